// On-device draft-tree construction: proposal top-k, best-first trees, tier
// utilities and the packed verify wave, so a wave is planned from the
// drafter's logits without a host round trip.
//
// Reference path replaced (host Python per request):
//   probabilities(logits, T, float64)        sampling.py:29-36
//   probability_tree(q, budget, ...)         tree.py:148-212 (torch.topk per
//                                            depth, then a best-first heap)
//   _prefix_tree / _draft_tree_expected_tokens
//                                            continuous_tree_block_decode.py:560-586
//   tree selection of _propose_many          continuous_tree_block_decode.py:839-883
//
// proposal_topk_kernel: one CTA per (request, depth) row.  A radix select
// over order-preserving integer keys of the logits (8-bit digits, one
// shared-memory histogram per digit) finds the k-th largest key; one more
// pass gathers the keys above it (sorted afterwards) and the first equal keys
// in index order, so ties go to the lower vocabulary index.  The log mass of
// a kept token is (l - l_max) / T - log(sum_j exp((l_j - l_max) / T)) in
// fp64; the sum uses exp(h + r) = exp(h) * exp(r) with h on a 1/64 grid
// (a per-CTA table) and a degree-5 Taylor polynomial for |r| <= 1/128.
//
// draft_tree_kernel: one warp per tree.  The frontier is a shared-memory
// array of candidates (score, parent, depth, rank, parent mass); each step the
// warp finds the smallest (score, parent, depth, rank) with a shuffle
// reduction, emits it as the next node and appends its next sibling and first
// child, with the reference's fp64 operation order, so the tree is bit-equal
// to the reference's for the same log masses.
#include <cuda_bf16.h>

#include <cmath>

#include "common.cuh"

namespace sg {
namespace {

constexpr int kTopkThreads = 512;
constexpr int kTopkMax = 1024;      // largest k
constexpr int kChunk = 8;           // elements per thread per ordered gather chunk
constexpr int kExpSteps = 32;       // exp table: h = -i / 32
constexpr int kExpEntries = 64 * kExpSteps + 1;  // covers d in [-64, 0]
constexpr int kCandMax = 2048;      // candidates of the bin select
constexpr int kBinsPerNat = 8;      // bin select: 256 bins over 32 nats below the row max
constexpr int kBins = 256;
constexpr int kTreeWarps = 4;       // trees per CTA
constexpr int kMaxLength = 64;      // draft depths
constexpr int kMaxTiers = 8;

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status != nullptr) atomicMax(status, code);
}

__device__ __forceinline__ uint32_t order_key(__nv_bfloat16 v) {
  const uint32_t b = __bfloat16_as_ushort(v);
  return b ^ ((b & 0x8000u) ? 0xFFFFu : 0x8000u);
}
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return b ^ ((b & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}
__device__ __forceinline__ double to_double(__nv_bfloat16 v) { return static_cast<double>(__bfloat162float(v)); }
__device__ __forceinline__ double to_double(float v) { return static_cast<double>(v); }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ bool finite_value(__nv_bfloat16 v) { return isfinite(__bfloat162float(v)); }
__device__ __forceinline__ bool finite_value(float v) { return isfinite(v); }

// exp(d) for d <= 0 from the per-CTA table of exp(-i/32): exp(h + r) =
// exp(h) * exp(r) with |r| <= 1/64 and the degree-6 Taylor polynomial of
// exp(r) (truncation below 5e-17 relative).
__device__ __forceinline__ double exp_nonpositive(double d, const double* table) {
  if (!(d >= -64.0)) return d < -745.0 || d != d ? 0.0 : exp(d);  // (a NaN row is reported by the caller)
  const double scaled = -d * kExpSteps;
  const int i = __double2int_rn(scaled);
  const double r = d + static_cast<double>(i) / kExpSteps;  // |r| <= 1/64, exact
  double p = 1.0 / 720.0;
  p = fma(p, r, 1.0 / 120.0);
  p = fma(p, r, 1.0 / 24.0);
  p = fma(p, r, 1.0 / 6.0);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return table[i] * p;
}

// Digit of the radix select: among keys matching `prefix` under `mask`, the
// value b of the next digit with count(keys with digit > b) < need <=
// count(digit >= b).  Returns b and lowers `need` by the count above it.
__device__ int select_digit(const uint32_t* hist, int& need, int* scratch) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    // lane l covers bins 255 - 8l .. 248 - 8l (descending)
    int local = 0;
    for (int j = 0; j < 8; ++j) local += hist[255 - 8 * lane - j];
    int incl = local;
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int excl = incl - local;
    if (excl < need && need <= incl) {
      int run = excl;
      for (int j = 0; j < 8; ++j) {
        const int b = 255 - 8 * lane - j;
        const int c = hist[b];
        if (need <= run + c) {
          scratch[0] = b;
          scratch[1] = run;
          break;
        }
        run += c;
      }
    }
  }
  __syncthreads();
  const int b = scratch[0];
  need -= scratch[1];
  __syncthreads();
  return b;
}

// Calls f(i, v) for every element of row x, 16-byte vector loads when the
// row allows them (each thread a strided run of whole vectors).
template <typename T, typename F>
__device__ __forceinline__ void for_each_element(const T* __restrict__ x, int vocab, F&& f) {
  constexpr int VEC = 16 / static_cast<int>(sizeof(T));
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && vocab % VEC == 0) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int c = threadIdx.x; c < vocab / VEC; c += kTopkThreads) {
      const uint4 w = xv[c];
      const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int j = 0; j < VEC; ++j) f(c * VEC + j, e[j]);
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += kTopkThreads) f(i, x[i]);
  }
}

__device__ __forceinline__ unsigned long long cand_word(uint32_t key, int i) {
  // descending order of this word = key descending, then index ascending
  return (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
}
__device__ __forceinline__ int cand_index(unsigned long long w) {
  return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(w & 0xFFFFFFFFull));
}

// Sorts cand[0, n) descending (bitonic network over the next power of two).
__device__ void sort_desc(unsigned long long* cand, int n) {
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = n + static_cast<int>(threadIdx.x); i < P; i += kTopkThreads) cand[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += kTopkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = cand[i], c = cand[j];
          if (desc ? (a < c) : (a > c)) {
            cand[i] = c;
            cand[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads, 2) proposal_topk_kernel(const T* __restrict__ logits,
                                                                     int64_t row_stride, int rows_per_group,
                                                                     int64_t group_stride, int vocab, int k,
                                                                     double inv_t, double* __restrict__ log_q,
                                                                     int64_t* __restrict__ ids,
                                                                     int32_t* status) {
  constexpr int kKeyBits = static_cast<int>(sizeof(T)) * 8;
  __shared__ uint32_t hist[kBins];
  __shared__ double exp_table[kExpEntries];
  __shared__ unsigned long long cand[kCandMax];
  __shared__ int eq_list[kTopkMax];
  __shared__ int scratch[4];
  __shared__ double red[kTopkThreads / 32];
  __shared__ uint32_t kmax[kTopkThreads / 32];
  __shared__ int n_cand;
  __shared__ int eq_base;
  __shared__ int warp_eq[kTopkThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int group = static_cast<int>(blockIdx.x) / rows_per_group;
  const int in_group = static_cast<int>(blockIdx.x) - group * rows_per_group;
  const T* x = logits + static_cast<int64_t>(group) * group_stride + static_cast<int64_t>(in_group) * row_stride;
  double* out_q = log_q + static_cast<int64_t>(blockIdx.x) * k;
  int64_t* out_id = ids + static_cast<int64_t>(blockIdx.x) * k;

  for (int i = tid; i < kExpEntries; i += kTopkThreads) exp_table[i] = exp(-static_cast<double>(i) / kExpSteps);
  for (int i = tid; i < kBins; i += kTopkThreads) hist[i] = 0u;
  if (tid == 0) n_cand = 0;

  // pass 0: the row maximum (largest order key)
  uint32_t my_max = 0;
  bool bad = false;
  for_each_element(x, vocab, [&](int, T v) {
    my_max = max(my_max, order_key(v));
    bad |= !finite_value(v);
  });
  for (int o = 16; o > 0; o >>= 1) my_max = max(my_max, __shfl_xor_sync(0xffffffffu, my_max, o));
  if (lane == 0) kmax[warp] = my_max;
  if (__syncthreads_or(bad) && tid == 0) report(status, SG_ERR_PROBABILITY);
  uint32_t mkey = kmax[0];
  for (int w = 1; w < kTopkThreads / 32; ++w) mkey = max(mkey, kmax[w]);
  double lmax;
  if constexpr (sizeof(T) == 2) {
    const uint32_t b = (mkey & 0x8000u) ? (mkey ^ 0x8000u) : (mkey ^ 0xFFFFu);
    lmax = to_double(__ushort_as_bfloat16(static_cast<unsigned short>(b)));
  } else {
    const uint32_t b = (mkey & 0x80000000u) ? (mkey ^ 0x80000000u) : (mkey ^ 0xFFFFFFFFu);
    lmax = static_cast<double>(__uint_as_float(b));
  }
  // bin of an element: floor(8 (max - l) / T) when below 256, else none
  // (fp32: the bins only partition the row, the same way in both passes)
  const float lmax_f = static_cast<float>(lmax), bin_scale = static_cast<float>(inv_t * kBinsPerNat);
  auto bin_of = [&](T v) -> int {
    const float d = (lmax_f - to_float(v)) * bin_scale;  // >= 0 (NaN: no bin)
    return d < static_cast<float>(kBins) ? static_cast<int>(d) : kBins;
  };

  // pass 1: normaliser (fp64) and the bin histogram
  double my_sum = 0.0;
  for_each_element(x, vocab, [&](int, T v) {
    my_sum += exp_nonpositive((to_double(v) - lmax) * inv_t, exp_table);
    const int b = bin_of(v);
    if (b < kBins) atomicAdd(&hist[b], 1u);
  });
  for (int o = 16; o > 0; o >>= 1) my_sum += __shfl_xor_sync(0xffffffffu, my_sum, o);
  if (lane == 0) red[warp] = my_sum;
  __syncthreads();
  double total = 0.0;
  for (int w = 0; w < kTopkThreads / 32; ++w) total += red[w];
  const double log_total = log(total);
  // smallest bin B with count(bins <= B) >= k
  if (warp == 0) {
    int local = 0;
    for (int j = 0; j < kBins / 32; ++j) local += hist[lane * (kBins / 32) + j];
    int incl = local;
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31 && incl < k) {
      scratch[0] = -1;  // fewer than k elements within 32 nats: radix select
      scratch[1] = 0;
    }
    const int excl = incl - local;
    if (excl < k && k <= incl) {
      int run = excl;
      for (int j = 0; j < kBins / 32; ++j) {
        run += hist[lane * (kBins / 32) + j];
        if (run >= k) {
          scratch[0] = lane * (kBins / 32) + j;
          scratch[1] = run;
          break;
        }
      }
    }
  }
  __syncthreads();
  const int sel_bin = scratch[0], n_sel = scratch[1];
  if (sel_bin >= 0 && n_sel <= kCandMax) {
    // pass 2: every element in bins <= B is a candidate; sort them
    for_each_element(x, vocab, [&](int i, T v) {
      if (bin_of(v) <= sel_bin) {
        const int slot = atomicAdd(&n_cand, 1);
        if (slot < kCandMax) cand[slot] = cand_word(order_key(v), i);
      }
    });
    __syncthreads();
    if (n_cand != n_sel) {
      if (tid == 0) report(status, SG_ERR_TREE);
      return;
    }
    sort_desc(cand, n_sel);
    for (int r = tid; r < k; r += kTopkThreads) {
      const int i = cand_index(cand[r]);
      out_id[r] = i;
      out_q[r] = (to_double(x[i]) - lmax) * inv_t - log_total;
    }
    return;
  }

  // Radix select over order keys (rows where more than kCandMax elements sit
  // in the selected bin or fewer than k within 32 nats): 8-bit digits, one
  // shared-memory histogram each, then the keys above the k-th key (sorted)
  // and the first equal keys in index order.
  uint32_t prefix = 0, mask = 0;
  int need = k;
  for (int digit = 0; digit < kKeyBits / 8; ++digit) {
    const int shift = kKeyBits - 8 * (digit + 1);
    __syncthreads();
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0u;
    __syncthreads();
    for_each_element(x, vocab, [&](int, T v) {
      const uint32_t key = order_key(v);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    });
    __syncthreads();
    const uint32_t b = static_cast<uint32_t>(select_digit(hist, need, scratch));
    prefix |= b << shift;
    mask |= 255u << shift;
  }
  if (tid == 0) {
    n_cand = 0;
    eq_base = 0;
  }
  __syncthreads();
  const uint32_t thr = prefix;
  for (int base = 0; base < vocab; base += kTopkThreads * kChunk) {
    const int i0 = base + tid * kChunk;
    int eq_local = 0;
    for (int j = 0; j < kChunk; ++j) {
      const int i = i0 + j;
      if (i >= vocab) break;
      const uint32_t key = order_key(x[i]);
      if (key > thr) {
        const int slot = atomicAdd(&n_cand, 1);
        if (slot < kTopkMax) cand[slot] = cand_word(key, i);
      } else if (key == thr) {
        ++eq_local;
      }
    }
    if (__syncthreads_count(eq_local) == 0) continue;
    int incl = eq_local;
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_eq[warp] = incl;
    __syncthreads();
    int before = eq_base + incl - eq_local;
    for (int w = 0; w < warp; ++w) before += warp_eq[w];
    for (int j = 0; j < kChunk && eq_local > 0; ++j) {
      const int i = i0 + j;
      if (i >= vocab) break;
      if (order_key(x[i]) == thr) {
        if (before < need) eq_list[before] = i;
        ++before;
        --eq_local;
      }
    }
    __syncthreads();
    if (tid == 0) {
      int add = 0;
      for (int w = 0; w < kTopkThreads / 32; ++w) add += warp_eq[w];
      eq_base += add;
    }
    __syncthreads();
  }
  __syncthreads();
  const int gt = k - need;
  if (tid == 0 && n_cand != gt) report(status, SG_ERR_TREE);
  sort_desc(cand, gt);
  for (int r = tid; r < k; r += kTopkThreads) {
    const int i = r < gt ? cand_index(cand[r]) : eq_list[r - gt];
    out_id[r] = i;
    out_q[r] = (to_double(x[i]) - lmax) * inv_t - log_total;
  }
}

// ---------------------------------------------------------------------------
// Best-first trees
// ---------------------------------------------------------------------------
struct TreeParams {
  const double* log_q;      // [trees, length, width]
  const int64_t* ids;       // [trees, length, width]
  int trees, length, width;
  const int32_t* budgets;   // [trees] or null (then `budget` for all)
  int budget;               // largest budget (row stride of the outputs)
  double rewards[kMaxLength];
  int caps[kMaxLength];     // per-depth rank caps (already clipped to width)
  int adaptive_min;         // -1: off
  double log_threshold;
  int tiers[kMaxTiers];
  int num_tiers;
  int64_t* tokens;          // [trees, budget]
  int64_t* parents;         // [trees, budget + 1]
  int32_t* depths;          // [trees, budget + 1]
  double* masses;           // [trees, budget + 1]
  int32_t* node_count;      // [trees]
  double* utilities;        // [trees, num_tiers] or null
  int32_t* status;
  int warps;                // trees per CTA
  int staged;               // 1: each tree's log masses and ids are copied to shared memory first
};

__device__ __forceinline__ bool cand_less(double sa, unsigned long long ta, double sb, unsigned long long tb) {
  return sa < sb || (sa == sb && ta < tb);
}

// Shared memory of one tree's warp: frontier (score, parent mass, tie key),
// node masses, and when staged the tree's log masses and 32-bit ids.
__host__ __device__ inline size_t tree_warp_bytes(int budget, int length, int width, bool staged) {
  const size_t cap = static_cast<size_t>(budget) + 2;
  size_t b = cap * 3 * 8 + (static_cast<size_t>(budget) + 1) * 8;
  if (staged) b += static_cast<size_t>(length) * width * 12;
  return (b + 15) & ~size_t(15);
}

__global__ void __launch_bounds__(kTreeWarps * 32) draft_tree_kernel(const TreeParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tree = blockIdx.x * p.warps + warp;
  const int cap = p.budget + 2;  // frontier capacity: one entry in, at most two out per node
  uint8_t* base = smem + static_cast<size_t>(warp) * tree_warp_bytes(p.budget, p.length, p.width, p.staged != 0);
  double* score = reinterpret_cast<double*>(base);
  double* plog = score + cap;
  unsigned long long* tie = reinterpret_cast<unsigned long long*>(plog + cap);
  double* node_mass = reinterpret_cast<double*>(tie + cap);
  if (tree >= p.trees) return;
  const double* lq = p.log_q + static_cast<int64_t>(tree) * p.length * p.width;
  const int64_t* tid_ids = p.ids + static_cast<int64_t>(tree) * p.length * p.width;
  double* lq_s = node_mass + (p.budget + 1);
  int32_t* ids_s = reinterpret_cast<int32_t*>(lq_s + static_cast<size_t>(p.length) * p.width);
  if (p.staged) {
    for (int j = lane; j < p.length * p.width; j += 32) {
      lq_s[j] = lq[j];
      ids_s[j] = static_cast<int32_t>(tid_ids[j]);
    }
    __syncwarp();
    lq = lq_s;
  }
  auto token_at = [&](int64_t j) -> int64_t { return p.staged ? ids_s[j] : tid_ids[j]; };
  int budget = p.budgets != nullptr ? p.budgets[tree] : p.budget;
  if (budget < 1 || budget > p.budget) {
    if (lane == 0) report(p.status, SG_ERR_TREE);
    budget = max(1, min(budget, p.budget));
  }
  int caps[kMaxLength];
  for (int d = 0; d < p.length; ++d) caps[d] = min(p.caps[d], budget);
  if (p.adaptive_min >= 0) {
    const int seen = min(4, p.length);
    double total = 0.0;
    for (int d = 0; d < seen; ++d) total += lq[static_cast<int64_t>(d) * p.width];
    if (total / seen >= p.log_threshold) budget = p.adaptive_min;
  }
  int64_t* out_tok = p.tokens + static_cast<int64_t>(tree) * p.budget;
  int64_t* out_par = p.parents + static_cast<int64_t>(tree) * (p.budget + 1);
  int32_t* out_dep = p.depths + static_cast<int64_t>(tree) * (p.budget + 1);
  double* out_mass = p.masses + static_cast<int64_t>(tree) * (p.budget + 1);
  if (lane == 0) {
    out_par[0] = -1;
    out_dep[0] = 0;
    out_mass[0] = 0.0;
    node_mass[0] = 0.0;
    score[0] = -(lq[0] + p.rewards[0]);
    plog[0] = 0.0;
    tie[0] = 0ull;
  }
  __syncwarp();
  int n = 1, count = 0;
  while (n > 0 && count < budget) {
    // smallest (score, parent, depth, rank)
    double bs = INFINITY;
    unsigned long long bt = ~0ull;
    int bslot = -1;
    for (int j = lane; j < n; j += 32)
      if (bslot < 0 || cand_less(score[j], tie[j], bs, bt)) {
        bs = score[j];
        bt = tie[j];
        bslot = j;
      }
    for (int o = 16; o > 0; o >>= 1) {
      const double os = __shfl_xor_sync(0xffffffffu, bs, o);
      const unsigned long long ot = __shfl_xor_sync(0xffffffffu, bt, o);
      const int oslot = __shfl_xor_sync(0xffffffffu, bslot, o);
      if (oslot >= 0 && (bslot < 0 || cand_less(os, ot, bs, bt))) {
        bs = os;
        bt = ot;
        bslot = oslot;
      }
    }
    const double parent_mass = plog[bslot];
    const int parent = static_cast<int>(bt >> 32);
    const int depth = static_cast<int>((bt >> 16) & 0xFFFFu);
    const int rank = static_cast<int>(bt & 0xFFFFu);
    __syncwarp();
    if (lane == 0) {
      // remove the expanded candidate (the last one takes its slot)
      --n;
      score[bslot] = score[n];
      plog[bslot] = plog[n];
      tie[bslot] = tie[n];
      const int node = count + 1;
      const int64_t row = static_cast<int64_t>(depth) * p.width;
      out_tok[count] = token_at(row + rank);
      out_par[node] = parent;
      out_dep[node] = depth + 1;
      out_mass[node] = -bs;
      node_mass[node] = -bs;
      if (rank + 1 < caps[depth]) {
        score[n] = -((parent_mass + lq[row + rank + 1]) + p.rewards[depth]);
        plog[n] = parent_mass;
        tie[n] = (static_cast<unsigned long long>(parent) << 32) | (static_cast<unsigned long long>(depth) << 16) |
                 static_cast<unsigned long long>(rank + 1);
        ++n;
      }
      if (depth + 1 < p.length) {
        score[n] = (bs - lq[row + p.width]) - p.rewards[depth + 1];
        plog[n] = -bs;
        tie[n] = (static_cast<unsigned long long>(node) << 32) | (static_cast<unsigned long long>(depth + 1) << 16);
        ++n;
      }
    }
    n = __shfl_sync(0xffffffffu, n, 0);
    ++count;
    __syncwarp();
  }
  if (lane == 0) p.node_count[tree] = count;
  if (p.utilities == nullptr) return;
  // tier utilities: 1 + the compensated (Neumaier) running sum of
  // exp(prefix mass) over the tier's first nodes, as the reference's float
  // `sum` accumulates it
  for (int j = 1 + lane; j <= count; j += 32) node_mass[j] = exp(node_mass[j]);
  __syncwarp();
  if (lane == 0) {
    double* util = p.utilities + static_cast<int64_t>(tree) * p.num_tiers;
    double total = 0.0, comp = 0.0;
    int next_tier = 0;
    for (int t = 0; t < p.num_tiers; ++t)
      if (p.tiers[t] > count) {
        util[t] = NAN;
        report(p.status, SG_ERR_TREE);
      }
    for (int j = 1; j <= count; ++j) {
      const double v = node_mass[j];
      if (j == 1) {
        total = v;
      } else {
        const double t = total + v;
        if (fabs(total) >= fabs(v))
          comp += (total - t) + v;
        else
          comp += (v - t) + total;
        total = t;
      }
      for (int t = next_tier; t < p.num_tiers; ++t)
        if (p.tiers[t] == j) util[t] = 1.0 + ((comp != 0.0 && isfinite(comp)) ? total + comp : total);
    }
  }
}

// Register-resident frontier (budgets with 2 * budget + 1 <= 32 * kRegSlots,
// staged log masses): lane l holds candidates l, l + 32, ... in registers
// and caches its own minimum; the warp minimum of the 128-bit key (order-
// preserving score bits, then parent / depth / rank) is found with up to four
// __reduce_min_sync steps on 32-bit words.  Same candidates, same order, same
// fp64 arithmetic as draft_tree_kernel.
constexpr int kRegSlots = 9;

__device__ __forceinline__ unsigned long long score_key(double v) {
  if (v == 0.0) v = 0.0;  // -0 and +0 compare equal
  const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(v));
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}
__device__ __forceinline__ double score_of(unsigned long long k) {
  const unsigned long long b = (k >> 63) ? (k & 0x7FFFFFFFFFFFFFFFull) : ~k;
  return __longlong_as_double(static_cast<long long>(b));
}

__global__ void __launch_bounds__(kTreeWarps * 32) draft_tree_reg_kernel(const TreeParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tree = blockIdx.x * p.warps + warp;
  uint8_t* base = smem + static_cast<size_t>(warp) * tree_warp_bytes(p.budget, p.length, p.width, true);
  double* node_mass = reinterpret_cast<double*>(base) + 3 * (p.budget + 2);
  double* lq = node_mass + (p.budget + 1);
  int32_t* ids_s = reinterpret_cast<int32_t*>(lq + static_cast<size_t>(p.length) * p.width);
  if (tree >= p.trees) return;
  {
    const double* lq_g = p.log_q + static_cast<int64_t>(tree) * p.length * p.width;
    const int64_t* ids_g = p.ids + static_cast<int64_t>(tree) * p.length * p.width;
    const int n = p.length * p.width;
    // eight independent loads in flight per lane
    for (int j0 = lane; j0 < n; j0 += 32 * 8) {
      double a[8];
      int64_t b[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + 32 * u;
        a[u] = j < n ? lq_g[j] : 0.0;
        b[u] = j < n ? ids_g[j] : 0;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + 32 * u;
        if (j < n) {
          lq[j] = a[u];
          ids_s[j] = static_cast<int32_t>(b[u]);
        }
      }
    }
    __syncwarp();
  }
  int budget = p.budgets != nullptr ? p.budgets[tree] : p.budget;
  if (budget < 1 || budget > p.budget) {
    if (lane == 0) report(p.status, SG_ERR_TREE);
    budget = max(1, min(budget, p.budget));
  }
  const int cap_budget = budget;  // rank caps use the budget before the adaptive change
  if (p.adaptive_min >= 0) {
    const int seen = min(4, p.length);
    double total = 0.0;
    for (int d = 0; d < seen; ++d) total += lq[static_cast<int64_t>(d) * p.width];
    if (total / seen >= p.log_threshold) budget = p.adaptive_min;
  }
  int64_t* out_tok = p.tokens + static_cast<int64_t>(tree) * p.budget;
  int64_t* out_par = p.parents + static_cast<int64_t>(tree) * (p.budget + 1);
  int32_t* out_dep = p.depths + static_cast<int64_t>(tree) * (p.budget + 1);
  double* out_mass = p.masses + static_cast<int64_t>(tree) * (p.budget + 1);

  unsigned long long sk[kRegSlots], tk[kRegSlots];
  double pl[kRegSlots];
#pragma unroll
  for (int j = 0; j < kRegSlots; ++j) {
    sk[j] = ~0ull;
    tk[j] = ~0ull;
    pl[j] = 0.0;
  }
  unsigned long long best_sk = ~0ull, best_tk = ~0ull;
  int best_slot = -1;
  auto recompute = [&]() {
    best_sk = ~0ull;
    best_tk = ~0ull;
    best_slot = -1;
#pragma unroll
    for (int j = 0; j < kRegSlots; ++j)
      if (sk[j] < best_sk || (sk[j] == best_sk && tk[j] < best_tk)) {
        best_sk = sk[j];
        best_tk = tk[j];
        best_slot = sk[j] == ~0ull ? -1 : j;
      }
  };
  int inserted = 0;
  auto insert = [&](double score, unsigned long long tie, double parent_mass) {
    const int owner = inserted & 31, slot = inserted >> 5;
    ++inserted;
    if (lane != owner) return;
    const unsigned long long k = score_key(score);
#pragma unroll
    for (int j = 0; j < kRegSlots; ++j)
      if (j == slot) {
        sk[j] = k;
        tk[j] = tie;
        pl[j] = parent_mass;
      }
    if (k < best_sk || (k == best_sk && tie < best_tk)) {
      best_sk = k;
      best_tk = tie;
      best_slot = slot;
    }
  };
  if (lane == 0) {
    out_par[0] = -1;
    out_dep[0] = 0;
    out_mass[0] = 0.0;
    node_mass[0] = 0.0;
  }
  insert(-(lq[0] + p.rewards[0]), 0ull, 0.0);
  int count = 0;
  while (count < budget) {
    // warp minimum of (best_sk, best_tk), word by word
    bool cand = true;
    unsigned mask = 0xffffffffu;
    const uint32_t words[4] = {static_cast<uint32_t>(best_sk >> 32), static_cast<uint32_t>(best_sk),
                               static_cast<uint32_t>(best_tk >> 32), static_cast<uint32_t>(best_tk)};
    bool empty = false;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t v = cand ? words[w] : 0xFFFFFFFFu;
      const uint32_t m = __reduce_min_sync(0xffffffffu, v);
      if (w == 0 && m == 0xFFFFFFFFu && __all_sync(0xffffffffu, best_slot < 0)) empty = true;
      cand = cand && v == m;
      mask = __ballot_sync(0xffffffffu, cand);
      if (__popc(mask) == 1) break;
    }
    if (empty) break;
    const int winner = __ffs(mask) - 1;
    double parent_mass = 0.0;
    if (lane == winner) {
      double v = 0.0;
#pragma unroll
      for (int j = 0; j < kRegSlots; ++j)
        if (j == best_slot) {
          v = pl[j];
          sk[j] = ~0ull;
          tk[j] = ~0ull;
        }
      parent_mass = v;
    }
    const unsigned long long bk = __shfl_sync(0xffffffffu, best_sk, winner);
    const unsigned long long bt = __shfl_sync(0xffffffffu, best_tk, winner);
    parent_mass = __shfl_sync(0xffffffffu, parent_mass, winner);
    if (lane == winner) recompute();
    const double bs = score_of(bk);
    const int parent = static_cast<int>(bt >> 32);
    const int depth = static_cast<int>((bt >> 16) & 0xFFFFu);
    const int rank = static_cast<int>(bt & 0xFFFFu);
    const int node = count + 1;
    const int64_t row = static_cast<int64_t>(depth) * p.width;
    if (lane == 0) {
      out_tok[count] = ids_s[row + rank];
      out_par[node] = parent;
      out_dep[node] = depth + 1;
      out_mass[node] = -bs;
      node_mass[node] = -bs;
    }
    if (rank + 1 < min(p.caps[depth], cap_budget))
      insert(-((parent_mass + lq[row + rank + 1]) + p.rewards[depth]),
             (static_cast<unsigned long long>(parent) << 32) | (static_cast<unsigned long long>(depth) << 16) |
                 static_cast<unsigned long long>(rank + 1),
             parent_mass);
    if (depth + 1 < p.length)
      insert((bs - lq[row + p.width]) - p.rewards[depth + 1],
             (static_cast<unsigned long long>(node) << 32) | (static_cast<unsigned long long>(depth + 1) << 16), -bs);
    ++count;
  }
  if (lane == 0) p.node_count[tree] = count;
  if (p.utilities == nullptr) return;
  __syncwarp();
  for (int j = 1 + lane; j <= count; j += 32) node_mass[j] = exp(node_mass[j]);
  __syncwarp();
  if (lane == 0) {
    double* util = p.utilities + static_cast<int64_t>(tree) * p.num_tiers;
    double total = 0.0, comp = 0.0;
    for (int t = 0; t < p.num_tiers; ++t)
      if (p.tiers[t] > count) {
        util[t] = NAN;
        report(p.status, SG_ERR_TREE);
      }
    for (int j = 1; j <= count; ++j) {
      const double v = node_mass[j];
      if (j == 1) {
        total = v;
      } else {
        const double t = total + v;
        if (fabs(total) >= fabs(v))
          comp += (total - t) + v;
        else
          comp += (v - t) + total;
        total = t;
      }
      for (int t = 0; t < p.num_tiers; ++t)
        if (p.tiers[t] == j) util[t] = 1.0 + ((comp != 0.0 && isfinite(comp)) ? total + comp : total);
    }
  }
}

// Packs each request's chosen tier (the first allocation[r] nodes of its
// tree) into the packed verify wave: row r's block starts with the anchor
// (its last generated token), then the nodes in best-first order (parents
// are local row indices; the anchor's is -1).
__global__ void __launch_bounds__(1024) pack_tree_wave_kernel(
    const int64_t* __restrict__ tokens, const int64_t* __restrict__ parents, int budget,
    const int32_t* __restrict__ node_count, const int32_t* __restrict__ allocation,
    const int64_t* __restrict__ anchor_tokens, int trees, int64_t max_rows, int64_t* __restrict__ row_offsets,
    int64_t* __restrict__ wave_parents, int64_t* __restrict__ wave_tokens, int32_t* status) {
  __shared__ int64_t offsets_s[1025];
  __shared__ int64_t warp_sum[32];
  __shared__ int bad;
  const int r = threadIdx.x, lane = r & 31, warp = r >> 5;
  if (r == 0) bad = 0;
  __syncthreads();
  // rows of request r (its anchor + allocation[r] nodes), block-wide scan
  int64_t rows = 0;
  if (r < trees) {
    int a = allocation[r];
    if (a < 0 || a > node_count[r] || a > budget) {
      bad = 1;
      a = 0;
    }
    rows = a + 1;
  }
  int64_t incl = rows;
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < static_cast<int>(blockDim.x >> 5) ? warp_sum[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    warp_sum[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int64_t before = incl - rows + (warp > 0 ? warp_sum[warp - 1] : 0);
  if (r < trees) offsets_s[r + 1] = before + rows;
  if (r == 0) offsets_s[0] = 0;
  __syncthreads();
  if (bad || offsets_s[trees] > max_rows) {
    if (r == 0) report(status, SG_ERR_TREE);
    for (int t = r; t <= trees; t += blockDim.x) row_offsets[t] = 0;
    return;
  }
  for (int t = r; t <= trees; t += blockDim.x) row_offsets[t] = offsets_s[t];
  // every row of the wave: one thread per (request, row) pair, requests in turn
  for (int t = warp; t < trees; t += blockDim.x >> 5) {
    const int64_t base = offsets_s[t];
    const int n = static_cast<int>(offsets_s[t + 1] - base);
    for (int j = lane; j < n; j += 32) {
      wave_parents[base + j] = j == 0 ? -1 : parents[static_cast<int64_t>(t) * (budget + 1) + j];
      wave_tokens[base + j] = j == 0 ? anchor_tokens[t] : tokens[static_cast<int64_t>(t) * budget + j - 1];
    }
  }
}

bool aligned_to(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace
}  // namespace sg

extern "C" int sg_proposal_topk(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows_per_group,
                                int64_t group_stride, int32_t rows, int32_t vocab, int32_t k, double temperature,
                                double* log_q, int64_t* ids, int32_t* status, void* stream) {
  using namespace sg;
  if (rows == 0) return SG_OK;
  if (logits == nullptr || log_q == nullptr || ids == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_proposal_topk: null pointer");
  if (rows < 0 || vocab < 1 || k < 1 || k > kTopkMax || k > vocab || row_stride < vocab || rows_per_group < 1 ||
      rows % rows_per_group != 0 || (rows > rows_per_group && group_stride < row_stride * rows_per_group))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_proposal_topk: bad sizes (1 <= k <= min(1024, vocab), rows a "
                                         "multiple of rows_per_group, groups not overlapping)");
  if (!(temperature > 0.0) || !std::isfinite(temperature))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_proposal_topk: temperature must be finite and > 0");
  if (dtype != SG_DTYPE_BF16 && dtype != SG_DTYPE_F32)
    return fail(SG_ERR_UNSUPPORTED, "sg_proposal_topk: logits must be bf16 or fp32");
  const uintptr_t el = dtype == SG_DTYPE_BF16 ? 2 : 4;
  if (!aligned_to(logits, el) || !aligned_to(log_q, 8) || !aligned_to(ids, 8) || !aligned_to(status, 4))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_proposal_topk: misaligned pointer");
  const double inv_t = 1.0 / temperature;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SG_DTYPE_BF16) {
    proposal_topk_kernel<__nv_bfloat16><<<rows, kTopkThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), row_stride, rows_per_group, group_stride, vocab, k, inv_t, log_q,
        ids, status);
  } else {
    proposal_topk_kernel<float><<<rows, kTopkThreads, 0, s>>>(static_cast<const float*>(logits), row_stride,
                                                              rows_per_group, group_stride, vocab, k, inv_t, log_q,
                                                              ids, status);
  }
  return check_launch("proposal_topk_kernel");
}

extern "C" int sg_build_draft_trees(const double* log_q, const int64_t* ids, int32_t num_trees, int32_t length,
                                    int32_t width, const int32_t* budgets, int32_t budget, const double* rewards,
                                    const int32_t* rank_caps, int32_t adaptive_min_budget,
                                    double confidence_threshold, const int32_t* tiers, int32_t num_tiers,
                                    int64_t* tokens, int64_t* parents, int32_t* depths, double* masses,
                                    int32_t* node_count, double* utilities, int32_t* status, void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (log_q == nullptr || ids == nullptr || tokens == nullptr || parents == nullptr || depths == nullptr ||
      masses == nullptr || node_count == nullptr || (num_tiers > 0 && (tiers == nullptr || utilities == nullptr)))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_build_draft_trees: null pointer");
  if (num_trees < 0 || length < 1 || length > kMaxLength || width < 1 || budget < 1 || budget > 4096 ||
      num_tiers < 0 || num_tiers > kMaxTiers)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_build_draft_trees: bad sizes (length <= 64, budget <= 4096, "
                                         "tiers <= 8)");
  if (!aligned_to(log_q, 8) || !aligned_to(ids, 8) || !aligned_to(tokens, 8) || !aligned_to(parents, 8) ||
      !aligned_to(masses, 8) || !aligned_to(depths, 4) || !aligned_to(node_count, 4) || !aligned_to(budgets, 4) ||
      !aligned_to(utilities, 8) || !aligned_to(status, 4))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_build_draft_trees: misaligned pointer");
  TreeParams p = {};
  p.log_q = log_q;
  p.ids = ids;
  p.trees = num_trees;
  p.length = length;
  p.width = width;
  p.budgets = budgets;
  p.budget = budget;
  for (int d = 0; d < length; ++d) {
    const double r = rewards != nullptr ? rewards[d] : 0.0;
    if (!std::isfinite(r)) return fail(SG_ERR_INVALID_ARGUMENT, "sg_build_draft_trees: rewards must be finite");
    p.rewards[d] = r;
    const int c = rank_caps != nullptr ? rank_caps[d] : budget;
    if (c < 1) return fail(SG_ERR_INVALID_ARGUMENT, "sg_build_draft_trees: rank caps must be >= 1");
    p.caps[d] = std::min(std::min(c, budget), width);
  }
  if (adaptive_min_budget >= 0) {
    if (!(confidence_threshold > 0.0) || adaptive_min_budget < 1 || adaptive_min_budget > budget)
      return fail(SG_ERR_INVALID_ARGUMENT,
                  "sg_build_draft_trees: adaptive budget needs a threshold > 0 and 1 <= min budget <= budget");
    p.log_threshold = std::log(confidence_threshold);
  }
  p.adaptive_min = adaptive_min_budget >= 0 ? adaptive_min_budget : -1;
  for (int t = 0; t < num_tiers; ++t) {
    if (tiers[t] < 1 || (t > 0 && tiers[t] <= tiers[t - 1]))
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_build_draft_trees: tiers must be increasing and >= 1");
    p.tiers[t] = tiers[t];
  }
  p.num_tiers = num_tiers;
  p.tokens = tokens;
  p.parents = parents;
  p.depths = depths;
  p.masses = masses;
  p.node_count = node_count;
  p.utilities = num_tiers > 0 ? utilities : nullptr;
  p.status = status;
  // largest trees-per-CTA whose warps can stage their tree in shared
  // memory; otherwise unstaged (log masses read from global memory)
  constexpr size_t kSmemLimit = 220 * 1024;
  p.warps = 0;
  for (int w = kTreeWarps; w >= 1 && p.warps == 0; w >>= 1)
    if (w * tree_warp_bytes(budget, length, width, true) <= kSmemLimit) {
      p.warps = w;
      p.staged = 1;
    }
  if (p.warps == 0) {
    for (int w = kTreeWarps; w >= 1 && p.warps == 0; w >>= 1)
      if (w * tree_warp_bytes(budget, length, width, false) <= kSmemLimit) p.warps = w;
    p.staged = 0;
  }
  if (p.warps == 0) return fail(SG_ERR_UNSUPPORTED, "sg_build_draft_trees: budget too large");
  const size_t smem = p.warps * tree_warp_bytes(budget, length, width, p.staged != 0);
  const bool in_registers = p.staged && 2 * budget + 1 <= 32 * kRegSlots;
  static std::atomic<int> reg_limits[kMaxDevices], smem_limits[kMaxDevices];
  auto kernel = in_registers ? draft_tree_reg_kernel : draft_tree_kernel;
  const int st = ensure_dynamic_smem(kernel, smem, in_registers ? reg_limits : smem_limits);
  if (st != SG_OK) return st;
  const int blocks = (num_trees + p.warps - 1) / p.warps;
  kernel<<<blocks, p.warps * 32, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("draft_tree_kernel");
}

extern "C" int sg_pack_tree_wave(const int64_t* tokens, const int64_t* parents, int32_t budget,
                                 const int32_t* node_count, const int32_t* allocation, const int64_t* anchor_tokens,
                                 int32_t num_trees, int64_t max_rows, int64_t* row_offsets, int64_t* wave_parents,
                                 int64_t* wave_tokens, int32_t* status, void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (tokens == nullptr || parents == nullptr || node_count == nullptr || allocation == nullptr ||
      anchor_tokens == nullptr || row_offsets == nullptr || wave_parents == nullptr || wave_tokens == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_pack_tree_wave: null pointer");
  if (num_trees < 0 || num_trees > 1024 || budget < 1 || max_rows < num_trees)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_pack_tree_wave: bad sizes (at most 1024 trees)");
  pack_tree_wave_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      tokens, parents, budget, node_count, allocation, anchor_tokens, num_trees, max_rows, row_offsets, wave_parents,
      wave_tokens, status);
  return check_launch("pack_tree_wave_kernel");
}
