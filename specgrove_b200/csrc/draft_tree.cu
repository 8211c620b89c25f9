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
constexpr int kExpSteps = 64;       // exp table: h = -i / 64
constexpr int kExpEntries = 64 * kExpSteps + 1;  // covers d in [-64, 0]
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
__device__ __forceinline__ bool finite_value(__nv_bfloat16 v) { return isfinite(__bfloat162float(v)); }
__device__ __forceinline__ bool finite_value(float v) { return isfinite(v); }

// exp(d) for d <= 0 from the per-CTA table of exp(-i/64).
__device__ __forceinline__ double exp_nonpositive(double d, const double* table) {
  if (!(d >= -64.0)) return d < -745.0 || d != d ? 0.0 : exp(d);  // (a NaN row is reported by the caller)
  const double scaled = -d * kExpSteps;
  const int i = __double2int_rn(scaled);
  const double r = d + static_cast<double>(i) / kExpSteps;  // |r| <= 1/128, exact
  double p = 1.0 / 120.0;
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

template <typename T>
__global__ void __launch_bounds__(kTopkThreads, 2) proposal_topk_kernel(const T* __restrict__ logits,
                                                                     int64_t row_stride, int rows_per_group,
                                                                     int64_t group_stride, int vocab, int k,
                                                                     double inv_t, double* __restrict__ log_q,
                                                                     int64_t* __restrict__ ids,
                                                                     int32_t* status) {
  constexpr int kKeyBits = static_cast<int>(sizeof(T)) * 8;
  __shared__ uint32_t hist[256];
  __shared__ double exp_table[kExpEntries];
  __shared__ unsigned long long cand[kTopkMax];
  __shared__ int eq_list[kTopkMax];
  __shared__ int scratch[4];
  __shared__ double red[kTopkThreads / 32];
  __shared__ uint32_t kmax[kTopkThreads / 32];
  __shared__ int n_gt;
  __shared__ int eq_base;
  __shared__ int warp_eq[kTopkThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int group = static_cast<int>(blockIdx.x) / rows_per_group;
  const int in_group = static_cast<int>(blockIdx.x) - group * rows_per_group;
  const T* x = logits + static_cast<int64_t>(group) * group_stride + static_cast<int64_t>(in_group) * row_stride;
  double* out_q = log_q + static_cast<int64_t>(blockIdx.x) * k;
  int64_t* out_id = ids + static_cast<int64_t>(blockIdx.x) * k;

  for (int i = tid; i < kExpEntries; i += kTopkThreads) exp_table[i] = exp(-static_cast<double>(i) / kExpSteps);

  uint32_t prefix = 0, mask = 0;
  int need = k;
  uint32_t my_max = 0;
  double my_sum = 0.0, lmax = 0.0;
  bool bad = false;
  for (int digit = 0; digit < kKeyBits / 8; ++digit) {
    const int shift = kKeyBits - 8 * (digit + 1);
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0u;
    __syncthreads();
    // whole warps iterate together so that equal bins of a warp can be
    // counted with one shared-memory atomic (a row's leading digits fall in
    // a handful of bins: per-element atomics would serialise on them)
    for (int base = 0; base < vocab; base += kTopkThreads) {
      const int i = base + tid;
      const bool in = i < vocab;
      const T v = in ? x[i] : T{};
      const uint32_t key = order_key(v);
      if (in && digit == 0) {
        my_max = max(my_max, key);
        bad |= !finite_value(v);
      }
      if (in && digit == 1) my_sum += exp_nonpositive((to_double(v) - lmax) * inv_t, exp_table);
      const bool counted = in && (key & mask) == prefix;
      const unsigned active = __ballot_sync(0xffffffffu, counted);
      if (counted) {
        const uint32_t bin = (key >> shift) & 255u;
        const unsigned same = __match_any_sync(active, bin);
        if (lane == __ffs(same) - 1) atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(same)));
      }
    }
    if (digit == 0) {
      // row maximum (the largest key) for the normaliser pass
      for (int o = 16; o > 0; o >>= 1) my_max = max(my_max, __shfl_xor_sync(0xffffffffu, my_max, o));
      if (lane == 0) kmax[warp] = my_max;
      if (__syncthreads_or(bad) && tid == 0) report(status, SG_ERR_PROBABILITY);
      uint32_t m = kmax[0];
      for (int w = 1; w < kTopkThreads / 32; ++w) m = max(m, kmax[w]);
      // the element holding the maximum key: decode the key back to a value
      if constexpr (sizeof(T) == 2) {
        const uint32_t b = (m & 0x8000u) ? (m ^ 0x8000u) : (m ^ 0xFFFFu);
        lmax = to_double(__ushort_as_bfloat16(static_cast<unsigned short>(b)));
      } else {
        const uint32_t b = (m & 0x80000000u) ? (m ^ 0x80000000u) : (m ^ 0xFFFFFFFFu);
        lmax = static_cast<double>(__uint_as_float(b));
      }
    } else {
      __syncthreads();
    }
    const uint32_t b = static_cast<uint32_t>(select_digit(hist, need, scratch));
    prefix |= b << shift;
    mask |= 255u << shift;
  }
  // normaliser
  for (int o = 16; o > 0; o >>= 1) my_sum += __shfl_xor_sync(0xffffffffu, my_sum, o);
  if (lane == 0) red[warp] = my_sum;
  if (tid == 0) {
    n_gt = 0;
    eq_base = 0;
  }
  __syncthreads();
  double total = 0.0;
  for (int w = 0; w < kTopkThreads / 32; ++w) total += red[w];
  const double log_total = log(total);

  // gather: keys above the threshold (any order), equal keys in index order
  const uint32_t thr = prefix;
  for (int base = 0; base < vocab; base += kTopkThreads * kChunk) {
    const int i0 = base + tid * kChunk;
    int eq_local = 0;
    for (int j = 0; j < kChunk; ++j) {
      const int i = i0 + j;
      if (i >= vocab) break;
      const uint32_t key = order_key(x[i]);
      if (key > thr) {
        const int slot = atomicAdd(&n_gt, 1);
        if (slot < kTopkMax) cand[slot] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - i);
      } else if (key == thr) {
        ++eq_local;
      }
    }
    if (__syncthreads_count(eq_local) == 0) continue;
    // exclusive scan of eq_local in thread order
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
  const int gt = k - need;  // == n_gt
  // sort the keys above the threshold, descending (bitonic over a power of two)
  int P = 1;
  while (P < gt) P <<= 1;
  for (int i = gt + tid; i < P; i += kTopkThreads) cand[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += kTopkThreads) {
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
  for (int r = tid; r < k; r += kTopkThreads) {
    const int i = r < gt ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(cand[r] & 0xFFFFFFFFull))
                         : eq_list[r - gt];
    out_id[r] = i;
    out_q[r] = (to_double(x[i]) - lmax) * inv_t - log_total;
  }
  if (tid == 0 && n_gt != gt) report(status, SG_ERR_TREE);
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
};

__device__ __forceinline__ bool cand_less(double sa, unsigned long long ta, double sb, unsigned long long tb) {
  return sa < sb || (sa == sb && ta < tb);
}

__global__ void __launch_bounds__(kTreeWarps * 32) draft_tree_kernel(const TreeParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tree = blockIdx.x * kTreeWarps + warp;
  const int cap = p.budget + 2;  // frontier capacity: one entry in, at most two out per node
  double* score = reinterpret_cast<double*>(smem) + static_cast<size_t>(warp) * cap * 3;
  double* plog = score + cap;
  unsigned long long* tie = reinterpret_cast<unsigned long long*>(plog + cap);
  double* node_mass = reinterpret_cast<double*>(smem) + static_cast<size_t>(kTreeWarps) * cap * 3 +
                      static_cast<size_t>(warp) * (p.budget + 1);
  if (tree >= p.trees) return;
  const double* lq = p.log_q + static_cast<int64_t>(tree) * p.length * p.width;
  const int64_t* tid_ids = p.ids + static_cast<int64_t>(tree) * p.length * p.width;
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
      out_tok[count] = tid_ids[row + rank];
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

// Packs each request's chosen tier (the first allocation[r] nodes of its
// tree) into the packed verify wave: row r's block starts with the anchor
// (its last generated token), then the nodes in best-first order (parents
// are local row indices; the anchor's is -1).
__global__ void pack_tree_wave_kernel(const int64_t* __restrict__ tokens, const int64_t* __restrict__ parents,
                                      int budget, const int32_t* __restrict__ node_count,
                                      const int32_t* __restrict__ allocation,
                                      const int64_t* __restrict__ anchor_tokens, int trees, int64_t max_rows,
                                      int64_t* __restrict__ row_offsets, int64_t* __restrict__ wave_parents,
                                      int64_t* __restrict__ wave_tokens, int32_t* status) {
  __shared__ int64_t offsets_s[1025];
  __shared__ int bad;
  if (threadIdx.x == 0) {
    bad = 0;
    int64_t run = 0;
    offsets_s[0] = 0;
    for (int r = 0; r < trees; ++r) {
      int a = allocation[r];
      if (a < 0 || a > node_count[r] || a > budget) {
        bad = 1;
        a = 0;
      }
      run += a + 1;
      offsets_s[r + 1] = run;
    }
    if (run > max_rows) bad = 1;
  }
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) report(status, SG_ERR_TREE);
    for (int r = threadIdx.x; r <= trees; r += blockDim.x) row_offsets[r] = 0;
    return;
  }
  for (int r = threadIdx.x; r <= trees; r += blockDim.x) row_offsets[r] = offsets_s[r];
  for (int r = 0; r < trees; ++r) {
    const int64_t base = offsets_s[r];
    const int n = static_cast<int>(offsets_s[r + 1] - base);
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      wave_parents[base + j] = j == 0 ? -1 : parents[static_cast<int64_t>(r) * (budget + 1) + j];
      wave_tokens[base + j] = j == 0 ? anchor_tokens[r] : tokens[static_cast<int64_t>(r) * budget + j - 1];
    }
  }
}

size_t tree_smem_bytes(int budget) {
  const size_t cap = static_cast<size_t>(budget) + 2;
  return kTreeWarps * (cap * 3 * 8 + (static_cast<size_t>(budget) + 1) * 8);
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
  const size_t smem = tree_smem_bytes(budget);
  if (smem > 227 * 1024) return fail(SG_ERR_UNSUPPORTED, "sg_build_draft_trees: budget too large");
  SG_CUDA_CHECK(cudaFuncSetAttribute(draft_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
  const int blocks = (num_trees + kTreeWarps - 1) / kTreeWarps;
  draft_tree_kernel<<<blocks, kTreeWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(p);
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
  pack_tree_wave_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      tokens, parents, budget, node_count, allocation, anchor_tokens, num_trees, max_rows, row_offsets, wave_parents,
      wave_tokens, status);
  return check_launch("pack_tree_wave_kernel");
}
