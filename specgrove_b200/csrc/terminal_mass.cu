// Terminal-mass tree verifier: the law of ancestral tree sampling drawn as
// one terminal node and one bonus token (sampling.py:542-735,
// tree_block_verify_terminal_mass with its default exit_mode "internal" and
// prefix_mode "batched"; the decoder's default verifier,
// continuous_tree_block_decode.py:1328).
//
// For node v with children C(v): its row mass is total(v) = sum_t p_v[t], its
// exit mass tail(v) = total(v) - sum_{c in C(v)} p_v[tok(c)] (1 for a leaf, as
// a fraction tail/total), each edge's normalised probability
// p_v[tok(c)] / total(v), and prefix(v) the product of the normalised edge
// probabilities from the root.  The terminal node is drawn from
// prefix(v) * exit(v), then the bonus token from v's row with its children's
// tokens removed (the whole row for a leaf).
//
// Arithmetic: row masses are exact 64.64 fixed-point sums of the fp32
// probabilities (the acceptance kernels' arithmetic, order independent),
// tail(v) = total(v) - children's masses exactly; they become fp64 by one
// correctly rounded conversion.  Normalisation, prefix products, terminal
// masses and the terminal-node draw run in fp64 on one thread in node order;
// the bonus token is the exact fixed-point inverse CDF over the exit row.
// The C oracle follows the same steps, so decisions agree bit for bit; the
// reference's own fp64 sums differ from these only by rounding.
//
// Two launches: row_mass_kernel sums the rows of internal nodes (one CTA
// per packed row with coalesced loads, leaves return at once),
// terminal_kernel (one CTA per tree) does the rest; its bonus draw sums the
// exit row in 512-token chunks (a warp each), finds the crossing chunk and
// scans it with one warp.
#include <cuda_runtime.h>

#include "common.cuh"
#include "layers.cuh"

namespace sg {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxChunks = 512;  // exit-row chunks of the bonus draw

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status != nullptr) atomicMax(status, code);
}

__device__ __forceinline__ Mass shfl_down_mass(Mass v, int d) {
  Mass r;
  r.lo = __shfl_down_sync(0xffffffffu, v.lo, d);
  r.hi = __shfl_down_sync(0xffffffffu, v.hi, d);
  return r;
}

__device__ __forceinline__ Mass shfl_up_mass(Mass v, int d) {
  Mass r;
  r.lo = __shfl_up_sync(0xffffffffu, v.lo, d);
  r.hi = __shfl_up_sync(0xffffffffu, v.hi, d);
  return r;
}

// Exact block sum (every thread returns the total).
__device__ Mass block_sum(Mass v, Mass* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = mass_add(v, shfl_down_mass(v, d));
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  Mass t = mass_zero();
  for (int w = 0; w < kWarps; ++w) t = mass_add(t, sh[w]);
  __syncthreads();
  return t;
}

// Exact mass of a whole row, coalesced: thread i takes float4s i, i + n,
// i + 2n, ... (the sum is exact, so the partition does not matter), eight
// loads in flight per thread.
__device__ Mass row_mass_strided(const uint32_t* bits, int64_t vocab, bool vec, uint32_t* bad) {
  Mass acc = mass_zero();
  const int64_t nthr = blockDim.x;
  if (vec) {
    const uint4* q4 = reinterpret_cast<const uint4*>(bits);
    const int64_t n4 = vocab / 4;
    int64_t i = threadIdx.x;
    for (; i + 7 * nthr < n4; i += 8 * nthr) {
      uint4 q[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = q4[i + k * nthr];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        mass_accumulate(acc, q[k].x, bad);
        mass_accumulate(acc, q[k].y, bad);
        mass_accumulate(acc, q[k].z, bad);
        mass_accumulate(acc, q[k].w, bad);
      }
    }
    for (; i < n4; i += nthr) {
      const uint4 q = q4[i];
      mass_accumulate(acc, q.x, bad);
      mass_accumulate(acc, q.y, bad);
      mass_accumulate(acc, q.z, bad);
      mass_accumulate(acc, q.w, bad);
    }
    for (int64_t t = n4 * 4 + threadIdx.x; t < vocab; t += nthr) mass_accumulate(acc, bits[t], bad);
  } else {
    for (int64_t t = threadIdx.x; t < vocab; t += nthr) mass_accumulate(acc, bits[t], bad);
  }
  return acc;
}

// Tree of packed row `row`: the largest t with row_offsets[t] <= row.
__device__ int tree_of_row(const int64_t* row_offsets, int num_trees, int64_t row) {
  int lo = 0, hi = num_trees - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (row_offsets[mid] <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kThreads) row_mass_kernel(const float* __restrict__ probs, int64_t vocab,
                                                           const int64_t* __restrict__ row_offsets,
                                                           const int64_t* __restrict__ parents, int num_trees,
                                                           Mass* __restrict__ totals, int32_t* status) {
  __shared__ Mass sh[kWarps];
  const int64_t row = blockIdx.x;
  const int t = tree_of_row(row_offsets, num_trees, row);
  const int64_t r0 = row_offsets[t], r1 = row_offsets[t + 1];
  if (row < r0 || row >= r1) {  // a row past the last tree
    if (threadIdx.x == 0) totals[row] = mass_zero();
    return;
  }
  const int64_t j = row - r0;
  int internal = 0;
  for (int64_t c = j + 1 + threadIdx.x; c < r1 - r0; c += blockDim.x)
    if (parents[r0 + c] == j) internal = 1;
  if (!__syncthreads_or(internal)) {
    if (threadIdx.x == 0) totals[row] = mass_zero();
    return;
  }
  const float* p = probs + row * vocab;
  const bool vec = (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
  uint32_t bad = 0;
  const Mass m = row_mass_strided(reinterpret_cast<const uint32_t*>(p), vocab, vec, &bad);
  const Mass total = block_sum(m, sh);
  const int any_bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    // an invalid probability marks the row (no valid sum reaches 2^127)
    totals[row] = any_bad ? Mass{~0ull, ~0ull} : total;
    if (any_bad) report(status, SG_ERR_PROBABILITY);
  }
}

struct TerminalArgs {
  const float* probs;
  int64_t vocab;
  const int64_t* row_offsets;
  const int64_t* parents;
  const int64_t* tokens;
  int num_trees;
  int max_depth;
  const double* uniforms;
  int uniform_stride;
  uint64_t seed;
  const int64_t* request_ids;
  const Mass* totals;
  int64_t total_rows;  // rows covered by `totals`
  int64_t* out;
  int32_t* status;
};

__global__ void __launch_bounds__(kThreads) terminal_kernel(const TerminalArgs a) {
  using layers::kMaxTreeRows;
  __shared__ int32_t par[kMaxTreeRows];
  __shared__ int64_t tok[kMaxTreeRows];
  __shared__ int32_t dep[kMaxTreeRows];
  __shared__ int64_t s_child_tok[kMaxTreeRows];
  __shared__ double prefix[kMaxTreeRows], term[kMaxTreeRows];
  __shared__ Mass covered[kMaxTreeRows], edge[kMaxTreeRows], tot[kMaxTreeRows];
  __shared__ bool internal[kMaxTreeRows];
  __shared__ int s_nchild, s_pick, s_fail, s_cross;
  __shared__ Mass s_exit_total, s_before, s_thr;
  __shared__ Mass s_chunk[kMaxChunks];
  __shared__ int64_t s_bonus;
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int64_t D = a.max_depth;
  int64_t* out = a.out + static_cast<int64_t>(t) * (D + 2);
  for (int64_t i = threadIdx.x; i < D + 2; i += blockDim.x) out[i] = -1;
  const int64_t r0 = a.row_offsets[t];
  const int64_t n64 = a.row_offsets[t + 1] - r0;
  const int n = static_cast<int>(n64);
  if (r0 < 0 || n64 < 1 || n64 > kMaxTreeRows || r0 + n64 > a.total_rows) {  // rows beyond total_rows have no sums
    if (threadIdx.x == 0) report(a.status, SG_ERR_TREE);
    return;
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    par[j] = static_cast<int32_t>(a.parents[r0 + j]);
    tok[j] = a.tokens[r0 + j];
  }
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  // topology: root first, parents precede, tokens in range, depth <= D
  if (threadIdx.x == 0) {
    int fail = par[0] != -1;
    dep[0] = 0;
    for (int j = 1; j < n && !fail; ++j) {
      if (par[j] < 0 || par[j] >= j || tok[j] < 0 || tok[j] >= a.vocab) fail = 1;
      else dep[j] = dep[par[j]] + 1;
      if (!fail && dep[j] > D) fail = 1;
    }
    s_fail = fail;
  }
  __syncthreads();
  if (!s_fail) {  // no node repeats a child token (pairs i < j)
    int dup = 0;
    for (int pair = threadIdx.x; pair < n * n; pair += blockDim.x) {
      const int i = pair / n, j = pair % n;
      if (i >= 1 && i < j && par[i] == par[j] && tok[i] == tok[j]) dup = 1;
    }
    if (__syncthreads_or(dup) && threadIdx.x == 0) s_fail = 1;
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) report(a.status, SG_ERR_TREE);
    return;
  }
  double u_node, u_bonus;
  if (a.uniforms != nullptr) {
    u_node = a.uniforms[static_cast<int64_t>(t) * a.uniform_stride];
    u_bonus = a.uniforms[static_cast<int64_t>(t) * a.uniform_stride + 1];
  } else {
    const uint64_t req = a.request_ids != nullptr ? static_cast<uint64_t>(a.request_ids[t]) : static_cast<uint64_t>(t);
    const U32x4 r = philox4x32_10(U32x4{0u, static_cast<uint32_t>(req), static_cast<uint32_t>(req >> 32), 2u},
                                  static_cast<uint32_t>(a.seed), static_cast<uint32_t>(a.seed >> 32));
    u_node = uniform53(r.x, r.y);
    u_bonus = uniform53(r.z, r.w);
  }
  // The edge probabilities and row totals come into shared memory in
  // parallel; the masses and the terminal-node draw then run on one thread in
  // node order.
  {
    uint32_t bad_e = 0;
    const uint32_t* rows = reinterpret_cast<const uint32_t*>(a.probs);
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      edge[j] = j > 0 ? mass_from_bits(rows[(r0 + par[j]) * a.vocab + tok[j]], &bad_e) : mass_zero();
      tot[j] = a.totals[r0 + j];
    }
    if (__syncthreads_or(bad_e) && threadIdx.x == 0) s_fail = SG_ERR_PROBABILITY;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    uint32_t bad = s_fail != 0;
    for (int j = 0; j < n; ++j) {
      covered[j] = mass_zero();
      internal[j] = false;
    }
    for (int j = 1; j < n; ++j) {
      covered[par[j]] = mass_add(covered[par[j]], edge[j]);
      internal[par[j]] = true;
    }
    double total_term = 0.0;
    prefix[0] = 1.0;
    int fail = bad ? SG_ERR_PROBABILITY : 0;
    for (int j = 0; j < n && !fail; ++j) {
      if (j > 0) {
        const Mass pt = tot[par[j]];
        if (pt.hi == ~0ull) {
          fail = SG_ERR_PROBABILITY;
          break;
        }
        prefix[j] = prefix[par[j]] * (mass_to_double(edge[j]) / mass_to_double(pt));
      }
      double exit_frac = 1.0;
      if (internal[j]) {
        const Mass total = tot[j];
        if (total.hi == ~0ull || mass_is_zero(total) || mass_lt(total, covered[j])) {
          fail = SG_ERR_PROBABILITY;
          break;
        }
        exit_frac = mass_to_double(mass_sub(total, covered[j])) / mass_to_double(total);
      }
      term[j] = prefix[j] * exit_frac;
      total_term += term[j];
    }
    int pick = -1;
    if (!fail && total_term > 0.0 && isfinite(total_term)) {
      const double thr = u_node * total_term;
      double cum = 0.0;
      for (int j = 0; j < n; ++j) {
        cum += term[j];
        if (term[j] > 0.0) pick = j;  // the last positive one, if rounding leaves cum <= thr
        if (cum > thr && term[j] > 0.0) break;
      }
    }
    if (!fail && pick < 0) fail = SG_ERR_PROBABILITY;
    s_fail = fail;
    s_pick = pick;
    if (!fail) {
      s_exit_total = internal[pick] ? mass_sub(tot[pick], covered[pick]) : mass_zero();
      int k = 0;
      for (int j = 1; j < n; ++j)
        if (par[j] == pick) s_child_tok[k++] = tok[j];
      s_nchild = k;
    }
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) report(a.status, s_fail);
    return;
  }
  const int v = s_pick;
  const int k = s_nchild;
  const float* row = a.probs + (r0 + v) * a.vocab;
  const uint32_t* rbits = reinterpret_cast<const uint32_t*>(row);
  const bool vec = (a.vocab & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // The exit row in chunks of `ch` tokens (a multiple of 512, at most
  // kMaxChunks chunks), each summed by one warp with coalesced loads; the
  // children's tokens leave their chunk's mass.
  const int64_t ch = 512 * ((a.vocab + 512 * kMaxChunks - 1) / (512 * kMaxChunks));
  const int nch = static_cast<int>((a.vocab + ch - 1) / ch);
  uint32_t bad = 0;
  for (int c = warp; c < nch; c += kWarps) {
    const int64_t c0 = c * ch, c1 = min64(a.vocab, c0 + ch);
    Mass acc = mass_zero();
    if (vec) {
      const uint4* q4 = reinterpret_cast<const uint4*>(rbits + c0);
      const int64_t n4 = (c1 - c0) / 4;  // a multiple of 4 tokens when vocab is
      for (int64_t x = lane; x < n4; x += 32) {
        const uint4 q = q4[x];
        mass_accumulate(acc, q.x, &bad);
        mass_accumulate(acc, q.y, &bad);
        mass_accumulate(acc, q.z, &bad);
        mass_accumulate(acc, q.w, &bad);
      }
    } else {
      for (int64_t x = c0 + lane; x < c1; x += 32) mass_accumulate(acc, rbits[x], &bad);
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) acc = mass_add(acc, shfl_down_mass(acc, d));
    if (lane == 0) {
      for (int e = 0; e < k; ++e) {
        const int64_t ct = s_child_tok[e];
        if (ct >= c0 && ct < c1) acc = mass_sub(acc, mass_from_bits(rbits[ct], &bad));
      }
      s_chunk[c] = acc;
    }
  }
  if (threadIdx.x == 0) s_bonus = -1;
  __syncthreads();
  // The crossing chunk: thread 0 walks the chunk masses in order.
  if (threadIdx.x == 0) {
    Mass total = s_exit_total;
    if (k == 0) {  // a leaf: its whole row
      total = mass_zero();
      for (int c = 0; c < nch; ++c) total = mass_add(total, s_chunk[c]);
    }
    s_cross = -1;
    if (!mass_is_zero(total)) {
      const Mass thr = mass_scale(u_bonus, total);
      Mass run = mass_zero();
      for (int c = 0; c < nch; ++c) {
        const Mass next = mass_add(run, s_chunk[c]);
        if (mass_lt(thr, next)) {
          s_cross = c;
          s_before = run;
          s_thr = thr;
          break;
        }
        run = next;
      }
    }
  }
  __syncthreads();
  if (s_cross < 0) {  // zero exit mass: no token to draw
    if (threadIdx.x == 0) report(a.status, SG_ERR_PROBABILITY);
    return;
  }
  if (warp == 0) {
    // Inside the crossing chunk: lane l takes tokens [c0 + l * per, ...), a
    // warp scan gives each lane the mass before its run, and the lane whose
    // run crosses the threshold walks it.
    const int64_t c0 = static_cast<int64_t>(s_cross) * ch, c1 = min64(a.vocab, c0 + ch);
    const int64_t per = ch / 32;
    const int64_t l0 = min64(c1, c0 + lane * per), l1 = min64(c1, l0 + per);
    auto excluded = [&](int64_t x) {
      bool e = false;
      for (int c = 0; c < k; ++c) e |= s_child_tok[c] == x;
      return e;
    };
    Mass mine = mass_zero();
    for (int64_t x = l0; x < l1; ++x)
      if (!excluded(x)) mine = mass_add(mine, mass_from_bits(rbits[x], &bad));
    Mass inc = mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const Mass o = shfl_up_mass(inc, d);
      if (lane >= d) inc = mass_add(inc, o);
    }
    Mass run = mass_add(s_before, mass_sub(inc, mine));
    const Mass thr = s_thr;
    if (!mass_lt(thr, run) && mass_lt(thr, mass_add(run, mine))) {
      for (int64_t x = l0; x < l1; ++x) {
        if (excluded(x)) continue;
        run = mass_add(run, mass_from_bits(rbits[x], &bad));
        if (mass_lt(thr, run)) {
          s_bonus = x;
          break;
        }
      }
    }
  }
  if (__syncthreads_or(bad)) {  // the terminal row holds an invalid probability
    if (threadIdx.x == 0) report(a.status, SG_ERR_PROBABILITY);
    return;
  }
  if (threadIdx.x == 0) {
    if (s_bonus < 0) {
      report(a.status, SG_ERR_PROBABILITY);
      return;
    }
    const int count = dep[v];
    for (int x = v, i = count - 1; x != 0; x = par[x], --i) out[i] = x;
    out[D] = count;
    out[D + 1] = s_bonus;
  }
}

}  // namespace
}  // namespace sg

extern "C" size_t sg_tree_verify_terminal_mass_workspace_bytes(int64_t total_rows) {
  if (total_rows < 0) return 0;
  return static_cast<size_t>(total_rows) * sizeof(sg::Mass) + 256;
}

extern "C" int sg_tree_verify_terminal_mass(const float* probs, int64_t vocab, const int64_t* row_offsets,
                                            const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                                            int64_t total_rows, int32_t max_depth, const double* uniforms,
                                            int32_t uniform_stride, uint64_t seed, const int64_t* request_ids,
                                            int64_t* out, int32_t* status, void* workspace, size_t workspace_bytes,
                                            void* stream_ptr) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (probs == nullptr || row_offsets == nullptr || parents == nullptr || tokens == nullptr || out == nullptr ||
      num_trees < 0 || total_rows < 1 || vocab < 1 || max_depth < 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_verify_terminal_mass: bad argument");
  if (uniforms != nullptr && uniform_stride < 2)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_verify_terminal_mass: uniform_stride must be >= 2");
  if (total_rows > (int64_t{1} << 31) - 1)
    return fail(SG_ERR_UNSUPPORTED, "sg_tree_verify_terminal_mass: too many rows");
  if (workspace == nullptr || workspace_bytes < sg_tree_verify_terminal_mass_workspace_bytes(total_rows) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return fail(SG_ERR_WORKSPACE, "sg_tree_verify_terminal_mass: workspace too small or not 16-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  Mass* totals = static_cast<Mass*>(workspace);
  row_mass_kernel<<<static_cast<unsigned>(total_rows), kThreads, 0, stream>>>(probs, vocab, row_offsets, parents,
                                                                             num_trees, totals, status);
  int st = check_launch("row_mass_kernel");
  if (st != SG_OK) return st;
  TerminalArgs a{probs, vocab, row_offsets, parents, tokens, num_trees, max_depth, uniforms, uniform_stride,
                 seed, request_ids, totals, total_rows, out, status};
  return launch_pdl("terminal_kernel", terminal_kernel, dim3(static_cast<unsigned>(num_trees)), dim3(kThreads), 0,
                    stream, a);
}
