// Tree-sampling acceptance over packed fp32 probability rows (sm_100a).
//
// One thread-block cluster walks one request tree top-down.  At each visited
// node the cluster's CTAs split the node's probability row, reduce it to exact
// 64.64 fixed-point masses per 1024-token block (a warp per block, 32 tokens
// per lane; probabilities below 1 take a one-word fixed-point path), exchange
// their slice totals through distributed shared memory, and the CTA whose
// slice holds the inverse-CDF threshold locates the token with one
// 1024-token rescan in index order.  The walk
// then follows the matching child edge (warp ballot over the tree's nodes).
//
// Semantics follow the reference kernels
//   fused_tree_sampling.py:538-627 (scan rule: token = first index whose
//   inclusive prefix exceeds u[depth] * row_total; fallback V-1; stop when no
//   child matches or depth == max_depth), and
//   fused_tree_sampling.py:688-824 (sparse exit: route among children by
//   cumulative child mass against u[2d]; on exit draw from the row without the
//   children against u[2d+1]; fallback = last non-child token),
// with the fp64 running sums replaced by exact fixed-point sums so that the
// decision is independent of the reduction order.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace sg {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBlockElems = 1024;  // one warp x 8 float4 per lane
constexpr int kVecs = kBlockElems / 128;  // float4 loads per lane per block
constexpr int kMaxChildren = 256;

struct AcceptParams {
  const float* probs;
  int64_t vocab;
  const int64_t* row_offsets;
  const int64_t* parents;
  const int64_t* tokens;
  int32_t num_trees;
  int32_t max_nodes;
  int32_t max_depth;
  int32_t rule;
  const double* uniforms;
  int32_t uniform_stride;
  uint64_t seed;
  const int64_t* request_ids;
  int64_t* out;
  int32_t* status;
  int32_t blocks_per_cta;  // 128-token blocks per CTA slice
  bool aligned4;           // rows 16-byte aligned and vocab % 4 == 0
};

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status != nullptr) atomicMax(status, code);
}

// General path for a float4 with a value >= 1, negative or not finite (rare
// in probability rows), kept out of line so the common path stays short.
__device__ __noinline__ void accumulate4_general(Mass& big, uint4 v, uint32_t* bad) {
  big = mass_add(big, mass_from_bits(v.x, bad));
  big = mass_add(big, mass_from_bits(v.y, bad));
  big = mass_add(big, mass_from_bits(v.z, bad));
  big = mass_add(big, mass_from_bits(v.w, bad));
}

// Exact masses of four fp32 values into (lo, carry) — all four below 1.0 —
// or into `big` through the general path.
__device__ __forceinline__ void accumulate4(uint64_t& lo, uint32_t& carry, Mass& big, uint4 v, uint32_t* bad) {
  if (__builtin_expect(max(max(v.x, v.y), max(v.z, v.w)) < 0x3f800000u, 1)) {
    add_with_carry(lo, carry, mass_lo_f64(v.x));
    add_with_carry(lo, carry, mass_lo_f64(v.y));
    add_with_carry(lo, carry, mass_lo_f64(v.z));
    add_with_carry(lo, carry, mass_lo_f64(v.w));
  } else {
    accumulate4_general(big, v, bad);
  }
}

__device__ __forceinline__ Mass warp_sum(Mass v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    Mass o;
    o.lo = __shfl_xor_sync(0xffffffffu, v.lo, d);
    o.hi = __shfl_xor_sync(0xffffffffu, v.hi, d);
    v = mass_add(v, o);
  }
  return v;
}

__device__ __forceinline__ Mass warp_inclusive_scan(Mass v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    Mass o;
    o.lo = __shfl_up_sync(0xffffffffu, v.lo, d);
    o.hi = __shfl_up_sync(0xffffffffu, v.hi, d);
    if (lane >= d) v = mass_add(v, o);
  }
  return v;
}

// Four consecutive probabilities starting at `index` (zero beyond vocab).
__device__ __forceinline__ uint4 load4(const float* row, int64_t index, int64_t vocab, bool aligned4) {
  if (aligned4 && index + 3 < vocab) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(row + index));
    return make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z),
                      __float_as_uint(v.w));
  }
  uint4 r = make_uint4(0u, 0u, 0u, 0u);
  if (index + 0 < vocab) r.x = __float_as_uint(__ldg(row + index + 0));
  if (index + 1 < vocab) r.y = __float_as_uint(__ldg(row + index + 1));
  if (index + 2 < vocab) r.z = __float_as_uint(__ldg(row + index + 2));
  if (index + 3 < vocab) r.w = __float_as_uint(__ldg(row + index + 3));
  return r;
}

template <int CLUSTER>
__global__ void __launch_bounds__(kThreads, 1) accept_probs_kernel(const AcceptParams p) {
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned crank = cluster.block_rank();
  const int tree = static_cast<int>(blockIdx.x) / CLUSTER;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  extern __shared__ __align__(16) unsigned char smem_raw[];
  Mass* blk = reinterpret_cast<Mass*>(smem_raw);                        // [blocks_per_cta]
  int* s_parent = reinterpret_cast<int*>(blk + p.blocks_per_cta);       // [max_nodes]
  int* s_token = s_parent + p.max_nodes;                                // [max_nodes]

  __shared__ Mass s_cta_total;
  __shared__ Mass s_warp[kWarps];
  __shared__ int s_selected;       // written into every CTA by the owner
  __shared__ int s_bad_tree;
  __shared__ int s_child_count;
  __shared__ int s_child_node[kMaxChildren];
  __shared__ int s_child_tok[kMaxChildren];
  __shared__ int s_cross_block;
  __shared__ Mass s_cross_residual;

  const int64_t row0 = p.row_offsets[tree];
  const int n = static_cast<int>(p.row_offsets[tree + 1] - row0);
  const int D = p.max_depth;
  int64_t* out = p.out + static_cast<int64_t>(tree) * (D + 2);
  const uint64_t request = p.request_ids ? static_cast<uint64_t>(p.request_ids[tree])
                                         : static_cast<uint64_t>(tree);

  if (tid == 0) s_bad_tree = (n < 1 || n > p.max_nodes) ? 1 : 0;
  __syncthreads();
  if (s_bad_tree) {
    if (crank == 0 && tid == 0) report(p.status, SG_ERR_TREE);
    if (crank == 0)
      for (int i = tid; i < D + 2; i += kThreads) out[i] = -1;
    cluster.sync();
    return;
  }
  // Stage and validate the tree (parents[j] < j, tokens in range).
  for (int j = tid; j < n; j += kThreads) {
    const int64_t par = p.parents[row0 + j];
    const int64_t tok = p.tokens[row0 + j];
    s_parent[j] = static_cast<int>(par);
    s_token[j] = static_cast<int>(tok);
    const bool ok = (j == 0) ? (par == -1) : (par >= 0 && par < j && tok >= 0 && tok < p.vocab);
    if (!ok) atomicOr(&s_bad_tree, 1);
  }
  if (crank == 0)
    for (int i = tid; i < D + 2; i += kThreads) out[i] = -1;
  __syncthreads();
  if (s_bad_tree) {
    if (crank == 0 && tid == 0) report(p.status, SG_ERR_TREE);
    cluster.sync();
    return;
  }

  const int64_t V = p.vocab;
  const int64_t nblk_total = (V + kBlockElems - 1) / kBlockElems;
  const int64_t slice_first = static_cast<int64_t>(crank) * p.blocks_per_cta;
  const int nb = static_cast<int>(max64(0, min64(p.blocks_per_cta, nblk_total - slice_first)));

  int cur = 0;
  int accepted = 0;
  uint32_t bad_prob = 0u;
  for (int depth = 0; depth <= D; ++depth) {
    const float* row = p.probs + (row0 + cur) * V;
    double u_main, u_exit;
    if (p.uniforms != nullptr) {
      const double* ut = p.uniforms + static_cast<int64_t>(tree) * p.uniform_stride;
      if (p.rule == SG_RULE_SPARSE_EXIT) {
        u_main = ut[2 * depth];
        u_exit = ut[2 * depth + 1];
      } else {
        u_main = ut[depth];
        u_exit = 0.0;
      }
    } else {
      const NodeUniforms nu = node_uniforms(p.seed, request, static_cast<uint32_t>(cur));
      u_main = nu.route;
      u_exit = nu.exit;
    }
    if (!(u_main >= 0.0 && u_main < 1.0) || !(u_exit >= 0.0 && u_exit < 1.0)) {
      if (tid == 0 && crank == 0) report(p.status, SG_ERR_INVALID_ARGUMENT);
      u_main = (u_main >= 0.0 && u_main < 1.0) ? u_main : 0.0;
      u_exit = (u_exit >= 0.0 && u_exit < 1.0) ? u_exit : 0.0;
    }

    const bool sparse = (p.rule == SG_RULE_SPARSE_EXIT);
    if (sparse) {
      // Children of `cur` in node (edge) order.
      if (warp == 0) {
        int count = 0;
        for (int base = 1; base < n; base += 32) {
          const int j = base + lane;
          const bool hit = (j < n) && s_parent[j] == cur;
          const unsigned mask = __ballot_sync(0xffffffffu, hit);
          if (hit) {
            const int slot = count + __popc(mask & ((1u << lane) - 1u));
            if (slot < kMaxChildren) {
              s_child_node[slot] = j;
              s_child_tok[slot] = s_token[j];
            }
          }
          count += __popc(mask);
        }
        if (lane == 0) s_child_count = count;
      }
      __syncthreads();
      if (s_child_count > kMaxChildren) {
        if (tid == 0 && crank == 0) report(p.status, SG_ERR_UNSUPPORTED);
        break;
      }
      // Route: first child whose exact cumulative mass exceeds u * 1.
      int route = -1;
      {
        const Mass thr = mass_scale(u_main, Mass{0ull, 1ull});
        Mass cum = mass_zero();
        uint32_t bad = 0u;
        for (int c = 0; c < s_child_count; ++c) {
          const float v = __ldg(row + s_child_tok[c]);
          cum = mass_add(cum, mass_from_bits(__float_as_uint(v), &bad));
          if (mass_lt(thr, cum)) {
            route = s_child_node[c];
            break;
          }
        }
        bad_prob |= bad;
      }
      if (route >= 0 && depth < D) {
        if (crank == 0 && tid == 0) out[accepted] = route;
        ++accepted;
        cur = route;
        __syncthreads();
        continue;
      }
    }

    // ---- full-row pass: exact mass of every 1024-token block of this slice
    // (lane l reads float4 l of each 512-byte segment, so every load
    // instruction is one contiguous 512 bytes; 8 loads per lane in flight).
    for (int b = warp; b < nb; b += kWarps) {
      uint4 v[kVecs];
#pragma unroll
      for (int k = 0; k < kVecs; ++k)
        v[k] = load4(row, (slice_first + b) * kBlockElems + k * 128 + lane * 4, V, p.aligned4);
      uint64_t lo = 0ull;
      uint32_t carry = 0u;
      Mass big = mass_zero();
#pragma unroll
      for (int k = 0; k < kVecs; ++k) accumulate4(lo, carry, big, v[k], &bad_prob);
      Mass s = mass_add(Mass{lo, carry}, big);
      s = warp_sum(s);
      if (lane == 0) blk[b] = s;
    }
    __syncthreads();
    if (sparse && tid == 0) {
      // Remove the children's mass from their blocks (exact subtraction).
      uint32_t bad = 0u;
      for (int c = 0; c < s_child_count; ++c) {
        const int64_t tok = s_child_tok[c];
        const int64_t b = tok / kBlockElems - slice_first;
        if (b >= 0 && b < nb) {
          const float v = __ldg(row + tok);
          blk[b] = mass_sub(blk[b], mass_from_bits(__float_as_uint(v), &bad));
        }
      }
    }
    __syncthreads();
    // CTA total.
    {
      Mass s = mass_zero();
      for (int b = tid; b < nb; b += kThreads) s = mass_add(s, blk[b]);
      s = warp_sum(s);
      if (lane == 0) s_warp[warp] = s;
      __syncthreads();
      if (warp == 0) {
        Mass t = (lane < kWarps) ? s_warp[lane] : mass_zero();
        t = warp_sum(t);
        if (lane == 0) s_cta_total = t;
      }
      if (tid == 0) s_selected = -1;
    }
    cluster.sync();

    // Grand total and this CTA's exclusive prefix (identical in every CTA).
    Mass total = mass_zero(), prefix = mass_zero(), mine = mass_zero();
#pragma unroll
    for (int r = 0; r < CLUSTER; ++r) {
      const Mass* remote = cluster.map_shared_rank(&s_cta_total, r);
      const Mass t = *remote;
      if (r < static_cast<int>(crank)) prefix = mass_add(prefix, t);
      if (r == static_cast<int>(crank)) mine = t;
      total = mass_add(total, t);
    }
    const Mass thr = mass_scale(sparse ? u_exit : u_main, total);
    const bool owner = !mass_is_zero(total) && !mass_lt(thr, prefix) &&
                       mass_lt(thr, mass_add(prefix, mine));
    if (owner) {
      // Find the crossing block: contiguous runs of blocks per thread.
      const Mass local = mass_sub(thr, prefix);
      const int per = (nb + kThreads - 1) / kThreads;
      const int b0 = min(nb, tid * per), b1 = min(nb, b0 + per);
      Mass s = mass_zero();
      for (int b = b0; b < b1; ++b) s = mass_add(s, blk[b]);
      Mass incl = warp_inclusive_scan(s, lane);
      if (lane == 31) s_warp[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        Mass w = (lane < kWarps) ? s_warp[lane] : mass_zero();
        Mass wi = warp_inclusive_scan(w, lane);
        if (lane < kWarps) s_warp[lane] = mass_sub(wi, w);  // exclusive
      }
      __syncthreads();
      const Mass excl = mass_add(s_warp[warp], mass_sub(incl, s));
      if (b0 < b1 && !mass_lt(local, excl) && mass_lt(local, mass_add(excl, s))) {
        Mass run = excl;
        for (int b = b0; b < b1; ++b) {
          const Mass next = mass_add(run, blk[b]);
          if (mass_lt(local, next)) {
            s_cross_block = b;
            s_cross_residual = mass_sub(local, run);
            break;
          }
          run = next;
        }
      }
      __syncthreads();
      if (warp == 0) {
        // Rescan the crossing block in index order: lane l owns tokens
        // [first, first + 32) with first = block start + 32 l.
        const int b = s_cross_block;
        const Mass resid = s_cross_residual;
        const int64_t first = (slice_first + b) * kBlockElems + lane * (kBlockElems / 32);
        uint32_t e[kBlockElems / 32];
#pragma unroll
        for (int k = 0; k < kBlockElems / 128; ++k) {
          const uint4 v = load4(row, first + k * 4, V, p.aligned4);
          e[4 * k] = v.x;
          e[4 * k + 1] = v.y;
          e[4 * k + 2] = v.z;
          e[4 * k + 3] = v.w;
        }
        uint32_t bad = 0u;
        if (sparse) {  // children are excluded from the exit draw
          for (int c = 0; c < s_child_count; ++c) {
            const int64_t off = s_child_tok[c] - first;
#pragma unroll
            for (int k = 0; k < kBlockElems / 32; ++k)
              if (off == k) e[k] = 0u;
          }
        }
        uint64_t lo = 0ull;
        uint32_t carry = 0u;
        Mass big = mass_zero();
#pragma unroll
        for (int k = 0; k < kBlockElems / 128; ++k)
          accumulate4(lo, carry, big, make_uint4(e[4 * k], e[4 * k + 1], e[4 * k + 2], e[4 * k + 3]), &bad);
        const Mass lane_sum = mass_add(Mass{lo, carry}, big);
        const Mass li = warp_inclusive_scan(lane_sum, lane);
        Mass run = mass_sub(li, lane_sum);
        int found = -1;
        if (!mass_lt(resid, run) && mass_lt(resid, li)) {
#pragma unroll
          for (int k = 0; k < kBlockElems / 32; ++k) {
            mass_accumulate(run, e[k], &bad);
            if (found < 0 && mass_lt(resid, run)) found = k;
          }
        }
        const unsigned who = __ballot_sync(0xffffffffu, found >= 0);
        if (who != 0u) {
          const int src = __ffs(who) - 1;
          const int fk = __shfl_sync(0xffffffffu, found, src);
          if (lane == 0) {
            const int token = static_cast<int>((slice_first + b) * kBlockElems + src * (kBlockElems / 32) + fk);
#pragma unroll
            for (int r = 0; r < CLUSTER; ++r) *cluster.map_shared_rank(&s_selected, r) = token;
          }
        }
      }
    }
    cluster.sync();

    int token = s_selected;
    if (token < 0) {
      // Zero total (or a final boundary): reference fallbacks.
      if (!sparse) {
        token = static_cast<int>(V - 1);
      } else {
        for (int64_t t = V - 1; t >= 0; --t) {
          bool is_child = false;
          for (int c = 0; c < s_child_count; ++c) is_child = is_child || (s_child_tok[c] == t);
          if (!is_child) {
            token = static_cast<int>(t);
            break;
          }
        }
      }
    }
    int child = -1;
    if (!sparse) {
      // First node with (parent, token) == (cur, token).
      for (int base = 1; base < n; base += 32) {
        const int j = base + lane;
        const bool hit = (j < n) && s_parent[j] == cur && s_token[j] == token;
        const unsigned mask = __ballot_sync(0xffffffffu, hit);
        if (mask != 0u) {
          child = base + __ffs(mask) - 1;
          break;
        }
      }
    }
    if (child >= 0 && depth < D) {
      if (crank == 0 && tid == 0) out[accepted] = child;
      ++accepted;
      cur = child;
      __syncthreads();
      continue;
    }
    if (crank == 0 && tid == 0) {
      out[D] = accepted;
      out[D + 1] = token;
    }
    break;
  }
  if (bad_prob) report(p.status, SG_ERR_PROBABILITY);
  cluster.sync();
}

__global__ void follow_kernel(const int64_t* __restrict__ posterior, const int64_t* __restrict__ row_offsets,
                              const int64_t* __restrict__ parents, const int64_t* __restrict__ tokens,
                              int32_t num_trees, int32_t max_nodes, int32_t max_depth,
                              int64_t* __restrict__ out_all, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int tree = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tree >= num_trees) return;
  const int64_t row0 = row_offsets[tree];
  const int n = static_cast<int>(row_offsets[tree + 1] - row0);
  const int D = max_depth;
  int64_t* out = out_all + static_cast<int64_t>(tree) * (D + 2);
  for (int i = lane; i < D + 2; i += 32) out[i] = -1;
  __syncwarp();
  if (n < 1 || n > max_nodes) {
    if (lane == 0) report(status, SG_ERR_TREE);
    return;
  }
  int cur = 0, accepted = 0;
  int64_t bonus = posterior[row0];
  for (int depth = 0; depth < D; ++depth) {
    int child = -1;
    for (int base = 1; base < n; base += 32) {
      const int j = base + lane;
      const bool hit = (j < n) && parents[row0 + j] == cur && tokens[row0 + j] == bonus;
      const unsigned mask = __ballot_sync(0xffffffffu, hit);
      if (mask != 0u) {
        child = base + __ffs(mask) - 1;
        break;
      }
    }
    if (child < 0) break;
    if (lane == 0) out[accepted] = child;
    ++accepted;
    cur = child;
    bonus = posterior[row0 + cur];
  }
  if (lane == 0) {
    out[D] = accepted;
    out[D + 1] = bonus;
  }
}

template <int CLUSTER>
int launch_accept(const AcceptParams& p, size_t smem, cudaStream_t stream) {
  auto kernel = accept_probs_kernel<CLUSTER>;
  SG_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.num_trees) * CLUSTER, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CLUSTER;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SG_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, p));
  return check_launch("accept_probs_kernel");
}

}  // namespace
}  // namespace sg

extern "C" int sg_tree_accept_probs(const float* probs, int64_t vocab, const int64_t* row_offsets,
                                    const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                                    int32_t max_nodes, int32_t max_depth, int32_t rule,
                                    const double* uniforms, int32_t uniform_stride, uint64_t seed,
                                    const int64_t* request_ids, int64_t* out, int32_t* status,
                                    void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (probs == nullptr || row_offsets == nullptr || parents == nullptr || tokens == nullptr ||
      out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: null pointer");
  if (num_trees < 0 || vocab < 1 || vocab > (int64_t(1) << 30) || max_depth < 0 ||
      max_nodes < 1 || max_nodes > (1 << 16))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: bad sizes");
  if (rule != SG_RULE_SCAN && rule != SG_RULE_SPARSE_EXIT)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: unknown rule");
  if (uniforms != nullptr) {
    const int need = (rule == SG_RULE_SCAN) ? max_depth + 1 : 2 * (max_depth + 1);
    if (uniform_stride < need)
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: uniforms do not cover every depth");
  }
  const int sms = device_sm_count();
  if (sms <= 0) return fail(SG_ERR_CUDA, "sg_tree_accept_probs: no CUDA device");
  int cluster = 1;
  while (cluster < 8 && static_cast<int64_t>(num_trees) * cluster * 2 <= sms) cluster *= 2;
  const int64_t nblk = (vocab + kBlockElems - 1) / kBlockElems;
  AcceptParams p;
  p.probs = probs;
  p.vocab = vocab;
  p.row_offsets = row_offsets;
  p.parents = parents;
  p.tokens = tokens;
  p.num_trees = num_trees;
  p.max_nodes = max_nodes;
  p.max_depth = max_depth;
  p.rule = rule;
  p.uniforms = uniforms;
  p.uniform_stride = uniform_stride;
  p.seed = seed;
  p.request_ids = request_ids;
  p.out = out;
  p.status = status;
  p.aligned4 = (vocab % 4 == 0) && (reinterpret_cast<uintptr_t>(probs) % 16 == 0);
  size_t smem = 0;
  for (;;) {
    p.blocks_per_cta = static_cast<int32_t>((nblk + cluster - 1) / cluster);
    smem = static_cast<size_t>(p.blocks_per_cta) * sizeof(Mass) + static_cast<size_t>(max_nodes) * 8;
    if (smem <= 160 * 1024 || cluster == 8) break;
    cluster *= 2;
  }
  if (smem > 200 * 1024) return fail(SG_ERR_UNSUPPORTED, "sg_tree_accept_probs: vocabulary too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (cluster) {
    case 1: return launch_accept<1>(p, smem, s);
    case 2: return launch_accept<2>(p, smem, s);
    case 4: return launch_accept<4>(p, smem, s);
    default: return launch_accept<8>(p, smem, s);
  }
}

extern "C" int sg_tree_follow(const int64_t* posterior, const int64_t* row_offsets, const int64_t* parents,
                              const int64_t* tokens, int32_t num_trees, int32_t max_nodes,
                              int32_t max_depth, int64_t* out, int32_t* status, void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (posterior == nullptr || row_offsets == nullptr || parents == nullptr || tokens == nullptr ||
      out == nullptr || num_trees < 0 || max_depth < 0 || max_nodes < 1)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_follow: bad arguments");
  const int warps_per_block = 4;
  const unsigned grid = static_cast<unsigned>((num_trees + warps_per_block - 1) / warps_per_block);
  follow_kernel<<<grid, warps_per_block * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      posterior, row_offsets, parents, tokens, num_trees, max_nodes, max_depth, out, status);
  return check_launch("follow_kernel");
}
