// Tree-sampling acceptance straight from logit rows (sm_100a): the
// direct-logits verifiers of the reference (fused_tree_sampling.py:942-1115
// fused_tree_sample_logits_scan_kernel, :1117-1236 its batched form, used by
// tree_verify_ancestral_logits_fused_scan(_batched), :2417-2533), which
// normalise and walk only the visited rows instead of materialising a
// node x vocabulary probability matrix.
//
// At each visited node (reference semantics):
//   x_j = double(logit_j) / T,  w_j = exp(x_j - max_j x_j)   (fp64)
//   token = first j whose inclusive prefix of w exceeds u[depth] * sum(w),
//   fallback V - 1; child = first edge (node order) with that (parent,
//   token); stop when there is none or depth == max_depth.
// The prefix sums are exact 64.64 fixed-point sums of floor(w_j * 2^64), so
// the decision does not depend on the reduction order (it can differ from
// the reference's fp64 running sum only when u * total lies within ~1e-16
// relative of a boundary).
//
// One thread-block cluster walks one tree.  Each visited row costs two
// cluster barriers: one after every CTA's slice maximum (read by all CTAs
// through distributed shared memory), one after the slice masses; the
// selection then runs identically in warp 0 of every CTA, as in the
// probability kernel (accept.cu).  Buffers written in a pass are double
// buffered by pass parity, so a buffer is rewritten only two passes later,
// after barriers every reader has passed.
#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include <mutex>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace sg {
namespace {

constexpr int kLThreads = 256;
constexpr int kLWarps = kLThreads / 32;
constexpr int kLBlock = 1024;  // tokens per block: 32 steps of 32 consecutive tokens
constexpr int kLMaxCluster = 8;

struct LogitsParams {
  const void* logits;
  int dtype;  // 0 fp32, 1 bf16
  int64_t vocab;
  const int64_t* row_offsets;
  const int64_t* parents;
  const int64_t* tokens;
  int32_t num_trees, max_nodes, max_depth;
  double inv_temp;
  const double* uniforms;
  int32_t uniform_stride;
  uint64_t seed;
  const int64_t* request_ids;
  int64_t* out;
  int32_t* status;
  int32_t blocks_per_cta;
};

__device__ __forceinline__ void lreport(int32_t* status, int code) {
  if (status != nullptr) atomicMax(status, code);
}

template <typename T>
__device__ __forceinline__ float logit_at(const T* row, int64_t j);
template <>
__device__ __forceinline__ float logit_at<float>(const float* row, int64_t j) {
  return __ldg(row + j);
}
template <>
__device__ __forceinline__ float logit_at<__nv_bfloat16>(const __nv_bfloat16* row, int64_t j) {
  return __bfloat162float(row[j]);
}

// floor(w * 2^64) of a weight w in [0, 1] as a 64.64 mass (w == 1: 2^64).
__device__ __forceinline__ Mass weight_mass(double w) {
  if (w >= 1.0) return Mass{0ull, 1ull};
  return Mass{__double2ull_rz(w * 0x1p64), 0ull};
}

__device__ __forceinline__ Mass lwarp_sum(Mass v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    Mass o;
    o.lo = __shfl_xor_sync(0xffffffffu, v.lo, d);
    o.hi = __shfl_xor_sync(0xffffffffu, v.hi, d);
    v = mass_add(v, o);
  }
  return v;
}

__device__ __forceinline__ Mass lwarp_scan(Mass v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    Mass o;
    o.lo = __shfl_up_sync(0xffffffffu, v.lo, d);
    o.hi = __shfl_up_sync(0xffffffffu, v.hi, d);
    if (lane >= d) v = mass_add(v, o);
  }
  return v;
}

__device__ __forceinline__ Mass lshfl(Mass v, int src) {
  return Mass{__shfl_sync(0xffffffffu, v.lo, src), __shfl_sync(0xffffffffu, v.hi, src)};
}

template <int CLUSTER, typename T>
__global__ void __launch_bounds__(kLThreads) accept_logits_kernel(const LogitsParams p) {
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned crank = cluster.block_rank();
  const int tree = static_cast<int>(blockIdx.x) / CLUSTER;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  extern __shared__ __align__(16) unsigned char lsmem[];
  Mass* blk = reinterpret_cast<Mass*>(lsmem);                     // [2][blocks_per_cta]
  int* s_parent = reinterpret_cast<int*>(blk + 2 * p.blocks_per_cta);
  int* s_token = s_parent + p.max_nodes;
  __shared__ float s_wmax[kLWarps];
  __shared__ float s_max[2];
  __shared__ Mass s_total[2];
  __shared__ int s_bad_tree, s_sel_token, s_sel_child;

  const int64_t row0 = p.row_offsets[tree];
  const int n = static_cast<int>(p.row_offsets[tree + 1] - row0);
  const int D = p.max_depth;
  int64_t* out = p.out + static_cast<int64_t>(tree) * (D + 2);
  const uint64_t request = p.request_ids ? static_cast<uint64_t>(p.request_ids[tree]) : static_cast<uint64_t>(tree);
  if (tid == 0) s_bad_tree = (n < 1 || n > p.max_nodes) ? 1 : 0;
  __syncthreads();
  if (!s_bad_tree) {
    for (int j = tid; j < n; j += kLThreads) {
      const int64_t par = p.parents[row0 + j], tok = p.tokens[row0 + j];
      s_parent[j] = static_cast<int>(par);
      s_token[j] = static_cast<int>(tok);
      const bool ok = (j == 0) ? (par == -1) : (par >= 0 && par < j && tok >= 0 && tok < p.vocab);
      if (!ok) atomicOr(&s_bad_tree, 1);
    }
  }
  if (crank == 0)
    for (int i = tid; i < D + 2; i += kLThreads) out[i] = -1;
  __syncthreads();
  if (s_bad_tree) {
    if (crank == 0 && tid == 0) lreport(p.status, SG_ERR_TREE);
    cluster.sync();
    return;
  }

  const T* base = static_cast<const T*>(p.logits);
  const int64_t V = p.vocab;
  const int64_t nblk_total = (V + kLBlock - 1) / kLBlock;
  const int64_t slice_first = static_cast<int64_t>(crank) * p.blocks_per_cta;
  const int nb = static_cast<int>(max64(0, min64(p.blocks_per_cta, nblk_total - slice_first)));
  const double inv = p.inv_temp;
  int cur = 0, accepted = 0, pass = 0;
  bool bad = false;
  for (int depth = 0; depth <= D; ++depth) {
    const T* row = base + (row0 + cur) * V;
    double u;
    if (p.uniforms != nullptr) {
      u = p.uniforms[static_cast<int64_t>(tree) * p.uniform_stride + depth];
    } else {
      u = node_uniforms(p.seed, request, static_cast<uint32_t>(cur)).route;
    }
    if (!(u >= 0.0 && u < 1.0)) {
      if (tid == 0 && crank == 0) lreport(p.status, SG_ERR_INVALID_ARGUMENT);
      u = 0.0;
    }
    const int buf = pass & 1;
    ++pass;
    // ---- pass 1: slice maximum of the logits (max of x = logit / T follows,
    // since scaling by a positive 1/T preserves the order of the doubles)
    float m = -INFINITY;
    for (int i = warp; i < nb; i += kLWarps) {
      const int64_t b0 = (slice_first + i) * kLBlock;
      for (int k = 0; k < kLBlock / 32; ++k) {
        const int64_t j = b0 + k * 32 + lane;
        if (j < V) {
          const float v = logit_at<T>(row, j);
          if (!(v == v)) bad = true;
          m = fmaxf(m, v);
        }
      }
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    if (lane == 0) s_wmax[warp] = m;
    __syncthreads();
    if (tid == 0) {
      float cm = -INFINITY;
      for (int w = 0; w < kLWarps; ++w) cm = fmaxf(cm, s_wmax[w]);
      s_max[buf] = cm;
    }
    cluster.sync();
    float rm = -INFINITY;
#pragma unroll
    for (int c = 0; c < CLUSTER; ++c) rm = fmaxf(rm, *cluster.map_shared_rank(&s_max[buf], c));
    const double xmax = static_cast<double>(rm) * inv;
    // ---- pass 2: exact mass of every block of the slice
    Mass* mb = blk + buf * p.blocks_per_cta;
    for (int i = warp; i < nb; i += kLWarps) {
      const int64_t b0 = (slice_first + i) * kLBlock;
      uint64_t lo = 0ull;
      uint64_t hi = 0ull;
      for (int k = 0; k < kLBlock / 32; ++k) {
        const int64_t j = b0 + k * 32 + lane;
        if (j < V) {
          const Mass w = weight_mass(exp(static_cast<double>(logit_at<T>(row, j)) * inv - xmax));
          lo += w.lo;
          hi += w.hi + (lo < w.lo ? 1ull : 0ull);
        }
      }
      const Mass s = lwarp_sum(Mass{lo, hi});
      if (lane == 0) mb[i] = s;
    }
    __syncthreads();
    if (warp == 0) {
      Mass s = mass_zero();
      for (int b = lane; b < nb; b += 32) s = mass_add(s, mb[b]);
      s = lwarp_sum(s);
      if (lane == 0) s_total[buf] = s;
    }
    cluster.sync();
    // ---- selection (warp 0 of every CTA, identical work)
    if (warp == 0) {
      const Mass t = (lane < CLUSTER) ? *cluster.map_shared_rank(&s_total[buf], lane) : mass_zero();
      const Mass incl = lwarp_scan(t, lane);
      const Mass total = lshfl(incl, CLUSTER - 1);
      const Mass thr = mass_scale(u, total);
      int token = -1;
      const unsigned own = __ballot_sync(0xffffffffu, lane < CLUSTER && mass_lt(thr, incl));
      if (!mass_is_zero(total) && own != 0u) {
        const int owner = __ffs(own) - 1;
        Mass resid = mass_sub(thr, lshfl(mass_sub(incl, t), owner));
        const Mass* ob = cluster.map_shared_rank(blk + buf * p.blocks_per_cta, owner);
        const int64_t o_first = static_cast<int64_t>(owner) * p.blocks_per_cta;
        const int o_nb = static_cast<int>(max64(0, min64(p.blocks_per_cta, nblk_total - o_first)));
        // crossing block (a warp scan over the owner's block masses, 32 at a time)
        int cb = -1;
        for (int b0 = 0; b0 < o_nb && cb < 0; b0 += 32) {
          const Mass bm = (b0 + lane < o_nb) ? ob[b0 + lane] : mass_zero();
          const Mass bi = lwarp_scan(bm, lane);
          const unsigned hit = __ballot_sync(0xffffffffu, b0 + lane < o_nb && mass_lt(resid, bi));
          if (hit != 0u) {
            const int L = __ffs(hit) - 1;
            cb = b0 + L;
            resid = mass_sub(resid, mass_sub(lshfl(bi, L), lshfl(bm, L)));
          } else {
            resid = mass_sub(resid, lshfl(bi, 31));
          }
        }
        if (cb >= 0) {
          // crossing token inside the block: 32 consecutive tokens at a time
          const int64_t b0 = (o_first + cb) * kLBlock;
          for (int k = 0; k < kLBlock / 32 && token < 0; ++k) {
            const int64_t j = b0 + k * 32 + lane;
            const Mass w =
                j < V ? weight_mass(exp(static_cast<double>(logit_at<T>(row, j)) * inv - xmax)) : mass_zero();
            const Mass wi = lwarp_scan(w, lane);
            const unsigned hit = __ballot_sync(0xffffffffu, j < V && mass_lt(resid, wi));
            if (hit != 0u)
              token = static_cast<int>(b0 + k * 32 + __ffs(hit) - 1);
            else
              resid = mass_sub(resid, lshfl(wi, 31));
          }
        }
      }
      if (token < 0) token = static_cast<int>(V - 1);  // reference fallback
      int child = -1;
      for (int b = 1; b < n; b += 32) {
        const int j = b + lane;
        const unsigned mask = __ballot_sync(0xffffffffu, j < n && s_parent[j] == cur && s_token[j] == token);
        if (mask != 0u) {
          child = b + __ffs(mask) - 1;
          break;
        }
      }
      if (lane == 0) {
        s_sel_token = token;
        s_sel_child = child;
      }
    }
    __syncthreads();
    const int token = s_sel_token, child = s_sel_child;
    if (child >= 0 && depth < D) {
      if (crank == 0 && tid == 0) out[accepted] = child;
      ++accepted;
      cur = child;
      continue;
    }
    if (crank == 0 && tid == 0) {
      out[D] = accepted;
      out[D + 1] = token;
    }
    break;
  }
  if (bad) lreport(p.status, SG_ERR_PROBABILITY);
  cluster.sync();  // no CTA leaves while another may read its shared memory
}

template <int C, typename T>
int launch_logits(const LogitsParams& p, size_t smem, cudaStream_t s) {
  auto kernel = accept_logits_kernel<C, T>;
  static std::atomic<int> limits[kMaxDevices];
  const int st = ensure_dynamic_smem(kernel, smem, limits);
  if (st != SG_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.num_trees) * C, 1, 1);
  cfg.blockDim = dim3(kLThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SG_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, p));
  return check_launch("accept_logits_kernel");
}

template <typename T>
int launch_logits_cluster(int c, const LogitsParams& p, size_t smem, cudaStream_t s) {
  switch (c) {
    case 1: return launch_logits<1, T>(p, smem, s);
    case 2: return launch_logits<2, T>(p, smem, s);
    case 4: return launch_logits<4, T>(p, smem, s);
    default: return launch_logits<8, T>(p, smem, s);
  }
}

}  // namespace
}  // namespace sg

extern "C" int sg_tree_accept_logits(const void* logits, int32_t dtype, int64_t vocab, const int64_t* row_offsets,
                                     const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                                     int32_t max_nodes, int32_t max_depth, double temperature,
                                     const double* uniforms, int32_t uniform_stride, uint64_t seed,
                                     const int64_t* request_ids, int64_t* out, int32_t* status, void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (logits == nullptr || row_offsets == nullptr || parents == nullptr || tokens == nullptr || out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_logits: null pointer");
  if (dtype != SG_DTYPE_F32 && dtype != SG_DTYPE_BF16)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_logits: dtype must be SG_DTYPE_F32 or SG_DTYPE_BF16");
  if (num_trees < 0 || vocab < 1 || vocab > (int64_t(1) << 30) || max_depth < 0 || max_nodes < 1 ||
      max_nodes > (1 << 16))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_logits: bad sizes");
  if (!(temperature > 0.0) || temperature == INFINITY)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_logits: temperature must be finite and positive");
  if (uniforms != nullptr && uniform_stride < max_depth + 1)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_logits: uniforms do not cover every depth");
  const int sms = device_sm_count();
  if (sms <= 0) return fail(SG_ERR_CUDA, "sg_tree_accept_logits: no CUDA device");
  const int64_t nblk = (vocab + kLBlock - 1) / kLBlock;
  // cluster: up to 8 CTAs per tree while every tree's cluster stays resident
  // (about 4 of these CTAs fit an SM; resident clusters never wait on others)
  int cluster = kLMaxCluster;
  while (cluster > 1 && (cluster > nblk || static_cast<int64_t>(num_trees) * cluster > 4LL * sms)) cluster >>= 1;
  const int bpc = static_cast<int>((nblk + cluster - 1) / cluster);
  const size_t smem = static_cast<size_t>(bpc) * 2 * sizeof(Mass) + static_cast<size_t>(max_nodes) * 8;
  if (smem > 200 * 1024) return fail(SG_ERR_UNSUPPORTED, "sg_tree_accept_logits: vocabulary or tree too large");
  LogitsParams p{logits, dtype, vocab, row_offsets, parents, tokens, num_trees, max_nodes, max_depth,
                 1.0 / temperature, uniforms, uniform_stride, seed, request_ids, out, status, bpc};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == SG_DTYPE_BF16 ? launch_logits_cluster<__nv_bfloat16>(cluster, p, smem, s)
                                : launch_logits_cluster<float>(cluster, p, smem, s);
}
