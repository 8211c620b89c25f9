// Memory-bound per-layer kernels of the packed verify pass.
//
// They restate the Qwen3 decoder-layer pieces that the reference runs through
// HF transformers (Qwen3Model via engine.py:499-517): embedding lookup,
// RMSNorm, per-head q/k RMSNorm + rotary embedding, and the packed-input
// construction of continuous_tree_block_decode.py:500-546 (positions =
// round_prefix_len + depth, ancestor-or-self visibility of Tree.visibility,
// tree.py:19-26) — here as per-row ancestor bitsets built on device.
#include <math.h>

#include "layers.cuh"

namespace sg {
namespace layers {
namespace {

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status != nullptr) atomicMax(status, code);
}

// One thread per tree: parents precede children, so one ordered pass gives
// depth and the ancestor-or-self bitset of every node.
__global__ void __launch_bounds__(kMaxTreeRows) tree_meta_kernel(
    const int64_t* __restrict__ row_offsets, const int64_t* __restrict__ parents,
    const int64_t* __restrict__ position_base, const int64_t* __restrict__ request_ids, int num_trees, int num_rows,
    RowMeta meta, int32_t* status) {
  // One CTA per tree, one thread per node: each node builds its own
  // ancestor-or-self bitset and depth by walking its parent chain in shared
  // memory, so no node waits for another.  A parent outside [0, j) is
  // reported and treated as the root, as is a root whose parent is not -1.
  __shared__ int s_parent[kMaxTreeRows];
  const int t = blockIdx.x;
  if (t >= num_trees) return;
  const int64_t r0 = row_offsets[t];
  const int64_t r1 = row_offsets[t + 1];
  const int n = static_cast<int>(r1 - r0);
  if (r0 < 0 || r1 > num_rows || n < 1 || n > kMaxTreeRows) {
    if (threadIdx.x == 0) report(status, SG_ERR_TREE);
    return;
  }
  const int j = threadIdx.x;
  if (j < n) {
    const int64_t par = parents[r0 + j];
    int p = 0;
    if (j == 0) {
      if (par != -1) report(status, SG_ERR_TREE);
      p = -1;
    } else if (par < 0 || par >= j) {
      report(status, SG_ERR_TREE);
    } else {
      p = static_cast<int>(par);
    }
    s_parent[j] = p;
  }
  __syncthreads();
  if (j >= n) return;
  uint32_t bits[kAncWords];
#pragma unroll
  for (int w = 0; w < kAncWords; ++w) bits[w] = 0u;
  int depth = 0;
  for (int a = j; a > 0; a = s_parent[a]) {  // parents are strictly smaller: the walk ends at the root
    bits[a >> 5] |= 1u << (a & 31);
    ++depth;
  }
  bits[0] |= 1u;  // the root
  const int64_t q = r0 + j;
  uint32_t* anc = meta.anc + q * kAncWords;
#pragma unroll
  for (int w = 0; w < kAncWords; ++w) anc[w] = bits[w];
  meta.position[q] = static_cast<int32_t>(position_base[t] + depth);
  meta.tree[q] = t;
  meta.local[q] = j;
  meta.request_id[q] = request_ids != nullptr ? request_ids[t] : t;
}

// Launch order of the tree attention: requests by decreasing K/V length
// (cache prefix + tree rows), ties by index, so the longest CTAs start first
// and the grid's tail is short.  One CTA; R is small.
// Work list of the persistent tree attention.  Requests are ranked by
// decreasing K/V length (ties by index) so the kernel's tail runs the short
// items; each expands to its (kv head, 128-row query block) items, packed as
// request << 16 | kv_head << 8 | block.  Also zeroes the per-layer work
// counters the attention CTAs draw items from.  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) attention_work_kernel(const int64_t* __restrict__ row_offsets,
                                                              const int64_t* __restrict__ cache_len, int num_trees,
                                                              int group, int num_kv_heads, int32_t* __restrict__ order,
                                                              int32_t* __restrict__ items, int item_capacity,
                                                              int32_t* __restrict__ num_items,
                                                              int32_t* __restrict__ counters, int num_counters) {
  __shared__ int s_scan[1024];
  const int tid = threadIdx.x;
  for (int i = tid; i < num_counters; i += blockDim.x) counters[i] = 0;
  for (int i = tid; i < num_trees; i += blockDim.x) {
    const int64_t li = cache_len[i] + row_offsets[i + 1] - row_offsets[i];
    int rank = 0;
    for (int j = 0; j < num_trees; ++j) {
      const int64_t lj = cache_len[j] + row_offsets[j + 1] - row_offsets[j];
      rank += (lj > li || (lj == li && j < i)) ? 1 : 0;
    }
    order[rank] = i;
  }
  __syncthreads();
  auto blocks = [&](int req) -> int {  // 128-row query blocks of one kv head
    const int64_t n = row_offsets[req + 1] - row_offsets[req];
    if (n < 1 || n > kMaxTreeRows) return 0;  // malformed: tree_meta reports it
    return static_cast<int>((n * group + 127) / 128);
  };
  const int per = (num_trees + 1023) / 1024;
  const int c0 = min(num_trees, tid * per);
  const int c1 = min(num_trees, c0 + per);
  int local = 0;
  for (int r = c0; r < c1; ++r) local += blocks(order[r]) * num_kv_heads;
  s_scan[tid] = local;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {  // inclusive scan
    const int v = tid >= off ? s_scan[tid - off] : 0;
    __syncthreads();
    s_scan[tid] += v;
    __syncthreads();
  }
  int at = s_scan[tid] - local;
  for (int r = c0; r < c1; ++r) {
    const int req = order[r];
    const int nb = blocks(req);
    for (int h = 0; h < num_kv_heads; ++h)
      for (int b = 0; b < nb; ++b, ++at)
        if (at < item_capacity) items[at] = (req << 16) | (h << 8) | b;
  }
  if (tid == 1023) *num_items = min(s_scan[1023], item_capacity);
}

__global__ void embed_kernel(const int64_t* __restrict__ tokens, const __nv_bfloat16* __restrict__ embed,
                             int64_t vocab, int hidden, float* __restrict__ x, int32_t* status) {
  const int row = blockIdx.x;
  int64_t tok = tokens[row];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) report(status, SG_ERR_TREE);
    tok = 0;
  }
  const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(embed + tok * hidden);
  float2* dst = reinterpret_cast<float2*>(x + static_cast<int64_t>(row) * hidden);
  for (int i = threadIdx.x; i < hidden / 2; i += blockDim.x) dst[i] = __bfloat1622float2(src[i]);
}

// y = bf16(x * rsqrt(mean(x^2) + eps) * w); one CTA of 256 threads per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                                      int hidden, float eps, __nv_bfloat16* __restrict__ out,
                                                      int64_t ld_out, float* __restrict__ ssq) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<int64_t>(row) * hidden);
  const int n4 = hidden / 4;
  // Rows of up to kKeep float4 per thread stay in registers between the sum of
  // squares and the scaling, so the row is read once.
  constexpr int kKeep = 8;
  const bool keep = n4 <= kKeep * static_cast<int>(blockDim.x);
  float4 kept[kKeep];
  float ss = 0.f;
  if (keep) {
#pragma unroll
    for (int k = 0; k < kKeep; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      kept[k] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += kept[k].x * kept[k].x + kept[k].y * kept[k].y + kept[k].z * kept[k].z + kept[k].w * kept[k].w;
    }
  } else {
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = xr[i];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  }
  __shared__ float red[8];
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) t += __shfl_xor_sync(0xffffffffu, t, d);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  // folded form (ssq given): the consumer GEMM applies rstd per row
  const float rstd = ssq != nullptr ? 1.0f : rsqrtf(red[0] / static_cast<float>(hidden) + eps);
  if (ssq != nullptr && threadIdx.x == 0) ssq[row] = red[0];
  const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(w);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<int64_t>(row) * ld_out);
  auto scale = [&](int i, float4 v) {
    const float2 wa = __bfloat1622float2(w2[2 * i]);
    const float2 wb = __bfloat1622float2(w2[2 * i + 1]);
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x * rstd * wa.x, v.y * rstd * wa.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z * rstd * wb.x, v.w * rstd * wb.y);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&a);
    packed.y = *reinterpret_cast<uint32_t*>(&b);
    o[i] = packed;
  };
  if (keep) {
#pragma unroll
    for (int k = 0; k < kKeep; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i < n4) scale(i, kept[k]);
    }
  } else {
    for (int i = threadIdx.x; i < n4; i += blockDim.x) scale(i, xr[i]);
  }
}

// One warp per (row, head).  Heads [0, nq) are queries, [nq, nq+nkv) keys,
// [nq+nkv, nq+2nkv) values.  Lane l holds dims l + 32 i; the rotary pairs
// (d, d + D/2) therefore sit in the same lane.
template <int D>
__global__ void __launch_bounds__(256) qkv_post_kernel(const QkvPost p) {
  constexpr int PER = D / 32;
  constexpr int HALF = D / 2;
  pdl_trigger();
  pdl_wait();
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = p.nq + 2 * p.nkv;
  if (warp_global >= p.rows * heads) return;
  const int row = warp_global / heads;
  const int head = warp_global % heads;
  const __nv_bfloat16* src = p.qkv + static_cast<int64_t>(row) * heads * D + static_cast<int64_t>(head) * D;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) v[i] = __bfloat162float(src[lane + 32 * i]);
  const bool is_q = head < p.nq;
  const bool is_k = !is_q && head < p.nq + p.nkv;
  if (is_q || is_k) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) ss += v[i] * v[i];
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps);
    const __nv_bfloat16* w = is_q ? p.q_norm : p.k_norm;
#pragma unroll
    for (int i = 0; i < PER; ++i) v[i] = v[i] * rstd * __bfloat162float(w[lane + 32 * i]);
    // rotate_half rotary embedding: out_d = x_d cos - x_{d+H} sin (d < H),
    //                                out_{d+H} = x_{d+H} cos + x_d sin.
    const float pos = static_cast<float>(p.position[row]);
#pragma unroll
    for (int i = 0; i < PER / 2; ++i) {
      const int d = lane + 32 * i;  // < HALF
      const float angle = pos * p.inv_freq[d];
      float s, c;
      sincosf(angle, &s, &c);
      const float x1 = v[i], x2 = v[i + PER / 2];
      v[i] = x1 * c - x2 * s;
      v[i + PER / 2] = x2 * c + x1 * s;
    }
    (void)HALF;
  }
  __nv_bfloat16* dst;
  if (is_q) {
    dst = p.q_out + static_cast<int64_t>(row) * p.nq * D + static_cast<int64_t>(head) * D;
  } else {
    const int kvh = is_k ? head - p.nq : head - p.nq - p.nkv;
    const int t = p.tree[row];
    if (t < 0) {  // row of a rejected tree (reported by tree_meta)
      return;
    }
    const int64_t arena_row = p.slots[t] * p.capacity + p.cache_len[t] + p.local[row];
    if (arena_row < 0 || arena_row >= p.plane_rows || p.cache_len[t] + p.local[row] >= p.capacity) {
      if (lane == 0) report(p.status, SG_ERR_CAPACITY);
      return;
    }
    __nv_bfloat16* plane = (is_k ? p.k_plane0 : p.v_plane0) + static_cast<int64_t>(kvh) * p.plane_stride;
    dst = plane + arena_row * D;
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(v[i]);
}

// Rotary table and K/V arena row of every packed row, once per pass (the
// angles and the arena row do not change from layer to layer).  One CTA of
// D/2 threads per row; thread 0 also resolves the row's arena row, -1 for a
// row of a rejected tree or one that would overflow its slot (reported).
__global__ void row_rope_kernel(const int32_t* __restrict__ position, const int32_t* __restrict__ tree,
                                const int32_t* __restrict__ local, const float* __restrict__ inv_freq,
                                const int64_t* __restrict__ slots, const int64_t* __restrict__ cache_len,
                                int64_t capacity, int64_t plane_rows, int half, float2* __restrict__ rope,
                                int64_t* __restrict__ arena_row, int32_t* status) {
  const int row = blockIdx.x;
  const int d = threadIdx.x;
  if (d < half) {
    const float angle = static_cast<float>(position[row]) * inv_freq[d];
    float sn, cs;
    sincosf(angle, &sn, &cs);
    rope[static_cast<int64_t>(row) * half + d] = make_float2(cs, sn);
  }
  if (d == 0) {
    int64_t ar = -1;
    const int t = tree[row];
    if (t >= 0) {
      const int64_t a = slots[t] * capacity + cache_len[t] + local[row];
      if (a < 0 || a >= plane_rows || cache_len[t] + local[row] >= capacity)
        report(status, SG_ERR_CAPACITY);
      else
        ar = a;
    }
    arena_row[row] = ar;
  }
}

// The same operation as qkv_post_kernel with one CTA per packed row, reading
// the pass's rotary table and arena rows.  A group of D/8 threads owns one
// head, each thread 8 consecutive dims moved as 16-byte vectors, with its 8
// (cos, sin) pairs and norm weights in registers; the rotary partner of dim
// d (< D/2) is dim d + D/2, held by the thread D/16 lanes away in the same
// group, and the norm's sum of squares is reduced inside the group.  Every
// lane takes every shuffle (value heads and idle lanes compute and then
// discard), so control flow stays uniform across a warp whose groups hold
// different head types, and no block-wide barrier is needed.
template <int D>
__global__ void __launch_bounds__(256) qkv_post_row_kernel(const QkvPost p) {
  constexpr int G = D / 8;      // threads per head
  constexpr int HALF_G = G / 2; // partner distance in lanes
  constexpr int HALF = D / 2;
  pdl_trigger();
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int j = tid % G;            // 8-dim chunk of the head
  const bool high = j >= HALF_G;    // dims >= D/2
  const int d0 = 8 * j;
  const int dl = 8 * (j % HALF_G);  // angle index of this chunk's dims
  float qw[8], kw[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {  // weights are not produced by a predecessor
    qw[e] = __bfloat162float(p.q_norm[d0 + e]);
    kw[e] = __bfloat162float(p.k_norm[d0 + e]);
  }
  pdl_wait();
  float cs[8], sn[8];
  const float2* rr = p.rope + static_cast<int64_t>(row) * HALF + dl;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 t = rr[e];
    cs[e] = t.x;
    sn[e] = t.y;
  }
  const int64_t arena_row = p.arena_row[row];
  const int heads = p.nq + 2 * p.nkv;
  const int iters = (heads * G + static_cast<int>(blockDim.x) - 1) / static_cast<int>(blockDim.x);
  for (int it = 0; it < iters; ++it) {
    const int head = (it * static_cast<int>(blockDim.x) + tid) / G;
    const bool valid = head < heads;
    float v[8];
    if (valid) {
      const uint4 raw = *reinterpret_cast<const uint4*>(p.qkv + static_cast<int64_t>(row) * heads * D +
                                                        static_cast<int64_t>(head) * D + d0);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    const bool is_q = head < p.nq;
    const bool is_k = !is_q && head < p.nq + p.nkv;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
#pragma unroll
    for (int d = HALF_G; d >= 1; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps);
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = v[e] * rstd * (is_q ? qw[e] : kw[e]);
      const float partner = __shfl_xor_sync(0xffffffffu, x, HALF_G);
      // rotate_half: out_d = x_d cos - x_{d+H} sin,  out_{d+H} = x_{d+H} cos + x_d sin
      r[e] = high ? x * cs[e] + partner * sn[e] : x * cs[e] - partner * sn[e];
    }
    if (!valid) continue;
    const bool qk = is_q || is_k;
    uint4 packed;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o2[e] = __floats2bfloat162_rn(qk ? r[2 * e] : v[2 * e], qk ? r[2 * e + 1] : v[2 * e + 1]);
    if (is_q) {
      *reinterpret_cast<uint4*>(p.q_out + static_cast<int64_t>(row) * p.nq * D + static_cast<int64_t>(head) * D +
                                d0) = packed;
    } else if (arena_row >= 0) {
      const int kvh = is_k ? head - p.nq : head - p.nq - p.nkv;
      __nv_bfloat16* plane = (is_k ? p.k_plane0 : p.v_plane0) + static_cast<int64_t>(kvh) * p.plane_stride;
      *reinterpret_cast<uint4*>(plane + arena_row * D + d0) = packed;
    }
  }
}

// lse and Gumbel-max token of every row from the per-vocab-tile partials
// (max, sum exp(l - max), best perturbed logit, its column).
__global__ void lm_combine_kernel(const float4* __restrict__ partials, int n_tiles, int rows,
                                  float* __restrict__ lse, int64_t* __restrict__ posterior,
                                  const int32_t* __restrict__ abort_status) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  if (abort_status != nullptr && *abort_status != 0) {
    if (lane == 0) {
      if (lse != nullptr) lse[row] = NAN;
      if (posterior != nullptr) posterior[row] = -1;
    }
    return;
  }
  const float4* pr = partials + static_cast<int64_t>(row) * n_tiles;
  float m = -INFINITY;
  for (int t = lane; t < n_tiles; t += 32) m = fmaxf(m, pr[t].x);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
  float s = 0.f, best = -INFINITY;
  int idx = 0x7fffffff;
  for (int t = lane; t < n_tiles; t += 32) {
    const float4 v = pr[t];
    s += v.y * __expf(v.x - m);
    const int col = __float_as_int(v.w);
    if (v.z > best || (v.z == best && col < idx)) {
      best = v.z;
      idx = col;
    }
  }
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, d);
    const float ob = __shfl_xor_sync(0xffffffffu, best, d);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, d);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  if (lane == 0) {
    if (lse != nullptr) lse[row] = m + logf(s);
    if (posterior != nullptr) posterior[row] = idx;
  }
}

// log p_parent(token) for every non-root row: logit recomputed as a dot
// product of the parent's final hidden row with the token's LM-head row.
__global__ void child_logprob_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ w,
                                     int hidden, int64_t vocab, const int64_t* __restrict__ tokens,
                                     const int64_t* __restrict__ parents, const int64_t* __restrict__ row_offsets,
                                     const int32_t* __restrict__ tree, const int32_t* __restrict__ local,
                                     const float* __restrict__ lse, float inv_temp, int rows,
                                     float* __restrict__ logprob, const float* __restrict__ ssq, int ss_parts,
                                     float inv_h, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  if (tree[row] < 0 || local[row] == 0) {
    if (lane == 0) logprob[row] = tree[row] < 0 ? NAN : 0.f;
    return;
  }
  const int64_t par = parents[row];
  const int64_t tok = tokens[row];
  if (par < 0 || par >= local[row] || tok < 0 || tok >= vocab) {  // invalid tree: reported by tree_meta
    if (lane == 0) logprob[row] = NAN;
    return;
  }
  const int64_t prow = row_offsets[tree[row]] + par;
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(h + prow * hidden);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(w + tok * hidden);
  float acc = 0.f;
  for (int i = lane; i < hidden / 2; i += 32) {
    const float2 x = __bfloat1622float2(a[i]);
    const float2 y = __bfloat1622float2(b[i]);
    acc += x.x * y.x + x.y * y.y;
  }
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  // h holds bf16(x * w) when the final norm is folded (ssq given): the row
  // scale rstd joins 1/T exactly as in the LM-head epilogue
  float xs = inv_temp;
  if (ssq != nullptr) {
    float t = 0.f;
    for (int i = 0; i < ss_parts; ++i) t += ssq[prow * ss_parts + i];
    xs = __fmul_rn(rsqrtf(__fmaf_rn(t, inv_h, eps)), inv_temp);
  }
  if (lane == 0) logprob[row] = acc * xs - lse[prow];
}

// One CTA per request: its kept rows go to dst rows base .. base + count,
// base = kept rows of the earlier requests (summed by the CTA itself).
// Counts or nodes outside the tree are reported and their rows skipped.
__global__ void __launch_bounds__(256) gather_kept_rows_kernel(const uint4* __restrict__ src, int64_t row_vecs,
                                                               const int64_t* __restrict__ row_offsets,
                                                               const int64_t* __restrict__ accept_out,
                                                               int num_trees, int max_depth, uint4* __restrict__ dst,
                                                               int64_t* __restrict__ dst_offsets, int32_t* status) {
  __shared__ int64_t s_part[8];
  const int t = blockIdx.x;
  const int stride = max_depth + 2;
  auto kept = [&](int tree) -> int64_t {
    const int64_t c = accept_out[static_cast<int64_t>(tree) * stride + max_depth];
    return (c >= 0 && c <= max_depth) ? c + 1 : 0;
  };
  int64_t part = 0;
  for (int u = threadIdx.x; u < t; u += blockDim.x) part += kept(u);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) part += __shfl_xor_sync(0xffffffffu, part, d);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = part;
  __syncthreads();
  int64_t base = 0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) base += s_part[w];
  const int64_t count = kept(t);
  if (threadIdx.x == 0) {
    if (count == 0) report(status, SG_ERR_TREE);
    if (t == 0) dst_offsets[0] = 0;
    dst_offsets[t + 1] = base + count;
  }
  const int64_t r0 = row_offsets[t], n = row_offsets[t + 1] - r0;
  for (int64_t j = 0; j < count; ++j) {
    const int64_t node = j == 0 ? 0 : accept_out[static_cast<int64_t>(t) * stride + j - 1];
    if (node < 0 || node >= n) {
      if (threadIdx.x == 0) report(status, SG_ERR_TREE);
      continue;
    }
    const uint4* s = src + (r0 + node) * row_vecs;
    uint4* o = dst + (base + j) * row_vecs;
    for (int64_t v = threadIdx.x; v < row_vecs; v += blockDim.x) o[v] = s[v];
  }
}

}  // namespace

int launch_gather_kept_rows(const void* src, int64_t row_bytes, const int64_t* row_offsets, const int64_t* accept_out,
                            int num_trees, int max_depth, void* dst, int64_t* dst_offsets, int32_t* status,
                            cudaStream_t stream) {
  if (num_trees <= 0) return SG_OK;
  if (row_bytes <= 0 || row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "gather of kept rows: rows and buffers must be 16-byte aligned");
  gather_kept_rows_kernel<<<num_trees, 256, 0, stream>>>(static_cast<const uint4*>(src), row_bytes / 16, row_offsets,
                                                         accept_out, num_trees, max_depth, static_cast<uint4*>(dst),
                                                         dst_offsets, status);
  return check_launch("gather_kept_rows_kernel");
}

int launch_attention_work(const int64_t* row_offsets, const int64_t* cache_len, int num_trees, int group,
                          int num_kv_heads, AttentionWork work, int num_layers, cudaStream_t stream) {
  if (num_trees <= 0) return SG_OK;
  if (num_trees > 65535 || num_kv_heads > 255 || group > 127)
    return fail(SG_ERR_UNSUPPORTED, "tree attention work list: > 65535 requests, > 255 kv heads or group > 127");
  attention_work_kernel<<<1, 1024, 0, stream>>>(row_offsets, cache_len, num_trees, group, num_kv_heads, work.order,
                                                work.items, work.item_capacity, work.num_items, work.counters,
                                                num_layers);
  return check_launch("attention_work_kernel");
}

int launch_tree_meta(const int64_t* row_offsets, const int64_t* parents, const int64_t* position_base,
                     const int64_t* request_ids, int num_trees, int num_rows, RowMeta meta, int32_t* status,
                     cudaStream_t stream) {
  if (num_trees <= 0) return SG_OK;
  // rows not claimed by a valid tree keep tree = -1 and are skipped downstream
  SG_CUDA_CHECK(cudaMemsetAsync(meta.tree, 0xff, static_cast<size_t>(num_rows) * sizeof(int32_t), stream));
  tree_meta_kernel<<<num_trees, kMaxTreeRows, 0, stream>>>(row_offsets, parents, position_base, request_ids,
                                                             num_trees, num_rows, meta, status);
  return check_launch("tree_meta_kernel");
}

int launch_row_rope(const RowMeta& meta, const float* inv_freq, int head_dim, int rows, const int64_t* slots,
                    const int64_t* cache_len, int64_t capacity, int64_t plane_rows, int32_t* status,
                    cudaStream_t stream) {
  if (rows <= 0) return SG_OK;
  const int half = head_dim / 2;
  row_rope_kernel<<<rows, half, 0, stream>>>(meta.position, meta.tree, meta.local, inv_freq, slots, cache_len,
                                             capacity, plane_rows, half, meta.rope, meta.arena_row, status);
  return check_launch("row_rope_kernel");
}

__global__ void __launch_bounds__(256) draft_meta_kernel(const int64_t* __restrict__ update_offsets,
                                                         const int64_t* __restrict__ cache_len,
                                                         const int64_t* __restrict__ anchors, int64_t mask_token,
                                                         int num_requests, int block, int update_rows,
                                                         RowMeta bm, RowMeta cm, int64_t* __restrict__ block_offsets,
                                                         int64_t* __restrict__ prefix_len,
                                                         int64_t* __restrict__ block_tokens,
                                                         int64_t* __restrict__ lengths_out, int32_t* status) {
  const int t = blockIdx.x;
  int64_t u0 = update_offsets[t], u1 = update_offsets[t + 1];
  if (u0 < 0 || u1 < u0 || u1 > update_rows || (t == num_requests - 1 && u1 != update_rows)) {
    if (threadIdx.x == 0) report(status, SG_ERR_TREE);
    u0 = u1 = 0;
  }
  const int64_t prefix = cache_len[t] + (u1 - u0);
  for (int j = threadIdx.x; j < block; j += blockDim.x) {
    const int64_t q = static_cast<int64_t>(t) * block + j;
    uint32_t* anc = bm.anc + q * kAncWords;
    for (int w = 0; w < kAncWords; ++w) {
      const int lo = 32 * w;
      anc[w] = block >= lo + 32 ? 0xFFFFFFFFu : (block > lo ? (1u << (block - lo)) - 1u : 0u);
    }
    bm.position[q] = static_cast<int32_t>(prefix + j);
    bm.tree[q] = t;
    bm.local[q] = j;
    bm.request_id[q] = t;
    block_tokens[q] = j == 0 ? anchors[t] : mask_token;
  }
  for (int64_t i = u0 + threadIdx.x; i < u1; i += blockDim.x) {
    cm.position[i] = static_cast<int32_t>(cache_len[t] + (i - u0));
    cm.tree[i] = t;
    cm.local[i] = static_cast<int32_t>(i - u0);
  }
  if (threadIdx.x == 0) {
    block_offsets[t] = static_cast<int64_t>(t) * block;
    if (t == num_requests - 1) block_offsets[num_requests] = static_cast<int64_t>(num_requests) * block;
    prefix_len[t] = prefix;
    if (lengths_out != nullptr) lengths_out[t] = prefix;
  }
}

int launch_draft_meta(const int64_t* update_offsets, const int64_t* cache_len, const int64_t* anchors,
                      int64_t mask_token, int num_requests, int block, int update_rows, RowMeta block_meta,
                      RowMeta ctx_meta, int64_t* block_offsets, int64_t* prefix_len, int64_t* block_tokens,
                      int64_t* lengths_out, int32_t* status, cudaStream_t stream) {
  if (num_requests <= 0) return SG_OK;
  if (block < 1 || block > kMaxTreeRows) return fail(SG_ERR_UNSUPPORTED, "draft_meta: block size must be 1..256");
  draft_meta_kernel<<<num_requests, 256, 0, stream>>>(update_offsets, cache_len, anchors, mask_token, num_requests,
                                                      block, update_rows, block_meta, ctx_meta, block_offsets,
                                                      prefix_len, block_tokens, lengths_out, status);
  return check_launch("draft_meta_kernel");
}

int launch_embed(const int64_t* tokens, const __nv_bfloat16* embed, int64_t vocab, int hidden, int rows, float* x,
                 int32_t* status, cudaStream_t stream) {
  if (rows <= 0) return SG_OK;
  embed_kernel<<<rows, 256, 0, stream>>>(tokens, embed, vocab, hidden, x, status);
  return check_launch("embed_kernel");
}

int launch_rmsnorm(const float* x, const __nv_bfloat16* weight, int hidden, int rows, float eps,
                   __nv_bfloat16* out, cudaStream_t stream, int64_t ld_out) {
  if (rows <= 0) return SG_OK;
  if (hidden % 4 != 0) return fail(SG_ERR_UNSUPPORTED, "rmsnorm: hidden % 4 != 0");
  if (ld_out == 0) ld_out = hidden;
  if (ld_out % 4 != 0) return fail(SG_ERR_UNSUPPORTED, "rmsnorm: output stride % 4 != 0");
  return launch_pdl("rmsnorm_kernel", rmsnorm_kernel, dim3(rows), dim3(256), 0, stream, x, weight, hidden, eps, out,
                    ld_out, static_cast<float*>(nullptr));
}

int launch_norm_fold(const float* x, const __nv_bfloat16* weight, int hidden, int rows, __nv_bfloat16* xw,
                     float* ssq, cudaStream_t stream) {
  if (rows <= 0) return SG_OK;
  if (hidden % 4 != 0) return fail(SG_ERR_UNSUPPORTED, "rmsnorm: hidden % 4 != 0");
  return launch_pdl("rmsnorm_kernel", rmsnorm_kernel, dim3(rows), dim3(256), 0, stream, x, weight, hidden, 0.f, xw,
                    static_cast<int64_t>(hidden), ssq);
}

int launch_qkv_post(const QkvPost& p, cudaStream_t stream) {
  if (p.rows <= 0) return SG_OK;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const bool vec = p.rope != nullptr && p.arena_row != nullptr && a16(p.qkv) && a16(p.q_out) &&
                   a16(p.k_plane0) && a16(p.v_plane0) && (p.plane_stride * 2) % 16 == 0;
  if (vec && p.head_dim == 128)
    return launch_pdl("qkv_post_row_kernel", qkv_post_row_kernel<128>, dim3(p.rows), dim3(256), 0, stream, p);
  if (vec && p.head_dim == 64)
    return launch_pdl("qkv_post_row_kernel", qkv_post_row_kernel<64>, dim3(p.rows), dim3(256), 0, stream, p);
  const int64_t warps = static_cast<int64_t>(p.rows) * (p.nq + 2 * p.nkv);
  const unsigned grid = static_cast<unsigned>((warps + 7) / 8);
  if (p.head_dim == 128)
    return launch_pdl("qkv_post_kernel", qkv_post_kernel<128>, dim3(grid), dim3(256), 0, stream, p);
  if (p.head_dim == 64)
    return launch_pdl("qkv_post_kernel", qkv_post_kernel<64>, dim3(grid), dim3(256), 0, stream, p);
  return fail(SG_ERR_UNSUPPORTED, "qkv_post: head_dim must be 64 or 128");
}

int launch_lm_combine(const float4* partials, int n_tiles, int rows, float* lse, int64_t* posterior,
                      const int32_t* abort_status, cudaStream_t stream) {
  if (rows <= 0) return SG_OK;
  lm_combine_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(partials, n_tiles, rows, lse, posterior, abort_status);
  return check_launch("lm_combine_kernel");
}

int launch_child_logprob(const __nv_bfloat16* h, const __nv_bfloat16* lm_head, int hidden, int64_t vocab,
                         const int64_t* tokens,
                         const int64_t* parents, const int64_t* row_offsets, const int32_t* tree,
                         const int32_t* local, const float* lse, float inv_temp, int rows, float* logprob,
                         cudaStream_t stream, const float* ssq, int ss_parts, float eps) {
  if (rows <= 0) return SG_OK;
  child_logprob_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(h, lm_head, hidden, vocab, tokens, parents, row_offsets, tree,
                                                           local, lse, inv_temp, rows, logprob, ssq, ss_parts,
                                                           1.0f / static_cast<float>(hidden), eps);
  return check_launch("child_logprob_kernel");
}

}  // namespace layers
}  // namespace sg
