// Memory-bound per-layer kernels of the packed verify pass (sm_100a).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace sg {
namespace layers {

constexpr int kMaxTreeRows = 256;               // rows per request tree (root included)
constexpr int kAncWords = kMaxTreeRows / 32;    // ancestor bitset words per row

// Per-row metadata derived on device from the wave's tree description.
struct RowMeta {
  uint32_t* anc;        // [Q][kAncWords] ancestor-or-self bitset over local rows
  int32_t* position;    // [Q] rotary position = position_base[req] + depth
  int32_t* tree;        // [Q] request (tree) index of the row
  int32_t* local;       // [Q] local node index
  int64_t* request_id;  // [Q] Philox key of the row's request
  int32_t* order;       // [R] requests by decreasing K/V length (attention launch order)
  float2* rope;         // [Q][D/2] (cos, sin) of the row's rotary angles, once per pass
  int64_t* arena_row;   // [Q] arena row of the row's K/V (-1: rejected tree or overflow)
};

// Per-pass rotary table and K/V arena row of every packed row (the same in
// every layer): rope[q][d] = sincos(position[q] * inv_freq[d]).
int launch_row_rope(const RowMeta& meta, const float* inv_freq, int head_dim, int rows, const int64_t* slots,
                    const int64_t* cache_len, int64_t capacity, int64_t plane_rows, int32_t* status,
                    cudaStream_t stream);

int launch_tree_meta(const int64_t* row_offsets, const int64_t* parents, const int64_t* position_base,
                     const int64_t* request_ids, int num_trees, int num_rows, RowMeta meta, int32_t* status,
                     cudaStream_t stream);

// Persistent tree attention work list (built once per pass).
struct AttentionWork {
  int32_t* order;       // [R] requests by decreasing K/V length
  int32_t* items;       // [item_capacity] request << 16 | kv_head << 8 | 128-row block
  int item_capacity;
  int32_t* num_items;   // [1]
  int32_t* counters;    // [num_layers] next item of each layer's attention launch
};
int launch_attention_work(const int64_t* row_offsets, const int64_t* cache_len, int num_trees, int group,
                          int num_kv_heads, AttentionWork work, int num_layers, cudaStream_t stream);

// Per-row metadata of a drafter step.  Request t's block rows t*B .. t*B+B-1
// see each other (all bits of the block set: the block is bidirectional) at
// positions prefix_t + j, prefix_t = cache_len[t] + its update rows; its
// context rows update_offsets[t] .. update_offsets[t+1]-1 sit at positions
// cache_len[t] + i.  Writes the block rows' offsets, prefix lengths and
// input tokens (anchor, then mask tokens) and lengths_out = prefix.
int launch_draft_meta(const int64_t* update_offsets, const int64_t* cache_len, const int64_t* anchors,
                      int64_t mask_token, int num_requests, int block, int update_rows, RowMeta block_meta,
                      RowMeta ctx_meta, int64_t* block_offsets, int64_t* prefix_len, int64_t* block_tokens,
                      int64_t* lengths_out, int32_t* status, cudaStream_t stream);

int launch_embed(const int64_t* tokens, const __nv_bfloat16* embed, int64_t vocab, int hidden, int rows,
                 float* x, int32_t* status, cudaStream_t stream);

int launch_rmsnorm(const float* x, const __nv_bfloat16* weight, int hidden, int rows, float eps,
                   __nv_bfloat16* out, cudaStream_t stream, int64_t ld_out = 0);

// The RMSNorm folded into the next GEMM: xw = bf16(x * weight) and ssq[row]
// = sum of x^2 (one part per row), the GEMM scaling each row by
// rsqrt(ssq / hidden + eps) in its epilogue.
int launch_norm_fold(const float* x, const __nv_bfloat16* weight, int hidden, int rows, __nv_bfloat16* xw,
                     float* ssq, cudaStream_t stream);

struct QkvPost {
  const __nv_bfloat16* qkv;     // [Q, (nq + 2 nkv) * D]
  const __nv_bfloat16* q_norm;  // [D]
  const __nv_bfloat16* k_norm;  // [D]
  const float* inv_freq;        // [D/2]
  const int32_t* position;      // [Q]
  const int32_t* tree;          // [Q]
  const int32_t* local;         // [Q]
  const int64_t* slots;         // [R]
  const int64_t* cache_len;     // [R]
  __nv_bfloat16* q_out;         // [Q, nq * D]
  __nv_bfloat16* k_plane0;      // K plane of kv head 0 of this layer
  __nv_bfloat16* v_plane0;      // V plane of kv head 0 of this layer
  int64_t plane_stride;         // elements between consecutive kv heads' planes
  int64_t capacity;             // rows per slot
  int64_t plane_rows;           // rows per plane (slots * capacity)
  const float2* rope;           // [Q][D/2] per-pass rotary table (launch_row_rope), or null
  const int64_t* arena_row;     // [Q] per-pass K/V arena row (launch_row_rope), or null
  int nq, nkv, head_dim, rows;
  float eps;
  int32_t* status;
};
int launch_qkv_post(const QkvPost& p, cudaStream_t stream);

// lse[row] and posterior[row] from the per-vocab-tile partials of the
// LM-head epilogue.  With a non-null `abort_status` holding a non-zero code
// (a GEMM that gave up a bounded wait), every row gets posterior -1, lse NaN.
int launch_lm_combine(const float4* partials, int n_tiles, int rows, float* lse, int64_t* posterior,
                      const int32_t* abort_status, cudaStream_t stream);

// Gather each request's kept rows ([0] + accepted nodes, read from the
// acceptance output accept_out[t, max_depth + 2]) of `src` (row_bytes per
// row, rows packed by row_offsets) into `dst`, requests in order, and write
// dst_offsets[t] .. dst_offsets[t + 1] for each.  row_bytes % 16 == 0.
int launch_gather_kept_rows(const void* src, int64_t row_bytes, const int64_t* row_offsets, const int64_t* accept_out,
                            int num_trees, int max_depth, void* dst, int64_t* dst_offsets, int32_t* status,
                            cudaStream_t stream);

int launch_child_logprob(const __nv_bfloat16* h, const __nv_bfloat16* lm_head, int hidden, int64_t vocab,
                         const int64_t* tokens,
                         const int64_t* parents, const int64_t* row_offsets, const int32_t* tree,
                         const int32_t* local, const float* lse, float inv_temp, int rows, float* logprob,
                         cudaStream_t stream, const float* ssq = nullptr, int ss_parts = 0, float eps = 0.f);

}  // namespace layers
}  // namespace sg
