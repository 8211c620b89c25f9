// Tree attention launcher interface (implementation in attention.cu).
#pragma once

#include <cuda_bf16.h>

#include "sm100.cuh"

namespace sg {
namespace attn {

struct Params {
  const __nv_bfloat16* q;    // [Q, nq, D]
  __nv_bfloat16* out;        // [Q, nq, D]
  const __nv_bfloat16* k0;   // K plane of kv head 0 (this layer)
  const __nv_bfloat16* v0;   // V plane of kv head 0 (this layer)
  int64_t plane_stride;      // elements between kv heads' planes
  int64_t capacity;          // rows per request slot
  int64_t plane_rows;        // rows per plane (slots * capacity)
  int64_t num_rows;          // packed query rows of the wave
  const int64_t* row_offsets;
  const int64_t* slots;
  const int64_t* cache_len;
  const uint32_t* anc;       // [Q][kAncWords]
  int nq, nkv, group;
  int plane_k0, plane_v0;    // arena plane of kv head 0's K and V for this layer
  const int32_t* items;      // persistent kernel: request << 16 | kv_head << 8 | 128-row block
  const int32_t* num_items;  // [1]
  int32_t* work_counter;     // next item; zero before the launch
  float scale_log2;          // softmax scale * log2(e)
  int32_t* status;
};

// Rows of the kv_map TMA box (a 128-key tile is loaded as two boxes).
constexpr int kKeyTile = 64;

// kv_map: 3-D TMA map over the whole arena (head_dim, plane rows, planes),
// box (64, kKeyTile, 1), 128-byte swizzle.
int launch(const CUtensorMap& kv_map, const Params& p, int num_requests, int max_rows_per_request, int head_dim,
           cudaStream_t stream);

}  // namespace attn
}  // namespace sg
