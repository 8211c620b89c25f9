// Accepted-path KV commit (sm_100a).
//
// Reference: _PersistentRequestCachePool.append_packed_sequence
// (continuous_tree_block_decode.py:215-261) gathers the kept packed rows
// (ΣL + query_offset + row) of every layer's K and V and index_copy_'s them
// to slot * capacity + old_length + i, with one index_select and one
// index_copy_ per layer and tensor.
//
// Here one launch moves every plane (layer x {K,V} x kv head) at once.  A CTA
// owns one request (group) and a run of planes: it stages the group's kept
// rows for those planes in shared memory with 16-byte loads, synchronises,
// and writes them back with 16-byte stores.  Staging the whole group before
// any store makes the in-place tail compaction (src and dst in the same plane,
// dst_rows[i] <= src_rows[i]) race-free; src and dst may alias, so neither is
// declared __restrict__ and loads use the coherent path.
#include <algorithm>

#include "common.cuh"

namespace sg {
namespace {

constexpr int kCommitThreads = 256;
constexpr int kStageBytes = 32 * 1024;

__global__ void __launch_bounds__(kCommitThreads)
kv_commit_kernel(unsigned char* dst, int64_t dst_plane_rows,
                 const unsigned char* src, int64_t src_plane_rows, int64_t num_planes,
                 int64_t row_bytes, const int64_t* __restrict__ src_rows,
                 const int64_t* __restrict__ dst_rows, const int64_t* __restrict__ group_offsets,
                 int planes_per_cta, int rows_per_chunk, bool vec16, int32_t* status) {
  __shared__ __align__(16) unsigned char stage[kStageBytes];
  __shared__ int64_t s_src[64];
  __shared__ int64_t s_dst[64];
  const int g = blockIdx.x;
  const int64_t plane0 = static_cast<int64_t>(blockIdx.y) * planes_per_cta;
  const int nplanes = static_cast<int>(min64(planes_per_cta, num_planes - plane0));
  if (nplanes <= 0) return;
  const int64_t r_begin = group_offsets[g];
  const int64_t r_end = group_offsets[g + 1];
  const int unit = vec16 ? 16 : 4;
  const int units_per_row = static_cast<int>(row_bytes / unit);

  for (int64_t c0 = r_begin; c0 < r_end; c0 += rows_per_chunk) {
    const int nrows = static_cast<int>(min64(rows_per_chunk, r_end - c0));
    if (threadIdx.x < nrows) {
      int64_t s = src_rows[c0 + threadIdx.x];
      int64_t d = dst_rows[c0 + threadIdx.x];
      if (s < 0 || s >= src_plane_rows || d < 0 || d >= dst_plane_rows) {
        if (status != nullptr) atomicMax(status, static_cast<int32_t>(SG_ERR_CAPACITY));
        s = -1;
        d = -1;
      }
      s_src[threadIdx.x] = s;
      s_dst[threadIdx.x] = d;
    }
    __syncthreads();
    const int total_units = nplanes * nrows * units_per_row;
    // gather
    for (int i = threadIdx.x; i < total_units; i += kCommitThreads) {
      const int u = i % units_per_row;
      const int rest = i / units_per_row;
      const int r = rest % nrows;
      const int pl = rest / nrows;
      const int64_t s = s_src[r];
      if (s < 0) continue;
      const unsigned char* from =
          src + ((plane0 + pl) * src_plane_rows + s) * row_bytes + static_cast<int64_t>(u) * unit;
      unsigned char* to = stage + static_cast<int64_t>(i) * unit;
      if (vec16)
        *reinterpret_cast<uint4*>(to) = *reinterpret_cast<const uint4*>(from);
      else
        *reinterpret_cast<uint32_t*>(to) = *reinterpret_cast<const uint32_t*>(from);
    }
    __syncthreads();
    // scatter
    for (int i = threadIdx.x; i < total_units; i += kCommitThreads) {
      const int u = i % units_per_row;
      const int rest = i / units_per_row;
      const int r = rest % nrows;
      const int pl = rest / nrows;
      const int64_t d = s_dst[r];
      if (d < 0) continue;
      unsigned char* to =
          dst + ((plane0 + pl) * dst_plane_rows + d) * row_bytes + static_cast<int64_t>(u) * unit;
      const unsigned char* from = stage + static_cast<int64_t>(i) * unit;
      if (vec16)
        *reinterpret_cast<uint4*>(to) = *reinterpret_cast<const uint4*>(from);
      else
        *reinterpret_cast<uint32_t*>(to) = *reinterpret_cast<const uint32_t*>(from);
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace sg

extern "C" int sg_kv_commit(void* dst, int64_t dst_plane_rows, const void* src, int64_t src_plane_rows,
                            int64_t num_planes, int64_t row_bytes, const int64_t* src_rows,
                            const int64_t* dst_rows, const int64_t* group_offsets, int32_t num_groups,
                            int32_t max_group_rows, int32_t* status, void* stream) {
  using namespace sg;
  if (num_groups == 0 || num_planes == 0) return SG_OK;
  if (dst == nullptr || src == nullptr || src_rows == nullptr || dst_rows == nullptr ||
      group_offsets == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_kv_commit: null pointer");
  if (num_groups < 0 || num_planes < 0 || dst_plane_rows < 1 || src_plane_rows < 1 || row_bytes < 4 ||
      row_bytes % 4 != 0 || max_group_rows < 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_kv_commit: bad sizes");
  if (row_bytes > kStageBytes)
    return fail(SG_ERR_UNSUPPORTED, "sg_kv_commit: row larger than the staging buffer");
  if (max_group_rows == 0) return SG_OK;
  const bool vec16 = (row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(src) % 16 == 0);
  int rows_per_chunk = static_cast<int>(std::min<int64_t>(64, max_group_rows));
  rows_per_chunk = static_cast<int>(std::min<int64_t>(rows_per_chunk, kStageBytes / row_bytes));
  if (rows_per_chunk < 1) rows_per_chunk = 1;
  int64_t planes_per_cta = kStageBytes / (static_cast<int64_t>(rows_per_chunk) * row_bytes);
  if (planes_per_cta < 1) planes_per_cta = 1;
  if (planes_per_cta > num_planes) planes_per_cta = num_planes;
  const int64_t grid_y = (num_planes + planes_per_cta - 1) / planes_per_cta;
  if (grid_y > 65535) return fail(SG_ERR_UNSUPPORTED, "sg_kv_commit: too many planes");
  dim3 grid(static_cast<unsigned>(num_groups), static_cast<unsigned>(grid_y), 1);
  kv_commit_kernel<<<grid, kCommitThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned char*>(dst), dst_plane_rows, static_cast<const unsigned char*>(src),
      src_plane_rows, num_planes, row_bytes, src_rows, dst_rows, group_offsets,
      static_cast<int>(planes_per_cta), rows_per_chunk, vec16, status);
  return check_launch("kv_commit_kernel");
}

// ---------------------------------------------------------------------------
// Commit straight from the acceptance output: keep rows [0] + accepted nodes
// of every tree, tree t's tail rows at slot[t] * capacity + lengths_in[t] + j.
// ---------------------------------------------------------------------------
namespace sg {
namespace {

constexpr int kMaxKeep = 64;
constexpr int kAcceptedThreads = 256;

constexpr int kCopyChunk = 4;     // rows a thread loads before it stores them
constexpr int kColsPerThread = 4; // 16- or 4-byte columns per thread

// One thread per (tree, kColsPerThread columns of the plane space), so one
// tree needs only a few CTAs and a whole wave fits on the GPU.  Kept row r of
// a tree is node out[r-1] of its tree (row 0, the root, is node 0), which
// the verify pass wrote at len + node; it moves to len + r.  The CTA stages
// the tree's path in shared memory and checks it once (node_r >= r, inside
// the slot's tail) before anything moves, so a bad path changes nothing.  A
// thread then copies its columns kCopyChunk rows at a time: all loads of a
// chunk are issued before its stores, so the row reads overlap.  In place
// this is safe because node_r >= r: a chunk writes rows below the first row
// of the next chunk, whose sources node_r' >= r' lie above them, and within a
// chunk every source is read before any destination is written.  Rows
// already in place (node_r == r, always the root) are skipped.
__global__ void __launch_bounds__(kAcceptedThreads)
kv_commit_accepted_kernel(unsigned char* arena, int64_t plane_rows, int64_t num_planes, int64_t row_bytes,
                          int64_t capacity, const int64_t* __restrict__ slots,
                          const int64_t* __restrict__ lengths_in, int64_t* __restrict__ lengths_out,
                          const int64_t* __restrict__ accept_out, int32_t max_depth, bool vec16,
                          int32_t* status) {
  __shared__ int s_node[kMaxKeep];
  __shared__ int s_bad;
  const int t = blockIdx.y;
  const int64_t* out = accept_out + static_cast<int64_t>(t) * (max_depth + 2);
  const int64_t slot = slots[t];
  const int64_t len = lengths_in[t];
  const int64_t count = out[max_depth];
  // path nodes, loaded alongside the count (validated below)
  const int64_t node_raw = (threadIdx.x < kMaxKeep - 1 && threadIdx.x < max_depth) ? out[threadIdx.x] : 0;
  int kept = static_cast<int>(count) + 1;
  const bool ok = count >= 0 && count <= max_depth && kept <= kMaxKeep && len >= 0 && len + kept <= capacity &&
                  slot >= 0 && (slot + 1) * capacity <= plane_rows;
  if (!ok) kept = 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (!ok && status != nullptr) atomicMax(status, static_cast<int32_t>(SG_ERR_CAPACITY));
    lengths_out[t] = len + kept;
  }
  if (kept <= 1) return;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  if (threadIdx.x < kept - 1) {
    const int r = threadIdx.x + 1;
    const bool good = node_raw >= r && len + node_raw < capacity;  // a root path in this slot's tail
    s_node[r - 1] = good ? static_cast<int>(node_raw) : r;
    if (!good) s_bad = 1;
  }
  __syncthreads();
  if (s_bad) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && status != nullptr)
      atomicMax(status, static_cast<int32_t>(SG_ERR_TREE));
    return;
  }
  const int unit = vec16 ? 16 : 4;
  const int64_t units_per_row = row_bytes / unit;
  const int64_t columns = num_planes * units_per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kAcceptedThreads;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kAcceptedThreads + threadIdx.x;
  unsigned char* colp[kColsPerThread];
#pragma unroll
  for (int j = 0; j < kColsPerThread; ++j) {
    const int64_t c = c0 + j * stride;
    const int64_t plane = c / units_per_row;
    const int64_t u = c % units_per_row;
    colp[j] = (c < columns) ? arena + (plane * plane_rows + slot * capacity + len) * row_bytes + u * unit : nullptr;
  }
  for (int r0 = 1; r0 < kept; r0 += kCopyChunk) {
    if (vec16) {
      uint4 v[kColsPerThread][kCopyChunk];
#pragma unroll
      for (int j = 0; j < kColsPerThread; ++j)
#pragma unroll
        for (int k = 0; k < kCopyChunk; ++k) {
          const int r = r0 + k;
          if (colp[j] != nullptr && r < kept && s_node[r - 1] != r)
            v[j][k] = *reinterpret_cast<const uint4*>(colp[j] + static_cast<int64_t>(s_node[r - 1]) * row_bytes);
        }
#pragma unroll
      for (int j = 0; j < kColsPerThread; ++j)
#pragma unroll
        for (int k = 0; k < kCopyChunk; ++k) {
          const int r = r0 + k;
          if (colp[j] != nullptr && r < kept && s_node[r - 1] != r)
            *reinterpret_cast<uint4*>(colp[j] + r * row_bytes) = v[j][k];
        }
    } else {
      uint32_t v[kColsPerThread][kCopyChunk];
#pragma unroll
      for (int j = 0; j < kColsPerThread; ++j)
#pragma unroll
        for (int k = 0; k < kCopyChunk; ++k) {
          const int r = r0 + k;
          if (colp[j] != nullptr && r < kept && s_node[r - 1] != r)
            v[j][k] = *reinterpret_cast<const uint32_t*>(colp[j] + static_cast<int64_t>(s_node[r - 1]) * row_bytes);
        }
#pragma unroll
      for (int j = 0; j < kColsPerThread; ++j)
#pragma unroll
        for (int k = 0; k < kCopyChunk; ++k) {
          const int r = r0 + k;
          if (colp[j] != nullptr && r < kept && s_node[r - 1] != r)
            *reinterpret_cast<uint32_t*>(colp[j] + r * row_bytes) = v[j][k];
        }
    }
  }
}

}  // namespace
}  // namespace sg

extern "C" int sg_kv_commit_accepted(void* arena, int64_t plane_rows, int64_t num_planes, int64_t row_bytes,
                                     int64_t capacity, const int64_t* slots, const int64_t* lengths_in,
                                     int64_t* lengths_out, const int64_t* accept_out, int32_t num_trees,
                                     int32_t max_depth, int32_t* status, void* stream) {
  using namespace sg;
  if (num_trees == 0 || num_planes == 0) return SG_OK;
  if (arena == nullptr || slots == nullptr || lengths_in == nullptr || lengths_out == nullptr ||
      accept_out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_kv_commit_accepted: null pointer");
  if (lengths_in == lengths_out)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_kv_commit_accepted: lengths_in and lengths_out must differ");
  if (num_trees < 0 || num_planes < 0 || plane_rows < 1 || capacity < 1 || row_bytes < 4 ||
      row_bytes % 4 != 0 || max_depth < 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_kv_commit_accepted: bad sizes");
  if (max_depth + 1 > kMaxKeep)
    return fail(SG_ERR_UNSUPPORTED, "sg_kv_commit_accepted: max_depth above 63");
  const bool vec16 = (row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(arena) % 16 == 0);
  const int64_t columns = num_planes * (row_bytes / (vec16 ? 16 : 4));
  const int64_t per_cta = static_cast<int64_t>(kAcceptedThreads) * kColsPerThread;
  const int64_t grid_x = (columns + per_cta - 1) / per_cta;
  if (grid_x > 0x7fffffff || num_trees > 65535)
    return fail(SG_ERR_UNSUPPORTED, "sg_kv_commit_accepted: more than 65535 trees or too many columns");
  dim3 grid(static_cast<unsigned>(grid_x), static_cast<unsigned>(num_trees), 1);
  kv_commit_accepted_kernel<<<grid, kAcceptedThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned char*>(arena), plane_rows, num_planes, row_bytes, capacity, slots, lengths_in,
      lengths_out, accept_out, max_depth, vec16, status);
  return check_launch("kv_commit_accepted_kernel");
}
