// Host helpers: TMA tensor-map encoding through the runtime's driver entry
// point (no link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <mutex>

#include "sm100.cuh"

namespace sg {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void resolve_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  std::call_once(g_encode_once, resolve_encode);
  if (g_encode == nullptr) return fail(SG_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || row_stride_bytes % 16 != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "TMA operand not 16-byte aligned");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u", static_cast<int>(r),
              static_cast<unsigned long long>(inner), static_cast<unsigned long long>(outer), box_inner,
              box_outer);
    return SG_ERR_CUDA;
  }
  return SG_OK;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                      uint64_t row_stride_bytes, uint64_t plane_stride_bytes, uint32_t box_inner,
                      uint32_t box_rows) {
  std::call_once(g_encode_once, resolve_encode);
  if (g_encode == nullptr) return fail(SG_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || row_stride_bytes % 16 != 0 || plane_stride_bytes % 16 != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "TMA operand not 16-byte aligned");
  cuuint64_t dims[3] = {inner, rows, planes};
  cuuint64_t strides[2] = {row_stride_bytes, plane_stride_bytes};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3d) failed (%d)", static_cast<int>(r));
    return SG_ERR_CUDA;
  }
  return SG_OK;
}

}  // namespace sg
