// C-ABI entry for the tcgen05 GEMM (plain library-style call used by tests and
// by hosts that drive the layer GEMMs themselves).
#include "gemm.cuh"

namespace sg {
namespace {

int check_gemm_args(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K) {
  if (A == nullptr || B == nullptr) return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: null operand");
  if (M < 0 || N <= 0 || K <= 0) return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: bad sizes");
  if (K % gemm::BK != 0) return fail(SG_ERR_UNSUPPORTED, "sg_gemm_bf16: K must be a multiple of 64");
  if (N % 32 != 0) return fail(SG_ERR_UNSUPPORTED, "sg_gemm_bf16: N must be a multiple of 32");
  if (lda < K || ldb < K || (lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: leading dimensions");
  return SG_OK;
}

}  // namespace
}  // namespace sg

namespace sg {
namespace {

// Layout of a split workspace: partial accumulators, then the flags.
bool split_from(void* workspace, size_t bytes, gemm::SplitWorkspace& ws) {
  const int sms = device_sm_count();
  const size_t pbytes = gemm::split_partial_bytes(sms);
  const size_t need = pbytes + gemm::split_partial_tiles(sms) * sizeof(int);
  if (workspace == nullptr || sms <= 0 || bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return false;
  ws.partials = static_cast<float*>(workspace);
  ws.flags = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + pbytes);
  ws.partial_tiles = gemm::split_partial_tiles(sms);
  return true;
}

int gemm_dispatch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int32_t M,
                  int32_t N, int32_t K, int32_t epilogue, void* aux, int64_t ld_aux, int32_t* status,
                  const gemm::SplitWorkspace* split, void* stream);

}  // namespace
}  // namespace sg

extern "C" size_t sg_gemm_split_workspace_bytes(void) {
  const int sms = sg::device_sm_count();
  return sg::gemm::split_partial_bytes(sms) + sg::gemm::split_partial_tiles(sms) * sizeof(int);
}

extern "C" int sg_gemm_split_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sg;
  gemm::SplitWorkspace ws;
  if (!split_from(workspace, workspace_bytes, ws))
    return fail(SG_ERR_WORKSPACE, "sg_gemm_split_workspace_init: workspace too small or not 256-byte aligned");
  SG_CUDA_CHECK(cudaMemsetAsync(ws.flags, 0, ws.partial_tiles * sizeof(int), static_cast<cudaStream_t>(stream)));
  return SG_OK;
}

extern "C" int sg_gemm_bf16_ws(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                               int32_t M, int32_t N, int32_t K, int32_t epilogue, void* aux, int64_t ld_aux,
                               int32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sg;
  gemm::SplitWorkspace ws;
  const bool use = split_from(workspace, workspace_bytes, ws);
  return gemm_dispatch(A, lda, B, ldb, C, ldc, M, N, K, epilogue, aux, ld_aux, status, use ? &ws : nullptr, stream);
}

extern "C" int sg_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                            int32_t M, int32_t N, int32_t K, int32_t epilogue, void* aux, int64_t ld_aux,
                            int32_t* status, void* stream) {
  return sg::gemm_dispatch(A, lda, B, ldb, C, ldc, M, N, K, epilogue, aux, ld_aux, status, nullptr, stream);
}

namespace sg {
namespace {
int gemm_dispatch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int32_t M,
                  int32_t N, int32_t K, int32_t epilogue, void* aux, int64_t ld_aux, int32_t* status,
                  const gemm::SplitWorkspace* split, void* stream) {
  if (M == 0) return SG_OK;
  int st = check_gemm_args(A, lda, B, ldb, M, N, K);
  if (st != SG_OK) return st;
  if (C == nullptr) return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: null output");
  CUtensorMap ta, tb;
  st = make_tmap_2d_bf16(&ta, A, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(lda) * 2,
                         gemm::BK, gemm::BM);
  if (st != SG_OK) return st;
  st = make_tmap_2d_bf16(&tb, B, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ldb) * 2,
                         gemm::BK, gemm::BN);
  if (st != SG_OK) return st;
  const gemm::Shape shape = gemm::make_shape(M, N, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (epilogue) {
    case SG_EPI_STORE_BF16: {
      if (ldc % 8 != 0) return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: ldc");
      gemm::EpiStoreBf16::Params p{static_cast<__nv_bfloat16*>(C), ldc, status};
      return gemm::launch<gemm::EpiStoreBf16>(ta, tb, shape, p, s, split);
    }
    case SG_EPI_STORE_F32: {
      if (ldc % 4 != 0) return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: ldc");
      gemm::EpiStoreF32::Params p{static_cast<float*>(C), ldc, status};
      return gemm::launch<gemm::EpiStoreF32>(ta, tb, shape, p, s, split);
    }
    case SG_EPI_RESIDUAL: {
      if (ldc % 4 != 0 || (aux != nullptr && ld_aux % 8 != 0))
        return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: residual strides");
      gemm::EpiResidual::Params p{static_cast<float*>(C), ldc, static_cast<__nv_bfloat16*>(aux), ld_aux, status};
      return gemm::launch<gemm::EpiResidual>(ta, tb, shape, p, s, split);
    }
    case SG_EPI_SWIGLU: {
      if (N % gemm::BN != 0 || ldc % 8 != 0)
        return fail(SG_ERR_UNSUPPORTED, "sg_gemm_bf16: SwiGLU needs N % 256 == 0");
      gemm::EpiSwiGlu::Params p{static_cast<__nv_bfloat16*>(C), ldc, status};
      return gemm::launch<gemm::EpiSwiGlu>(ta, tb, shape, p, s, split);
    }
    default:
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_gemm_bf16: unknown epilogue");
  }
}
}  // namespace
}  // namespace sg
