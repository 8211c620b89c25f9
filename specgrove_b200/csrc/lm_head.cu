// Final RMSNorm + LM head fused with softmax and sampling, outside the pass.
//
// The same three kernels as the sampling stage of sg_verify_pass (final
// norm, LM-head GEMM with the two-level sampling epilogue of gemm.cuh,
// lm_combine) over caller-given residual rows.  This is the seam of the
// reference's lazy-projection verifiers, which receive hidden states and the
// LM-head module instead of logits (continuous_tree_block_decode.py:1795-1808,
// 1933-1964; fused_tree_sampling.py:2758-3031).
#include "gemm.cuh"
#include "layers.cuh"
#include "lm_head.cuh"

namespace sg {

namespace {
size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
}  // namespace

size_t lm_head_scratch_need(int rows, int hidden, int vocab) {
  const size_t tiles = static_cast<size_t>((vocab + gemm::BN - 1) / gemm::BN);
  return 256 /* status word */ + align256(static_cast<size_t>(rows) * hidden * 2) +
         align256(static_cast<size_t>(rows) * tiles * sizeof(float4)) + static_cast<size_t>(rows) * sizeof(float);
}

int lm_head_check(const char* who, const float* x, const void* final_norm, const void* lm_head, int32_t rows,
                  int32_t hidden, int32_t vocab, const int32_t* row_node, const int64_t* row_request,
                  float temperature, const float* lse, const int64_t* posterior) {
  if (x == nullptr || final_norm == nullptr || lm_head == nullptr || row_node == nullptr ||
      row_request == nullptr || lse == nullptr || posterior == nullptr) {
    set_error("%s: null pointer", who);
    return SG_ERR_INVALID_ARGUMENT;
  }
  if (rows < 0 || hidden < 64 || hidden % gemm::BK != 0 || vocab < 32 || vocab % 32 != 0) {
    set_error("%s: bad sizes (rows >= 0, hidden % 64 == 0, vocab % 32 == 0)", who);
    return SG_ERR_INVALID_ARGUMENT;
  }
  if (!(temperature >= 0.f) || temperature == INFINITY) {
    set_error("%s: temperature must be finite and >= 0 (0 = greedy)", who);
    return SG_ERR_INVALID_ARGUMENT;
  }
  // x is read as float4 (rmsnorm), final_norm as bf16 pairs, lm_head by TMA;
  // the row keys and outputs as whole words.  A misaligned pointer would
  // raise a sticky device fault instead of an error code.
  if (!aligned(x, 16) || !aligned(final_norm, 4) || !aligned(lm_head, 16) || !aligned(row_node, 4) ||
      !aligned(row_request, 8) || !aligned(lse, 4) || !aligned(posterior, 8)) {
    set_error("%s: misaligned pointer (x and lm_head 16 B, row_request and posterior 8 B, others 4 B)", who);
    return SG_ERR_INVALID_ARGUMENT;
  }
  return SG_OK;
}

int lm_head_run(const float* x, const void* final_norm, const void* lm_head, int32_t rows, int32_t hidden,
                int32_t vocab, float rms_eps, const int32_t* row_node, const int64_t* row_request, uint64_t seed,
                float temperature, float* lse, int64_t* posterior, void* scratch, cudaStream_t s,
                const void* normed) {
  int32_t* status = static_cast<int32_t*>(scratch);
  __nv_bfloat16* xn = normed != nullptr ? static_cast<__nv_bfloat16*>(const_cast<void*>(normed))
                                        : reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(scratch) + 256);
  float4* partials = reinterpret_cast<float4*>(static_cast<uint8_t*>(scratch) + 256 +
                                               align256(static_cast<size_t>(rows) * hidden * 2));
  const int tiles = (vocab + gemm::BN - 1) / gemm::BN;
  // the final RMSNorm in the pass's form: a kernel writing normalised bf16
  // rows, or (folded) xn = bf16(x * final_norm) with each row's logits scaled
  // by rsqrt(mean(x^2) + eps)
  const bool fold = normed == nullptr && norm_fused();
  float* ssq = !fold ? nullptr
                     : reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(partials) +
                                                align256(static_cast<size_t>(rows) * tiles * 16));
  CUtensorMap a_map, b_map;
  int st;
  if ((st = make_tmap_2d_bf16(&a_map, xn, hidden, rows, static_cast<uint64_t>(hidden) * 2, gemm::BK, gemm::BM)) !=
      SG_OK)
    return st;
  if ((st = make_tmap_2d_bf16(&b_map, lm_head, hidden, vocab, static_cast<uint64_t>(hidden) * 2, gemm::BK,
                              gemm::BN)) != SG_OK)
    return st;
  // The status word starts at zero; every other scratch value read below is
  // written earlier in this call (all rows x hidden normalised values, all
  // rows x tiles partials).
  SG_CUDA_CHECK(cudaMemsetAsync(status, 0, sizeof(int32_t), s));
  if (fold &&
      (st = layers::launch_norm_fold(x, static_cast<const __nv_bfloat16*>(final_norm), hidden, rows, xn, ssq, s)) !=
          SG_OK)
    return st;
  if (normed == nullptr && !fold &&
      (st = layers::launch_rmsnorm(x, static_cast<const __nv_bfloat16*>(final_norm), hidden, rows, rms_eps, xn, s)) !=
          SG_OK)
    return st;
  gemm::EpiLmHead::Params pl;
  pl.partials = partials;
  pl.n_tiles = tiles;
  pl.row_local = row_node;
  pl.row_request = row_request;
  pl.seed = seed;
  pl.greedy = temperature == 0.f ? 1 : 0;
  pl.inv_temp = pl.greedy ? 1.0f : 1.0f / temperature;
  pl.status = status;
  pl.rn = gemm::RowNorm{ssq, 1, 1.0f / static_cast<float>(hidden), rms_eps};
  if ((st = gemm::launch<gemm::EpiLmHead>(a_map, b_map, gemm::make_shape(rows, vocab, hidden), pl, s)) != SG_OK)
    return st;
  // A GEMM that gave up on a bounded wait leaves partial results: the
  // combine then writes posterior = -1 and lse = NaN for every row.
  return layers::launch_lm_combine(partials, tiles, rows, lse, posterior, status, s);
}

}  // namespace sg

extern "C" size_t sg_lm_head_sample_workspace_bytes(int32_t rows, int32_t hidden, int32_t vocab) {
  if (rows < 0 || hidden < 0 || vocab < 0) return 0;
  return sg::lm_head_scratch_need(rows, hidden, vocab);
}

extern "C" int sg_lm_head_sample(const float* x, const void* final_norm, const void* lm_head, int32_t rows,
                                 int32_t hidden, int32_t vocab, float rms_eps, const int32_t* row_node,
                                 const int64_t* row_request, uint64_t seed, float temperature, float* lse,
                                 int64_t* posterior, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sg;
  if (rows == 0) return SG_OK;
  int st = lm_head_check("sg_lm_head_sample", x, final_norm, lm_head, rows, hidden, vocab, row_node, row_request,
                         temperature, lse, posterior);
  if (st != SG_OK) return st;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_lm_head_sample: workspace must be a 256-byte aligned device buffer");
  const size_t need = lm_head_scratch_need(rows, hidden, vocab);
  if (workspace_bytes < need) {
    set_error("sg_lm_head_sample: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    return SG_ERR_WORKSPACE;
  }
  return lm_head_run(x, final_norm, lm_head, rows, hidden, vocab, rms_eps, row_node, row_request, seed, temperature,
                     lse, posterior, workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int sg_lm_head_sample_bf16(const void* xn, const void* lm_head, int32_t rows, int32_t hidden,
                                      int32_t vocab, const int32_t* row_node, const int64_t* row_request,
                                      uint64_t seed, float temperature, float* lse, int64_t* posterior,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sg;
  if (rows == 0) return SG_OK;
  // the checks of the fp32 entry, with the normed rows standing in for x and
  // the final norm (16-byte aligned rows: TMA reads them directly)
  int st = lm_head_check("sg_lm_head_sample_bf16", static_cast<const float*>(xn), lm_head, lm_head, rows, hidden,
                         vocab, row_node, row_request, temperature, lse, posterior);
  if (st != SG_OK) return st;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_lm_head_sample_bf16: workspace must be a 256-byte aligned buffer");
  const size_t need = lm_head_scratch_need(rows, hidden, vocab);
  if (workspace_bytes < need) {
    set_error("sg_lm_head_sample_bf16: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    return SG_ERR_WORKSPACE;
  }
  return lm_head_run(nullptr, nullptr, lm_head, rows, hidden, vocab, 0.f, row_node, row_request, seed, temperature,
                     lse, posterior, workspace, static_cast<cudaStream_t>(stream), xn);
}
