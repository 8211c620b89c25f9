// Shared implementation of the stand-alone LM-head sampling entry points
// (sg_lm_head_sample with a caller workspace, sg_lm_head_sample_static with
// the library's static scratch).
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace sg {

// Form of the RMSNorms of the verify pass (engine.cu): false (the default)
// runs them as kernels that write normalised bf16 rows; true (SG_NORM_FUSED=1)
// folds them into GEMM epilogues (bf16(x * w) rows, each row's GEMM output
// scaled by rsqrt(mean(x^2) + eps)).  The stand-alone sampler follows the
// same form for the final norm, so it draws what the pass draws.
bool qkv_fused();
bool norm_fused();

// Scratch bytes for `rows` rows: a 256-byte status word, the normalised rows
// (bf16) and the per-(row, vocab tile) partials (float4), 256-byte aligned.
size_t lm_head_scratch_need(int rows, int hidden, int vocab);

// Argument checks shared by both entry points (pointers, sizes, alignment,
// temperature >= 0); sets the error detail under the caller's name.
int lm_head_check(const char* who, const float* x, const void* final_norm, const void* lm_head, int32_t rows,
                  int32_t hidden, int32_t vocab, const int32_t* row_node, const int64_t* row_request,
                  float temperature, const float* lse, const int64_t* posterior);

// Enqueue norm -> LM head + sampling -> combine with `scratch` (256-byte
// aligned, lm_head_scratch_need bytes).  temperature 0 selects greedy rows.
// With `normed` (bf16 [rows, hidden] already-normalised rows) the norm is
// skipped and x / final_norm are ignored.
int lm_head_run(const float* x, const void* final_norm, const void* lm_head, int32_t rows, int32_t hidden,
                int32_t vocab, float rms_eps, const int32_t* row_node, const int64_t* row_request, uint64_t seed,
                float temperature, float* lse, int64_t* posterior, void* scratch, cudaStream_t stream,
                const void* normed = nullptr);

}  // namespace sg
