// Fused LM-head sampling that allocates no device memory.
//
// Some hosts cannot call cudaMalloc when they want to sample: a serving
// process whose device memory is already handed over to its own pool
// allocator (a raw cudaMalloc outside that pool can fail or fragment it),
// or a foreign-language caller reaching this library through an FFI whose
// runtime only passes in buffers it allocated itself.  For them this entry
// point runs the same final RMSNorm -> LM-head GEMM (softmax + sampling
// epilogue) -> combine kernels as sg_verify_pass, but keeps its scratch (a
// status word, the normalised rows and the per-vocab-tile partials) in one
// fixed-size array that the library declares at file scope.  The array is
// part of the library image: every GPU that loads the library holds it until
// the process exits.
#include <mutex>

#include "lm_head.cuh"

namespace sg {
namespace {

// Scratch of the no-allocation sampler (layout of lm_head_run).
__device__ __align__(256) uint8_t g_lm_head_scratch[SG_LM_HEAD_STATIC_SCRATCH_BYTES];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Host code cannot use g_lm_head_scratch's name as a device address (it is a
// host-side stand-in); resolve the real address once per device.
int scratch_address(void** out) {
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(SG_ERR_UNSUPPORTED, "sg_lm_head_sample_static: device index");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_lm_head_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      set_error("sg_lm_head_sample_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(err));
      return SG_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return SG_OK;
}

}  // namespace
}  // namespace sg

extern "C" int sg_lm_head_sample_static(const float* x, const void* final_norm, const void* lm_head, int32_t rows,
                                        int32_t hidden, int32_t vocab, float rms_eps, const int32_t* row_node,
                                        const int64_t* row_request, uint64_t seed, float temperature, float* lse,
                                        int64_t* posterior, void* stream) {
  using namespace sg;
  if (rows == 0) return SG_OK;
  int st = lm_head_check("sg_lm_head_sample_static", x, final_norm, lm_head, rows, hidden, vocab, row_node,
                         row_request, temperature, lse, posterior);
  if (st != SG_OK) return st;
  const size_t need = lm_head_scratch_need(rows, hidden, vocab);
  if (need > SG_LM_HEAD_STATIC_SCRATCH_BYTES) {
    set_error("sg_lm_head_sample_static: %d rows x hidden %d x vocab %d need %zu scratch bytes, the static "
              "scratch holds %u",
              rows, hidden, vocab, need, static_cast<unsigned>(SG_LM_HEAD_STATIC_SCRATCH_BYTES));
    return SG_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  if ((st = scratch_address(&scratch)) != SG_OK) return st;
  return lm_head_run(x, final_norm, lm_head, rows, hidden, vocab, rms_eps, row_node, row_request, seed, temperature,
                     lse, posterior, scratch, static_cast<cudaStream_t>(stream));
}
