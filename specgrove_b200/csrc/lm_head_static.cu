// Fused LM-head sampling that allocates no device memory.
//
// Some hosts cannot call cudaMalloc when they want to sample: a serving
// process whose device memory is already handed over to its own pool
// allocator (a raw cudaMalloc outside that pool can fail or fragment it),
// or a foreign-language caller reaching this library through an FFI whose
// runtime only passes in buffers it allocated itself.  For them this entry
// point runs the same final RMSNorm -> LM-head GEMM (online softmax +
// Gumbel-max epilogue) -> combine kernels as sg_verify_pass, but keeps its
// scratch (the normalised rows and the per-vocab-tile partials) in one
// fixed-size array that the library declares at file scope.  The array is
// part of the library image: every GPU that loads the library holds it until
// the process exits.
#include <mutex>

#include "gemm.cuh"
#include "layers.cuh"

namespace sg {
namespace {

// Scratch of the no-allocation sampler: normalised rows (bf16) followed by
// the per-(row, vocab tile) partials (float4), both 256-byte aligned.
__device__ __align__(256) uint8_t g_lm_head_scratch[SG_LM_HEAD_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
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

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

size_t lm_head_static_scratch_need(int rows, int hidden, int vocab) {
  const size_t tiles = static_cast<size_t>((vocab + gemm::BN - 1) / gemm::BN);
  return align256(static_cast<size_t>(rows) * hidden * 2) + static_cast<size_t>(rows) * tiles * sizeof(float4);
}

}  // namespace sg

extern "C" int sg_lm_head_sample_static(const float* x, const void* final_norm, const void* lm_head, int32_t rows,
                                        int32_t hidden, int32_t vocab, float rms_eps, const int32_t* row_node,
                                        const int64_t* row_request, uint64_t seed, float temperature, float* lse,
                                        int64_t* posterior, void* stream) {
  using namespace sg;
  if (rows == 0) return SG_OK;
  if (x == nullptr || final_norm == nullptr || lm_head == nullptr || row_node == nullptr ||
      row_request == nullptr || lse == nullptr || posterior == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_lm_head_sample_static: null pointer");
  if (rows < 0 || hidden < 64 || hidden % gemm::BK != 0 || vocab < 32 || vocab % 32 != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_lm_head_sample_static: bad sizes (hidden % 64, vocab % 32)");
  if (!(temperature > 0.f)) return fail(SG_ERR_INVALID_ARGUMENT, "sg_lm_head_sample_static: temperature must be > 0");
  const size_t need = lm_head_static_scratch_need(rows, hidden, vocab);
  if (need > SG_LM_HEAD_STATIC_SCRATCH_BYTES) {
    set_error("sg_lm_head_sample_static: %d rows x hidden %d x vocab %d need %zu scratch bytes, the static "
              "scratch holds %u",
              rows, hidden, vocab, need, static_cast<unsigned>(SG_LM_HEAD_STATIC_SCRATCH_BYTES));
    return SG_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int st = scratch_address(&scratch);
  if (st != SG_OK) return st;
  __nv_bfloat16* xn = static_cast<__nv_bfloat16*>(scratch);
  float4* partials = reinterpret_cast<float4*>(static_cast<uint8_t*>(scratch) +
                                               align256(static_cast<size_t>(rows) * hidden * 2));
  const int tiles = (vocab + gemm::BN - 1) / gemm::BN;
  CUtensorMap a_map, b_map;
  if ((st = make_tmap_2d_bf16(&a_map, xn, hidden, rows, static_cast<uint64_t>(hidden) * 2, gemm::BK, gemm::BM)) !=
      SG_OK)
    return st;
  if ((st = make_tmap_2d_bf16(&b_map, lm_head, hidden, vocab, static_cast<uint64_t>(hidden) * 2, gemm::BK,
                              gemm::BN)) != SG_OK)
    return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Every scratch element read below is written earlier in this call (all
  // rows x hidden normalised values, all rows x tiles partials), so nothing
  // has to be cleared between calls.
  if ((st = layers::launch_rmsnorm(x, static_cast<const __nv_bfloat16*>(final_norm), hidden, rows, rms_eps, xn, s)) !=
      SG_OK)
    return st;
  gemm::EpiLmHead::Params pl;
  pl.partials = partials;
  pl.n_tiles = tiles;
  pl.row_local = row_node;
  pl.row_request = row_request;
  pl.seed = seed;
  pl.inv_temp = 1.0f / temperature;
  pl.status = nullptr;
  if ((st = gemm::launch<gemm::EpiLmHead>(a_map, b_map, gemm::make_shape(rows, vocab, hidden), pl, s)) != SG_OK)
    return st;
  return layers::launch_lm_combine(partials, tiles, rows, lse, posterior, s);
}
