// The packed tree-verification pass: one target forward over every request's
// selected tree rows, fused LM head + sampling, tree walk and KV commit.
//
// Reference call chain replaced (continuous_tree_block_decode.py:1748-2246):
//   _pack_cache_sequence (:313-361)  -> not needed: attention reads the arena
//   _packed_block_inputs (:500-546)  -> tree_meta_kernel (bitsets, positions)
//   engine.target_hidden_forward     -> embed + 36 x {norm, QKV GEMM, q/k norm
//     (engine.py:499-517)               + RoPE + arena tail write, tree
//                                       attention, O GEMM + residual, norm,
//                                       gate/up GEMM + SwiGLU, down GEMM +
//                                       residual}
//   lm_head + probabilities          -> LM-head GEMM with online softmax and
//     (:1809-1824)                      Gumbel-max sampling epilogue
//   verifier (:1965-2107)            -> tree walk over the sampled tokens
//   append_packed_sequence (:2121)   -> in-place arena commit
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>
#include <memory>
#include <vector>

#include "attention.cuh"
#include "gemm.cuh"
#include "layers.cuh"
#include "lm_head.cuh"

namespace sg {

// SG_QKV_FUSED=0 runs the q/k norm + RoPE + KV write as its own kernel after
// a plain q/k/v GEMM (the two forms compute the same values; the switch is
// for A/B timing).
bool qkv_fused() {
  static const bool fused = [] {
    const char* v = std::getenv("SG_QKV_FUSED");
    return v == nullptr || v[0] != '0';
  }();
  return fused;
}

// SG_NORM_FUSED=1 folds the input and post-attention RMSNorms into the
// neighbouring GEMM epilogues (the residual epilogue writes bf16(x * w) and
// per-tile sums of squares, the next GEMM scales each row by
// rsqrt(mean(x^2) + eps)) instead of running them as kernels.  Off by
// default: it measured even on the 2048-row wave and 5% slower on the
// 512-row wave, whose residual GEMMs run split over two CTAs per tile with
// the heavier epilogue on the owner's critical path.  The folded form needs
// the fused q/k/v epilogue.
// The pass's fp32 residual stream (read and written by every residual GEMM
// epilogue and norm of every layer) is kept persisting in L2: an access-policy
// window on every kernel of the pass over an L2 set-aside of this process's
// context, so the layer's weight and K/V streams do not evict it (about 1% of
// the configuration-4 pass).  SG_L2_PERSIST=0 turns it off.
bool l2_persist() {
  static const bool on = [] {
    const char* v = std::getenv("SG_L2_PERSIST");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

bool norm_fused() {
  static const bool fused = [] {
    const char* v = std::getenv("SG_NORM_FUSED");
    return v != nullptr && v[0] == '1';
  }();
  return fused && qkv_fused();
}

namespace {

// Narrow tile width for the residual (O and down) projections: 160 columns
// make a 2560-wide output 16 tiles per 128 rows instead of 10, so a
// 512-row wave keeps 64 SMs busy instead of 40 (configuration 3: 8.83 ->
// 8.35 ms per pass).  Where 256-wide tiles already fill a wave the narrow
// tile is slower (configuration 4: 37.1 against 35.0 ms: more A re-reads per
// flop), so each pass picks the width (residual_width).
constexpr int kNarrowBN = 160;

// Tile width of a pass's residual projections: the narrow tile when its
// waves, weighted by its width and a 1.25 efficiency penalty, beat the
// 256-wide tile's waves.
int residual_width(int rows, int hidden, int sms) {
  static const int forced = [] {  // SG_RESIDUAL_BN=160 or 256 pins the width (tests, A/B timing)
    const char* v = std::getenv("SG_RESIDUAL_BN");
    const int w = v != nullptr ? std::atoi(v) : 0;
    return w == kNarrowBN || w == gemm::BN ? w : 0;
  }();
  if (forced != 0) return forced;
  const int mt = (rows + gemm::BM - 1) / gemm::BM;
  const int t_wide = mt * ((hidden + gemm::BN - 1) / gemm::BN);
  const int t_narrow = mt * ((hidden + kNarrowBN - 1) / kNarrowBN);
  const double wide = static_cast<double>((t_wide + sms - 1) / sms);
  const double narrow = static_cast<double>((t_narrow + sms - 1) / sms) * kNarrowBN / gemm::BN * 1.25;
  return narrow < wide ? kNarrowBN : gemm::BN;
}

enum { W_IN_NORM = 0, W_QKV, W_Q_NORM, W_K_NORM, W_O, W_POST_NORM, W_GATE_UP, W_DOWN, W_COUNT };

struct LayerMaps {
  CUtensorMap qkv, o, gate_up, down;
  CUtensorMap o_narrow, down_narrow;  // the same weights with kNarrowBN-row boxes
};

struct Engine {
  sg_model_desc model;
  std::vector<const void*> layer_ptrs;
  sg_arena_desc arena;
  int max_rows, max_requests;
  int device;
  // tensor maps
  std::vector<LayerMaps> maps;
  CUtensorMap lm_map, xn_map, attn_map, h_map, kv_map;
  // workspace
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  float* x;
  size_t l2_window_bytes = 0;  // residual-stream bytes kept persisting in L2 (0: off)
  size_t l2_setaside = 0;      // the context's persisting L2 set-aside
  __nv_bfloat16 *xn, *qkv, *q, *attn, *h;
  float* ssq;      // [max_rows][ss_parts] row sums of squares of the residual (folded RMSNorms)
  int ss_parts;    // column tiles of the residual GEMMs
  float4* partials;
  float* lse_ws;
  int64_t* posterior_ws;
  layers::RowMeta meta;
  layers::AttentionWork work;
  int vocab_tiles;
  // Stream-K workspace for GEMMs with fewer tiles than SMs (small waves):
  // their k-blocks are spread over up to twice as many CTAs.
  gemm::SplitWorkspace split = {nullptr, nullptr, 0};
  int sms = 0;
  std::unique_ptr<struct DraftState> draft;  // set for a drafter engine
  ~Engine();
};

// The drafter's extra weights and per-call buffers (sg_draft_engine_create).
struct DraftState {
  sg_draft_desc desc;
  CUtensorMap fc_map;                 // B operand: fc [hidden, F * hidden]
  CUtensorMap th_map;                 // A operand: normed context rows [max_update, hidden]
  std::vector<CUtensorMap> kv_maps;   // B operand per layer: the k|v rows of the fused q|k|v weight
  void* buffer = nullptr;
  float* th32;                        // [max_update, hidden] fc output
  __nv_bfloat16* th;                  // [max_update, hidden] hidden_norm(fc(features))
  layers::RowMeta ctx_meta;           // context rows: position, tree, local, rope, arena_row
  int64_t* block_offsets;             // [max_requests + 1]
  int64_t* prefix;                    // [max_requests] cache rows + update rows
  int64_t* block_tokens;              // [max_requests * block]
  ~DraftState() {
    if (buffer != nullptr) cudaFree(buffer);
  }
};

Engine::~Engine() {
  if (workspace != nullptr) cudaFree(workspace);
}

template <typename T>
T* carve(uint8_t*& cursor, size_t count) {
  uintptr_t p = (reinterpret_cast<uintptr_t>(cursor) + 255) & ~uintptr_t(255);
  cursor = reinterpret_cast<uint8_t*>(p + count * sizeof(T));
  return reinterpret_cast<T*>(p);
}


inline void trace(const sg_wave_desc& w, int point, cudaStream_t stream) {
  if (w.trace_events != nullptr && w.trace_events[point] != nullptr)
    cudaEventRecord(static_cast<cudaEvent_t>(w.trace_events[point]), stream);
}

// Upper bound on the tree attention's (request, kv head, 128-row block)
// items: per kv head, sum over requests of ceil(n_i * G / 128) <= rows * G /
// 128 + requests, and requests <= rows.
int attention_item_capacity(const sg_model_desc& m, int rows) {
  const int G = m.num_q_heads / m.num_kv_heads;
  return m.num_kv_heads * ((rows * G + 127) / 128 + rows);
}

size_t workspace_size(const sg_model_desc& m, int rows, int sms) {
  const size_t H = m.hidden, D = m.head_dim, I = m.intermediate;
  const size_t qkv = (m.num_q_heads + 2 * m.num_kv_heads) * D;
  const size_t vt = (m.vocab + gemm::BN - 1) / gemm::BN;
  size_t s = 0;
  s += rows * H * 4 + 256;                    // x
  s += rows * H * 2 + 256;                    // xn
  s += rows * qkv * 2 + 256;                  // qkv
  s += rows * m.num_q_heads * D * 2 + 256;    // q
  s += rows * m.num_q_heads * D * 2 + 256;    // attn
  s += rows * I * 2 + 256;                    // h
  s += rows * vt * 16 + 256;                  // partials
  s += rows * 4 + 256;                        // lse
  s += rows * 8 + 256;                        // posterior
  s += rows * ((H + kNarrowBN - 1) / kNarrowBN) * 4 + 256;  // row sums of squares (folded norms)
  s += rows * layers::kAncWords * 4 + 256;    // anc
  s += rows * 4 * 3 + 3 * 256;                // position, tree, local
  s += rows * 8 + 256;                        // request id
  s += rows * 4 + 256;                        // attention order (R <= rows)
  s += rows * (D / 2) * 8 + 256;              // per-pass rotary table (cos, sin)
  s += rows * 8 + 256;                        // per-pass K/V arena row
  s += attention_item_capacity(m, rows) * 4 + 256;  // attention work list
  s += (m.num_layers + 1) * 4 + 256;          // item count, per-layer work counters
  s += gemm::split_partial_bytes(sms) + 256;  // stream-K partial accumulators
  s += gemm::split_partial_tiles(sms) * sizeof(int) + 256;  // stream-K flags
  return s + 4096;
}

int check_model(const sg_model_desc& m) {
  if (m.num_layers < 1 || m.hidden < 64 || m.num_q_heads < 1 || m.num_kv_heads < 1 ||
      m.num_q_heads % m.num_kv_heads != 0 || (m.head_dim != 64 && m.head_dim != 128) || m.intermediate < 64 ||
      m.vocab < 32)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_engine_create: bad model shape");
  if (m.hidden % gemm::BK != 0 || (m.num_q_heads * m.head_dim) % gemm::BK != 0 ||
      m.intermediate % gemm::BK != 0 || (2 * m.intermediate) % gemm::BN != 0 || m.vocab % 32 != 0 ||
      m.hidden % 32 != 0)
    return fail(SG_ERR_UNSUPPORTED, "sg_engine_create: shape not tileable (hidden, q width, intermediate % 64, "
                                    "2*intermediate % 256, vocab % 32)");
  if (m.embed == nullptr || m.final_norm == nullptr || m.lm_head == nullptr || m.inv_freq == nullptr ||
      m.layers == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_engine_create: null weight");
  return SG_OK;
}

}  // namespace
}  // namespace sg

using sg::Engine;

namespace sg {
namespace {

// Builds an engine (weights' tensor maps, workspace) for `model` over `arena`.
int create_engine(const sg_model_desc* model, const sg_arena_desc* arena, int32_t max_rows, int32_t max_requests,
                  std::unique_ptr<Engine>& e) {
  if (model == nullptr || arena == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_engine_create: null argument");
  int st = check_model(*model);
  if (st != SG_OK) return st;
  if (max_rows < 1 || max_requests < 1 || arena->storage == nullptr || arena->num_slots < 1 || arena->capacity < 1)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_engine_create: bad sizes");
  e.reset(new Engine());
  e->model = *model;
  e->layer_ptrs.assign(model->layers, model->layers + static_cast<size_t>(model->num_layers) * W_COUNT);
  e->model.layers = e->layer_ptrs.data();
  e->arena = *arena;
  e->max_rows = max_rows;
  e->max_requests = max_requests;
  SG_CUDA_CHECK(cudaGetDevice(&e->device));
  const sg_model_desc& m = e->model;
  const int H = m.hidden, D = m.head_dim, I = m.intermediate;
  const int qkv_n = (m.num_q_heads + 2 * m.num_kv_heads) * D;
  const int qw = m.num_q_heads * D;
  for (int l = 0; l < m.num_layers; ++l)
    for (int w = 0; w < W_COUNT; ++w)
      if (e->layer_ptrs[l * W_COUNT + w] == nullptr) return fail(SG_ERR_INVALID_ARGUMENT, "null layer weight");
  e->maps.resize(m.num_layers);
  for (int l = 0; l < m.num_layers; ++l) {
    const void* const* lw = &e->layer_ptrs[l * W_COUNT];
    LayerMaps& lm = e->maps[l];
    if ((st = make_tmap_2d_bf16(&lm.qkv, lw[W_QKV], H, qkv_n, H * 2, gemm::BK, gemm::BN)) != SG_OK) return st;
    if ((st = make_tmap_2d_bf16(&lm.o, lw[W_O], qw, H, qw * 2, gemm::BK, gemm::BN)) != SG_OK) return st;
    if ((st = make_tmap_2d_bf16(&lm.o_narrow, lw[W_O], qw, H, qw * 2, gemm::BK, kNarrowBN)) != SG_OK) return st;
    if ((st = make_tmap_2d_bf16(&lm.gate_up, lw[W_GATE_UP], H, 2 * I, H * 2, gemm::BK, gemm::BN)) != SG_OK)
      return st;
    if ((st = make_tmap_2d_bf16(&lm.down, lw[W_DOWN], I, H, I * 2, gemm::BK, gemm::BN)) != SG_OK) return st;
    if ((st = make_tmap_2d_bf16(&lm.down_narrow, lw[W_DOWN], I, H, I * 2, gemm::BK, kNarrowBN)) != SG_OK) return st;
  }
  if ((st = make_tmap_2d_bf16(&e->lm_map, m.lm_head, H, m.vocab, H * 2, gemm::BK, gemm::BN)) != SG_OK) return st;
  {
    const uint64_t plane_rows = static_cast<uint64_t>(arena->num_slots) * arena->capacity;
    const uint64_t planes = static_cast<uint64_t>(m.num_layers) * 2 * m.num_kv_heads;
    if ((st = make_tmap_3d_bf16(&e->kv_map, arena->storage, D, plane_rows, planes, D * 2, plane_rows * D * 2, 64,
                                attn::kKeyTile)) != SG_OK)
      return st;
  }

  e->sms = device_sm_count();
  if (e->sms <= 0) return fail(SG_ERR_CUDA, "sg_engine_create: no CUDA device");
  e->workspace_bytes = workspace_size(m, max_rows, e->sms);
  SG_CUDA_CHECK(cudaMalloc(&e->workspace, e->workspace_bytes));
  uint8_t* cur = static_cast<uint8_t*>(e->workspace);
  e->x = carve<float>(cur, static_cast<size_t>(max_rows) * H);
  if (l2_persist()) {
    // Set aside L2 for the fp32 residual stream (this process's context
    // only; never shrinks a larger set-aside made earlier in the process).
    int dev = 0, max_persist = 0, max_window = 0;
    SG_CUDA_CHECK(cudaGetDevice(&dev));
    SG_CUDA_CHECK(cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, dev));
    SG_CUDA_CHECK(cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, dev));
    const size_t want = std::min(static_cast<size_t>(max_rows) * H * sizeof(float), static_cast<size_t>(max_window));
    size_t cur_limit = 0;
    SG_CUDA_CHECK(cudaDeviceGetLimit(&cur_limit, cudaLimitPersistingL2CacheSize));
    const size_t setaside = std::min(want, static_cast<size_t>(max_persist));
    if (cur_limit < setaside) SG_CUDA_CHECK(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, setaside));
    SG_CUDA_CHECK(cudaDeviceGetLimit(&cur_limit, cudaLimitPersistingL2CacheSize));
    if (want > 0 && cur_limit > 0) {
      e->l2_window_bytes = want;
      e->l2_setaside = cur_limit;
    }
  }
  e->xn = carve<__nv_bfloat16>(cur, static_cast<size_t>(max_rows) * H);
  e->qkv = carve<__nv_bfloat16>(cur, static_cast<size_t>(max_rows) * qkv_n);
  e->q = carve<__nv_bfloat16>(cur, static_cast<size_t>(max_rows) * qw);
  e->attn = carve<__nv_bfloat16>(cur, static_cast<size_t>(max_rows) * qw);
  e->h = carve<__nv_bfloat16>(cur, static_cast<size_t>(max_rows) * I);
  e->vocab_tiles = (m.vocab + gemm::BN - 1) / gemm::BN;
  e->partials = carve<float4>(cur, static_cast<size_t>(max_rows) * e->vocab_tiles);
  e->lse_ws = carve<float>(cur, max_rows);
  e->posterior_ws = carve<int64_t>(cur, max_rows);
  e->ss_parts = (H + kNarrowBN - 1) / kNarrowBN;  // the most column tiles a residual GEMM writes
  e->ssq = carve<float>(cur, static_cast<size_t>(max_rows) * e->ss_parts);
  e->meta.anc = carve<uint32_t>(cur, static_cast<size_t>(max_rows) * layers::kAncWords);
  e->meta.position = carve<int32_t>(cur, max_rows);
  e->meta.tree = carve<int32_t>(cur, max_rows);
  e->meta.local = carve<int32_t>(cur, max_rows);
  e->meta.request_id = carve<int64_t>(cur, max_rows);
  e->meta.order = carve<int32_t>(cur, max_rows);
  e->meta.rope = carve<float2>(cur, static_cast<size_t>(max_rows) * (D / 2));
  e->meta.arena_row = carve<int64_t>(cur, max_rows);
  e->work.order = e->meta.order;
  e->work.item_capacity = attention_item_capacity(m, max_rows);
  e->work.items = carve<int32_t>(cur, e->work.item_capacity);
  e->work.num_items = carve<int32_t>(cur, 1);
  e->work.counters = carve<int32_t>(cur, m.num_layers);
  e->split.partial_tiles = gemm::split_partial_tiles(e->sms);
  e->split.partials = carve<float>(cur, e->split.partial_tiles * gemm::BM * gemm::BN);
  e->split.flags = carve<int>(cur, e->split.partial_tiles);
  if (static_cast<size_t>(cur - static_cast<uint8_t*>(e->workspace)) > e->workspace_bytes)
    return fail(SG_ERR_WORKSPACE, "sg_engine_create: workspace layout overflow");
  // Split flags start at zero; every split GEMM leaves them at zero.
  if (cudaMemset(e->split.flags, 0, e->split.partial_tiles * sizeof(int)) != cudaSuccess)
    return fail(SG_ERR_CUDA, "sg_engine_create: cudaMemset of the split flags failed");
  if ((st = make_tmap_2d_bf16(&e->xn_map, e->xn, H, max_rows, H * 2, gemm::BK, gemm::BM)) != SG_OK) return st;
  if ((st = make_tmap_2d_bf16(&e->attn_map, e->attn, qw, max_rows, qw * 2, gemm::BK, gemm::BM)) != SG_OK) return st;
  if ((st = make_tmap_2d_bf16(&e->h_map, e->h, I, max_rows, I * 2, gemm::BK, gemm::BM)) != SG_OK) return st;
  return SG_OK;
}

}  // namespace
}  // namespace sg

extern "C" int sg_engine_create(const sg_model_desc* model, const sg_arena_desc* arena, int32_t max_rows,
                                int32_t max_requests, void** engine_out) {
  using namespace sg;
  if (engine_out == nullptr) return fail(SG_ERR_INVALID_ARGUMENT, "sg_engine_create: null argument");
  *engine_out = nullptr;
  std::unique_ptr<Engine> e;
  const int st = create_engine(model, arena, max_rows, max_requests, e);
  if (st != SG_OK) return st;
  *engine_out = e.release();
  return SG_OK;
}

extern "C" int sg_engine_destroy(void* engine) {
  if (engine == nullptr) return SG_OK;
  delete static_cast<Engine*>(engine);
  return SG_OK;
}

extern "C" size_t sg_engine_workspace_bytes(void* engine) {
  return engine == nullptr ? 0 : static_cast<Engine*>(engine)->workspace_bytes;
}

namespace sg {
namespace {

// Per-call inputs of the decoder layer stack, shared by the verify pass and
// the drafter step.  Request r owns packed rows row_offsets[r] ..
// row_offsets[r + 1] - 1, after cache_len[r] rows of its arena slot; e->x
// holds the embedded rows and e->meta their per-row metadata.
struct StackArgs {
  int R = 0, Q = 0;
  const int64_t* row_offsets = nullptr;
  const int64_t* slots = nullptr;
  const int64_t* cache_len = nullptr;
  int max_rows_per_request = 0;
  int32_t* status = nullptr;
  const sg_wave_desc* wave = nullptr;  // trace events (verify pass)
  // drafter features (verify pass): layer l's residual stream into column
  // block feature_slot[l] of features_out
  const int* feature_slot = nullptr;
  int nfeat = 0;
  void* features_out = nullptr;
  // drafter context rows: their K/V are projected from draft->th into the
  // arena at draft->ctx_meta.arena_row in every layer, before its attention
  const DraftState* draft = nullptr;
  int ctx_rows = 0;
};

inline void trace_at(const StackArgs& a, int point, cudaStream_t stream) {
  if (a.wave != nullptr) trace(*a.wave, point, stream);
}

int run_stack(Engine* e, const StackArgs& a, cudaStream_t stream) {
  const sg_model_desc& m = e->model;
  const int H = m.hidden, D = m.head_dim, I = m.intermediate;
  const int nq = m.num_q_heads, nkv = m.num_kv_heads;
  const int qkv_n = (nq + 2 * nkv) * D;
  const int qw = nq * D;
  const int Q = a.Q;
  const int64_t plane_rows = e->arena.num_slots * e->arena.capacity;
  const int64_t plane_stride = plane_rows * D;  // elements between kv heads
  __nv_bfloat16* arena = static_cast<__nv_bfloat16*>(e->arena.storage);
  const bool nf = norm_fused();
  const int rbn = residual_width(Q, H, e->sms);
  const int P = (H + rbn - 1) / rbn;  // column tiles of this pass's residual GEMMs
  const float inv_h = 1.0f / static_cast<float>(H);
  int st;
  if (nf && (st = layers::launch_norm_fold(e->x, static_cast<const __nv_bfloat16*>(e->layer_ptrs[W_IN_NORM]), H, Q,
                                           e->xn, e->ssq, stream)) != SG_OK)
    return st;
  if ((st = layers::launch_attention_work(a.row_offsets, a.cache_len, a.R, nq / nkv, nkv, e->work, m.num_layers,
                                         stream)) != SG_OK)
    return st;
  trace_at(a, 1, stream);
  const gemm::Shape s_qkv = gemm::make_shape(Q, qkv_n, H);
  const gemm::Shape s_o = gemm::make_shape(Q, H, qw, rbn);
  const gemm::Shape s_gu = gemm::make_shape(Q, 2 * I, H);
  const gemm::Shape s_down = gemm::make_shape(Q, H, I, rbn);
  const gemm::Shape s_ctx = gemm::make_shape(a.ctx_rows, 2 * nkv * D, H);
  // Shapes with at most half a wave of tiles (few packed rows) and a long K
  // give each tile's k-blocks to two CTAs; everything else runs whole tiles,
  // which measured faster (a split tile's owner waits for its contributor,
  // adds the partial and only then runs the epilogue: about 15 µs that only
  // a long k-loop pays back, e.g. the 512-row down projection, K = 12288,
  // 85 -> 65 µs, but not the O projection, K = 4096, 34 -> 37 µs).
  auto small_wave = [&](const gemm::Shape& sh) -> const gemm::SplitWorkspace* {
    return 2 * sh.tiles <= e->sms && sh.k_blocks >= 96 ? &e->split : nullptr;
  };
  for (int l = 0; l < m.num_layers; ++l) {
    const void* const* lw = &e->layer_ptrs[static_cast<size_t>(l) * W_COUNT];
    const LayerMaps& lm = e->maps[l];
    __nv_bfloat16* k_plane0 = arena + static_cast<int64_t>(l) * 2 * nkv * plane_stride;
    __nv_bfloat16* v_plane0 = k_plane0 + static_cast<int64_t>(nkv) * plane_stride;

    if (a.draft != nullptr && a.ctx_rows > 0) {
      // drafter context rows: k|v projection of hidden_norm(fc(features))
      // with k_norm and RoPE, written at the rows' arena positions (no q)
      const DraftState& d = *a.draft;
      const auto* kn = static_cast<const __nv_bfloat16*>(lw[W_K_NORM]);
      if (D == 128) {
        gemm::EpiQkvPost<128>::Params pc{nullptr, 0, k_plane0, v_plane0, plane_stride, d.ctx_meta.arena_row,
                                         d.ctx_meta.rope, kn, kn, 0, nkv, m.rms_eps, a.status, gemm::RowNorm{}};
        st = gemm::launch<gemm::EpiQkvPost<128>>(d.th_map, d.kv_maps[l], s_ctx, pc, stream, small_wave(s_ctx));
      } else {
        gemm::EpiQkvPost<64>::Params pc{nullptr, 0, k_plane0, v_plane0, plane_stride, d.ctx_meta.arena_row,
                                        d.ctx_meta.rope, kn, kn, 0, nkv, m.rms_eps, a.status, gemm::RowNorm{}};
        st = gemm::launch<gemm::EpiQkvPost<64>>(d.th_map, d.kv_maps[l], s_ctx, pc, stream, small_wave(s_ctx));
      }
      if (st != SG_OK) return st;
    }
    if (!nf && (st = layers::launch_rmsnorm(e->x, static_cast<const __nv_bfloat16*>(lw[W_IN_NORM]), H, Q, m.rms_eps,
                                            e->xn, stream)) != SG_OK)
      return st;
    if (l == 0) trace_at(a, 2, stream);
    // input RMSNorm's row scale: sums from the fold kernel (layer 0, one part)
    // or from the previous down projection's tiles
    const gemm::RowNorm rn_in = nf ? gemm::RowNorm{e->ssq, l == 0 ? 1 : P, inv_h, m.rms_eps} : gemm::RowNorm{};
    if (qkv_fused()) {
      // q/k/v projection with q/k RMSNorm, RoPE and the KV-tail write in its epilogue
      if (D == 128) {
        gemm::EpiQkvPost<128>::Params pf{e->q, qw, k_plane0, v_plane0, plane_stride, e->meta.arena_row,
                                         e->meta.rope, static_cast<const __nv_bfloat16*>(lw[W_Q_NORM]),
                                         static_cast<const __nv_bfloat16*>(lw[W_K_NORM]), nq, nkv, m.rms_eps,
                                         a.status, rn_in};
        st = gemm::launch<gemm::EpiQkvPost<128>>(e->xn_map, lm.qkv, s_qkv, pf, stream, small_wave(s_qkv));
      } else {
        gemm::EpiQkvPost<64>::Params pf{e->q, qw, k_plane0, v_plane0, plane_stride, e->meta.arena_row,
                                        e->meta.rope, static_cast<const __nv_bfloat16*>(lw[W_Q_NORM]),
                                        static_cast<const __nv_bfloat16*>(lw[W_K_NORM]), nq, nkv, m.rms_eps,
                                        a.status, rn_in};
        st = gemm::launch<gemm::EpiQkvPost<64>>(e->xn_map, lm.qkv, s_qkv, pf, stream, small_wave(s_qkv));
      }
      if (st != SG_OK) return st;
      if (l == 0) {
        trace_at(a, 3, stream);
        trace_at(a, 4, stream);
      }
    } else {
      gemm::EpiStoreBf16::Params pq{e->qkv, qkv_n, a.status};
      if ((st = gemm::launch<gemm::EpiStoreBf16>(e->xn_map, lm.qkv, s_qkv, pq, stream, small_wave(s_qkv))) != SG_OK)
        return st;
      if (l == 0) trace_at(a, 3, stream);
      layers::QkvPost qp;
      qp.qkv = e->qkv;
      qp.q_norm = static_cast<const __nv_bfloat16*>(lw[W_Q_NORM]);
      qp.k_norm = static_cast<const __nv_bfloat16*>(lw[W_K_NORM]);
      qp.inv_freq = m.inv_freq;
      qp.position = e->meta.position;
      qp.tree = e->meta.tree;
      qp.local = e->meta.local;
      qp.slots = a.slots;
      qp.cache_len = a.cache_len;
      qp.q_out = e->q;
      qp.k_plane0 = k_plane0;
      qp.v_plane0 = v_plane0;
      qp.plane_stride = plane_stride;
      qp.capacity = e->arena.capacity;
      qp.plane_rows = plane_rows;
      qp.rope = e->meta.rope;
      qp.arena_row = e->meta.arena_row;
      qp.nq = nq;
      qp.nkv = nkv;
      qp.head_dim = D;
      qp.rows = Q;
      qp.eps = m.rms_eps;
      qp.status = a.status;
      if ((st = layers::launch_qkv_post(qp, stream)) != SG_OK) return st;
      if (l == 0) trace_at(a, 4, stream);
    }

    attn::Params ap;
    ap.q = e->q;
    ap.out = e->attn;
    ap.k0 = k_plane0;
    ap.v0 = v_plane0;
    ap.plane_stride = plane_stride;
    ap.capacity = e->arena.capacity;
    ap.plane_rows = plane_rows;
    ap.num_rows = Q;
    ap.row_offsets = a.row_offsets;
    ap.slots = a.slots;
    ap.cache_len = a.cache_len;
    ap.anc = e->meta.anc;
    ap.nq = nq;
    ap.nkv = nkv;
    ap.group = nq / nkv;
    ap.plane_k0 = l * 2 * nkv;
    ap.plane_v0 = l * 2 * nkv + nkv;
    ap.items = e->work.items;
    ap.num_items = e->work.num_items;
    ap.work_counter = e->work.counters + l;
    ap.status = a.status;
    ap.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
    if ((st = attn::launch(e->kv_map, ap, a.R, a.max_rows_per_request, D, stream)) != SG_OK) return st;
    if (l == 0) trace_at(a, 5, stream);

    gemm::EpiResidual::Params po{e->x, H, nullptr, 0, a.status};
    if (nf) {  // fold the post-attention RMSNorm into this epilogue and the gate/up GEMM
      po.xw = e->xn;
      po.ldw = H;
      po.norm_w = static_cast<const __nv_bfloat16*>(lw[W_POST_NORM]);
      po.ssq = e->ssq;
      po.ss_parts = P;
    }
    if ((st = rbn == kNarrowBN ? gemm::launch<gemm::EpiResidual, kNarrowBN>(e->attn_map, lm.o_narrow, s_o, po, stream,
                                                                            small_wave(s_o))
                               : gemm::launch<gemm::EpiResidual>(e->attn_map, lm.o, s_o, po, stream, small_wave(s_o))) !=
        SG_OK)
      return st;
    if (l == 0) trace_at(a, 6, stream);
    if (!nf && (st = layers::launch_rmsnorm(e->x, static_cast<const __nv_bfloat16*>(lw[W_POST_NORM]), H, Q,
                                            m.rms_eps, e->xn, stream)) != SG_OK)
      return st;
    if (l == 0) trace_at(a, 7, stream);
    gemm::EpiSwiGlu::Params pg{e->h, I, a.status,
                               nf ? gemm::RowNorm{e->ssq, P, inv_h, m.rms_eps} : gemm::RowNorm{}};
    if ((st = gemm::launch<gemm::EpiSwiGlu>(e->xn_map, lm.gate_up, s_gu, pg, stream, small_wave(s_gu))) != SG_OK)
      return st;
    if (l == 0) trace_at(a, 8, stream);
    // the residual stream after this layer is hidden_states[l + 1]; the last
    // layer's entry is the final-normed stream, copied after the final norm
    __nv_bfloat16* feat = nullptr;
    if (a.feature_slot != nullptr && a.feature_slot[l] >= 0 && l + 1 < m.num_layers)
      feat = static_cast<__nv_bfloat16*>(a.features_out) + static_cast<int64_t>(a.feature_slot[l]) * H;
    gemm::EpiResidual::Params pd{e->x, H, feat, static_cast<int64_t>(a.nfeat) * H, a.status};
    if (nf && l + 1 < m.num_layers) {  // fold the next layer's input RMSNorm
      pd.xw = e->xn;
      pd.ldw = H;
      pd.norm_w = static_cast<const __nv_bfloat16*>(e->layer_ptrs[static_cast<size_t>(l + 1) * W_COUNT + W_IN_NORM]);
      pd.ssq = e->ssq;
      pd.ss_parts = P;
    }
    if ((st = rbn == kNarrowBN ? gemm::launch<gemm::EpiResidual, kNarrowBN>(e->h_map, lm.down_narrow, s_down, pd,
                                                                            stream, small_wave(s_down))
                               : gemm::launch<gemm::EpiResidual>(e->h_map, lm.down, s_down, pd, stream,
                                                                 small_wave(s_down))) != SG_OK)
      return st;
    if (l == 0) trace_at(a, 9, stream);
  }
  return SG_OK;
}

}  // namespace
}  // namespace sg

extern "C" int sg_verify_pass(void* engine, const sg_wave_desc* wave, void* stream_ptr) {
  using namespace sg;
  if (engine == nullptr || wave == nullptr) return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: null argument");
  Engine* e = static_cast<Engine*>(engine);
  const sg_wave_desc& w = *wave;
  const sg_model_desc& m = e->model;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int R = w.num_requests, Q = w.num_rows;
  if (R < 1 || Q < R || Q > e->max_rows || R > e->max_requests || w.max_depth < 0 ||
      w.max_rows_per_request < 1 || w.max_rows_per_request > layers::kMaxTreeRows)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: wave sizes out of range");
  if (w.row_offsets == nullptr || w.parents == nullptr || w.tokens == nullptr || w.slots == nullptr ||
      w.cache_lengths == nullptr || w.position_base == nullptr || w.accept_out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: null wave array");
  if (w.commit && w.lengths_out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: commit needs lengths_out");
  if (!(w.temperature >= 0.f) || w.temperature == INFINITY)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: temperature must be finite and >= 0 (0 = greedy)");
  const bool greedy = w.temperature == 0.f;
  const float inv_temp = greedy ? 1.0f : 1.0f / w.temperature;
  struct WindowScope {  // the residual stream's L2 window for this pass's launches
    L2Window saved;
    WindowScope(const Engine* e, int rows) : saved(l2_window()) {
      if (e->l2_window_bytes == 0) return;
      const size_t bytes = std::min(e->l2_window_bytes, static_cast<size_t>(rows) * e->model.hidden * sizeof(float));
      const float ratio = std::min(1.0f, static_cast<float>(e->l2_setaside) / static_cast<float>(bytes));
      l2_window() = L2Window{e->x, bytes, ratio};
    }
    ~WindowScope() { l2_window() = saved; }
  } window_scope(e, Q);
  // feature slot of every layer (-1: not a drafter feature layer)
  std::vector<int> feature_slot(static_cast<size_t>(m.num_layers), -1);
  const int nfeat = w.num_feature_layers;
  if (nfeat < 0 || (nfeat > 0 && (w.feature_layers == nullptr || w.features_out == nullptr ||
                                  (reinterpret_cast<uintptr_t>(w.features_out) & 15u) != 0)))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: feature layers need a 16-byte aligned features_out");
  for (int f = 0; f < nfeat; ++f) {
    const int l = w.feature_layers[f];
    if (l < 0 || l >= m.num_layers) return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: feature layer out of range");
    feature_slot[l] = f;
  }
  if (w.features_kept != nullptr && (nfeat == 0 || w.features_kept_offsets == nullptr))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: features_kept needs feature layers and offsets");
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev != e->device) return fail(SG_ERR_INVALID_ARGUMENT, "sg_verify_pass: engine belongs to another device");

  const int H = m.hidden, D = m.head_dim;
  const int nkv = m.num_kv_heads;
  const int64_t plane_rows = e->arena.num_slots * e->arena.capacity;
  __nv_bfloat16* arena = static_cast<__nv_bfloat16*>(e->arena.storage);
  int st;

  trace(w, 0, stream);
  if ((st = layers::launch_tree_meta(w.row_offsets, w.parents, w.position_base, w.request_ids, R, Q, e->meta, w.status,
                                     stream)) != SG_OK)
    return st;
  if ((st = layers::launch_row_rope(e->meta, m.inv_freq, D, Q, w.slots, w.cache_lengths, e->arena.capacity,
                                    plane_rows, w.status, stream)) != SG_OK)
    return st;
  if ((st = layers::launch_embed(w.tokens, static_cast<const __nv_bfloat16*>(m.embed), m.vocab, H, Q, e->x, w.status,
                                 stream)) != SG_OK)
    return st;
  const bool nf = norm_fused();
  const float inv_h = 1.0f / static_cast<float>(H);
  StackArgs sa;
  sa.R = R;
  sa.Q = Q;
  sa.row_offsets = w.row_offsets;
  sa.slots = w.slots;
  sa.cache_len = w.cache_lengths;
  sa.max_rows_per_request = w.max_rows_per_request;
  sa.status = w.status;
  sa.wave = &w;
  sa.feature_slot = feature_slot.data();
  sa.nfeat = nfeat;
  sa.features_out = w.features_out;
  if ((st = run_stack(e, sa, stream)) != SG_OK) return st;
  trace(w, 10, stream);
  if (w.hidden_out != nullptr)
    SG_CUDA_CHECK(cudaMemcpyAsync(w.hidden_out, e->x, static_cast<size_t>(Q) * H * 4, cudaMemcpyDeviceToDevice,
                                  stream));
  // final RMSNorm: folded into the LM head (one fold kernel per pass, the
  // same computation as sg_lm_head_sample), or as a kernel
  if (nf) {
    if ((st = layers::launch_norm_fold(e->x, static_cast<const __nv_bfloat16*>(m.final_norm), H, Q, e->xn, e->ssq,
                                       stream)) != SG_OK)
      return st;
  } else if ((st = layers::launch_rmsnorm(e->x, static_cast<const __nv_bfloat16*>(m.final_norm), H, Q, m.rms_eps,
                                          e->xn, stream)) != SG_OK) {
    return st;
  }
  if (nf && feature_slot[m.num_layers - 1] >= 0) {  // the final-normed stream, for the drafter
    if ((st = layers::launch_rmsnorm(e->x, static_cast<const __nv_bfloat16*>(m.final_norm), H, Q, m.rms_eps,
                                     static_cast<__nv_bfloat16*>(w.features_out) +
                                         static_cast<int64_t>(feature_slot[m.num_layers - 1]) * H,
                                     stream, static_cast<int64_t>(nfeat) * H)) != SG_OK)
      return st;
  } else if (feature_slot[m.num_layers - 1] >= 0) {
    const size_t pitch = static_cast<size_t>(nfeat) * H * 2;
    SG_CUDA_CHECK(cudaMemcpy2DAsync(static_cast<uint8_t*>(w.features_out) +
                                        static_cast<size_t>(feature_slot[m.num_layers - 1]) * H * 2,
                                    pitch, e->xn, static_cast<size_t>(H) * 2, static_cast<size_t>(H) * 2, Q,
                                    cudaMemcpyDeviceToDevice, stream));
  }
  trace(w, 11, stream);
  gemm::EpiLmHead::Params pl;
  pl.partials = e->partials;
  pl.n_tiles = e->vocab_tiles;
  pl.row_local = e->meta.local;
  pl.row_request = e->meta.request_id;
  pl.seed = w.seed;
  pl.inv_temp = inv_temp;
  pl.greedy = greedy ? 1 : 0;
  pl.status = w.status;
  pl.rn = nf ? gemm::RowNorm{e->ssq, 1, inv_h, m.rms_eps} : gemm::RowNorm{};
  if ((st = gemm::launch<gemm::EpiLmHead>(e->xn_map, e->lm_map, gemm::make_shape(Q, m.vocab, H), pl, stream)) !=
      SG_OK)
    return st;
  trace(w, 12, stream);
  float* lse = w.lse != nullptr ? w.lse : e->lse_ws;
  int64_t* posterior = w.posterior != nullptr ? w.posterior : e->posterior_ws;
  if ((st = layers::launch_lm_combine(e->partials, e->vocab_tiles, Q, lse, posterior, nullptr, stream)) != SG_OK)
    return st;
  if (w.child_logprob != nullptr &&
      (st = layers::launch_child_logprob(e->xn, static_cast<const __nv_bfloat16*>(m.lm_head), H, m.vocab, w.tokens, w.parents,
                                         w.row_offsets, e->meta.tree, e->meta.local, lse, inv_temp, Q,
                                         w.child_logprob, stream, nf ? e->ssq : nullptr, 1, m.rms_eps)) != SG_OK)
    return st;
  trace(w, 13, stream);
  if ((st = sg_tree_follow(posterior, w.row_offsets, w.parents, w.tokens, R, w.max_rows_per_request, w.max_depth,
                           w.accept_out, w.status, stream)) != SG_OK)
    return st;
  if (w.features_kept != nullptr &&
      (st = layers::launch_gather_kept_rows(w.features_out, static_cast<int64_t>(nfeat) * H * 2, w.row_offsets,
                                            w.accept_out, R, w.max_depth, w.features_kept, w.features_kept_offsets,
                                            w.status, stream)) != SG_OK)
    return st;
  trace(w, 14, stream);
  if (w.commit) {
    if ((st = sg_kv_commit_accepted(arena, plane_rows, static_cast<int64_t>(m.num_layers) * 2 * nkv,
                                    static_cast<int64_t>(D) * 2, e->arena.capacity, w.slots, w.cache_lengths,
                                    w.lengths_out, w.accept_out, R, w.max_depth, w.status, stream)) != SG_OK)
      return st;
  }
  trace(w, 15, stream);
  return SG_OK;
}

// ---------------------------------------------------------------------------
// Drafter step (DFlash block drafter, dflash.py:147-200, as the decoder calls
// it with a persistent per-request draft cache,
// continuous_tree_block_decode.py:889-962).
// ---------------------------------------------------------------------------
extern "C" int sg_draft_engine_create(const sg_model_desc* model, const sg_draft_desc* draft,
                                      const sg_arena_desc* arena, int32_t max_requests, void** engine_out) {
  using namespace sg;
  if (draft == nullptr || engine_out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_engine_create: null argument");
  *engine_out = nullptr;
  if (draft->fc == nullptr || draft->hidden_norm == nullptr || draft->num_feature_layers < 1 ||
      draft->block_size < 1 || draft->block_size > layers::kMaxTreeRows || draft->max_update_rows < 1 ||
      max_requests < 1)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_engine_create: bad drafter description");
  const int64_t block_rows = static_cast<int64_t>(max_requests) * draft->block_size;
  const int max_rows = static_cast<int>(std::max<int64_t>(block_rows, draft->max_update_rows));
  std::unique_ptr<Engine> e;
  int st = create_engine(model, arena, max_rows, max_requests, e);
  if (st != SG_OK) return st;
  const sg_model_desc& m = e->model;
  const int H = m.hidden, D = m.head_dim, F = draft->num_feature_layers;
  const int qw = m.num_q_heads * D, kvw = 2 * m.num_kv_heads * D;
  if (kvw % 32 != 0) return fail(SG_ERR_UNSUPPORTED, "sg_draft_engine_create: k|v width % 32 != 0");
  std::unique_ptr<DraftState> d(new DraftState());
  d->desc = *draft;
  if ((st = make_tmap_2d_bf16(&d->fc_map, draft->fc, static_cast<uint64_t>(F) * H, H,
                              static_cast<uint64_t>(F) * H * 2, gemm::BK, gemm::BN)) != SG_OK)
    return st;
  d->kv_maps.resize(m.num_layers);
  for (int l = 0; l < m.num_layers; ++l) {
    const uint8_t* qkv = static_cast<const uint8_t*>(e->layer_ptrs[static_cast<size_t>(l) * W_COUNT + W_QKV]);
    if ((st = make_tmap_2d_bf16(&d->kv_maps[l], qkv + static_cast<size_t>(qw) * H * 2, H, kvw,
                                static_cast<uint64_t>(H) * 2, gemm::BK, gemm::BN)) != SG_OK)
      return st;
  }
  const size_t U = draft->max_update_rows;
  size_t bytes = 0;
  bytes += U * H * 4 + 256;                                   // th32
  bytes += U * H * 2 + 256;                                   // th
  bytes += U * 4 * 3 + 3 * 256;                               // ctx position, tree, local
  bytes += U * (D / 2) * 8 + 256;                             // ctx rope
  bytes += U * 8 + 256;                                       // ctx arena rows
  bytes += (static_cast<size_t>(max_requests) + 1) * 8 + 256; // block offsets
  bytes += static_cast<size_t>(max_requests) * 8 + 256;       // prefix lengths
  bytes += static_cast<size_t>(block_rows) * 8 + 256;         // block tokens
  SG_CUDA_CHECK(cudaMalloc(&d->buffer, bytes));
  uint8_t* cur = static_cast<uint8_t*>(d->buffer);
  d->th32 = carve<float>(cur, U * H);
  d->th = carve<__nv_bfloat16>(cur, U * H);
  d->ctx_meta = layers::RowMeta{};
  d->ctx_meta.position = carve<int32_t>(cur, U);
  d->ctx_meta.tree = carve<int32_t>(cur, U);
  d->ctx_meta.local = carve<int32_t>(cur, U);
  d->ctx_meta.rope = carve<float2>(cur, U * (D / 2));
  d->ctx_meta.arena_row = carve<int64_t>(cur, U);
  d->block_offsets = carve<int64_t>(cur, static_cast<size_t>(max_requests) + 1);
  d->prefix = carve<int64_t>(cur, max_requests);
  d->block_tokens = carve<int64_t>(cur, block_rows);
  if (static_cast<size_t>(cur - static_cast<uint8_t*>(d->buffer)) > bytes)
    return fail(SG_ERR_WORKSPACE, "sg_draft_engine_create: buffer layout overflow");
  if ((st = make_tmap_2d_bf16(&d->th_map, d->th, H, U, static_cast<uint64_t>(H) * 2, gemm::BK, gemm::BM)) != SG_OK)
    return st;
  e->draft = std::move(d);
  *engine_out = e.release();
  return SG_OK;
}

extern "C" int sg_draft_pass(void* engine, const sg_draft_wave* wave, void* stream_ptr) {
  using namespace sg;
  if (engine == nullptr || wave == nullptr) return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_pass: null argument");
  Engine* e = static_cast<Engine*>(engine);
  if (!e->draft) return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_pass: not a drafter engine (sg_draft_engine_create)");
  DraftState& d = *e->draft;
  const sg_draft_wave& w = *wave;
  const sg_model_desc& m = e->model;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int R = w.num_requests, U = w.num_update_rows, B = d.desc.block_size;
  if (R < 1 || R > e->max_requests || static_cast<int64_t>(R) * B > e->max_rows || U < 0 ||
      U > d.desc.max_update_rows)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_pass: sizes out of range");
  const bool ctx_only = w.context_only != 0;
  if (w.slots == nullptr || w.cache_lengths == nullptr || w.update_offsets == nullptr ||
      (!ctx_only && (w.anchor_tokens == nullptr || w.logits_out == nullptr)) || (U > 0 && w.features == nullptr))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_pass: null wave array");
  if ((U > 0 && (reinterpret_cast<uintptr_t>(w.features) & 15u) != 0) ||
      (!ctx_only && (reinterpret_cast<uintptr_t>(w.logits_out) & 15u) != 0))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_pass: features and logits_out must be 16-byte aligned");
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev != e->device) return fail(SG_ERR_INVALID_ARGUMENT, "sg_draft_pass: engine belongs to another device");
  const int H = m.hidden, D = m.head_dim, F = d.desc.num_feature_layers;
  const int Q = R * B;
  const int64_t plane_rows = e->arena.num_slots * e->arena.capacity;
  int st;
  // context rows of a malformed request keep tree -1 (no arena row)
  if (U > 0) SG_CUDA_CHECK(cudaMemsetAsync(d.ctx_meta.tree, 0xFF, static_cast<size_t>(U) * 4, stream));
  if ((st = layers::launch_draft_meta(w.update_offsets, w.cache_lengths, ctx_only ? w.slots : w.anchor_tokens,
                                      d.desc.mask_token_id, R, B, U, e->meta, d.ctx_meta, d.block_offsets, d.prefix,
                                      d.block_tokens, w.lengths_out, w.status, stream)) != SG_OK)
    return st;
  // block rows after the committed context, context rows at cache_len ..
  if (!ctx_only && (st = layers::launch_row_rope(e->meta, m.inv_freq, D, Q, w.slots, d.prefix, e->arena.capacity,
                                                 plane_rows, w.status, stream)) != SG_OK)
    return st;
  if ((st = layers::launch_row_rope(d.ctx_meta, m.inv_freq, D, U, w.slots, w.cache_lengths, e->arena.capacity,
                                    plane_rows, w.status, stream)) != SG_OK)
    return st;
  if (!ctx_only && (st = layers::launch_embed(d.block_tokens, static_cast<const __nv_bfloat16*>(m.embed), m.vocab, H,
                                              Q, e->x, w.status, stream)) != SG_OK)
    return st;
  if (U > 0) {
    // target_hidden = hidden_norm(fc(features))
    CUtensorMap feat_map;
    if ((st = make_tmap_2d_bf16(&feat_map, w.features, static_cast<uint64_t>(F) * H, U,
                                static_cast<uint64_t>(F) * H * 2, gemm::BK, gemm::BM)) != SG_OK)
      return st;
    const gemm::Shape s_fc = gemm::make_shape(U, H, F * H);
    gemm::EpiStoreF32::Params pf{d.th32, H, w.status};
    if ((st = gemm::launch<gemm::EpiStoreF32>(feat_map, d.fc_map, s_fc, pf, stream,
                                              2 * s_fc.tiles <= e->sms ? &e->split : nullptr)) != SG_OK)
      return st;
    if ((st = layers::launch_rmsnorm(d.th32, static_cast<const __nv_bfloat16*>(d.desc.hidden_norm), H, U, m.rms_eps,
                                     d.th, stream)) != SG_OK)
      return st;
  }
  if (ctx_only) {
    // the context rows' k|v in every layer (the block is not run)
    if (U == 0) return SG_OK;
    const int nkv = m.num_kv_heads;
    const int64_t plane_stride = plane_rows * D;
    __nv_bfloat16* arena = static_cast<__nv_bfloat16*>(e->arena.storage);
    const gemm::Shape s_ctx = gemm::make_shape(U, 2 * nkv * D, H);
    const gemm::SplitWorkspace* split = 2 * s_ctx.tiles <= e->sms ? &e->split : nullptr;
    for (int l = 0; l < m.num_layers; ++l) {
      __nv_bfloat16* k_plane0 = arena + static_cast<int64_t>(l) * 2 * nkv * plane_stride;
      __nv_bfloat16* v_plane0 = k_plane0 + static_cast<int64_t>(nkv) * plane_stride;
      const auto* kn = static_cast<const __nv_bfloat16*>(e->layer_ptrs[static_cast<size_t>(l) * W_COUNT + W_K_NORM]);
      if (D == 128) {
        gemm::EpiQkvPost<128>::Params pc{nullptr, 0, k_plane0, v_plane0, plane_stride, d.ctx_meta.arena_row,
                                         d.ctx_meta.rope, kn, kn, 0, nkv, m.rms_eps, w.status, gemm::RowNorm{}};
        st = gemm::launch<gemm::EpiQkvPost<128>>(d.th_map, d.kv_maps[l], s_ctx, pc, stream, split);
      } else {
        gemm::EpiQkvPost<64>::Params pc{nullptr, 0, k_plane0, v_plane0, plane_stride, d.ctx_meta.arena_row,
                                        d.ctx_meta.rope, kn, kn, 0, nkv, m.rms_eps, w.status, gemm::RowNorm{}};
        st = gemm::launch<gemm::EpiQkvPost<64>>(d.th_map, d.kv_maps[l], s_ctx, pc, stream, split);
      }
      if (st != SG_OK) return st;
    }
    return SG_OK;
  }
  StackArgs sa;
  sa.R = R;
  sa.Q = Q;
  sa.row_offsets = d.block_offsets;
  sa.slots = w.slots;
  sa.cache_len = d.prefix;
  sa.max_rows_per_request = B;
  sa.status = w.status;
  sa.draft = &d;
  sa.ctx_rows = U;
  if ((st = run_stack(e, sa, stream)) != SG_OK) return st;
  // drafter's final norm, target's LM head: bf16 logits of every block row
  if ((st = layers::launch_rmsnorm(e->x, static_cast<const __nv_bfloat16*>(m.final_norm), H, Q, m.rms_eps, e->xn,
                                   stream)) != SG_OK)
    return st;
  gemm::EpiStoreBf16::Params pl{static_cast<__nv_bfloat16*>(w.logits_out), m.vocab, w.status};
  return gemm::launch<gemm::EpiStoreBf16>(e->xn_map, e->lm_map, gemm::make_shape(Q, m.vocab, H), pl, stream);
}
