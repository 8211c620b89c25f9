// Request-isolated packed tree attention on tcgen05 tensor cores (sm_100a).
//
// Reference semantics: the packed additive mask of
// continuous_tree_block_decode.py:500-546 — tree row j of request i sees the
// request's own KV prefix [0, L_i) and its own ancestors-or-self in the tree
// (Tree.visibility, tree.py:19-26), nothing of other requests — applied by HF
// SDPA inside Qwen3Model (engine.py:499-517) with GQA.
//
// No mask tensor and no packed KV copy exist.  One CTA owns (request, kv
// head, block of 128 query rows); its rows are the request's tree rows x the
// kv head's query-head group (row r -> token r / G, head h*G + r % G), so
// every K/V byte streamed from the request's arena slot serves all G heads.
//
//   warp 0      TMA: K and V tiles of 64 keys (64-dim boxes, 128B swizzle)
//               from the arena into a 4-stage shared-memory ring
//   warp 1      MMA: S_j = Q K_j^T into one of two TMEM buffers, then
//               O += P_j V_j into a TMEM accumulator (V read MN-major)
//   warps 2..9  softmax, two threads per query row (TMEM lane), each owning
//               half of the tile's key columns: read S_j,
//               mask tree keys with a 256-bit ancestor bitset (prefix keys
//               need none), online max in the log2 domain with lazy O
//               rescaling (only when the row max grows by more than 2^8),
//               write P_j (bf16) to shared memory; finally O / l -> global.
// The QK^T of tile j+1 is issued before waiting for P_j, so it overlaps the
// softmax of tile j.
#include <cuda_bf16.h>
#include <math.h>
#include <stdlib.h>

#include "attention.cuh"
#include "layers.cuh"
#include "sm100.cuh"

namespace sg {
namespace attn {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr uint32_t ATOM = 128 * 128;       // 128 rows x 64 bf16 swizzle block (16 KB)
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Tile geometry: BN keys per K/V tile, STAGES-deep K/V ring.
template <int D, int BN, int STAGES, int SPLIT>
struct Layout {
  static constexpr int THREADS = 64 + 128 * SPLIT;       // TMA warp, MMA warp, 4*SPLIT softmax warps
  static constexpr int HALVES = D / 64;                  // 64-element swizzle blocks along D
  static constexpr uint32_t KV_HALF = BN * 128;          // BN rows x 64 elements
  static constexpr uint32_t Q_BYTES = HALVES * ATOM;
  static constexpr uint32_t KV_BYTES = HALVES * KV_HALF; // one K or V tile
  static constexpr uint32_t P_BYTES = (BN / 64) * ATOM;  // 128 rows x BN keys (x2 buffers)
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr uint32_t OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr uint32_t OFF_RED = OFF_P + 2 * P_BYTES;   // [3 * SPLIT][128] floats
  static constexpr uint32_t OFF_BAR = OFF_RED + 3 * SPLIT * 128 * 4;
  static constexpr size_t SMEM = OFF_BAR + 512;
  static constexpr uint32_t O_COL = 2 * BN;              // S double buffer, then O
  static constexpr uint32_t TMEM_COLS = (O_COL + D) <= 256 ? 256 : 512;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int D, int BN, int STAGES, int SPLIT>
__global__ void __launch_bounds__(Layout<D, BN, STAGES, SPLIT>::THREADS, 1)
tree_attention_tc_kernel(const __grid_constant__ CUtensorMap kv_map, const Params p) {
  using L = Layout<D, BN, STAGES, SPLIT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0u) {  // 128B-swizzle atoms need 1 KB alignment
    if (threadIdx.x == 0 && p.status != nullptr) atomicMax(p.status, static_cast<int32_t>(SG_ERR_UNSUPPORTED));
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;                 // [STAGES]
  uint64_t* kv_empty = bars + STAGES;       // [STAGES]
  uint64_t* s_full = bars + 2 * STAGES;     // [2] S_j ready in TMEM buffer j % 2
  uint64_t* q_full = s_full + 2;
  uint64_t* p_full = q_full + 1;            // P_j written (and O rescaled if needed)
  uint64_t* o_done = p_full + 1;            // [2] PV_j (reading P buffer j % 2) complete
  uint64_t* xchg = o_done + 2;              // [4 quarters][3]: row max of tiles j%2, final sums
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xchg + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  pdl_trigger();
  pdl_wait();  // q, the K/V tail and the launch order come from earlier kernels
  const int mtile = blockIdx.x;
  const int kvh = blockIdx.y;
  const int req = p.order != nullptr ? p.order[blockIdx.z] : static_cast<int>(blockIdx.z);
  const int64_t q0 = p.row_offsets[req];
  const int64_t q1 = p.row_offsets[req + 1];
  if (q0 < 0 || q1 > p.num_rows || q1 - q0 < 1 || q1 - q0 > layers::kMaxTreeRows) return;
  const int n = static_cast<int>(q1 - q0);
  const int G = p.group;
  const int rows_total = n * G;
  const int m_base = mtile * BM;
  if (m_base >= rows_total) return;
  const int64_t Lp = p.cache_len[req];
  const int64_t kv_total = Lp + n;
  const int64_t slot = p.slots[req];
  // Never read outside the request's own slot (the QKV kernel reports the
  // capacity error for such a request).
  if (slot < 0 || (slot + 1) * p.capacity > p.plane_rows || Lp < 0 || kv_total > p.capacity) return;
  const int tiles = static_cast<int>((kv_total + BN - 1) / BN);
  const int row0 = static_cast<int>(slot * p.capacity);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&s_full[i], 1);
    mbar_init(q_full, 128);
    mbar_init(p_full, 128 * SPLIT);
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    for (int i = 0; i < 12; ++i) mbar_init(&xchg[i], 32 * SPLIT);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&kv_map);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t O_COL = L::O_COL;

  auto give_up = [&]() {
    *abort_flag = 1;
    if (p.status != nullptr) atomicMax(p.status, static_cast<int32_t>(SG_ERR_CUDA));
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int plane_k = p.plane_k0 + kvh, plane_v = p.plane_v0 + kvh;
      for (int j = 0; j < tiles && !*abort_flag; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1u)) {
          give_up();
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * L::KV_BYTES);
        const int row = row0 + j * BN;
#pragma unroll
        for (int h = 0; h < L::HALVES; ++h)
#pragma unroll
          for (int rb = 0; rb < BN / kKeyTile; ++rb) {  // the map's box is kKeyTile rows
            const uint32_t off = h * L::KV_HALF + rb * kKeyTile * 128;
            tma_load_3d(smem + L::OFF_K + s * L::KV_BYTES + off, &kv_map, h * 64, row + rb * kKeyTile, plane_k,
                        &kv_full[s]);
            tma_load_3d(smem + L::OFF_V + s * L::KV_BYTES + off, &kv_map, h * 64, row + rb * kKeyTile, plane_v,
                        &kv_full[s]);
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_bf16_f32(BM, BN);
      const uint32_t idesc_pv = idesc_bf16_f32(BM, D) | (1u << 16);  // B (V) is MN-major
      const uint32_t q_addr = smem_u32(smem + L::OFF_Q);
      const uint32_t p_addr = smem_u32(smem + L::OFF_P);
      auto issue_qk = [&](int j) -> bool {
        const int s = j % STAGES;
        if (!mbar_wait(&kv_full[s], (j / STAGES) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::OFF_K + s * L::KV_BYTES);
        const int sb = j & 1;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t qoff = (ks >> 2) * ATOM + (ks & 3) * 32;
          const uint32_t koff = (ks >> 2) * L::KV_HALF + (ks & 3) * 32;
          mma_bf16(tmem + sb * BN, desc_k_sw128(q_addr + qoff), desc_k_sw128(k_addr + koff), idesc_qk,
                   ks > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[sb]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0);
      if (ok) {
        tc_fence_after();
        ok = issue_qk(0);
      }
      for (int j = 0; ok && j < tiles; ++j) {
        if (j + 1 < tiles && !issue_qk(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(p_full, j & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int s = j % STAGES;
        const uint32_t v_addr = smem_u32(smem + L::OFF_V + s * L::KV_BYTES);
        const uint32_t pb_addr = p_addr + (j & 1) * L::P_BYTES;
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks) {
          const uint64_t adesc = desc_k_sw128(pb_addr + (ks >> 2) * ATOM + (ks & 3) * 32);
          const uint64_t bdesc = desc_mn_sw128(v_addr + ks * 16 * 128, L::KV_HALF, 1024);
          mma_bf16(tmem + O_COL, adesc, bdesc, idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&kv_empty[s]);
        mma_commit(&o_done[j & 1]);
      }
      if (!ok) give_up();
    }
  } else {
    // --------------------------------------------------------------- softmax
    // SPLIT warps per TMEM lane quarter; warp w owns rows 32*(w % 4) + lane
    // (the TMEM lanes it may access) and columns [half*CW, half*CW + CW).
    constexpr int CW = BN / SPLIT;  // S (key) columns per thread
    constexpr int DW = D / SPLIT;   // O columns per thread
    const int sw = warp - 2;
    const int quarter = warp & 3;
    const int half = sw >> 2;
    const int r = quarter * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int m_row = m_base + r;
    const bool valid = m_row < rows_total;
    const int tok = valid ? m_row / G : 0;
    const int head = kvh * G + (valid ? m_row % G : 0);
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);  // [2 tiles][SPLIT][128] maxima, then sums
    if (half == 0) {  // Q row -> shared memory (K-major, 128B swizzle)
      const uint4* src = reinterpret_cast<const uint4*>(p.q + ((q0 + tok) * p.nq + head) * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 v = valid ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(smem + L::OFF_Q + (c >> 3) * ATOM + swz128(r, c & 7)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(q_full);
    }
    uint32_t anc[layers::kAncWords];
    const uint32_t* ap = p.anc + (q0 + tok) * layers::kAncWords;
#pragma unroll
    for (int w = 0; w < layers::kAncWords; ++w) anc[w] = ap[w];
    const float c2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < tiles; ++j) {
      if (*abort_flag) {
        ok = false;
        break;
      }
      const int s = j % STAGES;
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[CW];  // raw scores, masked keys = -inf
      {
        uint32_t raw[CW];
#pragma unroll
        for (int c = 0; c < CW / 32; ++c)
          tmem_ld32_nowait(tmem + lane_base + sb * BN + half * CW + c * 32, raw + c * 32);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < CW; ++e) sv[e] = __uint_as_float(raw[e]);
      }
      const int64_t key0 = static_cast<int64_t>(j) * BN + half * CW;
      if (key0 + CW > Lp) {  // these columns reach the tree keys or the end
#pragma unroll
        for (int e = 0; e < CW; ++e) {
          const int64_t key = key0 + e;
          bool vis = true;
          if (key >= Lp) {
            const int k = static_cast<int>(key - Lp);
            vis = key < kv_total && ((anc[k >> 5] >> (k & 31)) & 1u);
          }
          if (!vis) sv[e] = -INFINITY;
        }
      }
      float mt;
      {  // pairwise max
        float t[CW / 2];
#pragma unroll
        for (int e = 0; e < CW / 2; ++e) t[e] = fmaxf(sv[2 * e], sv[2 * e + 1]);
#pragma unroll
        for (int w = CW / 4; w >= 1; w >>= 1)
#pragma unroll
          for (int e = 0; e < w; ++e) t[e] = fmaxf(t[e], t[e + w]);
        mt = t[0] * c2;
      }
      if constexpr (SPLIT > 1) {  // combine the row max over the column halves
        red[((j & 1) * SPLIT + half) * 128 + r] = mt;
        mbar_arrive(&xchg[quarter * 3 + (j & 1)]);
        if (!mbar_wait(&xchg[quarter * 3 + (j & 1)], (j >> 1) & 1)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int h = 0; h < SPLIT; ++h) mt = fmaxf(mt, red[((j & 1) * SPLIT + h) * 128 + r]);
      }
      // P buffer j % 2 was last read by PV_{j-2}
      if (j >= 2 && !mbar_wait(&o_done[j & 1], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      const bool grow = mt > m_run + kRescaleThreshold;
      if (j == 0) {
        m_run = mt;
      } else if (__any_sync(0xffffffffu, grow)) {
        // Rescaling O needs PV_{j-1} complete (rare: the max grew by > 2^8).
        if (!mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float m_new = grow ? mt : m_run;
        const float alpha = fast_exp2(m_run - m_new);
#pragma unroll
        for (int c = 0; c < DW / 32; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_base + O_COL + half * DW + c * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= alpha;
          tmem_st32(tmem + lane_base + O_COL + half * DW + c * 32, o);
        }
        tmem_wait_st();
        l_run *= alpha;
        m_run = m_new;
      }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint8_t* prow = smem + L::OFF_P + (j & 1) * L::P_BYTES;
      const float neg_m = -m_run;
#pragma unroll
      for (int c = 0; c < CW / 8; ++c) {
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          e8[e] = fast_exp2(fmaf(sv[c * 8 + e], c2, neg_m));
          acc[e] += e8[e];
        }
        uint4 w;
        w.x = pack_bf16x2(e8[0], e8[1]);
        w.y = pack_bf16x2(e8[2], e8[3]);
        w.z = pack_bf16x2(e8[4], e8[5]);
        w.w = pack_bf16x2(e8[6], e8[7]);
        const int chunk = half * (CW / 8) + c;  // 16-byte chunk index in the P row
        *reinterpret_cast<uint4*>(prow + (chunk >> 3) * ATOM + swz128(r, chunk & 7)) = w;
      }
      l_run += ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      if (half == 0 && r < BN && static_cast<int64_t>(j) * BN + r >= kv_total) {
        // Keys past the request's tail come from stale arena rows (possibly
        // NaN bit patterns); P is 0 there, but 0 * NaN is NaN in the MMA, so
        // zero this row of the V tile before P_j is released.
        uint8_t* vrow = smem + L::OFF_V + s * L::KV_BYTES + r * 128;
#pragma unroll
        for (int h = 0; h < L::HALVES; ++h)
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(vrow + h * L::KV_HALF + c * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && !mbar_wait(&o_done[(tiles - 1) & 1], ((tiles - 1) >> 1) & 1)) ok = false;
    if (!ok) {
      give_up();
    } else {
      if constexpr (SPLIT > 1) {  // total row sum over the column halves
        red[(2 * SPLIT + half) * 128 + r] = l_run;
        mbar_arrive(&xchg[quarter * 3 + 2]);
        if (mbar_wait(&xchg[quarter * 3 + 2], 0)) {
          l_run = 0.f;
#pragma unroll
          for (int h = 0; h < SPLIT; ++h) l_run += red[(2 * SPLIT + h) * 128 + r];
        } else {
          give_up();
        }
      }
      tc_fence_after();
      const float inv = 1.f / l_run;
      __nv_bfloat16* dst = p.out + ((q0 + tok) * p.nq + head) * D + half * DW;
#pragma unroll
      for (int c = 0; c < DW / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + O_COL + half * DW + c * 32, o);
        if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(o[q * 8 + 0] * inv, o[q * 8 + 1] * inv);
            w.y = pack_bf16x2(o[q * 8 + 2] * inv, o[q * 8 + 3] * inv);
            w.z = pack_bf16x2(o[q * 8 + 4] * inv, o[q * 8 + 5] * inv);
            w.w = pack_bf16x2(o[q * 8 + 6] * inv, o[q * 8 + 7] * inv);
            d4[q] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <int D, int BN, int STAGES, int SPLIT>
int launch_cfg(const CUtensorMap& map, const Params& p, dim3 grid, cudaStream_t stream) {
  using L = Layout<D, BN, STAGES, SPLIT>;
  auto kernel = tree_attention_tc_kernel<D, BN, STAGES, SPLIT>;
  static int configured = 0;
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (!(configured & (1 << dev))) {
    SG_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L::SMEM)));
    configured |= 1 << dev;
  }
  return launch_pdl("tree_attention_tc_kernel", kernel, grid, dim3(L::THREADS), L::SMEM, stream, map, p);
}

}  // namespace

int launch(const CUtensorMap& kv_map, const Params& p, int num_requests, int max_rows_per_request, int head_dim,
           cudaStream_t stream) {
  if (num_requests <= 0) return SG_OK;
  if (max_rows_per_request > layers::kMaxTreeRows)
    return fail(SG_ERR_UNSUPPORTED, "tree attention: more than 256 rows in one request");
  const int mtiles = (max_rows_per_request * p.group + BM - 1) / BM;
  dim3 grid(static_cast<unsigned>(mtiles), static_cast<unsigned>(p.nkv), static_cast<unsigned>(num_requests));
  // 64-key tiles, a 4-deep K/V ring, double-buffered P and 8 softmax warps
  // (two per TMEM lane quarter, each owning half of the key columns) in one
  // CTA per SM (~195 KB of shared memory at head_dim 128).  SG_ATTN_SPLIT=1
  // selects one softmax warp per quarter (same results; a tuning alternative).
  static const int split = [] {
    const char* v = getenv("SG_ATTN_SPLIT");
    return v != nullptr ? atoi(v) : 2;
  }();
  if (head_dim == 128) {
    if (split == 1) return launch_cfg<128, kKeyTile, 4, 1>(kv_map, p, grid, stream);
    return launch_cfg<128, kKeyTile, 4, 2>(kv_map, p, grid, stream);
  }
  if (head_dim == 64) return launch_cfg<64, kKeyTile, 4, 2>(kv_map, p, grid, stream);
  return fail(SG_ERR_UNSUPPORTED, "tree attention: head_dim must be 64 or 128");
}

}  // namespace attn
}  // namespace sg
