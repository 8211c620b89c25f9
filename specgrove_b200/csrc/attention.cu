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
//   warp 0      TMA: K and V tiles of 128 keys (64-dim boxes, 128B swizzle)
//               from the arena into a 2-stage shared-memory ring
//   warp 1      MMA: S_j = Q K_j^T into one of two TMEM buffers, then
//               O += P_j V_j into a TMEM accumulator (V read MN-major)
//   warps 2..5  softmax, one thread per query row (= TMEM lane): read S_j,
//               mask tree keys with a 256-bit ancestor bitset (prefix keys
//               need none), online max in the log2 domain with lazy O
//               rescaling (only when the row max grows by more than 2^8),
//               write P_j (bf16) to shared memory; finally O / l -> global.
// The QK^T of tile j+1 is issued before waiting for P_j, so it overlaps the
// softmax of tile j.
#include <cuda_bf16.h>
#include <math.h>

#include "attention.cuh"
#include "layers.cuh"
#include "sm100.cuh"

namespace sg {
namespace attn {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ATOM = 128 * 128;       // 128 rows x 64 bf16 swizzle block (16 KB)
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct Layout {
  static constexpr int HALVES = D / 64;                // 64-element swizzle blocks along D
  static constexpr uint32_t Q_BYTES = HALVES * ATOM;
  static constexpr uint32_t KV_BYTES = HALVES * ATOM;  // one K or V tile of 128 keys
  static constexpr uint32_t P_BYTES = 2 * ATOM;        // 128 rows x 128 keys
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + 2 * KV_BYTES;
  static constexpr uint32_t OFF_P = OFF_V + 2 * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_P + P_BYTES;
  static constexpr size_t SMEM = OFF_BAR + 256 + 1024;
};

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1)
tree_attention_tc_kernel(const __grid_constant__ CUtensorMap kv_map, const Params p) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;       // [2]
  uint64_t* kv_empty = bars + 2;  // [2]
  uint64_t* s_full = bars + 4;    // [2]
  uint64_t* q_full = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int mtile = blockIdx.x;
  const int kvh = blockIdx.y;
  const int req = blockIdx.z;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    mbar_init(q_full, 128);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&kv_map);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t O_COL = 2 * BN;

  auto give_up = [&]() {
    *abort_flag = 1;
    if (p.status != nullptr) atomicMax(p.status, static_cast<int32_t>(SG_ERR_CUDA));
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int plane_k = p.plane_k0 + kvh, plane_v = p.plane_v0 + kvh;
      for (int j = 0; j < tiles && !*abort_flag; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[s], ph ^ 1u)) {
          give_up();
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * L::KV_BYTES);
        const int row = row0 + j * BN;
#pragma unroll
        for (int h = 0; h < L::HALVES; ++h) {
          tma_load_3d(smem + L::OFF_K + s * L::KV_BYTES + h * ATOM, &kv_map, h * 64, row, plane_k, &kv_full[s]);
          tma_load_3d(smem + L::OFF_V + s * L::KV_BYTES + h * ATOM, &kv_map, h * 64, row, plane_v, &kv_full[s]);
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
        const int s = j & 1;
        if (!mbar_wait(&kv_full[s], (j >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::OFF_K + s * L::KV_BYTES);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * ATOM + (ks & 3) * 32;
          mma_bf16(tmem + s * BN, desc_k_sw128(q_addr + off), desc_k_sw128(k_addr + off), idesc_qk,
                   ks > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[s]);
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
        const int s = j & 1;
        const uint32_t v_addr = smem_u32(smem + L::OFF_V + s * L::KV_BYTES);
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks) {
          const uint64_t adesc = desc_k_sw128(p_addr + (ks >> 2) * ATOM + (ks & 3) * 32);
          const uint64_t bdesc = desc_mn_sw128(v_addr + ks * 16 * 128, ATOM, 1024);
          mma_bf16(tmem + O_COL, adesc, bdesc, idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&kv_empty[s]);
        mma_commit(o_done);
      }
      if (!ok) give_up();
    }
  } else {
    // ---------------------------------------------------- softmax, one row/thread
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int m_row = m_base + r;
    const bool valid = m_row < rows_total;
    const int tok = valid ? m_row / G : 0;
    const int head = kvh * G + (valid ? m_row % G : 0);
    {  // Q row -> shared memory (K-major, 128B swizzle)
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
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        float t[32];
        tmem_ld32(tmem + lane_base + s * BN + c * 32, t);
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[c * 32 + e] = t[e] * c2;
      }
      const int64_t key0 = static_cast<int64_t>(j) * BN;
      if (key0 + BN > Lp) {  // tile reaches the tree keys or the end
#pragma unroll
        for (int e = 0; e < BN; ++e) {
          const int64_t key = key0 + e;
          bool vis = true;
          if (key >= Lp) {
            const int k = static_cast<int>(key - Lp);
            vis = key < kv_total && ((anc[k >> 5] >> (k & 31)) & 1u);
          }
          if (!vis) sv[e] = -INFINITY;
        }
      }
      float mt = -INFINITY;
#pragma unroll
      for (int e = 0; e < BN; ++e) mt = fmaxf(mt, sv[e]);
      if (j > 0 && !mbar_wait(o_done, (j - 1) & 1)) {  // PV_{j-1} done: P free, O stable
        ok = false;
        break;
      }
      tc_fence_after();
      const bool grow = mt > m_run + kRescaleThreshold;
      if (j == 0) {
        m_run = mt;
      } else if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mt : m_run;
        const float alpha = exp2f(m_run - m_new);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_base + O_COL + c * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= alpha;
          tmem_st32(tmem + lane_base + O_COL + c * 32, o);
        }
        tmem_wait_st();
        l_run *= alpha;
        m_run = m_new;
      }
      float rs = 0.f;
      uint8_t* prow = smem + L::OFF_P;
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          e8[e] = exp2f(sv[c * 8 + e] - m_run);
          rs += e8[e];
        }
        uint4 w;
        w.x = pack_bf16x2(e8[0], e8[1]);
        w.y = pack_bf16x2(e8[2], e8[3]);
        w.z = pack_bf16x2(e8[4], e8[5]);
        w.w = pack_bf16x2(e8[6], e8[7]);
        *reinterpret_cast<uint4*>(prow + (c >> 3) * ATOM + swz128(r, c & 7)) = w;
      }
      l_run += rs;
      if (key0 + r >= kv_total) {
        // Keys past the request's tail come from stale arena rows (possibly
        // NaN bit patterns); P is 0 there, but 0 * NaN is NaN in the MMA, so
        // zero this row of the V tile before P_j is released.
        uint8_t* vrow = smem + L::OFF_V + s * L::KV_BYTES + r * 128;
#pragma unroll
        for (int h = 0; h < L::HALVES; ++h)
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vrow + h * ATOM + c * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && !mbar_wait(o_done, (tiles - 1) & 1)) ok = false;
    if (!ok) {
      give_up();
    } else {
      tc_fence_after();
      const float inv = 1.f / l_run;
      __nv_bfloat16* dst = p.out + ((q0 + tok) * p.nq + head) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + O_COL + c * 32, o);
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
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int D>
int launch_d(const CUtensorMap& map, const Params& p, dim3 grid, cudaStream_t stream) {
  static int configured = 0;
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (!(configured & (1 << dev))) {
    SG_CUDA_CHECK(cudaFuncSetAttribute(tree_attention_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Layout<D>::SMEM)));
    configured |= 1 << dev;
  }
  tree_attention_tc_kernel<D><<<grid, THREADS, Layout<D>::SMEM, stream>>>(map, p);
  return check_launch("tree_attention_tc_kernel");
}

}  // namespace

int launch(const CUtensorMap& kv_map, const Params& p, int num_requests, int max_rows_per_request, int head_dim,
           cudaStream_t stream) {
  if (num_requests <= 0) return SG_OK;
  if (max_rows_per_request > layers::kMaxTreeRows)
    return fail(SG_ERR_UNSUPPORTED, "tree attention: more than 256 rows in one request");
  const int mtiles = (max_rows_per_request * p.group + BM - 1) / BM;
  dim3 grid(static_cast<unsigned>(mtiles), static_cast<unsigned>(p.nkv), static_cast<unsigned>(num_requests));
  if (head_dim == 128) return launch_d<128>(kv_map, p, grid, stream);
  if (head_dim == 64) return launch_d<64>(kv_map, p, grid, stream);
  return fail(SG_ERR_UNSUPPORTED, "tree attention: head_dim must be 64 or 128");
}

}  // namespace attn
}  // namespace sg
