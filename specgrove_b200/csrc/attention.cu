// Request-isolated packed tree attention on tcgen05 tensor cores (sm_100a).
//
// Reference semantics: the packed additive mask of
// continuous_tree_block_decode.py:500-546 — tree row j of request i sees the
// request's own KV prefix [0, L_i) and its own ancestors-or-self in the tree
// (Tree.visibility, tree.py:19-26), nothing of other requests — applied by HF
// SDPA inside Qwen3Model (engine.py:499-517) with GQA.
//
// No mask tensor and no packed KV copy exist.  A work item is (request, kv
// head, block of 128 query rows); its rows are the request's tree rows x the
// kv head's query-head group (row r -> token r / G, head h*G + r % G), so
// every K/V byte streamed from the request's arena slot serves all G heads.
// One persistent CTA per SM works through the items (longest requests first);
// the kernel and its warp roles are described above tree_attention_tm_kernel.
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
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 64 bits of a 256-bit set held as four 64-bit words, starting at bit pos
// (0 <= pos < 256; bits past 255 read as 0).  Register selects only, no
// dynamically indexed (local-memory) array.
__device__ __forceinline__ uint64_t bits64_at(const uint64_t (&w)[4], int pos) {
  const int wi = pos >> 6, bo = pos & 63;
  const uint64_t lo = wi == 0 ? w[0] : wi == 1 ? w[1] : wi == 2 ? w[2] : w[3];
  const uint64_t hi = wi == 0 ? w[1] : wi == 1 ? w[2] : wi == 2 ? w[3] : 0ull;
  return bo == 0 ? lo : (lo >> bo) | (hi << (64 - bo));
}

// Visibility of 64 consecutive keys of one query row: bit e is set when key
// (kk + e) of the request's tree is visible, where negative indices are the
// cached prefix (always visible) and tree key t < n is visible when bit t of
// the row's ancestor-or-self set is.
__device__ __forceinline__ uint64_t visible64(const uint64_t (&anc)[4], int64_t kk, int n) {
  uint64_t vis = 0;
  if (kk < 0) vis = kk <= -64 ? ~0ull : (1ull << static_cast<int>(-kk)) - 1;  // prefix keys
  const int64_t s0 = kk < 0 ? 0 : kk;                                          // first tree key
  const int e0 = static_cast<int>(s0 - kk);                                    // its bit
  if (e0 < 64 && s0 < n) {
    uint64_t t = bits64_at(anc, static_cast<int>(s0));
    const int64_t cnt = n - s0;  // tree keys left
    if (cnt < 64) t &= (1ull << static_cast<int>(cnt)) - 1;
    vis |= t << e0;
  }
  return vis;
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// ---------------------------------------------------------------------------
// Persistent tensor-memory-resident kernel, 128-key tiles, split-KV softmax.
//
// One CTA per SM draws work items — (request, kv head, 128-row query block),
// longest requests first — from a per-launch atomic counter, and every role
// streams across item boundaries: the TMA warp fetches the next item and
// starts its K/V loads while the current item's last tiles are computed.
//
// Q and P live in TMEM and feed the MMAs as the A operand, so shared memory
// holds only the K/V ring and the tensor core reads just K or V from it.
// S = Q K^T of a 128-key tile is one N=128 MMA chain.  The two softmax warps
// of a TMEM lane quarter (one SM sub-partition) each own one 64-key half of
// every tile with their own running max, sum and O accumulator (split-KV
// inside the CTA), so they never exchange anything per tile; the halves merge
// once per item.  The MMA thread follows a fixed schedule with blocking
// waits: QK^T of tile j as soon as K_j has landed and S_{j-1} has been read,
// then PV of tile j-1 (two independent N=D chains, one per half) once P_{j-1}
// is written.  The exponentials of tile j overlap PV_{j-1}.
//
// TMEM columns (512): O_half0 [0, D), O_half1 [D, 2D), Q [2D, 2.5D) as bf16
// pairs, P_half0 / P_half1 (32 columns each, bf16 pairs), S (128 fp32).
template <int D, int KST, int VST>
struct TmLayout {
  static constexpr int BN = 128;                          // keys per tile
  static constexpr int HK = BN / 2;                       // keys per softmax half
  static constexpr int THREADS = 96 + 256;                // K TMA, MMA, V TMA, 8 softmax warps
  static constexpr int HALVES = D / 64;                   // 64-dim swizzle blocks
  static constexpr uint32_t KV_HALF = BN * 128;           // 128 keys x 64 dims
  static constexpr uint32_t KV_BYTES = HALVES * KV_HALF;  // one K or V tile
  static constexpr uint32_t OFF_K = 0;                    // KST-slot K ring
  static constexpr uint32_t OFF_V = KST * KV_BYTES;       // VST-slot V ring
  static constexpr uint32_t OFF_RED = (KST + VST) * KV_BYTES;  // [2 halves][2: max, sum][128] floats
  static constexpr uint32_t OFF_ITEM = OFF_RED + 4 * 128 * 4;  // [2] published work items
  static constexpr uint32_t OFF_BAR = OFF_ITEM + 128;
  // 2 * (KST + VST) ring barriers + 13 others (8 bytes each), then the TMEM
  // base address and the abort flag.
  static constexpr uint32_t BAR_BYTES = (2 * (KST + VST) + 13) * 8 + 8;
  static constexpr size_t SMEM = OFF_BAR + ((BAR_BYTES + 127) / 128) * 128;
  static constexpr uint32_t O_COL = 0;                    // + half * D
  static constexpr uint32_t Q_COL = 2 * D;
  static constexpr uint32_t P_COL = Q_COL + D / 2;        // + half * HK / 2
  static constexpr uint32_t S_COL = P_COL + HK;           // + half * HK
  static_assert(S_COL + BN <= 512, "TMEM column map");
  static_assert(SMEM <= 232448, "shared memory");
};

// One work item as published by the TMA warp (tiles < 0: no more work).
struct WorkItem {
  int64_t q0;        // first packed query row of the request
  int64_t lp;        // cached prefix length L
  int32_t kvh;
  int32_t m_base;    // first query row (token-major x group) of the block
  int32_t n;         // tree rows of the request
  int32_t tiles;     // 128-key tiles over L + n keys
  int32_t row0;      // first arena row of the request's slot
  int32_t active_q;  // TMEM lane quarters holding at least one query row
};
static_assert(sizeof(WorkItem) <= 64, "work item slot");

template <int D, int KST, int VST>
__global__ void __launch_bounds__(TmLayout<D, KST, VST>::THREADS, 1)
tree_attention_tm_kernel(const __grid_constant__ CUtensorMap kv_map, const Params p) {
  using L = TmLayout<D, KST, VST>;
  constexpr int BN = L::BN;
  constexpr int HK = L::HK;
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((smem_u32(smem) & 1023u) != 0u) {
    if (threadIdx.x == 0 && p.status != nullptr) atomicMax(p.status, static_cast<int32_t>(SG_ERR_UNSUPPORTED));
    return;
  }
  WorkItem* items = reinterpret_cast<WorkItem*>(smem + L::OFF_ITEM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* k_full = bars;                // [KST] K tile landed
  uint64_t* k_empty = k_full + KST;       // [KST] K tile consumed by QK^T
  uint64_t* v_full = k_empty + KST;       // [VST] V tile landed
  uint64_t* v_empty = v_full + VST;       // [VST] V tile consumed by PV
  uint64_t* s_full = v_empty + VST;       // S of a tile written
  uint64_t* s_free = s_full + 1;          // S read by every softmax thread
  uint64_t* p_full = s_free + 1;          // P (both halves) written
  uint64_t* o_done = p_full + 1;          // PV of a tile complete
  uint64_t* q_full = o_done + 1;          // Q rows of an item in TMEM
  uint64_t* merge = q_full + 1;           // [4 quarters] per-item (max, sum) exchange
  uint64_t* item_full = merge + 4;        // [2] work item published
  static_assert(2 * (KST + VST) + 13 == 2 * KST + 2 * VST + 4 + 1 + 4 + 2 + 2, "barrier count");
  uint64_t* item_empty = item_full + 2;   // [2] work item read by every consumer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    // Per-tile and per-item barriers count every softmax thread.
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(p_full, 256);
    mbar_init(o_done, 1);
    mbar_init(q_full, 256);
    for (int i = 0; i < 4; ++i) mbar_init(&merge[i], 64);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 2 + 256);  // MMA thread, V producer, softmax
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&kv_map);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // q, the K/V tail and the work list come from earlier kernels

  auto give_up = [&]() {
    *abort_flag = 1;
    if (p.status != nullptr) atomicMax(p.status, static_cast<int32_t>(SG_ERR_CUDA));
  };
  // Producers: load the item's K (or V) tiles into their ring, tile index gt
  // onwards (across items).
  auto load_tiles = [&](const WorkItem& it, int64_t gt, int plane0, uint32_t off_ring, uint64_t* full,
                        uint64_t* empty, int stages) -> bool {
    const int plane = plane0 + it.kvh;
    for (int j = 0; j < it.tiles; ++j, ++gt) {
      const int s = static_cast<int>(gt % stages);
      if (*abort_flag || !mbar_wait(&empty[s], static_cast<uint32_t>((gt / stages) & 1) ^ 1u)) {
        give_up();
        return false;
      }
      mbar_arrive_expect_tx(&full[s], L::KV_BYTES);
      const int row = it.row0 + j * BN;
#pragma unroll
      for (int h = 0; h < L::HALVES; ++h)
#pragma unroll
        for (int rb = 0; rb < BN / kKeyTile; ++rb)  // the map's box is kKeyTile rows
          tma_load_3d(smem + off_ring + s * L::KV_BYTES + h * L::KV_HALF + rb * kKeyTile * 128, &kv_map, h * 64,
                      row + rb * kKeyTile, plane, &full[s]);
    }
    return true;
  };
  // Consumers: wait for work item `seq`, copy it, release the slot.
  auto next_item = [&](int seq, WorkItem& it) -> bool {
    if (!mbar_wait(&item_full[seq & 1], (seq >> 1) & 1)) return false;
    it = items[seq & 1];
    mbar_arrive(&item_empty[seq & 1]);
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------ scheduler + TMA producer
    if (lane == 0) {
      const int total = *p.num_items;
      int64_t gt = 0;  // tiles loaded so far (across items)
      for (int seq = 0;; ++seq) {
        WorkItem it;
        it.tiles = -1;
        while (!*abort_flag) {
          const int i = atomicAdd(p.work_counter, 1);
          if (i >= total) break;
          const int code = p.items[i];
          const int req = code >> 16;
          const int64_t q0 = p.row_offsets[req];
          const int64_t q1 = p.row_offsets[req + 1];
          const int64_t lp = p.cache_len[req];
          const int64_t slot = p.slots[req];
          if (q0 < 0 || q1 > p.num_rows || q1 - q0 < 1 || q1 - q0 > layers::kMaxTreeRows) continue;
          const int n = static_cast<int>(q1 - q0);
          const int m_base = (code & 0xff) * BM;
          if (m_base >= n * p.group) continue;
          // Never read outside the request's own slot (the QKV kernel reports
          // the capacity error for such a request).
          if (slot < 0 || (slot + 1) * p.capacity > p.plane_rows || lp < 0 || lp + n > p.capacity) continue;
          it.q0 = q0;
          it.lp = lp;
          it.kvh = (code >> 8) & 0xff;
          it.m_base = m_base;
          it.n = n;
          it.tiles = static_cast<int>((lp + n + BN - 1) / BN);
          it.row0 = static_cast<int>(slot * p.capacity);
          it.active_q = min(4, (n * p.group - m_base + 31) / 32);
          break;
        }
        if (!mbar_wait(&item_empty[seq & 1], ((seq >> 1) & 1) ^ 1u)) {
          give_up();
          break;
        }
        items[seq & 1] = it;
        mbar_arrive(&item_full[seq & 1]);
        if (it.tiles < 0) break;
        if (!load_tiles(it, gt, p.plane_k0, L::OFF_K, k_full, k_empty, KST)) break;
        gt += it.tiles;
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ V producer
    // Follows the published items with its own ring, so K loads never queue
    // behind a V tile whose slot PV has not released yet.
    if (lane == 0) {
      int64_t gt = 0;
      for (int seq = 0;; ++seq) {
        WorkItem it;
        if (!next_item(seq, it)) {
          give_up();
          break;
        }
        if (it.tiles < 0) break;
        if (!load_tiles(it, gt, p.plane_v0, L::OFF_V, v_full, v_empty, VST)) break;
        gt += it.tiles;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_bf16_f32(BM, BN);
      const uint32_t idesc_pv = idesc_bf16_f32(BM, D) | (1u << 16);  // B (V) is MN-major
      int64_t gt = 0;  // tiles consumed so far (across items)
      bool ok = true;
      for (int seq = 0; ok; ++seq) {
        WorkItem it;
        if (!next_item(seq, it)) {
          ok = false;
          break;
        }
        if (it.tiles < 0) break;
        if (!mbar_wait(q_full, seq & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int j = 0; j <= it.tiles; ++j) {
          const int64_t g = gt + j;
          if (j < it.tiles) {  // S_j = Q K_j^T
            const int s = static_cast<int>(g % KST);
            if (!mbar_wait(&k_full[s], static_cast<uint32_t>((g / KST) & 1)) ||
                (g > 0 && !mbar_wait(s_free, static_cast<uint32_t>((g - 1) & 1)))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t k_addr = smem_u32(smem + L::OFF_K + s * L::KV_BYTES);
#pragma unroll
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint32_t koff = (ks >> 2) * L::KV_HALF + (ks & 3) * 32;
              mma_bf16_ta(tmem + L::S_COL, tmem + L::Q_COL + ks * 8, desc_k_sw128(k_addr + koff), idesc_qk,
                          ks > 0 ? 1u : 0u);
            }
            mma_commit(&k_empty[s]);
            mma_commit(s_full);
          }
          if (j > 0) {  // O_h += P_{j-1,h} V_{j-1,h}
            const int s = static_cast<int>((g - 1) % VST);
            if (!mbar_wait(p_full, static_cast<uint32_t>((g - 1) & 1)) ||
                !mbar_wait(&v_full[s], static_cast<uint32_t>(((g - 1) / VST) & 1))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(smem + L::OFF_V + s * L::KV_BYTES);
#pragma unroll
            for (int ks = 0; ks < HK / 16; ++ks)
#pragma unroll
              for (int h = 0; h < 2; ++h) {  // the two halves' chains interleave
                const uint64_t bdesc = desc_mn_sw128(v_addr + (h * HK + ks * 16) * 128, L::KV_HALF, 1024);
                mma_bf16_ta(tmem + L::O_COL + h * D, tmem + L::P_COL + h * (HK / 2) + ks * 8, bdesc, idesc_pv,
                            (j > 1 || ks > 0) ? 1u : 0u);
              }
            mma_commit(&v_empty[s]);
            mma_commit(o_done);
          }
        }
        gt += it.tiles;
      }
      if (!ok) give_up();
    }
  } else {
    // --------------------------------------------------------------- softmax
    // Warp w serves TMEM lane quarter w % 4 (the lanes it may access) and key
    // half hf = (w - 3) / 4 of every tile, one 64-key row per thread.  A warp
    // whose quarter holds no query row of an item still takes every barrier
    // step of every tile (it only skips the work): parity waits are exact
    // only for a waiter at most one phase away from the barrier, so no warp
    // may skip phases and later rejoin.
    const int quarter = warp & 3;
    const int hf = (warp - 3) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float c2 = p.scale_log2;
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);
    int gt = 0;  // tiles consumed so far (across items)
    int merges = 0;  // items this quarter was active in (merge barrier phase)
    bool ok = true;
    // Row of the query block this thread serves in item w (token, head).
    auto row_of = [&](const WorkItem& w, bool& valid, int& tok, int& head) {
      const int m_row = w.m_base + r;
      valid = quarter < w.active_q && m_row < w.n * p.group;
      tok = valid ? m_row / p.group : 0;
      head = w.kvh * p.group + (valid ? m_row % p.group : 0);
    };
    // This thread's half of item w's Q row -> TMEM (two bf16 per column,
    // 16 columns at a time), then arrive on q_full.  Called for the next item
    // once S of the current item's last tile has been read, i.e. after the
    // current item's last QK^T completed, so QK^T of the next item overlaps
    // the current item's last exponentials, PV and epilogue.  The next item's
    // first PV, which overwrites O, still waits for every thread's P of that
    // item, issued only after this thread's epilogue.
    auto stage_q = [&](const WorkItem& w) {
      if (quarter < w.active_q) {
        bool valid;
        int tok, head;
        row_of(w, valid, tok, head);
        constexpr int QW = D / 4;  // columns per thread
        const uint4* src = reinterpret_cast<const uint4*>(p.q + ((w.q0 + tok) * p.nq + head) * D + hf * (D / 2));
#pragma unroll
        for (int ch = 0; ch < QW / 16; ++ch) {
          uint32_t qw[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 v = valid ? src[ch * 4 + c] : make_uint4(0u, 0u, 0u, 0u);
            qw[4 * c + 0] = v.x;
            qw[4 * c + 1] = v.y;
            qw[4 * c + 2] = v.z;
            qw[4 * c + 3] = v.w;
          }
          tmem_st16u(tmem + lane_base + L::Q_COL + hf * QW + ch * 16, qw);
        }
        tmem_wait_st();
        prefetch_l1(p.anc + (w.q0 + tok) * layers::kAncWords);  // read when the item starts
      }
      tc_fence_before();
      mbar_arrive(q_full);
    };
    auto load_anc = [&](const WorkItem& w, uint64_t (&a4)[4]) {  // ancestor-or-self set (256 bits)
      bool valid;
      int tok, head;
      row_of(w, valid, tok, head);
      const uint4* ap = reinterpret_cast<const uint4*>(p.anc + (w.q0 + tok) * layers::kAncWords);
      const uint4 a = ap[0], b = ap[1];
      a4[0] = (static_cast<uint64_t>(a.y) << 32) | a.x;
      a4[1] = (static_cast<uint64_t>(a.w) << 32) | a.z;
      a4[2] = (static_cast<uint64_t>(b.y) << 32) | b.x;
      a4[3] = (static_cast<uint64_t>(b.w) << 32) | b.z;
    };
    WorkItem it;
    if (!next_item(0, it)) ok = false;
    uint64_t anc[4] = {0ull, 0ull, 0ull, 0ull};
    if (ok && it.tiles >= 0) {
      stage_q(it);
      if (quarter < it.active_q) load_anc(it, anc);
    }
    for (int seq = 0; ok && it.tiles >= 0; ++seq) {
      const int tiles = it.tiles;
      // At the item's last tile, once its S has been read: wait for the next
      // item and stage its Q, reading it in place (its slot is released only
      // when this item is done, so it cannot be overwritten meanwhile).
      auto at_last_tile = [&]() -> bool {
        if (!mbar_wait(&item_full[(seq + 1) & 1], ((seq + 1) >> 1) & 1)) return false;
        const WorkItem& nx = items[(seq + 1) & 1];
        if (nx.tiles >= 0) stage_q(nx);
        return true;
      };
      // One tile before that: if the next item is already published, pull
      // this thread's Q half-row and ancestor row into L1 (no wait).
      auto prefetch_next = [&]() {
        if (!mbar_test(&item_full[(seq + 1) & 1], ((seq + 1) >> 1) & 1)) return;
        const WorkItem& nx = items[(seq + 1) & 1];
        if (nx.tiles < 0 || quarter >= nx.active_q) return;
        bool valid;
        int tok, head;
        row_of(nx, valid, tok, head);
        prefetch_l1(p.q + ((nx.q0 + tok) * p.nq + head) * D + hf * (D / 2));
        prefetch_l1(p.anc + (nx.q0 + tok) * layers::kAncWords);
      };
      // Move on: copy the next item out of its slot and release the slot.
      auto advance = [&]() {
        it = items[(seq + 1) & 1];
        mbar_arrive(&item_empty[(seq + 1) & 1]);
        if (it.tiles >= 0 && quarter < it.active_q) load_anc(it, anc);
      };
      if (quarter >= it.active_q) {
        // Idle quarter: take every barrier step of every tile (no work).
        for (int j = 0; j < tiles && ok; ++j) {
          const int g = gt + j;
          if (!mbar_wait(s_full, static_cast<uint32_t>(g) & 1u)) ok = false;
          mbar_arrive(s_free);
          if (ok && j == tiles - 1 && !at_last_tile()) ok = false;
          if (ok && j > 0 && !mbar_wait(o_done, static_cast<uint32_t>(g - 1) & 1u)) ok = false;
          mbar_arrive(p_full);
        }
        if (ok && !mbar_wait(o_done, static_cast<uint32_t>(gt + tiles - 1) & 1u)) ok = false;
        gt += tiles;
        if (ok) advance();
        continue;
      }
      bool valid;
      int tok, head;
      row_of(it, valid, tok, head);
      const int lp = static_cast<int>(it.lp);  // < capacity
      const int kv_total = lp + it.n;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < tiles; ++j) {
        const int g = gt + j;
        if (!mbar_wait(s_full, static_cast<uint32_t>(g) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[HK];
        {
          uint32_t raw[HK];
          tmem_ld32_nowait(tmem + lane_base + L::S_COL + hf * HK, raw);
          tmem_ld32_nowait(tmem + lane_base + L::S_COL + hf * HK + 32, raw + 32);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < HK; ++e) sv[e] = __uint_as_float(raw[e]);
        }
        tc_fence_before();
        mbar_arrive(s_free);
        if (j == tiles - 2) prefetch_next();
        if (j == tiles - 1 && !at_last_tile()) {
          ok = false;
          break;
        }
        const int key0 = j * BN + hf * HK;
        if (key0 + HK > lp) {  // this half reaches the tree keys or the end
          const uint64_t vis = visible64(anc, key0 - lp, it.n);
#pragma unroll
          for (int e = 0; e < HK; ++e)
            if (!((vis >> e) & 1ull)) sv[e] = -INFINITY;
        }
        float mt;
        {  // row max of the 64 scores: three-input max tree (64 -> 22 -> 8 -> 3 -> 1)
          float t[22];
#pragma unroll
          for (int e = 0; e < 21; ++e) t[e] = fmax3f(sv[3 * e], sv[3 * e + 1], sv[3 * e + 2]);
          t[21] = sv[63];
          float u[8];
#pragma unroll
          for (int e = 0; e < 7; ++e) u[e] = fmax3f(t[3 * e], t[3 * e + 1], t[3 * e + 2]);
          u[7] = t[21];
          mt = fmax3f(fmax3f(u[0], u[1], u[2]), fmax3f(u[3], u[4], u[5]), fmaxf(u[6], u[7])) * c2;
        }
        // Lazy rescaling: move the reference max only when the tile max
        // exceeds it by more than 2^8 (the first tile always sets it).
        const bool grow = j == 0 || mt > m_run + kRescaleThreshold;
        const bool rescale = j > 0 && __any_sync(0xffffffffu, grow);
        float alpha = 1.f;
        if (grow) {
          alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mt);
          m_run = mt;
        }
        // A row whose keys so far are all masked has m_run = -inf; its P is
        // then 0 (not NaN) with the offset taken as 0.
        const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        uint32_t pw[HK / 2];
#pragma unroll
        for (int c = 0; c < HK / 8; ++c) {
          float e8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            e8[e] = fast_exp2(fmaf(sv[c * 8 + e], c2, neg_m));
            acc[e] += e8[e];
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) pw[c * 4 + e] = pack_bf16x2(e8[2 * e], e8[2 * e + 1]);
        }
        l_run = l_run * alpha + (((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7])));
        // P and this half's O accumulator were last used by PV of tile g-1
        if (j > 0 && !mbar_wait(o_done, static_cast<uint32_t>(g - 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (rescale) {  // rare: the row max grew by more than 2^8
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_base + L::O_COL + hf * D + c * 32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tmem + lane_base + L::O_COL + hf * D + c * 32, o);
          }
        }
        tmem_st32u(tmem + lane_base + L::P_COL + hf * (HK / 2), pw);
        tmem_wait_st();
        if (key0 + HK > kv_total) {
          // Keys past the request's tail come from stale arena rows (possibly
          // NaN bit patterns); P is 0 there, but 0 * NaN is NaN in the MMA,
          // so zero those rows of this half of the V tile (once it has
          // landed) before P is released.  The V slot's barrier is at most
          // one phase from this wait: PV of tile g - VST completed (o_done
          // of g - 1) and the slot cannot refill before PV of tile g.
          const int s = g % VST;
          if (!mbar_wait(&v_full[s], static_cast<uint32_t>(g / VST) & 1u)) {
            ok = false;
            break;
          }
          for (int v = r; v < HK; v += 32 * it.active_q) {
            if (key0 + v < kv_total) continue;
            uint8_t* vrow = smem + L::OFF_V + s * L::KV_BYTES + (hf * HK + v) * 128;
#pragma unroll
            for (int h = 0; h < L::HALVES; ++h)
#pragma unroll
              for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(vrow + h * L::KV_HALF + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (ok && !mbar_wait(o_done, static_cast<uint32_t>(gt + tiles - 1) & 1u)) ok = false;
      if (!ok) break;
      // Merge the two halves' (max, sum, O): each warp writes out half of the
      // O columns.  The next item's first PV overwrites O only after every
      // softmax thread arrived on that item's q_full.
      red[(hf * 2 + 0) * 128 + r] = m_run;
      red[(hf * 2 + 1) * 128 + r] = l_run;
      tc_fence_before();
      mbar_arrive(&merge[quarter]);
      if (!mbar_wait(&merge[quarter], merges & 1)) {
        ok = false;
        break;
      }
      ++merges;
      {
        const float m0 = red[0 * 128 + r], l0 = red[1 * 128 + r];
        const float m1 = red[2 * 128 + r], l1 = red[3 * 128 + r];
        const float m = fmaxf(m0, m1);
        const float w0 = m0 == -INFINITY ? 0.f : fast_exp2(m0 - m);
        const float w1 = m1 == -INFINITY ? 0.f : fast_exp2(m1 - m);
        const float inv = 1.f / (l0 * w0 + l1 * w1);
        tc_fence_after();
        __nv_bfloat16* dst = p.out + ((it.q0 + tok) * p.nq + head) * D + hf * (D / 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          float o0[32], o1[32];
          const uint32_t col = hf * (D / 2) + c * 32;
          tmem_ld32(tmem + lane_base + L::O_COL + col, o0);
          tmem_ld32(tmem + lane_base + L::O_COL + D + col, o1);
#pragma unroll
          for (int e = 0; e < 32; ++e) o0[e] = (o0[e] * w0 + o1[e] * w1) * inv;
          if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack_bf16x2(o0[q * 8 + 0], o0[q * 8 + 1]);
              w.y = pack_bf16x2(o0[q * 8 + 2], o0[q * 8 + 3]);
              w.z = pack_bf16x2(o0[q * 8 + 4], o0[q * 8 + 5]);
              w.w = pack_bf16x2(o0[q * 8 + 6], o0[q * 8 + 7]);
              d4[q] = w;
            }
          }
        }
      }
      gt += tiles;
      advance();
    }
    if (!ok) give_up();
  }
  // Roles ran on one lane of warps 0-2: reconverge each warp before the CTA
  // barrier that precedes freeing TMEM.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, int KST, int VST>
int launch_tm(const CUtensorMap& map, const Params& p, int num_requests, cudaStream_t stream) {
  using L = TmLayout<D, KST, VST>;
  auto kernel = tree_attention_tm_kernel<D, KST, VST>;
  static std::atomic<int> limits[kMaxDevices];
  const int st = ensure_dynamic_smem(kernel, L::SMEM, limits);
  if (st != SG_OK) return st;
  if (p.items == nullptr || p.num_items == nullptr || p.work_counter == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "tree attention: missing work list");
  // One CTA per SM; every (request, kv head) has at least one item.
  const int ctas = static_cast<int>(min64(device_sm_count(), static_cast<int64_t>(num_requests) * p.nkv));
  return launch_pdl("tree_attention_tm_kernel", kernel, dim3(static_cast<unsigned>(ctas)), dim3(L::THREADS), L::SMEM,
                    stream, map, p);
}

}  // namespace

int launch(const CUtensorMap& kv_map, const Params& p, int num_requests, int max_rows_per_request, int head_dim,
           cudaStream_t stream) {
  if (num_requests <= 0) return SG_OK;
  if (max_rows_per_request > layers::kMaxTreeRows)
    return fail(SG_ERR_UNSUPPORTED, "tree attention: more than 256 rows in one request");
  // head_dim 128: 4-slot K ring and 3-slot V ring of 128-key tiles (231.8 KB
  // of shared memory); head_dim 64: 6 + 6 slots of half the size.
  if (head_dim == 128) return launch_tm<128, 4, 3>(kv_map, p, num_requests, stream);
  if (head_dim == 64) return launch_tm<64, 6, 6>(kv_map, p, num_requests, stream);
  return fail(SG_ERR_UNSUPPORTED, "tree attention: head_dim must be 64 or 128");
}

}  // namespace attn
}  // namespace sg
