// Persistent, warp-specialised tcgen05 GEMM for sm_100a:
//   acc[M, N] = A[M, K] . B[N, K]^T      (bf16 operands, fp32 accumulate in TMEM)
// A and B are K-major (row-major with K contiguous), as packed activation rows
// and nn.Linear weights are.  Tiles are 128 x 256 with K-blocks of 64:
//   warp 0      TMA producer: A/B tiles -> 128B-swizzled shared memory ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16)
//               into one of two TMEM accumulators (2 x 256 columns)
//   warps 2..5  epilogue: tcgen05.ld the accumulator (32 rows per warp),
//               apply the fused epilogue, store; frees the accumulator so the
//               next tile's MMAs overlap this tile's epilogue.
// Tiles are visited n-major (all M tiles of a weight panel back to back) so a
// weight panel is read from HBM once and served from L2 to the other M tiles.
//
// Wave tail (stream-K): with T tiles on P CTAs, the T mod P tiles left after
// the last full wave would leave SMs idle for a whole tile.  Their k-blocks
// are instead split evenly over the CTAs, each taking one contiguous run of
// (tile, k-block) iterations.  The CTA whose run holds a tile's first k-block
// owns it: the other CTAs on that tile (at most two) write fp32 partial
// accumulators to a workspace and count themselves done on a flag; the owner
// adds the partials in k order (a fixed order, so results are reproducible),
// then runs the fused epilogue and resets the flags.  All CTAs of the grid
// (one per SM) are resident together, and every flag wait is bounded.
// An owner segment always ends its CTA's run, so when its accumulator is
// complete the operand ring is idle: the partials come into it by bulk copy
// (half a tile of every contributor per round) and the owner adds them from
// shared memory.
#pragma once

#include <type_traits>

#include "sm100.cuh"

namespace sg {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_TILE = BM * BK * 2;
constexpr int B_TILE = BN * BK * 2;
constexpr int STAGE_BYTES = A_TILE + B_TILE;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr int BARRIER_BYTES = 256;
constexpr int EPI_STAGE_BYTES = 32 * 8 * 16;  // per epilogue warp: 32 rows x 8 x 16 B
constexpr size_t SMEM_BYTES =
    static_cast<size_t>(STAGES) * STAGE_BYTES + 1024 + BARRIER_BYTES + 4 * EPI_STAGE_BYTES;
constexpr uint32_t IDESC = sm100::idesc_bf16_f32(BM, BN);

// Per tile width: the default 256 columns, or 160 for the residual
// projections (a 4096-wide output is 26 tiles per 128 rows, 2.81 waves of
// 148 SMs at 2048 rows against 1.73 for 256-wide tiles).  Narrower tiles
// leave room for a fifth ring stage, and two fp32 partials of a split tile
// fit the ring in one combine round.
template <int TBN>
struct Cfg {
  static_assert(TBN % 32 == 0 && TBN >= 32 && TBN <= 256, "tile width");
  static constexpr int B_TILE = TBN * BK * 2;
  static constexpr int STAGE_BYTES = A_TILE + B_TILE;
  static constexpr int STAGES = TBN == 256 ? 4 : 5;
  static constexpr size_t SMEM_BYTES =
      static_cast<size_t>(STAGES) * STAGE_BYTES + 1024 + BARRIER_BYTES + 4 * EPI_STAGE_BYTES;
  static constexpr uint32_t IDESC = sm100::idesc_bf16_f32(BM, TBN);
  static constexpr int ROUNDS = TBN == 256 ? 2 : 1;  // stream-K combine rounds (2 partials per round fit the ring)
  static_assert(2 * BM * (TBN / ROUNDS) * 4 <= STAGES * STAGE_BYTES, "combine round exceeds the ring");
  static_assert(BM * TBN * 4 <= STAGES * STAGE_BYTES, "staged tile exceeds the ring");
  static_assert(2 * TBN <= static_cast<int>(TMEM_COLS), "two accumulators exceed TMEM");
};

// Stream-K plan for the tiles after the last full wave (sk_ctas == 0: none).
struct Split {
  int t_dp;         // tiles [0, t_dp) run whole, round-robin over the grid
  int sk_ctas;      // CTAs [0, sk_ctas) share the k-blocks of tiles [t_dp, tiles)
  int per, rem;     // CTA c takes per (+1 when c < rem) consecutive iterations
  int max_slots;    // partial buffers per split tile (contributors per tile)
  float* partials;  // [split tile][slot][tile width / 4][BM] float4 (slot stride BM * BN floats)
  int* flags;       // [split tile][slot]: 128 once the contributor's threads are done
};

struct Shape {
  int M, N, K;
  int bn;  // tile width (columns)
  int m_tiles, n_tiles, k_blocks, tiles;
  Split sp;
};

inline Shape make_shape(int M, int N, int K, int bn = BN) {
  Shape s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.bn = bn;
  s.m_tiles = (M + BM - 1) / BM;
  s.n_tiles = (N + bn - 1) / bn;
  s.k_blocks = K / BK;
  s.tiles = s.m_tiles * s.n_tiles;
  s.sp = Split{s.tiles, 0, 0, 0, 0, nullptr, nullptr};
  return s;
}

// Workspace of the stream-K tail: partial accumulators and flags.  Flags
// must be zero before the first launch (each launch leaves them zero).
struct SplitWorkspace {
  float* partials;
  int* flags;
  size_t partial_tiles;  // capacity in (tile, slot) partial buffers
};

constexpr int kMaxSlots = 2;  // contributors per split tile (each run >= half a tile)

// Worst-case (tile, slot) buffers any shape needs on `sms` CTAs.
inline size_t split_partial_tiles(int sms) { return static_cast<size_t>(sms) * kMaxSlots; }
inline size_t split_partial_bytes(int sms) { return split_partial_tiles(sms) * BM * BN * sizeof(float); }

// Plan the tail split of `s` on `sms` CTAs; leaves s.sp without a split when
// it would not help or the workspace is missing.
inline void plan_split(Shape& s, int sms, const SplitWorkspace* ws) {
  s.sp = Split{s.tiles, 0, 0, 0, 0, nullptr, nullptr};
  if (ws == nullptr || ws->partials == nullptr || ws->flags == nullptr || sms <= 0 || s.k_blocks < 2) return;
  const int tail = s.tiles % sms;  // all tiles when there is no full wave
  if (tail == 0) return;
  const int64_t iters = static_cast<int64_t>(tail) * s.k_blocks;
  const int min_run = (s.k_blocks + 1) / 2;  // keeps contributors per tile <= 2
  const int ctas = static_cast<int>(min64(sms, iters / min_run));
  if (ctas <= tail) return;  // no more CTAs than tiles: nothing to gain
  if (static_cast<size_t>(tail) * kMaxSlots > ws->partial_tiles) return;
  s.sp.t_dp = s.tiles - tail;
  s.sp.sk_ctas = ctas;
  s.sp.per = static_cast<int>(iters / ctas);
  s.sp.rem = static_cast<int>(iters % ctas);
  s.sp.max_slots = kMaxSlots;
  s.sp.partials = ws->partials;
  s.sp.flags = ws->flags;
}

__device__ __forceinline__ void tile_coords(const Shape& s, int tile, int& m0, int& n0) {
  m0 = (tile % s.m_tiles) * BM;
  n0 = (tile / s.m_tiles) * s.bn;
}

// One unit of a CTA's work: k-blocks [kb0, kb1) of a tile.
enum SegKind { kSegWhole = 0, kSegOwner = 1, kSegContrib = 2 };
struct Seg {
  int tile, kb0, kb1, kind;
  int slot;      // contributor: its partial buffer
  int ncontrib;  // owner: partial buffers to add (slots 0 .. ncontrib-1)
};

// Walks this CTA's segments: whole tiles blockIdx.x, +gridDim.x, ... below
// t_dp, then its run of tail iterations.  Every warp role walks the same list.
struct SegIter {
  int dp_next, it, end;
  __device__ void begin(const Shape& s) {
    dp_next = static_cast<int>(blockIdx.x);
    const int c = static_cast<int>(blockIdx.x);
    if (c < s.sp.sk_ctas) {
      it = c * s.sp.per + min(c, s.sp.rem);
      end = it + s.sp.per + (c < s.sp.rem ? 1 : 0);
    } else {
      it = end = 0;
    }
  }
  __device__ static int cta_of(const Split& sp, int i) {  // CTA whose run holds tail iteration i
    const int big = sp.rem * (sp.per + 1);
    return i < big ? i / (sp.per + 1) : sp.rem + (i - big) / sp.per;
  }
  __device__ bool next(const Shape& s, Seg& g) {
    if (dp_next < s.sp.t_dp) {
      g = Seg{dp_next, 0, s.k_blocks, kSegWhole, 0, 0};
      dp_next += static_cast<int>(gridDim.x);
      return true;
    }
    if (it >= end) return false;
    const int K = s.k_blocks;
    const int ti = it / K, kb0 = it % K;
    const int kb1 = min(K, kb0 + (end - it));
    g = Seg{s.sp.t_dp + ti, kb0, kb1, kSegWhole, 0, 0};
    if (kb0 == 0 && kb1 < K) {
      g.kind = kSegOwner;
      g.ncontrib = cta_of(s.sp, ti * K + K - 1) - static_cast<int>(blockIdx.x);
    } else if (kb0 > 0) {
      g.kind = kSegContrib;
      g.slot = static_cast<int>(blockIdx.x) - cta_of(s.sp, ti * K) - 1;
    }
    it += kb1 - kb0;
    return true;
  }
  __device__ bool more(const Shape& s) const { return dp_next < s.sp.t_dp || it < end; }
};

// An epilogue that reads a [BM, BN] fp32 tile of global memory may set
// kStagesTile and provide tile_src(...) and apply_staged(...): on the CTA's
// last segment (when the operand ring is idle) the tile's rows come into the
// ring by bulk copy, one row per epilogue thread, and the epilogue reads them
// from shared memory instead of issuing dependent global loads.
template <class E, class = void>
struct stages_tile : std::false_type {};
template <class E>
struct stages_tile<E, std::void_t<decltype(E::kStagesTile)>> : std::bool_constant<E::kStagesTile> {};

// Epi must provide:
//   struct Params;  (int32_t* status member)
//   static __device__ void apply(const Params&, const Shape&, uint32_t taddr,
//                                int m0, int n0, int quarter, int lane,
//                                uint4* stage);  // the warp's staging slice
template <class Epi, int TBN = BN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
            const Shape shape, const typename Epi::Params ep) {
  using namespace sm100;
  using C = Cfg<TBN>;
  constexpr int STAGES = C::STAGES;
  constexpr int STAGE_BYTES = C::STAGE_BYTES;
  constexpr int B_TILE = C::B_TILE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint4* epi_stage = reinterpret_cast<uint4*>(smem + STAGES * STAGE_BYTES + BARRIER_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* pbar = bars + 2 * STAGES + 5;  // stream-K partials -> operand ring
  uint64_t* cbar = bars + 2 * STAGES + 6;  // the owner's 128 threads are done with a round of the ring
  uint64_t* xbar = bars + 2 * STAGES + 7;  // the last tile's epilogue input -> operand ring

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(pbar, 1);
    mbar_init(cbar, 128);
    mbar_init(xbar, 128);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // activations and the residual stream come from the previous kernel

  auto fail_wait = [&](void) {
    *abort_flag = 1;
    if (ep.status != nullptr) atomicMax(ep.status, static_cast<int32_t>(SG_ERR_CUDA));
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      SegIter si;
      si.begin(shape);
      Seg g;
      while (!*abort_flag && si.next(shape, g)) {
        int m0, n0;
        tile_coords(shape, g.tile, m0, n0);
        for (int kb = g.kb0; kb < g.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u)) {
            fail_wait();
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_TILE, &tma_a, kb * BK, m0, &full[stage]);
          tma_load_2d(sB + stage * B_TILE, &tma_b, kb * BK, n0, &full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      SegIter si;
      si.begin(shape);
      Seg g;
      while (!*abort_flag && si.next(shape, g)) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u)) {
          fail_wait();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * TBN);
        bool ok = true;
        for (int kb = g.kb0; kb < g.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            fail_wait();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_TILE);
          const uint32_t b_base = smem_u32(sB + stage * B_TILE);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16(d, desc_k_sw128(a_base + k * 32), desc_k_sw128(b_base + k * 32), C::IDESC,
                     ((kb - g.kb0) | k) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int r = quarter * 32 + lane;  // row within the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    SegIter si;
    si.begin(shape);
    Seg g;
    while (si.next(shape, g)) {
      if (*abort_flag) break;
      if (!mbar_wait(&tfull[acc], acc_phase)) {
        fail_wait();
        break;
      }
      tc_fence_after();
      int m0, n0;
      tile_coords(shape, g.tile, m0, n0);
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * TBN);
      const Split& sp = shape.sp;
      const int sk_tile = g.tile - sp.t_dp;
      if (g.kind == kSegContrib) {
        // Partial accumulator -> workspace (L2), then count this thread done.
        const int fi = sk_tile * sp.max_slots + g.slot;
        float* dst = sp.partials + static_cast<size_t>(fi) * (BM * BN);
        // float4 of column quad j of row r at [j][r]: a warp's store is 512
        // contiguous bytes.
        float4* d4 = reinterpret_cast<float4*>(dst) + r;
#pragma unroll 1
        for (int c = 0; c < TBN / 32; ++c) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(d4 + (c * 8 + q) * BM, make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]));
        }
        __threadfence();
        atomicAdd(&sp.flags[fi], 1);
      } else {
        if (g.kind == kSegOwner) {
          // Wait for the contributors' partials (each flag counts 128 threads).
          bool ready = true;
          for (int slot = 0; slot < g.ncontrib && ready; ++slot) {
            const volatile int* f = sp.flags + sk_tile * sp.max_slots + slot;
            uint32_t i = 0;
            while (*f < 128 && ++i < kWaitLimit) __nanosleep(32);
            ready = *f >= 128;
          }
          if (!ready) {
            fail_wait();
            break;
          }
          __threadfence();
          // acc += partials in k order, written back to TMEM for the epilogue.
          // Round h brings columns [h TBN / ROUNDS, (h + 1) TBN / ROUNDS) of
          // every contributor (contiguous quads of the partial) into the idle
          // ring; thread 0 of the epilogue warps issues the copies.
          constexpr uint32_t kHalf = BM * (TBN / C::ROUNDS) * sizeof(float);
          constexpr int kRoundChunks = TBN / (32 * C::ROUNDS);
          const float4* ring4 = reinterpret_cast<const float4*>(smem);
          const bool issuer = threadIdx.x == 64;
          for (int h = 0; h < C::ROUNDS && ready; ++h) {
            if (issuer) {
              if (h > 0 && !mbar_wait(cbar, 0u)) {  // round 0 fully read
                fail_wait();
                ready = false;
                break;
              }
              if (h == 0) fence_proxy_async_global();  // the contributors' stores precede the bulk reads
              mbar_arrive_expect_tx(pbar, static_cast<uint32_t>(g.ncontrib) * kHalf);
              for (int slot = 0; slot < g.ncontrib; ++slot)
                bulk_g2s(smem + slot * kHalf,
                         reinterpret_cast<const uint8_t*>(sp.partials +
                                                          static_cast<size_t>(sk_tile * sp.max_slots + slot) *
                                                              (BM * BN)) +
                             h * kHalf,
                         kHalf, pbar);
            }
            if (!mbar_wait(pbar, static_cast<uint32_t>(h))) {
              fail_wait();
              ready = false;
              break;
            }
#pragma unroll 1
            for (int c = 0; c < kRoundChunks; ++c) {
              float v[32];
              const uint32_t col = static_cast<uint32_t>((h * kRoundChunks + c) * 32);
              tmem_ld32(taddr + col, v);
              for (int slot = 0; slot < g.ncontrib; ++slot) {
                const float4* src = ring4 + slot * (kHalf / 16) + r;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  const float4 pq = src[(c * 8 + q) * BM];
                  v[q * 4] += pq.x;
                  v[q * 4 + 1] += pq.y;
                  v[q * 4 + 2] += pq.z;
                  v[q * 4 + 3] += pq.w;
                }
              }
              tmem_st32(taddr + col, v);
            }
            fence_proxy_async_smem();  // this thread's reads of the ring precede the next round's copies
            mbar_arrive(cbar);
          }
          if (!ready) break;
          tmem_wait_st();
          // Each owner thread counts itself past the flag (128 -> 256); the
          // last one resets it to 0 for the next launch, so no owner thread
          // still polling can see it drop below 128.
          for (int slot = 0; slot < g.ncontrib; ++slot) {
            int* f = &sp.flags[sk_tile * sp.max_slots + slot];
            if (atomicAdd(f, 1) == 255) atomicExch(f, 0);
          }
        }
        uint4* wst = epi_stage + (warp - 2) * (EPI_STAGE_BYTES / 16);
        bool staged = false;
        if constexpr (stages_tile<Epi>::value) {
          if (!si.more(shape)) {
            // The last segment: the ring is idle (no loads follow, the
            // accumulator is complete).  After an owner's combine, wait until
            // every thread is done with the partials' second round.
            const int et = static_cast<int>(threadIdx.x) - 64;
            const float* src = nullptr;
            uint32_t bytes = 0;
            if (Epi::tile_src(ep, shape, m0 + et, n0, src, bytes)) {
              if (g.kind == kSegOwner && !mbar_wait(cbar, static_cast<uint32_t>((C::ROUNDS - 1) & 1))) {
                fail_wait();
                break;
              }
              mbar_arrive_expect_tx(xbar, bytes);
              if (bytes != 0) bulk_g2s(smem + et * (TBN * sizeof(float)), src, bytes, xbar);
              if (!mbar_wait(xbar, 0u)) {
                fail_wait();
                break;
              }
              Epi::apply_staged(ep, shape, taddr, m0, n0, quarter, lane, wst, reinterpret_cast<const float*>(smem));
              staged = true;
            }
          }
        }
        if (!staged) Epi::apply(ep, shape, taddr, m0, n0, quarter, lane, wst);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  // Roles ran on one lane of warps 0 and 1: reconverge each warp before the
  // CTA barrier; warp 1 frees TMEM only once the epilogue warps have arrived.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// --------------------------------------------------------------- epilogues
//
// Epilogue warps read TMEM one row per thread (tcgen05.ld 32x32b).  Writing
// rows straight to row-major memory would make every warp instruction touch
// 32 different rows; instead each warp stages 32 rows x 128 bytes in its own
// shared-memory slice (16-byte units XOR-swizzled by row, conflict-free) and
// reads it back transposed, so 8 lanes cover one row's 128-byte line and a
// warp instruction moves 4 whole lines.

// Row `lane`'s 16-byte unit q -> stage; unit q of row `row` <- stage.
__device__ __forceinline__ void stage_put(uint4* st, int lane, int q, uint4 v) { st[lane * 8 + (q ^ (lane & 7))] = v; }
__device__ __forceinline__ uint4 stage_get(const uint4* st, int row, int q) { return st[row * 8 + (q ^ (row & 7))]; }

__device__ __forceinline__ uint4 f4_as_u4(float a, float b, float c, float d) {
  return make_uint4(__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d));
}

// Stage 64 bf16 per row (8 x 16 B) and store them row-major: out + row * ld
// + col0, columns [col0, col0 + valid) of rows [row0, row0 + 32) below M.
__device__ __forceinline__ void store_bf16_rows(uint4* st, int lane, const uint32_t (&w)[32], __nv_bfloat16* out,
                                                int64_t ld, int row0, int M, int col0, int valid) {
#pragma unroll
  for (int q = 0; q < 8; ++q) stage_put(st, lane, q, make_uint4(w[q * 4], w[q * 4 + 1], w[q * 4 + 2], w[q * 4 + 3]));
  __syncwarp();
  const int q = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = i * 4 + (lane >> 3);
    const int row = row0 + rr;
    const uint4 v = stage_get(st, rr, q);
    if (row < M && q * 8 < valid)
      *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * ld + col0 + q * 8) = v;
  }
  __syncwarp();
}

// C (bf16, row stride ldc) = acc
struct EpiStoreBf16 {
  struct Params {
    __nv_bfloat16* out;
    int64_t ldo;
    int32_t* status;
  };
  static __device__ __forceinline__ void apply(const Params& p, const Shape& s, uint32_t taddr, int m0, int n0,
                                               int quarter, int lane, uint4* st) {
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      const int col = n0 + c * 64;
      if (col >= s.N) break;
      float v[64];
      sm100::tmem_ld32_nowait(taddr + c * 64, reinterpret_cast<uint32_t*>(v));
      sm100::tmem_ld32_nowait(taddr + c * 64 + 32, reinterpret_cast<uint32_t*>(v) + 32);
      sm100::tmem_wait_ld();
      uint32_t w[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) w[e] = sm100::pack_bf16x2(v[2 * e], v[2 * e + 1]);
      store_bf16_rows(st, lane, w, p.out, p.ldo, m0 + quarter * 32, s.M, col, s.N - col);
    }
  }
};

// C (fp32) = acc
struct EpiStoreF32 {
  struct Params {
    float* out;
    int64_t ldo;
    int32_t* status;
  };
  static __device__ __forceinline__ void apply(const Params& p, const Shape& s, uint32_t taddr, int m0, int n0,
                                               int quarter, int lane, uint4* st) {
    const int row0 = m0 + quarter * 32;
    const int q = lane & 7;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int col = n0 + c * 32;
      if (col >= s.N) break;
      float v[32];
      sm100::tmem_ld32(taddr + c * 32, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) stage_put(st, lane, k, f4_as_u4(v[k * 4], v[k * 4 + 1], v[k * 4 + 2], v[k * 4 + 3]));
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = i * 4 + (lane >> 3);
        const int row = row0 + rr;
        const uint4 u = stage_get(st, rr, q);
        if (row < s.M)
          *reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(row) * p.ldo + col + q * 4) = u;
      }
      __syncwarp();
    }
  }
};

// Row scale of the RMSNorm folded into a GEMM: the producer of the GEMM's A
// operand wrote bf16(x * w) and, per row, partial sums of squares of x over
// `parts` column tiles; rstd = rsqrt(mean(x^2) + eps) multiplies the
// accumulator of the row (A = x * rstd * w up to one bf16 rounding).
struct RowNorm {
  const float* ssq;  // [rows][parts], or null: no scaling
  int parts;
  float inv_h;       // 1 / hidden
  float eps;
  __device__ __forceinline__ float rstd(int row, bool valid) const {
    if (ssq == nullptr) return 1.0f;
    if (!valid) return 0.0f;
    const float* s = ssq + static_cast<int64_t>(row) * parts;
    float t = 0.f;
    for (int i = 0; i < parts; ++i) t += s[i];
    return rsqrtf(__fmaf_rn(t, inv_h, eps));
  }
};

// Residual stream update: x (fp32) += acc.  Optional outputs, all from the
// updated x: x_bf16 = bf16(x) (the drafter's hidden state), xw = bf16(x *
// norm_w) (the next GEMM's A operand with the next RMSNorm's weight folded
// in), ssq[row][n0 / s.bn] = sum of x^2 over this tile's columns (the next
// GEMM's row scale, RowNorm).
struct EpiResidual {
  struct Params {
    float* x;
    int64_t ldx;
    __nv_bfloat16* x_bf16;  // may be null
    int64_t ldb;
    int32_t* status;
    __nv_bfloat16* xw;            // may be null
    int64_t ldw;
    const __nv_bfloat16* norm_w;  // [N] weight of the next RMSNorm (with xw)
    float* ssq;                   // may be null; [rows][ss_parts]
    int ss_parts;
  };
  static constexpr bool kStagesTile = true;
  static constexpr bool kAnyWidth = true;  // reads the tile width from the shape
  // Row `row` of the tile's x: its source and byte count (0 past M).  False
  // when x's rows are not 16-byte aligned (the epilogue then loads directly);
  // the same answer for every row of a launch.
  static __device__ __forceinline__ bool tile_src(const Params& p, const Shape& s, int row, int n0, const float*& src,
                                                  uint32_t& bytes) {
    if (((reinterpret_cast<uintptr_t>(p.x) & 15u) != 0) || (p.ldx & 3) != 0) return false;
    src = p.x + static_cast<int64_t>(row) * p.ldx + n0;
    bytes = row < s.M ? static_cast<uint32_t>(min(s.bn, s.N - n0)) * 4u : 0u;
    return true;
  }
  static __device__ __forceinline__ void apply(const Params& p, const Shape& s, uint32_t taddr, int m0, int n0,
                                               int quarter, int lane, uint4* st) {
    apply_staged(p, s, taddr, m0, n0, quarter, lane, st, nullptr);
  }
  // xs: the tile's x rows in shared memory ([BM][s.bn] fp32), or null to load
  // them from global memory.
  static __device__ __forceinline__ void apply_staged(const Params& p, const Shape& s, uint32_t taddr, int m0,
                                                      int n0, int quarter, int lane, uint4* st, const float* xs) {
    const int row0 = m0 + quarter * 32;
    const int q = lane & 7;
    float ssr[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // rows i * 4 + lane / 8, this lane's columns
#pragma unroll 1
    for (int c = 0; c < s.bn / 32; ++c) {
      const int col = n0 + c * 32;
      if (col >= s.N) break;
      float v[32];
      sm100::tmem_ld32(taddr + c * 32, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) stage_put(st, lane, k, f4_as_u4(v[k * 4], v[k * 4 + 1], v[k * 4 + 2], v[k * 4 + 3]));
      __syncwarp();
      // Lane (i, lane / 8, q) handles 4 columns of row i * 4 + lane / 8: the
      // x loads of all 8 passes go out first, then the adds and stores.
      float4 xv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = row0 + i * 4 + (lane >> 3);
        if (xs != nullptr)
          xv[i] = *reinterpret_cast<const float4*>(xs + (quarter * 32 + i * 4 + (lane >> 3)) * s.bn + c * 32 + q * 4);
        else
          xv[i] = row < s.M ? *reinterpret_cast<const float4*>(p.x + static_cast<int64_t>(row) * p.ldx + col + q * 4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = i * 4 + (lane >> 3);
        const int row = row0 + rr;
        const uint4 a = stage_get(st, rr, q);
        float4 x = xv[i];
        x.x += __uint_as_float(a.x);
        x.y += __uint_as_float(a.y);
        x.z += __uint_as_float(a.z);
        x.w += __uint_as_float(a.w);
        if (row < s.M) {
          *reinterpret_cast<float4*>(p.x + static_cast<int64_t>(row) * p.ldx + col + q * 4) = x;
          if (p.x_bf16 != nullptr)
            *reinterpret_cast<uint2*>(p.x_bf16 + static_cast<int64_t>(row) * p.ldb + col + q * 4) =
                make_uint2(sm100::pack_bf16x2(x.x, x.y), sm100::pack_bf16x2(x.z, x.w));
          if (p.xw != nullptr) {
            const uint2 wr = *reinterpret_cast<const uint2*>(p.norm_w + col + q * 4);
            const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wr.x));
            const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wr.y));
            *reinterpret_cast<uint2*>(p.xw + static_cast<int64_t>(row) * p.ldw + col + q * 4) =
                make_uint2(sm100::pack_bf16x2(x.x * w01.x, x.y * w01.y), sm100::pack_bf16x2(x.z * w23.x, x.w * w23.y));
          }
          ssr[i] += (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
        }
      }
      __syncwarp();
    }
    if (p.ssq != nullptr) {
      // the 8 lanes of a row (same lane / 8) hold its 8 column groups
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float v = ssr[i];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        const int row = row0 + i * 4 + (lane >> 3);
        if (q == 0 && row < s.M) p.ssq[static_cast<int64_t>(row) * p.ss_parts + n0 / s.bn] = v;
      }
    }
  }
};

// SwiGLU on a weight whose rows are interleaved in 128-row blocks
// [gate_0..127, up_0..127, gate_128..255, up_128..255, ...]: each 256-column
// tile holds matching gate and up columns; out[row, n0/2 + j] = silu(g_j) * u_j.
struct EpiSwiGlu {
  struct Params {
    __nv_bfloat16* out;
    int64_t ldo;
    int32_t* status;
    RowNorm rn;  // the post-attention RMSNorm's row scale (ssq null: none)
  };
  static __device__ __forceinline__ void apply(const Params& p, const Shape& s, uint32_t taddr, int m0, int n0,
                                               int quarter, int lane, uint4* st) {
    if (n0 >= s.N) return;
    const int row = m0 + quarter * 32 + lane;
    const float rs = p.rn.rstd(row, row < s.M);
#pragma unroll 1
    for (int c = 0; c < BN / 128; ++c) {  // 64 output columns per pass
      uint32_t w[32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float g[32], u[32];
        sm100::tmem_ld32_nowait(taddr + c * 64 + h * 32, reinterpret_cast<uint32_t*>(g));
        sm100::tmem_ld32_nowait(taddr + BN / 2 + c * 64 + h * 32, reinterpret_cast<uint32_t*>(u));
        sm100::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float g0 = g[2 * e] * rs, g1 = g[2 * e + 1] * rs;
          w[h * 16 + e] = sm100::pack_bf16x2(g0 / (1.0f + __expf(-g0)) * (u[2 * e] * rs),
                                             g1 / (1.0f + __expf(-g1)) * (u[2 * e + 1] * rs));
        }
      }
      store_bf16_rows(st, lane, w, p.out, p.ldo, m0 + quarter * 32, s.M, n0 / 2 + c * 64, 64);
    }
  }
};


// Stage 64 bf16 per row (8 x 16 B) and store row rr of the warp's 32 rows at
// dst(rr) (a pointer to its 64 columns, or null to skip the row); the
// transposed read-back lets 8 lanes cover one row's 128-byte line.
template <class RowPtr>
__device__ __forceinline__ void store_bf16_rows_to(uint4* st, int lane, const uint32_t (&w)[32], RowPtr dst) {
#pragma unroll
  for (int q = 0; q < 8; ++q) stage_put(st, lane, q, make_uint4(w[q * 4], w[q * 4 + 1], w[q * 4 + 2], w[q * 4 + 3]));
  __syncwarp();
  const int q = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = i * 4 + (lane >> 3);
    const uint4 v = stage_get(st, rr, q);
    __nv_bfloat16* d = dst(rr);
    if (d != nullptr) *reinterpret_cast<uint4*>(d + q * 8) = v;
  }
  __syncwarp();
}

// The q/k/v projection with the per-head work of the Qwen3 attention input
// fused in (HF Qwen3Attention: q_norm / k_norm RMSNorm over each head, then
// rotate-half RoPE at the row's position): a 256-column tile holds whole
// heads (256 % D == 0), and each epilogue thread owns one row, so the head's
// sum of squares and its rotary pairs (d, d + D/2) are in the thread's own
// accumulator columns.  Query heads go to q_out [rows, nq * D]; key and value
// heads straight to the request's KV-arena tail (arena_row[row], -1: skip).
// Angles come from the pass's rotary table rope[row][d] = (cos, sin).
template <int D>
struct EpiQkvPost {
  struct Params {
    __nv_bfloat16* q_out;
    int64_t ldq;
    __nv_bfloat16* k_plane0;     // K plane of kv head 0 of this layer
    __nv_bfloat16* v_plane0;     // V plane of kv head 0 of this layer
    int64_t plane_stride;        // elements between consecutive kv heads' planes
    const int64_t* arena_row;    // [rows]
    const float2* rope;          // [rows][D/2]
    const __nv_bfloat16* q_norm; // [D]
    const __nv_bfloat16* k_norm; // [D]
    int nq, nkv;
    float eps;
    int32_t* status;
    RowNorm rn;  // the input RMSNorm's row scale (ssq null: none)
  };
  static __device__ __forceinline__ void apply(const Params& p, const Shape& s, uint32_t taddr, int m0, int n0,
                                               int quarter, int lane, uint4* st) {
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    constexpr int HALF = D / 2;
    const int row0 = m0 + quarter * 32;
    const int row = row0 + lane;
    const bool rv = row < s.M;
    const float rs = p.rn.rstd(row, rv);
    const int heads = min(BN, s.N - n0) / D;
#pragma unroll 1
    for (int hi = 0; hi < heads; ++hi) {
      const int head = n0 / D + hi;
      const uint32_t hbase = taddr + static_cast<uint32_t>(hi * D);
      const bool is_q = head < p.nq;
      const bool is_k = !is_q && head < p.nq + p.nkv;
      // destination of row rr's columns [c0, c0 + 64) of this head
      auto dst = [&](int c0) {
        return [&, c0](int rr) -> __nv_bfloat16* {
          const int r = row0 + rr;
          if (r >= s.M) return nullptr;
          if (is_q) return p.q_out + static_cast<int64_t>(r) * p.ldq + static_cast<int64_t>(head) * D + c0;
          const int64_t ar = p.arena_row[r];
          if (ar < 0) return nullptr;
          const int kvh = is_k ? head - p.nq : head - p.nq - p.nkv;
          return (is_k ? p.k_plane0 : p.v_plane0) + static_cast<int64_t>(kvh) * p.plane_stride + ar * D + c0;
        };
      };
      if (!is_q && !is_k) {  // value head: plain copy
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          float a[32], b[32];
          sm100::tmem_ld32(hbase + c * 64, a);
          sm100::tmem_ld32(hbase + c * 64 + 32, b);
          uint32_t w[32];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            w[e] = sm100::pack_bf16x2(a[2 * e] * rs, a[2 * e + 1] * rs);
            w[16 + e] = sm100::pack_bf16x2(b[2 * e] * rs, b[2 * e + 1] * rs);
          }
          store_bf16_rows_to(st, lane, w, dst(c * 64));
        }
        continue;
      }
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float a[32];
        sm100::tmem_ld32(hbase + c * 32, a);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float v = a[e] * rs;
          ss += v * v;
        }
      }
      // head RMSNorm of the input-normed projection: scale rs, then rstd
      const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps) * rs;
      const __nv_bfloat16* wn = is_q ? p.q_norm : p.k_norm;
      const float2* rp = p.rope + static_cast<int64_t>(rv ? row : row0) * HALF;
      uint32_t lo[HALF / 2], up[HALF / 2];  // packed bf16 pairs of dims [0, D/2) and [D/2, D)
#pragma unroll
      for (int c = 0; c < HALF / 32; ++c) {
        float a[32], b[32];
        sm100::tmem_ld32(hbase + c * 32, a);
        sm100::tmem_ld32(hbase + HALF + c * 32, b);
        // The row's (cos, sin) pairs of these 32 dims as 16 float4 loads
        // issued together (one memory round trip, not one per dim pair).
        float4 cs4[16];
        const float4* rp4 = reinterpret_cast<const float4*>(rp + c * 32);
#pragma unroll
        for (int k = 0; k < 16; ++k) cs4[k] = rv ? rp4[k] : make_float4(1.f, 0.f, 1.f, 0.f);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float ra[2], rb[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int d = c * 32 + e + k;
            const float4 q4 = cs4[e / 2];
            const float2 cs = k == 0 ? make_float2(q4.x, q4.y) : make_float2(q4.z, q4.w);
            const float xa = a[e + k] * rstd * __bfloat162float(wn[d]);
            const float xb = b[e + k] * rstd * __bfloat162float(wn[d + HALF]);
            // rotate_half: out_d = x_d cos - x_{d+H} sin,  out_{d+H} = x_{d+H} cos + x_d sin
            ra[k] = xa * cs.x - xb * cs.y;
            rb[k] = xb * cs.x + xa * cs.y;
          }
          lo[c * 16 + e / 2] = sm100::pack_bf16x2(ra[0], ra[1]);
          up[c * 16 + e / 2] = sm100::pack_bf16x2(rb[0], rb[1]);
        }
      }
      if constexpr (D == 128) {
        store_bf16_rows_to(st, lane, lo, dst(0));
        store_bf16_rows_to(st, lane, up, dst(64));
      } else {
        uint32_t w[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          w[e] = lo[e];
          w[16 + e] = up[e];
        }
        store_bf16_rows_to(st, lane, w, dst(0));
      }
    }
  }
};

// LM head fused with softmax and sampling: full-vocabulary logits never reach
// HBM.  Per (row, 256-column vocab tile) the epilogue writes
// {tile max m_t, tile mass S_t = sum exp(x - m_t), tile key, tile column};
// lm_combine_kernel turns the tiles into lse[row] and the row's posterior
// token (the column of the largest key).  x = logit / T.
//
// Sampled rows (T > 0) use a two-level exact draw of softmax(x):
//   1. a Gumbel race over the tiles: key_t = m_t + log S_t + G_t, G_t =
//      -log E_t, E_t ~ Exp(1); argmax_t key_t picks tile t with probability
//      S_t e^{m_t} / sum_s S_s e^{m_s} (Gumbel-max over the tile masses);
//   2. inside the tile, column j = the first whose running sum of
//      exp(x - m_t) exceeds U * S_t (inverse CDF), drawn whether or not the
//      tile wins, so no second pass over the vocabulary is needed.
// P(j) = (S_t e^{m_t} / Z) (e^{x_j - m_t} / S_t) = e^{x_j} / Z: the law of
// softmax(x), the law of the reference's per-row multinomial
// (sampling.py:29-42, 903-950).  Both draws come from one Philox4x32-10 call
// keyed by the seed with counter (tile, node, request lo, 0x80000000 |
// request hi), a stream disjoint from the acceptance walk's (whose 4th
// counter word is 0): words (x, y) give E_t from 64 bits, word z the 24-bit
// uniform U.  E_t keeps full fp32 relative precision near 0, where the
// winning keys come from (exp_variate), so near-ties between tiles resolve
// to within fp32 rounding of the keys, ~1e-6.
// Greedy rows (T = 0, the reference's argmax verifier over bf16 logits,
// continuous_tree_block_decode.py:45-71, 1809-1811): key = bf16(logit),
// column = first maximum, mass terms at T = 1 (lse of the raw logits).
__host__ __device__ __forceinline__ float exp_variate(uint64_t w) {
  // V = (2k + 1) / 2^53 with k = w >> 12, a uniform in (0, 1); E = -ln(1 - V).
  // Below 1/2, E = -log1p(-V); above, 1 - V = (2k' + 1) / 2^53 with
  // k' = 2^52 - 1 - k exactly, and E = -ln(1 - V).  Both operands are exact
  // up to one fp32 rounding of the odd integer.
  const uint64_t k = w >> 12;
  const bool low = (k >> 51) == 0ull;
  const uint64_t kk = low ? k : ((1ull << 52) - 1ull) - k;
#ifdef __CUDA_ARCH__
  const float v = __ull2float_rn(2ull * kk + 1ull) * 0x1p-53f;
#else
  const float v = static_cast<float>(2ull * kk + 1ull) * 0x1p-53f;
#endif
  return low ? -log1pf(-v) : -logf(v);
}

__device__ __forceinline__ float lm_tile_weight(float v, float inv_temp, float m) {
  return __expf(__fsub_rn(__fmul_rn(v, inv_temp), m));
}

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

struct EpiLmHead {
  struct Params {
    float4* partials;          // [rows, n_tiles]
    int n_tiles;
    const int32_t* row_local;  // [rows] node index within the tree
    const int64_t* row_request;// [rows] request key
    uint64_t seed;
    float inv_temp;            // 1 / T (1 for greedy rows)
    int greedy;                // 1: argmax of bf16 logits
    int32_t* status;
    RowNorm rn;                // the final RMSNorm's row scale (ssq null: none)
  };
  static __device__ __forceinline__ void apply(const Params& p, const Shape& s, uint32_t taddr, int m0, int n0,
                                               int quarter, int lane, uint4*) {
    constexpr int kChunks = BN / 32;
    const int row = m0 + quarter * 32 + lane;
    const bool rv = row < s.M;
    const int nch = min(BN, s.N - n0) / 32;  // N % 32 == 0; uniform over the CTA
    // logit = rstd * acc; x = logit / T = acc * xs (one rounded factor for every pass)
    const float rs = p.rn.rstd(row, rv);
    const float xs = __fmul_rn(rs, p.inv_temp);
    // pass 1: tile max of x = logit / T (greedy: first maximum of bf16(logit))
    float m = -INFINITY, gbest = -INFINITY;
    int gcol = n0;
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      float v[32];
      sm100::tmem_ld32(taddr + c * 32, v);
      if (p.greedy) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          m = fmaxf(m, __fmul_rn(v[e], xs));
          const float b = bf16_round(__fmul_rn(v[e], rs));
          if (b > gbest) {
            gbest = b;
            gcol = n0 + c * 32 + e;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) m = fmaxf(m, __fmul_rn(v[e], xs));
      }
    }
    // pass 2: per-chunk masses with the tile max (sequential fp32 sums)
    float cs[kChunks];
    float S = 0.f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      cs[c] = 0.f;
      if (c < nch) {
        float v[32];
        sm100::tmem_ld32(taddr + c * 32, v);
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) a = __fadd_rn(a, lm_tile_weight(v[e], xs, m));
        cs[c] = a;
        S = __fadd_rn(S, a);
      }
    }
    float key = gbest;
    int col = gcol;
    if (!p.greedy) {
      const uint32_t node = rv ? static_cast<uint32_t>(p.row_local[row]) : 0u;
      const uint64_t req = rv ? static_cast<uint64_t>(p.row_request[row]) : 0ull;
      const U32x4 r = philox4x32_10(U32x4{static_cast<uint32_t>(n0 / BN), node, static_cast<uint32_t>(req),
                                          0x80000000u | (static_cast<uint32_t>(req >> 32) & 0x7fffffffu)},
                                    static_cast<uint32_t>(p.seed), static_cast<uint32_t>(p.seed >> 32));
      const float E = exp_variate((static_cast<uint64_t>(r.y) << 32) | r.x);
      key = __fsub_rn(__fadd_rn(m, logf(S)), logf(E));
      const float thr = __fmul_rn((static_cast<float>(r.z >> 8) + 0.5f) * (1.0f / 16777216.0f), S);
      // chunk holding the crossing: the first c with base_c + cs[c] > thr
      float base = 0.f;
      int kc = -1;
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        if (kc < 0 && c < nch) {
          const float nb = __fadd_rn(base, cs[c]);
          if (thr < nb)
            kc = c;
          else
            base = nb;
        }
      }
      col = -1;
      if (kc < 0) {  // rounding left thr at the total: the last column (the reference's V - 1 rule)
        kc = nch;
        col = n0 + nch * 32 - 1;
      }
      // pass 3: the crossing inside chunk kc.  Each chunk's running sum
      // repeats pass 2's operations in the same order, so at the chunk's end
      // base + a equals nb > thr: the crossing always lies inside it.  TMEM
      // loads are warp-wide, so the warp walks the range of its lanes' chunks.
      const int c_lo = __reduce_min_sync(0xffffffffu, kc);
      const int c_hi = min(__reduce_max_sync(0xffffffffu, kc), nch - 1);
#pragma unroll 1
      for (int c = c_lo; c <= c_hi; ++c) {
        float v[32];
        sm100::tmem_ld32(taddr + c * 32, v);
        if (c == kc) {
          float a = 0.f;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            a = __fadd_rn(a, lm_tile_weight(v[e], xs, m));
            if (col < 0 && thr < __fadd_rn(base, a)) col = n0 + c * 32 + e;
          }
          if (col < 0) col = n0 + c * 32 + 31;
        }
      }
    }
    if (rv) p.partials[static_cast<int64_t>(row) * p.n_tiles + n0 / BN] = make_float4(m, S, key, __int_as_float(col));
  }
};

// Host launcher: persistent grid of min(tiles, SMs) CTAs.
template <class E, class = void>
struct any_width : std::false_type {};
template <class E>
struct any_width<E, std::void_t<decltype(E::kAnyWidth)>> : std::bool_constant<E::kAnyWidth> {};

// Launch with tile width TBN; shape_in must come from make_shape(..., TBN)
// and the B tensor map's box must be {BK, TBN}.
template <class Epi, int TBN = BN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Shape& shape_in, const typename Epi::Params& ep,
           cudaStream_t stream, const SplitWorkspace* split = nullptr) {
  static_assert(TBN == BN || any_width<Epi>::value, "this epilogue assumes 256-column tiles");
  if (shape_in.bn != TBN) return fail(SG_ERR_INVALID_ARGUMENT, "gemm: shape planned for another tile width");
  // Devices on which this instantiation's shared-memory limit is raised.
  // Setting it twice (two host threads racing on the first call) is harmless.
  static std::atomic<uint64_t> configured_devices{0};
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(SG_ERR_UNSUPPORTED, "gemm: device index >= 64");
  const uint64_t bit = 1ull << dev;
  if (!(configured_devices.load(std::memory_order_acquire) & bit)) {
    SG_CUDA_CHECK(cudaFuncSetAttribute(gemm_kernel<Epi, TBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg<TBN>::SMEM_BYTES)));
    configured_devices.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int sms = device_sm_count();
  Shape shape = shape_in;
  plan_split(shape, sms, split);
  int grid = shape.tiles < sms ? shape.tiles : sms;
  if (shape.sp.sk_ctas > grid) grid = shape.sp.sk_ctas;
  if (grid <= 0) return SG_OK;
  return launch_pdl("gemm_kernel", gemm_kernel<Epi, TBN>, dim3(grid), dim3(THREADS), Cfg<TBN>::SMEM_BYTES, stream, ta,
                    tb, shape, ep);
}

}  // namespace gemm
}  // namespace sg
