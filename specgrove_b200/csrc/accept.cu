// Tree-sampling acceptance over packed fp32 probability rows (sm_100a).
//
// One thread-block cluster (up to 8 CTAs) walks one request tree top-down;
// the cluster size is the largest for which every tree's cluster is resident
// at once.  At each visited node the cluster's CTAs split the node's
// probability row into 1024-token blocks.  Each CTA streams its slice through
// a ring of 4 KB shared-memory slots filled by bulk asynchronous copies
// (cp.async.bulk completing on an mbarrier, no multicast); the warp that owns
// a slot waits for it, reduces the block to an exact 64.64 fixed-point mass
// and refills the slot, so a CTA keeps 48 KB of the row in flight without
// holding it in registers.  Block masses are double-buffered by pass, so one
// cluster barrier per visited node suffices: after it, warp 0 of every CTA
// reads the slice totals and the owning CTA's block masses through
// distributed shared memory, finds the crossing block, rescans it in index
// order (lane sums, then the crossing lane's 32 tokens spread over the warp)
// and reaches the same token and child as every other CTA of the cluster.
//
// Semantics follow the reference kernels
//   fused_tree_sampling.py:538-627 (scan rule: token = first index whose
//   inclusive prefix exceeds u[depth] * row_total; fallback V-1; stop when no
//   child matches or depth == max_depth), and
//   fused_tree_sampling.py:688-824 (sparse exit: route among children by
//   cumulative child mass against u[2d]; on exit draw from the row without the
//   children against u[2d+1]; fallback = last non-child token),
// with the fp64 running sums replaced by exact fixed-point sums so that the
// decision is independent of the reduction order.
#include <cooperative_groups.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace cg = cooperative_groups;

namespace sg {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kMinCtasPerSm = 4;
constexpr int kBlockElems = 1024;  // one warp x 8 float4 per lane
constexpr int kBlockBytes = kBlockElems * 4;
constexpr int kVecs = kBlockElems / 128;  // float4 per lane per block
constexpr int kSlots = 12;                // ring of 4 KB slots per CTA (48 KB), 3 per warp
constexpr int kMaxChildren = 256;
constexpr int kMaxCluster = 8;
// Block i of a slice goes to slot i % kSlots and is reduced by warp
// i % kWarps.  With kSlots a multiple of kWarps every slot has one owner
// warp, which both waits for each of its fills and issues the next one, so a
// slot's barrier is never more than the one awaited phase ahead of its
// waiter (a parity wait cannot tell phase k from phase k - 2).
static_assert(kSlots % kWarps == 0, "each ring slot must belong to exactly one warp");

struct AcceptParams {
  const float* probs;
  int64_t vocab;
  const int64_t* row_offsets;
  const int64_t* parents;
  const int64_t* tokens;
  int32_t num_trees;
  int32_t max_nodes;
  int32_t max_depth;
  int32_t rule;
  const double* uniforms;
  int32_t uniform_stride;
  uint64_t seed;
  const int64_t* request_ids;
  int64_t* out;
  int32_t* status;
  int32_t blocks_per_cta;  // 1024-token blocks per CTA slice
  bool aligned4;           // rows 16-byte aligned and vocab % 4 == 0
};

__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status != nullptr) atomicMax(status, code);
}

// General path for a float4 with a value >= 1, negative or not finite (rare
// in probability rows), kept out of line so the common path stays short.
__device__ __noinline__ void accumulate4_general(Mass& big, uint4 v, uint32_t* bad) {
  big = mass_add(big, mass_from_bits(v.x, bad));
  big = mass_add(big, mass_from_bits(v.y, bad));
  big = mass_add(big, mass_from_bits(v.z, bad));
  big = mass_add(big, mass_from_bits(v.w, bad));
}

// Exact masses of four fp32 values into (lo, carry) — all four below 1.0 —
// or into `big` through the general path.
__device__ __forceinline__ void accumulate4(uint64_t& lo, uint32_t& carry, Mass& big, uint4 v, uint32_t* bad) {
  if (__builtin_expect(max(max(v.x, v.y), max(v.z, v.w)) < 0x3f800000u, 1)) {
    add_with_carry(lo, carry, mass_lo_f64(v.x));
    add_with_carry(lo, carry, mass_lo_f64(v.y));
    add_with_carry(lo, carry, mass_lo_f64(v.z));
    add_with_carry(lo, carry, mass_lo_f64(v.w));
  } else {
    accumulate4_general(big, v, bad);
  }
}

__device__ __forceinline__ Mass warp_sum(Mass v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    Mass o;
    o.lo = __shfl_xor_sync(0xffffffffu, v.lo, d);
    o.hi = __shfl_xor_sync(0xffffffffu, v.hi, d);
    v = mass_add(v, o);
  }
  return v;
}

__device__ __forceinline__ Mass warp_inclusive_scan(Mass v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    Mass o;
    o.lo = __shfl_up_sync(0xffffffffu, v.lo, d);
    o.hi = __shfl_up_sync(0xffffffffu, v.hi, d);
    if (lane >= d) v = mass_add(v, o);
  }
  return v;
}

// Four consecutive probabilities starting at `index` (zero beyond vocab).
__device__ __forceinline__ uint4 load4(const float* row, int64_t index, int64_t vocab, bool aligned4) {
  if (aligned4 && index + 3 < vocab) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(row + index));
    return make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z),
                      __float_as_uint(v.w));
  }
  uint4 r = make_uint4(0u, 0u, 0u, 0u);
  if (index + 0 < vocab) r.x = __float_as_uint(__ldg(row + index + 0));
  if (index + 1 < vocab) r.y = __float_as_uint(__ldg(row + index + 1));
  if (index + 2 < vocab) r.z = __float_as_uint(__ldg(row + index + 2));
  if (index + 3 < vocab) r.w = __float_as_uint(__ldg(row + index + 3));
  return r;
}

__device__ __forceinline__ Mass shfl_mass(Mass v, int src) {
  Mass r;
  r.lo = __shfl_sync(0xffffffffu, v.lo, src);
  r.hi = __shfl_sync(0xffffffffu, v.hi, src);
  return r;
}

// Bulk asynchronous copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) from global memory into this CTA's shared memory, completing on
// `bar` (no multicast).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm100::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

// Fill ring slot `slot` with block `b` of `row` (blocks past the end of the
// row are never issued; the row's last block may be short).
__device__ __forceinline__ void fill_slot(float* ring, uint64_t* full, int slot, const float* row,
                                          int64_t b, int64_t vocab) {
  const int64_t base = b * kBlockElems;
  const uint32_t bytes = static_cast<uint32_t>(min64(kBlockElems, vocab - base) * 4);
  sm100::mbar_arrive_expect_tx(&full[slot], bytes);
  bulk_load(ring + slot * kBlockElems, row + base, bytes, &full[slot]);
}

// Exact mass of block `gb` (global block index) of `row` read from a ring
// slot: lane l holds float4 l of each 512-byte segment.
__device__ __forceinline__ Mass slot_mass(const float* slot, int64_t gb, int64_t vocab, int lane, uint32_t* bad) {
  const float4* src = reinterpret_cast<const float4*>(slot);
  const int64_t base = gb * kBlockElems;
  // Four independent carry chains (float4 k goes to chain k % 4) keep the
  // dependent adds per lane short.
  constexpr int kChains = 4;
  uint64_t lo[kChains] = {};
  uint32_t carry[kChains] = {};
  Mass big = mass_zero();
#pragma unroll
  for (int k = 0; k < kVecs; ++k) {
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (base + k * 128 + lane * 4 < vocab) {  // vocab % 4 == 0 on this path
      const float4 f = src[k * 32 + lane];
      v = make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
    }
    accumulate4(lo[k % kChains], carry[k % kChains], big, v, bad);
  }
  Mass sum = big;
#pragma unroll
  for (int c = 0; c < kChains; ++c) sum = mass_add(sum, Mass{lo[c], carry[c]});
  return warp_sum(sum);
}

// The same mass read straight from global memory (rows that are not 16-byte
// aligned or whose vocabulary is not a multiple of 4).
__device__ __forceinline__ Mass global_mass(const float* row, int64_t gb, int64_t vocab, bool aligned4, int lane,
                                            uint32_t* bad) {
  uint4 v[kVecs];
#pragma unroll
  for (int k = 0; k < kVecs; ++k) v[k] = load4(row, gb * kBlockElems + k * 128 + lane * 4, vocab, aligned4);
  uint64_t lo = 0ull;
  uint32_t carry = 0u;
  Mass big = mass_zero();
#pragma unroll
  for (int k = 0; k < kVecs; ++k) accumulate4(lo, carry, big, v[k], bad);
  return warp_sum(mass_add(Mass{lo, carry}, big));
}

// Warp-wide: the token of block `gb` of `row` at which the running mass of
// the block first exceeds `resid` (resid < the block's mass), or -1.  Lane l
// owns the 32 consecutive tokens from gb * 1024 + 32 l; children of a
// sparse-exit node count as zero.  A scan of the lane sums picks the lane
// that holds the crossing, whose 32 values are then spread one per lane for a
// second scan, so no lane walks its tokens serially.
__device__ __forceinline__ int crossing_token(const float* row, int64_t gb, int64_t vocab, bool aligned4, Mass resid,
                                              bool sparse, const int* child_tok, int child_count, int lane,
                                              uint32_t* bad) {
  const int64_t first = gb * kBlockElems + lane * (kBlockElems / 32);
  uint32_t e[kBlockElems / 32];
#pragma unroll
  for (int k = 0; k < kBlockElems / 128; ++k) {
    const uint4 v = load4(row, first + k * 4, vocab, aligned4);
    e[4 * k] = v.x;
    e[4 * k + 1] = v.y;
    e[4 * k + 2] = v.z;
    e[4 * k + 3] = v.w;
  }
  if (sparse) {  // children are excluded from the exit draw
    for (int c = 0; c < child_count; ++c) {
      const int64_t off = child_tok[c] - first;
#pragma unroll
      for (int k = 0; k < kBlockElems / 32; ++k)
        if (off == k) e[k] = 0u;
    }
  }
  uint64_t lo = 0ull;
  uint32_t carry = 0u;
  Mass big = mass_zero();
#pragma unroll
  for (int k = 0; k < kBlockElems / 128; ++k)
    accumulate4(lo, carry, big, make_uint4(e[4 * k], e[4 * k + 1], e[4 * k + 2], e[4 * k + 3]), bad);
  const Mass lane_sum = mass_add(Mass{lo, carry}, big);
  const Mass li = warp_inclusive_scan(lane_sum, lane);
  const Mass le = mass_sub(li, lane_sum);
  const unsigned hit = __ballot_sync(0xffffffffu, !mass_lt(resid, le) && mass_lt(resid, li));
  if (hit == 0u) return -1;
  const int L = __ffs(hit) - 1;
  const Mass resid2 = mass_sub(resid, shfl_mass(le, L));
  // Lane j takes token j of lane L's run.
  uint32_t mine = 0u;
#pragma unroll
  for (int k = 0; k < kBlockElems / 32; ++k) {
    const uint32_t v = __shfl_sync(0xffffffffu, e[k], L);
    if (k == lane) mine = v;
  }
  const Mass ti = warp_inclusive_scan(mass_from_bits(mine, bad), lane);
  const unsigned hit2 = __ballot_sync(0xffffffffu, mass_lt(resid2, ti));
  if (hit2 == 0u) return -1;
  return static_cast<int>(first - lane * (kBlockElems / 32)) + L * (kBlockElems / 32) + (__ffs(hit2) - 1);
}

template <int CLUSTER, bool BULK>
__global__ void __launch_bounds__(kThreads, kMinCtasPerSm) accept_probs_kernel(const AcceptParams p) {
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned crank = cluster.block_rank();
  const int tree = static_cast<int>(blockIdx.x) / CLUSTER;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  // Dynamic shared memory: [ring: kSlots x 4 KB (BULK only)]
  // [block masses: 2 x blocks_per_cta] [parents: max_nodes] [tokens: max_nodes]
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);
  Mass* blk = reinterpret_cast<Mass*>(smem_raw + (BULK ? kSlots * kBlockBytes : 0));
  int* s_parent = reinterpret_cast<int*>(blk + 2 * p.blocks_per_cta);
  int* s_token = s_parent + p.max_nodes;

  __shared__ __align__(8) uint64_t s_full[kSlots];
  __shared__ Mass s_total[2];  // this CTA's slice total, by pass parity
  __shared__ int s_bad_tree;
  __shared__ int s_child_count;
  __shared__ int s_child_node[kMaxChildren];
  __shared__ int s_child_tok[kMaxChildren];
  __shared__ int s_sel_token;
  __shared__ int s_sel_child;

  if (BULK && tid == 0) {
    for (int s = 0; s < kSlots; ++s) sm100::mbar_init(&s_full[s], 1);
    sm100::fence_barrier_init();
  }

  const int64_t row0 = p.row_offsets[tree];
  const int n = static_cast<int>(p.row_offsets[tree + 1] - row0);
  const int D = p.max_depth;
  int64_t* out = p.out + static_cast<int64_t>(tree) * (D + 2);
  const uint64_t request = p.request_ids ? static_cast<uint64_t>(p.request_ids[tree])
                                         : static_cast<uint64_t>(tree);

  if (tid == 0) s_bad_tree = (n < 1 || n > p.max_nodes) ? 1 : 0;
  __syncthreads();
  if (s_bad_tree) {
    if (crank == 0 && tid == 0) report(p.status, SG_ERR_TREE);
    if (crank == 0)
      for (int i = tid; i < D + 2; i += kThreads) out[i] = -1;
    cluster.sync();
    return;
  }
  // Stage and validate the tree (parents[j] < j, tokens in range).
  for (int j = tid; j < n; j += kThreads) {
    const int64_t par = p.parents[row0 + j];
    const int64_t tok = p.tokens[row0 + j];
    s_parent[j] = static_cast<int>(par);
    s_token[j] = static_cast<int>(tok);
    const bool ok = (j == 0) ? (par == -1) : (par >= 0 && par < j && tok >= 0 && tok < p.vocab);
    if (!ok) atomicOr(&s_bad_tree, 1);
  }
  if (crank == 0)
    for (int i = tid; i < D + 2; i += kThreads) out[i] = -1;
  __syncthreads();
  if (s_bad_tree) {
    if (crank == 0 && tid == 0) report(p.status, SG_ERR_TREE);
    cluster.sync();
    return;
  }

  const int64_t V = p.vocab;
  const int64_t nblk_total = (V + kBlockElems - 1) / kBlockElems;
  const int64_t slice_first = static_cast<int64_t>(crank) * p.blocks_per_cta;
  const int nb = static_cast<int>(max64(0, min64(p.blocks_per_cta, nblk_total - slice_first)));

  int cur = 0;
  int accepted = 0;
  int pass = 0;  // full-row passes so far (identical in every CTA of the cluster)
  uint32_t bad_prob = 0u;
  bool wait_failed = false;
  for (int depth = 0; depth <= D; ++depth) {
    const float* row = p.probs + (row0 + cur) * V;
    double u_main, u_exit;
    if (p.uniforms != nullptr) {
      const double* ut = p.uniforms + static_cast<int64_t>(tree) * p.uniform_stride;
      if (p.rule == SG_RULE_SPARSE_EXIT) {
        u_main = ut[2 * depth];
        u_exit = ut[2 * depth + 1];
      } else {
        u_main = ut[depth];
        u_exit = 0.0;
      }
    } else {
      const NodeUniforms nu = node_uniforms(p.seed, request, static_cast<uint32_t>(cur));
      u_main = nu.route;
      u_exit = nu.exit;
    }
    if (!(u_main >= 0.0 && u_main < 1.0) || !(u_exit >= 0.0 && u_exit < 1.0)) {
      if (tid == 0 && crank == 0) report(p.status, SG_ERR_INVALID_ARGUMENT);
      u_main = (u_main >= 0.0 && u_main < 1.0) ? u_main : 0.0;
      u_exit = (u_exit >= 0.0 && u_exit < 1.0) ? u_exit : 0.0;
    }

    const bool sparse = (p.rule == SG_RULE_SPARSE_EXIT);
    if (sparse) {
      // Children of `cur` in node (edge) order.
      if (warp == 0) {
        int count = 0;
        for (int base = 1; base < n; base += 32) {
          const int j = base + lane;
          const bool hit = (j < n) && s_parent[j] == cur;
          const unsigned mask = __ballot_sync(0xffffffffu, hit);
          if (hit) {
            const int slot = count + __popc(mask & ((1u << lane) - 1u));
            if (slot < kMaxChildren) {
              s_child_node[slot] = j;
              s_child_tok[slot] = s_token[j];
            }
          }
          count += __popc(mask);
        }
        if (lane == 0) s_child_count = count;
      }
      __syncthreads();
      if (s_child_count > kMaxChildren) {
        if (tid == 0 && crank == 0) report(p.status, SG_ERR_UNSUPPORTED);
        break;
      }
      // Route: first child whose exact cumulative mass exceeds u * 1.
      int route = -1;
      {
        const Mass thr = mass_scale(u_main, Mass{0ull, 1ull});
        Mass cum = mass_zero();
        uint32_t bad = 0u;
        for (int c = 0; c < s_child_count; ++c) {
          const float v = __ldg(row + s_child_tok[c]);
          cum = mass_add(cum, mass_from_bits(__float_as_uint(v), &bad));
          if (mass_lt(thr, cum)) {
            route = s_child_node[c];
            break;
          }
        }
        bad_prob |= bad;
      }
      if (route >= 0 && depth < D) {
        if (crank == 0 && tid == 0) out[accepted] = route;
        ++accepted;
        cur = route;
        __syncthreads();
        continue;
      }
    }

    // ---- full-row pass: exact mass of every 1024-token block of this slice.
    const int buf = pass & 1;
    Mass* mb = blk + buf * p.blocks_per_cta;
    if (BULK) {
      // Slot s receives blocks s, s + kSlots, ... of the slice: `fills` per
      // pass, so the phase of its barrier for block i of pass `pass` is
      // (pass * fills + i / kSlots) & 1.  Every slot is idle here (each
      // earlier fill was consumed before the block-wide barrier that ended
      // the previous pass).  Slot s is only ever awaited and refilled by
      // warp s % kWarps, which consumes fill k before it issues fill k + 1.
      if (tid == 0)
        for (int s = 0; s < kSlots && s < nb; ++s) fill_slot(ring, s_full, s, row, slice_first + s, V);
      for (int i = warp; i < nb; i += kWarps) {
        const int s = i % kSlots;
        const int fills = (nb - s + kSlots - 1) / kSlots;
        const uint32_t parity = static_cast<uint32_t>(pass * fills + i / kSlots) & 1u;
        if (!sm100::mbar_wait(&s_full[s], parity)) wait_failed = true;
        const Mass m = slot_mass(ring + s * kBlockElems, slice_first + i, V, lane, &bad_prob);
        if (lane == 0) mb[i] = m;
        __syncwarp();
        if (lane == 0 && i + kSlots < nb) {
          sm100::fence_proxy_async_smem();  // this warp's reads of the slot precede the refill
          fill_slot(ring, s_full, s, row, slice_first + i + kSlots, V);
        }
      }
    } else {
      for (int i = warp; i < nb; i += kWarps) {
        const Mass m = global_mass(row, slice_first + i, V, p.aligned4, lane, &bad_prob);
        if (lane == 0) mb[i] = m;
      }
    }
    ++pass;
    __syncthreads();
    if (sparse) {
      if (tid == 0) {
        // Remove the children's mass from their blocks (exact subtraction).
        uint32_t bad = 0u;
        for (int c = 0; c < s_child_count; ++c) {
          const int64_t tok = s_child_tok[c];
          const int64_t b = tok / kBlockElems - slice_first;
          if (b >= 0 && b < nb) {
            const float v = __ldg(row + tok);
            mb[b] = mass_sub(mb[b], mass_from_bits(__float_as_uint(v), &bad));
          }
        }
      }
      __syncthreads();
    }
    // CTA total (warp 0; at most a few dozen blocks per slice).
    if (warp == 0) {
      Mass s = mass_zero();
      for (int b = lane; b < nb; b += 32) s = mass_add(s, mb[b]);
      s = warp_sum(s);
      if (lane == 0) s_total[buf] = s;
    }
    // The one cluster barrier of this node: every slice total and block mass
    // of this pass is visible cluster-wide after it.  Buffers of parity `buf`
    // are rewritten two passes later, after the next barrier, which no CTA
    // passes before every CTA has finished reading them below.
    cluster.sync();

    if (warp == 0) {
      // Slice totals -> grand total, owning CTA, threshold inside its slice.
      const Mass t = (lane < CLUSTER) ? *cluster.map_shared_rank(&s_total[buf], lane) : mass_zero();
      const Mass incl = warp_inclusive_scan(t, lane);
      const Mass total = shfl_mass(incl, CLUSTER - 1);
      const Mass thr = mass_scale(sparse ? u_exit : u_main, total);
      int token = -1;
      const unsigned own = __ballot_sync(0xffffffffu, lane < CLUSTER && mass_lt(thr, incl));
      if (!mass_is_zero(total) && own != 0u) {
        const int owner = __ffs(own) - 1;
        const Mass local = mass_sub(thr, shfl_mass(mass_sub(incl, t), owner));
        // The owner's block masses (distributed shared memory): lane l sums a
        // contiguous run, a warp scan locates the run and then the block that
        // holds the threshold.
        const Mass* ob = cluster.map_shared_rank(blk + buf * p.blocks_per_cta, owner);
        const int64_t o_first = static_cast<int64_t>(owner) * p.blocks_per_cta;
        const int o_nb = static_cast<int>(max64(0, min64(p.blocks_per_cta, nblk_total - o_first)));
        const int per = (o_nb + 31) / 32;
        const int b0 = min(o_nb, lane * per), b1 = min(o_nb, b0 + per);
        Mass run_sum = mass_zero();
        for (int b = b0; b < b1; ++b) run_sum = mass_add(run_sum, ob[b]);
        const Mass run_incl = warp_inclusive_scan(run_sum, lane);
        const Mass run_excl = mass_sub(run_incl, run_sum);
        const bool mine = b0 < b1 && !mass_lt(local, run_excl) && mass_lt(local, run_incl);
        int cb = -1;
        Mass resid = mass_zero();
        if (mine) {
          Mass run = run_excl;
          for (int b = b0; b < b1; ++b) {
            const Mass next = mass_add(run, ob[b]);
            if (mass_lt(local, next)) {
              cb = b;
              resid = mass_sub(local, run);
              break;
            }
            run = next;
          }
        }
        const unsigned who = __ballot_sync(0xffffffffu, mine && cb >= 0);
        if (who != 0u) {
          const int src_lane = __ffs(who) - 1;
          cb = __shfl_sync(0xffffffffu, cb, src_lane);
          resid = shfl_mass(resid, src_lane);
          uint32_t bad = 0u;
          token = crossing_token(row, o_first + cb, V, p.aligned4, resid, sparse, s_child_tok, s_child_count,
                                 lane, &bad);
        }
      }
      if (token < 0) {
        // Zero total (or a final boundary): reference fallbacks.
        if (!sparse) {
          token = static_cast<int>(V - 1);
        } else {
          for (int64_t t2 = V - 1; t2 >= 0; --t2) {
            bool is_child = false;
            for (int c = 0; c < s_child_count; ++c) is_child = is_child || (s_child_tok[c] == t2);
            if (!is_child) {
              token = static_cast<int>(t2);
              break;
            }
          }
        }
      }
      int child = -1;
      if (!sparse) {
        // First node with (parent, token) == (cur, token).
        for (int base = 1; base < n; base += 32) {
          const int j = base + lane;
          const bool hit = (j < n) && s_parent[j] == cur && s_token[j] == token;
          const unsigned mask = __ballot_sync(0xffffffffu, hit);
          if (mask != 0u) {
            child = base + __ffs(mask) - 1;
            break;
          }
        }
      }
      if (lane == 0) {
        s_sel_token = token;
        s_sel_child = child;
      }
    }
    __syncthreads();
    const int token = s_sel_token;
    const int child = s_sel_child;
    if (child >= 0 && depth < D) {
      if (crank == 0 && tid == 0) out[accepted] = child;
      ++accepted;
      cur = child;
      continue;
    }
    if (crank == 0 && tid == 0) {
      out[D] = accepted;
      out[D + 1] = token;
    }
    break;
  }
  if (bad_prob) report(p.status, SG_ERR_PROBABILITY);
  if (wait_failed) report(p.status, SG_ERR_CUDA);
  // No CTA leaves while another may still read its shared memory.
  cluster.sync();
}

__global__ void follow_kernel(const int64_t* __restrict__ posterior, const int64_t* __restrict__ row_offsets,
                              const int64_t* __restrict__ parents, const int64_t* __restrict__ tokens,
                              int32_t num_trees, int32_t max_nodes, int32_t max_depth,
                              int64_t* __restrict__ out_all, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int tree = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tree >= num_trees) return;
  const int64_t row0 = row_offsets[tree];
  const int n = static_cast<int>(row_offsets[tree + 1] - row0);
  const int D = max_depth;
  int64_t* out = out_all + static_cast<int64_t>(tree) * (D + 2);
  for (int i = lane; i < D + 2; i += 32) out[i] = -1;
  __syncwarp();
  if (n < 1 || n > max_nodes) {
    if (lane == 0) report(status, SG_ERR_TREE);
    return;
  }
  int cur = 0, accepted = 0;
  int64_t bonus = posterior[row0];
  for (int depth = 0; depth < D; ++depth) {
    int child = -1;
    for (int base = 1; base < n; base += 32) {
      const int j = base + lane;
      const bool hit = (j < n) && parents[row0 + j] == cur && tokens[row0 + j] == bonus;
      const unsigned mask = __ballot_sync(0xffffffffu, hit);
      if (mask != 0u) {
        child = base + __ffs(mask) - 1;
        break;
      }
    }
    if (child < 0) break;
    if (lane == 0) out[accepted] = child;
    ++accepted;
    cur = child;
    bonus = posterior[row0 + cur];
  }
  if (lane == 0) {
    out[D] = accepted;
    out[D + 1] = bonus;
  }
}

template <int CLUSTER, bool BULK>
int launch_accept(const AcceptParams& p, size_t smem, cudaStream_t stream) {
  auto kernel = accept_probs_kernel<CLUSTER, BULK>;
  static std::atomic<int> limits[kMaxDevices];
  const int st = ensure_dynamic_smem(kernel, smem, limits);
  if (st != SG_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.num_trees) * CLUSTER, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CLUSTER;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SG_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, p));
  return check_launch("accept_probs_kernel");
}

template <bool BULK>
int launch_accept_cluster(int cluster, const AcceptParams& p, size_t smem, cudaStream_t s) {
  switch (cluster) {
    case 1: return launch_accept<1, BULK>(p, smem, s);
    case 2: return launch_accept<2, BULK>(p, smem, s);
    case 4: return launch_accept<4, BULK>(p, smem, s);
    default: return launch_accept<8, BULK>(p, smem, s);
  }
}

// Resident CTAs per SM of the kernel variant for `cluster` with `smem` bytes
// of dynamic shared memory (cached per variant and size).
template <bool BULK>
int resident_ctas(int cluster, size_t smem) {
  static std::mutex mu;
  static size_t cached_smem[kMaxCluster + 1] = {};
  static int cached_occ[kMaxCluster + 1] = {};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (cached_smem[cluster] == smem) return cached_occ[cluster];
  }
  int occ = 0;
  cudaError_t err = cudaSuccess;
  auto query = [&](auto kernel) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err == cudaSuccess) err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, smem);
  };
  switch (cluster) {
    case 1: query(accept_probs_kernel<1, BULK>); break;
    case 2: query(accept_probs_kernel<2, BULK>); break;
    case 4: query(accept_probs_kernel<4, BULK>); break;
    default: query(accept_probs_kernel<8, BULK>); break;
  }
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cached_smem[cluster] = smem;
  cached_occ[cluster] = occ;
  return occ;
}

size_t accept_smem(int cluster, int64_t nblk, int32_t max_nodes, bool bulk) {
  const int64_t per_cta = (nblk + cluster - 1) / cluster;
  return (bulk ? static_cast<size_t>(kSlots) * kBlockBytes : 0) + static_cast<size_t>(per_cta) * 2 * sizeof(Mass) +
         static_cast<size_t>(max_nodes) * 8;
}

// SG_ACCEPT_CLUSTER=1|2|4|8 fixes the cluster size (launch-shape sweeps).
int accept_cluster_override() {
  static const int value = [] {
    const char* env = std::getenv("SG_ACCEPT_CLUSTER");
    if (env == nullptr) return 0;
    const int v = std::atoi(env);
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
  }();
  return value;
}

}  // namespace
}  // namespace sg

extern "C" int sg_tree_accept_probs(const float* probs, int64_t vocab, const int64_t* row_offsets,
                                    const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                                    int32_t max_nodes, int32_t max_depth, int32_t rule,
                                    const double* uniforms, int32_t uniform_stride, uint64_t seed,
                                    const int64_t* request_ids, int64_t* out, int32_t* status,
                                    void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (probs == nullptr || row_offsets == nullptr || parents == nullptr || tokens == nullptr ||
      out == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: null pointer");
  if (num_trees < 0 || vocab < 1 || vocab > (int64_t(1) << 30) || max_depth < 0 ||
      max_nodes < 1 || max_nodes > (1 << 16))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: bad sizes");
  if (rule != SG_RULE_SCAN && rule != SG_RULE_SPARSE_EXIT)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: unknown rule");
  if (uniforms != nullptr) {
    const int need = (rule == SG_RULE_SCAN) ? max_depth + 1 : 2 * (max_depth + 1);
    if (uniform_stride < need)
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_accept_probs: uniforms do not cover every depth");
  }
  const int sms = device_sm_count();
  if (sms <= 0) return fail(SG_ERR_CUDA, "sg_tree_accept_probs: no CUDA device");
  const int64_t nblk = (vocab + kBlockElems - 1) / kBlockElems;
  AcceptParams p;
  p.probs = probs;
  p.vocab = vocab;
  p.row_offsets = row_offsets;
  p.parents = parents;
  p.tokens = tokens;
  p.num_trees = num_trees;
  p.max_nodes = max_nodes;
  p.max_depth = max_depth;
  p.rule = rule;
  p.uniforms = uniforms;
  p.uniform_stride = uniform_stride;
  p.seed = seed;
  p.request_ids = request_ids;
  p.out = out;
  p.status = status;
  p.aligned4 = (vocab % 4 == 0) && (reinterpret_cast<uintptr_t>(probs) % 16 == 0);
  const bool bulk = p.aligned4;
  // Cluster size: the largest power of two up to 8 (and up to the number of
  // blocks in a row) for which every tree's cluster is resident at once, so
  // that a visited row is split over as many SMs as the batch allows.
  int cluster = 1;
  const int forced = accept_cluster_override();
  if (forced > 0) {
    cluster = forced;
  } else {
    for (int c = kMaxCluster; c >= 1; c >>= 1) {
      if (c > 1 && c > nblk) continue;
      const size_t sm = accept_smem(c, nblk, max_nodes, bulk);
      if (sm > 200 * 1024) break;  // smaller clusters need even more
      const int occ = bulk ? resident_ctas<true>(c, sm) : resident_ctas<false>(c, sm);
      if (c == 1 || static_cast<int64_t>(num_trees) * c <= static_cast<int64_t>(sms) * occ) {
        cluster = c;
        break;
      }
    }
  }
  // Large vocabularies need more CTAs per row to fit the block masses.
  size_t smem = accept_smem(cluster, nblk, max_nodes, bulk);
  while (smem > 200 * 1024 && cluster < kMaxCluster) {
    cluster *= 2;
    smem = accept_smem(cluster, nblk, max_nodes, bulk);
  }
  if (smem > 200 * 1024) return fail(SG_ERR_UNSUPPORTED, "sg_tree_accept_probs: vocabulary or tree too large");
  p.blocks_per_cta = static_cast<int32_t>((nblk + cluster - 1) / cluster);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return bulk ? launch_accept_cluster<true>(cluster, p, smem, s) : launch_accept_cluster<false>(cluster, p, smem, s);
}

extern "C" int sg_tree_follow(const int64_t* posterior, const int64_t* row_offsets, const int64_t* parents,
                              const int64_t* tokens, int32_t num_trees, int32_t max_nodes,
                              int32_t max_depth, int64_t* out, int32_t* status, void* stream) {
  using namespace sg;
  if (num_trees == 0) return SG_OK;
  if (posterior == nullptr || row_offsets == nullptr || parents == nullptr || tokens == nullptr ||
      out == nullptr || num_trees < 0 || max_depth < 0 || max_nodes < 1)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_tree_follow: bad arguments");
  const int warps_per_block = 4;
  const unsigned grid = static_cast<unsigned>((num_trees + warps_per_block - 1) / warps_per_block);
  follow_kernel<<<grid, warps_per_block * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      posterior, row_offsets, parents, tokens, num_trees, max_nodes, max_depth, out, status);
  return check_launch("follow_kernel");
}
