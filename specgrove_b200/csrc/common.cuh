// Shared device/host helpers for the specgrove_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "specgrove_b200.h"

namespace sg {

// ---------------------------------------------------------------------------
// Host-side error plumbing: a thread-local detail string and a launch counter.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void count_launch(uint64_t n = 1);

inline int fail(int status, const char* what) {
  set_error("%s", what);
  return status;
}

inline int check_launch(const char* kernel) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("%s launch failed: %s", kernel, cudaGetErrorString(err));
    return SG_ERR_CUDA;
  }
  count_launch();
  return SG_OK;
}

#define SG_CUDA_CHECK(call)                                                  \
  do {                                                                       \
    cudaError_t err_ = (call);                                               \
    if (err_ != cudaSuccess) {                                               \
      ::sg::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,             \
                      cudaGetErrorString(err_));                             \
      return SG_ERR_CUDA;                                                    \
    }                                                                        \
  } while (0)

int device_sm_count();

// Largest CUDA device index + 1 that the per-device caches of this library
// (kernel attributes, static scratch addresses) handle.
constexpr int kMaxDevices = 64;

// Raises `kernel`'s dynamic shared-memory limit on the current device to at
// least `bytes`, calling cudaFuncSetAttribute only when the recorded limit
// (limits[device], one array per kernel) is lower; so repeated launches (and
// launches inside CUDA graph capture) make no attribute call.
template <typename Kernel>
int ensure_dynamic_smem(Kernel kernel, size_t bytes, std::atomic<int>* limits) {
  int dev = 0;
  SG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(SG_ERR_UNSUPPORTED, "device index beyond the per-device caches");
  const int want = static_cast<int>(bytes);
  if (limits[dev].load(std::memory_order_acquire) >= want) return SG_OK;
  SG_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want));
  int cur = limits[dev].load(std::memory_order_relaxed);
  while (cur < want && !limits[dev].compare_exchange_weak(cur, want, std::memory_order_acq_rel)) {
  }
  return SG_OK;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the previous kernel in the stream is still finishing: it triggers its
// own dependents at entry (pdl_trigger), does setup that touches no global
// data (barrier init, TMEM allocation, tensor-map prefetch), then calls
// pdl_wait before its first global read, which returns once every preceding
// kernel has completed and its writes are visible.  In a kernel launched
// without the attribute both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() {
#ifdef __CUDA_ARCH__
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_wait() {
#ifdef __CUDA_ARCH__
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

bool pdl_enabled();  // SG_PDL=0 disables programmatic dependent launch

// L2 residency window: while set (on this host thread), every launch_pdl
// kernel marks its accesses to [base, base + bytes) as persisting in L2 (the
// rest of the window's misses stream), so a buffer that each layer reads and
// writes survives the layer's weight and K/V streams in the L2 set-aside.
struct L2Window {
  const void* base = nullptr;
  size_t bytes = 0;
  float hit_ratio = 0.f;
};
L2Window& l2_window();

template <typename... Params, typename... Args>
int launch_pdl(const char* name, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  const L2Window& win = l2_window();
  if (win.bytes != 0) {
    attr[n].id = cudaLaunchAttributeAccessPolicyWindow;
    attr[n].val.accessPolicyWindow.base_ptr = const_cast<void*>(win.base);
    attr[n].val.accessPolicyWindow.num_bytes = win.bytes;
    attr[n].val.accessPolicyWindow.hitRatio = win.hit_ratio;
    attr[n].val.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
    attr[n].val.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
  if (err != cudaSuccess) {
    set_error("%s launch failed: %s", name, cudaGetErrorString(err));
    return SG_ERR_CUDA;
  }
  return check_launch(name);
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// ---------------------------------------------------------------------------
// Exact probability mass: unsigned 64.64 fixed point held in two 64-bit limbs.
//
// Every fp32 value p in [0, 2^40) becomes floor(p * 2^64) — exact for all
// normal values >= 2^-40 and truncated below — and sums of such values are
// exact integers, so prefix sums and totals do not depend on the reduction
// order.  The GPU kernels and the CPU oracle therefore make bit-identical
// inverse-CDF decisions whatever their thread counts or cluster sizes.
// ---------------------------------------------------------------------------
struct Mass {
  uint64_t lo, hi;
};

__host__ __device__ __forceinline__ Mass mass_zero() { return Mass{0ull, 0ull}; }

__host__ __device__ __forceinline__ Mass mass_add(Mass a, Mass b) {
  Mass r;
  r.lo = a.lo + b.lo;
  r.hi = a.hi + b.hi + (r.lo < a.lo ? 1ull : 0ull);
  return r;
}

__host__ __device__ __forceinline__ Mass mass_sub(Mass a, Mass b) {
  Mass r;
  r.lo = a.lo - b.lo;
  r.hi = a.hi - b.hi - (a.lo < b.lo ? 1ull : 0ull);
  return r;
}

__host__ __device__ __forceinline__ bool mass_lt(Mass a, Mass b) {
  return a.hi < b.hi || (a.hi == b.hi && a.lo < b.lo);
}

__host__ __device__ __forceinline__ bool mass_is_zero(Mass a) {
  return (a.lo | a.hi) == 0ull;
}

// fp32 bit pattern -> 64.64 mass.  Sets *bad for negative (other than -0.0),
// non-finite or >= 2^40 inputs and returns zero for them.
__host__ __device__ __forceinline__ Mass mass_from_bits(uint32_t bits, uint32_t* bad) {
  if ((bits & 0x7fffffffu) == 0u) return mass_zero();  // +0.0 and -0.0
  const uint32_t e = (bits >> 23) & 0xffu;
  if ((bits >> 31) != 0u || e >= 167u) {  // negative, inf/nan, or >= 2^40
    *bad = 1u;
    return mass_zero();
  }
  uint64_t m = bits & 0x7fffffu;
  int eff = 1;
  if (e != 0u) {
    m |= 0x800000ull;
    eff = static_cast<int>(e);
  }
  // value = m * 2^(eff - 150); mass = value * 2^64 = m * 2^(eff - 86)
  const int s = eff - 86;
  Mass r;
  if (s >= 0) {
    r.lo = (s < 64) ? (m << s) : 0ull;
    r.hi = (s == 0) ? 0ull : ((s < 64) ? (m >> (64 - s)) : (m << (s - 64)));
  } else {
    r.lo = (-s < 64) ? (m >> (-s)) : 0ull;
    r.hi = 0ull;
  }
  return r;
}

// floor(p * 2^64) of a non-negative fp32 p below 1.0 (bit pattern below
// 0x3f800000): the low word of its 64.64 mass, whose high word is zero.  Equal
// to mass_from_bits on every such input (checked exhaustively).
__host__ __device__ __forceinline__ uint64_t mass_lo_below_one(uint32_t bits) {
  const uint32_t e = bits >> 23;  // 0 .. 126
  const uint32_t m = (bits & 0x7fffffu) | (e != 0u ? 0x800000u : 0u);
  const int s = static_cast<int>(e != 0u ? e : 1u) - 86;  // mass = m * 2^s
  if (s >= 0) return static_cast<uint64_t>(m) << s;       // s <= 40
  const int r = -s;
  return r < 32 ? static_cast<uint64_t>(m >> r) : 0ull;   // m < 2^24
}

#ifdef __CUDACC__
// Same value on the device in four instructions: the fp32 bits shifted left
// by 29 plus 960 << 52 are exactly the fp64 bit pattern of p * 2^64 (the
// exponent rebased from 127 to 1023 + 64; fp32 denormals land below 1), and
// the truncating conversion to an unsigned 64-bit integer is the floor.
// Equal to mass_lo_below_one on every input below 1.0 (checked exhaustively).
__device__ __forceinline__ uint64_t mass_lo_f64(uint32_t bits) {
  const uint64_t d = (static_cast<uint64_t>(bits) << 29) + 0x3C00000000000000ull;
  return __double2ull_rz(__longlong_as_double(static_cast<long long>(d)));
}

// (lo, carry) += v as one carry chain.
__device__ __forceinline__ void add_with_carry(uint64_t& lo, uint32_t& carry, uint64_t v) {
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u32 %1, %1, 0;" : "+l"(lo), "+r"(carry) : "l"(v));
}
#endif

// Exact running sum of fp32 masses: probabilities below 1 take the one-word
// path (low word plus a carry count in the high word); anything else goes
// through mass_from_bits.
__host__ __device__ __forceinline__ void mass_accumulate(Mass& acc, uint32_t bits, uint32_t* bad) {
  if (bits < 0x3f800000u) {
#ifdef __CUDA_ARCH__
    const uint64_t v = mass_lo_f64(bits);
#else
    const uint64_t v = mass_lo_below_one(bits);
#endif
    acc.lo += v;
    acc.hi += (acc.lo < v) ? 1ull : 0ull;
  } else {
    acc = mass_add(acc, mass_from_bits(bits, bad));
  }
}

// The mass's value (an integer: p * 2^64 units) as the nearest double: the
// top 64 significant bits with the rest folded into a sticky low bit, one
// round-to-nearest conversion, then an exact power-of-two scale.
__host__ __device__ __forceinline__ double mass_to_double(Mass m) {
#ifdef __CUDA_ARCH__
  if (m.hi == 0ull) return __ull2double_rn(m.lo);
  const int lz = __clzll(static_cast<long long>(m.hi));
#else
  if (m.hi == 0ull) return static_cast<double>(m.lo);
  const int lz = __builtin_clzll(m.hi);
#endif
  const uint64_t top = lz != 0 ? (m.hi << lz) | (m.lo >> (64 - lz)) : m.hi;
  const uint64_t rest = lz != 0 ? (m.lo << lz) : m.lo;
  const uint64_t v = top | (rest != 0ull ? 1ull : 0ull);
#ifdef __CUDA_ARCH__
  return ldexp(__ull2double_rn(v), 64 - lz);
#else
  return __builtin_ldexp(static_cast<double>(v), 64 - lz);
#endif
}

__host__ __device__ __forceinline__ uint64_t mul_hi64(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
  return __umul64hi(a, b);
#else
  return static_cast<uint64_t>((static_cast<unsigned __int128>(a) * b) >> 64);
#endif
}

// floor(u * total) for a double u in [0, 1), computed exactly.
__host__ __device__ __forceinline__ Mass mass_scale(double u, Mass total) {
  uint64_t bits;
#ifdef __CUDA_ARCH__
  bits = static_cast<uint64_t>(__double_as_longlong(u));
#else
  __builtin_memcpy(&bits, &u, sizeof(bits));
#endif
  const uint64_t e = (bits >> 52) & 0x7ffull;
  uint64_t m = bits & ((1ull << 52) - 1ull);
  int shift;  // u = m * 2^-shift
  if (e == 0ull) {
    shift = 1074;
  } else {
    m |= (1ull << 52);
    shift = 1075 - static_cast<int>(e);
  }
  if (m == 0ull || shift >= 192 + 53) return mass_zero();
  // 192-bit product total * m
  const uint64_t p0 = total.lo * m;
  const uint64_t p1a = mul_hi64(total.lo, m);
  const uint64_t q0 = total.hi * m;
  const uint64_t q1 = mul_hi64(total.hi, m);
  const uint64_t l1 = p1a + q0;
  const uint64_t l2 = q1 + (l1 < p1a ? 1ull : 0ull);
  uint64_t limb[3] = {p0, l1, l2};
  // shift right by `shift` (>= 1 for u < 1) keeping 128 bits
  Mass r = mass_zero();
  const int word = shift >> 6;
  const int bit = shift & 63;
  uint64_t w0 = 0, w1 = 0, w2 = 0;  // limbs shifted down by `word` words
  if (word == 0) { w0 = limb[0]; w1 = limb[1]; w2 = limb[2]; }
  else if (word == 1) { w0 = limb[1]; w1 = limb[2]; }
  else if (word == 2) { w0 = limb[2]; }
  if (bit == 0) {
    r.lo = w0;
    r.hi = w1;
  } else {
    r.lo = (w0 >> bit) | (w1 << (64 - bit));
    r.hi = (w1 >> bit) | (w2 << (64 - bit));
  }
  return r;
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011), the published counter-based generator.
// ---------------------------------------------------------------------------
struct U32x4 {
  uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ U32x4 philox4x32_10(U32x4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    if (round > 0) {
      k0 += W0;
      k1 += W1;
    }
    const uint64_t p0 = static_cast<uint64_t>(M0) * ctr.x;
    const uint64_t p1 = static_cast<uint64_t>(M1) * ctr.z;
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    U32x4 next;
    next.x = hi1 ^ ctr.y ^ k0;
    next.y = lo1;
    next.z = hi0 ^ ctr.w ^ k1;
    next.w = lo0;
    ctr = next;
  }
  return ctr;
}

__host__ __device__ __forceinline__ double uniform53(uint32_t a, uint32_t b) {
  const uint64_t v = (static_cast<uint64_t>(b) << 32) | a;
  return static_cast<double>(v >> 11) * (1.0 / 9007199254740992.0);
}

// The two uniforms of one tree node: counter (node, request lo, request hi, 0),
// key = seed.  u.x drives the scan / routing draw, u.y the sparse-exit draw.
struct NodeUniforms {
  double route, exit;
};

__host__ __device__ __forceinline__ NodeUniforms node_uniforms(uint64_t seed, uint64_t request,
                                                               uint32_t node) {
  U32x4 c{node, static_cast<uint32_t>(request), static_cast<uint32_t>(request >> 32), 0u};
  U32x4 r = philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  return NodeUniforms{uniform53(r.x, r.y), uniform53(r.z, r.w)};
}

}  // namespace sg
