// Shared device and host helpers for the bpt_b200 kernels (sm_100a only).
//
// - status codes and the thread-local error message behind bpt_last_error()
// - mbarrier + cp.async.bulk (the TMA engine's 1-D bulk copy) wrappers; every wait is bounded
// - programmatic dependent launch (PDL): griddepcontrol wrappers and a launch helper
// - small numeric helpers: bf16/fp16 loads, packed fp32x2 FMA, e4m3 conversion
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/bpt_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "bpt_b200 kernels are written for sm_100a only"
#endif

namespace bpt {

// ---- host-side status ----------------------------------------------------------------------------------------

int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
int num_sms();
int set_max_smem(const void* kernel, int bytes);
// The driver's cuTensorMapEncodeTiled (a PFN_cuTensorMapEncodeTiled_v12000), or null if the driver lacks it.
void* tensor_map_encoder();

#define BPT_REQUIRE(cond, status, ...)                 \
  do {                                                \
    if (!(cond)) return ::bpt::set_error(status, __VA_ARGS__); \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- device-side error flag ------------------------------------------------------------------------------------
// Kernels never trap. A bounded wait that runs out, or an index that fails its bounds check, records a code here
// and the kernel skips the work it cannot do; the host reads it with bpt_device_error().

extern __device__ int g_device_error;

enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrTimeout = 1,      // an mbarrier wait gave up
  kDevErrBlockIndex = 2,   // a block-table entry outside [0, num_blocks)
  kDevErrSlotIndex = 3,    // a write slot outside the block
};

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_device_error, 0, code); }

// Limits of the bounded waits: ~200 ms in normal operation (far beyond any healthy wait), ~2 ms under
// BPT_FLAG_TEST_STALL, where a test makes a wait run out on purpose.
constexpr uint64_t kWaitNs = 200000000ull;
constexpr uint64_t kTestWaitNs = 2000000ull;

// ---- PDL ---------------------------------------------------------------------------------------------------------

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---- mbarrier + bulk copy ------------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// The same test, letting the hardware suspend the thread until the phase completes or about `ns` nanoseconds
// pass, so a waiting warp does not take issue slots from the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete, for at most ~limit_ns. Returns false (and records
// kDevErrTimeout) if it gave up: the caller then skips the data that never arrived.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 200000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_suspend(bar, parity, 1000u)) return true;
    if ((i & 15u) == 0 && global_timer_ns() - start > limit_ns) {
      record_error(kDevErrTimeout);
      return false;
    }
  }
}

// The same wait for a long one (a whole tile's copies): after the first test the thread sleeps `sleep_ns`
// between tests, so waiting warps leave the issue slots to the warps that have work.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t sleep_ns,
                                                uint64_t limit_ns = 200000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15u) == 0 && global_timer_ns() - start > limit_ns) {
      record_error(kDevErrTimeout);
      return false;
    }
  }
}

// The same wait, made uniform across a warp: lane 0 spins (bounded), the verdict is broadcast, and on success
// every lane re-observes the completed phase so that each gets the barrier's acquire ordering.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 200000000ull) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, limit_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok != 0;
}

// 1-D bulk copy global -> shared through the TMA engine, completing on `bar` (complete_tx). Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 eviction hint: the data is read once (weights, KV pages), so evict it first.
__device__ __forceinline__ void bulk_g2s_evict_first(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                                     uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Orders this thread's earlier generic-proxy accesses of shared memory (and those it acquired from other threads)
// before its later async-proxy ones, e.g. reads of a ring stage before the bulk copy that overwrites it.
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 4-D tiled tensor copy global -> shared through the TMA engine with an L2 eviction hint, completing on `bar`.
// `map` is a __grid_constant__ kernel parameter; the innermost coordinate times the element size must be a multiple
// of 16 bytes.
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const void* map, int c0, int c1, int c2, int c3,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- numerics ------------------------------------------------------------------------------------------------------

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

template <int DT>
__device__ __forceinline__ float load_as_float(const void* p, int64_t i) {
  if constexpr (DT == BPT_DTYPE_F32) return static_cast<const float*>(p)[i];
  if constexpr (DT == BPT_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
  if constexpr (DT == BPT_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return 0.f;
}

template <int DT>
__device__ __forceinline__ void store_from_float(void* p, int64_t i, float v) {
  if constexpr (DT == BPT_DTYPE_F32) static_cast<float*>(p)[i] = v;
  if constexpr (DT == BPT_DTYPE_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  if constexpr (DT == BPT_DTYPE_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// d = a * b + c on two fp32 lanes at once (sm_100 packed FMA).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Two E4M3 bytes (low byte first) -> two fp32 values, exactly.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t two) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(two));
  __half2 h = *reinterpret_cast<__half2*>(&h2);
  return __half22float2(h);
}

// Two fp32 values -> two E4M3 bytes (round to nearest even, saturating to +-448), lo in the low byte.
__device__ __forceinline__ uint16_t float2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// y / b, correctly rounded, from r = RN(1 / b) (computed once per divisor, e.g. with __frcp_rn): q = RN(y * r) is
// within one ulp of y / b, and with the exact remainder e = y - q * b (one FMA), RN(q + e * r) is the correctly
// rounded quotient (Markstein's theorem; P. Markstein, IBM J. Res. Dev. 34(1), 1990; Muller et al., Handbook of
// Floating-Point Arithmetic, 2nd ed., 4.9), barring underflow of e, i.e. for quotients far above 2^-100.
__device__ __forceinline__ float div_by(float y, float b, float r) {
  const float q = __fmul_rn(y, r);
  const float e = __fmaf_rn(-q, b, y);
  return __fmaf_rn(e, r, q);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace bpt
