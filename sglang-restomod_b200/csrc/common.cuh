// Shared device helpers for the sm_100a kernels of this library.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
// mbarrier-tracked bulk copies (the TMA engine's 1-D form), the hardware
// FP8/FP4 -> f16x2 conversions, and the m16n8k16 f16 MMA used by the
// weight-streaming decode kernels. Waits are bounded by a wall-clock limit and
// report through a device status word instead of hanging.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// Device-side error bits, OR-ed into the library's status word.
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,   // an mbarrier wait gave up (never expected)
  kDevBadExpert = 2,     // an expert id outside [0, E) reached a GEMM
  kDevBadRoute = 4,      // a route index outside the activation rows
  kDevPeerTimeout = 8,   // an expert-parallel wait on another rank gave up
};

// A wait that has not completed after this many nanoseconds records
// kDevWaitTimeout and lets the kernel return. A bulk copy finishes in
// microseconds, so two seconds only trips on a real fault.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "  selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the given phase parity (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "  selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on the given phase parity. Returns false (and sets the status
// bit) when the limit passes; the caller then stops issuing work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        if (status) atomicOr(status, kDevWaitTimeout);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------- bulk copies
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D bulk copy global -> shared through the TMA engine; completion is
// reported as transaction bytes on `bar`. Both addresses 16-byte aligned and
// `bytes` a multiple of 16 (the callers' layouts guarantee it).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 16-byte asynchronous global -> shared copy (L2 only), tracked by an
// mbarrier through cp_async_arrive_noinc below.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}

// 4-byte asynchronous global -> shared copy (through L1), tracked like
// cp_async_16.
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed.
// The barrier's expected count must include this arrival (noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while
// the previous kernel in the stream is still running. It must execute
// griddep_wait() before it reads anything that kernel wrote.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Lets the next kernel in the stream (if launched with PDL) start launching.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with programmatic stream serialization (PDL) enabled.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// --------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------ conversions
// Two E4M3 bytes (low byte -> low half) to f16x2; exact, every E4M3 value is
// an f16 value.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// Four bytes of E2M1 nibble pairs to four f16x2 (byte i -> out[i]; within a
// byte the low nibble -> the low half). Exact.
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&out)[4]) {
  asm("{\n"
      "  .reg .b8 b0, b1, b2, b3;\n"
      "  mov.b32 {b0, b1, b2, b3}, %4;\n"
      "  cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "  cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "  cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "  cvt.rn.f16x2.e2m1x2 %3, b3;\n"
      "}\n"
      : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
      : "r"(w));
}

// Eight bf16 to eight f16, each rounded to nearest even.
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 raw) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[j]);
    __half2 h = __floats2half2_rn(__low2float(b), __high2float(b));
    o[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// ------------------------------------------------------------------- MMA
// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_shared_u128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint32_t ld_shared_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
  return v;
}

// Read-only 16-byte global load kept in L1 (activations are re-read by every
// warp of a CTA).
__device__ __forceinline__ uint4 ldg_u128(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// SiLU with the fast reciprocal divide (about 2 ulp; -0 for g below -88).
__device__ __forceinline__ float silu_f32(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

}  // namespace b200
