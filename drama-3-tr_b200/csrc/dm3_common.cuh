// Shared device helpers for the drama-3 MoE / block-FP8 kernels (sm_100a only).
//
// Everything here is thin inline PTX: mbarrier + cp.async.bulk staging (TMA bulk copies
// into the issuing CTA only), gpu-scope acquire/release flags with time-bounded spins, the FP8
// mma.sync tile used for the skinny (<= 4 row) products, and the exact bf16 -> e4m3 hi/lo
// split that lets a bf16 activation be multiplied against raw e4m3 weights on the FP8 pipe.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "drama3 kernels are written for sm_100a only"
#endif

namespace dm3 {

// Status bits written into a workspace status word by kernels; the host reads them back.
enum : uint32_t {
  STATUS_OK = 0u,
  STATUS_TIMEOUT = 1u,      // a bounded wait ran out (flag, counter or mbarrier)
  STATUS_BAD_EXPERT = 2u,   // an expert id outside [0, n_experts) was skipped
};

// Upper bound of every spin in these kernels, in nanoseconds of %globaltimer: 1 s unless
// dm3_set_wait_limit_ns changed it on the device. Each translation unit holds its own copy (a
// static device variable), which set_wait_limit_here writes on the current device.
constexpr uint64_t kDefaultWaitLimitNs = 1000000000ull;
static __device__ uint64_t g_wait_limit_ns = kDefaultWaitLimitNs;
__device__ __forceinline__ uint64_t wait_limit_ns() { return g_wait_limit_ns; }
static inline cudaError_t set_wait_limit_here(uint64_t ns) {
  return cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase completes or
// about hint_ns nanoseconds pass, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// As mbar_wait, sleeping between checks (for waits that other warps' work would otherwise share
// issue slots with).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, 100000u)) {
    if (globaltimer() - t0 > wait_limit_ns()) return false;
  }
  return true;
}
// Waits for the phase with the given parity to complete; false when the time limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > wait_limit_ns()) return false;
  }
  return true;
}

// ---------------------------------------------------------------- async copies
// Bulk global->shared copy (non-tensor TMA). dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Orders prior generic-proxy accesses (seen through an acquire) before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }

// ---------------------------------------------------------------- gpu-scope flags
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acqrel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Spins until *p >= target (gpu-scope acquire); false when the time limit ran out.
__device__ __forceinline__ bool wait_geq(const uint32_t* p, uint32_t target) {
  if (ld_acquire(p) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire(p) < target) {
    if (globaltimer() - t0 > wait_limit_ns()) return false;
    __nanosleep(64);
  }
  return true;
}

// ---------------------------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- named barrier
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- FP8 tensor-core tile
// D[16x8] += A[16x32] (e4m3, row) * B[32x8] (e4m3, col), fp32 accumulate.
// Lane (g = lane/4, q = lane%4) holds A rows g and g+8 at k = {4q..4q+3, 16+4q..16+4q+3},
// B column g at the same k, and C rows g, g+8 at columns 2q, 2q+1.
// Not volatile: a pure function of its operands, so the compiler may schedule independent MMAs
// back to back.
__device__ __forceinline__ void mma_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_smem16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// ---------------------------------------------------------------- exact bf16 -> e4m3 hi/lo split
// Power-of-two prescale 2^e that maps amax into [128, 256): every bf16 value v with
// |v| >= amax * 2^-9 then splits exactly as v*2^e = hi + lo with hi, lo both e4m3.
__device__ __forceinline__ int split_exponent(float amax) {
  const uint32_t bits = __float_as_uint(amax) & 0x7fffffffu;
  const int ex = static_cast<int>(bits >> 23);
  if (bits == 0u) return 0;
  int e = 134 - ex;
  if (e > 126) e = 126;
  if (e < -126) e = -126;
  return e;
}
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float(static_cast<uint32_t>(127 + e) << 23); }

__device__ __forceinline__ uint16_t pack_e4m3x2(float lo_elem, float hi_elem) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}
__device__ __forceinline__ float2 unpack_e4m3x2(uint16_t v) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(v));
  __half2 h = *reinterpret_cast<__half2*>(&h2);
  return __half22float2(h);
}
// Splits two prescaled values into (hi pair, lo pair) of packed e4m3.
__device__ __forceinline__ void split2(float a, float b, uint16_t& hi, uint16_t& lo) {
  hi = pack_e4m3x2(a, b);
  const float2 back = unpack_e4m3x2(hi);
  lo = pack_e4m3x2(a - back.x, b - back.y);
}

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

}  // namespace dm3
