// Expert-parallel arena shared by the prefill and decode kernels (sm_100a only), and the
// system-scope flag helpers of the NVLink exchanges.
#pragma once

#include <cstddef>
#include <cstdint>

#include "dm3_common.cuh"
#include "dm3_internal.h"

namespace dm3 {
namespace ep {

__host__ __device__ inline size_t aup(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Every rank holds one arena, mapped by all ranks (CUDA IPC over NVLink):
//   ctrl     [16] u32: the call epoch, CTA counters
//   rflag    [world] u32, rcount [world] u32: written by source rank s after its pairs for this
//            rank have landed in stage[s] (count first, then the epoch with a system-scope release)
//   retflag  [world] u32: written by destination rank d after every output row for this rank's
//            pairs has landed in ret
//   rmeta    [world][tl * K] int2: (local expert << 20 | source pair index,
//            the token's row slot in stage << 9 | x split exponent + 256)
//   stage    [world][tl * K][2][H] e4m3: the x rows (one per token and destination rank, numbered
//            in pair order), split exactly into hi + lo
//   ret      [tl * K][H] fp32: the down-projection row of each of this rank's pairs
//   redflag  [world] u32, red [2][world][2][kMaxT][H] fp32: the sharded decode layer's
//            all-reduce, rank s's routed and shared partial sums (written by s; the region of the
//            call's epoch parity, so a rank one call ahead never overwrites what is still read)
enum : int { EP_EPOCH = 0, EP_DISP_COUNT = 1, EP_DOWN_COUNT = 2, EP_RED_EPOCH = 3, EP_RED_COUNT = 4 };
struct EpLayout {
  size_t ctrl, rflag, rcount, retflag, redflag, rmeta, stage, ret, red, total;
  int slots;  // pairs per source region
};
__host__ __device__ inline EpLayout ep_layout(int world, int tl, int K, int H) {
  EpLayout A;
  A.slots = tl * K;
  size_t o = 0;
  A.ctrl = o;
  o += 64;
  A.rflag = o;
  o += 64;
  A.rcount = o;
  o += 64;
  A.retflag = o;
  o += 64;
  A.redflag = o;
  o += 64;
  A.rmeta = o = aup(o, 128);
  o += static_cast<size_t>(world) * A.slots * 8;
  A.stage = o = aup(o, 1024);
  o += static_cast<size_t>(world) * A.slots * 2 * H;
  A.ret = o = aup(o, 1024);
  o += static_cast<size_t>(A.slots) * H * 4;
  A.red = o = aup(o, 1024);
  o += static_cast<size_t>(2) * world * 2 * kMaxT * H * 4;
  A.total = aup(o, 4096);
  return A;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
// Waits (bounded) until the flag holds the epoch; false when the time limit ran out.
__device__ __forceinline__ bool wait_epoch(const uint32_t* flagp, uint32_t epoch) {
  if (ld_acquire_sys(flagp) == epoch) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_sys(flagp) != epoch) {
    if (globaltimer() - t0 > wait_limit_ns()) return false;
    __nanosleep(100);
  }
  return true;
}

}  // namespace ep
}  // namespace dm3
