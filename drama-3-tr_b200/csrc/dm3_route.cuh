// Device helpers shared by the decode and prefill routers and activation splits (sm_100a only):
// order-preserving float keys, a warp-wide top-8 over 64-bit keys, and the exact split of 16 bf16
// values into e4m3 hi + lo bytes.
#pragma once

#include <cuda_bf16.h>

#include "dm3_common.cuh"

namespace dm3 {

// Order-preserving map of a float to an unsigned key (larger float, larger key; -0 and +0 equal).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f + 0.f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ void cswap_desc(uint64_t& a, uint64_t& b) {
  const uint64_t hi = a > b ? a : b, lo = a > b ? b : a;
  a = hi;
  b = lo;
}

// The 8 largest of 256 packed keys held 8 per lane, sorted descending; every lane ends with the
// same 8. Each lane sorts its own 8 (Batcher's 19-comparator network), then five butterfly rounds
// merge with the partner lane's list: the elementwise max of one list and the other reversed is
// the top 8 of both as a bitonic sequence, which three half-cleaner stages sort again.
__device__ __forceinline__ void warp_top8(uint64_t (&k)[8]) {
  cswap_desc(k[0], k[1]); cswap_desc(k[2], k[3]); cswap_desc(k[4], k[5]); cswap_desc(k[6], k[7]);
  cswap_desc(k[0], k[2]); cswap_desc(k[1], k[3]); cswap_desc(k[4], k[6]); cswap_desc(k[5], k[7]);
  cswap_desc(k[1], k[2]); cswap_desc(k[5], k[6]);
  cswap_desc(k[0], k[4]); cswap_desc(k[1], k[5]); cswap_desc(k[2], k[6]); cswap_desc(k[3], k[7]);
  cswap_desc(k[2], k[4]); cswap_desc(k[3], k[5]);
  cswap_desc(k[1], k[2]); cswap_desc(k[3], k[4]); cswap_desc(k[5], k[6]);
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint64_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __shfl_xor_sync(0xffffffffu, k[i], d);
#pragma unroll
    for (int i = 0; i < 8; ++i) k[i] = k[i] > o[7 - i] ? k[i] : o[7 - i];
    cswap_desc(k[0], k[4]); cswap_desc(k[1], k[5]); cswap_desc(k[2], k[6]); cswap_desc(k[3], k[7]);
    cswap_desc(k[0], k[2]); cswap_desc(k[1], k[3]); cswap_desc(k[4], k[6]); cswap_desc(k[5], k[7]);
    cswap_desc(k[0], k[1]); cswap_desc(k[2], k[3]); cswap_desc(k[4], k[5]); cswap_desc(k[6], k[7]);
  }
}

// 16 consecutive bf16 values, prescaled by sc, split exactly into e4m3 hi and lo bytes.
__device__ __forceinline__ void split16(const uint4 (&v)[2], float sc, uint4& hi, uint4& lo) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(v);
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint16_t h0, l0, h1, l1;
    split2(__bfloat162float(e[4 * i]) * sc, __bfloat162float(e[4 * i + 1]) * sc, h0, l0);
    split2(__bfloat162float(e[4 * i + 2]) * sc, __bfloat162float(e[4 * i + 3]) * sc, h1, l1);
    h[i] = h0 | (static_cast<uint32_t>(h1) << 16);
    l[i] = l0 | (static_cast<uint32_t>(l1) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ float abs_max16(const uint4 (&v)[2]) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(v);
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(__bfloat162float(e[i])));
  return m;
}

}  // namespace dm3
