// Block-FP8 GEMV for B200 (sm_100a): y[M, N] = x[M, K] * dequant(q[N, K])^T (+ bias), M <= 4.
//
// A decode GEMV moves N x K weight bytes once and does 2 M flops per byte: it is bound by HBM and
// by the latency of its short dependent chain, not by arithmetic.
// * One CTA per SM owns a balanced range of output rows. A producer warp copies them, 16 rows x
//   2048 bytes of K per stage, into a shared-memory ring with cp.async.bulk (one copy per row, at a
//   padded pitch so that fragment loads are free of bank conflicts), starting before
//   griddepcontrol.wait: weights are never produced by the preceding kernel, so a chain of GEMVs
//   streams each call's weights beside the previous call.
// * After the wait, each of 8 consumer warps splits its two 128-wide K blocks (per 2048-byte chunk)
//   of the M <= 4 rows of x exactly into e4m3 hi + lo (power-of-two prescale per row and K block),
//   then multiplies the raw e4m3 weight rows by them with the FP8 mma.sync m16n8k32 (16 weight rows
//   x 8 columns: hi of rows 0-3, lo of rows 0-3): four MMAs per K block and 16 rows. (Widening every
//   weight byte e4m3 -> f16 -> f32 on the CUDA cores and using packed fp32 FMAs measured 1.6x slower
//   at 2048 x 4096: the conversions are low-throughput instructions.) Each K block's fp32 partial is
//   scaled by its block scale, as the reference Triton kernel does (fp8_linear.py:21-26).
// * When each of the CTA's 16-row tiles has its own ring slot, a tile's MMAs are issued as soon as
//   its copy lands and the scaling and sums of all tiles follow the last tile's MMAs; otherwise the
//   stages are consumed one at a time.
// * The warps' partials of a row are added in a fixed order, so results do not depend on timing.
// * A gathered row list (the audio head's rows of the full vocabulary matrix) only changes the
//   source address of each row copy.
#include "dm3_common.cuh"
#include "dm3_internal.h"

namespace dm3 {
namespace gemv {

constexpr int kWarps = 8;                    // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + the producer warp
constexpr int kTileRows = 16;
constexpr int kChunk = 2048;                 // bytes of K per stage (16 blocks: 2 per warp)
constexpr int kPitch = kChunk + 64;          // row pitch of a stage: rows g, g + 1 64 bytes apart mod 128
constexpr int kStageBytes = kTileRows * kPitch;
constexpr int kRingSlots = 3;
constexpr int kMaxRows = 64;                 // rows per CTA; larger N takes more CTAs than SMs
constexpr int kSmemBudget = 115200;          // two CTAs (this call and the next of a chain) per SM

static __device__ uint32_t g_status;

struct Params {
  const __nv_bfloat16* x;
  int M, K, N;
  const uint8_t* q;
  int64_t ldq;
  const int64_t* rows;  // optional gather list [N] (a parameter: read before griddepcontrol.wait)
  int64_t n_rows_q;
  const float* s;
  int64_t lds;
  int srows;
  const void* bias;
  int bias_kind;
  void* y;
  int64_t ldy;
  int y_fp32;
  int nch;    // 2048-byte chunks of K
  int slots;  // ring slots
  int off_sc, off_red, off_bar;
};

__device__ __forceinline__ int64_t src_row(const Params& p, int r) {
  if (p.rows == nullptr) return r;
  int64_t v = p.rows[r];
  // out-of-range indices are rejected by the host wrapper; clamp so a bad list can never fault
  if (v < 0) v = 0;
  if (v >= p.n_rows_q) v = p.n_rows_q - 1;
  return v;
}

template <int NCH>
__global__ void __launch_bounds__(kThreads, NCH <= 2 ? 2 : 1) gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + kRingSlots;
  float* sc = reinterpret_cast<float*>(smem + p.off_sc);
  float* red = reinterpret_cast<float*>(smem + p.off_red);  // [tile][warp][16 rows][4 x rows]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row_begin = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.N) / gridDim.x);
  const int row_end = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.N) / gridDim.x);
  const int R = row_end - row_begin;
  const int n_tiles = (R + kTileRows - 1) / kTileRows;
  const int n_stages = n_tiles * p.nch;
  const int nkb = p.K >> 7;

  if (tid == 0) {
    for (int i = 0; i < p.slots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch();

  if (warp == kWarps) {
    // ---------------------------------------------------------------- producer
    for (int i = 0; i < n_stages; ++i) {
      const int slot = i % p.slots;
      if (i >= p.slots) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&empty[slot], ((i / p.slots) - 1) & 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) atomicOr(&g_status, STATUS_TIMEOUT);
          break;  // the consumers are gone: nothing more can be delivered
        }
      }
      const int t = i / p.nch, c = i - t * p.nch;
      const int r0 = row_begin + t * kTileRows;
      const int nr = min(kTileRows, row_end - r0);
      const int k0 = c * kChunk;
      const int kc = min(kChunk, p.K - k0);
      uint8_t* dst = smem + slot * kStageBytes;
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nr * kc));
      __syncwarp();
      if (lane < nr) bulk_g2s(dst + lane * kPitch, p.q + src_row(p, r0 + lane) * p.ldq + k0, kc, &full[slot]);
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  // the scales of this CTA's rows (parameters, like the weights)
  for (int i = tid; i < R * nkb; i += kWarps * 32) {
    const int r = i / nkb, kb = i - r * nkb;
    sc[i] = __ldg(p.s + (src_row(p, row_begin + r) / p.srows) * p.lds + kb);
  }
  const int g = lane >> 2, q = lane & 3;
  // split x into this warp's B fragments: K blocks c * 16 + 2 * warp + i of every chunk c.
  // The split goes through this warp's 1 KB of the (not yet used) partial-sum area.
  uint8_t* xw = reinterpret_cast<uint8_t*>(red) + warp * 1024;
  griddep_wait();  // x is produced by the preceding kernel
  uint4 bfr[NCH][2][2];
  float ef[NCH][2][2];  // inverse prescale of this lane's two x rows, per K block
  {
    const bool two = p.M <= 2;
    const int m = two ? lane >> 4 : lane >> 3;       // x row this lane splits
    const int cw = two ? 8 : 16;                     // values per lane
    const int c0 = (two ? (lane & 15) : (lane & 7)) * cw;
    // every load first: one memory round trip for all of the warp's K blocks
    uint4 raw[NCH][2][2];
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int kb = c * 16 + 2 * warp + i;
        raw[c][i][0] = raw[c][i][1] = make_uint4(0u, 0u, 0u, 0u);
        if (kb < nkb && m < p.M) {
          const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(m) * p.K + kb * 128 + c0);
          raw[c][i][0] = src[0];
          if (!two) raw[c][i][1] = src[1];
        }
      }
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      uint32_t hi[2][4], lo[2][4];
      float inv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int kb = c * 16 + 2 * warp + i;
        const bool kv = kb < nkb;
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.f;
        if (kv && m < p.M) {
          const uint4 u0 = raw[c][i][0];
          const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[2 * e] = __uint_as_float(w0[e] << 16);
            v[2 * e + 1] = __uint_as_float(w0[e] & 0xffff0000u);
          }
          if (!two) {
            const uint4 u1 = raw[c][i][1];
            const uint32_t w1[4] = {u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              v[8 + 2 * e] = __uint_as_float(w1[e] << 16);
              v[8 + 2 * e + 1] = __uint_as_float(w1[e] & 0xffff0000u);
            }
          }
        }
        float amax = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
        // the lanes holding the same x row of this K block
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        if (two) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 8));
        const int ex = split_exponent(amax);
        const float pre = exp2i(ex);
        inv[i] = exp2i(-ex);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint16_t h0, l0, h1, l1;
          split2(v[4 * e] * pre, v[4 * e + 1] * pre, h0, l0);
          split2(v[4 * e + 2] * pre, v[4 * e + 3] * pre, h1, l1);
          hi[i][e] = h0 | (static_cast<uint32_t>(h1) << 16);
          lo[i][e] = l0 | (static_cast<uint32_t>(l1) << 16);
        }
      }
      // B fragment columns: m = hi of x row m, 4 + m = lo. With M <= 2 both K blocks share the
      // buffer: block i's hi and lo of x row m go to rows 2i + m and 4 + 2i + m, and lane group g
      // reads row g ^ 2i, so that columns 0, 1, 4, 5 of block i's fragment hold its x rows 0, 1. Its
      // columns 2, 3, 6, 7 then hold the other block's values: they meet zero prescale factors and
      // land in partial sums of x rows 2, 3, which are never read. With M > 2 the blocks take the
      // buffer in turn.
      const int src0 = (2 * (q & 1)) << (two ? 4 : 3), src1 = (2 * (q & 1) + 1) << (two ? 4 : 3);
      if (two) {
        __syncwarp();  // the previous chunk's fragments are loaded
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          *reinterpret_cast<uint2*>(xw + (2 * i + m) * 128 + c0) = make_uint2(hi[i][0], hi[i][1]);
          *reinterpret_cast<uint2*>(xw + (4 + 2 * i + m) * 128 + c0) = make_uint2(lo[i][0], lo[i][1]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float i0 = __shfl_sync(0xffffffffu, inv[i], src0 & 31);
          const float i1 = __shfl_sync(0xffffffffu, inv[i], src1 & 31);
          ef[c][i][0] = (q & 1) ? 0.f : i0;
          ef[c][i][1] = (q & 1) ? 0.f : i1;
          const uint8_t* row = xw + (g ^ (2 * i)) * 128 + 16 * q;
          bfr[c][i][0] = ld_smem16(row);
          bfr[c][i][1] = ld_smem16(row + 64);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          __syncwarp();
          *reinterpret_cast<uint4*>(xw + m * 128 + c0) = make_uint4(hi[i][0], hi[i][1], hi[i][2], hi[i][3]);
          *reinterpret_cast<uint4*>(xw + (4 + m) * 128 + c0) = make_uint4(lo[i][0], lo[i][1], lo[i][2], lo[i][3]);
          // inverse prescales of x rows 0-3 from the lanes that computed them
          ef[c][i][0] = __shfl_sync(0xffffffffu, inv[i], src0 & 31);
          ef[c][i][1] = __shfl_sync(0xffffffffu, inv[i], src1 & 31);
          __syncwarp();
          bfr[c][i][0] = ld_smem16(xw + g * 128 + 16 * q);
          bfr[c][i][1] = ld_smem16(xw + g * 128 + 64 + 16 * q);
        }
      }
    }
  }
  named_bar(1, kWarps * 32);  // scales visible; every warp is done with its split buffer

  bool failed = false;
  if (NCH == 1 && n_stages <= p.slots) {
    // Every tile of the CTA sits in its own ring slot (one chunk of K; all copies were issued before
    // griddepcontrol.wait). Each tile's MMAs are issued as soon as its copy has landed and the sums
    // of all tiles follow the last tile's MMAs: the tensor-core results then arrive once for the
    // whole CTA rather than once per tile, and a tile that lands late still overlaps the MMAs of
    // the tiles before it.
    bool ok = true;
    float d[kRingSlots][2][4];
#pragma unroll
    for (int t = 0; t < kRingSlots; ++t) {
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[t][j][e] = 0.f;
      if (t < n_stages && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(&full[t], 0));
        if (ok) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int kb = 2 * warp + j;
            if (kb < nkb) {
              const uint8_t* rlo = smem + t * kStageBytes + g * kPitch + kb * 128 + 16 * q;
              const uint8_t* rhi = rlo + 8 * kPitch;
              const uint4 a0 = ld_smem16(rlo), a1 = ld_smem16(rlo + 64);
              const uint4 h0 = ld_smem16(rhi), h1 = ld_smem16(rhi + 64);
              const uint4 b0 = bfr[0][j][0], b1 = bfr[0][j][1];
              mma_e4m3(d[t][j], a0.x, h0.x, a0.y, h0.y, b0.x, b0.y);
              mma_e4m3(d[t][j], a0.z, h0.z, a0.w, h0.w, b0.z, b0.w);
              mma_e4m3(d[t][j], a1.x, h1.x, a1.y, h1.y, b1.x, b1.y);
              mma_e4m3(d[t][j], a1.z, h1.z, a1.w, h1.w, b1.z, b1.w);
            }
          }
        }
      }
    }
    if (!ok) {
      if (lane == 0) atomicOr(&g_status, STATUS_TIMEOUT);
    } else {
#pragma unroll
      for (int t = 0; t < kRingSlots; ++t) {
        if (t < n_stages) {
          const int rl = min(t * kTileRows + g, R - 1), rh = min(t * kTileRows + g + 8, R - 1);
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int kb = 2 * warp + j;
            if (kb < nkb) {
              const float sl = sc[rl * nkb + kb], sh = sc[rh * nkb + kb];
              acc[0] = fmaf(d[t][j][0], sl * ef[0][j][0], acc[0]);
              acc[1] = fmaf(d[t][j][1], sl * ef[0][j][1], acc[1]);
              acc[2] = fmaf(d[t][j][2], sh * ef[0][j][0], acc[2]);
              acc[3] = fmaf(d[t][j][3], sh * ef[0][j][1], acc[3]);
            }
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 2);
          if (q < 2) {
            float* rw = red + ((t * kWarps + warp) * kTileRows) * 4;
            *reinterpret_cast<float2*>(rw + g * 4 + 2 * q) = make_float2(acc[0], acc[1]);
            *reinterpret_cast<float2*>(rw + (g + 8) * 4 + 2 * q) = make_float2(acc[2], acc[3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0)
      for (int s = 0; s < n_stages; ++s) mbar_arrive(&empty[s]);
  } else {
  for (int i = 0; i < n_stages; ++i) {
    const int slot = i % p.slots;
    if (!failed) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[slot], (i / p.slots) & 1));
      if (!ok) {
        failed = true;
        if (lane == 0) atomicOr(&g_status, STATUS_TIMEOUT);
      }
    }
    const int t = i / p.nch, c = i - t * p.nch;
    if (!failed) {
      const uint8_t* rlo = smem + slot * kStageBytes + g * kPitch;
      const uint8_t* rhi = rlo + 8 * kPitch;
      const int rl = min(t * kTileRows + g, R - 1), rh = min(t * kTileRows + g + 8, R - 1);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < NCH; ++cc) {
        if (cc != c) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int kbl = 2 * warp + j;  // K block within the chunk
          const int kb = c * 16 + kbl;
          if (kb < nkb) {
            const uint4 a0 = ld_smem16(rlo + kbl * 128 + 16 * q), a1 = ld_smem16(rlo + kbl * 128 + 64 + 16 * q);
            const uint4 h0 = ld_smem16(rhi + kbl * 128 + 16 * q), h1 = ld_smem16(rhi + kbl * 128 + 64 + 16 * q);
            const uint4 b0 = bfr[cc][j][0], b1 = bfr[cc][j][1];
            float t4[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int e = 0; e < 4; ++e) t4[u][e] = 0.f;
            mma_e4m3(t4[0], a0.x, h0.x, a0.y, h0.y, b0.x, b0.y);
            mma_e4m3(t4[1], a0.z, h0.z, a0.w, h0.w, b0.z, b0.w);
            mma_e4m3(t4[2], a1.x, h1.x, a1.y, h1.y, b1.x, b1.y);
            mma_e4m3(t4[3], a1.z, h1.z, a1.w, h1.w, b1.z, b1.w);
            const float sl = sc[rl * nkb + kb], sh = sc[rh * nkb + kb];
            const float f00 = sl * ef[cc][j][0], f01 = sl * ef[cc][j][1];
            const float f10 = sh * ef[cc][j][0], f11 = sh * ef[cc][j][1];
            acc[0] = fmaf((t4[0][0] + t4[1][0]) + (t4[2][0] + t4[3][0]), f00, acc[0]);
            acc[1] = fmaf((t4[0][1] + t4[1][1]) + (t4[2][1] + t4[3][1]), f01, acc[1]);
            acc[2] = fmaf((t4[0][2] + t4[1][2]) + (t4[2][2] + t4[3][2]), f10, acc[2]);
            acc[3] = fmaf((t4[0][3] + t4[1][3]) + (t4[2][3] + t4[3][3]), f11, acc[3]);
          }
        }
      }
      // hi (columns 2q, 2q + 1 for q < 2) + lo (the same x rows in lane q + 2)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 2);
      if (q < 2) {
        // chunk partials of a tile accumulate in place (chunks of a tile arrive in order)
        float* rw = red + ((t * kWarps + warp) * kTileRows) * 4;
        if (c == 0) {
          *reinterpret_cast<float2*>(rw + g * 4 + 2 * q) = make_float2(acc[0], acc[1]);
          *reinterpret_cast<float2*>(rw + (g + 8) * 4 + 2 * q) = make_float2(acc[2], acc[3]);
        } else {
          float2* a = reinterpret_cast<float2*>(rw + g * 4 + 2 * q);
          float2* b = reinterpret_cast<float2*>(rw + (g + 8) * 4 + 2 * q);
          *a = make_float2(a->x + acc[0], a->y + acc[1]);
          *b = make_float2(b->x + acc[2], b->y + acc[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  }
  named_bar(1, kWarps * 32);
  for (int i = tid; i < R * p.M; i += kWarps * 32) {
    const int m = i / R, r = i - m * R;
    const int t = r / kTileRows, rr = r - t * kTileRows;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[((t * kWarps + w) * kTileRows + rr) * 4 + m];
    const int n = row_begin + r;
    if (p.bias_kind == 1) v += __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
    if (p.bias_kind == 2) v += static_cast<const float*>(p.bias)[n];
    if (p.y_fp32)
      static_cast<float*>(p.y)[m * p.ldy + n] = v;
    else
      static_cast<__nv_bfloat16*>(p.y)[m * p.ldy + n] = __float2bfloat16_rn(v);
  }
}

}  // namespace gemv

// ------------------------------------------------------------------ host launcher
int launch_gemv_tc(const __nv_bfloat16* x, int M, int K, int N, const uint8_t* q, int64_t ldq, const float* s,
                   int64_t lds, int srows, const void* bias, int bias_kind, void* y, int64_t ldy, int y_fp32,
                   cudaStream_t stream);

namespace gemv {
// Grid, ring and shared-memory layout of a launch.
struct Plan {
  int grid, max_rows, nch, stages, slots, off_sc, off_red, off_bar, smem;
};
inline Plan plan_of(int K, int N, int sms) {
  Plan P{};
  P.grid = sms > (N + kMaxRows - 1) / kMaxRows ? sms : (N + kMaxRows - 1) / kMaxRows;
  if (P.grid > N) P.grid = N;
  P.max_rows = (N + P.grid - 1) / P.grid;
  const int tiles = (P.max_rows + kTileRows - 1) / kTileRows;
  P.nch = (K + kChunk - 1) / kChunk;
  P.stages = tiles * P.nch;
  const int sc_bytes = (P.max_rows * (K / 128) * 4 + 15) / 16 * 16;
  int red_bytes = tiles * kWarps * kTileRows * 4 * 4;
  if (red_bytes < kWarps * 1024) red_bytes = kWarps * 1024;  // the split buffers share it
  P.slots = kRingSlots < P.stages ? kRingSlots : P.stages;
  while (P.slots > 1 && P.slots * kStageBytes + sc_bytes + red_bytes + 2 * kRingSlots * 8 > kSmemBudget) --P.slots;
  P.off_sc = P.slots * kStageBytes;
  P.off_red = P.off_sc + sc_bytes;
  P.off_bar = P.off_red + red_bytes;
  P.smem = P.off_bar + 2 * kRingSlots * 8;
  return P;
}
}  // namespace gemv

// Every row of a CTA is one chunk of K and all of the CTA's stages fit the ring.
bool gemv_rows_fit(int K, int N, int sms) {
  const gemv::Plan P = gemv::plan_of(K, N, sms);
  return P.nch == 1 && P.stages <= P.slots;
}

namespace {
template <int NCH>
cudaError_t launch_gemv_nch(const gemv::Params& p, int grid, int smem, cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && !configured[dev]) {
    e = cudaFuncSetAttribute(gemv::gemv_kernel<NCH>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(gemv::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv::gemv_kernel<NCH>, p);
}
}  // namespace

int launch_gemv(const __nv_bfloat16* x, int M, int K, int N, const uint8_t* q, int64_t ldq, const int64_t* rows,
                int64_t n_rows_q, const float* s, int64_t lds, int srows, const void* bias, int bias_kind, void* y,
                int64_t ldy, int y_fp32, cudaStream_t stream) {
  using namespace gemv;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return 2;
  }
  const Plan P = plan_of(K, N, sm_count(dev));
  Params p{};
  p.x = x;
  p.M = M;
  p.K = K;
  p.N = N;
  p.q = q;
  p.ldq = ldq;
  p.rows = rows;
  p.n_rows_q = n_rows_q;
  p.s = s;
  p.lds = lds;
  p.srows = srows;
  p.bias = bias;
  p.bias_kind = bias_kind;
  p.y = y;
  p.ldy = ldy;
  p.y_fp32 = y_fp32;
  p.nch = P.nch;
  p.slots = P.slots;
  p.off_sc = P.off_sc;
  p.off_red = P.off_red;
  p.off_bar = P.off_bar;
  const int grid = P.grid, off = P.smem;
  cudaError_t err;
  if (p.nch == 1)
    err = launch_gemv_nch<1>(p, grid, off, stream);
  else if (p.nch == 2)
    err = launch_gemv_nch<2>(p, grid, off, stream);
  else
    err = launch_gemv_nch<4>(p, grid, off, stream);
  if (err != cudaSuccess) {
    set_error(std::string("gemv launch: ") + cudaGetErrorString(err));
    return 2;
  }
  note_launches(1);
  return 0;
}

// Reads and clears this file's status word (asynchronously on the stream).
int gemv_status_async(uint32_t* host_value, cudaStream_t stream) {
  const uint32_t zero = 0;
  if (cudaMemcpyFromSymbolAsync(host_value, gemv::g_status, 4, 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(gemv::g_status, &zero, 4, 0, cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return 2;
  return 0;
}

}  // namespace dm3

// ------------------------------------------------------------------ C ABI
namespace {
bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_gemv(const void* x, int M, int K, int N, const void* q, int64_t ldq, const float* s, int64_t lds,
               int srows, int bias_kind, const void* bias, void* y, int64_t ldy) {
  using dm3::set_error;
  if (M < 1 || M > dm3::kMaxT) return set_error("M must be in [1, 4]"), 1;
  if (K < 128 || K % 128 || K > dm3::kMaxGemvK) return set_error("K must be a multiple of 128 in [128, 8192]"), 1;
  if (N < 1) return set_error("N must be >= 1"), 1;
  if (!x || !q || !s || !y) return set_error("null pointer argument"), 1;
  if (!a16(x) || !a16(q)) return set_error("x and q must be 16-byte aligned"), 1;
  if (ldq < K || ldq % 16) return set_error("ldq must be >= K and a multiple of 16"), 1;
  if (srows != 1 && srows != 128) return set_error("srows must be 1 or 128"), 1;
  if (lds < K / 128) return set_error("lds must be >= K / 128"), 1;
  if (bias_kind < 0 || bias_kind > 2 || (bias_kind && !bias)) return set_error("bad bias"), 1;
  if (ldy < N) return set_error("ldy must be >= N"), 1;
  return 0;
}
}  // namespace

extern "C" int dm3_fp8_gemv(const void* x, int M, int K, int N, const void* q, int64_t ldq, const float* s,
                            int64_t lds, int srows, const void* bias, int bias_kind, void* y, int64_t ldy,
                            int y_fp32, void* stream) {
  dm3::note_launches(0);
  const int rc = check_gemv(x, M, K, N, q, ldq, s, lds, srows, bias_kind, bias, y, ldy);
  if (rc) return rc;
  // This file's kernel when every row of a CTA is one 2048-byte chunk and all of a CTA's rows fit its
  // ring (all weights then arrive before griddepcontrol.wait returns): measured faster on every such
  // shape. Otherwise the tensor-core kernel (split-K over a thread-block cluster, gemv_tc.cu), which
  // keeps its latency at K = 4096 and 8192 and for 2048 x 8192.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return dm3::set_error("cudaGetDevice failed"), 2;
  if (!dm3::gemv_rows_fit(K, N, dm3::sm_count(dev))) {
    const int rt = dm3::launch_gemv_tc(static_cast<const __nv_bfloat16*>(x), M, K, N, static_cast<const uint8_t*>(q),
                                       ldq, s, lds, srows, bias, bias_kind, y, ldy, y_fp32,
                                       static_cast<cudaStream_t>(stream));
    if (rt >= 0) return rt;
  }
  return dm3::launch_gemv(static_cast<const __nv_bfloat16*>(x), M, K, N, static_cast<const uint8_t*>(q), ldq,
                          nullptr, N, s, lds, srows, bias, bias_kind, y, ldy, y_fp32,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int dm3_fp8_gemv_gather(const void* x, int M, int K, int N, const void* q, int64_t ldq,
                                   int64_t n_rows_q, const int64_t* rows, const float* s, int64_t lds, int srows,
                                   void* y, int64_t ldy, int y_fp32, void* stream) {
  dm3::note_launches(0);
  const int rc = check_gemv(x, M, K, N, q, ldq, s, lds, srows, 0, nullptr, y, ldy);
  if (rc) return rc;
  if (!rows || n_rows_q < 1) return dm3::set_error("rows and n_rows_q are required"), 1;
  return dm3::launch_gemv(static_cast<const __nv_bfloat16*>(x), M, K, N, static_cast<const uint8_t*>(q), ldq,
                          rows, n_rows_q, s, lds, srows, nullptr, 0, y, ldy, y_fp32,
                          static_cast<cudaStream_t>(stream));
}

namespace dm3 {
// This file's copy of the device wait limit on the current device (dm3_set_wait_limit_ns).
int wait_limit_gemv(uint64_t ns) { return static_cast<int>(set_wait_limit_here(ns)); }
}  // namespace dm3
