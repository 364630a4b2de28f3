// Block-FP8 GEMV for B200 (sm_100a): y[M, N] = x[M, K] * dequant(q[N, K])^T, M <= 4.
//
// Each CTA owns a contiguous, balanced range of output rows (one CTA per SM). A producer warp
// streams tiles of up to 16 weight rows into a 2-stage shared-memory ring with cp.async.bulk
// (one copy per tile when the rows are contiguous, one per row for a gathered head) together with
// the tile's scale rows; 8 consumer warps split the K blocks of a tile and run FP8 m16n8k32
// mma.sync on the raw e4m3 bytes against the exact e4m3 hi/lo split of x.
// Per 128-wide K block the fp32 partial is multiplied by its block scale, as the reference
// Triton kernel does (fp8_linear.py:21-26).
//
// Programmatic dependent launch: the weight copies of the first tiles are issued before
// griddepcontrol.wait (weights are never produced by the preceding kernel), so a chain of
// GEMVs in a CUDA graph overlaps each kernel's DRAM ramp-up with the previous one's tail.
#include "dm3_common.cuh"
#include "dm3_internal.h"

namespace dm3 {
namespace gemv {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kStages = 2;
constexpr int kPad = 64;

struct Params {
  const __nv_bfloat16* x;
  int M, K, N;
  const uint8_t* q;
  int64_t ldq;
  const int64_t* rows;  // optional gather list [N]
  int64_t n_rows_q;
  const float* s;
  int64_t lds;
  int srows;
  const void* bias;
  int bias_kind;
  void* y;
  int64_t ldy;
  int y_fp32;
  int tile_rows;  // rows per stage (<= 16)
  int sc_bulk;    // scale rows staged by bulk copy (16-byte aligned rows); else read from global
};

struct Smem {
  int pitch, stage_bytes, stage, xq, red, misc, total;
};

__host__ __device__ inline Smem smem_layout(int K, int tile_rows) {
  Smem S;
  S.pitch = K + kPad;  // activation columns (thread-written, padded); weight rows are unpadded
  const int sb = tile_rows * K + tile_rows * (K / 128) * 4;
  S.stage_bytes = (sb + 127) / 128 * 128;
  int o = 0;
  S.stage = o;
  o += kStages * S.stage_bytes;
  S.xq = o;
  o += 8 * S.pitch;
  S.red = o;
  o += kConsumerWarps * 16 * 4 * 4;
  S.misc = o;
  o += 256;
  S.total = o;
  return S;
}

struct Misc {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  float xinv[kMaxT];
};

__device__ __forceinline__ int64_t src_row(const Params& p, int r) {
  if (p.rows == nullptr) return r;
  int64_t v = p.rows[r];
  // out-of-range indices are rejected by the host wrapper; clamp so a bad list can never fault
  if (v < 0) v = 0;
  if (v >= p.n_rows_q) v = p.n_rows_q - 1;
  return v;
}

__global__ void __launch_bounds__(kThreads) gemv_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Smem S = smem_layout(p.K, p.tile_rows);
  Misc* misc = reinterpret_cast<Misc*>(smem + S.misc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row_begin = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.N) / gridDim.x);
  const int row_end = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.N) / gridDim.x);
  const int TR = p.tile_rows;
  const int n_tiles = (row_end - row_begin + TR - 1) / TR;
  const int nkb = p.K / 128;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&misc->full[s], 1);
      mbar_init(&misc->empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch();

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------------- producer
    // Weights do not depend on the preceding kernel, so copies start before griddepcontrol.wait.
    uint32_t empty_par = 1;
    const bool contiguous = p.rows == nullptr && p.ldq == p.K;
    for (int i = 0; i < n_tiles; ++i) {
      const int stage = i % kStages;
      if (i > 0 && stage == 0) empty_par ^= 1u;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&misc->empty[stage], empty_par);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;  // consumers gone: nothing more can be delivered
      const int r0 = row_begin + i * TR;
      const int nr = min(TR, row_end - r0);
      uint8_t* st = smem + S.stage + stage * S.stage_bytes;
      uint64_t* full = &misc->full[stage];
      float* sd = reinterpret_cast<float*>(st + TR * p.K);
      const uint32_t srow = nkb * 4;
      // scale rows: 1x128 with contiguous rows -> one copy; 128x128 -> the (at most two) block rows
      // at positions 0, 1; gathered rows -> one copy per row
      const bool sc_one = p.sc_bulk && p.srows == 1 && p.rows == nullptr && p.lds == nkb;
      const bool sc_blk = p.sc_bulk && p.srows == 128 && p.rows == nullptr;
      const int sb0 = r0 / 128, sb1 = (r0 + nr - 1) / 128;
      uint32_t sbytes = 0;
      if (p.sc_bulk) sbytes = sc_one ? nr * srow : (sc_blk ? (sb1 - sb0 + 1) * srow : nr * srow);
      if (lane == 0) {
        mbar_arrive_expect_tx(full, static_cast<uint32_t>(nr * p.K) + sbytes);
        if (contiguous) bulk_g2s(st, p.q + static_cast<int64_t>(r0) * p.K, nr * p.K, full);
        if (sc_one) {
          bulk_g2s(sd, p.s + static_cast<int64_t>(r0) * nkb, nr * srow, full);
        } else if (sc_blk) {
          for (int b = sb0; b <= sb1; ++b) bulk_g2s(sd + (b - sb0) * nkb, p.s + static_cast<int64_t>(b) * p.lds, srow, full);
        }
      }
      __syncwarp();
      if (lane < nr) {
        const int64_t src = src_row(p, r0 + lane);
        if (!contiguous) bulk_g2s(st + lane * p.K, p.q + src * p.ldq, p.K, full);
        if (p.sc_bulk && !sc_one && !sc_blk)
          bulk_g2s(sd + lane * nkb, p.s + (src / p.srows) * p.lds, srow, full);
      }
    }
  } else {
    // ---------------------------------------------------------------- consumers
    griddep_wait();  // x is produced by the preceding kernel
    uint8_t* xq = smem + S.xq;
    if (warp < p.M) {
      const __nv_bfloat16* xr = p.x + static_cast<size_t>(warp) * p.K;
      float amax = 0.f;
      for (int k = lane * 8; k < p.K; k += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(e[i])));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const int e = split_exponent(amax);
      const float sc = exp2i(e);
      if (lane == 0) misc->xinv[warp] = exp2i(-e);
      uint8_t* hi = xq + warp * S.pitch;
      uint8_t* lo = xq + (4 + warp) * S.pitch;
      for (int k = lane * 8; k < p.K; k += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const __nv_bfloat16* e8 = reinterpret_cast<const __nv_bfloat16*>(&v);
        uint16_t h4[4], l4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          split2(__bfloat162float(e8[2 * i]) * sc, __bfloat162float(e8[2 * i + 1]) * sc, h4[i], l4[i]);
        *reinterpret_cast<uint2*>(hi + k) =
            make_uint2(h4[0] | (uint32_t(h4[1]) << 16), h4[2] | (uint32_t(h4[3]) << 16));
        *reinterpret_cast<uint2*>(lo + k) =
            make_uint2(l4[0] | (uint32_t(l4[1]) << 16), l4[2] | (uint32_t(l4[3]) << 16));
      }
    }
    named_bar(1, kConsumers);
    const int g = lane >> 2, q = lane & 3;
    const bool bvalid = (g & 3) < p.M;
    const uint8_t* bcol = xq + g * S.pitch;
    float* red = reinterpret_cast<float*>(smem + S.red);
    uint32_t full_par = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int stage = i % kStages;
      if (i > 0 && stage == 0) full_par ^= 1u;
      if (!mbar_wait(&misc->full[stage], full_par)) break;
      const int r0 = row_begin + i * TR;
      const int nr = min(TR, row_end - r0);
      const uint8_t* st = smem + S.stage + stage * S.stage_bytes;
      const float* sc = reinterpret_cast<const float*>(st + TR * p.K);
      const bool lo_ok = g < nr, hi_ok = g + 8 < nr;
      const uint8_t* row_lo = st + g * p.K;
      const uint8_t* row_hi = st + (g + 8) * p.K;
      // where each of this lane's two rows finds its scale row
      const bool sc_blk = p.srows == 128 && p.rows == nullptr;
      int si_lo = g, si_hi = g + 8;
      if (sc_blk) {
        si_lo = (r0 + g) / 128 - r0 / 128;
        si_hi = (r0 + g + 8) / 128 - r0 / 128;
      }
      const float* gs_lo = p.s + (lo_ok ? (src_row(p, r0 + g) / p.srows) * p.lds : 0);
      const float* gs_hi = p.s + (hi_ok ? (src_row(p, r0 + g + 8) / p.srows) * p.lds : 0);
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
      // this warp's k blocks: warp, warp + 8, ...; two per pass, all fragments loaded up front
      for (int kb0 = warp; kb0 < nkb; kb0 += 2 * kConsumerWarps) {
        const int kb1 = kb0 + kConsumerWarps;
        const bool v1 = kb1 < nkb;
        const int kbs[2] = {kb0, v1 ? kb1 : kb0};
        float part[2][4];
        tile_kblocks<2>(part, row_lo, row_hi, bcol, lo_ok, hi_ok, bvalid, kbs, q);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          float s0 = 0.f, s1 = 0.f;
          if (i == 0 || v1) {
            if (p.sc_bulk) {
              if (lo_ok) s0 = sc[si_lo * nkb + kbs[i]];
              if (hi_ok) s1 = sc[si_hi * nkb + kbs[i]];
            } else {
              if (lo_ok) s0 = __ldg(gs_lo + kbs[i]);
              if (hi_ok) s1 = __ldg(gs_hi + kbs[i]);
            }
          }
          tot[0] = fmaf(part[i][0], s0, tot[0]);
          tot[1] = fmaf(part[i][1], s0, tot[1]);
          tot[2] = fmaf(part[i][2], s1, tot[2]);
          tot[3] = fmaf(part[i][3], s1, tot[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) tot[j] += __shfl_down_sync(0xffffffffu, tot[j], 2);
      if (q < 2) {
        float* rw = red + warp * 64;
        rw[g * 4 + 2 * q] = tot[0];
        rw[g * 4 + 2 * q + 1] = tot[1];
        rw[(g + 8) * 4 + 2 * q] = tot[2];
        rw[(g + 8) * 4 + 2 * q + 1] = tot[3];
      }
      named_bar(1, kConsumers);
      if (tid < 64) {
        const int r = tid >> 2, t = tid & 3;
        if (r < nr && t < p.M) {
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) v += red[w * 64 + r * 4 + t];
          v *= misc->xinv[t];
          const int n = r0 + r;
          if (p.bias_kind == 1) v += __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
          if (p.bias_kind == 2) v += static_cast<const float*>(p.bias)[n];
          if (p.y_fp32)
            static_cast<float*>(p.y)[t * p.ldy + n] = v;
          else
            static_cast<__nv_bfloat16*>(p.y)[t * p.ldy + n] = __float2bfloat16_rn(v);
        }
      }
      named_bar(1, kConsumers);
      if (lane == 0) mbar_arrive(&misc->empty[stage]);
    }
  }
}

}  // namespace gemv

// ------------------------------------------------------------------ host launcher
int launch_gemv_tc(const __nv_bfloat16* x, int M, int K, int N, const uint8_t* q, int64_t ldq, const float* s,
                   int64_t lds, int srows, const void* bias, int bias_kind, void* y, int64_t ldy, int y_fp32,
                   cudaStream_t stream);

int launch_gemv(const __nv_bfloat16* x, int M, int K, int N, const uint8_t* q, int64_t ldq, const int64_t* rows,
                int64_t n_rows_q, const float* s, int64_t lds, int srows, const void* bias, int bias_kind, void* y,
                int64_t ldy, int y_fp32, cudaStream_t stream) {
  gemv::Params p{};
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
  p.tile_rows = K <= 2048 ? 16 : (K <= 4096 ? 8 : 4);
  const int nkb = K / 128;
  p.sc_bulk = (reinterpret_cast<uintptr_t>(s) & 15u) == 0 && (nkb * 4) % 16 == 0 && (lds * 4) % 16 == 0;
  const gemv::Smem S = gemv::smem_layout(K, p.tile_rows);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return 2;
  }
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(gemv::gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess) {
      set_error("cudaFuncSetAttribute(gemv) failed");
      return 2;
    }
    configured[dev] = true;
  }
  const int sms = sm_count(dev);
  const int grid = N < sms ? N : sms;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(gemv::kThreads);
  cfg.dynamicSmemBytes = S.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemv::gemv_kernel, p);
  if (err != cudaSuccess) {
    set_error(std::string("gemv launch: ") + cudaGetErrorString(err));
    return 2;
  }
  note_launches(1);
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
  // contiguous weight rows: the tensor-core kernel (split-K over a thread-block cluster)
  const int rt = dm3::launch_gemv_tc(static_cast<const __nv_bfloat16*>(x), M, K, N, static_cast<const uint8_t*>(q),
                                     ldq, s, lds, srows, bias, bias_kind, y, ldy, y_fp32,
                                     static_cast<cudaStream_t>(stream));
  if (rt >= 0) return rt;
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
