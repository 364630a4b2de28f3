// Block-FP8 GEMM on the tcgen05 tensor cores (sm_100a): y[M, N] = x[M, K] * dequant(q[N, K])^T
// (+ bias) for many activation rows, the path where the reference dequantises the whole weight
// and calls F.linear (fp8_linear.py:60-61; the prompt-reading chunks of engine.py:283-288 run every
// converted projection this way).
//
// Two kernels chained by programmatic dependent launch:
//   split  one warp per token row: the row's absolute maximum gives a power-of-two prescale 2^e
//          (amax -> [128, 256)); x * 2^e is split exactly into e4m3 hi + lo, stored as row t of the
//          hi plane and of the lo plane of the activation image, and 2^-e is kept per token
//   gemm   persistent CTAs over tiles of 128 weight rows x tb tokens (tb = 16, 32, 64 or 128):
//          warp 0 lane 0 feeds a ring of 4 stages by TMA (the weight slab, 128 rows x 128 bytes of K,
//          and the tile's hi and lo activation slabs, tb rows each, 128-byte swizzle; weights of the
//          first stages go out before griddepcontrol.wait); warp 1 lane 0 issues tcgen05.mma
//          kind::f8f6f4 (M = 128, N = tb, K = 32), the hi and the lo slab into the same accumulator,
//          one accumulator per 128-wide k block, four of them in flight in TMEM; warps 2-9 (two groups
//          of four, each owning half of the tile's tokens) read every k block's accumulator with all
//          loads issued before one wait and accumulate it times the weight's block scale in fp32
//          registers, then write y = acc * 2^-e (+ bias).
// Every product is exact (e4m3 x e4m3) and the block scale multiplies each 128-wide k-block partial
// in fp32, as the reference's dequantise-then-multiply does up to summation order.
#include <cstdint>
#include <string>

#include "dm3_common.cuh"
#include "dm3_internal.h"
#include "dm3_tc.cuh"

namespace dm3 {
namespace gemm {

constexpr int kRows = 128;                       // weight rows per tile (the MMA's M)
constexpr int kMaxTok = 128;                     // tokens per tile at most (the MMA's N)
constexpr int kStages = 4;
constexpr int kASlab = kRows * 128;              // 16 KB
constexpr int kBSlab = kMaxTok * 128;            // one activation plane's slab, up to 16 KB
constexpr int kStage = kASlab + 2 * kBSlab;       // weights, hi rows, lo rows
constexpr int kNacc = 4;
constexpr uint32_t kAccCols = 128;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 96 + 32 * kEpiWarps;   // producer, MMA issuer, 8 epilogue warps, 2nd MMA issuer
constexpr int kSplitWarps = 8;
constexpr int kStatusWord = 4;                   // the same slot as every other workspace's status

struct Params {
  const __nv_bfloat16* x;
  int M, K, N;
  const float* s;
  int64_t lds;
  int srows;
  const void* bias;
  int bias_kind;  // 0 none, 1 bf16, 2 fp32
  void* y;
  int64_t ldy;
  int y_fp32;
  uint8_t* ximg;     // [2][M][K] e4m3: the hi plane, then the lo plane
  float* xinv;       // [M]
  uint32_t* ctrl;    // control words; ctrl[kStatusWord] is the sticky status word
  int tb;            // tokens per tile
  int n_tok_tiles, n_tiles;
};

// Workspace: control words, 2^-e per token, the activation image.
struct Layout {
  size_t ctrl, xinv, ximg, total;
};
__host__ __device__ inline Layout layout(int M, int K) {
  Layout L;
  L.ctrl = 0;
  L.xinv = 256;
  L.ximg = (L.xinv + static_cast<size_t>(M) * 4 + 1023) / 1024 * 1024;  // [2][M][K]
  L.total = L.ximg + static_cast<size_t>(2) * M * K;
  return L;
}

struct Aux {
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[kNacc], acc_empty[kNacc];
  uint64_t mma_done, mma_done2;
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ void flag(const Params& p, uint32_t bits) { atomicOr(p.ctrl + kStatusWord, bits); }

// A bounded wait that, once any wait of the CTA has run out, returns false at once.
__device__ __forceinline__ bool wait_or_abort(const Params& p, uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (mbar_wait_sleep(bar, parity)) return true;
  if (!*abort) flag(p, STATUS_TIMEOUT);
  *abort = 1;
  return false;
}

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

// One warp per token row: absolute maximum, then the exact hi / lo split into row t of each plane.
__global__ void __launch_bounds__(32 * kSplitWarps) split_kernel(const __grid_constant__ Params p) {
  const int t = blockIdx.x * kSplitWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  griddep_wait();
  griddep_launch();
  if (t >= p.M) return;
  const uint4* row = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * p.K);
  const int chunks = p.K / 16;  // 16 elements (two uint4) per chunk
  float m = 0.f;
  for (int c = lane; c < chunks; c += 32) {
    const uint4 a = __ldg(row + 2 * c), b = __ldg(row + 2 * c + 1);
    const uint4 v[2] = {a, b};
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(v);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(__bfloat162float(e[i])));
  }
  m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
  const int ex = split_exponent(m);
  const float sc = exp2i(ex);
  uint8_t* hi_row = p.ximg + static_cast<size_t>(t) * p.K;
  uint8_t* lo_row = hi_row + static_cast<size_t>(p.M) * p.K;
  for (int c = lane; c < chunks; c += 32) {
    const uint4 v[2] = {__ldg(row + 2 * c), __ldg(row + 2 * c + 1)};
    uint4 hi, lo;
    split16(v, sc, hi, lo);
    *reinterpret_cast<uint4*>(hi_row + 16 * c) = hi;
    *reinterpret_cast<uint4*>(lo_row + 16 * c) = lo;
  }
  if (lane == 0) p.xinv[t] = exp2i(-ex);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_x) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Aux& aux = *reinterpret_cast<Aux*>(smem + kStages * kStage);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = p.K / 128;
  const int tb = p.tb;
  const int my_tiles = p.n_tiles > static_cast<int>(blockIdx.x) ? (p.n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  volatile int* abort = &aux.abort;

  if (tid == 0) {
    tc::prefetch_map(&map_w);
    tc::prefetch_map(&map_x);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&aux.full[s], 1);
      mbar_init(&aux.empty[s], 1);
    }
    for (int a = 0; a < kNacc; ++a) {
      mbar_init(&aux.acc_full[a], 1);
      mbar_init(&aux.acc_empty[a], kEpiWarps);
    }
    mbar_init(&aux.mma_done, 1);
    mbar_init(&aux.mma_done2, 1);
    aux.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(&aux.tmem, 512);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux.tmem;

  if (warp == 0) {
    // ================================================================ TMA producer (lane 0)
    if (lane == 0) {
      const int total = my_tiles * nkb;
      const uint32_t bbytes = static_cast<uint32_t>(2 * tb * 128);  // hi and lo slabs
      auto tile_of = [&](int k, int& rt, int& tt) {
        const int i = blockIdx.x + k * gridDim.x;
        rt = i / p.n_tok_tiles;
        tt = i % p.n_tok_tiles;
      };
      auto issue_a = [&](int s) {
        int rt, tt;
        tile_of(s / nkb, rt, tt);
        uint64_t* bar = &aux.full[s % kStages];
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kASlab) + bbytes);
        tc::tma_load_3d(smem + (s % kStages) * kStage, &map_w, (s % nkb) * 128, rt * kRows, 0, bar);
      };
      auto issue_b = [&](int s) {
        int rt, tt;
        tile_of(s / nkb, rt, tt);
        uint8_t* dst = smem + (s % kStages) * kStage + kASlab;
        tc::tma_load_3d(dst, &map_x, (s % nkb) * 128, tb * tt, 0, &aux.full[s % kStages]);
        tc::tma_load_3d(dst + kBSlab, &map_x, (s % nkb) * 128, tb * tt, 1, &aux.full[s % kStages]);
      };
      // weights never come from the preceding kernel: the first ring goes out before the wait
      const int first = min(total, kStages);
      for (int s = 0; s < first; ++s) issue_a(s);
      griddep_wait();
      griddep_launch();
      for (int s = 0; s < first; ++s) issue_b(s);
      int issued = first;
      for (int s = first; s < total; ++s) {
        if (!wait_or_abort(p, &aux.empty[s % kStages], ((s / kStages) & 1) ^ 1u, abort)) break;
        issue_a(s);
        issue_b(s);
        issued = s + 1;
      }
      // nothing may still be copying into shared memory when the CTA exits (bounded waits)
      for (int s = max(0, issued - kStages); s < issued; ++s) mbar_wait(&aux.full[s % kStages], (s / kStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2 + kEpiWarps) {
    // ================================================================ MMA issuers (lane 0): warp 1 the even
    // stages, the last warp the odd ones (their accumulators differ: ab = s % 4). One issuer waits
    // about as long for each tcgen05.mma to be accepted as the tensor core takes to run a
    // skinny one; two issuers keep it busy (9-15% faster at M = 16-256).
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_e4m3(kRows, tb);
      const int total = my_tiles * nkb;
      const int par = warp == 1 ? 0 : 1;
      for (int s = par; s < total; s += 2) {
        const int ab = s % kNacc;
        if (!wait_or_abort(p, &aux.acc_empty[ab], ((s / kNacc) & 1) ^ 1u, abort)) break;
        if (!wait_or_abort(p, &aux.full[s % kStages], (s / kStages) & 1, abort)) break;
        tc::fence_after_sync();
        const uint32_t a = smem_u32(smem + (s % kStages) * kStage);
        const uint32_t b = a + kASlab;
        // x = hi + lo exactly: both halves accumulate into the same columns
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          tc::mma_f8(tmem + ab * kAccCols, tc::smem_desc(a + 32 * k4), tc::smem_desc(b + 32 * k4), idesc, k4 > 0);
          tc::mma_f8(tmem + ab * kAccCols, tc::smem_desc(a + 32 * k4), tc::smem_desc(b + kBSlab + 32 * k4), idesc,
                     true);
        }
        tc::mma_commit(&aux.empty[s % kStages]);
        tc::mma_commit(&aux.acc_full[ab]);
      }
      // every MMA issued has completed before TMEM is released (bounded)
      tc::mma_commit(par ? &aux.mma_done2 : &aux.mma_done);
      mbar_wait(par ? &aux.mma_done2 : &aux.mma_done, 0);
    }
    __syncwarp();
  } else {
    // ================================================================ epilogue (warps 2-9)
    const int grp = (warp - 2) >> 2;         // token half of the tile
    const int q = warp & 3;                  // TMEM lane quarter this warp may read
    const int r = 32 * q + lane;             // weight row within the tile
    const int half = tb / 2;                 // tokens (= accumulator columns) of this group
    griddep_wait();                          // 2^-e of the tokens comes from the split kernel
    int use = 0;
    for (int k = 0; k < my_tiles; ++k) {
      const int i = blockIdx.x + k * gridDim.x;
      const int rt = i / p.n_tok_tiles, tt = i % p.n_tok_tiles;
      const int n = rt * kRows + r;
      const int tok0 = tt * tb + grp * half;
      const float* srow = p.s + static_cast<size_t>((n < p.N ? n : p.N - 1) / p.srows) * p.lds;
      float acc[kMaxTok / 2];
#pragma unroll
      for (int j = 0; j < kMaxTok / 2; ++j) acc[j] = 0.f;
      float sc = __ldg(srow);
      bool ok = !*abort;
      for (int kb = 0; kb < nkb; ++kb, ++use) {
        const float sc_next = kb + 1 < nkb ? __ldg(srow + kb + 1) : 0.f;
        const int ab = use % kNacc;
        bool ready = ok;
        if (ok && lane == 0) ready = wait_or_abort(p, &aux.acc_full[ab], (use / kNacc) & 1, abort);
        ready = __shfl_sync(0xffffffffu, ready, 0);
        ok = ok && ready;
        tc::fence_after_sync();
        if (ok) {
          const uint32_t ta = tmem + (static_cast<uint32_t>(32 * q) << 16) + ab * kAccCols + grp * half;
          // every load of this k block is issued before the one wait
          float v[kMaxTok / 2];
          if (half == 64) {
            tc::tmem_ld32(ta, *reinterpret_cast<float(*)[32]>(&v[0]));
            tc::tmem_ld32(ta + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
          } else if (half == 32) {
            tc::tmem_ld32(ta, *reinterpret_cast<float(*)[32]>(&v[0]));
          } else if (half == 16) {
            tc::tmem_ld16(ta, *reinterpret_cast<float(*)[16]>(&v[0]));
          } else {
            tc::tmem_ld8(ta, *reinterpret_cast<float(*)[8]>(&v[0]));
          }
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < kMaxTok / 2; ++j)
            if (j < half) acc[j] = fmaf(sc, v[j], acc[j]);
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&aux.acc_empty[ab]);
        }
        sc = sc_next;
      }
      if (!ok) break;
      // y = acc * 2^-e (+ bias): lanes hold consecutive rows of one token, so each store is coalesced
      float bias = 0.f;
      if (n < p.N) {
        if (p.bias_kind == 1) bias = __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
        if (p.bias_kind == 2) bias = static_cast<const float*>(p.bias)[n];
      }
      const float xi_lane = tok0 + lane < p.M && lane < half ? __ldcg(p.xinv + tok0 + lane) : 0.f;
      const float xi_hi = tok0 + 32 + lane < p.M && 32 + lane < half ? __ldcg(p.xinv + tok0 + 32 + lane) : 0.f;
#pragma unroll
      for (int j = 0; j < kMaxTok / 2; ++j) {
        const float xj = __shfl_sync(0xffffffffu, j < 32 ? xi_lane : xi_hi, j & 31);
        const int t = tok0 + j;
        if (j < half && t < p.M && n < p.N) {
          const float v = fmaf(acc[j], xj, bias);
          if (p.y_fp32)
            static_cast<float*>(p.y)[static_cast<size_t>(t) * p.ldy + n] = v;
          else
            static_cast<__nv_bfloat16*>(p.y)[static_cast<size_t>(t) * p.ldy + n] = __float2bfloat16_rn(v);
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

constexpr size_t kSmem = static_cast<size_t>(kStages) * kStage + ((sizeof(Aux) + 127) / 128) * 128 + 1024;

}  // namespace gemm
}  // namespace dm3

// ------------------------------------------------------------------ C ABI
extern "C" size_t dm3_fp8_gemm_workspace_bytes(int M, int K) {
  if (M < 1 || K < 128) return 0;
  return dm3::gemm::layout(M, K).total;
}

extern "C" int dm3_fp8_gemm(const void* x, int M, int K, int N, const void* q, int64_t ldq, const float* s,
                            int64_t lds, int srows, const void* bias, int bias_kind, void* y, int64_t ldy, int y_fp32,
                            void* workspace, size_t workspace_bytes, void* stream) {
  using dm3::set_error;
  namespace g = dm3::gemm;
  dm3::note_launches(0);
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (M < 1 || M > (1 << 20)) return set_error("M must be in [1, 1048576]"), 1;
  if (K < 128 || K % 128 || K > 65536) return set_error("K must be a multiple of 128 in [128, 65536]"), 1;
  if (N < 1) return set_error("N must be >= 1"), 1;
  if (!x || !q || !s || !y || !workspace) return set_error("null pointer argument"), 1;
  if (!a16(x) || !a16(q)) return set_error("x and q must be 16-byte aligned"), 1;
  if (ldq < K || ldq % 16) return set_error("ldq must be >= K and a multiple of 16"), 1;
  if (srows != 1 && srows != 128) return set_error("srows must be 1 or 128"), 1;
  if (lds < K / 128) return set_error("lds must be >= K / 128"), 1;
  if (bias_kind < 0 || bias_kind > 2 || (bias_kind != 0 && !bias)) return set_error("bad bias arguments"), 1;
  if (ldy < N) return set_error("ldy must be >= N"), 1;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return set_error("workspace must be 256-byte aligned"), 1;
  if (workspace_bytes < g::layout(M, K).total) return set_error("workspace too small"), 4;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error("cudaGetDevice failed"), 2;
  const int sms = dm3::sm_count(dev);
  const g::Layout L = g::layout(M, K);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  g::Params p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.M = M;
  p.K = K;
  p.N = N;
  p.s = s;
  p.lds = lds;
  p.srows = srows;
  p.bias = bias;
  p.bias_kind = bias_kind;
  p.y = y;
  p.ldy = ldy;
  p.y_fp32 = y_fp32;
  p.ximg = ws + L.ximg;
  p.xinv = reinterpret_cast<float*>(ws + L.xinv);
  p.ctrl = reinterpret_cast<uint32_t*>(ws + L.ctrl);
  p.tb = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  p.n_tok_tiles = (M + p.tb - 1) / p.tb;
  const int n_row_tiles = (N + g::kRows - 1) / g::kRows;
  p.n_tiles = n_row_tiles * p.n_tok_tiles;

  CUtensorMap mw, mx;
  if (!dm3::tensor_map_3d(&mw, q, static_cast<uint64_t>(K), static_cast<uint64_t>(N), 1, static_cast<uint64_t>(ldq),
                          static_cast<uint64_t>(ldq) * static_cast<uint64_t>(N), g::kRows) ||
      !dm3::tensor_map_3d(&mx, p.ximg, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 2, static_cast<uint64_t>(K),
                          static_cast<uint64_t>(M) * static_cast<uint64_t>(K), static_cast<uint32_t>(p.tb)))
    return 2;
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(g::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(g::kSmem)) != cudaSuccess)
      return set_error("cudaFuncSetAttribute(gemm) failed"), 2;
    configured[dev] = true;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = dm3::pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((M + g::kSplitWarps - 1) / g::kSplitWarps);
  cfg.blockDim = dim3(32 * g::kSplitWarps);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&cfg, g::split_kernel, p);
  if (err != cudaSuccess) return set_error(std::string("gemm split launch: ") + cudaGetErrorString(err)), 2;
  cfg.gridDim = dim3(p.n_tiles < sms ? p.n_tiles : sms);
  cfg.blockDim = dim3(g::kThreads);
  cfg.dynamicSmemBytes = g::kSmem;
  err = cudaLaunchKernelEx(&cfg, g::gemm_kernel, p, mw, mx);
  if (err != cudaSuccess) return set_error(std::string("gemm launch: ") + cudaGetErrorString(err)), 2;
  dm3::note_launches(2);
  return 0;
}

namespace dm3 {
// This file's copy of the device wait limit on the current device (dm3_set_wait_limit_ns).
int wait_limit_gemm(uint64_t ns) { return static_cast<int>(set_wait_limit_here(ns)); }
}  // namespace dm3
