// Prefill (prompt-reading) MoE layer for B200 (sm_100a): hundreds of tokens against 256 block-FP8
// experts, as seven chained kernels under programmatic dependent launch.
//
//   logits    approximate router logits x . W^T on the tensor cores (tcgen05 kind::f16, bf16 x bf16
//             products, fp32 accumulation in TMEM), plus the squared norms of the router rows
//   select    one warp per token: a proven error window around every approximate logit picks the
//             few experts that can still reach the top k; only those are recomputed exactly (fp64
//             sums of the exact bf16 products, rounded once), so the chosen experts and their
//             weights are those of exact logits; softmax / top-k / renormalise as Speaker.__call__
//             (engine.py:233-235) and the shared expert's sigmoid gate (engine.py:158)
//   plan      one CTA: the (token, k) pairs stably sorted by expert (the dispatch order), per-expert
//             offsets, and tiles of up to 64 tokens of one expert (the shared expert takes all T)
//   dispatch  every (expert, token) position gets the token's row split exactly into e4m3 hi + lo
//             rows (x * 2^e, one power of two per token), in the permuted order
//   up        items (tile, 128 gate rows + the matching 128 up rows): tcgen05 kind::f8f6f4 with
//             M = 128 weight rows, N = 2 x tokens (hi / lo rows interleaved), one fp32 accumulator
//             pair per 128-wide k slab that the epilogue scales by the weight's block scale into
//             registers; SwiGLU; h rounded to bf16 and split exactly into e4m3 hi + lo per (token,
//             128-block of h)
//   down      items (tile, 128 output rows) against h, per-slab scales (weight block x h block);
//             one fp32 row per (expert, token) position
//   combine   per token the routing-weighted sum of its k rows (fixed order), + bias, + the gated
//             shared expert, with the reference's bf16 rounding points
//
// Warp roles of the up / down kernels (one CTA per SM, 10 warps): warp 0 issues TMA loads (weight
// slabs of 128 rows x 128 bytes and the tile's activation slab), warp 1 issues the MMAs, warps 2-9
// read the accumulators (warp % 4 selects the TMEM lane quarter, (warp - 2) / 4 the half of the
// tile's tokens). Every wait is bounded; a wait that runs out sets the status word and the CTA's
// abort flag, after which no thread waits again and every loop still runs to its end, so no
// barrier is left without its arrivals.
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <utility>

#include "dm3_common.cuh"
#include "dm3_ep.cuh"
#include "dm3_internal.h"
#include "dm3_route.cuh"
#include "dm3_tc.cuh"

namespace dm3 {
namespace pf {

constexpr int kTileTok = 64;                 // tokens per expert tile
constexpr int kRows = 128;                   // weight rows per MMA tile (M)
constexpr int kSlab = kRows * 128;           // one 128-byte K slab of a 128-row tile
// warp 0 TMA, warp 1 MMA, then groups of 8 epilogue warps: the up kernel has two groups that take
// alternate items, so one group's SwiGLU tail overlaps the other group's accumulator reads
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = kEpiWarps * 32;
__host__ __device__ constexpr int epi_groups(bool down) { return down ? 1 : 2; }
__host__ __device__ constexpr int expert_threads(bool down) { return 96 + epi_groups(down) * kEpiThreads; }
constexpr int kStages = 4;                   // ring of TMA stages
constexpr int kStage = 3 * kSlab;            // two weight slabs, the activation slab (<= 128 rows)
// TMEM accumulator buffers: up 4 of 128 columns (gate, then up rows; a token's hi and lo rows add into
// one column), down 2 of 256 (two 128-row halves, each token's hi / lo rows in adjacent columns)
__host__ __device__ constexpr int n_acc(bool down) { return down ? 2 : 4; }
__host__ __device__ constexpr uint32_t acc_cols(bool down) { return down ? 256u : 128u; }
constexpr int kLgK = 512;                    // K per logits CTA
constexpr int kLgSlabs = kLgK / 64;          // 64 bf16 per 128-byte slab
constexpr int kLgTok = 32;                   // tokens per logits CTA (N)
constexpr int kLgThreads = 192;              // warp 0 TMA + MMA, warp 1 TMEM, warps 2-5 epilogue
constexpr int kLgBSlab = kLgTok * 128;
constexpr int kLgSmem = kLgSlabs * (kSlab + kLgBSlab) + 1024 + 256;
constexpr int kCombineThreads = 256;
constexpr int kBarEpi = 1;                   // named barriers of the up epilogue groups (1, 2)

// control words; the status word sits where the decode workspace keeps it, so one reader serves both
enum : int { C_STATUS = 4, C_NTILES = 8, C_NVALID = 9, C_WORDS = 16 };

constexpr int kMaxRanks = 8;

struct Params {
  int T, H, I, E, K;  // tokens, hidden, intermediate, routed experts (router width), top-k
  int mode;           // 0: routing given (ids / rw), 1: router
  const __nv_bfloat16* x;
  const __nv_bfloat16* router_w;  // [E][H] bf16
  int logits_bf16;
  const float* logit_bias;
  const __nv_bfloat16* sh_gate;  // [H] or null
  const int64_t* ids;
  const __nv_bfloat16* rw;
  const uint8_t* w13;
  int64_t w13_stride;
  const float* s13;
  int64_t s13_stride;
  const uint8_t* w2;
  int64_t w2_stride;
  const float* s2;
  int64_t s2_stride;
  int srows;
  const uint8_t* sh_w13;
  const float* sh_s13;
  const uint8_t* sh_w2;
  const float* sh_s2;
  int sh_srows;
  const float* out_bias;
  __nv_bfloat16* y;
  int64_t* ids_out;
  __nv_bfloat16* w_out;
  int64_t* perm_out;
  int64_t* offsets_out;
  uint8_t* ws;
  // expert parallel (world > 1): this rank routes its own T tokens over all E experts and owns the
  // el experts [rank * el, (rank + 1) * el), whose weights w13 / w2 hold; ep_arena[r] is rank r's
  // arena mapped in this process (ep_arena[rank] its own), ep_tl the token capacity of every rank
  int world, rank, ep_tl, ep_el;
  uint8_t* ep_arena[kMaxRanks];
  // optional placement [E]: (owning rank << 16) | index among that rank's experts; null places
  // expert e on rank e / el at index e % el
  const int* ep_owner;
};

__device__ __forceinline__ int ep_place(const Params& p, int e) {
  return p.ep_owner ? __ldg(p.ep_owner + e) : ((e / p.ep_el) << 16) | (e % p.ep_el);
}

// ------------------------------------------------------------------ workspace layout
// Positions: the P = T * K routed (token, k) pairs in dispatch order (expert-major, stable), then
// one position per token for the shared expert. Every per-position buffer is indexed by position.
struct Layout {
  size_t ctrl, lpart, wnorm, pair_e, pair_w, gate, xexp, pos_tok, pxinv, perm, inv, tiles, pimg, himg, hinv, outp, total;
  int ks, max_tiles, npos;
  int cap;  // routed positions [0, cap); the shared expert's positions are cap + t
};

__host__ __device__ inline size_t aup(size_t v, size_t a) { return (v + a - 1) / a * a; }

// cap: routed positions; T * K on one GPU, world * (token capacity per rank) * K under expert
// parallelism (the pairs every rank may send here).
__host__ __device__ inline Layout layout(int T, int H, int I, int E, int K, int cap = -1) {
  Layout L;
  const size_t P = static_cast<size_t>(T) * K;
  L.cap = cap < 0 ? static_cast<int>(P) : cap;
  L.ks = (H + kLgK - 1) / kLgK;
  L.npos = L.cap + T;
  L.max_tiles = (L.cap + kTileTok - 1) / kTileTok + (E < L.cap ? E : L.cap) + (T + kTileTok - 1) / kTileTok + 1;
  size_t o = 0;
  L.ctrl = o;
  o += C_WORDS * 4;
  L.lpart = o = aup(o, 128);
  o += static_cast<size_t>(L.ks) * T * E * 4;
  L.wnorm = o = aup(o, 128);
  o += static_cast<size_t>(L.ks) * E * 4;
  L.pair_e = o = aup(o, 128);
  o += P * 4;
  L.pair_w = o = aup(o, 128);
  o += P * 4;
  L.gate = o = aup(o, 128);
  o += static_cast<size_t>(T) * 4;
  L.xexp = o = aup(o, 128);
  o += static_cast<size_t>(T) * 4;
  L.pos_tok = o = aup(o, 128);
  o += static_cast<size_t>(L.npos) * 4;
  L.pxinv = o = aup(o, 128);  // [npos] 2^-e of the position's token split
  o += static_cast<size_t>(L.npos) * 4;
  L.perm = o = aup(o, 128);
  o += P * 4;
  L.inv = o = aup(o, 128);
  o += P * 4;
  L.tiles = o = aup(o, 128);
  o += static_cast<size_t>(L.max_tiles) * 16;
  L.pimg = o = aup(o, 1024);  // [2][npos][H] e4m3: the hi rows of every position, then the lo rows
  o += static_cast<size_t>(L.npos) * 2 * H;
  L.himg = o = aup(o, 1024);  // [npos][2][I] e4m3
  o += static_cast<size_t>(L.npos) * 2 * I;
  L.hinv = o = aup(o, 128);   // [npos][I / 128] fp32: 2^-e of each 128-block of h
  o += static_cast<size_t>(L.npos) * (I / 128) * 4;
  L.outp = o = aup(o, 128);   // [npos][H] fp32: down-projection row of each position (unweighted)
  o += static_cast<size_t>(L.npos) * H * 4;
  L.total = aup(o, 256);
  return L;
}

__host__ __device__ inline Layout layout_of(const Params& p) {
  return layout(p.T, p.H, p.I, p.E, p.K, p.world > 1 ? p.world * p.ep_tl * p.K : -1);
}

using ep::EpLayout;
using ep::ep_layout;
using ep::EP_EPOCH;
using ep::EP_DISP_COUNT;
using ep::EP_DOWN_COUNT;
using ep::ld_acquire_sys;
using ep::st_release_sys;
using ep::wait_epoch;

template <typename T>
__device__ __forceinline__ T* ws_at(const Params& p, size_t off) {
  return reinterpret_cast<T*>(p.ws + off);
}
__device__ __forceinline__ void flag(const Params& p, uint32_t bits) {
  atomicOr(reinterpret_cast<uint32_t*>(p.ws) + C_STATUS, bits);
}

// Waits unless the CTA has aborted; a wait that runs out aborts the CTA (and reports it once).
__device__ __forceinline__ bool wait_or_abort(const Params& p, uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (mbar_wait_sleep(bar, parity)) return true;
  if (!*abort) flag(p, STATUS_TIMEOUT);
  *abort = 1;
  return false;
}

// ------------------------------------------------------------------ logits kernel
// CTA (m, n, ks): router rows [128 m, +128) x tokens [32 n, +32) over k in [512 ks, +512). Both
// operands arrive by TMA (the router rows before griddepcontrol.wait, x after it); one thread
// issues 32 MMAs (M = 128, N = 32, K = 16) into 32 TMEM columns. The partial logits are written
// as lpart[ks][t][e]; CTAs with n = 0 also write the squared norms of their router rows over their
// k range, which bound the summation error of the approximate logits.
__global__ void __launch_bounds__(kLgThreads, 1)
    logits_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map_r,
                  const __grid_constant__ CUtensorMap map_x) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sa = smem;
  uint8_t* sb = smem + kLgSlabs * kSlab;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + kLgSlabs * kLgBSlab);
  uint64_t* done = full + kLgSlabs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const Layout L = layout_of(p);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kRows, t0 = blockIdx.y * kLgTok, ks = blockIdx.z;
  const int nsl = min(kLgSlabs, p.H / 64 - ks * kLgSlabs);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLgSlabs; ++s) mbar_init(&full[s], 1);
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 32);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_map(&map_r);
      tc::prefetch_map(&map_x);
      for (int s = 0; s < nsl; ++s) {
        mbar_arrive_expect_tx(&full[s], kSlab + kLgBSlab);
        tc::tma_load_3d(sa + s * kSlab, &map_r, (ks * kLgK + s * 64) * 2, m0, 0, &full[s]);
      }
      griddep_wait();  // x comes from the preceding kernel
      griddep_launch();
      for (int s = 0; s < nsl; ++s) tc::tma_load_3d(sb + s * kLgBSlab, &map_x, (ks * kLgK + s * 64) * 2, t0, 0, &full[s]);
      const uint32_t idesc = tc::idesc_bf16(kRows, kLgTok);
      bool ok = true;
      for (int s = 0; s < nsl && ok; ++s) {
        if (!mbar_wait(&full[s], 0)) {
          flag(p, STATUS_TIMEOUT);
          ok = false;
          break;
        }
        const uint32_t a = smem_u32(sa + s * kSlab), b = smem_u32(sb + s * kLgBSlab);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::mma_bf16(tmem, tc::smem_desc(a + 32 * k), tc::smem_desc(b + 32 * k), idesc, s > 0 || k > 0);
      }
      tc::mma_commit(done);  // also issued after a failed wait: every MMA issued so far completes
    }
    __syncwarp();
  } else if (warp >= 2) {
    const int q = warp & 3;
    const int r = 32 * q + lane;
    // squared norms of this CTA's share of the 128 router rows over this k range (the token-tile
    // CTAs split the rows; 16 threads per row; the slab swizzle only permutes 16-byte chunks
    // inside a row's 128 bytes)
    const int rp = (kRows + gridDim.y - 1) / gridDim.y;
    const int r_lo = blockIdx.y * rp, r_hi = min(kRows, r_lo + rp);
    if (r_lo < r_hi) {
      bool landed = true;
      for (int s = 0; s < nsl && landed; ++s) landed = mbar_wait(&full[s], 0);
      if (!landed && r == 0) flag(p, STATUS_TIMEOUT);
      for (int base = r_lo; base < r_hi; base += 8) {
        const int row = base + (r >> 4), part = r & 15;
        float n2 = 0.f;
        if (landed && row < r_hi) {
          for (int ci = part; ci < nsl * 8; ci += 16) {
            const uint4 v = *reinterpret_cast<const uint4*>(sa + (ci >> 3) * kSlab + (row >> 3) * 1024 + (row & 7) * 128 + (ci & 7) * 16);
            const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float f = __bfloat162float(e[i]);
              n2 = fmaf(f, f, n2);
            }
          }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
        if (part == 0 && row < r_hi && m0 + row < p.E) ws_at<float>(p, L.wnorm)[ks * p.E + m0 + row] = n2;
      }
    }
    const bool ready = mbar_wait(done, 0);
    if (!ready && lane == 0) flag(p, STATUS_TIMEOUT);
    tc::fence_after_sync();
    float v[32];
    tc::tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16), v);
    tc::tmem_wait_ld();
    if (ready && m0 + r < p.E) {
      float* out = ws_at<float>(p, L.lpart) + (static_cast<size_t>(ks) * p.T + t0) * p.E + m0 + r;
#pragma unroll
      for (int j = 0; j < kLgTok; ++j)
        if (t0 + j < p.T) out[static_cast<size_t>(j) * p.E] = v[j];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 32);
}

// ------------------------------------------------------------------ select kernel
constexpr int kSelThreads = 256;  // one CTA per token; thread e owns expert e, 8 elements of x
constexpr int kSelChunk = 8;      // candidate rows fetched together
constexpr int kMaxKs = (kMaxH + kLgK - 1) / kLgK;

struct SelSmem {
  double part[kSelThreads / 32][kSelChunk];
  uint64_t keys[kMaxRouter];
  float fx[kMaxRouter];
  int cand[kMaxRouter + 1];
  uint8_t is_cand[kMaxRouter];
  float red[2][kSelThreads / 32];
  int wcount[kSelThreads / 32];
  float theta, gcoef;
  int ncand;
};

// The logit the softmax sees: fp32 (or rounded to bf16 for a bf16 router) + the optional bias.
// Non-decreasing in v, so bounds on v give bounds on it.
__device__ __forceinline__ float logit_map(const Params& p, float v, int e) {
  if (p.logits_bf16) v = bf16_round(v);
  if (p.logit_bias) v += __ldg(p.logit_bias + e);
  return v;
}

// One CTA per token. Routing given (mode 0): validates the ids and records the pairs. Router
// (mode 1): approximate logit a_e = sum of the logits kernel's partials; its error is below
// d_e = 2^-10 |x| |w_e| (the fp32 tensor-core sums err by far less than 2^-16 of sum |x_k w_ek|,
// which Cauchy-Schwarz bounds by |x| |w_e|). theta = the k-th largest of map(a_e - d_e); an expert
// with map(a_e + d_e) < theta has k experts strictly above it and cannot be selected, every other
// one is a candidate whose logit is recomputed exactly: the exact bf16 products summed in fp64
// (within 2^-42 of exact for 2048 terms) and rounded once to fp32, as the oracle's float64 matmul.
// Candidate rows are fetched kSelChunk at a time by the whole CTA (8 elements per thread), so a
// chunk costs one memory round trip. Selection, softmax and renormalisation follow the decode
// router (ties to the lower index) with the exact values of every candidate; the softmax
// denominator takes the approximate values of the others, whose share cancels in the
// renormalised weights.
__global__ void __launch_bounds__(kSelThreads, 4) select_kernel(const __grid_constant__ Params p) {
  __shared__ SelSmem sm;
  const Layout L = layout_of(p);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x;
  const int H = p.H, E = p.E, K = p.K;
  griddep_wait();
  griddep_launch();
  // this thread's 8 elements of the token row, |x|^2 and max |x|
  const bool xin = 8 * tid < H;
  const uint4 xv = xin ? __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * H + 8 * tid))
                       : make_uint4(0u, 0u, 0u, 0u);
  float xn2 = 0.f, xm = 0.f;
  {
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(xe[j]);
      xn2 = fmaf(f, f, xn2);
      xm = fmaxf(xm, fabsf(f));
    }
  }
  // approximate logit of expert tid (all partials requested before the reductions)
  float a = 0.f, w2 = 0.f;
  if (p.mode == 1 && tid < E) {
    float ap[kMaxKs], wp[kMaxKs];
#pragma unroll
    for (int s = 0; s < kMaxKs; ++s) {
      ap[s] = s < L.ks ? __ldcg(ws_at<const float>(p, L.lpart) + (static_cast<size_t>(s) * p.T + t) * E + tid) : 0.f;
      wp[s] = s < L.ks ? __ldcg(ws_at<const float>(p, L.wnorm) + s * E + tid) : 0.f;
    }
#pragma unroll
    for (int s = 0; s < kMaxKs; ++s) {
      a += ap[s];
      w2 += wp[s];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    xn2 += __shfl_xor_sync(0xffffffffu, xn2, o);
    xm = fmaxf(xm, __shfl_xor_sync(0xffffffffu, xm, o));
  }
  if (lane == 0) {
    sm.red[0][warp] = xn2;
    sm.red[1][warp] = xm;
  }
  __syncthreads();
  xn2 = 0.f;
  xm = 0.f;
#pragma unroll
  for (int w = 0; w < kSelThreads / 32; ++w) {
    xn2 += sm.red[0][w];
    xm = fmaxf(xm, sm.red[1][w]);
  }
  if (tid == 0) ws_at<int>(p, L.xexp)[t] = split_exponent(xm);
  int* pair_e = ws_at<int>(p, L.pair_e) + t * K;
  float* pair_w = ws_at<float>(p, L.pair_w) + t * K;
  if (p.mode == 0) {
    if (tid < K) {
      const int64_t id = p.ids[t * K + tid];
      const bool ok = id >= 0 && id < E;
      if (!ok) flag(p, STATUS_BAD_EXPERT);
      pair_e[tid] = ok ? static_cast<int>(id) : -1;
      pair_w[tid] = __bfloat162float(p.rw[t * K + tid]);
    }
    if (tid == 0) ws_at<float>(p, L.gate)[t] = 1.f;
    return;
  }
  // windows and the threshold
  float fu = -FLT_MAX;
  if (tid < E) {
    const float d = __fmul_ru(ldexpf(sqrtf(xn2 * w2), -10), 1.001f) + 1e-30f;
    sm.fx[tid] = logit_map(p, a, tid);
    fu = logit_map(p, __fadd_ru(a, d), tid);
    sm.keys[tid] = (static_cast<uint64_t>(order_key(logit_map(p, __fsub_rd(a, d), tid))) << 32) | static_cast<uint32_t>(~tid);
  } else if (tid < kMaxRouter) {
    sm.keys[tid] = 0ull;
  }
  __syncthreads();
  if (warp == 0) {
    // theta = the K-th largest of the 32 lane maxima of the lower bounds: at most the K-th largest
    // lower bound, so the candidate set below only grows (by a few experts) and still holds every
    // expert that can be selected; it costs one round of 32 shuffles instead of a full top-8 merge
    uint64_t mk = 0ull;
#pragma unroll
    for (int i = 0; i < 8; ++i) mk = max(mk, sm.keys[lane + 32 * i]);
    int beats = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) beats += __shfl_sync(0xffffffffu, mk, j) > mk ? 1 : 0;
    const unsigned who = __ballot_sync(0xffffffffu, beats == K - 1);
    if (lane == __ffs(who) - 1) sm.theta = key_value(static_cast<uint32_t>(mk >> 32));
  }
  __syncthreads();
  // candidate list (ascending expert order), then the shared gate row
  const bool cand = tid < E && fu >= sm.theta;
  const unsigned bal = __ballot_sync(0xffffffffu, cand);
  if (lane == 0) sm.wcount[warp] = __popc(bal);
  if (tid < kMaxRouter) sm.is_cand[tid] = cand ? 1 : 0;
  __syncthreads();
  int before = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kSelThreads / 32; ++w) {
    before += w < warp ? sm.wcount[w] : 0;
    total += sm.wcount[w];
  }
  if (cand) sm.cand[before + __popc(bal & ((1u << lane) - 1u))] = tid;
  const bool gate_row = p.sh_gate != nullptr;
  if (tid == 0) {
    if (gate_row) sm.cand[total] = E;  // the shared expert's gate row
    sm.ncand = total + (gate_row ? 1 : 0);
  }
  __syncthreads();
  const int nc = sm.ncand;
  double xd[8];  // this thread's x elements, exact in fp64 (converted once for every candidate)
  {
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
    for (int j = 0; j < 8; ++j) xd[j] = static_cast<double>(__bfloat162float(xe[j]));
  }
  for (int c0 = 0; c0 < nc; c0 += kSelChunk) {
    uint4 wv[kSelChunk];
#pragma unroll
    for (int c = 0; c < kSelChunk; ++c) {
      wv[c] = make_uint4(0u, 0u, 0u, 0u);
      if (c0 + c < nc && xin) {
        const int row = sm.cand[c0 + c];
        const __nv_bfloat16* wr = row < E ? p.router_w + static_cast<size_t>(row) * H : p.sh_gate;
        wv[c] = __ldg(reinterpret_cast<const uint4*>(wr + 8 * tid));
      }
    }
    double a[kSelChunk];
#pragma unroll
    for (int c = 0; c < kSelChunk; ++c) {
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv[c]);
      a[c] = 0.0;
#pragma unroll
      for (int j = 0; j < 8; ++j) a[c] = fma(xd[j], static_cast<double>(__bfloat162float(we[j])), a[c]);
    }
    // the 8 rows' sums over the warp by a transposing reduction: each halving step keeps half of the
    // rows and sends the other half (9 shuffles of doubles instead of 40); lane l ends with row l / 4
    static_assert(kSelChunk == 8, "the transposing reduction is written for 8 rows");
    {
      const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const double keep = u16 ? a[4 + i] : a[i], send = u16 ? a[i] : a[4 + i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const double keep = u8 ? a[2 + i] : a[i], send = u8 ? a[i] : a[2 + i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      {
        const double keep = u4 ? a[1] : a[0], send = u4 ? a[0] : a[1];
        a[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      a[0] += __shfl_xor_sync(0xffffffffu, a[0], 2);
      a[0] += __shfl_xor_sync(0xffffffffu, a[0], 1);
    }
    if ((lane & 3) == 0) sm.part[warp][lane >> 2] = a[0];
    __syncthreads();
    if (tid < kSelChunk && c0 + tid < nc) {
      double sum = 0.0;
#pragma unroll
      for (int w = 0; w < kSelThreads / 32; ++w) sum += sm.part[w][tid];
      const float v = __double2float_rn(sum);
      const int row = sm.cand[c0 + tid];
      if (row < E)
        sm.fx[row] = logit_map(p, v, row);
      else
        sm.gcoef = bf16_round(1.f / (1.f + expf(-bf16_round(v))));
    }
    __syncthreads();
  }
  if (warp != 0) return;
  // selection among the candidates (exact values), softmax over all, renormalise
  float fx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    fx[i] = e < E ? sm.fx[e] : -FLT_MAX;
  }
  int sel_e[8];
  float sel_v[8];
  const int nr = nc - (gate_row ? 1 : 0);  // routed candidates, in ascending expert order
  if (nr <= 32) {
    // lane c ranks candidate c by counting the larger keys: the order of the top-8 merge (exact
    // logit descending, ties to the lower expert); the selections are the ranks below K
    const int ce = lane < nr ? sm.cand[lane] : 0;
    const uint64_t ck = lane < nr ? (static_cast<uint64_t>(order_key(sm.fx[ce])) << 32) | static_cast<uint32_t>(~ce) : 0ull;
    int rank = 0;
    for (int j = 0; j < nr; ++j) rank += __shfl_sync(0xffffffffu, ck, j) > ck ? 1 : 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const unsigned who = __ballot_sync(0xffffffffu, lane < nr && rank == j);
      const int src = who ? __ffs(who) - 1 : 0;
      const uint64_t kj = __shfl_sync(0xffffffffu, ck, src);
      sel_e[j] = who ? static_cast<int>(~static_cast<uint32_t>(kj)) : 0;
      sel_v[j] = who ? key_value(static_cast<uint32_t>(kj >> 32)) : -FLT_MAX;
    }
  } else {
    uint64_t k[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      k[i] = (e < E && sm.is_cand[e]) ? (static_cast<uint64_t>(order_key(fx[i])) << 32) | static_cast<uint32_t>(~e) : 0ull;
    }
    warp_top8(k);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sel_e[j] = static_cast<int>(~static_cast<uint32_t>(k[j]));
      sel_v[j] = key_value(static_cast<uint32_t>(k[j] >> 32));
    }
  }
  const float m = sel_v[0];
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (lane + 32 * i < E) z += expf(fx[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  int my_e = 0;
  float my_v = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (lane == j) {
      my_e = sel_e[j];
      my_v = sel_v[j];
    }
  const float my_p = expf(my_v - m) / z;
  float psum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    const float pj = __shfl_sync(0xffffffffu, my_p, j);
    if (j < K) psum += pj;
  }
  if (lane < K) {
    const __nv_bfloat16 wb = __float2bfloat16_rn(my_p / psum);
    pair_e[lane] = my_e;
    pair_w[lane] = __bfloat162float(wb);
    if (p.ids_out) p.ids_out[t * K + lane] = my_e;
    if (p.w_out) p.w_out[t * K + lane] = wb;
  }
  if (lane == 0) ws_at<float>(p, L.gate)[t] = gate_row ? sm.gcoef : 1.f;
}

// ------------------------------------------------------------------ dispatch kernel
// Plan and dispatch in one launch. The dispatch order is the stable sort of the (token, k) pairs
// by expert (argsort(ids.flatten(), stable=True)): pair i of expert e goes to position
// off[e] + (pairs of expert e before i). A "pair CTA" owns pairs [a, b): it counts every pair's
// expert and those before a (one pass over the T * K expert ids, from L2), scans the counts into
// offsets, ranks its own pairs in order, and writes each pair's position and copies its token's
// hi + lo rows (the exact e4m3 split of x * 2^e, e from the token's absolute maximum, made once per
// token by the select kernel) to it. "Shared CTAs" write the shared expert's positions P + t. CTA 0 also writes the tile list (ceil(n_e / 64) tiles
// per expert in expert order, then the shared expert's tiles), the per-expert offsets and the
// counts the expert kernels read.
constexpr int kDispThreads = 256;
constexpr int kDispWarps = kDispThreads / 32;
constexpr int kMaxPpc = 1024;  // pairs per CTA (T * K <= 256 * kMaxPpc)

// Pairs per dispatch CTA: at least 16 (two rows per warp to split and place; every CTA also counts all
// pairs, so fewer pairs per CTA trade row latency for redundant counting: 16 measured 3.3 µs faster
// per prefill layer than 32 at T = 512)
__host__ __device__ inline int pairs_per_cta(int P) {
  const int ppc = (P + 255) / 256;
  return ppc < 16 ? 16 : (ppc + 15) / 16 * 16;
}

// Splits token row t into the hi / lo rows of position pos (one warp).
__device__ __forceinline__ void split_row(const Params& p, const Layout& L, int pos, int t, int lane) {
  const int ex = __ldcg(ws_at<const int>(p, L.xexp) + t);
  const float sc = exp2i(ex);
  if (lane == 0) ws_at<float>(p, L.pxinv)[pos] = exp2i(-ex);
  const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * p.H);
  uint8_t* hi_row = p.ws + L.pimg + static_cast<size_t>(pos) * p.H;
  uint8_t* lo_row = p.ws + L.pimg + static_cast<size_t>(L.npos + pos) * p.H;
  constexpr int kC = kMaxH / 16 / 32;  // 16-element chunks per lane at H = 2048
  uint4 v[kC][2];
#pragma unroll
  for (int i = 0; i < kC; ++i) {
    const int c = lane + 32 * i;
    if (c < p.H / 16) {
      v[i][0] = __ldg(src + 2 * c);
      v[i][1] = __ldg(src + 2 * c + 1);
    }
  }
#pragma unroll
  for (int i = 0; i < kC; ++i) {
    const int c = lane + 32 * i;
    if (c < p.H / 16) {
      uint4 hi, lo;
      split16(v[i], sc, hi, lo);
      *reinterpret_cast<uint4*>(hi_row + 16 * c) = hi;
      *reinterpret_cast<uint4*>(lo_row + 16 * c) = lo;
    }
  }
}

// The received pairs of an expert-parallel destination, in (source rank, slot) order: pair r is
// slot r - pre[s] of source s's region.
struct RecvPairs {
  int pre[kMaxRanks + 1];
  __device__ __forceinline__ void locate(int r, int world, int& src, int& slot) const {
    src = 0;
#pragma unroll
    for (int s = 1; s < kMaxRanks; ++s)
      if (s < world && r >= pre[s]) src = s;
    slot = r - pre[src];
  }
};

// Copies a received pair's hi / lo rows (adjacent in the staging area) into position pos of the hi
// and lo planes (one warp).
__device__ __forceinline__ void copy_row(const Params& p, const Layout& L, const uint8_t* srow, int pos, int lane) {
  uint4* hi_row = reinterpret_cast<uint4*>(p.ws + L.pimg + static_cast<size_t>(pos) * p.H);
  uint4* lo_row = reinterpret_cast<uint4*>(p.ws + L.pimg + static_cast<size_t>(L.npos + pos) * p.H);
  const int h16 = p.H / 16, n16 = 2 * h16;
  constexpr int kC = 2 * kMaxH / 16 / 32;
  uint4 v[kC];
#pragma unroll
  for (int i = 0; i < kC; ++i)
    if (lane + 32 * i < n16) v[i] = __ldcg(reinterpret_cast<const uint4*>(srow) + lane + 32 * i);
#pragma unroll
  for (int i = 0; i < kC; ++i) {
    const int c = lane + 32 * i;
    if (c < h16)
      hi_row[c] = v[i];
    else if (c < n16)
      lo_row[c - h16] = v[i];
  }
}

__global__ void __launch_bounds__(kDispThreads) dispatch_kernel(const __grid_constant__ Params p) {
  __shared__ int hist[kMaxRouter], before[kMaxRouter], off[kMaxRouter + 1], tbase[kMaxRouter + 1];
  __shared__ int spos[kMaxPpc];
  __shared__ RecvPairs rp;
  __shared__ int s_ok;
  const Layout L = layout_of(p);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool ep = p.world > 1;
  const int K = p.K, T = p.T;
  const int E = ep ? p.ep_el : p.E;  // experts whose tiles are built here
  const int cap = L.cap;             // pair slots (single GPU: T * K)
  const int ppc = pairs_per_cta(cap);
  const int n_pair_ctas = (cap + ppc - 1) / ppc;
  griddep_wait();
  griddep_launch();
  if (static_cast<int>(blockIdx.x) >= n_pair_ctas) {
    // the shared expert's positions: one warp per local token
    const int t = (blockIdx.x - n_pair_ctas) * kDispWarps + warp;
    if (p.sh_w13 != nullptr && t < T) {
      if (lane == 0) ws_at<int>(p, L.pos_tok)[cap + t] = t;
      split_row(p, L, cap + t, t, lane);
    }
    return;
  }
  // the pairs: this rank's own (single GPU) or the ones every source rank sent here
  const uint8_t* arena = ep ? p.ep_arena[p.rank] : nullptr;
  const EpLayout A = ep_layout(p.world > 1 ? p.world : 1, p.ep_tl, K, p.H);
  int R = cap;
  if (ep) {
    if (tid == 0) s_ok = 1;
    __syncthreads();
    const uint32_t epoch = __ldcg(reinterpret_cast<const uint32_t*>(arena + A.ctrl) + EP_EPOCH);
    if (tid < p.world && !wait_epoch(reinterpret_cast<const uint32_t*>(arena + A.rflag) + tid, epoch)) {
      flag(p, STATUS_TIMEOUT);
      s_ok = 0;
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int s = 0; s <= kMaxRanks; ++s) {
        rp.pre[s] = acc;
        if (s < p.world && s_ok) acc += min(static_cast<int>(__ldcg(reinterpret_cast<const uint32_t*>(arena + A.rcount) + s)), A.slots);
      }
      if (!s_ok) rp.pre[kMaxRanks] = 0;
    }
    __syncthreads();
    R = s_ok ? rp.pre[p.world] : 0;
  }
  const int2* rmeta = ep ? reinterpret_cast<const int2*>(arena + A.rmeta) : nullptr;
  const int* pair_e = ws_at<const int>(p, L.pair_e);
  auto expert_of = [&](int i) -> int {
    if (!ep) return __ldcg(pair_e + i);
    int src, slot;
    rp.locate(i, p.world, src, slot);
    return __ldcg(&rmeta[src * A.slots + slot].x) >> 20;
  };
  const int a = blockIdx.x * ppc, b = min(R, a + ppc);
  for (int e = tid; e < kMaxRouter; e += kDispThreads) {
    hist[e] = 0;
    before[e] = 0;
  }
  __syncthreads();
  for (int i0 = 4 * tid; i0 < R; i0 += 4 * kDispThreads) {
    int ev[4];
    if (!ep && i0 + 3 < R && (R & 3) == 0) {
      const int4 v = __ldcg(reinterpret_cast<const int4*>(pair_e + i0));
      ev[0] = v.x, ev[1] = v.y, ev[2] = v.z, ev[3] = v.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) ev[u] = i0 + u < R ? expert_of(i0 + u) : -1;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (ev[u] >= 0) {
        atomicAdd(&hist[ev[u]], 1);
        if (i0 + u < a) atomicAdd(&before[ev[u]], 1);
      }
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scans of the counts and of the tile counts (8 experts per lane, in order)
    const int per_l = (E + 31) / 32;
    int s = 0, st = 0;
    for (int j = 0; j < per_l; ++j) {
      const int e = lane * per_l + j;
      if (e < E) {
        s += hist[e];
        st += (hist[e] + kTileTok - 1) / kTileTok;
      }
    }
    int incl = s, inclt = st;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, o), y = __shfl_up_sync(0xffffffffu, inclt, o);
      if (lane >= o) {
        incl += x;
        inclt += y;
      }
    }
    int base = incl - s, tb = inclt - st;
    for (int j = 0; j < per_l; ++j) {
      const int e = lane * per_l + j;
      if (e < E) {
        off[e] = base;
        tbase[e] = tb;
        base += hist[e];
        tb += (hist[e] + kTileTok - 1) / kTileTok;
      }
    }
    if (lane == 31) {
      off[E] = incl;
      tbase[E] = inclt;
    }
    __syncwarp();
    // ranks of this CTA's pairs, in pair order, 32 at a time
    int* pos_tok = ws_at<int>(p, L.pos_tok);
    int* inv = ws_at<int>(p, L.inv);
    for (int i0 = a; i0 < b; i0 += 32) {
      const int i = i0 + lane;
      const int e = i < b ? expert_of(i) : -1;
      const unsigned m = __match_any_sync(0xffffffffu, e);
      const int rank = e >= 0 ? before[e] + __popc(m & ((1u << lane) - 1u)) : 0;
      __syncwarp();
      if (e >= 0 && lane == __ffs(m) - 1) before[e] += __popc(m);
      __syncwarp();
      const int pos = e >= 0 ? off[e] + rank : -1;
      if (i < b) {
        spos[i - a] = pos;
        if (!ep) {
          inv[i] = pos;
          if (pos >= 0) {
            pos_tok[pos] = i / K;
            if (p.perm_out) p.perm_out[pos] = i;
          }
        }
      }
    }
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    const int nt_routed = tbase[E];
    const int nt_sh = p.sh_w13 != nullptr ? (T + kTileTok - 1) / kTileTok : 0;
    int4* tiles = ws_at<int4>(p, L.tiles);
    for (int e = tid; e < E; e += kDispThreads) {
      const int n = hist[e];
      for (int j = 0; j * kTileTok < n; ++j)
        tiles[tbase[e] + j] = make_int4(e, off[e] + j * kTileTok, min(kTileTok, n - j * kTileTok), 0);
    }
    for (int j = tid; j < nt_sh; j += kDispThreads)
      tiles[nt_routed + j] = make_int4(-1, cap + j * kTileTok, min(kTileTok, T - j * kTileTok), 0);
    if (p.offsets_out)
      for (int e = tid; e <= E; e += kDispThreads) p.offsets_out[e] = off[e];
    if (tid == 0) {
      uint32_t* c = ws_at<uint32_t>(p, L.ctrl);
      c[C_NTILES] = static_cast<uint32_t>(nt_routed + nt_sh);
      c[C_NVALID] = static_cast<uint32_t>(off[E]);
    }
  }
  // the permuted activation rows of this CTA's pairs
  for (int j = warp; j < b - a; j += kDispWarps) {
    const int pos = spos[j];
    if (pos < 0) continue;
    if (!ep) {
      split_row(p, L, pos, (a + j) / K, lane);
    } else {
      int src, slot;
      rp.locate(a + j, p.world, src, slot);
      const int2 m = __ldcg(&rmeta[src * A.slots + slot]);
      const int row = m.y >> 9, ex = (m.y & 0x1FF) - 256;  // the pair's token row, its split exponent
      if (lane == 0) {
        ws_at<float>(p, L.pxinv)[pos] = exp2i(-ex);
        ws_at<int>(p, L.pos_tok)[pos] = (src << 20) | (m.x & 0xFFFFF);  // where the output row goes
      }
      copy_row(p, L, arena + A.stage + (static_cast<size_t>(src) * A.slots + row) * 2 * p.H, pos, lane);
    }
  }
}

// ------------------------------------------------------------------ expert-parallel dispatch
// Source side: every pair of this rank's tokens goes to the rank owning its expert. CTA c owns
// pairs [a, b); it counts each destination's pairs (all, and those before a), ranks its own in
// order within their destination, and writes each pair's split x rows and metadata into the
// destination's stage / rmeta region of this source over NVLink. The last CTA to finish (counted on
// a local counter after a system-scope fence by each CTA) writes every destination's count and then
// its flag (the call's epoch, with a system-scope release), and advances the local epoch.
__global__ void __launch_bounds__(kDispThreads) ep_dispatch_kernel(const __grid_constant__ Params p) {
  __shared__ int dcount[kMaxRanks], dbefore[kMaxRanks], rbefore[kMaxRanks];
  __shared__ int spos[kMaxPpc], srow[kMaxPpc];
  __shared__ int s_last;
  const Layout L = layout_of(p);
  const EpLayout A = ep_layout(p.world, p.ep_tl, p.K, p.H);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K, P = p.T * K, W = p.world;
  const int ppc = pairs_per_cta(P);
  const int a = blockIdx.x * ppc, b = min(P, a + ppc);
  uint32_t* own_ctrl = reinterpret_cast<uint32_t*>(p.ep_arena[p.rank] + A.ctrl);
  griddep_wait();
  griddep_launch();
  const uint32_t epoch = __ldcg(own_ctrl + EP_EPOCH) + 1u;
  if (tid < kMaxRanks) {
    dcount[tid] = 0;
    dbefore[tid] = 0;
    rbefore[tid] = 0;
  }
  __syncthreads();
  const int* pair_e = ws_at<const int>(p, L.pair_e);
  // A token's row goes to a destination once, with its first pair (in k order) to that rank; the
  // token's other pairs there point at that row. Rows are numbered per destination in pair order.
  // (When K does not divide a CTA's pair range or a 32-lane round, every pair carries its own row.)
  const bool share = (ppc % K) == 0 && (32 % K) == 0;
  auto dest = [&](int i) { return ep_place(p, __ldcg(pair_e + i)) >> 16; };
  if (share) {
    // one token per thread: its pairs' ranks, and which pair is the first to each rank
    for (int t = tid; t < p.T; t += kDispThreads) {
      int dk[kMaxTopK];
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k) dk[k] = k < K ? dest(t * K + k) : -1;
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k) {
        if (k >= K) break;
        const int d = dk[k];
        atomicAdd(&dcount[d], 1);
        if (t * K + k < a) {
          atomicAdd(&dbefore[d], 1);
          bool first = true;
#pragma unroll
          for (int k2 = 0; k2 < kMaxTopK; ++k2)
            if (k2 < k && dk[k2] == d) first = false;
          if (first) atomicAdd(&rbefore[d], 1);
        }
      }
    }
  } else {
    for (int i = tid; i < P; i += kDispThreads) {
      const int d = dest(i);
      atomicAdd(&dcount[d], 1);
      if (i < a) {
        atomicAdd(&dbefore[d], 1);
        atomicAdd(&rbefore[d], 1);
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    // pair slots and row slots of this CTA's pairs, in pair order (when rows are shared, a token's K
    // pairs lie in one 32-lane round)
    for (int i0 = a; i0 < b; i0 += 32) {
      const int i = i0 + lane;
      const int d = i < b ? dest(i) : -1;
      const unsigned m = __match_any_sync(0xffffffffu, d);
      const int rank = d >= 0 ? dbefore[d] + __popc(m & ((1u << lane) - 1u)) : 0;
      bool owner = d >= 0;
      if (share) {
        const int k = i % K;
        for (int j = 1; j < kMaxTopK; ++j) {
          const int dj = __shfl_sync(0xffffffffu, d, lane >= j ? lane - j : lane);
          if (j <= k && dj == d) owner = false;
        }
      }
      const unsigned mo = m & __ballot_sync(0xffffffffu, owner);
      int row = d >= 0 ? rbefore[d] + __popc(mo & ((1u << lane) - 1u)) : 0;
      // a shared row's slot is that of the token's first pair to the same rank
      const unsigned mt = __match_any_sync(0xffffffffu, share ? (i / K) * kMaxRanks + (d < 0 ? 0 : d) : i);
      const int row_owner = __ffs(mt & __ballot_sync(0xffffffffu, owner)) - 1;
      const int shared_row = __shfl_sync(0xffffffffu, row, row_owner < 0 ? lane : row_owner);
      if (!owner) row = shared_row;
      __syncwarp();
      if (d >= 0 && lane == __ffs(m) - 1) {
        dbefore[d] += __popc(m);
        rbefore[d] += __popc(mo);
      }
      __syncwarp();
      if (i < b) {
        spos[i - a] = (d << 24) | rank;
        srow[i - a] = owner ? row : -1 - row;
      }
    }
  }
  __syncthreads();
  for (int j = warp; j < b - a; j += kDispWarps) {
    const int i = a + j, t = i / K;
    const int d = spos[j] >> 24, slot = spos[j] & 0xFFFFFF;
    const bool owner = srow[j] >= 0;
    const int row = owner ? srow[j] : -1 - srow[j];
    const int e_local = ep_place(p, __ldcg(pair_e + i)) & 0xFFFF;
    uint8_t* dst_arena = p.ep_arena[d];
    const size_t sidx = static_cast<size_t>(p.rank) * A.slots + slot;
    const size_t ridx = static_cast<size_t>(p.rank) * A.slots + row;
    const int ex = __ldcg(ws_at<const int>(p, L.xexp) + t);
    // metadata: (local expert, pair index), (the token's row slot, split exponent + 256 in 9 bits)
    if (lane == 0)
      reinterpret_cast<int2*>(dst_arena + A.rmeta)[sidx] =
          make_int2((e_local << 20) | i, (row << 9) | ((ex + 256) & 0x1FF));
    if (!owner) continue;  // the token's row already goes to this rank with an earlier pair
    const float sc = exp2i(ex);
    const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * p.H);
    uint8_t* hi_row = dst_arena + A.stage + ridx * 2 * p.H;
    uint8_t* lo_row = hi_row + p.H;
    constexpr int kC = kMaxH / 16 / 32;
    uint4 v[kC][2];
#pragma unroll
    for (int c0 = 0; c0 < kC; ++c0) {
      const int c = lane + 32 * c0;
      if (c < p.H / 16) {
        v[c0][0] = __ldg(src + 2 * c);
        v[c0][1] = __ldg(src + 2 * c + 1);
      }
    }
#pragma unroll
    for (int c0 = 0; c0 < kC; ++c0) {
      const int c = lane + 32 * c0;
      if (c < p.H / 16) {
        uint4 hi, lo;
        split16(v[c0], sc, hi, lo);
        *reinterpret_cast<uint4*>(hi_row + 16 * c) = hi;
        *reinterpret_cast<uint4*>(lo_row + 16 * c) = lo;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();  // cumulative: this CTA's peer writes, seen through the barrier
    s_last = atomicAdd(own_ctrl + EP_DISP_COUNT, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (s_last) {
    if (tid < W) {
      __threadfence_system();
      uint8_t* dst_arena = p.ep_arena[tid];
      reinterpret_cast<uint32_t*>(dst_arena + A.rcount)[p.rank] = static_cast<uint32_t>(dcount[tid]);
      st_release_sys(reinterpret_cast<uint32_t*>(dst_arena + A.rflag) + p.rank, epoch);
    }
    if (tid == 0) {
      own_ctrl[EP_DISP_COUNT] = 0u;
      own_ctrl[EP_EPOCH] = epoch;
    }
  }
}

// ------------------------------------------------------------------ up / down kernels
constexpr int kMaxItems = 64;  // items per CTA whose descriptors are staged in shared memory

struct Aux {
  int4 items[kMaxItems];  // (expert or -1, first position, tokens, row block) of the CTA's items
  uint64_t full[8], empty[8];
  uint64_t acc_full[4], acc_empty[4];
  // up: turn[g] completes when the other epilogue group has released every accumulator of the
  // item before group g's next one, so no group waits on an accumulator barrier more than one
  // phase ahead of the MMAs
  uint64_t turn[2];
  uint64_t mma_done, mma_done2;
  uint32_t tmem;
  int abort;
  int last;  // expert parallel, down: this CTA finished last
  float amax[2][2][2][4][32];  // up: [group][item parity][token half][lane quarter][token] |h| maxima
};

// Activation box of a tile of n tokens (index 0-3 for n <= 8, 16, 32, 64). Up: n rows of the hi
// plane and n of the lo plane, each rounded up to 16, 16, 32 or 64 rows (the MMA's N; M = 128 needs a
// multiple of 16). Down: the 2n interleaved hi / lo rows, rounded up to 16, 32, 64 or 128.
__device__ __forceinline__ int box_index(int n) { return n <= 8 ? 0 : n <= 16 ? 1 : n <= 32 ? 2 : 3; }
__host__ __device__ constexpr int up_box_rows(int bi) { return bi <= 1 ? 16 : (8 << bi); }

// Item k of this CTA (k-th of blockIdx.x, blockIdx.x + gridDim.x, ...): staged in shared memory at
// kernel start, read from the tile list beyond kMaxItems.
__device__ __forceinline__ int4 item_desc(const Aux& aux, const int4* tiles, int nrb, int k) {
  if (k < kMaxItems) return aux.items[k];
  const int idx = blockIdx.x + k * gridDim.x;
  const int4 tl = __ldcg(tiles + idx / nrb);
  return make_int4(tl.x, tl.y, tl.z, idx % nrb);
}

template <bool DOWN>
__global__ void __launch_bounds__(expert_threads(DOWN), 1)
    expert_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map_w,
                  const __grid_constant__ CUtensorMap map_sh, const __grid_constant__ CUtensorMap map_b0,
                  const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_b2,
                  const __grid_constant__ CUtensorMap map_b3) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int kBOff = 2 * kSlab;  // activation slab inside a stage
  constexpr int kNacc = n_acc(DOWN);
  constexpr uint32_t kAccCols = acc_cols(DOWN);
  Aux& aux = *reinterpret_cast<Aux*>(smem + kStages * kStage);
  const Layout L = layout_of(p);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // items: up 128 gate rows + the matching 128 up rows; down 256 output rows (two 128-row halves)
  const int nrb = DOWN ? p.H / (2 * kRows) : p.I / kRows;
  const int nkb = (DOWN ? p.I : p.H) / 128;    // k slabs per item
  // the tile list is written by the dispatch kernel: the up kernel (its successor) waits for it,
  // the down kernel (two launches later) finds it complete
  if (!DOWN) griddep_wait();
  const int ntiles = static_cast<int>(__ldcg(ws_at<const uint32_t>(p, L.ctrl) + C_NTILES));
  const int n_items = ntiles * nrb;
  const int my_items = n_items > static_cast<int>(blockIdx.x) ? (n_items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int4* tiles = ws_at<const int4>(p, L.tiles);
  volatile int* abort = &aux.abort;

  if (tid < my_items && tid < kMaxItems) {
    const int idx = blockIdx.x + tid * gridDim.x;
    const int4 tl = __ldcg(tiles + idx / nrb);
    aux.items[tid] = make_int4(tl.x, tl.y, tl.z, idx % nrb);
  }
  if (tid == 0) {
    tc::prefetch_map(&map_w);
    if (p.sh_w13) tc::prefetch_map(&map_sh);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&aux.full[s], 1);
      mbar_init(&aux.empty[s], 1);
    }
    for (int a = 0; a < kNacc; ++a) {
      mbar_init(&aux.acc_full[a], 1);
      mbar_init(&aux.acc_empty[a], kEpiWarps);
    }
    mbar_init(&aux.turn[0], kEpiWarps);
    mbar_init(&aux.turn[1], kEpiWarps);
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
      const int total = my_items * nkb;
      auto issue_a = [&](int s, const int4& it, int kb) {
        const CUtensorMap* map = it.x < 0 ? &map_sh : &map_w;
        const int plane = it.x < 0 ? 0 : it.x;
        uint8_t* dst = smem + (s % kStages) * kStage;
        uint64_t* bar = &aux.full[s % kStages];
        const int bi = box_index(it.z);
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kBOff + (DOWN ? (16 << bi) : 2 * up_box_rows(bi)) * 128));
        const int row0 = DOWN ? 2 * kRows * it.w : kRows * it.w;
        const int row1 = DOWN ? row0 + kRows : p.I + kRows * it.w;
        tc::tma_load_3d(dst, map, kb * 128, row0, plane, bar);
        tc::tma_load_3d(dst + kSlab, map, kb * 128, row1, plane, bar);
      };
      auto issue_b = [&](int s, const int4& it, int kb) {
        const int bi = box_index(it.z);
        const CUtensorMap* map = bi == 0 ? &map_b0 : bi == 1 ? &map_b1 : bi == 2 ? &map_b2 : &map_b3;
        uint8_t* dst = smem + (s % kStages) * kStage + kBOff;
        if (DOWN) {
          tc::tma_load_3d(dst, map, kb * 128, 2 * it.y, 0, &aux.full[s % kStages]);
        } else {
          // the tile's hi rows, then its lo rows, from the two planes of the activation image
          tc::tma_load_3d(dst, map, kb * 128, it.y, 0, &aux.full[s % kStages]);
          tc::tma_load_3d(dst + up_box_rows(bi) * 128, map, kb * 128, it.y, 1, &aux.full[s % kStages]);
        }
      };
      // the weight slabs of the first ring before the wait; activation slabs (from the preceding
      // kernel) after it
      const int first = min(total, kStages);
      for (int s = 0; s < first; ++s) issue_a(s, item_desc(aux, tiles, nrb, s / nkb), s % nkb);
      griddep_wait();
      griddep_launch();
      for (int s = 0; s < first; ++s) issue_b(s, item_desc(aux, tiles, nrb, s / nkb), s % nkb);
      int k = first / nkb, kb = first % nkb;
      int4 it = item_desc(aux, tiles, nrb, k < my_items ? k : 0);
      for (int s = first; s < total; ++s) {
        wait_or_abort(p, &aux.empty[s % kStages], ((s / kStages) & 1) ^ 1u, abort);
        issue_a(s, it, kb);
        issue_b(s, it, kb);
        if (++kb == nkb) {
          kb = 0;
          if (++k < my_items) it = item_desc(aux, tiles, nrb, k);
        }
      }
      // nothing may still be copying into shared memory when the CTA exits (bounded waits, also
      // after an abort)
      for (int s = max(0, total - kStages); s < total; ++s) mbar_wait(&aux.full[s % kStages], (s / kStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1 || warp == expert_threads(DOWN) / 32 - 1) {
    // ================================================================ MMA issuers (lane 0): warp 1 the
    // even accumulator uses (buffer 0), the last warp the odd ones (buffer 1)
    const int par = warp == 1 ? 0 : 1;
    if (lane == 0) {
      int s = 0, use = 0;
      for (int k = 0; k < my_items; ++k) {
        const int4 it = item_desc(aux, tiles, nrb, k);
        const int bi = box_index(it.z);
        const int nb = DOWN ? (16 << bi) : up_box_rows(bi);  // the MMA's N
        const uint32_t idesc = tc::idesc_e4m3(kRows, nb);
        for (int kb = 0; kb < nkb; ++kb, ++s, ++use) {
          const int ab = use % kNacc;
          if ((ab & 1) != par) continue;
          wait_or_abort(p, &aux.acc_empty[ab], ((use / kNacc) & 1) ^ 1u, abort);
          wait_or_abort(p, &aux.full[s % kStages], (s / kStages) & 1, abort);
          tc::fence_after_sync();
          const uint32_t a = smem_u32(smem + (s % kStages) * kStage);
          const uint32_t b = a + kBOff;
          const uint32_t d = tmem + ab * kAccCols;
          if (DOWN) {
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              tc::mma_f8(d, tc::smem_desc(a + 32 * k4), tc::smem_desc(b + 32 * k4), idesc, k4 > 0);
              tc::mma_f8(d + 128, tc::smem_desc(a + kSlab + 32 * k4), tc::smem_desc(b + 32 * k4), idesc, k4 > 0);
            }
          } else {
            // x = hi + lo exactly: both halves of a token add into its column (gate rows in columns
            // [0, 64), up rows in [64, 128))
            const uint32_t blo = b + nb * 128;
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              tc::mma_f8(d, tc::smem_desc(a + 32 * k4), tc::smem_desc(b + 32 * k4), idesc, k4 > 0);
              tc::mma_f8(d, tc::smem_desc(a + 32 * k4), tc::smem_desc(blo + 32 * k4), idesc, true);
              tc::mma_f8(d + 64, tc::smem_desc(a + kSlab + 32 * k4), tc::smem_desc(b + 32 * k4), idesc, k4 > 0);
              tc::mma_f8(d + 64, tc::smem_desc(a + kSlab + 32 * k4), tc::smem_desc(blo + 32 * k4), idesc, true);
            }
          }
          tc::mma_commit(&aux.empty[s % kStages]);
          tc::mma_commit(&aux.acc_full[ab]);
        }
      }
      tc::mma_commit(par ? &aux.mma_done2 : &aux.mma_done);
      wait_or_abort(p, par ? &aux.mma_done2 : &aux.mma_done, 0, abort);
    }
    __syncwarp();
  } else {
    // ================================================================ epilogue (warps 2-9 [, 10-17])
    constexpr int kGroups = epi_groups(DOWN);
    const int grp = (warp - 2) >> 3;  // this warp's group: items grp, grp + kGroups, ...
    const int q = warp & 3, hf = ((warp - 2) >> 2) & 1;
    const int r = 32 * q + lane;
    if (DOWN) griddep_wait();  // the h blocks' scales come from the up kernel
    // per-item token data, fetched one item ahead: up 2^-e of each token's x split, down the
    // token's 2^-e of each 128-block of h
    // (down, expert parallel: the token's output row destination, source rank << 20 | pair index)
    auto token_data = [&](const int4& it, float (&v)[kMaxI / 128], int& rm) {
      const int nh = min(max(it.z - 32 * hf, 0), 32);
      const int pos = it.y + 32 * hf + lane;
#pragma unroll
      for (int kb = 0; kb < kMaxI / 128; ++kb) v[kb] = 0.f;
      rm = -1;
      if (lane < nh) {
        if (!DOWN) {
          v[0] = __ldcg(ws_at<const float>(p, L.pxinv) + pos);
        } else {
#pragma unroll
          for (int kb = 0; kb < kMaxI / 128; ++kb)
            if (kb < nkb) v[kb] = __ldcg(ws_at<const float>(p, L.hinv) + static_cast<size_t>(pos) * nkb + kb);
          if (p.world > 1 && it.x >= 0) rm = __ldcg(ws_at<const int>(p, L.pos_tok) + pos);
        }
      }
    };
    auto scale_row = [&](const int4& it, bool second) -> const float* {
      // block scales of this thread's weight row in the item's first or second 128-row half:
      // [rows / srows][nkb] per expert
      const bool shared_tile = it.x < 0;
      const int srows = shared_tile ? p.sh_srows : p.srows;
      if (!DOWN) {
        const float* s13 = shared_tile ? p.sh_s13 : p.s13 + static_cast<size_t>(it.x) * p.s13_stride;
        const int row = (second ? p.I : 0) + kRows * it.w + r;
        return s13 + static_cast<size_t>(row / srows) * nkb;
      }
      const float* s2 = shared_tile ? p.sh_s2 : p.s2 + static_cast<size_t>(it.x) * p.s2_stride;
      return s2 + static_cast<size_t>((2 * kRows * it.w + (second ? kRows : 0) + r) / srows) * nkb;
    };
    int4 it_next = grp < my_items ? item_desc(aux, tiles, nrb, grp) : make_int4(0, 0, 0, 0);
    float td_next[kMaxI / 128];
    int rm_next = -1;
    float sg_next = 0.f, su_next = 0.f;  // the next item's first-slab scales
    if (grp < my_items) {
      token_data(it_next, td_next, rm_next);
      sg_next = __ldg(scale_row(it_next, false));
      su_next = __ldg(scale_row(it_next, true));
    }
    for (int k = grp; k < my_items; k += kGroups) {
      int use = k * nkb;  // accumulator uses run over (item, slab) in the MMA's order
      const int4 it = it_next;
      float td[kMaxI / 128];
#pragma unroll
      for (int i = 0; i < kMaxI / 128; ++i) td[i] = td_next[i];
      float sg = sg_next, su = su_next;
      const int rm = rm_next;
      if (k + kGroups < my_items) {
        it_next = item_desc(aux, tiles, nrb, k + kGroups);
        token_data(it_next, td_next, rm_next);
        sg_next = __ldg(scale_row(it_next, false));
        su_next = __ldg(scale_row(it_next, true));
      }
      if (kGroups > 1 && k > 0) {
        // item k's accumulators follow item k - 1's, which the other group reads
        bool t_ok = true;
        if (lane == 0) t_ok = wait_or_abort(p, &aux.turn[k & 1], ((k - 1) >> 1) & 1, abort);
        __syncwarp();
        (void)t_ok;
      }
      const int nh = min(max(it.z - 32 * hf, 0), 32);  // this warp's tokens of the tile
      const int pbase = it.y + 32 * hf;
      const bool shared_tile = it.x < 0;
      const float* sgp = scale_row(it, false);
      const float* sup = scale_row(it, true);
      float a0[32], a1[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) a0[j] = a1[j] = 0.f;
      // the up kernel's 16 slabs stay a rolled loop: unrolled, its code would push the item tail
      // out of the instruction cache on every item
#pragma unroll(DOWN ? kMaxI / 128 : 1)
      for (int kb = 0; kb < (DOWN ? kMaxI / 128 : nkb); ++kb) {
        if (kb < nkb) {
          // the next slab's scales are requested before this slab's accumulator is read
          float sg_n = 0.f, su_n = 0.f;
          if (kb + 1 < nkb) {
            sg_n = __ldg(sgp + kb + 1);
            su_n = __ldg(sup + kb + 1);
          }
          const int ab = use % kNacc;
          bool ready = true;
          if (lane == 0) ready = wait_or_abort(p, &aux.acc_full[ab], (use / kNacc) & 1, abort);
          ready = __shfl_sync(0xffffffffu, ready, 0);
          ++use;
          tc::fence_after_sync();
          if (nh > 0 && ready) {
            const uint32_t ta =
                tmem + (static_cast<uint32_t>(32 * q) << 16) + ab * kAccCols + (DOWN ? 64 : 32) * hf;
            if (!DOWN) {
              // the thread's 32 tokens: one column each (hi + lo summed by the MMAs), gate rows, then up
              // rows; 16 columns per load keep the two groups within their registers
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                float v[16];
                tc::tmem_ld16(ta + 16 * c, v);
                tc::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) a0[16 * c + j] = fmaf(sg, v[j], a0[16 * c + j]);
              }
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                float v[16];
                tc::tmem_ld16(ta + 64 + 16 * c, v);
                tc::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) a1[16 * c + j] = fmaf(su, v[j], a1[16 * c + j]);
              }
            } else {
              float v0[32], v1[32];
              tc::tmem_ld32(ta, v0);
              tc::tmem_ld32(ta + 32, v1);
              tc::tmem_wait_ld();
              float hk = td[0];
#pragma unroll
              for (int i = 1; i < kMaxI / 128; ++i)
                if (kb == i) hk = td[i];
              float hj[32];  // 2^-e of each token's h block
#pragma unroll
              for (int j = 0; j < 32; ++j) hj[j] = __shfl_sync(0xffffffffu, hk, j);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                a0[j] = fmaf(sg * hj[j], v0[2 * j] + v0[2 * j + 1], a0[j]);
                a0[16 + j] = fmaf(sg * hj[16 + j], v1[2 * j] + v1[2 * j + 1], a0[16 + j]);
              }
              tc::tmem_ld32(ta + 128, v0);
              tc::tmem_ld32(ta + 160, v1);
              tc::tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                a1[j] = fmaf(su * hj[j], v0[2 * j] + v0[2 * j + 1], a1[j]);
                a1[16 + j] = fmaf(su * hj[16 + j], v1[2 * j] + v1[2 * j + 1], a1[16 + j]);
              }
            }
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&aux.acc_empty[ab]);
          sg = sg_n;
          su = su_n;
        }
      }
      if (kGroups > 1) {
        // every accumulator of item k is released: the other group may start item k + 1
        __syncwarp();
        if (lane == 0) mbar_arrive(&aux.turn[(k + 1) & 1]);
      }
      if (!DOWN) {
        // SwiGLU, h rounded to bf16 (the reference's activation dtype; the shared expert is a chain
        // of bf16 modules), then the per-(token, 128-block) absolute maxima across the 4 quarters
        const int par = (k / kGroups) & 1;
        const float xi = td[0];
        // branch-free over the 32 tokens: the shared expert's extra bf16 roundings are selects, the
        // tokens past the tile's end are zeroed
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float xj = __shfl_sync(0xffffffffu, xi, j);
          float g = a0[j] * xj, u = a1[j] * xj;
          g = shared_tile ? bf16_round(g) : g;
          u = shared_tile ? bf16_round(u) : u;
          float sl = __fdividef(g, 1.f + __expf(-g));
          sl = shared_tile ? bf16_round(sl) : sl;
          const float h = j < nh ? bf16_round(sl * u) : 0.f;
          a0[j] = h;
          a1[j] = fabsf(h);
        }
        // transposing max over the warp's 32 rows: after the halving steps lane j holds the
        // maximum of token j (31 shuffles for all 32 tokens)
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
          const bool upper = (lane & d) != 0;
#pragma unroll
          for (int i = 0; i < d; ++i) {
            const float send = upper ? a1[i] : a1[i + d];
            const float keep = upper ? a1[i + d] : a1[i];
            a1[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, d));
          }
        }
        aux.amax[grp][par][hf][q][lane] = a1[0];
        named_bar(kBarEpi + grp, kEpiThreads);
        float e2[32];
        const int e_mine =
            split_exponent(fmaxf(fmaxf(aux.amax[grp][par][hf][0][lane], aux.amax[grp][par][hf][1][lane]),
                                 fmaxf(aux.amax[grp][par][hf][2][lane], aux.amax[grp][par][hf][3][lane])));
#pragma unroll
        for (int j = 0; j < 32; ++j) e2[j] = exp2i(__shfl_sync(0xffffffffu, e_mine, j));
        uint8_t* himg = p.ws + L.himg + static_cast<size_t>(2 * pbase) * p.I + kRows * it.w + r;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          if (j < nh) {
            uint16_t hi, lo;
            split2(a0[j] * e2[j], a0[j + 1] * e2[j + 1], hi, lo);
            himg[static_cast<size_t>(2 * j) * p.I] = static_cast<uint8_t>(hi & 0xFF);
            himg[static_cast<size_t>(2 * j + 1) * p.I] = static_cast<uint8_t>(lo & 0xFF);
            if (j + 1 < nh) {
              himg[static_cast<size_t>(2 * j + 2) * p.I] = static_cast<uint8_t>(hi >> 8);
              himg[static_cast<size_t>(2 * j + 3) * p.I] = static_cast<uint8_t>(lo >> 8);
            }
          }
        }
        if (q == 0 && lane < nh)
          ws_at<float>(p, L.hinv)[static_cast<size_t>(pbase + lane) * (p.I / 128) + it.w] = exp2i(-e_mine);
      } else {
        const int col = 2 * kRows * it.w + r;
        if (p.world > 1 && !shared_tile) {
          // expert parallel: each row goes straight to its source rank's return buffer over NVLink
          const EpLayout A = ep_layout(p.world, p.ep_tl, p.K, p.H);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int rmj = __shfl_sync(0xffffffffu, rm, j);
            if (j < nh) {
              float* out = reinterpret_cast<float*>(p.ep_arena[rmj >> 20] + A.ret) +
                           static_cast<size_t>(rmj & 0xFFFFF) * p.H + col;
              __stcg(out, a0[j]);
              __stcg(out + kRows, a1[j]);
            }
          }
        } else {
          float* out = ws_at<float>(p, L.outp) + static_cast<size_t>(pbase) * p.H + col;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nh) {
              __stcg(out + static_cast<size_t>(j) * p.H, a0[j]);
              __stcg(out + static_cast<size_t>(j) * p.H + kRows, a1[j]);
            }
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
  if (DOWN && p.world > 1) {
    // the last CTA tells every source rank that its output rows have landed: a system-scope fence
    // per CTA (cumulative over the CTA's stores, ordered by the barrier above), a local counter,
    // then a release of the call's epoch into each source's retflag
    const EpLayout A = ep_layout(p.world, p.ep_tl, p.K, p.H);
    uint32_t* own_ctrl = reinterpret_cast<uint32_t*>(p.ep_arena[p.rank] + A.ctrl);
    if (tid == 0) {
      __threadfence_system();
      aux.last = atomicAdd(own_ctrl + EP_DOWN_COUNT, 1u) == gridDim.x - 1 ? 1 : 0;
    }
    __syncthreads();
    if (aux.last) {
      const uint32_t epoch = __ldcg(own_ctrl + EP_EPOCH);
      if (tid < p.world) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(p.ep_arena[tid] + A.retflag) + p.rank, epoch);
      }
      if (tid == 0) own_ctrl[EP_DOWN_COUNT] = 0u;
    }
  }
}

// ------------------------------------------------------------------ combine kernel
// y = bf16(bf16(bf16(sum_j w_tj * row(t, j)) + bias) + bf16(gate_t * bf16(shared row))): the
// rounding points of fp8_moe_forward's bf16 output, the speaker's bias add (engine.py:237) and
// speaker_forward's bf16 tensor sum (engine.py:158). One thread per 8 outputs.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const __grid_constant__ Params p) {
  const Layout L = layout_of(p);
  const int c8 = p.H / 8;
  const int g = blockIdx.x * kCombineThreads + threadIdx.x;
  const int t = g / c8, n = (g % c8) * 8;
  const bool active = t < p.T;
  float bias[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (active && p.out_bias) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.out_bias + n)), b1 = __ldg(reinterpret_cast<const float4*>(p.out_bias + n + 4));
    bias[0] = b0.x, bias[1] = b0.y, bias[2] = b0.z, bias[3] = b0.w, bias[4] = b1.x, bias[5] = b1.y, bias[6] = b1.z, bias[7] = b1.w;
  }
  const bool ep = p.world > 1;
  const int K = p.K;
  // the pairs' positions and weights (dispatch and select, which completed before the up kernel
  // started) and the shared gate are read before the wait; only the rows come from the down kernel
  int pos[kMaxTopK];
  float w[kMaxTopK];
  float gate = 0.f;
  if (active) {
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      // expert parallel: pair t * K + j's row is row t * K + j of the return buffer
      pos[j] = j < K ? (ep ? t * K + j : __ldcg(ws_at<const int>(p, L.inv) + t * K + j)) : -1;
      w[j] = j < K ? __ldcg(ws_at<const float>(p, L.pair_w) + t * K + j) : 0.f;
    }
    if (p.sh_w13 != nullptr) gate = __ldcg(ws_at<const float>(p, L.gate) + t);
  }
  griddep_wait();
  griddep_launch();
  const EpLayout A = ep_layout(ep ? p.world : 1, p.ep_tl, p.K, p.H);
  if (ep) {
    // every destination rank has written this rank's output rows (bounded wait on its flag; a wait
    // that runs out is reported in the status word)
    const uint8_t* arena = p.ep_arena[p.rank];
    const uint32_t epoch = __ldcg(reinterpret_cast<const uint32_t*>(arena + A.ctrl) + EP_EPOCH);
    if (threadIdx.x < p.world && !wait_epoch(reinterpret_cast<const uint32_t*>(arena + A.retflag) + threadIdx.x, epoch))
      flag(p, STATUS_TIMEOUT);
    __syncthreads();
  }
  if (!active) return;
  const float* outp = ws_at<const float>(p, L.outp);
  const float* rows = ep ? reinterpret_cast<const float*>(p.ep_arena[p.rank] + A.ret) : outp;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (pos[j] >= 0) {
      const float4* row = reinterpret_cast<const float4*>(rows + static_cast<size_t>(pos[j]) * p.H + n);
      const float4 o0 = __ldcg(row), o1 = __ldcg(row + 1);
      acc[0] = fmaf(w[j], o0.x, acc[0]), acc[1] = fmaf(w[j], o0.y, acc[1]), acc[2] = fmaf(w[j], o0.z, acc[2]);
      acc[3] = fmaf(w[j], o0.w, acc[3]), acc[4] = fmaf(w[j], o1.x, acc[4]), acc[5] = fmaf(w[j], o1.y, acc[5]);
      acc[6] = fmaf(w[j], o1.z, acc[6]), acc[7] = fmaf(w[j], o1.w, acc[7]);
    }
  }
  const bool sh = p.sh_w13 != nullptr;
  float shv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (sh) {
    const float4* row = reinterpret_cast<const float4*>(outp + static_cast<size_t>(L.cap + t) * p.H + n);
    const float4 o0 = __ldcg(row), o1 = __ldcg(row + 1);
    shv[0] = o0.x, shv[1] = o0.y, shv[2] = o0.z, shv[3] = o0.w, shv[4] = o1.x, shv[5] = o1.y, shv[6] = o1.z, shv[7] = o1.w;
  }
  __align__(16) __nv_bfloat16 out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float a = bf16_round(acc[i]);
    if (p.out_bias) a = bf16_round(a + bias[i]);
    if (sh) a += bf16_round(gate * bf16_round(shv[i]));
    out[i] = __float2bfloat16_rn(a);
  }
  *reinterpret_cast<uint4*>(p.y + static_cast<size_t>(t) * p.H + n) = *reinterpret_cast<const uint4*>(out);
}

}  // namespace pf

// ------------------------------------------------------------------ host launcher
namespace {

template <typename... KArgs, typename... Args>
int pf_launch(void (*kernel)(KArgs...), dim3 grid, int block, size_t smem, cudaStream_t stream, const char* name,
              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    set_error(std::string(name) + " launch failed: " + cudaGetErrorString(err));
    return 2;
  }
  return 0;
}

constexpr size_t kExpertSmem(bool) {
  return static_cast<size_t>(pf::kStages * pf::kStage) + 1024 +
         ((sizeof(pf::Aux) + 127) / 128) * 128;
}

}  // namespace

size_t prefill_ws_bytes(int T, int H, int I, int E, int K) { return pf::layout(T, H, I, E, K).total; }

// Launches the prefill chain; route = false starts at the select kernel (routing given).
// phases: 1 = routing and (expert parallel) sending the pairs to their owners; 2 = dispatch into
// expert tiles, the expert products, (expert parallel) returning the rows, combine.
int launch_prefill(const pf::Params& p, cudaStream_t stream, int phases = 3) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev);
  const pf::Layout L = pf::layout_of(p);
  static bool attrs_set = false;
  if (!attrs_set) {
    cudaFuncSetAttribute(pf::logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::kLgSmem);
    cudaFuncSetAttribute(pf::expert_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kExpertSmem(false)));
    cudaFuncSetAttribute(pf::expert_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(kExpertSmem(true)));
    attrs_set = true;
  }
  const int H = p.H, I = p.I, E = p.E;
  const int E_w = p.world > 1 ? p.ep_el : E;  // experts held by this rank's weight tensors
  const uint64_t rows2 = static_cast<uint64_t>(2) * L.npos;
  CUtensorMap mr, mx, m13, msh13, m2, msh2, mb_up[4], mb_dn[4];
  bool ok = true;
  if (p.mode == 1 && (phases & 1)) {
    ok = ok && tensor_map_3d(&mr, p.router_w, 2ull * H, E, 1, 2ull * H, 2ull * H * E, 128);
    ok = ok && tensor_map_3d(&mx, p.x, 2ull * H, p.T, 1, 2ull * H, 2ull * H * p.T, pf::kLgTok);
  }
  if (phases & 2) ok = ok && tensor_map_3d(&m13, p.w13, H, 2ull * I, E_w, H, p.w13_stride, 128);
  if (phases & 2) ok = ok && tensor_map_3d(&m2, p.w2, I, H, E_w, I, p.w2_stride, 128);
  if (p.sh_w13 && (phases & 2)) {
    ok = ok && tensor_map_3d(&msh13, p.sh_w13, H, 2ull * I, 1, H, 2ull * I * H, 128);
    ok = ok && tensor_map_3d(&msh2, p.sh_w2, I, H, 1, I, static_cast<uint64_t>(H) * I, 128);
  } else {
    msh13 = m13;
    msh2 = m2;
  }
  for (int b = 0; b < 4 && (phases & 2); ++b) {
    // up: the hi plane (d2 = 0) and the lo plane (d2 = 1) of [2][npos][H]
    ok = ok && tensor_map_3d(&mb_up[b], p.ws + L.pimg, H, L.npos, 2, H, static_cast<uint64_t>(L.npos) * H,
                             static_cast<uint32_t>(pf::up_box_rows(b)));
    ok = ok && tensor_map_3d(&mb_dn[b], p.ws + L.himg, I, rows2, 1, I, rows2 * I, 16u << b);
  }
  if (!ok) return 2;
  int n = 0;
  if (phases & 1) {
    if (p.mode == 1) {
      const dim3 g((E + pf::kRows - 1) / pf::kRows, (p.T + pf::kLgTok - 1) / pf::kLgTok, L.ks);
      if (pf_launch(pf::logits_kernel, g, pf::kLgThreads, pf::kLgSmem, stream, "prefill logits", p, mr, mx)) return 2;
      ++n;
    }
    if (pf_launch(pf::select_kernel, dim3(p.T), pf::kSelThreads, 0, stream, "prefill select", p)) return 2;
    ++n;
    if (p.world > 1) {
      const int P = p.T * p.K;
      if (pf_launch(pf::ep_dispatch_kernel, dim3((P + pf::pairs_per_cta(P) - 1) / pf::pairs_per_cta(P)),
                    pf::kDispThreads, 0, stream, "expert-parallel dispatch", p))
        return 2;
      ++n;
    }
  }
  if (!(phases & 2)) {
    note_launches(n);
    return 0;
  }
  const int disp_ctas = (L.cap + pf::pairs_per_cta(L.cap) - 1) / pf::pairs_per_cta(L.cap) +
                        (p.sh_w13 ? (p.T + pf::kDispWarps - 1) / pf::kDispWarps : 0);
  if (pf_launch(pf::dispatch_kernel, dim3(disp_ctas), pf::kDispThreads, 0, stream, "prefill dispatch", p)) return 2;
  if (pf_launch(pf::expert_kernel<false>, dim3(sms), pf::expert_threads(false), kExpertSmem(false), stream,
                "prefill up", p, m13,
                msh13, mb_up[0], mb_up[1], mb_up[2], mb_up[3]))
    return 2;
  if (pf_launch(pf::expert_kernel<true>, dim3(sms), pf::expert_threads(true), kExpertSmem(true), stream,
                "prefill down", p, m2,
                msh2, mb_dn[0], mb_dn[1], mb_dn[2], mb_dn[3]))
    return 2;
  const int c_threads = p.T * (H / 8);
  if (pf_launch(pf::combine_kernel, dim3((c_threads + pf::kCombineThreads - 1) / pf::kCombineThreads),
                pf::kCombineThreads, 0, stream, "prefill combine", p))
    return 2;
  note_launches(n + 4);
  return 0;
}

// Router only: logits + select (ids_out / w_out).
int launch_route(const pf::Params& p, cudaStream_t stream) {
  const pf::Layout L = pf::layout_of(p);
  static bool attrs_set = false;
  if (!attrs_set) {
    cudaFuncSetAttribute(pf::logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::kLgSmem);
    attrs_set = true;
  }
  CUtensorMap mr, mx;
  if (!tensor_map_3d(&mr, p.router_w, 2ull * p.H, p.E, 1, 2ull * p.H, 2ull * p.H * p.E, 128) ||
      !tensor_map_3d(&mx, p.x, 2ull * p.H, p.T, 1, 2ull * p.H, 2ull * p.H * p.T, pf::kLgTok))
    return 2;
  const dim3 g((p.E + pf::kRows - 1) / pf::kRows, (p.T + pf::kLgTok - 1) / pf::kLgTok, L.ks);
  if (pf_launch(pf::logits_kernel, g, pf::kLgThreads, pf::kLgSmem, stream, "route logits", p, mr, mx)) return 2;
  if (pf_launch(pf::select_kernel, dim3(p.T), pf::kSelThreads, 0, stream, "route select", p))
    return 2;
  note_launches(2);
  return 0;
}

}  // namespace dm3

// ------------------------------------------------------------------ C ABI
namespace {

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_prefill(int T, int H, int I, int E, int top_k, const void* x, const void* w13, int64_t w13_stride,
                  const float* s13, const void* w2, int64_t w2_stride, const float* s2, int srows, const void* y,
                  const void* ws, size_t ws_bytes) {
  if (T < 1 || static_cast<int64_t>(T) * top_k > 256 * dm3::pf::kMaxPpc)
    return dm3::set_error("T * top_k must be in [1, 262144]"), 1;
  if (H < 256 || H % 256 || H > dm3::kMaxH) return dm3::set_error("H must be a multiple of 256 in [256, 2048]"), 1;
  if (I < 128 || I % 128 || I > dm3::kMaxI) return dm3::set_error("I must be a multiple of 128 in [128, 512]"), 1;
  if (top_k < 1 || top_k > dm3::kMaxTopK) return dm3::set_error("top_k must be in [1, 8]"), 1;
  if (E < top_k || E > dm3::kMaxRouter) return dm3::set_error("the expert count must be in [top_k, 256]"), 1;
  if (!x || !w13 || !s13 || !w2 || !s2 || !y || !ws) return dm3::set_error("null pointer argument"), 1;
  if (!al16(x) || !al16(w13) || !al16(w2) || !al16(y)) return dm3::set_error("x, y and weights must be 16-byte aligned"), 1;
  if (w13_stride % 16 || w2_stride % 16 || w13_stride < 2LL * I * H || w2_stride < static_cast<int64_t>(H) * I)
    return dm3::set_error("expert strides must be multiples of 16 bytes covering one expert"), 1;
  if (srows != 1 && srows != 128) return dm3::set_error("srows must be 1 or 128"), 1;
  if (reinterpret_cast<uintptr_t>(ws) % 256) return dm3::set_error("workspace must be 256-byte aligned"), 1;
  if (ws_bytes < dm3::prefill_ws_bytes(T, H, I, E, top_k)) return dm3::set_error("workspace too small"), 4;
  return 0;
}

dm3::pf::Params prefill_params(const void* x, int T, int H, int I, int E, int top_k, const void* w13,
                               int64_t w13_stride, const float* s13, int64_t s13_stride, const void* w2,
                               int64_t w2_stride, const float* s2, int64_t s2_stride, int srows, void* y,
                               int64_t* perm_out, int64_t* offsets_out, void* ws) {
  dm3::pf::Params p{};
  p.T = T;
  p.H = H;
  p.I = I;
  p.E = E;
  p.K = top_k;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.w13 = static_cast<const uint8_t*>(w13);
  p.w13_stride = w13_stride;
  p.s13 = s13;
  p.s13_stride = s13_stride;
  p.w2 = static_cast<const uint8_t*>(w2);
  p.w2_stride = w2_stride;
  p.s2 = s2;
  p.s2_stride = s2_stride;
  p.srows = srows;
  p.sh_srows = 128;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.perm_out = perm_out;
  p.offsets_out = offsets_out;
  p.ws = static_cast<uint8_t*>(ws);
  return p;
}

}  // namespace

extern "C" size_t dm3_moe_prefill_workspace_bytes(int T, int H, int I, int n_experts, int top_k) {
  if (T < 1 || H < 128 || I < 128 || n_experts < 1 || top_k < 1) return 0;
  return dm3::prefill_ws_bytes(T, H, I, n_experts, top_k);
}

extern "C" int dm3_moe_prefill(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                               int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride,
                               const float* s13, int64_t s13_stride, const void* w2, int64_t w2_stride,
                               const float* s2, int64_t s2_stride, int srows, const void* sh_w13, const float* sh_s13,
                               const void* sh_w2, const float* sh_s2, int sh_srows, const void* sh_gate,
                               const float* out_bias, void* y, int64_t* ids_out, void* w_out, int64_t* perm_out,
                               int64_t* offsets_out, void* workspace, size_t workspace_bytes, void* stream) {
  dm3::note_launches(0);
  int rc = check_prefill(T, H, I, n_router, top_k, x, w13, w13_stride, s13, w2, w2_stride, s2, srows, y, workspace,
                         workspace_bytes);
  if (rc) return rc;
  if (!router_w || !al16(router_w)) return dm3::set_error("router weight (bf16) must be given, 16-byte aligned"), 1;
  if (out_bias && !al16(out_bias)) return dm3::set_error("out_bias must be 16-byte aligned"), 1;
  if (sh_w13) {
    if (!sh_s13 || !sh_w2 || !sh_s2) return dm3::set_error("shared expert needs w13, s13, w2, s2"), 1;
    if (!al16(sh_w13) || !al16(sh_w2)) return dm3::set_error("shared expert weights must be 16-byte aligned"), 1;
    if (sh_srows != 1 && sh_srows != 128) return dm3::set_error("sh_srows must be 1 or 128"), 1;
    if (sh_gate && !al16(sh_gate)) return dm3::set_error("shared gate must be 16-byte aligned"), 1;
  }
  dm3::pf::Params p = prefill_params(x, T, H, I, n_router, top_k, w13, w13_stride, s13, s13_stride, w2, w2_stride, s2,
                                     s2_stride, srows, y, perm_out, offsets_out, workspace);
  p.mode = 1;
  p.router_w = static_cast<const __nv_bfloat16*>(router_w);
  p.logits_bf16 = logits_bf16;
  p.logit_bias = logit_bias;
  p.sh_w13 = static_cast<const uint8_t*>(sh_w13);
  p.sh_s13 = sh_s13;
  p.sh_w2 = static_cast<const uint8_t*>(sh_w2);
  p.sh_s2 = sh_s2;
  p.sh_srows = sh_w13 ? sh_srows : 128;
  p.sh_gate = sh_w13 ? static_cast<const __nv_bfloat16*>(sh_gate) : nullptr;
  p.out_bias = out_bias;
  p.ids_out = ids_out;
  p.w_out = static_cast<__nv_bfloat16*>(w_out);
  return dm3::launch_prefill(p, static_cast<cudaStream_t>(stream));
}

extern "C" int dm3_moe_grouped(const void* x, int T, int H, int I, const int64_t* ids, const void* weights,
                               int top_k, int n_experts, const void* w13, int64_t w13_stride, const float* s13,
                               int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2,
                               int64_t s2_stride, int srows, void* y, int64_t* perm_out, int64_t* offsets_out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  dm3::note_launches(0);
  int rc = check_prefill(T, H, I, n_experts, top_k, x, w13, w13_stride, s13, w2, w2_stride, s2, srows, y, workspace,
                         workspace_bytes);
  if (rc) return rc;
  if (!ids || !weights) return dm3::set_error("ids and weights are required"), 1;
  dm3::pf::Params p = prefill_params(x, T, H, I, n_experts, top_k, w13, w13_stride, s13, s13_stride, w2, w2_stride, s2,
                                     s2_stride, srows, y, perm_out, offsets_out, workspace);
  p.mode = 0;
  p.ids = ids;
  p.rw = static_cast<const __nv_bfloat16*>(weights);
  return dm3::launch_prefill(p, static_cast<cudaStream_t>(stream));
}

extern "C" size_t dm3_route_workspace_bytes(int T, int H, int n_router, int top_k) {
  if (T < 1 || H < 128 || n_router < 1 || top_k < 1) return 0;
  return dm3::pf::layout(T, H, 128, n_router, top_k).pos_tok;
}

extern "C" int dm3_route(const void* x, int T, int H, const void* router_w, int n_router, int top_k, int logits_bf16,
                         const float* logit_bias, int64_t* ids_out, void* w_out, void* workspace,
                         size_t workspace_bytes, void* stream) {
  dm3::note_launches(0);
  if (T < 1) return dm3::set_error("T must be >= 1"), 1;
  if (H < 128 || H % 128 || H > dm3::kMaxH) return dm3::set_error("H must be a multiple of 128 in [128, 2048]"), 1;
  if (top_k < 1 || top_k > dm3::kMaxTopK) return dm3::set_error("top_k must be in [1, 8]"), 1;
  if (n_router < top_k || n_router > dm3::kMaxRouter) return dm3::set_error("n_router must be in [top_k, 256]"), 1;
  if (!x || !router_w || !ids_out || !w_out || !workspace) return dm3::set_error("null pointer argument"), 1;
  if (!al16(x) || !al16(router_w)) return dm3::set_error("x and router weight must be 16-byte aligned"), 1;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return dm3::set_error("workspace must be 256-byte aligned"), 1;
  if (workspace_bytes < dm3_route_workspace_bytes(T, H, n_router, top_k)) return dm3::set_error("workspace too small"), 4;
  dm3::pf::Params p{};
  p.T = T;
  p.H = H;
  p.I = 128;
  p.E = n_router;
  p.K = top_k;
  p.mode = 1;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.router_w = static_cast<const __nv_bfloat16*>(router_w);
  p.logits_bf16 = logits_bf16;
  p.logit_bias = logit_bias;
  p.ids_out = ids_out;
  p.w_out = static_cast<__nv_bfloat16*>(w_out);
  p.ws = static_cast<uint8_t*>(workspace);
  return dm3::launch_route(p, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ expert-parallel C ABI
extern "C" size_t dm3_ep_arena_bytes(int world, int tokens_per_rank, int top_k, int H) {
  if (world < 2 || world > dm3::pf::kMaxRanks || tokens_per_rank < 1 || top_k < 1 || H < 128) return 0;
  return dm3::pf::ep_layout(world, tokens_per_rank, top_k, H).total;
}

extern "C" int dm3_ep_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return dm3::set_error("dm3_ep_alloc: bad arguments"), 1;
  *ptr = nullptr;
  cudaError_t err = cudaMalloc(ptr, bytes);
  if (err == cudaSuccess) err = cudaMemset(*ptr, 0, bytes);
  if (err != cudaSuccess) return dm3::set_error(std::string("dm3_ep_alloc: ") + cudaGetErrorString(err)), 2;
  return 0;
}

extern "C" int dm3_ep_free(void* ptr) {
  if (ptr && cudaFree(ptr) != cudaSuccess) return dm3::set_error("dm3_ep_free failed"), 2;
  return 0;
}

extern "C" int dm3_ep_ipc_handle(void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return dm3::set_error("dm3_ep_ipc_handle: null argument"), 1;
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, ptr);
  if (err != cudaSuccess) return dm3::set_error(std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(err)), 2;
  std::memcpy(handle_out, &h, sizeof(h));
  return 0;
}

extern "C" int dm3_ep_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return dm3::set_error("dm3_ep_ipc_open: null argument"), 1;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return dm3::set_error(std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(err)), 2;
  return 0;
}

extern "C" int dm3_ep_ipc_close(void* ptr) {
  if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return dm3::set_error("cudaIpcCloseMemHandle failed"), 2;
  return 0;
}

extern "C" size_t dm3_moe_prefill_ep_workspace_bytes(int world, int tokens_per_rank, int H, int I, int n_router,
                                                     int top_k) {
  if (world < 2 || world > dm3::pf::kMaxRanks || tokens_per_rank < 1 || H < 128 || I < 128 || n_router < 1 ||
      top_k < 1)
    return 0;
  return dm3::pf::layout(tokens_per_rank, H, I, n_router, top_k, world * tokens_per_rank * top_k).total;
}

namespace {

int check_ep(int world, int rank, int T, int tokens_per_rank, int n_router, void* const* arenas) {
  if (world < 2 || world > dm3::pf::kMaxRanks) return dm3::set_error("world must be in [2, 8]"), 1;
  if (rank < 0 || rank >= world) return dm3::set_error("rank out of range"), 1;
  if (T > tokens_per_rank) return dm3::set_error("T exceeds the arena's tokens per rank"), 1;
  if (n_router % world) return dm3::set_error("the expert count must divide evenly over the ranks"), 1;
  if (static_cast<int64_t>(world) * tokens_per_rank * 8 > 256 * dm3::pf::kMaxPpc)
    return dm3::set_error("world * tokens_per_rank * top_k exceeds the dispatch capacity"), 1;
  if (!arenas) return dm3::set_error("arena pointers are required"), 1;
  for (int r = 0; r < world; ++r)
    if (!arenas[r] || (reinterpret_cast<uintptr_t>(arenas[r]) & 4095u)) return dm3::set_error("bad arena pointer"), 1;
  return 0;
}

void set_ep(dm3::pf::Params& p, int world, int rank, int tokens_per_rank, void* const* arenas) {
  p.world = world;
  p.rank = rank;
  p.ep_tl = tokens_per_rank;
  p.ep_el = p.E / world;
  for (int r = 0; r < dm3::pf::kMaxRanks; ++r) p.ep_arena[r] = r < world ? static_cast<uint8_t*>(arenas[r]) : nullptr;
}

}  // namespace

// phases as launch_prefill: 1 = ep_dispatch, 2 = ep_combine, 3 = both
static int prefill_ep(int phases, const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                      int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride, const float* s13,
                      int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride,
                      int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                      int sh_srows, const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out,
                      void* w_out, int world, int rank, int tokens_per_rank, void* const* arenas, const int* owner,
                      void* workspace, size_t workspace_bytes, void* stream) {
  dm3::note_launches(0);
  int rc = check_ep(world, rank, T, tokens_per_rank, n_router, arenas);
  if (rc) return rc;
  // expert weights are only read by the second phase; the checks below take any non-null
  // placeholders for the first
  rc = check_prefill(T, H, I, n_router, top_k, x, w13, w13_stride, s13, w2, w2_stride, s2, srows, y, workspace,
                     SIZE_MAX);
  if (rc) return rc;
  if (workspace_bytes < dm3_moe_prefill_ep_workspace_bytes(world, tokens_per_rank, H, I, n_router, top_k))
    return dm3::set_error("workspace too small"), 4;
  if (!router_w || !al16(router_w)) return dm3::set_error("router weight (bf16) must be given, 16-byte aligned"), 1;
  if (out_bias && !al16(out_bias)) return dm3::set_error("out_bias must be 16-byte aligned"), 1;
  if (sh_w13) {
    if (!sh_s13 || !sh_w2 || !sh_s2) return dm3::set_error("shared expert needs w13, s13, w2, s2"), 1;
    if (!al16(sh_w13) || !al16(sh_w2)) return dm3::set_error("shared expert weights must be 16-byte aligned"), 1;
    if (sh_srows != 1 && sh_srows != 128) return dm3::set_error("sh_srows must be 1 or 128"), 1;
    if (sh_gate && !al16(sh_gate)) return dm3::set_error("shared gate must be 16-byte aligned"), 1;
  }
  dm3::pf::Params p = prefill_params(x, T, H, I, n_router, top_k, w13, w13_stride, s13, s13_stride, w2, w2_stride, s2,
                                     s2_stride, srows, y, nullptr, nullptr, workspace);
  p.mode = 1;
  p.router_w = static_cast<const __nv_bfloat16*>(router_w);
  p.logits_bf16 = logits_bf16;
  p.logit_bias = logit_bias;
  p.sh_w13 = static_cast<const uint8_t*>(sh_w13);
  p.sh_s13 = sh_s13;
  p.sh_w2 = static_cast<const uint8_t*>(sh_w2);
  p.sh_s2 = sh_s2;
  p.sh_srows = sh_w13 ? sh_srows : 128;
  p.sh_gate = sh_w13 ? static_cast<const __nv_bfloat16*>(sh_gate) : nullptr;
  p.out_bias = out_bias;
  p.ids_out = ids_out;
  p.w_out = static_cast<__nv_bfloat16*>(w_out);
  set_ep(p, world, rank, tokens_per_rank, arenas);
  p.ep_owner = owner;
  return dm3::launch_prefill(p, static_cast<cudaStream_t>(stream), phases);
}

extern "C" int dm3_moe_prefill_ep(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                                  int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride,
                                  const float* s13, int64_t s13_stride, const void* w2, int64_t w2_stride,
                                  const float* s2, int64_t s2_stride, int srows, const void* sh_w13,
                                  const float* sh_s13, const void* sh_w2, const float* sh_s2, int sh_srows,
                                  const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out, void* w_out,
                                  int world, int rank, int tokens_per_rank, void* const* arenas, const int* owner,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  return prefill_ep(3, x, T, H, I, router_w, n_router, top_k, logits_bf16, logit_bias, w13, w13_stride, s13,
                    s13_stride, w2, w2_stride, s2, s2_stride, srows, sh_w13, sh_s13, sh_w2, sh_s2, sh_srows, sh_gate,
                    out_bias, y, ids_out, w_out, world, rank, tokens_per_rank, arenas, owner, workspace,
                    workspace_bytes, stream);
}

extern "C" int dm3_ep_dispatch(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                               int logits_bf16, const float* logit_bias, const void* sh_gate, int64_t* ids_out,
                               void* w_out, int world, int rank, int tokens_per_rank, void* const* arenas,
                               const int* owner, void* workspace, size_t workspace_bytes, void* stream) {
  // the expert operands are not read by this phase: the router weight stands in for them in the
  // argument checks (and, when the shared gate is given, for the shared expert's presence)
  return prefill_ep(1, x, T, H, I, router_w, n_router, top_k, logits_bf16, logit_bias, router_w, 2LL * I * H,
                    reinterpret_cast<const float*>(router_w), 0, router_w, static_cast<int64_t>(H) * I,
                    reinterpret_cast<const float*>(router_w), 0, 128, sh_gate ? router_w : nullptr,
                    reinterpret_cast<const float*>(router_w), router_w, reinterpret_cast<const float*>(router_w), 128,
                    sh_gate, nullptr, const_cast<void*>(x), ids_out, w_out, world, rank, tokens_per_rank, arenas,
                    owner, workspace, workspace_bytes, stream);
}

extern "C" int dm3_ep_combine(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                              const void* w13, int64_t w13_stride, const float* s13, int64_t s13_stride,
                              const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride, int srows,
                              const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                              int sh_srows, const void* sh_gate, const float* out_bias, void* y, int world, int rank,
                              int tokens_per_rank, void* const* arenas, void* workspace, size_t workspace_bytes,
                              void* stream) {
  return prefill_ep(2, x, T, H, I, router_w, n_router, top_k, 1, nullptr, w13, w13_stride, s13, s13_stride, w2,
                    w2_stride, s2, s2_stride, srows, sh_w13, sh_s13, sh_w2, sh_s2, sh_srows, sh_gate, out_bias, y,
                    nullptr, nullptr, world, rank, tokens_per_rank, arenas, nullptr, workspace, workspace_bytes, stream);
}

namespace dm3 {
// This file's copy of the device wait limit on the current device (dm3_set_wait_limit_ns).
int wait_limit_moe_prefill(uint64_t ns) { return static_cast<int>(set_wait_limit_here(ns)); }
}  // namespace dm3
