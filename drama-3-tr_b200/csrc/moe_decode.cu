// Decode MoE layer for B200 (sm_100a) as four chained kernels, each launched with programmatic
// dependent launch so that a kernel's constant-weight loads start while its predecessor finishes:
//
//   route    router logits (exact products, summed in fp64 and rounded once), four warps per
//            router row
//   up       gate and up rows of every selected expert (+ the shared expert) on the tensor cores:
//            items of 64 gate + the matching 64 up rows over all of H; SwiGLU in the epilogue;
//            h written as bf16
//   down     128-row blocks of every selected expert's down projection against its h; routed
//            partials carry their routing weight
//   combine  sum over slots per output element with the reference's rounding points (+ bias,
//            + the sigmoid-gated shared expert), written as bf16
//
// Kernel boundaries are the only synchronisation between CTAs: no gpu-scope fence or flag is
// used on the streaming path.
//
// Up / down kernels (one CTA per SM, 8 warps):
//   warp 0     TMA producer: 128-byte-swizzled weight slabs (128 rows x 128 bytes of K) into a ring
//              of 32 KB stages, straight from the e4m3 expert tensors
//   warp 1     MMA issuer: tcgen05.mma kind::f8f6f4, M = 128 weight rows, N = 16 activation columns
//              (rows 0-3 the exact e4m3 "hi" split of each token, 4-7 the "lo" remainder, 8-15 zero),
//              K = 32 per instruction; every 128-wide k block accumulates into its own 16 TMEM
//              columns so that its block scale can be applied in fp32 afterwards
//   warps 2-3  activation split: the tokens' bf16 rows (x, or h of the item's expert) prescaled by a
//              power of two and split exactly into e4m3 hi + lo, written in the swizzled layout
//   warps 4-7  epilogue: TMEM -> registers (one weight row per thread), block scales, SwiGLU or the
//              routing weight, stores
//
// Ordering under programmatic dependent launch: every kernel calls griddepcontrol.launch_dependents
// only after its own griddepcontrol.wait, so once a kernel is running, everything two launches
// back has completed. The down kernel relies on that to select experts before its wait.
#include <atomic>
#include <cfloat>
#include <cstddef>
#include <cmath>
#include <mutex>
#include <string>
#include <utility>

#include "dm3_common.cuh"
#include "dm3_ep.cuh"
#include "dm3_internal.h"
#include "dm3_route.cuh"
#include "dm3_tc.cuh"

namespace dm3 {
namespace moe {

constexpr int kThreads = 256;       // 8 warps
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpEpi = 4;
constexpr int kSplitThreads = 192;  // up: every warp but the producer and the table warp (4)
constexpr int kEpiThreads = 128;    // warps 4-7
constexpr int kGroup = 32;          // k elements per activation exponent of h (one MMA K step)
constexpr int kTileRows = 128;      // weight rows per MMA tile (M)
constexpr int kUpHalf = 64;         // gate rows (and as many up rows) per up item
constexpr int kBlockRows = 128;     // output rows per down item (= rows per partial block)
constexpr int kN = 16;              // activation columns of the MMA (N)
constexpr int kSlabBytes = kTileRows * 128;   // one 128-byte K slab of a weight tile
constexpr int kStageBytes = 2 * kSlabBytes;   // two slabs per ring stage
constexpr int kBSlabBytes = kN * 128;         // one K slab of the activation tile
constexpr int kUpStages = 5, kDownStages = 6;
constexpr int kUpAcc = 2, kDownAcc = 2;       // TMEM accumulator buffers
constexpr uint32_t kUpTmemCols = 512, kDownTmemCols = 512;
constexpr int kRouteWarps = 4;      // router rows per route CTA
constexpr int kRouteSplit = 4;      // warps per router row (each sums a quarter of H)
constexpr int kRouteThreads = kRouteWarps * kRouteSplit * 32;
constexpr int kCombineThreads = 256;
// named barriers (0 is __syncthreads)
constexpr int kBarTable = 1, kBarSplit = 2, kBarEpi = 3;

struct Params {
  int T, H, I, top_k;
  const __nv_bfloat16* x;
  int mode;  // 0 = routing given (ids/weights), 1 = router in-kernel
  int fused;  // 1: the cluster kernel (layer_kernel) selects experts and combines; the route kernel only
              // computes logits and splits x
  const int64_t* ids;
  const __nv_bfloat16* rw;
  const void* router_w;
  int router_bf16, n_router, logits_bf16;
  const float* logit_bias;
  int64_t* ids_out;
  __nv_bfloat16* w_out;
  int n_experts;
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
  const __nv_bfloat16* sh_gate;
  const float* out_bias;
  __nv_bfloat16* y;
  uint8_t* ws;
  int sh_slot;  // slot 0 is the shared expert on this rank (the layer has one; rank 0 when sharded)
  // sharded over `world` ranks (world > 1): this rank runs the experts [rank * ep_el, +ep_el) of
  // the routing every rank computes alike, whose weights w13 / w2 hold; the partial sums meet in an
  // all-reduce over the expert-parallel arenas (ep_arena[r] = rank r's, mapped here)
  int world, rank, ep_tl, ep_el;
  uint8_t* ep_arena[8];
};


// ------------------------------------------------------------------ workspace layout
// Control words, the shared gate of the call, the router logits, the bf16 SwiGLU activations h and
// the fp32 per-slot partial outputs. Offsets do not depend on the row count, so one workspace
// serves every T of a given (H, I). Nothing in it carries state from one call to the next except
// the sticky status word (the route kernel's CTA counter is back at zero after every call).
struct WsLayout {
  size_t ctrl, slot_expert, coef, gate, logits, himg, himg_stride, hinv, ximg, xinv, partial, facc, total;
};
enum : int { CTRL_ROUTE_COUNT = 0, CTRL_STATUS = 4, CTRL_NSLOTS = 5, CTRL_WORDS = 16 };

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline WsLayout ws_layout(int H, int I) {
  WsLayout L;
  size_t o = 0;
  L.ctrl = o;
  o += CTRL_WORDS * 4;
  L.slot_expert = o;
  o += align_up(kMaxSlots * 4, 16);
  L.coef = o;
  o += align_up(kMaxSlots * kMaxT * 4, 16);
  L.gate = o;  // [kMaxT] the shared expert's sigmoid gate per row
  o += align_up(kMaxT * 4, 16);
  L.logits = o;
  o += align_up(kMaxT * (kMaxRouter + 1) * 4, 16);
  // per slot: h split into e4m3 hi (rows 0-3) and lo (rows 4-7) as the down kernel's activation
  // tile, 16 rows x I bytes in the swizzled slab layout (rows 8-15 are never written)
  o = align_up(o, 1024);
  L.himg_stride = static_cast<size_t>(I / 128) * kBSlabBytes;
  L.himg = o;
  o += L.himg_stride * kMaxSlots;
  L.hinv = o;  // [kMaxSlots][kMaxI / kGroup][kMaxT] fp32: 2^-e of each 32-element group of h
  o += static_cast<size_t>(kMaxSlots) * (kMaxI / kGroup) * kMaxT * 4;
  // x split by the route kernel into the up kernel's activation tile (16 rows x H), and 2^-e per row
  o = align_up(o, 1024);
  L.ximg = o;
  o += static_cast<size_t>(H / 128) * kBSlabBytes;
  L.xinv = o;
  o += kMaxT * 4;
  o = align_up(o, 128);
  L.partial = o;  // [H / 128][kMaxSlots][kMaxT][128] fp32: one output block's slots are adjacent
  o += static_cast<size_t>(H / kBlockRows) * kMaxSlots * kMaxT * kBlockRows * 4;
  o = align_up(o, 256);
  L.facc = o;  // [2][kMaxT][H] int64: the cluster kernel's fixed-point sums (routed, shared); zero between calls
  o += static_cast<size_t>(2) * kMaxT * H * 8;
  L.total = align_up(o, 256);
  return L;
}

__device__ __forceinline__ float* partial_block(const Params& p, const WsLayout& L, int nb, int slot) {
  return reinterpret_cast<float*>(p.ws + L.partial) +
         (static_cast<size_t>(nb) * kMaxSlots + slot) * kMaxT * kBlockRows;
}

// The route table of one call in shared memory, and the scratch that builds it.
struct Table {
  int expert[kMaxSlots];             // routed expert of each slot (slot 0 = shared expert when present)
  float coef[kMaxSlots * kMaxT];     // [slot][row] routing weight (the shared slot: its sigmoid gate)
  int kbuf[32];
  float wbuf[32];
};

// Barriers, the table and small per-item values of the up / down kernels.
struct Aux {
  uint64_t full[8], empty[8];        // TMA ring: bytes landed / MMAs done reading
  uint64_t acc_full[4], acc_empty[4];  // TMEM accumulators: MMAs done / epilogue done reading
  uint64_t b_ready[2], b_free[2];    // activation tiles (down): copied in / MMAs done reading
  uint32_t tmem;
  int epi_ok[4];                     // up: each epilogue warp's accumulator wait succeeded
  int n_slots;
  float xinv[kMaxT];                 // up: 2^-e of each token's split
  uint32_t xmax[kMaxT];              // up: |x| maxima (float bits)
  float upv[kUpHalf][kMaxT];         // up: the up-row values handed to the gate-row threads
  Table tab;
};

// Shared memory of the up / down kernels, from a 1024-byte aligned base: the ring of weight
// stages, the activation tile(s), then Aux.
struct SmemLayout {
  int nstages, stage, b, b_bytes, aux, total;
};

__host__ __device__ inline SmemLayout smem_layout(bool down, int H, int I) {
  SmemLayout S;
  S.nstages = down ? kDownStages : kUpStages;
  S.stage = 0;
  S.b = S.nstages * kStageBytes;
  S.b_bytes = (down ? I : H) / 128 * kBSlabBytes;  // one activation tile
  S.aux = S.b + (down ? 2 : 1) * S.b_bytes;
  S.total = S.aux + static_cast<int>(align_up(sizeof(Aux), 128)) + 1024;  // + alignment slack
  return S;
}

__device__ __forceinline__ uint32_t* ctrl(const Params& p, const WsLayout& L) {
  return reinterpret_cast<uint32_t*>(p.ws + L.ctrl);
}

__device__ __forceinline__ void flag_error(const Params& p, const WsLayout& L, uint32_t bits) {
  atomicOr(ctrl(p, L) + CTRL_STATUS, bits);
}

// Expert operands of a slot: slot 0 is the shared expert when one is present.
struct ExpertRef {
  const uint8_t* w13;
  const float* s13;
  const uint8_t* w2;
  const float* s2;
  int srows;
};

__device__ __forceinline__ ExpertRef expert_ref(const Params& p, int slot, const int* tab_expert) {
  ExpertRef r;
  if (slot == 0 && p.sh_slot) {
    r.w13 = p.sh_w13;
    r.s13 = p.sh_s13;
    r.w2 = p.sh_w2;
    r.s2 = p.sh_s2;
    r.srows = p.sh_srows;
  } else {
    const int e = tab_expert[slot];
    r.w13 = p.w13 + static_cast<size_t>(e) * p.w13_stride;
    r.s13 = p.s13 + static_cast<size_t>(e) * p.s13_stride;
    r.w2 = p.w2 + static_cast<size_t>(e) * p.w2_stride;
    r.s2 = p.s2 + static_cast<size_t>(e) * p.s2_stride;
    r.srows = p.srows;
  }
  return r;
}

// ------------------------------------------------------------------ route table helpers
// Builds slots from (token, expert, weight) pairs held one per lane (lanes >= n invalid), for
// routing given by the caller (any expert count). Slot order: distinct experts ascending. Returns
// the slot count. One warp; tab.kbuf / tab.wbuf are its scratch.
__device__ int build_slots(int lane, int n, int t, int e, float w, int T, Table& tab) {
  const bool valid = lane < n && e >= 0;
  const int key = valid ? e : 0x7fffffff;
  tab.kbuf[lane] = key;
  tab.wbuf[lane] = w;
  const unsigned same = __match_any_sync(0xffffffffu, key);
  const bool first = valid && (__ffs(same) - 1 == lane);
  const unsigned firsts = __ballot_sync(0xffffffffu, first);
  __syncwarp();
  int rank = 0;  // distinct experts below this one
  for (unsigned f = firsts; f; f &= f - 1u) rank += tab.kbuf[__ffs(f) - 1] < key ? 1 : 0;
  // one writer per (slot, row): a repeated pair (only possible with malformed ids) is summed in lane order
  const int key2 = valid ? ((rank << 3) | t) : -1 - lane;
  const unsigned grp = __match_any_sync(0xffffffffu, key2);
  for (int i = lane; i < kMaxSlots * kMaxT; i += 32) tab.coef[i] = 0.f;
  __syncwarp();
  if (valid && (__ffs(grp) - 1 == lane)) {
    float wsum = 0.f;
    for (unsigned g = grp; g; g &= g - 1u) wsum += tab.wbuf[__ffs(g) - 1];
    tab.expert[rank] = e;
    tab.coef[rank * kMaxT + t] = wsum;
  }
  __syncwarp();
  (void)T;
  return __popc(firsts);
}

// Route table from the caller's ids / weights (routing given), for one warp.
__device__ int table_from_ids(const Params& p, const WsLayout& L, int lane, Table& tab, bool report_bad_ids) {
  const int n = p.T * p.top_k;
  int t = 0, e = -1;
  float w = 0.f;
  if (lane < n) {
    t = lane / p.top_k;
    const int64_t id = p.ids[lane];
    if (id >= 0 && id < p.n_experts) {
      e = static_cast<int>(id);
      w = __bfloat162float(p.rw[lane]);
    } else if (report_bad_ids) {
      flag_error(p, L, STATUS_BAD_EXPERT);
    }
  }
  return build_slots(lane, n, t, e, w, p.T, tab);
}

// Route table the route kernel left in the workspace, for one warp (one L2 round trip).
__device__ int table_from_ws(const Params& p, const WsLayout& L, int lane, Table& tab) {
  constexpr int kE = (kMaxSlots + 31) / 32, kC = (kMaxSlots * kMaxT + 31) / 32;
  const int* gse = reinterpret_cast<const int*>(p.ws + L.slot_expert);
  const float* gco = reinterpret_cast<const float*>(p.ws + L.coef);
  // every load is issued before the first use: one L2 round trip
  const uint32_t n_slots = __ldcg(ctrl(p, L) + CTRL_NSLOTS);
  int ev[kE];
  float cv[kC];
#pragma unroll
  for (int q = 0; q < kE; ++q) ev[q] = lane + 32 * q < kMaxSlots ? __ldcg(gse + lane + 32 * q) : 0;
#pragma unroll
  for (int q = 0; q < kC; ++q) cv[q] = lane + 32 * q < kMaxSlots * kMaxT ? __ldcg(gco + lane + 32 * q) : 0.f;
#pragma unroll
  for (int q = 0; q < kE; ++q)
    if (lane + 32 * q < kMaxSlots) tab.expert[lane + 32 * q] = ev[q];
#pragma unroll
  for (int q = 0; q < kC; ++q)
    if (lane + 32 * q < kMaxSlots * kMaxT) tab.coef[lane + 32 * q] = cv[q];
  __syncwarp();
  return static_cast<int>(n_slots);
}

// ------------------------------------------------------------------ route kernel
// Shared-memory tail of the route kernel: the logits of every row (the last column is the shared
// expert's gate), the selections and the table scratch of the last CTA.
struct RouteTail {
  // the fields the route kernel itself uses come first: with a cluster kernel after it, the route
  // kernel's shared memory ends at `logits`
  uint64_t bar;
  int last;
  uint32_t xmax[kMaxT];
  double part[kRouteWarps][kMaxT][kRouteSplit];  // fp64 sum of each warp's quarter of a row
  float logits[kMaxT][kMaxRouter + 1];
  int sel_e[kMaxT * kMaxTopK];
  float sel_w[kMaxT * kMaxTopK];
  float shared_coef[kMaxT];
  uint32_t bitmap[kMaxRouter / 32];
};

__device__ __forceinline__ void cswap_desc32(uint32_t& a, uint32_t& b) {
  const uint32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}

// warp_top8 for 32-bit keys (same network and merge rounds).
__device__ __forceinline__ void warp_top8_32(uint32_t (&k)[8]) {
  cswap_desc32(k[0], k[1]); cswap_desc32(k[2], k[3]); cswap_desc32(k[4], k[5]); cswap_desc32(k[6], k[7]);
  cswap_desc32(k[0], k[2]); cswap_desc32(k[1], k[3]); cswap_desc32(k[4], k[6]); cswap_desc32(k[5], k[7]);
  cswap_desc32(k[1], k[2]); cswap_desc32(k[5], k[6]);
  cswap_desc32(k[0], k[4]); cswap_desc32(k[1], k[5]); cswap_desc32(k[2], k[6]); cswap_desc32(k[3], k[7]);
  cswap_desc32(k[2], k[4]); cswap_desc32(k[3], k[5]);
  cswap_desc32(k[1], k[2]); cswap_desc32(k[3], k[4]); cswap_desc32(k[5], k[6]);
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __shfl_xor_sync(0xffffffffu, k[i], d);
#pragma unroll
    for (int i = 0; i < 8; ++i) k[i] = max(k[i], o[7 - i]);
    cswap_desc32(k[0], k[4]); cswap_desc32(k[1], k[5]); cswap_desc32(k[2], k[6]); cswap_desc32(k[3], k[7]);
    cswap_desc32(k[0], k[2]); cswap_desc32(k[1], k[3]); cswap_desc32(k[4], k[6]); cswap_desc32(k[5], k[7]);
    cswap_desc32(k[0], k[1]); cswap_desc32(k[2], k[3]); cswap_desc32(k[4], k[5]); cswap_desc32(k[6], k[7]);
  }
}

// Top-k of row t by one warp from the logits in shared memory. Mirrors Speaker.__call__
// (engine.py:233-235): probs = softmax(logits), (w, ids) = probs.topk(k),
// w = (w / w.sum()).to(bf16). Selection uses the logits themselves (softmax is monotonic) with
// ties to the lower index: keys pack (logit order, ~index) so one comparison decides both. When
// every logit is a bf16 value (bf16 logits without a bias) the order fits 16 bits and a key is
// 32 bits; otherwise 64.
__device__ void route_row(const Params& p, RouteTail& rt, int t, int lane, bool emit = true) {
  const int E = p.n_router, K = p.top_k;
  float lv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) lv[i] = lane + 32 * i < E ? rt.logits[t][lane + 32 * i] : -FLT_MAX;
  int sel_e[8];
  float sel_v[8];
  if (p.logits_bf16 && p.logit_bias == nullptr) {
    uint32_t k[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      k[i] = e < E ? ((order_key(lv[i]) >> 16) << 16) | static_cast<uint32_t>(0xFFFF - e) : 0u;
    }
    warp_top8_32(k);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sel_e[j] = 0xFFFF - static_cast<int>(k[j] & 0xFFFFu);
      // the low half of a bf16 value's float bits is zero, which the key inverts for negative values
      sel_v[j] = key_value((k[j] & 0x80000000u) ? (k[j] & 0xFFFF0000u) : (k[j] | 0x0000FFFFu));
    }
  } else {
    uint64_t k[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      k[i] = e < E ? (static_cast<uint64_t>(order_key(lv[i])) << 32) | static_cast<uint32_t>(~e) : 0ull;
    }
    warp_top8(k);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sel_e[j] = static_cast<int>(~static_cast<uint32_t>(k[j]));
      sel_v[j] = key_value(static_cast<uint32_t>(k[j] >> 32));
    }
  }
  // softmax denominator; the maximum logit is the first selection's value (every lane holds the
  // merged top 8)
  const float m = sel_v[0];
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (lane + 32 * i < E) z += expf(lv[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  // lane j < K: probability of the j-th selection; the sum runs in selection order
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
    rt.sel_e[t * K + lane] = my_e;
    rt.sel_w[t * K + lane] = __bfloat162float(wb);
    if (emit && p.ids_out) p.ids_out[t * K + lane] = my_e;
    if (emit && p.w_out) p.w_out[t * K + lane] = wb;
  }
  if (lane == 0) rt.shared_coef[t] = p.sh_gate ? bf16_round(1.f / (1.f + expf(-rt.logits[t][E]))) : 1.f;
}

// The route table of the call from the selections, by one warp, into the workspace: slot 0 is the
// shared expert when present, then the distinct routed experts ascending (rank = count of selected
// experts below, from a bitmap of the router's experts).
__device__ void write_table(const Params& p, const WsLayout& L, RouteTail& rt, int lane) {
  const int n = p.T * p.top_k;
  const bool valid = lane < n;
  const int e = valid ? rt.sel_e[lane] : 0;
  const int t = valid ? lane / p.top_k : 0;
  // sharded: only the experts this rank holds get slots, numbered by their local index
  const bool own = valid && (p.world <= 1 || e / p.ep_el == p.rank);
  if (lane < kMaxRouter / 32) rt.bitmap[lane] = 0u;
  __syncwarp();
  if (own) atomicOr(&rt.bitmap[e >> 5], 1u << (e & 31));
  __syncwarp();
  int srank = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kMaxRouter / 32; ++w) {
    const uint32_t word = rt.bitmap[w];
    total += __popc(word);
    if (w < (e >> 5)) srank += __popc(word);
  }
  srank += __popc(rt.bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
  const bool sh = p.sh_slot != 0;
  const int base = sh ? 1 : 0;
  int* gse = reinterpret_cast<int*>(p.ws + L.slot_expert);
  float* gco = reinterpret_cast<float*>(p.ws + L.coef);
  for (int i = lane; i < kMaxSlots * kMaxT; i += 32) gco[i] = 0.f;
  __syncwarp();
  if (own) {
    gse[base + srank] = p.world > 1 ? e - p.rank * p.ep_el : e;  // rows that chose the same expert write the same value
    gco[(base + srank) * kMaxT + t] = rt.sel_w[lane];
  }
  if (sh && lane < p.T) gco[lane] = rt.shared_coef[lane];
  if (lane < p.T) reinterpret_cast<float*>(p.ws + L.gate)[lane] = rt.shared_coef[lane];
  if (sh && lane == 0) gse[0] = -1;
  if (lane == 0) ctrl(p, L)[CTRL_NSLOTS] = static_cast<uint32_t>(base + total);
}

// Shared memory of the route kernel: the CTA's router rows (staged by bulk copies before the
// wait), the activation rows, then RouteTail.
// rw router rows per CTA, T activation rows.
__host__ __device__ inline size_t route_tail_offset(int H, bool w32, int rw, int T) {
  return align_up(static_cast<size_t>(rw) * H * (w32 ? 4 : 2) + static_cast<size_t>(T) * H * 2, 16);
}
// The route kernel's shared memory; `fused` (a cluster kernel follows) needs no selection scratch,
// which keeps a route CTA small enough to sit on an SM beside a cluster CTA of the previous layer.
__host__ __device__ inline size_t route_smem_bytes(int H, bool w32, int rw, int T, bool fused) {
  return route_tail_offset(H, w32, rw, T) + align_up(fused ? offsetof(RouteTail, logits) : sizeof(RouteTail), 16);
}

// Router logits, then the route table. Four warps per router row (plus the shared expert's gate
// row), each summing a quarter of H. The CTA's rows are copied into shared memory by the bulk-copy
// engine before griddepcontrol.wait (router weights never depend on the preceding kernel); the
// activation rows are staged after it. Every product is exact in fp64 (bf16 x bf16 or bf16 x fp32)
// and the products are summed in fp64, so the logit is the sum rounded once to fp32 (then to bf16
// for a bf16 router), + the optional logit bias. (Summing in fp64 replaced an fp32 hi + lo pair
// with the same precision for this purpose: its dependent chains were about 1 µs longer.) The shared gate row is rounded to bf16 as a bf16 linear's output.
// Each CTA also splits its share of x into the up kernel's activation tile (the exact e4m3 hi / lo
// of x * 2^e per row). The last CTA to finish (one gpu-scope fence per CTA, with no copies in
// flight) selects the experts of every row (one warp per row) and writes the table.
template <bool W32, int RW>
__global__ void __launch_bounds__(RW * kRouteSplit * 32) route_kernel(const __grid_constant__ Params p) {
  constexpr int kThr = RW * kRouteSplit * 32;
  extern __shared__ __align__(16) uint8_t rsm[];
  const WsLayout L = ws_layout(p.H, p.I);
  const int H = p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rw = warp / kRouteSplit, quarter = warp % kRouteSplit;  // row within the CTA, quarter of H
  const bool sh_gate_row = p.sh_w13 != nullptr && p.sh_gate != nullptr;
  const int rows = p.n_router + (sh_gate_row ? 1 : 0);
  const int row0 = blockIdx.x * RW;
  const int row = row0 + rw;
  const int wsz = W32 ? 4 : 2;
  uint8_t* wrows = rsm;  // [RW][H] weights
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(rsm + static_cast<size_t>(RW) * H * wsz);
  RouteTail& rt = *reinterpret_cast<RouteTail*>(rsm + route_tail_offset(H, W32, RW, p.T));
  if (threadIdx.x == 0) {
    mbar_init(&rt.bar, 1);
    fence_mbar_init();
    uint32_t bytes = 0;
    for (int r = row0; r < min(rows, row0 + RW); ++r) bytes += r < p.n_router ? H * wsz : H * 2;
    mbar_arrive_expect_tx(&rt.bar, bytes);
    for (int r = row0; r < min(rows, row0 + RW); ++r) {
      if (r < p.n_router)
        bulk_g2s(wrows + static_cast<size_t>(r - row0) * H * wsz,
                 static_cast<const uint8_t*>(p.router_w) + static_cast<size_t>(r) * H * wsz, H * wsz, &rt.bar);
      else
        bulk_g2s(wrows + static_cast<size_t>(r - row0) * H * wsz, p.sh_gate, H * 2, &rt.bar);
    }
  }
  if (threadIdx.x < kMaxT) rt.xmax[threadIdx.x] = 0u;
  __syncthreads();  // the maxima are zero before any thread folds into them
  griddep_wait();
  griddep_launch();
  {
    constexpr int kPer = kMaxT * kMaxH / 8 / kThr;
    const int n16 = p.T * H / 8;
    const uint4* xsrc = reinterpret_cast<const uint4*>(p.x);
    uint4 v[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int c = threadIdx.x + q * kThr;
      v[q] = c < n16 ? xsrc[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int c = threadIdx.x + q * kThr;
      if (c < n16) {
        reinterpret_cast<uint4*>(xs)[c] = v[q];
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v[q]);
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(__bfloat162float(e[i])));
        // a warp's chunks lie in one row (H / 8 is a multiple of 32): one shared atomic per warp (the
        // maxima only serve the x split, which the cluster kernel does itself)
        if (!p.fused) {
          const uint32_t wm = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
          if (lane == 0) atomicMax(&rt.xmax[c / (H / 8)], wm);
        }
      }
    }
  }
  if (threadIdx.x == 0 && !mbar_wait(&rt.bar, 0)) flag_error(p, L, STATUS_TIMEOUT);
  __syncthreads();
  // this CTA's share of the x split: 16-element chunks c = blockIdx.x + gridDim.x * j
  if (!p.fused) {
    uint8_t* img = p.ws + L.ximg;
    const int chunks = H / 16;
    for (int c = blockIdx.x + gridDim.x * static_cast<int>(threadIdx.x); c < p.T * chunks;
         c += gridDim.x * kThr) {
      const int t = c / chunks, k = (c % chunks) * 16;
      const uint4 v2[2] = {*reinterpret_cast<const uint4*>(xs + t * H + k), *reinterpret_cast<const uint4*>(xs + t * H + k + 8)};
      uint4 hi, lo;
      split16(v2, exp2i(split_exponent(__uint_as_float(rt.xmax[t]))), hi, lo);
      *reinterpret_cast<uint4*>(img + tc::swz_offset(t, k, kN)) = hi;
      *reinterpret_cast<uint4*>(img + tc::swz_offset(4 + t, k, kN)) = lo;
    }
    if (blockIdx.x == 0 && threadIdx.x < kMaxT)
      reinterpret_cast<float*>(p.ws + L.xinv)[threadIdx.x] = exp2i(-split_exponent(__uint_as_float(rt.xmax[threadIdx.x])));
  }
  float* logits = reinterpret_cast<float*>(p.ws + L.logits);
  if (row < rows) {
    const bool row_w32 = W32 && row < p.n_router;  // the shared gate row is bf16 in either case
    const uint8_t* wr = wrows + static_cast<size_t>(rw) * H * wsz;
    const int k0 = quarter * (H / kRouteSplit), k1 = k0 + H / kRouteSplit;
    for (int t = 0; t < p.T; ++t) {
      const __nv_bfloat16* xr = xs + t * H;
      double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 1
      for (int k = k0 + lane * 8; k < k1; k += 256) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xr + k);
        const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
        float w[8];
        if (row_w32) {
          const uint4 w0 = *reinterpret_cast<const uint4*>(wr + k * 4), w1 = *reinterpret_cast<const uint4*>(wr + k * 4 + 16);
          w[0] = __uint_as_float(w0.x), w[1] = __uint_as_float(w0.y), w[2] = __uint_as_float(w0.z), w[3] = __uint_as_float(w0.w);
          w[4] = __uint_as_float(w1.x), w[5] = __uint_as_float(w1.y), w[6] = __uint_as_float(w1.z), w[7] = __uint_as_float(w1.w);
        } else {
          const uint4 wv = *reinterpret_cast<const uint4*>(wr + k * 2);
          const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = __bfloat162float(we[i]);
        }
        // each product is exact in fp64 (bf16 x bf16 or bf16 x fp32), added with one rounding
#pragma unroll
        for (int i = 0; i < 8; ++i)
          acc[i & 3] = fma(static_cast<double>(__bfloat162float(xe[i])), static_cast<double>(w[i]), acc[i & 3]);
      }
      double sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) rt.part[rw][t][quarter] = sum;
    }
  }
  __syncthreads();
  if (threadIdx.x < RW * kMaxT) {
    const int r = threadIdx.x / kMaxT, t = threadIdx.x % kMaxT;
    if (row0 + r < rows && t < p.T) {
      double sum = rt.part[r][t][0];
#pragma unroll
      for (int q = 1; q < kRouteSplit; ++q) sum += rt.part[r][t][q];
      float v = __double2float_rn(sum);  // the logit rounded once
      if (row0 + r < p.n_router) {
        if (p.logits_bf16) v = bf16_round(v);
        if (p.logit_bias) v += p.logit_bias[row0 + r];
      } else {
        v = bf16_round(v);
      }
      logits[t * (kMaxRouter + 1) + row0 + r] = v;
    }
  }
  if (p.fused) return;  // the cluster kernel reads the logits once this kernel has completed
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(ctrl(p, L) + CTRL_ROUTE_COUNT, 1u);
    rt.last = old == gridDim.x - 1;
    if (rt.last) __threadfence();
  }
  __syncthreads();
  if (!rt.last) return;
  // last CTA: every logit is visible
  {
    constexpr int kPer = (kMaxT * (kMaxRouter + 1) + kThr - 1) / kThr;
    float v[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = threadIdx.x + q * kThr;
      v[q] = i < p.T * (kMaxRouter + 1) && i % (kMaxRouter + 1) < rows ? __ldcg(logits + i) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = threadIdx.x + q * kThr;
      if (i < kMaxT * (kMaxRouter + 1)) (&rt.logits[0][0])[i] = v[q];
    }
  }
  __syncthreads();
  if (warp < p.T) route_row(p, rt, warp, lane);
  __syncthreads();
  if (warp == 0) {
    write_table(p, L, rt, lane);
    if (lane == 0) ctrl(p, L)[CTRL_ROUTE_COUNT] = 0u;  // every CTA has counted: ready for the next call
  }
}

// Up: the activation tile of all H. Row t holds the e4m3 hi part of x[t] * 2^e_t (e_t maps the
// row's absolute maximum into [128, 256)), row 4 + t the lo remainder. Rows of absent tokens and
// rows 8-15 only feed accumulator columns that nothing reads, so they are left as they are. Run by
// the kSplitThreads split threads; every load is issued before the first use, and the threads
// fence their writes for the tensor core.
__device__ void split_x(const Params& p, uint8_t* bt, Aux& aux, int sidx) {
  const int H = p.H, chunks = H / 16, n = p.T * chunks;
  constexpr int kMaxTasks = (kMaxT * (kMaxH / 16) + kSplitThreads - 1) / kSplitThreads;
  if (sidx < kMaxT) aux.xmax[sidx] = 0u;
  named_bar(kBarSplit, kSplitThreads);
  uint4 v[kMaxTasks][2];
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = sidx + q * kSplitThreads;
    if (task < n) {
      const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(task / chunks) * H + (task % chunks) * 16);
      v[q][0] = src[0];
      v[q][1] = src[1];
    }
  }
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = sidx + q * kSplitThreads;
    if (task < n) atomicMax(&aux.xmax[task / chunks], __float_as_uint(abs_max16(v[q])));
  }
  named_bar(kBarSplit, kSplitThreads);
  if (sidx < kMaxT) aux.xinv[sidx] = exp2i(-split_exponent(__uint_as_float(aux.xmax[sidx])));
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = sidx + q * kSplitThreads;
    if (task < n) {
      const int t = task / chunks, c = task % chunks;
      uint4 hi, lo;
      split16(v[q], exp2i(split_exponent(__uint_as_float(aux.xmax[t]))), hi, lo);
      *reinterpret_cast<uint4*>(bt + tc::swz_offset(t, c * 16, kN)) = hi;
      *reinterpret_cast<uint4*>(bt + tc::swz_offset(4 + t, c * 16, kN)) = lo;
    }
  }
  tc::fence_proxy_async_smem();
}

// ------------------------------------------------------------------ epilogues
// Sum over accumulators (16 TMEM columns each, starting at the thread's lane address) of
// scale x (hi + lo) for this thread's weight row; scale(j) is the accumulator's combined scale.
template <int MaxAcc, typename ScaleFn>
__device__ __forceinline__ void reduce_acc(uint32_t taddr, int nacc, ScaleFn scale, float (&acc)[kMaxT]) {
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) acc[t] = 0.f;
#pragma unroll
  for (int j0 = 0; j0 < MaxAcc; j0 += 8) {
    if (j0 < nacc) {
      float v[8][8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < nacc) tc::tmem_ld8(taddr + (j0 + j) * 16, v[j]);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < nacc)
#pragma unroll
          for (int t = 0; t < kMaxT; ++t) acc[t] = fmaf(scale(j0 + j, t), v[j][t] + v[j][4 + t], acc[t]);
    }
  }
}

// The block scales of this thread's weight row (issued before the accumulator wait).
__device__ __forceinline__ void load_scales(const float* srow, int nkb, float* sc, int max_kb) {
#pragma unroll
  for (int kb = 0; kb < max_kb; ++kb) sc[kb] = kb < nkb ? __ldg(srow + kb) : 0.f;
}

// Up: thread r holds gate row 64*blk + r (r < 64) or up row I + 64*blk + r - 64; the up values go
// through shared memory to the gate threads, which apply SwiGLU, round h to bf16 (the reference's
// activation dtype) and write it straight into the down kernel's activation tile: each warp's 32
// values of a token form one group whose power-of-two scale maps its absolute maximum into
// [128, 256), and h * 2^e splits exactly into e4m3 hi + lo. The four epilogue warps meet at a
// named barrier (the caller makes their loop decisions uniform). Releases the accumulator buffer
// (acc_empty) as soon as it has been read.
__device__ void epilogue_up(const Params& p, const WsLayout& L, Aux& aux, uint32_t taddr, uint64_t* acc_empty,
                            int slot, int blk, int e, int lane, const float (&sc)[kMaxH / 128]) {
  const int r = 32 * e + lane;
  const int nkb = p.H / 128;
  float acc[kMaxT];
  reduce_acc<kMaxH / 128>(taddr, nkb, [&](int j, int) { return sc[j]; }, acc);
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(acc_empty);
  if (r >= kUpHalf)
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) aux.upv[r - kUpHalf][t] = acc[t] * aux.xinv[t];
  named_bar(kBarEpi, kEpiThreads);
  if (r >= kUpHalf) return;
  const bool shared_slot = slot == 0 && p.sh_slot;
  float hb[kMaxT];
  uint32_t am[kMaxT];
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) {
    hb[t] = 0.f;
    if (t < p.T) {
      // silu(g) = g * 1 / (1 + e^-g) with the fast exponential and an IEEE reciprocal; h is rounded
      // to bf16 right after, far above their error
      float gt = acc[t] * aux.xinv[t];
      float ut = aux.upv[r][t];
      if (shared_slot) {
        // the shared expert is a chain of bf16 modules: down(silu(gate(x)) * up(x))
        gt = bf16_round(gt);
        ut = bf16_round(ut);
        hb[t] = bf16_round(bf16_round(gt * __frcp_rn(1.f + __expf(-gt))) * ut);
      } else {
        hb[t] = bf16_round(gt * __frcp_rn(1.f + __expf(-gt)) * ut);
      }
    }
    am[t] = t < p.T ? __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(hb[t]))) : 0u;
  }
  uint8_t* img = p.ws + L.himg + static_cast<size_t>(slot) * L.himg_stride;
  const int kk = kUpHalf * blk + r;  // k index of the down projection
  float ex[kMaxT];
#pragma unroll
  for (int t = 0; t < kMaxT; t += 2) {
    if (t >= p.T) {
      ex[t] = ex[t + 1] = 1.f;
      continue;
    }
    const int e0 = split_exponent(__uint_as_float(am[t])), e1 = split_exponent(__uint_as_float(am[t + 1]));
    ex[t] = exp2i(-e0);
    ex[t + 1] = exp2i(-e1);
    uint16_t hi, lo;
    split2(hb[t] * exp2i(e0), hb[t + 1] * exp2i(e1), hi, lo);
    img[tc::swz_offset(t, kk, kN)] = static_cast<uint8_t>(hi & 0xFF);
    img[tc::swz_offset(4 + t, kk, kN)] = static_cast<uint8_t>(lo & 0xFF);
    if (t + 1 < p.T) {
      img[tc::swz_offset(t + 1, kk, kN)] = static_cast<uint8_t>(hi >> 8);
      img[tc::swz_offset(5 + t, kk, kN)] = static_cast<uint8_t>(lo >> 8);
    }
  }
  if (lane == 0) {
    float* hinv = reinterpret_cast<float*>(p.ws + L.hinv) + (static_cast<size_t>(slot) * (kMaxI / kGroup) + kk / kGroup) * kMaxT;
    *reinterpret_cast<float4*>(hinv) = make_float4(ex[0], ex[1], ex[2], ex[3]);
  }
}

// Down: thread r holds output row 128*nb + r of one slot; accumulator j covers the 32 k of one
// group of h, weighted by the weight's 128-block scale and the group's 2^-e. The partial carries the
// routing weight (the shared slot stays raw: the combine kernel rounds and gates it). Releases the
// accumulator buffer once it has been read.
__device__ void epilogue_down(const Params& p, const WsLayout& L, Aux& aux, uint32_t taddr, uint64_t* acc_empty,
                              int slot, int nb, int e, int lane, const float (&sc)[kMaxI / 128],
                              const float4 (&hv)[kMaxI / kGroup]) {
  const int r = 32 * e + lane;
  const int ngroups = p.I / kGroup;
  float acc[kMaxT];
  reduce_acc<kMaxI / kGroup>(
      taddr, ngroups,
      [&](int j, int t) {
        const float4 h = hv[j];
        return sc[j / (128 / kGroup)] * (t == 0 ? h.x : t == 1 ? h.y : t == 2 ? h.z : h.w);
      },
      acc);
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(acc_empty);
  const bool shared_slot = slot == 0 && p.sh_slot;
  float* part = partial_block(p, L, nb, slot);
  for (int t = 0; t < p.T; ++t)
    __stcg(part + t * kBlockRows + r, acc[t] * (shared_slot ? 1.f : aux.tab.coef[slot * kMaxT + t]));
}

// ------------------------------------------------------------------ up / down kernels
// One body for both streaming kernels (DOWN = false: up items, true: down items). Items are
// assigned statically (CTA c takes items c, c + gridDim, ...), so CTAs never wait on each other.
// map_w covers the routed experts ([E][rows][K] bytes), map_sh the shared expert.
//
// Route table: warp 4 reads the one the route kernel wrote (or builds it from the caller's ids).
// The up kernel reads it after griddepcontrol.wait; the down kernel before it, since everything it
// needs from the route kernel (or from the kernel that produced the ids) completed before the up
// kernel released its dependents. The down kernel's activation tiles come from the up kernel and
// are copied in after the wait.
template <bool DOWN>
__global__ void __launch_bounds__(kThreads, 1)
    expert_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map_w,
                  const __grid_constant__ CUtensorMap map_sh) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const SmemLayout S = smem_layout(DOWN, p.H, p.I);
  const WsLayout L = ws_layout(p.H, p.I);
  Aux& aux = *reinterpret_cast<Aux*>(smem + S.aux);
  Table& tab = aux.tab;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool sh = p.sh_slot != 0;
  const int per_slot = DOWN ? p.H / kBlockRows : p.I / kUpHalf;
  const int nkb = (DOWN ? p.I : p.H) / 128;  // 128-wide k blocks (slabs) per item
  const int nchunks = (nkb + 1) / 2;         // ring stages per item
  const int nacc = DOWN ? kDownAcc : kUpAcc;
  const uint32_t acc_cols = DOWN ? kDownTmemCols / kDownAcc : kUpTmemCols / kUpAcc;
  const uint32_t tmem_cols = DOWN ? kDownTmemCols : kUpTmemCols;

  if (tid == 0) {
    // the TMA descriptors are fetched while the CTA sets up
    tc::prefetch_map(&map_w);
    if (sh) tc::prefetch_map(&map_sh);
    for (int s = 0; s < S.nstages; ++s) {
      mbar_init(&aux.full[s], 1);   // the producer's arrive.expect_tx; the TMA bytes complete it
      mbar_init(&aux.empty[s], 1);  // tcgen05.commit after the stage's MMAs
    }
    for (int a = 0; a < nacc; ++a) {
      mbar_init(&aux.acc_full[a], 1);           // tcgen05.commit after the item's last MMA
      mbar_init(&aux.acc_empty[a], kEpiThreads / 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&aux.b_ready[b], 1);  // the producer's arrive.expect_tx; the copy completes it
      mbar_init(&aux.b_free[b], 1);   // tcgen05.commit after the item's MMAs
    }
    fence_mbar_init();
  }
  if (warp == kWarpMma) tc::tmem_alloc(&aux.tmem, tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux.tmem;

  if (warp == kWarpTma) {
    // ================================================================ TMA producer (lane 0 issues)
    int stage = 0;
    uint32_t empty_par = 1;
    bool ok = true;
    auto issue = [&](int idx, int c) -> bool {
      if (!mbar_wait(&aux.empty[stage], empty_par)) {
        flag_error(p, L, STATUS_TIMEOUT);
        return false;
      }
      const int slot = idx / per_slot, blk = idx % per_slot;
      const bool shared_slot = sh && slot == 0;
      const CUtensorMap* map = shared_slot ? &map_sh : &map_w;
      const int ex = shared_slot ? 0 : tab.expert[slot];
      uint8_t* dst = smem + S.stage + stage * kStageBytes;
      const int kb0 = 2 * c, nsl = min(2, nkb - kb0);
      mbar_arrive_expect_tx(&aux.full[stage], static_cast<uint32_t>(nsl * kSlabBytes));
      for (int j = 0; j < nsl; ++j) {
        const int kx = (kb0 + j) * 128;
        if (!DOWN) {
          tc::tma_load_3d(dst + j * kSlabBytes, map, kx, kUpHalf * blk, ex, &aux.full[stage]);
          tc::tma_load_3d(dst + j * kSlabBytes + kSlabBytes / 2, map, kx, p.I + kUpHalf * blk, ex, &aux.full[stage]);
        } else {
          tc::tma_load_3d(dst + j * kSlabBytes, map, kx, kBlockRows * blk, ex, &aux.full[stage]);
        }
      }
      if (++stage == S.nstages) {
        stage = 0;
        empty_par ^= 1u;
      }
      return true;
    };
    int k = 0, c = 0;  // item ordinal and chunk of the next weight stage
    auto item_of = [&](int kk) { return static_cast<int>(blockIdx.x) + kk * static_cast<int>(gridDim.x); };
    auto advance = [&]() {
      if (++c == nchunks) {
        c = 0;
        ++k;
      }
    };
    if (lane == 0) {
      if (!DOWN && sh) {
        // shared-expert stages need no routing: up to one ring of them before the table exists
        for (int n = 0; ok && n < S.nstages && item_of(k) < per_slot; ++n) {
          ok = issue(item_of(k), c);
          advance();
        }
      }
      if (!DOWN && p.mode == 1) {
        // the route kernel left x split into this kernel's activation tile: one bulk copy from L2
        griddep_wait();
        griddep_launch();
        mbar_arrive_expect_tx(&aux.b_ready[0], static_cast<uint32_t>(S.b_bytes));
        bulk_g2s(smem + S.b, p.ws + L.ximg, static_cast<uint32_t>(S.b_bytes), &aux.b_ready[0]);
      }
    }
    __syncwarp();
    named_bar(kBarTable, kThreads);
    const int n_items = aux.n_slots * per_slot;
    if (lane == 0) {
      if (!DOWN) {
        while (ok && item_of(k) < n_items) {
          ok = issue(item_of(k), c);
          advance();
        }
      } else {
        // weights of the first ring before the wait; afterwards each item's activation tile (from
        // the up kernel) is copied in ahead of any further weight stage of a later item
        for (int n = 0; ok && n < S.nstages && item_of(k) < n_items; ++n) {
          ok = issue(item_of(k), c);
          advance();
        }
        griddep_wait();
        griddep_launch();
        fence_proxy_async();
        int kb = 0;  // next item whose activation tile is copied
        while (ok) {
          if (item_of(kb) < n_items && kb <= k) {
            const int bb = kb & 1;
            if (!mbar_wait(&aux.b_free[bb], ((kb >> 1) & 1) ^ 1u)) {
              flag_error(p, L, STATUS_TIMEOUT);
              break;
            }
            const int slot = item_of(kb) / per_slot;
            mbar_arrive_expect_tx(&aux.b_ready[bb], static_cast<uint32_t>(S.b_bytes));
            bulk_g2s(smem + S.b + bb * S.b_bytes, p.ws + L.himg + static_cast<size_t>(slot) * L.himg_stride,
                     static_cast<uint32_t>(S.b_bytes), &aux.b_ready[bb]);
            ++kb;
          } else if (item_of(k) < n_items) {
            ok = issue(item_of(k), c);
            advance();
          } else {
            break;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ================================================================ MMA issuer (lane 0 issues)
    if (!DOWN && p.mode == 0) {
      griddep_wait();  // x comes from the preceding kernel
      griddep_launch();
      split_x(p, smem + S.b, aux, lane);  // the MMA warp helps split x (split index 0-31)
    }
    named_bar(kBarTable, kThreads);
    const int n_items = aux.n_slots * per_slot;
    if (lane == 0) {
      bool ok = true;
      if (!DOWN && p.mode == 1 && !mbar_wait(&aux.b_ready[0], 0)) {
        flag_error(p, L, STATUS_TIMEOUT);
        ok = false;
      }
      const uint32_t idesc = tc::idesc_e4m3(kTileRows, kN);
      int stage = 0;
      uint32_t full_par = 0;
      for (int k = 0; ok; ++k) {
        const int idx = blockIdx.x + k * gridDim.x;
        if (idx >= n_items) break;
        const int ab = k % nacc, bb = k & 1;
        if (!mbar_wait(&aux.acc_empty[ab], ((k / nacc) & 1) ^ 1u) ||
            (DOWN && !mbar_wait(&aux.b_ready[bb], (k >> 1) & 1))) {
          flag_error(p, L, STATUS_TIMEOUT);
          break;
        }
        tc::fence_after_sync();  // the epilogue's reads of this accumulator are ordered before the MMAs
        const uint32_t bt = smem_u32(smem + S.b + (DOWN ? bb * S.b_bytes : 0));
        const uint32_t d = tmem + ab * acc_cols;
        for (int c = 0; c < nchunks; ++c) {
          // the TMA's bytes completing the stage's barrier make them visible to the tensor core
          if (!mbar_wait(&aux.full[stage], full_par)) {
            flag_error(p, L, STATUS_TIMEOUT);
            ok = false;
            break;
          }
          const uint32_t a = smem_u32(smem + S.stage + stage * kStageBytes);
          for (int j = 0; j < 2 && 2 * c + j < nkb; ++j) {
            const int kb = 2 * c + j;
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              // up: one accumulator per 128-wide k block; down: one per 32-wide group of h
              const uint32_t col = DOWN ? (kb * 4 + k4) * 16 : kb * 16;
              tc::mma_f8(d + col, tc::smem_desc(a + j * kSlabBytes + 32 * k4),
                         tc::smem_desc(bt + kb * kBSlabBytes + 32 * k4), idesc, DOWN ? false : k4 > 0);
            }
          }
          tc::mma_commit(&aux.empty[stage]);  // the stage is free once these MMAs have read it
          if (++stage == S.nstages) {
            stage = 0;
            full_par ^= 1u;
          }
        }
        if (!ok) break;
        tc::mma_commit(&aux.acc_full[ab]);
        if (DOWN) tc::mma_commit(&aux.b_free[bb]);
      }
    }
    __syncwarp();
  } else if (warp < kWarpEpi) {
    // ================================================================ warps 2-3: split x (up, routing given)
    if (!DOWN && p.mode == 0) {
      griddep_wait();
      griddep_launch();
      split_x(p, smem + S.b, aux, 32 + (warp - 2) * 32 + lane);
    }
    named_bar(kBarTable, kThreads);
  } else {
    // ================================================================ epilogue (+ route table)
    const int e = warp - kWarpEpi;  // TMEM lane quarter (warp % 4)
    if (!DOWN) {
      griddep_wait();
      griddep_launch();
    }
    if (warp == kWarpEpi) {
      const int n = p.mode == 1 ? table_from_ws(p, L, lane, tab) : table_from_ids(p, L, lane, tab, !DOWN);
      if (lane == 0) aux.n_slots = n;
      if (!DOWN && p.mode == 1 && lane < kMaxT) aux.xinv[lane] = __ldcg(reinterpret_cast<const float*>(p.ws + L.xinv) + lane);
    } else if (!DOWN && p.mode == 0) {
      split_x(p, smem + S.b, aux, 96 + (warp - kWarpEpi - 1) * 32 + lane);
    }
    named_bar(kBarTable, kThreads);
    if (DOWN) {
      griddep_wait();
      griddep_launch();
      if (p.mode == 0 && blockIdx.x == 0 && warp == kWarpEpi && lane == 0)
        ctrl(p, L)[CTRL_NSLOTS] = static_cast<uint32_t>(aux.n_slots);  // for the combine kernel
    }
    const int n_items = aux.n_slots * per_slot;
    for (int k = 0;; ++k) {
      const int idx = blockIdx.x + k * gridDim.x;
      if (idx >= n_items) break;
      const int ab = k % nacc;
      const int slot = idx / per_slot, blk = idx % per_slot;
      const ExpertRef ex = expert_ref(p, slot, tab.expert);
      const int r = 32 * e + lane;
      float sc13[kMaxH / 128], sc2[kMaxI / 128];
      float4 hv[kMaxI / kGroup];
      if (!DOWN) {
        const int wrow = r < kUpHalf ? kUpHalf * blk + r : p.I + kUpHalf * blk + (r - kUpHalf);
        load_scales(ex.s13 + static_cast<size_t>(wrow / ex.srows) * nkb, nkb, sc13, kMaxH / 128);
      } else {
        load_scales(ex.s2 + static_cast<size_t>((kBlockRows * blk + r) / ex.srows) * nkb, nkb, sc2, kMaxI / 128);
        const float4* hsrc =
            reinterpret_cast<const float4*>(p.ws + L.hinv) + static_cast<size_t>(slot) * (kMaxI / kGroup);
#pragma unroll
        for (int g = 0; g < kMaxI / kGroup; ++g)
          hv[g] = g < p.I / kGroup ? __ldcg(hsrc + g) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      bool ready = true;
      if (lane == 0) ready = mbar_wait(&aux.acc_full[ab], (k / nacc) & 1);
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!DOWN) {
        // the up epilogue's warps meet at named barriers: they continue or stop together
        if (lane == 0) aux.epi_ok[e] = ready ? 1 : 0;
        named_bar(kBarEpi, kEpiThreads);
        ready = aux.epi_ok[0] && aux.epi_ok[1] && aux.epi_ok[2] && aux.epi_ok[3];
        named_bar(kBarEpi, kEpiThreads);  // epi_ok may be rewritten for the next item
      }
      if (!ready) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * e) << 16) + ab * acc_cols;
      if (!DOWN)
        epilogue_up(p, L, aux, taddr, &aux.acc_empty[ab], slot, blk, e, lane, sc13);
      else
        epilogue_down(p, L, aux, taddr, &aux.acc_empty[ab], slot, blk, e, lane, sc2, hv);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kWarpMma) tc::tmem_dealloc(tmem, tmem_cols);
}

// ------------------------------------------------------------------ combine kernel
// y = bf16(bf16(bf16(sum of routed partials) + bias) + bf16(sigmoid gate * bf16(shared))): the
// rounding points of fp8_moe_forward's bf16 output, Speaker's bias add (engine.py:236-237) and
// speaker_forward's bf16 tensor sum (engine.py:158). One thread per output element.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const __grid_constant__ Params p) {
  const WsLayout L = ws_layout(p.H, p.I);
  const int e = blockIdx.x * kCombineThreads + threadIdx.x;
  const int t = e / p.H, n = e % p.H;
  const bool active = t < p.T;
  float bias = 0.f;
  if (active && p.out_bias) bias = __ldg(p.out_bias + n);
  griddep_wait();
  griddep_launch();
  const bool sh = p.sh_w13 != nullptr;  // the layer has a shared expert (computed where sh_slot)
  float R = 0.f, S = 0.f;               // routed sum, raw shared-expert output
  if (active) {
    // the slot count and every slot's partial are requested at once: one L2 round trip; slots past
    // the count hold stale data and are masked
    const int nb = n / kBlockRows, r = n % kBlockRows;
    const float* col = partial_block(p, L, nb, 0) + t * kBlockRows + r;
    const uint32_t n_slots = __ldcg(ctrl(p, L) + CTRL_NSLOTS);
    float v[kMaxSlots];
#pragma unroll
    for (int s = 0; s < kMaxSlots; ++s) v[s] = __ldcg(col + s * kMaxT * kBlockRows);
    R = (!p.sh_slot && n_slots > 0u) ? v[0] : 0.f;
#pragma unroll
    for (int s = 1; s < kMaxSlots; ++s) R += static_cast<uint32_t>(s) < n_slots ? v[s] : 0.f;
    S = (p.sh_slot && n_slots > 0u) ? v[0] : 0.f;
  }
  if (p.world > 1) {
    // one-shot all-reduce over NVLink: every rank stores its two partials into every rank's arena
    // (region of the call's epoch parity), the last CTA raises this rank's flag on every rank, and
    // each CTA sums the ranks' partials in rank order once every flag holds the epoch
    __shared__ int s_last;
    const ep::EpLayout A = ep::ep_layout(p.world, p.ep_tl, p.top_k, p.H);
    uint32_t* own_ctrl = reinterpret_cast<uint32_t*>(p.ep_arena[p.rank] + A.ctrl);
    const uint32_t epoch = __ldcg(own_ctrl + ep::EP_RED_EPOCH) + 1u;
    const size_t region = static_cast<size_t>(epoch & 1u) * p.world * 2 * kMaxT * p.H;
    if (active)
      for (int d = 0; d < p.world; ++d) {
        float* red = reinterpret_cast<float*>(p.ep_arena[d] + A.red) + region;
        __stcg(red + (static_cast<size_t>(p.rank * 2 + 0) * kMaxT + t) * p.H + n, R);
        __stcg(red + (static_cast<size_t>(p.rank * 2 + 1) * kMaxT + t) * p.H + n, S);
      }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();  // cumulative over the CTA's stores, ordered by the barrier above
      s_last = atomicAdd(own_ctrl + ep::EP_RED_COUNT, 1u) == gridDim.x - 1 ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {
      if (threadIdx.x < p.world) {
        __threadfence_system();
        ep::st_release_sys(reinterpret_cast<uint32_t*>(p.ep_arena[threadIdx.x] + A.redflag) + p.rank, epoch);
      }
      if (threadIdx.x == 0) {
        own_ctrl[ep::EP_RED_COUNT] = 0u;
        own_ctrl[ep::EP_RED_EPOCH] = epoch;
      }
    }
    if (threadIdx.x < p.world &&
        !ep::wait_epoch(reinterpret_cast<const uint32_t*>(p.ep_arena[p.rank] + A.redflag) + threadIdx.x, epoch))
      flag_error(p, L, STATUS_TIMEOUT);
    __syncthreads();
    if (active) {
      const float* red = reinterpret_cast<const float*>(p.ep_arena[p.rank] + A.red) + region;
      R = 0.f;
      S = 0.f;
      for (int s = 0; s < p.world; ++s) {
        R += __ldcg(red + (static_cast<size_t>(s * 2 + 0) * kMaxT + t) * p.H + n);
        S += __ldcg(red + (static_cast<size_t>(s * 2 + 1) * kMaxT + t) * p.H + n);
      }
    }
  }
  if (!active) return;
  const float gate = sh ? __ldcg(reinterpret_cast<const float*>(p.ws + L.gate) + t) : 0.f;
  float acc = bf16_round(R);
  if (p.out_bias) acc = bf16_round(acc + bias);
  if (sh) acc += bf16_round(gate * bf16_round(S));
  p.y[static_cast<size_t>(t) * p.H + n] = __float2bfloat16_rn(acc);
}

#include "moe_cluster.cuh"

}  // namespace moe
}  // namespace dm3

// ------------------------------------------------------------------ host launcher
namespace dm3 {

size_t moe_ws_bytes(int H, int I) { return moe::ws_layout(H, I).total; }

namespace {

template <typename... KArgs, typename... Args>
int launch_one(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t stream, const char* name,
               Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
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
    set_error(std::string(name) + " launch: " + cudaGetErrorString(err));
    return 2;
  }
  return 0;
}

}  // namespace

int launch_moe(const moe::Params& p, cudaStream_t stream) {
  const moe::SmemLayout su = moe::smem_layout(false, p.H, p.I), sd = moe::smem_layout(true, p.H, p.I);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return 2;
  }
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    // One shared-memory carveout for all four kernels: an SM switching carveouts between
    // consecutive kernels must drain first, which would undo the overlap of dependent launches.
    bool ok = cudaFuncSetAttribute(moe::expert_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   227 * 1024) == cudaSuccess &&
              cudaFuncSetAttribute(moe::expert_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   227 * 1024) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(moe::expert_kernel<false>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(moe::expert_kernel<true>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    for (auto k : {moe::route_kernel<false, 4>, moe::route_kernel<true, 4>, moe::route_kernel<false, 2>,
                   moe::route_kernel<true, 2>}) {
      ok = ok && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(moe::route_smem_bytes(kMaxH, true, 4, kMaxT, false))) ==
                     cudaSuccess;
      ok = ok && cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    }
    ok = ok && cudaFuncSetAttribute(moe::combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(moe::layer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    227 * 1024) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(moe::layer_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    if (!ok) {
      set_error("cudaFuncSetAttribute(moe) failed");
      return 2;
    }
    configured[dev] = true;
  }
  // TMA maps of the expert weights: routed experts [E][2I][H] and [E][H][I] bytes with the caller's
  // expert strides; the shared expert as a single expert. Up items take 64-row boxes (gate and up
  // halves), down items 128-row boxes.
  const uint64_t H = static_cast<uint64_t>(p.H), I = static_cast<uint64_t>(p.I);
  CUtensorMap m13, m2, msh13, msh2;
  if (!tensor_map_3d(&m13, p.w13, H, 2 * I, static_cast<uint64_t>(p.n_experts), H, static_cast<uint64_t>(p.w13_stride),
                     moe::kUpHalf) ||
      !tensor_map_3d(&m2, p.w2, I, H, static_cast<uint64_t>(p.n_experts), I, static_cast<uint64_t>(p.w2_stride),
                     moe::kBlockRows))
    return 2;
  if (p.sh_w13) {
    if (!tensor_map_3d(&msh13, p.sh_w13, H, 2 * I, 1, H, 2 * I * H, moe::kUpHalf) ||
        !tensor_map_3d(&msh2, p.sh_w2, I, H, 1, I, H * I, moe::kBlockRows))
      return 2;
  } else {
    msh13 = m13;
    msh2 = m2;
  }
  const int sms = sm_count(dev);
  int launches = 0;
  if (p.fused) {
    // route (logits + x split), then the cluster kernel: one cluster of kCl CTAs per (possible slot,
    // quarter of I)
    const int rows = p.n_router + (p.sh_w13 && p.sh_gate ? 1 : 0);
    const bool w32 = p.router_bf16 == 0;
    // two router rows per CTA: one small route CTA per SM, beside the previous layer's cluster CTA
    if (int rc = launch_one(w32 ? moe::route_kernel<true, 2> : moe::route_kernel<false, 2>, (rows + 1) / 2,
                            2 * moe::kRouteSplit * 32, moe::route_smem_bytes(p.H, w32, 2, p.T, true), stream,
                            "moe route", p))
      return rc;
    const int clusters = (p.T * p.top_k + (p.sh_slot ? 1 : 0)) * (p.I / 128);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(clusters * moe::kCl);
    cfg.blockDim = dim3(moe::kThreads);
    cfg.dynamicSmemBytes = moe::fsmem_layout(p.H, p.I).total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = moe::kCl;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, moe::layer_kernel, p, m13, m2, msh13, msh2);
    if (err != cudaSuccess) {
      set_error(std::string("moe cluster launch: ") + cudaGetErrorString(err));
      return 2;
    }
    const int pairs = p.T * p.H / 2;
    if (int rc = launch_one(moe::finish_kernel, (pairs + moe::kFinishThreads - 1) / moe::kFinishThreads,
                            moe::kFinishThreads, 0, stream, "moe finish", p))
      return rc;
    note_launches(3);
    return 0;
  }
  if (p.mode == 1) {
    const int rows = p.n_router + (p.sh_w13 && p.sh_gate ? 1 : 0);
    const bool w32 = p.router_bf16 == 0;
    if (int rc = launch_one(w32 ? moe::route_kernel<true, 4> : moe::route_kernel<false, 4>,
                            (rows + moe::kRouteWarps - 1) / moe::kRouteWarps, moe::kRouteThreads,
                            moe::route_smem_bytes(p.H, w32, moe::kRouteWarps, p.T, false), stream, "moe route", p))
      return rc;
    ++launches;
  }
  if (int rc = launch_one(moe::expert_kernel<false>, sms, moe::kThreads, su.total, stream, "moe up", p, m13, msh13))
    return rc;
  if (int rc = launch_one(moe::expert_kernel<true>, sms, moe::kThreads, sd.total, stream, "moe down", p, m2, msh2))
    return rc;
  if (int rc = launch_one(moe::combine_kernel, (p.T * p.H + moe::kCombineThreads - 1) / moe::kCombineThreads,
                          moe::kCombineThreads, 0, stream, "moe combine", p))
    return rc;
  note_launches(launches + 3);
  return 0;
}

}  // namespace dm3

// ------------------------------------------------------------------ C ABI
namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int T, int H, int I, int top_k, const void* x, const void* w13, int64_t w13_stride,
                 const void* s13, const void* w2, int64_t w2_stride, const void* s2, int srows, void* y,
                 void* workspace, size_t workspace_bytes) {
  using namespace dm3;
  if (T < 1 || T > kMaxT) return set_error("T must be in [1, 4] for the decode kernel"), 1;
  if (H < 128 || H > kMaxH || H % 128) return set_error("H must be a multiple of 128 in [128, 2048]"), 1;
  if (I < 128 || I > kMaxI || I % 128) return set_error("I must be a multiple of 128 in [128, 512]"), 1;
  if (top_k < 1 || top_k > kMaxTopK) return set_error("top_k must be in [1, 8]"), 1;
  if (!x || !w13 || !s13 || !w2 || !s2 || !y || !workspace) return set_error("null pointer argument"), 1;
  if (!aligned16(x) || !aligned16(w13) || !aligned16(w2) || !aligned16(workspace))
    return set_error("x, w13, w2 and workspace must be 16-byte aligned"), 1;
  if (w13_stride % 16 || w2_stride % 16) return set_error("expert strides must be multiples of 16 bytes"), 1;
  if (srows != 1 && srows != 128) return set_error("srows must be 1 or 128"), 1;
  if (workspace_bytes < dm3::moe_ws_bytes(H, I)) return set_error("workspace too small"), 4;
  return 0;
}

}  // namespace

extern "C" size_t dm3_moe_workspace_bytes(int T, int H, int I) {
  (void)T;  // offsets do not depend on the row count, so one workspace serves every T of (H, I)
  return dm3::moe_ws_bytes(H, I);
}

extern "C" int dm3_moe_forward(const void* x, int T, int H, int I, const int64_t* ids, const void* weights,
                               int top_k, int n_experts, const void* w13, int64_t w13_stride, const float* s13,
                               int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2,
                               int64_t s2_stride, int srows, void* y, void* workspace, size_t workspace_bytes,
                               void* stream) {
  dm3::note_launches(0);
  int rc = check_common(T, H, I, top_k, x, w13, w13_stride, s13, w2, w2_stride, s2, srows, y, workspace,
                        workspace_bytes);
  if (rc) return rc;
  if (!ids || !weights) return dm3::set_error("ids and weights are required"), 1;
  if (n_experts < 1) return dm3::set_error("n_experts must be >= 1"), 1;
  if (T * top_k > 32) return dm3::set_error("T * top_k must be <= 32"), 1;
  dm3::moe::Params p{};
  p.T = T;
  p.H = H;
  p.I = I;
  p.top_k = top_k;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.mode = 0;
  p.ids = ids;
  p.rw = static_cast<const __nv_bfloat16*>(weights);
  p.n_experts = n_experts;
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
  p.ws = static_cast<uint8_t*>(workspace);
  return dm3::launch_moe(p, static_cast<cudaStream_t>(stream));
}

static int moe_layer_impl(const void* x, int T, int H, int I, const void* router_w, int router_dtype, int n_router,
                          int top_k, int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride,
                          const float* s13, int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2,
                          int64_t s2_stride, int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2,
                          const float* sh_s2, int sh_srows, const void* sh_gate, const float* out_bias, void* y,
                          int64_t* ids_out, void* w_out, void* workspace, size_t workspace_bytes, void* stream,
                          int world, int rank, int tokens_per_rank, void* const* arenas) {
  dm3::note_launches(0);
  int rc = check_common(T, H, I, top_k, x, w13, w13_stride, s13, w2, w2_stride, s2, srows, y, workspace,
                        workspace_bytes);
  if (rc) return rc;
  if (!router_w) return dm3::set_error("router weight is required"), 1;
  if (router_dtype != 0 && router_dtype != 1) return dm3::set_error("router_dtype must be 0 (fp32) or 1 (bf16)"), 1;
  if (n_router < top_k || n_router > dm3::kMaxRouter) return dm3::set_error("n_router must be in [top_k, 256]"), 1;
  if (!aligned16(router_w)) return dm3::set_error("router weight must be 16-byte aligned"), 1;
  if (T * top_k > 32) return dm3::set_error("T * top_k must be <= 32"), 1;
  if (sh_w13) {
    if (!sh_s13 || !sh_w2 || !sh_s2) return dm3::set_error("shared expert needs w13, s13, w2, s2"), 1;
    if (!aligned16(sh_w13) || !aligned16(sh_w2)) return dm3::set_error("shared expert weights must be 16-byte aligned"), 1;
    if (sh_srows != 1 && sh_srows != 128) return dm3::set_error("sh_srows must be 1 or 128"), 1;
    if (sh_gate && !aligned16(sh_gate)) return dm3::set_error("shared gate must be 16-byte aligned"), 1;
  }
  dm3::moe::Params p{};
  p.T = T;
  p.H = H;
  p.I = I;
  p.top_k = top_k;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.mode = 1;
  p.router_w = router_w;
  p.router_bf16 = router_dtype;
  p.n_router = n_router;
  p.logits_bf16 = logits_bf16;
  p.logit_bias = logit_bias;
  p.ids_out = ids_out;
  p.w_out = static_cast<__nv_bfloat16*>(w_out);
  p.n_experts = n_router;
  p.w13 = static_cast<const uint8_t*>(w13);
  p.w13_stride = w13_stride;
  p.s13 = s13;
  p.s13_stride = s13_stride;
  p.w2 = static_cast<const uint8_t*>(w2);
  p.w2_stride = w2_stride;
  p.s2 = s2;
  p.s2_stride = s2_stride;
  p.srows = srows;
  p.sh_w13 = static_cast<const uint8_t*>(sh_w13);
  p.sh_s13 = sh_s13;
  p.sh_w2 = static_cast<const uint8_t*>(sh_w2);
  p.sh_s2 = sh_s2;
  p.sh_srows = sh_w13 ? sh_srows : 128;
  p.sh_gate = static_cast<const __nv_bfloat16*>(sh_gate);
  p.out_bias = out_bias;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ws = static_cast<uint8_t*>(workspace);
  p.sh_slot = sh_w13 != nullptr && (world <= 1 || rank == 0) ? 1 : 0;
  if (world > 1) {
    if (world > 8 || rank < 0 || rank >= world || n_router % world || !arenas || tokens_per_rank < 1)
      return dm3::set_error("bad expert-parallel arguments (world in [2, 8], rank, n_router % world, arenas)"), 1;
    for (int r = 0; r < world; ++r)
      if (!arenas[r]) return dm3::set_error("null arena pointer"), 1;
    p.world = world;
    p.rank = rank;
    p.ep_tl = tokens_per_rank;
    p.ep_el = n_router / world;
    p.n_experts = p.ep_el;  // w13 / w2 hold this rank's experts
    for (int r = 0; r < 8; ++r) p.ep_arena[r] = r < world ? static_cast<uint8_t*>(arenas[r]) : nullptr;
  }
  // one kernel of thread-block clusters for the expert phase where the shape allows it
  p.fused = world <= 1 && dm3::moe::cluster_shape_ok(H, I) && dm3::cluster_path_enabled() ? 1 : 0;
  return dm3::launch_moe(p, static_cast<cudaStream_t>(stream));
}

extern "C" int dm3_moe_layer(const void* x, int T, int H, int I, const void* router_w, int router_dtype,
                             int n_router, int top_k, int logits_bf16, const float* logit_bias, const void* w13,
                             int64_t w13_stride, const float* s13, int64_t s13_stride, const void* w2,
                             int64_t w2_stride, const float* s2, int64_t s2_stride, int srows, const void* sh_w13,
                             const float* sh_s13, const void* sh_w2, const float* sh_s2, int sh_srows,
                             const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out, void* w_out,
                             void* workspace, size_t workspace_bytes, void* stream) {
  return moe_layer_impl(x, T, H, I, router_w, router_dtype, n_router, top_k, logits_bf16, logit_bias, w13, w13_stride,
                        s13, s13_stride, w2, w2_stride, s2, s2_stride, srows, sh_w13, sh_s13, sh_w2, sh_s2, sh_srows,
                        sh_gate, out_bias, y, ids_out, w_out, workspace, workspace_bytes, stream, 1, 0, 0, nullptr);
}

extern "C" int dm3_moe_layer_ep(const void* x, int T, int H, int I, const void* router_w, int router_dtype,
                                int n_router, int top_k, int logits_bf16, const float* logit_bias, const void* w13,
                                int64_t w13_stride, const float* s13, int64_t s13_stride, const void* w2,
                                int64_t w2_stride, const float* s2, int64_t s2_stride, int srows,
                                const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                                int sh_srows, const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out,
                                void* w_out, int world, int rank, int tokens_per_rank, void* const* arenas,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (world < 2) return dm3::set_error("dm3_moe_layer_ep needs world >= 2"), 1;
  return moe_layer_impl(x, T, H, I, router_w, router_dtype, n_router, top_k, logits_bf16, logit_bias, w13, w13_stride,
                        s13, s13_stride, w2, w2_stride, s2, s2_stride, srows, sh_w13, sh_s13, sh_w2, sh_s2, sh_srows,
                        sh_gate, out_bias, y, ids_out, w_out, workspace, workspace_bytes, stream, world, rank,
                        tokens_per_rank, arenas);
}

extern "C" int dm3_moe_status(void* workspace, uint32_t* status, void* stream) {
  if (!workspace || !status) return dm3::set_error("null pointer argument"), 1;
  uint32_t* word = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + dm3::moe::ws_layout(128, 128).ctrl) +
                   dm3::moe::CTRL_STATUS;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, word, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemsetAsync(word, 0, 4, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
    return dm3::set_error("reading the workspace status failed"), 2;
  *status = v;
  return (v & dm3::STATUS_TIMEOUT) ? 3 : 0;
}

// ------------------------------------------------------------------ allocation-free variant
// For callers that cannot allocate device memory at all: a caller running inside another
// runtime's memory pool, a plugin host that hands out only its own buffers, or code on a path
// where cudaMalloc is forbidden (it may synchronise the device and is not allowed during stream
// capture). The fused layer's scratch then lives in this file-scope device array instead of a
// caller-provided workspace. Every GPU that loads the library reserves it until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = 1572864;  // 1.5 MiB: the workspace of H <= 2048, I <= 512
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
// Device address of g_noalloc_scratch per device (the host-side symbol is not a device address),
// published once the array has been zeroed on that device.
std::atomic<void*> g_noalloc_ptr[64];
std::mutex g_noalloc_mu;

// The array's device address on device `dev` (current), zeroing it on the first call there: the
// memset is waited for before the address is published, so no caller can launch on a half-cleared
// array. Null (with the error set) when the runtime refuses, e.g. during stream capture.
void* noalloc_scratch(int dev, cudaStream_t stream) {
  void* ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (ptr != nullptr) return ptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  ptr = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
  if (ptr != nullptr) return ptr;
  cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (err != cudaSuccess) return dm3::set_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(err)), nullptr;
  err = cudaMemsetAsync(ptr, 0, kNoAllocScratchBytes, stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess)
    return dm3::set_error(std::string("clearing the static scratch (make the first call outside stream capture): ") +
                          cudaGetErrorString(err)),
           nullptr;
  g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
  return ptr;
}

}  // namespace

extern "C" int dm3_moe_layer_noalloc(const void* x, int T, int H, int I, const void* router_w, int router_dtype,
                                     int n_router, int top_k, int logits_bf16, const float* logit_bias,
                                     const void* w13, int64_t w13_stride, const float* s13, int64_t s13_stride,
                                     const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride, int srows,
                                     const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                                     int sh_srows, const void* sh_gate, const float* out_bias, void* y,
                                     int64_t* ids_out, void* w_out, void* stream) {
  dm3::note_launches(0);
  if (H > dm3::kMaxH || I > dm3::kMaxI || (H > 0 && I > 0 && dm3::moe_ws_bytes(H, I) > kNoAllocScratchBytes))
    return dm3::set_error("the static 1.5 MiB scratch holds the layer of H <= 2048 and I <= 512 only"), 4;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return dm3::set_error("no usable current CUDA device"), 2;
  void* scratch = noalloc_scratch(dev, static_cast<cudaStream_t>(stream));
  if (scratch == nullptr) return 2;
  return dm3_moe_layer(x, T, H, I, router_w, router_dtype, n_router, top_k, logits_bf16, logit_bias, w13, w13_stride,
                       s13, s13_stride, w2, w2_stride, s2, s2_stride, srows, sh_w13, sh_s13, sh_w2, sh_s2, sh_srows,
                       sh_gate, out_bias, y, ids_out, w_out, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int dm3_moe_noalloc_status(uint32_t* status, void* stream) {
  if (!status) return dm3::set_error("null pointer argument"), 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return dm3::set_error("no usable current CUDA device"), 2;
  *status = 0;
  void* scratch = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) return 0;  // no call has run on this device yet
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* word = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(scratch) + dm3::moe::ws_layout(128, 128).ctrl) +
                   dm3::moe::CTRL_STATUS;
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, word, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
    return dm3::set_error("reading the static scratch's status failed"), 2;
  // a call that stopped early may have left counters and partial sums behind: clear the whole array
  if (v != 0 && (cudaMemsetAsync(scratch, 0, kNoAllocScratchBytes, s) != cudaSuccess ||
                 cudaStreamSynchronize(s) != cudaSuccess))
    return dm3::set_error("clearing the static scratch failed"), 2;
  *status = v;
  return (v & dm3::STATUS_TIMEOUT) ? 3 : 0;
}

namespace dm3 {
// This file's copy of the device wait limit on the current device (dm3_set_wait_limit_ns).
int wait_limit_moe_decode(uint64_t ns) { return static_cast<int>(set_wait_limit_here(ns)); }
}  // namespace dm3
