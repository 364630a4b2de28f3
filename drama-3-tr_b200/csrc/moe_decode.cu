// Fused decode MoE layer for B200 (sm_100a): one persistent launch per layer covers
//   router logits (exact fp64 dot, rounded once) -> softmax / top-k / renormalise
//   -> gate/up products over block-FP8 experts -> SwiGLU (bf16 h)
//   -> down products -> weighted combine with the sigmoid-gated shared expert (+ bias).
//
// Work is a queue of items claimed with atomics, in dependency order:
//   R items   router rows (+ the shared-expert gate row)
//   G items   8 gate rows + the matching 8 up rows of one expert (slot), over all of H
//   D items   64 rows of one expert's down projection, over all of I
//   F items   final sum over slots of 64 output rows (+ bias) -> bf16
// Every item waits only on items with smaller indices, and a CTA handles its items in increasing
// order, so progress never needs co-residency of the grid. Each CTA runs
//   2 x 4 consumer warps  FP8 mma.sync on tiles staged in shared memory; the two groups take
//                         alternate stages of the ring, so two items are computed at once
//   1 producer warp       claims items, issues one cp.async.bulk per contiguous weight block
//                         (and its scale rows) into a 4-stage ring
//   1 signal warp         publishes finished items at gpu scope (fence + red.release), batching
//                         the fence so neither consumers nor stage reuse wait on a round trip
// Activations (x, and h for the down projection) are split exactly into e4m3 hi + lo columns of
// one m16n8k32 tile (cols 0-3 hi of rows 0-3, cols 4-7 lo), so raw e4m3 weight bytes feed the
// tensor core with no dequantisation pass; the per-128 block scales are applied to each 128-wide
// k block partial in fp32.
#include <cfloat>
#include <cmath>

#include "dm3_common.cuh"
#include "dm3_internal.h"

namespace dm3 {
namespace moe {

constexpr int kStages = 4;  // even: stage s belongs to consumer group s % 2
constexpr int kGroups = 2;
constexpr int kGroupWarps = 4;
constexpr int kGroupThreads = kGroupWarps * 32;
constexpr int kConsumerWarps = kGroups * kGroupWarps;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kGRows = 8;   // gate rows per G item (plus the same number of up rows)
constexpr int kDRows = 64;  // down-projection rows per D item
constexpr int kFRows = 64;  // output rows per F item
constexpr int kRRows = 2;   // router rows per R item
constexpr int kPad = 64;    // smem row padding (bytes) of the thread-written activation tiles
constexpr int kBarAll = 3;  // named barrier of all consumer warps (groups use 1 and 2)

enum : int { ITEM_NONE = 0, ITEM_R = 1, ITEM_G = 2, ITEM_D = 3, ITEM_F = 4, ITEM_END = 5 };

struct Params {
  int T, H, I, top_k;
  const __nv_bfloat16* x;
  int mode;  // 0 = routing given (ids/weights), 1 = router in-kernel
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
  // scale rows travel by bulk copy when their addresses and sizes are 16-byte multiples;
  // otherwise consumers read them from global memory
  int sc13_bulk, sc2_bulk, sh_sc13_bulk, sh_sc2_bulk;
};

// ------------------------------------------------------------------ workspace layout
// Control words, then per-slot / per-block counters, the route table, logits, the bf16 SwiGLU
// activations (with their per-row absolute maxima) and the fp32 per-slot partial outputs.
struct WsLayout {
  size_t ctrl, g_done, d_done, slot_expert, coef, logits, hblk, partial, total;
  size_t hblk_stride;  // bytes per slot: kMaxT*I bf16 + 16 bytes of amax words (T-independent)
  size_t amax_off;     // offset of the amax words inside a slot block
};
enum : int { CTRL_QUEUE = 0, CTRL_ROUTE_COUNT = 1, CTRL_ROUTE_FLAG = 2, CTRL_EXIT = 3, CTRL_STATUS = 4,
             CTRL_NSLOTS = 5, CTRL_WORDS = 16 };

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline WsLayout ws_layout(int T, int H, int I) {
  WsLayout L;
  size_t o = 0;
  L.ctrl = o;
  o += CTRL_WORDS * 4;
  L.g_done = o;
  o += align_up(kMaxSlots * 4, 16);
  L.d_done = o;
  o += align_up((kMaxH / kDRows) * 4, 16);
  L.slot_expert = o;
  o += align_up(kMaxSlots * 4, 16);
  L.coef = o;
  o += align_up(kMaxSlots * kMaxT * 4, 16);
  L.logits = o;
  o += align_up(kMaxT * (kMaxRouter + 1) * 4, 16);
  o = align_up(o, 128);
  L.amax_off = static_cast<size_t>(kMaxT) * I * 2;
  L.hblk_stride = align_up(L.amax_off + 16, 128);
  L.hblk = o;
  o += L.hblk_stride * kMaxSlots;
  L.partial = o;
  o += static_cast<size_t>(kMaxSlots) * T * H * 4;
  L.total = align_up(o, 256);
  return L;
}

// ------------------------------------------------------------------ shared-memory layout
struct Desc {
  int kind, a, b, c;  // R: a = first row, b = rows; G: a = slot, b = block; D: a = slot, b = n-block
};

struct SmemLayout {
  int stage_bytes, stage, xq, xb, grp, grp_bytes, table, misc, total;
  int xp, hp;           // padded row pitches of the activation tiles (bytes)
  int g_sc, d_sc, d_h;  // offsets inside a stage: G scales, D scales, D staged h block
};

__host__ __device__ inline SmemLayout smem_layout(int T, int H, int I) {
  SmemLayout S;
  S.xp = H + kPad;
  S.hp = I + kPad;
  const int nkh = H / 128, nki = I / 128;
  S.g_sc = 2 * kGRows * H;
  S.d_sc = kDRows * I;
  S.d_h = kDRows * I + kDRows * nki * 4;
  const int r_bytes = kRRows * H * 4;
  const int g_bytes = S.g_sc + 2 * kGRows * nkh * 4;
  const int d_bytes = S.d_h + static_cast<int>(align_up(kMaxT * I * 2 + 16, 16));
  int sb = r_bytes > g_bytes ? r_bytes : g_bytes;
  sb = sb > d_bytes ? sb : d_bytes;
  S.stage_bytes = static_cast<int>(align_up(sb, 128));
  int o = 0;
  S.stage = o;
  o += kStages * S.stage_bytes;
  S.xq = o;
  o += 8 * S.xp;
  S.xb = o;
  o += static_cast<int>(align_up(T * H * 2, 128));
  // per consumer group: hq (8 x hp), red (4 warps x 32 lanes x 4 floats), hinv (4 floats)
  S.grp_bytes = static_cast<int>(align_up(8 * S.hp + kGroupWarps * 32 * 16 + 16, 128));
  S.grp = o;
  o += kGroups * S.grp_bytes;
  S.table = o;  // slot_expert[kMaxSlots] int, coef[kMaxSlots][kMaxT] float
  o += static_cast<int>(align_up(kMaxSlots * 4 + kMaxSlots * kMaxT * 4 + 64, 128));
  S.misc = o;  // descs, barriers, xinv, flags
  o += 1024;
  S.total = o;
  return S;
}

struct Misc {
  Desc desc[kStages];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t done[kStages];
  float xinv[kMaxT];
  int n_slots;
  int abort;
};

struct Group {  // per-consumer-group scratch
  uint8_t* hq;
  float* red;
  float* hinv;
};

__device__ __forceinline__ Group group_scratch(uint8_t* smem, const SmemLayout& S, int gid) {
  uint8_t* b = smem + S.grp + gid * S.grp_bytes;
  Group g;
  g.hq = b;
  g.red = reinterpret_cast<float*>(b + 8 * S.hp);
  g.hinv = reinterpret_cast<float*>(b + 8 * S.hp + kGroupWarps * 32 * 16);
  return g;
}

struct Counts {
  int nR, nGS, nDS;  // R items, shared G items, shared D items
  int g_per_slot, d_per_slot, n_f;
};

__device__ __forceinline__ Counts item_counts(const Params& p) {
  Counts c;
  const bool sh = p.sh_w13 != nullptr;
  const int rows = p.mode == 1 ? p.n_router + (sh && p.sh_gate ? 1 : 0) : 0;
  c.nR = (rows + kRRows - 1) / kRRows;
  c.g_per_slot = p.I / kGRows;
  c.d_per_slot = p.H / kDRows;
  c.nGS = sh ? c.g_per_slot : 0;
  c.nDS = sh ? c.d_per_slot : 0;
  c.n_f = p.H / kFRows;
  return c;
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
  int srows, sc13_bulk, sc2_bulk;
};

__device__ __forceinline__ ExpertRef expert_ref(const Params& p, int slot, const int* tab_expert) {
  ExpertRef r;
  if (slot == 0 && p.sh_w13 != nullptr) {
    r.w13 = p.sh_w13;
    r.s13 = p.sh_s13;
    r.w2 = p.sh_w2;
    r.s2 = p.sh_s2;
    r.srows = p.sh_srows;
    r.sc13_bulk = p.sh_sc13_bulk;
    r.sc2_bulk = p.sh_sc2_bulk;
  } else {
    const int e = tab_expert[slot];
    r.w13 = p.w13 + static_cast<size_t>(e) * p.w13_stride;
    r.s13 = p.s13 + static_cast<size_t>(e) * p.s13_stride;
    r.w2 = p.w2 + static_cast<size_t>(e) * p.w2_stride;
    r.s2 = p.s2 + static_cast<size_t>(e) * p.s2_stride;
    r.srows = p.srows;
    r.sc13_bulk = p.sc13_bulk;
    r.sc2_bulk = p.sc2_bulk;
  }
  return r;
}

// ------------------------------------------------------------------ route table helpers
// Builds slots from (token, expert, weight) pairs held one per lane (lanes >= n invalid).
// Slot order: optional shared expert first, then distinct routed experts ascending.
// Writes slot_expert / coef into the given arrays (smem or global) and returns the slot count.
__device__ int build_slots(int lane, int n, int t, int e, float w, int shared, int T, int* slot_expert,
                           float* coef, const float shared_coef[kMaxT]) {
  const bool valid = lane < n && e >= 0;
  const int key = valid ? e : 0x7fffffff;
  const unsigned same = __match_any_sync(0xffffffffu, key);
  const bool first = valid && (__ffs(same) - 1 == lane);
  const unsigned firsts = __ballot_sync(0xffffffffu, first);
  int rank = 0;
  for (int j = 0; j < 32; ++j) {
    const int kj = __shfl_sync(0xffffffffu, key, j);
    if (((firsts >> j) & 1u) && kj < key) ++rank;
  }
  const int n_routed = __popc(firsts);
  const int base = shared ? 1 : 0;
  const int n_slots = base + n_routed;
  // one writer per (slot, row): a repeated pair (only possible with malformed ids) is summed in lane order
  const int key2 = valid ? ((rank << 3) | t) : -1 - lane;
  const unsigned grp = __match_any_sync(0xffffffffu, key2);
  float wsum = 0.f;
  for (int j = 0; j < 32; ++j) {
    const float wj = __shfl_sync(0xffffffffu, w, j);
    if ((grp >> j) & 1u) wsum += wj;
  }
  for (int i = lane; i < kMaxSlots * kMaxT; i += 32) coef[i] = 0.f;
  __syncwarp();
  if (first) slot_expert[base + rank] = e;
  if (valid && (__ffs(grp) - 1 == lane)) coef[(base + rank) * kMaxT + t] = wsum;
  if (shared && lane == 0) {
    slot_expert[0] = -1;
    for (int tt = 0; tt < T; ++tt) coef[tt] = shared_coef[tt];
  }
  __syncwarp();
  return n_slots;
}

// ------------------------------------------------------------------ consumer: x split
// Each of the first T consumer warps loads one activation row, keeps a bf16 copy for the router
// and writes its exact e4m3 hi / lo split (prescaled by a power of two) as B-operand columns.
__device__ void prepare_x(const Params& p, uint8_t* xq, __nv_bfloat16* xb, Misc* misc, int warp, int lane,
                          int xp) {
  const int H = p.H;
  if (warp < p.T) {
    const __nv_bfloat16* xr = p.x + static_cast<size_t>(warp) * H;
    float amax = 0.f;
    for (int k = lane * 8; k < H; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      *reinterpret_cast<uint4*>(xb + static_cast<size_t>(warp) * H + k) = v;
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(e[i])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const int e = split_exponent(amax);
    const float sc = exp2i(e);
    if (lane == 0) misc->xinv[warp] = exp2i(-e);
    uint8_t* hi = xq + warp * xp;
    uint8_t* lo = xq + (4 + warp) * xp;
    for (int k = lane * 8; k < H; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xb + static_cast<size_t>(warp) * H + k);
      const __nv_bfloat16* e8 = reinterpret_cast<const __nv_bfloat16*>(&v);
      uint16_t h4[4], l4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        split2(__bfloat162float(e8[2 * i]) * sc, __bfloat162float(e8[2 * i + 1]) * sc, h4[i], l4[i]);
      *reinterpret_cast<uint2*>(hi + k) = make_uint2(h4[0] | (uint32_t(h4[1]) << 16), h4[2] | (uint32_t(h4[3]) << 16));
      *reinterpret_cast<uint2*>(lo + k) = make_uint2(l4[0] | (uint32_t(l4[1]) << 16), l4[2] | (uint32_t(l4[3]) << 16));
    }
  }
}

// ------------------------------------------------------------------ consumer: R item
// Router logits for d.b rows: exact dot products in fp64 (bf16 x bf16 / fp32 products are exact
// and 2048 of them sum without loss in practice), rounded once to fp32 (and to bf16 for a bf16
// router), + the optional logit bias. The shared expert's gate row is rounded to bf16 as a bf16
// linear's output.
__device__ void consume_r(const Params& p, const WsLayout& L, const uint8_t* stage, const Desc& d,
                          const __nv_bfloat16* xb, int gw, int lane) {
  const int H = p.H;
  float* logits = reinterpret_cast<float*>(p.ws + L.logits);
  const int n = d.b * p.T;
  for (int job = gw; job < n; job += kGroupWarps) {
    const int r = job / p.T, t = job % p.T;
    const int row = d.a + r;
    const bool is_router = row < p.n_router;
    const bool row_f32 = is_router && !p.router_bf16;
    const uint8_t* w = stage + r * H * 4;
    const __nv_bfloat16* xr = xb + static_cast<size_t>(t) * H;
    double acc = 0.0;
    for (int k = lane; k < H; k += 32) {
      const double xv = static_cast<double>(__bfloat162float(xr[k]));
      const double wv = row_f32 ? static_cast<double>(reinterpret_cast<const float*>(w)[k])
                                : static_cast<double>(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[k]));
      acc = fma(xv, wv, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      float v = __double2float_rn(acc);
      if (is_router) {
        if (p.logits_bf16) v = bf16_round(v);
        if (p.logit_bias) v += p.logit_bias[row];
      } else {
        v = bf16_round(v);
      }
      logits[t * (kMaxRouter + 1) + row] = v;
    }
  }
}

// ------------------------------------------------------------------ consumer: G item
// 8 gate rows (tile rows 0-7) and the matching 8 up rows (tile rows 8-15) of one expert against the
// split activations: lane (g, q) ends with gate row g and up row g for rows 2q, 2q+1 (hi columns,
// after folding the lo columns in), so SwiGLU happens in registers. The group's 4 warps split
// the 128-wide k blocks and reduce through shared memory.
__device__ void consume_g(const Params& p, const WsLayout& L, const SmemLayout& S, const uint8_t* xq,
                          const uint8_t* stage, const Desc& d, const Misc* misc, const Group& G, const int* tab_expert,
                          int gw, int lane, int bar_id) {
  const int H = p.H;
  const int g = lane >> 2, q = lane & 3;
  const int nkb = H / 128;
  const int slot = d.a;
  const ExpertRef ex = expert_ref(p, slot, tab_expert);
  const float* sc = reinterpret_cast<const float*>(stage + S.g_sc);
  const int gate_row = d.b * kGRows + g, up_row = p.I + d.b * kGRows + g;
  const int sg_row = ex.srows == 1 ? g : 0;  // index into the staged gate scale rows
  const uint8_t* row_lo = stage + g * H;
  const uint8_t* row_hi = stage + (kGRows + g) * H;
  const uint8_t* bcol = xq + g * S.xp;
  const bool bvalid = (g & 3) < p.T;
  float tot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int kb = gw; kb < nkb; kb += kGroupWarps) {
    float part[1][4];
    const int kbs[1] = {kb};
    tile_kblocks<1>(part, row_lo, row_hi, bcol, true, true, bvalid, kbs, q);
    const float a0[4] = {part[0][0], part[0][1], part[0][2], part[0][3]}, a1[4] = {0.f, 0.f, 0.f, 0.f};
    float sgv, suv;
    if (ex.sc13_bulk) {
      sgv = sc[sg_row * nkb + kb];
      suv = sc[(kGRows + sg_row) * nkb + kb];
    } else {
      sgv = __ldg(ex.s13 + static_cast<size_t>(gate_row / ex.srows) * nkb + kb);
      suv = __ldg(ex.s13 + static_cast<size_t>(up_row / ex.srows) * nkb + kb);
    }
    tot[0] = fmaf(a0[0] + a1[0], sgv, tot[0]);
    tot[1] = fmaf(a0[1] + a1[1], sgv, tot[1]);
    tot[2] = fmaf(a0[2] + a1[2], suv, tot[2]);
    tot[3] = fmaf(a0[3] + a1[3], suv, tot[3]);
  }
  // fold lo columns (q = 2, 3) onto hi columns (q = 0, 1)
#pragma unroll
  for (int i = 0; i < 4; ++i) tot[i] += __shfl_down_sync(0xffffffffu, tot[i], 2);
  *reinterpret_cast<float4*>(G.red + (gw * 32 + lane) * 4) = make_float4(tot[0], tot[1], tot[2], tot[3]);
  named_bar(bar_id, kGroupThreads);
  if (gw == 0) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kGroupWarps; ++w) {
      const float4 r = *reinterpret_cast<const float4*>(G.red + (w * 32 + lane) * 4);
      v[0] += r.x;
      v[1] += r.y;
      v[2] += r.z;
      v[3] += r.w;
    }
    const bool shared_slot = slot == 0 && p.sh_w13 != nullptr;
    uint8_t* hb = p.ws + L.hblk + static_cast<size_t>(slot) * L.hblk_stride;
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(hb);
    uint32_t* amax_w = reinterpret_cast<uint32_t*>(hb + L.amax_off);
    float am[2] = {0.f, 0.f};
    if (q < 2) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int t = 2 * q + c;
        if (t < p.T) {
          float gt = v[c] * misc->xinv[t];
          float ut = v[2 + c] * misc->xinv[t];
          float hv;
          if (shared_slot) {
            // the shared expert is a chain of bf16 modules: down(silu(gate(x)) * up(x))
            gt = bf16_round(gt);
            ut = bf16_round(ut);
            hv = bf16_round(gt / (1.f + expf(-gt))) * ut;
          } else {
            hv = gt / (1.f + expf(-gt)) * ut;
          }
          const __nv_bfloat16 hbv = __float2bfloat16_rn(hv);
          h[static_cast<size_t>(t) * p.I + gate_row] = hbv;
          am[c] = fabsf(__bfloat162float(hbv));
        }
      }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      am[0] = fmaxf(am[0], __shfl_xor_sync(0xffffffffu, am[0], o));
      am[1] = fmaxf(am[1], __shfl_xor_sync(0xffffffffu, am[1], o));
    }
    if (g == 0 && q < 2) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int t = 2 * q + c;
        if (t < p.T) atomicMax(amax_w + t, __float_as_uint(am[c]));
      }
    }
  }
  named_bar(bar_id, kGroupThreads);  // red is reused by the group's next item
}

// ------------------------------------------------------------------ consumer: D item
// 64 rows of one expert's down projection against its staged h (bf16, split into e4m3 hi / lo
// columns here); each group warp owns 16 rows over all of I. Routed slots carry their routing
// weight into the partial; the shared slot stays raw and is gated in the F item.
__device__ void consume_d(const Params& p, const WsLayout& L, const SmemLayout& S, const uint8_t* stage,
                          const Desc& d, const Group& G, const float* coef_tab, const int* tab_expert, int gw,
                          int lane, int gtid, int bar_id) {
  const int I = p.I, T = p.T;
  const int nkb = I / 128;
  const int slot = d.a;
  const ExpertRef ex = expert_ref(p, slot, tab_expert);
  const uint8_t* hsrc = stage + S.d_h;
  const float* sc = reinterpret_cast<const float*>(stage + S.d_sc);
  {
    const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(hsrc);
    const float* amax = reinterpret_cast<const float*>(hsrc + static_cast<size_t>(kMaxT) * I * 2);
    const int pairs = T * I / 2;
    for (int i = gtid; i < pairs; i += kGroupThreads) {
      const int t = (2 * i) / I, k = (2 * i) % I;
      const float s = exp2i(split_exponent(amax[t]));
      uint16_t hi, lo;
      split2(__bfloat162float(hv[2 * i]) * s, __bfloat162float(hv[2 * i + 1]) * s, hi, lo);
      *reinterpret_cast<uint16_t*>(G.hq + t * S.hp + k) = hi;
      *reinterpret_cast<uint16_t*>(G.hq + (4 + t) * S.hp + k) = lo;
    }
    if (gtid < T) G.hinv[gtid] = exp2i(-split_exponent(amax[gtid]));
  }
  named_bar(bar_id, kGroupThreads);
  const int g = lane >> 2, q = lane & 3;
  const int r_lo = gw * 16 + g, r_hi = gw * 16 + 8 + g;
  const uint8_t* row_lo = stage + r_lo * I;
  const uint8_t* row_hi = stage + r_hi * I;
  const uint8_t* bcol = G.hq + g * S.hp;
  const bool bvalid = (g & 3) < T;
  const int n_lo = d.b * kDRows + r_lo, n_hi = d.b * kDRows + r_hi;
  float tot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int kb = 0; kb < nkb; ++kb) {
    float part[1][4];
    const int kbs[1] = {kb};
    tile_kblocks<1>(part, row_lo, row_hi, bcol, true, true, bvalid, kbs, q);
    const float a0[4] = {part[0][0], part[0][1], part[0][2], part[0][3]}, a1[4] = {0.f, 0.f, 0.f, 0.f};
    float s0, s1;
    if (ex.sc2_bulk) {
      s0 = sc[(ex.srows == 1 ? r_lo : 0) * nkb + kb];
      s1 = sc[(ex.srows == 1 ? r_hi : 0) * nkb + kb];
    } else {
      s0 = __ldg(ex.s2 + static_cast<size_t>(n_lo / ex.srows) * nkb + kb);
      s1 = __ldg(ex.s2 + static_cast<size_t>(n_hi / ex.srows) * nkb + kb);
    }
    tot[0] = fmaf(a0[0] + a1[0], s0, tot[0]);
    tot[1] = fmaf(a0[1] + a1[1], s0, tot[1]);
    tot[2] = fmaf(a0[2] + a1[2], s1, tot[2]);
    tot[3] = fmaf(a0[3] + a1[3], s1, tot[3]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) tot[i] += __shfl_down_sync(0xffffffffu, tot[i], 2);
  if (q < 2) {
    float* part = reinterpret_cast<float*>(p.ws + L.partial) + static_cast<size_t>(slot) * T * p.H;
    const bool shared_slot = slot == 0 && p.sh_w13 != nullptr;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int t = 2 * q + c;
      if (t < T) {
        const float k = G.hinv[t] * (shared_slot ? 1.f : coef_tab[slot * kMaxT + t]);
        __stcg(part + static_cast<size_t>(t) * p.H + n_lo, tot[c] * k);
        __stcg(part + static_cast<size_t>(t) * p.H + n_hi, tot[2 + c] * k);
      }
    }
  }
  named_bar(bar_id, kGroupThreads);  // hq / hinv are reused by the group's next item
}

// ------------------------------------------------------------------ route finalisation
// Run by one warp after every R item finished: top-k per row over the logits, renormalised
// weights, slot table. Mirrors Speaker.__call__ (engine.py:233-235): probs = softmax(logits),
// (w, ids) = probs.topk(k), w = (w / w.sum()).to(bf16). Selection uses the logits themselves
// (softmax is monotonic), ties to the lower index.
__device__ void finalize_route(const Params& p, const WsLayout& L, int lane) {
  const int T = p.T, E = p.n_router, K = p.top_k;
  const float* logits = reinterpret_cast<const float*>(p.ws + L.logits);
  int my_t = 0, my_e = -1;
  float my_w = 0.f;
  float shared_coef[kMaxT] = {1.f, 1.f, 1.f, 1.f};
  for (int t = 0; t < T; ++t) {
    float lv[kMaxRouter / 32];
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < kMaxRouter / 32; ++i) {
      const int e = lane + 32 * i;
      lv[i] = e < E ? __ldcg(logits + t * (kMaxRouter + 1) + e) : -FLT_MAX;
      m = fmaxf(m, lv[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float z = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxRouter / 32; ++i)
      if (lane + 32 * i < E) z += expf(lv[i] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    unsigned taken = 0u;
    float pj[kMaxTopK];
    int ej[kMaxTopK];
    for (int j = 0; j < K; ++j) {
      float bv = -FLT_MAX;
      int be = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < kMaxRouter / 32; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !(taken & (1u << i)) && (lv[i] > bv || (lv[i] == bv && e < be))) {
          bv = lv[i];
          be = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ov > bv || (ov == bv && oe < be)) {
          bv = ov;
          be = oe;
        }
      }
      if ((be & 31) == lane) taken |= 1u << (be >> 5);
      ej[j] = be;
      pj[j] = expf(bv - m) / z;
    }
    float s = 0.f;
    for (int j = 0; j < K; ++j) s += pj[j];
    for (int j = 0; j < K; ++j) {
      const __nv_bfloat16 wb = __float2bfloat16_rn(pj[j] / s);
      if (lane == t * K + j) {
        my_t = t;
        my_e = ej[j];
        my_w = __bfloat162float(wb);
      }
      if (lane == 0) {
        if (p.ids_out) p.ids_out[t * K + j] = ej[j];
        if (p.w_out) p.w_out[t * K + j] = wb;
      }
    }
    if (p.sh_gate) {
      const float gl = __ldcg(logits + t * (kMaxRouter + 1) + E);
      shared_coef[t] = bf16_round(1.f / (1.f + expf(-gl)));
    }
  }
  int* slot_expert = reinterpret_cast<int*>(p.ws + L.slot_expert);
  float* coef = reinterpret_cast<float*>(p.ws + L.coef);
  const int n_slots = build_slots(lane, T * K, my_t, my_e, my_w, p.sh_w13 != nullptr, T, slot_expert, coef,
                                  shared_coef);
  if (lane == 0) {
    uint32_t* c = reinterpret_cast<uint32_t*>(p.ws + L.ctrl);
    c[CTRL_NSLOTS] = static_cast<uint32_t>(n_slots);
    __threadfence();
    st_release(c + CTRL_ROUTE_FLAG, 1u);
  }
  __syncwarp();
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) moe_decode_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const SmemLayout S = smem_layout(p.T, p.H, p.I);
  const WsLayout L = ws_layout(p.T, p.H, p.I);
  const Counts C = item_counts(p);
  Misc* misc = reinterpret_cast<Misc*>(smem + S.misc);
  int* tab_expert = reinterpret_cast<int*>(smem + S.table);
  float* tab_coef = reinterpret_cast<float*>(smem + S.table + kMaxSlots * 4);
  uint32_t* ctl = reinterpret_cast<uint32_t*>(p.ws + L.ctrl);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool sh = p.sh_w13 != nullptr;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&misc->full[s], 1);  // the producer's arrive.expect_tx; bytes complete the phase
      mbar_init(&misc->empty[s], kGroupWarps + 1);  // the owning group's warps + the signal warp
      mbar_init(&misc->done[s], kGroupWarps);
    }
    misc->abort = 0;
    misc->n_slots = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();
  griddep_launch();

  if (warp == kProducerWarp) {
    // ================================================================ producer
    bool have_table = false;
    int n_slots = 0;
    int total = 0x7fffffff;
    auto load_table = [&]() -> bool {
      if (p.mode == 0) {
        // routing given: every CTA builds the slot table from ids / weights
        const int n = p.T * p.top_k;
        int t = 0, e = -1;
        float w = 0.f;
        if (lane < n) {
          t = lane / p.top_k;
          const int64_t id = p.ids[lane];
          if (id >= 0 && id < p.n_experts) {
            e = static_cast<int>(id);
            w = __bfloat162float(p.rw[lane]);
          } else {
            flag_error(p, L, STATUS_BAD_EXPERT);
          }
        }
        const float one[kMaxT] = {1.f, 1.f, 1.f, 1.f};
        n_slots = build_slots(lane, n, t, e, w, sh ? 1 : 0, p.T, tab_expert, tab_coef, one);
      } else {
        bool ok = true;
        if (lane == 0) ok = wait_geq(ctl + CTRL_ROUTE_FLAG, 1u);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
          return false;
        }
        n_slots = static_cast<int>(__ldcg(ctl + CTRL_NSLOTS));
        const int* gse = reinterpret_cast<const int*>(p.ws + L.slot_expert);
        const float* gco = reinterpret_cast<const float*>(p.ws + L.coef);
        for (int i = lane; i < kMaxSlots; i += 32) tab_expert[i] = __ldcg(gse + i);
        for (int i = lane; i < kMaxSlots * kMaxT; i += 32) tab_coef[i] = __ldcg(gco + i);
      }
      __syncwarp();
      const int routed = n_slots - (sh ? 1 : 0);
      total = C.nR + C.nGS + routed * C.g_per_slot + C.nDS + routed * C.d_per_slot + C.n_f;
      if (lane == 0) misc->n_slots = n_slots;
      have_table = true;
      return true;
    };
    if (p.mode == 0) load_table();

    int stage = 0;
    uint32_t empty_par = 1;
    int ends = 0;
    // items are claimed kClaim at a time, one chunk ahead of use, so the claim's round trip overlaps
    // the copies of the current chunk; a CTA still handles its items in increasing order
    constexpr uint32_t kClaim = 2;
    uint32_t cur = 0, ahead = 0, sub = 0;
    if (lane == 0) {
      cur = atomicAdd(ctl + CTRL_QUEUE, kClaim);
      ahead = atomicAdd(ctl + CTRL_QUEUE, kClaim);
    }
    for (;;) {
      Desc d{ITEM_END, 0, 0, 0};
      if (ends == 0) {
        const int idx = static_cast<int>(__shfl_sync(0xffffffffu, cur + sub, 0));
        if (lane == 0 && ++sub == kClaim) {
          sub = 0;
          cur = ahead;
          ahead = atomicAdd(ctl + CTRL_QUEUE, kClaim);
        }
        if (misc->abort) {
          d.kind = ITEM_END;
        } else if (idx < C.nR) {
          const int rows = p.n_router + ((sh && p.sh_gate) ? 1 : 0);
          d.kind = ITEM_R;
          d.a = idx * kRRows;
          d.b = min(kRRows, rows - d.a);
        } else if (idx < C.nR + C.nGS) {
          d.kind = ITEM_G;
          d.a = 0;
          d.b = idx - C.nR;
        } else if (!have_table && !load_table()) {
          if (lane == 0) misc->abort = 1;
          d.kind = ITEM_END;
        } else if (idx < total) {
          const int routed = n_slots - (sh ? 1 : 0);
          int j = idx - C.nR - C.nGS;
          if (j < routed * C.g_per_slot) {
            d.kind = ITEM_G;
            d.a = (sh ? 1 : 0) + j / C.g_per_slot;
            d.b = j % C.g_per_slot;
          } else {
            j -= routed * C.g_per_slot;
            if (j < C.nDS + routed * C.d_per_slot) {
              d.kind = ITEM_D;
              d.a = j / C.d_per_slot;
              d.b = j % C.d_per_slot;
            } else {
              d.kind = ITEM_F;
              d.b = j - C.nDS - routed * C.d_per_slot;
            }
          }
        }
      }

      if (d.kind == ITEM_F) {
        // final sum over slots of 64 output rows, done by the producer warp itself:
        // y = bf16(bf16(bf16(sum of routed) + bias) + bf16(sigmoid gate * bf16(shared))), the rounding
        // points of fp8_moe_forward's bf16 output, Speaker's bias add (engine.py:236-237) and
        // speaker_forward's bf16 tensor sum (engine.py:158)
        const uint32_t* d_done = reinterpret_cast<const uint32_t*>(p.ws + L.d_done);
        bool ok = true;
        if (lane == 0) ok = wait_geq(d_done + d.b, static_cast<uint32_t>(n_slots));
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) {
            flag_error(p, L, STATUS_TIMEOUT);
            misc->abort = 1;
          }
          continue;
        }
        const float* part = reinterpret_cast<const float*>(p.ws + L.partial);
        const int s0 = sh ? 1 : 0;
        for (int r = lane; r < kFRows; r += 32) {
          const int n = d.b * kFRows + r;
          for (int t = 0; t < p.T; ++t) {
            float acc = 0.f;
            for (int s = s0; s < n_slots; ++s) acc += __ldcg(part + (static_cast<size_t>(s) * p.T + t) * p.H + n);
            acc = bf16_round(acc);
            if (p.out_bias) acc = bf16_round(acc + p.out_bias[n]);
            if (sh) {
              const float shv = bf16_round(__ldcg(part + static_cast<size_t>(t) * p.H + n));
              acc += bf16_round(tab_coef[t] * shv);
            }
            p.y[static_cast<size_t>(t) * p.H + n] = __float2bfloat16_rn(acc);
          }
        }
        continue;
      }

      // wait for the stage to be free
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&misc->empty[stage], empty_par);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;  // the consumers cannot be reached any more
      }
      uint8_t* st = smem + S.stage + stage * S.stage_bytes;
      uint64_t* full = &misc->full[stage];
      if (lane == 0) {
        misc->desc[stage] = d;
        if (d.kind == ITEM_R) {
          const int esz = p.router_bf16 ? 2 : 4;
          uint32_t bytes = 0;
          for (int r = 0; r < d.b; ++r) bytes += (d.a + r < p.n_router ? esz : 2) * p.H;
          mbar_arrive_expect_tx(full, bytes);
          for (int r = 0; r < d.b; ++r) {
            const int row = d.a + r;
            if (row < p.n_router)
              bulk_g2s(st + r * p.H * 4, static_cast<const uint8_t*>(p.router_w) + static_cast<size_t>(row) * p.H * esz,
                       esz * p.H, full);
            else
              bulk_g2s(st + r * p.H * 4, p.sh_gate, 2 * p.H, full);
          }
        } else if (d.kind == ITEM_G) {
          const ExpertRef ex = expert_ref(p, d.a, tab_expert);
          const int nkb = p.H / 128;
          const int r0 = d.b * kGRows, u0 = p.I + d.b * kGRows;
          const uint32_t blk = kGRows * p.H;
          const uint32_t sbytes = ex.sc13_bulk ? (ex.srows == 1 ? 2u * kGRows * nkb * 4 : 2u * nkb * 4) : 0u;
          mbar_arrive_expect_tx(full, 2 * blk + sbytes);
          bulk_g2s(st, ex.w13 + static_cast<size_t>(r0) * p.H, blk, full);
          bulk_g2s(st + blk, ex.w13 + static_cast<size_t>(u0) * p.H, blk, full);
          if (ex.sc13_bulk) {
            float* sd = reinterpret_cast<float*>(st + S.g_sc);
            const uint32_t n = ex.srows == 1 ? kGRows * nkb * 4 : nkb * 4;
            bulk_g2s(sd, ex.s13 + static_cast<size_t>(r0 / ex.srows) * nkb, n, full);
            bulk_g2s(sd + kGRows * nkb, ex.s13 + static_cast<size_t>(u0 / ex.srows) * nkb, n, full);
          }
        } else if (d.kind == ITEM_D) {
          const ExpertRef ex = expert_ref(p, d.a, tab_expert);
          const int nkb = p.I / 128;
          const int n0 = d.b * kDRows;
          const uint32_t blk = kDRows * p.I;
          const uint32_t sbytes = ex.sc2_bulk ? (ex.srows == 1 ? kDRows * nkb * 4u : nkb * 4u) : 0u;
          const uint32_t hbytes = static_cast<uint32_t>(L.amax_off + 16);
          mbar_arrive_expect_tx(full, blk + sbytes + hbytes);
          bulk_g2s(st, ex.w2 + static_cast<size_t>(n0) * p.I, blk, full);
          if (ex.sc2_bulk)
            bulk_g2s(st + S.d_sc, ex.s2 + static_cast<size_t>(n0 / ex.srows) * nkb, sbytes, full);
          // h of this slot: wait until all its G items are published, then stage it
          const uint32_t* g_done = reinterpret_cast<const uint32_t*>(p.ws + L.g_done);
          if (!wait_geq(g_done + d.a, static_cast<uint32_t>(C.g_per_slot))) {
            flag_error(p, L, STATUS_TIMEOUT);
            misc->abort = 1;
          }
          fence_proxy_async();
          bulk_g2s(st + S.d_h, p.ws + L.hblk + static_cast<size_t>(d.a) * L.hblk_stride, hbytes, full);
        } else {
          mbar_arrive(full);  // END: no data
        }
      }
      __syncwarp();
      if (++stage == kStages) {
        stage = 0;
        empty_par ^= 1u;
      }
      if (d.kind == ITEM_END && ++ends == kGroups) break;  // one END per consumer group
    }
  } else if (warp < kConsumerWarps) {
    // ================================================================ consumers (two groups)
    const int gid = warp / kGroupWarps, gw = warp % kGroupWarps;
    const int gtid = tid - gid * kGroupThreads;
    const int bar_id = 1 + gid;
    const Group G = group_scratch(smem, S, gid);
    const uint8_t* xq = smem + S.xq;
    prepare_x(p, smem + S.xq, reinterpret_cast<__nv_bfloat16*>(smem + S.xb), misc, warp, lane, S.xp);
    named_bar(kBarAll, kConsumers);
    int stage = gid;
    uint32_t full_par = 0;
    for (;;) {
      if (!mbar_wait(&misc->full[stage], full_par)) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      const Desc d = misc->desc[stage];
      if (d.kind == ITEM_END) break;
      const uint8_t* st = smem + S.stage + stage * S.stage_bytes;
      if (d.kind == ITEM_R) {
        consume_r(p, L, st, d, reinterpret_cast<const __nv_bfloat16*>(smem + S.xb), gw, lane);
      } else if (d.kind == ITEM_G) {
        consume_g(p, L, S, xq, st, d, misc, G, tab_expert, gw, lane, bar_id);
      } else if (d.kind == ITEM_D) {
        consume_d(p, L, S, st, d, G, tab_coef, tab_expert, gw, lane, gtid, bar_id);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&misc->done[stage]);
        mbar_arrive(&misc->empty[stage]);
      }
      stage += kGroups;
      if (stage >= kStages) {
        stage -= kStages;
        full_par ^= 1u;
      }
    }
  } else {
    // ================================================================ signal warp
    // Publishes finished items at gpu scope. A stage is handed back to the producer as soon as the
    // consumers are done with it; the gpu-scope fence is then paid once per batch of finished items.
    constexpr int kMaxPending = 8;
    int pend_kind[kMaxPending], pend_idx[kMaxPending];
    int npend = 0;
    int stage = 0;
    uint32_t par = 0;
    bool finished = false;
    auto take = [&](const Desc& d) {
      pend_kind[npend] = d.kind;
      pend_idx[npend] = d.kind == ITEM_D ? d.b : d.a;
      ++npend;
      if (lane == 0) mbar_arrive(&misc->empty[stage]);
      if (++stage == kStages) {
        stage = 0;
        par ^= 1u;
      }
    };
    while (!finished) {
      // blocking: the next item in ring order is finished (or the stream ended)
      if (!mbar_wait(&misc->full[stage], par)) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      Desc d = misc->desc[stage];
      if (d.kind == ITEM_END) break;
      if (!mbar_wait(&misc->done[stage], par)) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      take(d);
      // non-blocking: collect every further item that is already finished
      while (npend < kMaxPending && mbar_try_wait(&misc->full[stage], par)) {
        d = misc->desc[stage];
        if (d.kind == ITEM_END) {
          finished = true;
          break;
        }
        if (!mbar_try_wait(&misc->done[stage], par)) break;
        take(d);
      }
      // publish the batch: the consumers' stores (ordered before their mbarrier arrivals) become
      // visible at gpu scope before any counter moves
      bool do_finalize = false;
      if (lane == 0) {
        __threadfence();
        for (int i = 0; i < npend; ++i) {
          if (pend_kind[i] == ITEM_G) {
            red_release_add(reinterpret_cast<uint32_t*>(p.ws + L.g_done) + pend_idx[i], 1u);
          } else if (pend_kind[i] == ITEM_D) {
            red_release_add(reinterpret_cast<uint32_t*>(p.ws + L.d_done) + pend_idx[i], 1u);
          } else if (pend_kind[i] == ITEM_R) {
            if (atom_add_acqrel(ctl + CTRL_ROUTE_COUNT, 1u) == static_cast<uint32_t>(C.nR - 1)) do_finalize = true;
          }
        }
      }
      npend = 0;
      if (__shfl_sync(0xffffffffu, do_finalize, 0)) finalize_route(p, L, lane);
    }
  }

  // ================================================================ exit + self-clean
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t old = atom_add_acqrel(ctl + CTRL_EXIT, 1u);
    if (old == gridDim.x - 1) {
      // last CTA out: reset every counter for the next call on this workspace
      ctl[CTRL_QUEUE] = 0u;
      ctl[CTRL_ROUTE_COUNT] = 0u;
      ctl[CTRL_ROUTE_FLAG] = 0u;
      ctl[CTRL_NSLOTS] = 0u;
      uint32_t* gd = reinterpret_cast<uint32_t*>(p.ws + L.g_done);
      for (int i = 0; i < kMaxSlots; ++i) gd[i] = 0u;
      uint32_t* dd = reinterpret_cast<uint32_t*>(p.ws + L.d_done);
      for (int i = 0; i < kMaxH / kDRows; ++i) dd[i] = 0u;
      for (int s = 0; s < kMaxSlots; ++s) {
        uint32_t* am = reinterpret_cast<uint32_t*>(p.ws + L.hblk + static_cast<size_t>(s) * L.hblk_stride +
                                                   L.amax_off);
        am[0] = am[1] = am[2] = am[3] = 0u;
      }
      ctl[CTRL_EXIT] = 0u;
      __threadfence();
    }
  }
}

}  // namespace moe
}  // namespace dm3

// ------------------------------------------------------------------ host launcher
namespace dm3 {

size_t moe_ws_bytes(int T, int H, int I) { return moe::ws_layout(T, H, I).total; }

int moe_smem_bytes(int T, int H, int I) { return moe::smem_layout(T, H, I).total; }

int launch_moe(const moe::Params& p, cudaStream_t stream) {
  const moe::SmemLayout S = moe::smem_layout(p.T, p.H, p.I);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return 2;
  }
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(moe::moe_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess) {
      set_error("cudaFuncSetAttribute(moe) failed");
      return 2;
    }
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(sm_count(dev));
  cfg.blockDim = dim3(moe::kThreads);
  cfg.dynamicSmemBytes = S.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, moe::moe_decode_kernel, p);
  if (err != cudaSuccess) {
    set_error(std::string("moe launch: ") + cudaGetErrorString(err));
    return 2;
  }
  note_launches(1);
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
  if (workspace_bytes < dm3::moe_ws_bytes(kMaxT, H, I)) return set_error("workspace too small"), 4;
  return 0;
}

// Scale rows are staged by bulk copy when every address and size involved is a 16-byte multiple:
// 1x128 rows always are (8 or 64 rows of K/128 floats); 128x128 rows need K/128 % 4 == 0.
void set_bulk_flags(dm3::moe::Params& p, int64_t s13_stride, int64_t s2_stride) {
  const int nkh = p.H / 128, nki = p.I / 128;
  p.sc13_bulk = aligned16(p.s13) && (s13_stride * 4) % 16 == 0 && (p.srows == 1 || nkh % 4 == 0);
  p.sc2_bulk = aligned16(p.s2) && (s2_stride * 4) % 16 == 0 && (p.srows == 1 || nki % 4 == 0);
  p.sh_sc13_bulk = p.sh_w13 && aligned16(p.sh_s13) && (p.sh_srows == 1 || nkh % 4 == 0);
  p.sh_sc2_bulk = p.sh_w13 && aligned16(p.sh_s2) && (p.sh_srows == 1 || nki % 4 == 0);
}

}  // namespace

extern "C" size_t dm3_moe_workspace_bytes(int T, int H, int I) {
  (void)T;  // sized for kMaxT rows so one workspace serves every T of a given (H, I)
  return dm3::moe_ws_bytes(dm3::kMaxT, H, I);
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
  set_bulk_flags(p, s13_stride, s2_stride);
  return dm3::launch_moe(p, static_cast<cudaStream_t>(stream));
}

extern "C" int dm3_moe_layer(const void* x, int T, int H, int I, const void* router_w, int router_dtype,
                             int n_router, int top_k, int logits_bf16, const float* logit_bias, const void* w13,
                             int64_t w13_stride, const float* s13, int64_t s13_stride, const void* w2,
                             int64_t w2_stride, const float* s2, int64_t s2_stride, int srows, const void* sh_w13,
                             const float* sh_s13, const void* sh_w2, const float* sh_s2, int sh_srows,
                             const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out, void* w_out,
                             void* workspace, size_t workspace_bytes, void* stream) {
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
  set_bulk_flags(p, s13_stride, s2_stride);
  return dm3::launch_moe(p, static_cast<cudaStream_t>(stream));
}

extern "C" int dm3_moe_status(void* workspace, uint32_t* status, void* stream) {
  if (!workspace || !status) return dm3::set_error("null pointer argument"), 1;
  uint32_t* word = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + dm3::moe::ws_layout(1, 128, 128).ctrl) +
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

constexpr size_t kNoAllocScratchBytes = 1310720;  // 1.25 MiB: the workspace of H <= 2048, I <= 512
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
// Device address of g_noalloc_scratch per device; the host-side symbol is not a device address.
void* g_noalloc_ptr[64] = {nullptr};

}  // namespace

extern "C" int dm3_moe_layer_noalloc(const void* x, int T, int H, int I, const void* router_w, int router_dtype,
                                     int n_router, int top_k, int logits_bf16, const float* logit_bias,
                                     const void* w13, int64_t w13_stride, const float* s13, int64_t s13_stride,
                                     const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride, int srows,
                                     const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                                     int sh_srows, const void* sh_gate, const float* out_bias, void* y,
                                     int64_t* ids_out, void* w_out, void* stream) {
  dm3::note_launches(0);
  if (H > 0 && I > 0 && H <= dm3::kMaxH && I <= dm3::kMaxI &&
      dm3::moe_ws_bytes(dm3::kMaxT, H, I) > kNoAllocScratchBytes)
    return dm3::set_error("H and I need more scratch than the 1.25 MiB static array holds"), 4;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return dm3::set_error("no usable current CUDA device"), 2;
  if (g_noalloc_ptr[dev] == nullptr) {
    // first call on this device: look up the array's device address and zero it once
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess) return dm3::set_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(err)), 2;
    err = cudaMemsetAsync(ptr, 0, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return dm3::set_error(std::string("clearing the static scratch: ") + cudaGetErrorString(err)), 2;
    g_noalloc_ptr[dev] = ptr;
  }
  return dm3_moe_layer(x, T, H, I, router_w, router_dtype, n_router, top_k, logits_bf16, logit_bias, w13, w13_stride,
                       s13, s13_stride, w2, w2_stride, s2, s2_stride, srows, sh_w13, sh_s13, sh_w2, sh_s2, sh_srows,
                       sh_gate, out_bias, y, ids_out, w_out, g_noalloc_ptr[dev], kNoAllocScratchBytes, stream);
}
