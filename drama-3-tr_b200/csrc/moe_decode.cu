// Decode MoE layer for B200 (sm_100a) as four chained kernels, each launched with programmatic
// dependent launch so that a kernel's constant-weight loads start while its predecessor finishes:
//
//   route    router logits (exact fp64 dot products, rounded once), one warp per router row; the
//            last CTA to finish runs softmax / top-k / renormalise and writes the slot table
//   up       gate and up rows of every selected expert (+ the shared expert) in items of 8 + 8
//            rows over all of H; SwiGLU in registers; h written as bf16
//   down     64-row blocks of every selected expert's down projection against its h; routed
//            partials carry their routing weight
//   combine  sum over slots per output element with the reference's rounding points (+ bias,
//            + the sigmoid-gated shared expert), written as bf16
//
// Kernel boundaries are the only synchronisation between CTAs on the streaming path: a gpu-scope
// fence issued while bulk copies are in flight costs microseconds, so none is. The one fence is in
// the route kernel, whose CTAs have nothing in flight by then.
//
// The up and down kernels run one producer warp, which stages each item with cp.async.bulk into a
// 4-stage shared-memory ring, and two groups of four consumer warps that take alternate stages and
// multiply the raw e4m3 weight bytes by the exact e4m3 hi / lo split of the activations (cols 0-3
// hi of rows 0-3, cols 4-7 lo) with mma.sync m16n8k32; the per-128 block scales are applied to each
// 128-wide k-block partial in fp32.
//
// Ordering under programmatic dependent launch: every kernel calls griddepcontrol.launch_dependents
// only after its own griddepcontrol.wait, so once a kernel is running, everything two launches
// back has completed. The down kernel relies on that to read the route table before its wait.
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
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kGRows = 8;         // gate rows per up item (plus the same number of up rows)
constexpr int kDRows = 64;        // down-projection rows per down item (= output rows per partial block)
constexpr int kRouteWarps = 4;    // router rows per route CTA (one warp per row)
constexpr int kCombineThreads = 256;
constexpr int kPad = 64;          // smem row padding (bytes) of the thread-written activation tiles
constexpr int kBarAll = 3;        // named barrier of all consumer warps (groups use 1 and 2)

enum : int { ITEM_G = 2, ITEM_D = 3, ITEM_END = 5 };

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
// Control words, the route table, the router logits, the bf16 SwiGLU activations h and the fp32
// per-slot partial outputs. Offsets do not depend on the row count, so one workspace serves every
// T of a given (H, I). Only the route counter is ever non-zero between calls, and the route kernel
// resets it.
struct WsLayout {
  size_t ctrl, slot_expert, coef, logits, h, h_stride, partial, total;
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
  L.logits = o;
  o += align_up(kMaxT * (kMaxRouter + 1) * 4, 16);
  o = align_up(o, 128);
  L.h_stride = align_up(static_cast<size_t>(kMaxT) * I * 2, 128);  // per slot: h[t][I] bf16
  L.h = o;
  o += L.h_stride * kMaxSlots;
  L.partial = o;  // [H / 64][kMaxSlots][kMaxT][64] fp32: one output block's slots are adjacent
  o += static_cast<size_t>(H / kDRows) * kMaxSlots * kMaxT * kDRows * 4;
  L.total = align_up(o, 256);
  return L;
}

__device__ __forceinline__ float* partial_block(const Params& p, const WsLayout& L, int nb, int slot) {
  return reinterpret_cast<float*>(p.ws + L.partial) + (static_cast<size_t>(nb) * kMaxSlots + slot) * kMaxT * kDRows;
}

// ------------------------------------------------------------------ shared-memory layout (up / down)
struct Desc {
  int kind, a, b, c;  // a = slot; up: b = 8-row block of gate / up rows; down: b = 64-row block
};

struct SmemLayout {
  int stage_bytes, stage, xq, grp, grp_bytes, table, misc, total;
  int xp, hp;           // padded row pitches of the activation tiles (bytes)
  int g_sc, d_sc, d_h;  // offsets inside a stage: up-item scales, down-item scales, staged h
};

__host__ __device__ inline SmemLayout smem_layout(int H, int I) {
  SmemLayout S;
  S.xp = H + kPad;
  S.hp = I + kPad;
  const int nkh = H / 128, nki = I / 128;
  S.g_sc = 2 * kGRows * H;
  S.d_sc = kDRows * I;
  S.d_h = kDRows * I + kDRows * nki * 4;
  const int g_bytes = S.g_sc + 2 * kGRows * nkh * 4;
  const int d_bytes = S.d_h + static_cast<int>(align_up(kMaxT * I * 2, 16));
  S.stage_bytes = static_cast<int>(align_up(g_bytes > d_bytes ? g_bytes : d_bytes, 128));
  int o = 0;
  S.stage = o;
  o += kStages * S.stage_bytes;
  S.xq = o;
  o += 8 * S.xp;
  // per consumer group: hq (8 x hp), red (4 warps x 32 lanes x 4 floats), h row maxima (4 floats)
  S.grp_bytes = static_cast<int>(align_up(8 * S.hp + kGroupWarps * 32 * 16 + 16, 128));
  S.grp = o;
  o += kGroups * S.grp_bytes;
  S.table = o;  // slot_expert[kMaxSlots] int, coef[kMaxSlots][kMaxT] float
  o += static_cast<int>(align_up(kMaxSlots * 4 + kMaxSlots * kMaxT * 4 + 64, 128));
  S.misc = o;
  o += 512;
  S.total = o;
  return S;
}

struct Misc {
  Desc desc[kStages];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  float xinv[kMaxT];
};

struct Group {  // per-consumer-group scratch
  uint8_t* hq;
  float* red;
  float* hmax;
};

__device__ __forceinline__ Group group_scratch(uint8_t* smem, const SmemLayout& S, int gid) {
  uint8_t* b = smem + S.grp + gid * S.grp_bytes;
  Group g;
  g.hq = b;
  g.red = reinterpret_cast<float*>(b + 8 * S.hp);
  g.hmax = reinterpret_cast<float*>(b + 8 * S.hp + kGroupWarps * 32 * 16);
  return g;
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

// The slot table of this call, for one warp, into shared memory: built from the caller's ids /
// weights (routing given) or copied from the table the route kernel wrote. Returns the slot count.
__device__ int load_table(const Params& p, const WsLayout& L, int lane, int* tab_expert, float* tab_coef,
                          bool report_bad_ids) {
  if (p.mode == 0) {
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
    const float one[kMaxT] = {1.f, 1.f, 1.f, 1.f};
    return build_slots(lane, n, t, e, w, p.sh_w13 != nullptr ? 1 : 0, p.T, tab_expert, tab_coef, one);
  }
  const int n_slots = static_cast<int>(__ldcg(ctrl(p, L) + CTRL_NSLOTS));
  const int* gse = reinterpret_cast<const int*>(p.ws + L.slot_expert);
  const float* gco = reinterpret_cast<const float*>(p.ws + L.coef);
  for (int i = lane; i < kMaxSlots; i += 32) tab_expert[i] = __ldcg(gse + i);
  for (int i = lane; i < kMaxSlots * kMaxT; i += 32) tab_coef[i] = __ldcg(gco + i);
  __syncwarp();
  return n_slots;
}

// ------------------------------------------------------------------ route kernel
// Router logits in shared memory of the last route CTA: [kMaxT][kMaxRouter + 1] floats (the last
// column is the shared expert's gate), then the selected experts and weights of every row.
struct RouteSmem {
  float logits[kMaxT][kMaxRouter + 1];
  int sel_e[kMaxT * kMaxTopK];
  float sel_w[kMaxT * kMaxTopK];
  float shared_coef[kMaxT];
  int last;
};

// Top-k of row t by one warp from the logits in shared memory, and the renormalised weights.
// Mirrors Speaker.__call__ (engine.py:233-235): probs = softmax(logits), (w, ids) = probs.topk(k),
// w = (w / w.sum()).to(bf16). Selection uses the logits themselves (softmax is monotonic), ties to
// the lower index.
__device__ void route_row(const Params& p, RouteSmem& rs, int t, int lane) {
  const int E = p.n_router, K = p.top_k;
  float lv[kMaxRouter / 32];
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kMaxRouter / 32; ++i) {
    const int e = lane + 32 * i;
    lv[i] = e < E ? rs.logits[t][e] : -FLT_MAX;
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
  float psum = 0.f, my_p = 0.f;
  int my_e = -1;
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
    const float pj = expf(bv - m) / z;
    psum += pj;
    if (lane == j) {
      my_e = be;
      my_p = pj;
    }
  }
  if (lane < K) {
    const __nv_bfloat16 wb = __float2bfloat16_rn(my_p / psum);
    rs.sel_e[t * K + lane] = my_e;
    rs.sel_w[t * K + lane] = __bfloat162float(wb);
    if (p.ids_out) p.ids_out[t * K + lane] = my_e;
    if (p.w_out) p.w_out[t * K + lane] = wb;
  }
  if (lane == 0)
    rs.shared_coef[t] = p.sh_gate ? bf16_round(1.f / (1.f + expf(-rs.logits[t][E]))) : 1.f;
}

// One warp per router row (plus the shared expert's gate row). The row is fetched into registers
// before griddepcontrol.wait (router weights never depend on the preceding kernel); the activation
// rows are staged in shared memory after it, all loads in flight at once. Each logit is an exact
// fp64 dot product (bf16 x bf16 and bf16 x fp32 products are exact in fp64) rounded once to fp32
// (then to bf16 for a bf16 router), + the optional logit bias; the shared gate row is rounded to
// bf16 as a bf16 linear's output. The last CTA to finish (one gpu-scope fence per CTA, with no
// copies in flight) runs the top-k of every row in parallel and writes the slot table.
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(const Params p) {
  const WsLayout L = ws_layout(p.H, p.I);
  __shared__ __align__(16) __nv_bfloat16 xs[kMaxT * kMaxH];
  __shared__ RouteSmem rs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool sh_gate_row = p.sh_w13 != nullptr && p.sh_gate != nullptr;
  const int rows = p.n_router + (sh_gate_row ? 1 : 0);
  const int row = blockIdx.x * kRouteWarps + warp;
  const bool is_router = row < p.n_router;
  const bool row_f32 = is_router && !p.router_bf16;
  // this lane's slice of the row: bf16 elements lane*8 + 256*j, or fp32 elements lane*4 + 128*j
  constexpr int kMaxChunks = kMaxH * 4 / (32 * 16);  // 16-byte chunks per lane of an fp32 row of kMaxH
  uint4 wv[kMaxChunks];
  const int chunks = row_f32 ? p.H / 128 : p.H / 256;
  if (row < rows) {
    const uint4* src = row_f32 ? reinterpret_cast<const uint4*>(static_cast<const float*>(p.router_w) +
                                                               static_cast<size_t>(row) * p.H)
                     : is_router ? reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.router_w) +
                                                                 static_cast<size_t>(row) * p.H)
                                 : reinterpret_cast<const uint4*>(p.sh_gate);
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) wv[j] = j < chunks ? __ldg(src + lane + 32 * j) : make_uint4(0u, 0u, 0u, 0u);
  }
  griddep_wait();
  griddep_launch();
  {
    constexpr int kPerThread = kMaxT * kMaxH / 8 / (kRouteWarps * 32);
    const int n16 = p.T * p.H / 8;
    const uint4* xsrc = reinterpret_cast<const uint4*>(p.x);
    uint4 v[kPerThread];
#pragma unroll
    for (int i = 0; i < kPerThread; ++i) {
      const int c = threadIdx.x + i * kRouteWarps * 32;
      v[i] = c < n16 ? xsrc[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kPerThread; ++i) {
      const int c = threadIdx.x + i * kRouteWarps * 32;
      if (c < n16) reinterpret_cast<uint4*>(xs)[c] = v[i];
    }
  }
  __syncthreads();
  float* logits = reinterpret_cast<float*>(p.ws + L.logits);
  if (row < rows) {
    for (int t = 0; t < p.T; ++t) {
      const __nv_bfloat16* xr = xs + t * p.H;
      double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
      for (int j = 0; j < kMaxChunks; ++j) {
        if (j < chunks) {
          if (row_f32) {
            const float* w = reinterpret_cast<const float*>(&wv[j]);
            const uint2 xv = *reinterpret_cast<const uint2*>(xr + lane * 4 + 128 * j);
            const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              acc[i] = fma(static_cast<double>(__bfloat162float(xe[i])), static_cast<double>(w[i]), acc[i]);
          } else {
            const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&wv[j]);
            const uint4 xv = *reinterpret_cast<const uint4*>(xr + lane * 8 + 256 * j);
            const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              acc[i & 3] = fma(static_cast<double>(__bfloat162float(xe[i])),
                               static_cast<double>(__bfloat162float(w[i])), acc[i & 3]);
          }
        }
      }
      double sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        float v = __double2float_rn(sum);
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
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(ctrl(p, L) + CTRL_ROUTE_COUNT, 1u);
    rs.last = old == gridDim.x - 1;
    if (rs.last) __threadfence();
  }
  __syncthreads();
  if (!rs.last) return;
  // last CTA: every logit is visible; stage them, one warp per row for the top-k, then the table
  for (int i = threadIdx.x; i < p.T * (kMaxRouter + 1); i += kRouteWarps * 32) {
    const int t = i / (kMaxRouter + 1), e = i % (kMaxRouter + 1);
    rs.logits[t][e] = e < rows ? __ldcg(logits + i) : 0.f;
  }
  __syncthreads();
  if (warp < p.T) route_row(p, rs, warp, lane);
  __syncthreads();
  if (warp == 0) {
    const int K = p.top_k;
    const int n = p.T * K;
    const int my_t = lane < n ? lane / K : 0;
    const int my_e = lane < n ? rs.sel_e[lane] : -1;
    const float my_w = lane < n ? rs.sel_w[lane] : 0.f;
    int* slot_expert = reinterpret_cast<int*>(p.ws + L.slot_expert);
    float* coef = reinterpret_cast<float*>(p.ws + L.coef);
    const int n_slots = build_slots(lane, n, my_t, my_e, my_w, p.sh_w13 != nullptr, p.T, slot_expert, coef,
                                    rs.shared_coef);
    if (lane == 0) {
      ctrl(p, L)[CTRL_NSLOTS] = static_cast<uint32_t>(n_slots);
      ctrl(p, L)[CTRL_ROUTE_COUNT] = 0u;  // every CTA has counted: ready for the next call
    }
  }
}

// ------------------------------------------------------------------ up: x split
// Each of the first T consumer warps loads one activation row and writes its exact e4m3 hi / lo
// split (prescaled by a power of two) as B-operand columns.
__device__ void prepare_x(const Params& p, uint8_t* xq, Misc* misc, int warp, int lane, int xp) {
  const int H = p.H;
  if (warp < p.T) {
    const __nv_bfloat16* xr = p.x + static_cast<size_t>(warp) * H;
    float amax = 0.f;
    for (int k = lane * 8; k < H; k += 256) {
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
    uint8_t* hi = xq + warp * xp;
    uint8_t* lo = xq + (4 + warp) * xp;
    for (int k = lane * 8; k < H; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
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

// ------------------------------------------------------------------ up: one item
// 8 gate rows (tile rows 0-7) and the matching 8 up rows (tile rows 8-15) of one expert against the
// split activations: lane (g, q) ends with gate row g and up row g for rows 2q, 2q+1 (hi columns,
// after folding the lo columns in), so SwiGLU happens in registers. The group's 4 warps split the
// 128-wide k blocks and reduce through shared memory.
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
  for (int kb0 = gw; kb0 < nkb; kb0 += 2 * kGroupWarps) {
    const int kb1 = kb0 + kGroupWarps;
    const bool v1 = kb1 < nkb;
    const int kbs[2] = {kb0, v1 ? kb1 : kb0};
    float part[2][4];
    tile_kblocks<2>(part, row_lo, row_hi, bcol, true, true, bvalid, kbs, q);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (i == 1 && !v1) break;
      float sgv, suv;
      if (ex.sc13_bulk) {
        sgv = sc[sg_row * nkb + kbs[i]];
        suv = sc[(kGRows + sg_row) * nkb + kbs[i]];
      } else {
        sgv = __ldg(ex.s13 + static_cast<size_t>(gate_row / ex.srows) * nkb + kbs[i]);
        suv = __ldg(ex.s13 + static_cast<size_t>(up_row / ex.srows) * nkb + kbs[i]);
      }
      tot[0] = fmaf(part[i][0], sgv, tot[0]);
      tot[1] = fmaf(part[i][1], sgv, tot[1]);
      tot[2] = fmaf(part[i][2], suv, tot[2]);
      tot[3] = fmaf(part[i][3], suv, tot[3]);
    }
  }
  // fold lo columns (q = 2, 3) onto hi columns (q = 0, 1)
#pragma unroll
  for (int i = 0; i < 4; ++i) tot[i] += __shfl_down_sync(0xffffffffu, tot[i], 2);
  *reinterpret_cast<float4*>(G.red + (gw * 32 + lane) * 4) = make_float4(tot[0], tot[1], tot[2], tot[3]);
  named_bar(bar_id, kGroupThreads);
  if (gw == 0 && q < 2) {
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
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.ws + L.h + static_cast<size_t>(slot) * L.h_stride);
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
        h[static_cast<size_t>(t) * p.I + gate_row] = __float2bfloat16_rn(hv);
      }
    }
  }
  named_bar(bar_id, kGroupThreads);  // red is reused by the group's next item
}

// ------------------------------------------------------------------ down: one item
// 64 rows of one expert's down projection against its staged h: the group finds each row's
// absolute maximum, writes the exact e4m3 hi / lo split, then each warp owns 16 rows over all of I.
// Routed slots carry their routing weight into the partial; the shared slot stays raw (the combine
// kernel rounds and gates it).
__device__ void consume_d(const Params& p, const WsLayout& L, const SmemLayout& S, const uint8_t* stage,
                          const Desc& d, const Group& G, const float* coef_tab, const int* tab_expert, int gw,
                          int lane, int gtid, int bar_id) {
  const int I = p.I, T = p.T;
  const int nkb = I / 128;
  const int slot = d.a;
  const ExpertRef ex = expert_ref(p, slot, tab_expert);
  const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(stage + S.d_h);
  const float* sc = reinterpret_cast<const float*>(stage + S.d_sc);
  if (gw < T) {  // warp t: the absolute maximum of h row t
    float am = 0.f;
    for (int k = lane * 8; k < I; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(hv + static_cast<size_t>(gw) * I + k);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(__bfloat162float(e[i])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if (lane == 0) G.hmax[gw] = am;
  }
  named_bar(bar_id, kGroupThreads);
  for (int i = gtid; i < T * I / 2; i += kGroupThreads) {
    const int t = (2 * i) / I, k = (2 * i) % I;
    const float s = exp2i(split_exponent(G.hmax[t]));
    uint16_t hi, lo;
    split2(__bfloat162float(hv[2 * i]) * s, __bfloat162float(hv[2 * i + 1]) * s, hi, lo);
    *reinterpret_cast<uint16_t*>(G.hq + t * S.hp + k) = hi;
    *reinterpret_cast<uint16_t*>(G.hq + (4 + t) * S.hp + k) = lo;
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
  for (int kb0 = 0; kb0 < nkb; kb0 += 2) {
    const bool v1 = kb0 + 1 < nkb;
    const int kbs[2] = {kb0, v1 ? kb0 + 1 : kb0};
    float part[2][4];
    tile_kblocks<2>(part, row_lo, row_hi, bcol, true, true, bvalid, kbs, q);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (i == 1 && !v1) break;
      float s0, s1;
      if (ex.sc2_bulk) {
        s0 = sc[(ex.srows == 1 ? r_lo : 0) * nkb + kbs[i]];
        s1 = sc[(ex.srows == 1 ? r_hi : 0) * nkb + kbs[i]];
      } else {
        s0 = __ldg(ex.s2 + static_cast<size_t>(n_lo / ex.srows) * nkb + kbs[i]);
        s1 = __ldg(ex.s2 + static_cast<size_t>(n_hi / ex.srows) * nkb + kbs[i]);
      }
      tot[0] = fmaf(part[i][0], s0, tot[0]);
      tot[1] = fmaf(part[i][1], s0, tot[1]);
      tot[2] = fmaf(part[i][2], s1, tot[2]);
      tot[3] = fmaf(part[i][3], s1, tot[3]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) tot[i] += __shfl_down_sync(0xffffffffu, tot[i], 2);
  if (q < 2) {
    float* part = partial_block(p, L, d.b, slot);
    const bool shared_slot = slot == 0 && p.sh_w13 != nullptr;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int t = 2 * q + c;
      if (t < T) {
        const float k = exp2i(-split_exponent(G.hmax[t])) * (shared_slot ? 1.f : coef_tab[slot * kMaxT + t]);
        __stcg(part + t * kDRows + r_lo, tot[c] * k);
        __stcg(part + t * kDRows + r_hi, tot[2 + c] * k);
      }
    }
  }
  named_bar(bar_id, kGroupThreads);  // hq / hmax are reused by the group's next item
}

// ------------------------------------------------------------------ up / down kernels
// One body for both streaming kernels (DOWN = false: up items, true: down items). Items are
// assigned statically (CTA c takes items c, c + gridDim, ...), so CTAs never wait on each other.
template <bool DOWN>
__global__ void __launch_bounds__(kThreads, 1) expert_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const SmemLayout S = smem_layout(p.H, p.I);
  const WsLayout L = ws_layout(p.H, p.I);
  Misc* misc = reinterpret_cast<Misc*>(smem + S.misc);
  int* tab_expert = reinterpret_cast<int*>(smem + S.table);
  float* tab_coef = reinterpret_cast<float*>(smem + S.table + kMaxSlots * 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool sh = p.sh_w13 != nullptr;
  const int per_slot = DOWN ? p.H / kDRows : p.I / kGRows;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&misc->full[s], 1);             // the producer's arrive.expect_tx; the bytes complete it
      mbar_init(&misc->empty[s], kGroupWarps);  // the owning group's warps
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ================================================================ producer
    // Up: shared-expert items need no routing and are staged before griddepcontrol.wait; the table
    // (the route kernel's, or built from ids a preceding kernel wrote) is read after it.
    // Down: the route table is final before this kernel starts, so weights are staged before the
    // wait; h comes from the up kernel and is staged after it.
    bool waited = false;
    int n_slots = sh ? 1 : 0;
    bool have_table = false;
    int pend[kStages];  // stages whose h copy waits for the up kernel (down, before the wait)
    int npend = 0;
    auto get_table = [&]() {
      n_slots = load_table(p, L, lane, tab_expert, tab_coef, !DOWN);
      have_table = true;
      // with routing given, the up kernel publishes the slot count for the combine kernel (after its
      // wait, so the previous call's combine has finished reading it)
      if (!DOWN && p.mode == 0 && blockIdx.x == 0 && lane == 0) ctrl(p, L)[CTRL_NSLOTS] = static_cast<uint32_t>(n_slots);
    };
    auto wait_predecessor = [&]() {
      griddep_wait();
      griddep_launch();
      waited = true;
      if (DOWN) {
        if (lane == 0) {
          fence_proxy_async();
          for (int i = 0; i < npend; ++i)
            bulk_g2s(smem + S.stage + pend[i] * S.stage_bytes + S.d_h,
                     p.ws + L.h + static_cast<size_t>(misc->desc[pend[i]].a) * L.h_stride,
                     static_cast<uint32_t>(p.T) * p.I * 2, &misc->full[pend[i]]);
        }
        npend = 0;
        __syncwarp();
      }
    };
    if (DOWN) get_table();
    int stage = 0;
    uint32_t empty_par = 1;
    for (int idx = blockIdx.x;; idx += gridDim.x) {
      if (!DOWN && !have_table && !(sh && idx < per_slot)) {
        wait_predecessor();
        get_table();
      }
      if (idx >= n_slots * per_slot) break;
      if (DOWN && !waited && npend == kStages) wait_predecessor();  // every stage waits for its h
      const Desc d{DOWN ? ITEM_D : ITEM_G, idx / per_slot, idx % per_slot, 0};
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&misc->empty[stage], empty_par);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      uint8_t* st = smem + S.stage + stage * S.stage_bytes;
      uint64_t* full = &misc->full[stage];
      if (lane == 0) {
        misc->desc[stage] = d;
        const ExpertRef ex = expert_ref(p, d.a, tab_expert);
        if (!DOWN) {
          const int nkb = p.H / 128;
          const int r0 = d.b * kGRows, u0 = p.I + d.b * kGRows;
          const uint32_t blk = kGRows * p.H;
          const uint32_t n = ex.srows == 1 ? kGRows * nkb * 4 : nkb * 4;
          mbar_arrive_expect_tx(full, 2 * blk + (ex.sc13_bulk ? 2 * n : 0u));
          bulk_g2s(st, ex.w13 + static_cast<size_t>(r0) * p.H, blk, full);
          bulk_g2s(st + blk, ex.w13 + static_cast<size_t>(u0) * p.H, blk, full);
          if (ex.sc13_bulk) {
            float* sd = reinterpret_cast<float*>(st + S.g_sc);
            bulk_g2s(sd, ex.s13 + static_cast<size_t>(r0 / ex.srows) * nkb, n, full);
            bulk_g2s(sd + kGRows * nkb, ex.s13 + static_cast<size_t>(u0 / ex.srows) * nkb, n, full);
          }
        } else {
          const int nkb = p.I / 128;
          const int n0 = d.b * kDRows;
          const uint32_t blk = kDRows * p.I;
          const uint32_t sbytes = ex.sc2_bulk ? (ex.srows == 1 ? kDRows * nkb * 4u : nkb * 4u) : 0u;
          const uint32_t hbytes = static_cast<uint32_t>(p.T) * p.I * 2;
          mbar_arrive_expect_tx(full, blk + sbytes + hbytes);
          bulk_g2s(st, ex.w2 + static_cast<size_t>(n0) * p.I, blk, full);
          if (ex.sc2_bulk) bulk_g2s(st + S.d_sc, ex.s2 + static_cast<size_t>(n0 / ex.srows) * nkb, sbytes, full);
          if (waited) bulk_g2s(st + S.d_h, p.ws + L.h + static_cast<size_t>(d.a) * L.h_stride, hbytes, full);
        }
      }
      if (DOWN && !waited) pend[npend++] = stage;
      __syncwarp();
      if (++stage == kStages) {
        stage = 0;
        empty_par ^= 1u;
      }
    }
    if (!waited) wait_predecessor();
    // one END per consumer group, in ring order
    for (int e = 0; e < kGroups; ++e) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&misc->empty[stage], empty_par);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (lane == 0) {
        if (!ok) flag_error(p, L, STATUS_TIMEOUT);
        misc->desc[stage] = Desc{ITEM_END, 0, 0, 0};
        mbar_arrive(&misc->full[stage]);
      }
      __syncwarp();
      if (++stage == kStages) {
        stage = 0;
        empty_par ^= 1u;
      }
    }
  } else {
    // ================================================================ consumers (two groups)
    const int gid = warp / kGroupWarps, gw = warp % kGroupWarps;
    const int gtid = tid - gid * kGroupThreads;
    const int bar_id = 1 + gid;
    const Group G = group_scratch(smem, S, gid);
    const uint8_t* xq = smem + S.xq;
    griddep_wait();
    griddep_launch();
    if (!DOWN) {
      prepare_x(p, smem + S.xq, misc, warp, lane, S.xp);
      named_bar(kBarAll, kConsumers);
    }
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
      if (!DOWN)
        consume_g(p, L, S, xq, st, d, misc, G, tab_expert, gw, lane, bar_id);
      else
        consume_d(p, L, S, st, d, G, tab_coef, tab_expert, gw, lane, gtid, bar_id);
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->empty[stage]);
      stage += kGroups;
      if (stage >= kStages) {
        stage -= kStages;
        full_par ^= 1u;
      }
    }
  }
}

// ------------------------------------------------------------------ combine kernel
// y = bf16(bf16(bf16(sum of routed partials) + bias) + bf16(sigmoid gate * bf16(shared))): the
// rounding points of fp8_moe_forward's bf16 output, Speaker's bias add (engine.py:236-237) and
// speaker_forward's bf16 tensor sum (engine.py:158). One thread per output element.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const Params p) {
  const WsLayout L = ws_layout(p.H, p.I);
  const int e = blockIdx.x * kCombineThreads + threadIdx.x;
  const int t = e / p.H, n = e % p.H;
  const bool active = t < p.T;
  float bias = 0.f;
  if (active && p.out_bias) bias = __ldg(p.out_bias + n);
  griddep_wait();
  griddep_launch();
  if (!active) return;
  const bool sh = p.sh_w13 != nullptr;
  // the slot count, the shared gate and every slot's partial are requested at once: one L2 round
  // trip; slots past the count hold stale data and are masked
  const int nb = n / kDRows, r = n % kDRows;
  const float* col = partial_block(p, L, nb, 0) + t * kDRows + r;
  const uint32_t n_slots = __ldcg(ctrl(p, L) + CTRL_NSLOTS);
  const float gate = sh ? __ldcg(reinterpret_cast<const float*>(p.ws + L.coef) + t) : 0.f;
  float v[kMaxSlots];
#pragma unroll
  for (int s = 0; s < kMaxSlots; ++s) v[s] = __ldcg(col + s * kMaxT * kDRows);
  float acc = (!sh && n_slots > 0u) ? v[0] : 0.f;
#pragma unroll
  for (int s = 1; s < kMaxSlots; ++s) acc += static_cast<uint32_t>(s) < n_slots ? v[s] : 0.f;
  acc = bf16_round(acc);
  if (p.out_bias) acc = bf16_round(acc + bias);
  if (sh) acc += bf16_round(gate * bf16_round(v[0]));
  p.y[static_cast<size_t>(t) * p.H + n] = __float2bfloat16_rn(acc);
}

}  // namespace moe
}  // namespace dm3

// ------------------------------------------------------------------ host launcher
namespace dm3 {

size_t moe_ws_bytes(int H, int I) { return moe::ws_layout(H, I).total; }

namespace {

template <typename Kernel>
int launch_one(Kernel kernel, int grid, int block, size_t smem, cudaStream_t stream, const moe::Params& p,
               const char* name) {
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
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, p);
  if (err != cudaSuccess) {
    set_error(std::string(name) + " launch: " + cudaGetErrorString(err));
    return 2;
  }
  return 0;
}

}  // namespace

int launch_moe(const moe::Params& p, cudaStream_t stream) {
  const moe::SmemLayout S = moe::smem_layout(p.H, p.I);
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
    ok = ok && cudaFuncSetAttribute(moe::route_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    ok = ok && cudaFuncSetAttribute(moe::combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared) == cudaSuccess;
    if (!ok) {
      set_error("cudaFuncSetAttribute(moe) failed");
      return 2;
    }
    configured[dev] = true;
  }
  const int sms = sm_count(dev);
  int launches = 0;
  if (p.mode == 1) {
    const int rows = p.n_router + (p.sh_w13 && p.sh_gate ? 1 : 0);
    if (int rc = launch_one(moe::route_kernel, (rows + moe::kRouteWarps - 1) / moe::kRouteWarps,
                            moe::kRouteWarps * 32, 0, stream, p, "moe route"))
      return rc;
    ++launches;
  }
  if (int rc = launch_one(moe::expert_kernel<false>, sms, moe::kThreads, S.total, stream, p, "moe up")) return rc;
  if (int rc = launch_one(moe::expert_kernel<true>, sms, moe::kThreads, S.total, stream, p, "moe down")) return rc;
  if (int rc = launch_one(moe::combine_kernel, (p.T * p.H + moe::kCombineThreads - 1) / moe::kCombineThreads,
                          moe::kCombineThreads, 0, stream, p, "moe combine"))
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
      dm3::moe_ws_bytes(H, I) > kNoAllocScratchBytes)
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
