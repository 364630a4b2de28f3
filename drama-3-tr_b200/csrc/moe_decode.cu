// Decode MoE layer for B200 (sm_100a) as four chained kernels, each launched with programmatic
// dependent launch so that a kernel's constant-weight loads start while its predecessor finishes:
//
//   route    router logits (exact products, summed in a hi + lo pair and rounded once), one warp
//            per router row
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
#include <cfloat>
#include <cmath>
#include <utility>

#include "dm3_common.cuh"
#include "dm3_internal.h"
#include "dm3_tc.cuh"

namespace dm3 {
namespace moe {

constexpr int kThreads = 256;       // 8 warps
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpSplit = 2, kWarpEpi = 4;
constexpr int kSplitThreads = 64;   // warps 2-3
constexpr int kEpiThreads = 128;    // warps 4-7
constexpr int kTileRows = 128;      // weight rows per MMA tile (M)
constexpr int kUpHalf = 64;         // gate rows (and as many up rows) per up item
constexpr int kBlockRows = 128;     // output rows per down item (= rows per partial block)
constexpr int kN = 16;              // activation columns of the MMA (N)
constexpr int kSlabBytes = kTileRows * 128;   // one 128-byte K slab of a weight tile
constexpr int kStageBytes = 2 * kSlabBytes;   // two slabs per ring stage
constexpr int kBSlabBytes = kN * 128;         // one K slab of the activation tile
constexpr int kUpStages = 5, kDownStages = 6;
constexpr int kUpAcc = 2, kDownAcc = 4;       // TMEM accumulator buffers
constexpr uint32_t kUpTmemCols = 512, kDownTmemCols = 256;
constexpr int kRouteWarps = 4;      // router rows per route CTA (one warp per row)
constexpr int kCombineThreads = 256;
// named barriers (0 is __syncthreads)
constexpr int kBarSelect = 1, kBarTable = 2, kBarSplit = 3;

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
};


// ------------------------------------------------------------------ workspace layout
// Control words, the shared gate of the call, the router logits, the bf16 SwiGLU activations h and
// the fp32 per-slot partial outputs. Offsets do not depend on the row count, so one workspace
// serves every T of a given (H, I). Nothing in it carries state from one call to the next except
// the sticky status word.
struct WsLayout {
  size_t ctrl, slot_expert, coef, logits, h, h_stride, partial, total;
};
enum : int { CTRL_STATUS = 4, CTRL_NSLOTS = 5, CTRL_WORDS = 16 };

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
  L.partial = o;  // [H / 128][kMaxSlots][kMaxT][128] fp32: one output block's slots are adjacent
  o += static_cast<size_t>(H / kBlockRows) * kMaxSlots * kMaxT * kBlockRows * 4;
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
  int sel_e[kMaxT * kMaxTopK];       // selected experts of each row, in selection order
  float sel_w[kMaxT * kMaxTopK];     // their renormalised bf16 weights
  float shared_coef[kMaxT];
  int kbuf[32];
  float wbuf[32];
};

// Barriers, the table and small per-item values of the up / down kernels.
struct Aux {
  uint64_t full[8], empty[8];        // TMA ring: bytes landed / MMAs done reading
  uint64_t acc_full[4], acc_empty[4];  // TMEM accumulators: MMAs done / epilogue done reading
  uint64_t b_ready[2], b_free[2];    // activation tiles (down): split written / epilogue done
  uint64_t upv_full, upv_empty;      // up: up-row values written / read
  uint32_t tmem;
  int split_ok;
  int n_slots;
  float xinv[kMaxT];                 // up: 2^-e of each token's split
  uint32_t hmax[2][kMaxT];           // down: |h| maxima of each tile's tokens (float bits)
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
  if (slot == 0 && p.sh_w13 != nullptr) {
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
// Builds slots from (token, expert, weight) pairs held one per lane (lanes >= n invalid).
// Slot order: optional shared expert first, then distinct routed experts ascending. Returns the
// slot count. One warp; tab.kbuf / tab.wbuf are its scratch.
__device__ int build_slots(int lane, int n, int t, int e, float w, bool shared, int T, Table& tab) {
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
  const int base = shared ? 1 : 0;
  // one writer per (slot, row): a repeated pair (only possible with malformed ids) is summed in lane order
  const int key2 = valid ? ((rank << 3) | t) : -1 - lane;
  const unsigned grp = __match_any_sync(0xffffffffu, key2);
  for (int i = lane; i < kMaxSlots * kMaxT; i += 32) tab.coef[i] = 0.f;
  __syncwarp();
  if (valid && (__ffs(grp) - 1 == lane)) {
    float wsum = 0.f;
    for (unsigned g = grp; g; g &= g - 1u) wsum += tab.wbuf[__ffs(g) - 1];
    tab.expert[base + rank] = e;
    tab.coef[(base + rank) * kMaxT + t] = wsum;
  }
  if (shared && lane == 0) {
    tab.expert[0] = -1;
    for (int tt = 0; tt < T; ++tt) tab.coef[tt] = tab.shared_coef[tt];
  }
  __syncwarp();
  return base + __popc(firsts);
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
  return build_slots(lane, n, t, e, w, false, p.T, tab);
}

// Route table from the row selections route_row left in tab.sel_e / sel_w, for one warp.
__device__ int table_from_selection(const Params& p, int lane, Table& tab) {
  const int n = p.T * p.top_k;
  const int t = lane < n ? lane / p.top_k : 0;
  const int e = lane < n ? tab.sel_e[lane] : -1;
  const float w = lane < n ? tab.sel_w[lane] : 0.f;
  return build_slots(lane, n, t, e, w, p.sh_w13 != nullptr, p.T, tab);
}

// ------------------------------------------------------------------ route kernel
// Order-preserving map of a float to an unsigned key (larger float, larger key; -0 and +0 equal).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f + 0.f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Top-k of row t by one warp from the route kernel's logits, and the renormalised weights, into
// tab.sel_e / sel_w / shared_coef. Mirrors Speaker.__call__ (engine.py:233-235):
// probs = softmax(logits), (w, ids) = probs.topk(k), w = (w / w.sum()).to(bf16). Selection uses the
// logits themselves (softmax is monotonic), ties to the lower index; each step is one warp-wide
// max of the lanes' best keys and one min of the expert indices that hold it.
__device__ void route_row(const Params& p, const WsLayout& L, int t, int lane, Table& tab, bool write_out) {
  const int E = p.n_router, K = p.top_k;
  const float* lg = reinterpret_cast<const float*>(p.ws + L.logits) + t * (kMaxRouter + 1);
  float lv[kMaxRouter / 32];
  uint32_t key[kMaxRouter / 32];
#pragma unroll
  for (int i = 0; i < kMaxRouter / 32; ++i) lv[i] = lane + 32 * i < E ? __ldcg(lg + lane + 32 * i) : -FLT_MAX;
  const float gl = (lane == 0 && p.sh_gate) ? __ldcg(lg + E) : 0.f;
  uint32_t kmax = 0u;
#pragma unroll
  for (int i = 0; i < kMaxRouter / 32; ++i) {
    key[i] = lane + 32 * i < E ? order_key(lv[i]) : 0u;
    kmax = max(kmax, key[i]);
  }
  const float m = key_value(__reduce_max_sync(0xffffffffu, kmax));
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxRouter / 32; ++i)
    if (lane + 32 * i < E) z += expf(lv[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  unsigned taken = 0u;
  int my_e = -1;
  float my_v = 0.f;
  for (int j = 0; j < K; ++j) {
    uint32_t bk = 0u;
    int bi = 0;
#pragma unroll
    for (int i = 0; i < kMaxRouter / 32; ++i)
      if (!((taken >> i) & 1u) && key[i] > bk) {
        bk = key[i];
        bi = i;
      }
    const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
    const uint32_t cand = (bk == mk && bk != 0u) ? static_cast<uint32_t>(lane + 32 * bi) : 0xffffffffu;
    const uint32_t be = __reduce_min_sync(0xffffffffu, cand);
    if (static_cast<int>(be & 31u) == lane) taken |= 1u << (be >> 5);
    if (lane == j) {
      my_e = static_cast<int>(be);
      my_v = key_value(mk);
    }
  }
  const float my_p = lane < K ? expf(my_v - m) / z : 0.f;
  float psum = 0.f;
  for (int j = 0; j < K; ++j) psum += __shfl_sync(0xffffffffu, my_p, j);
  if (lane < K) {
    const __nv_bfloat16 wb = __float2bfloat16_rn(my_p / psum);
    tab.sel_e[t * K + lane] = my_e;
    tab.sel_w[t * K + lane] = __bfloat162float(wb);
    if (write_out && p.ids_out) p.ids_out[t * K + lane] = my_e;
    if (write_out && p.w_out) p.w_out[t * K + lane] = wb;
  }
  if (lane == 0) tab.shared_coef[t] = p.sh_gate ? bf16_round(1.f / (1.f + expf(-gl))) : 1.f;
}

// Adds a to the unevaluated sum hi + lo without rounding error in hi (Knuth's TwoSum; the error
// term goes to lo).
__device__ __forceinline__ void two_sum_acc(float& hi, float& lo, float a) {
  const float s = hi + a;
  const float bb = s - hi;
  lo += (hi - (s - bb)) + (a - bb);
  hi = s;
}

// Router logits: one warp per router row (plus the shared expert's gate row). The row is fetched
// into registers before griddepcontrol.wait (router weights never depend on the preceding kernel);
// the activation rows are staged in shared memory after it, all loads in flight at once. Every
// product is exact in fp32 (bf16 x bf16; bf16 x fp32 keeps its rounding error through an fma) and
// is summed as a hi + lo pair, which carries about 48 significant bits, so the logit is the sum
// rounded once to fp32 (then to bf16 for a bf16 router), + the optional logit bias. The shared gate
// row is rounded to bf16 as a bf16 linear's output. The top-k runs in the kernels that use it.
__global__ void __launch_bounds__(kRouteWarps * 32) route_kernel(const Params p) {
  const WsLayout L = ws_layout(p.H, p.I);
  __shared__ __align__(16) __nv_bfloat16 xs[kMaxT * kMaxH];
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
  if (row >= rows) return;
  float* logits = reinterpret_cast<float*>(p.ws + L.logits);
  for (int t = 0; t < p.T; ++t) {
    const __nv_bfloat16* xr = xs + t * p.H;
    float hi[4] = {0.f, 0.f, 0.f, 0.f}, lo[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kMaxChunks; ++j) {
      if (j < chunks) {
        if (row_f32) {
          const float* w = reinterpret_cast<const float*>(&wv[j]);
          const uint2 xv = *reinterpret_cast<const uint2*>(xr + lane * 4 + 128 * j);
          const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float xf = __bfloat162float(xe[i]);
            const float pr = xf * w[i];
            lo[i] += fmaf(xf, w[i], -pr);  // the product's rounding error, exact
            two_sum_acc(hi[i], lo[i], pr);
          }
        } else {
          const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&wv[j]);
          const uint4 xv = *reinterpret_cast<const uint4*>(xr + lane * 8 + 256 * j);
          const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            two_sum_acc(hi[i & 3], lo[i & 3], __bfloat162float(xe[i]) * __bfloat162float(w[i]));
        }
      }
    }
    float h = hi[0], l = lo[0];
#pragma unroll
    for (int i = 1; i < 4; ++i) {
      l += lo[i];
      two_sum_acc(h, l, hi[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oh = __shfl_xor_sync(0xffffffffu, h, o);
      l += __shfl_xor_sync(0xffffffffu, l, o);
      two_sum_acc(h, l, oh);
    }
    if (lane == 0) {
      float v = h + l;
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

// ------------------------------------------------------------------ activation split
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

// Up: the activation tile of all H. Row t holds the e4m3 hi part of x[t] * 2^e_t (e_t maps the
// row's absolute maximum into [128, 256)), row 4 + t the lo remainder, every other row zero.
// Run by the 64 split threads; they fence their writes for the tensor core.
__device__ void split_x(const Params& p, uint8_t* bt, Aux& aux, int ptid) {
  const int H = p.H, wl = ptid >> 5, lane = ptid & 31;
  for (int t = wl; t < p.T; t += 2) {
    const __nv_bfloat16* xr = p.x + static_cast<size_t>(t) * H;
    float amax = 0.f;
    for (int k = lane * 8; k < H; k += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(__bfloat162float(e[i])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) {
      aux.hmax[0][t] = __float_as_uint(amax);
      aux.xinv[t] = exp2i(-split_exponent(amax));
    }
  }
  named_bar(kBarSplit, kSplitThreads);
  const int chunks = H / 16;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int task = ptid; task < kMaxT * chunks; task += kSplitThreads) {
    const int t = task / chunks, c = task % chunks;
    uint4 hi = z, lo = z;
    if (t < p.T) {
      const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * H + c * 16);
      const uint4 v[2] = {src[0], src[1]};
      split16(v, exp2i(split_exponent(__uint_as_float(aux.hmax[0][t]))), hi, lo);
    }
    *reinterpret_cast<uint4*>(bt + tc::swz_offset(t, c * 16, kN)) = hi;
    *reinterpret_cast<uint4*>(bt + tc::swz_offset(4 + t, c * 16, kN)) = lo;
  }
  for (int i = ptid; i < (H / 128) * 64; i += kSplitThreads)  // rows 8-15 of every slab
    *reinterpret_cast<uint4*>(bt + (i / 64) * kBSlabBytes + 1024 + (i % 64) * 16) = z;
  tc::fence_proxy_async_smem();
}

// Down: the activation tile of one slot's h (rows t < T; the zero rows are written once per
// kernel). hmax receives each row's absolute maximum for the epilogue.
__device__ void split_h(const Params& p, const WsLayout& L, uint8_t* bt, uint32_t* hmax, int slot, int ptid) {
  const int I = p.I, chunks = I / 16, n = p.T * chunks;
  constexpr int kMaxTasks = kMaxT * kMaxI / 16 / kSplitThreads;
  if (ptid < kMaxT) hmax[ptid] = 0u;
  named_bar(kBarSplit, kSplitThreads);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(p.ws + L.h + static_cast<size_t>(slot) * L.h_stride);
  uint4 v[kMaxTasks][2];
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = ptid + q * kSplitThreads;
    if (task < n) {
      const uint4* src = reinterpret_cast<const uint4*>(h + (task / chunks) * I + (task % chunks) * 16);
      v[q][0] = __ldcg(src);
      v[q][1] = __ldcg(src + 1);
      atomicMax(&hmax[task / chunks], __float_as_uint(abs_max16(v[q])));
    }
  }
  named_bar(kBarSplit, kSplitThreads);
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = ptid + q * kSplitThreads;
    if (task < n) {
      const int t = task / chunks, c = task % chunks;
      uint4 hi, lo;
      split16(v[q], exp2i(split_exponent(__uint_as_float(hmax[t]))), hi, lo);
      *reinterpret_cast<uint4*>(bt + tc::swz_offset(t, c * 16, kN)) = hi;
      *reinterpret_cast<uint4*>(bt + tc::swz_offset(4 + t, c * 16, kN)) = lo;
    }
  }
  tc::fence_proxy_async_smem();
}

// ------------------------------------------------------------------ epilogues
// Sum over k blocks of scale x (hi + lo) for this thread's weight row, from nkb accumulators of
// 16 TMEM columns each starting at column `col`.
template <int MaxKb>
__device__ __forceinline__ void reduce_kblocks(uint32_t taddr, int nkb, const float* sc, float (&acc)[kMaxT]) {
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) acc[t] = 0.f;
#pragma unroll
  for (int kb0 = 0; kb0 < MaxKb; kb0 += 8) {
    if (kb0 < nkb) {
      float v[8][8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (kb0 + j < nkb) tc::tmem_ld8(taddr + (kb0 + j) * 16, v[j]);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (kb0 + j < nkb)
#pragma unroll
          for (int t = 0; t < kMaxT; ++t) acc[t] = fmaf(sc[kb0 + j], v[j][t] + v[j][4 + t], acc[t]);
    }
  }
}

// Up: thread r holds gate row 64*blk + r (r < 64) or up row I + 64*blk + r - 64; the up values go
// through shared memory to the gate threads, which apply SwiGLU and store h. Releases the
// accumulator buffer (acc_empty) as soon as it has been read.
__device__ void epilogue_up(const Params& p, const WsLayout& L, Aux& aux, uint32_t taddr, uint64_t* acc_empty,
                            int slot, int blk, int e, int lane, int k) {
  const int r = 32 * e + lane;
  const int nkb = p.H / 128;
  const ExpertRef ex = expert_ref(p, slot, aux.tab.expert);
  const int wrow = r < kUpHalf ? kUpHalf * blk + r : p.I + kUpHalf * blk + (r - kUpHalf);
  const float* srow = ex.s13 + static_cast<size_t>(wrow / ex.srows) * nkb;
  float sc[kMaxH / 128];
#pragma unroll
  for (int kb = 0; kb < kMaxH / 128; ++kb) sc[kb] = kb < nkb ? __ldg(srow + kb) : 0.f;
  float acc[kMaxT];
  reduce_kblocks<kMaxH / 128>(taddr, nkb, sc, acc);
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(acc_empty);
  // hand-off of the up values through shared memory, guarded by two mbarriers (bounded waits)
  const uint32_t par = static_cast<uint32_t>(k & 1);
  if (r >= kUpHalf) {
    bool ok = true;
    if (lane == 0) ok = mbar_wait(&aux.upv_empty, par ^ 1u);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok && lane == 0) flag_error(p, L, STATUS_TIMEOUT);
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) aux.upv[r - kUpHalf][t] = acc[t] * aux.xinv[t];
    __syncwarp();
    if (lane == 0) mbar_arrive(&aux.upv_full);
    return;
  }
  bool ok = true;
  if (lane == 0) ok = mbar_wait(&aux.upv_full, par);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) {
    if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
    return;
  }
  {
    const bool shared_slot = slot == 0 && p.sh_w13 != nullptr;
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.ws + L.h + static_cast<size_t>(slot) * L.h_stride);
    for (int t = 0; t < p.T; ++t) {
      float gt = acc[t] * aux.xinv[t];
      float ut = aux.upv[r][t];
      float hv;
      if (shared_slot) {
        // the shared expert is a chain of bf16 modules: down(silu(gate(x)) * up(x))
        gt = bf16_round(gt);
        ut = bf16_round(ut);
        hv = bf16_round(gt / (1.f + expf(-gt))) * ut;
      } else {
        hv = gt / (1.f + expf(-gt)) * ut;
      }
      h[static_cast<size_t>(t) * p.I + kUpHalf * blk + r] = __float2bfloat16_rn(hv);
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&aux.upv_empty);  // upv may be rewritten for the next item
}

// Down: thread r holds output row 128*nb + r of one slot; the partial is weighted by the routing
// weight (the shared slot stays raw: the combine kernel rounds and gates it). Releases the
// accumulator buffer and the activation tile once both have been read.
__device__ void epilogue_down(const Params& p, const WsLayout& L, Aux& aux, uint32_t taddr, uint64_t* acc_empty,
                              uint64_t* b_free, const uint32_t* hmax, int slot, int nb, int e, int lane) {
  const int r = 32 * e + lane, n = kBlockRows * nb + r;
  const int nkb = p.I / 128;
  const ExpertRef ex = expert_ref(p, slot, aux.tab.expert);
  const float* srow = ex.s2 + static_cast<size_t>(n / ex.srows) * nkb;
  float sc[kMaxI / 128];
#pragma unroll
  for (int kb = 0; kb < kMaxI / 128; ++kb) sc[kb] = kb < nkb ? __ldg(srow + kb) : 0.f;
  float acc[kMaxT];
  reduce_kblocks<kMaxI / 128>(taddr, nkb, sc, acc);
  tc::fence_before_sync();
  float k[kMaxT];
  const bool shared_slot = slot == 0 && p.sh_w13 != nullptr;
#pragma unroll
  for (int t = 0; t < kMaxT; ++t)
    k[t] = exp2i(-split_exponent(__uint_as_float(hmax[t]))) * (shared_slot ? 1.f : aux.tab.coef[slot * kMaxT + t]);
  __syncwarp();
  if (lane == 0) {
    mbar_arrive(acc_empty);
    mbar_arrive(b_free);
  }
  float* part = partial_block(p, L, nb, slot);
  for (int t = 0; t < p.T; ++t) __stcg(part + t * kBlockRows + r, acc[t] * k[t]);
}

// ------------------------------------------------------------------ up / down kernels
// One body for both streaming kernels (DOWN = false: up items, true: down items). Items are
// assigned statically (CTA c takes items c, c + gridDim, ...), so CTAs never wait on each other.
// map_w covers the routed experts ([E][rows][K] bytes), map_sh the shared expert.
//
// Route table: with the router in the layer, epilogue warps 4 .. 4+T-1 select one row's experts
// each (up: after the wait, since the route kernel is the predecessor; down: before it, since the
// route kernel has completed by the time the down kernel starts) and warp 4 builds the table; with
// routing given, warp 4 builds it from the caller's ids.
template <bool DOWN>
__global__ void __launch_bounds__(kThreads, 1)
    expert_kernel(const Params p, const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_sh) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const SmemLayout S = smem_layout(DOWN, p.H, p.I);
  const WsLayout L = ws_layout(p.H, p.I);
  Aux& aux = *reinterpret_cast<Aux*>(smem + S.aux);
  Table& tab = aux.tab;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool sh = p.sh_w13 != nullptr;
  const int per_slot = DOWN ? p.H / kBlockRows : p.I / kUpHalf;
  const int nkb = (DOWN ? p.I : p.H) / 128;  // 128-wide k blocks (slabs) per item
  const int nchunks = (nkb + 1) / 2;         // ring stages per item
  const int nacc = DOWN ? kDownAcc : kUpAcc;
  const uint32_t acc_cols = DOWN ? kDownTmemCols / kDownAcc : kUpTmemCols / kUpAcc;
  const uint32_t tmem_cols = DOWN ? kDownTmemCols : kUpTmemCols;

  if (tid == 0) {
    for (int s = 0; s < S.nstages; ++s) {
      mbar_init(&aux.full[s], 1);   // the producer's arrive.expect_tx; the TMA bytes complete it
      mbar_init(&aux.empty[s], 1);  // tcgen05.commit after the stage's MMAs
    }
    for (int a = 0; a < nacc; ++a) {
      mbar_init(&aux.acc_full[a], 1);           // tcgen05.commit after the item's last MMA
      mbar_init(&aux.acc_empty[a], kEpiThreads / 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&aux.b_ready[b], kSplitThreads);
      mbar_init(&aux.b_free[b], kEpiThreads / 32);
    }
    mbar_init(&aux.upv_full, 2);   // the two up-row warps
    mbar_init(&aux.upv_empty, 2);  // the two gate-row warps
    fence_mbar_init();
  }
  if (warp == kWarpMma) tc::tmem_alloc(&aux.tmem, tmem_cols);
  if (DOWN && warp >= kWarpSplit && warp < kWarpEpi) {
    // the rows of the activation tiles that no item writes stay zero
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid - kWarpSplit * 32; i < 2 * S.b_bytes / 16; i += kSplitThreads)
      reinterpret_cast<uint4*>(smem + S.b)[i] = z;
    tc::fence_proxy_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = aux.tmem;

  if (warp == kWarpTma) {
    // ================================================================ TMA producer
    int stage = 0;
    uint32_t empty_par = 1;
    bool ok = true;
    auto issue = [&](int idx, int c) -> bool {
      bool ready = true;
      if (lane == 0) ready = mbar_wait(&aux.empty[stage], empty_par);
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        return false;
      }
      if (lane == 0) {
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
      }
      __syncwarp();
      if (++stage == S.nstages) {
        stage = 0;
        empty_par ^= 1u;
      }
      return true;
    };
    if (lane == 0) {
      tc::prefetch_map(&map_w);
      if (sh) tc::prefetch_map(&map_sh);
    }
    int k = 0, c = 0;  // item ordinal and chunk of the next stage
    if (!DOWN && sh) {
      // shared-expert stages need no routing: up to one ring of them before the table exists
      for (int n = 0; ok && n < S.nstages; ++n) {
        const int idx = blockIdx.x + k * gridDim.x;
        if (idx >= per_slot) break;
        ok = issue(idx, c);
        if (++c == nchunks) {
          c = 0;
          ++k;
        }
      }
    }
    named_bar(kBarSelect, kThreads);
    named_bar(kBarTable, kThreads);
    const int n_items = aux.n_slots * per_slot;
    while (ok) {
      const int idx = blockIdx.x + k * gridDim.x;
      if (idx >= n_items) break;
      ok = issue(idx, c);
      if (++c == nchunks) {
        c = 0;
        ++k;
      }
    }
  } else if (warp == kWarpMma) {
    // ================================================================ MMA issuer
    named_bar(kBarSelect, kThreads);
    named_bar(kBarTable, kThreads);
    tc::fence_after_sync();
    const int n_items = aux.n_slots * per_slot;
    const uint32_t idesc = tc::idesc_e4m3(kTileRows, kN);
    int stage = 0;
    uint32_t full_par = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int idx = blockIdx.x + k * gridDim.x;
      if (idx >= n_items) break;
      const int ab = k % nacc, bb = k & 1;
      bool ready = true;
      if (lane == 0) {
        ready = mbar_wait(&aux.acc_empty[ab], ((k / nacc) & 1) ^ 1u);
        if (ready && DOWN) ready = mbar_wait(&aux.b_ready[bb], (k >> 1) & 1);
      }
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      const uint32_t bt = smem_u32(smem + S.b + (DOWN ? bb * S.b_bytes : 0));
      const uint32_t d = tmem + ab * acc_cols;
      for (int c = 0; c < nchunks; ++c) {
        if (lane == 0) ready = mbar_wait(&aux.full[stage], full_par);
        ready = __shfl_sync(0xffffffffu, ready, 0);
        if (!ready) {
          if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
          ok = false;
          break;
        }
        tc::fence_after_sync();
        if (lane == 0) {
          const uint32_t a = smem_u32(smem + S.stage + stage * kStageBytes);
          for (int j = 0; j < 2 && 2 * c + j < nkb; ++j) {
            const int kb = 2 * c + j;
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              tc::mma_f8(d + kb * 16, tc::smem_desc(a + j * kSlabBytes + 32 * k4),
                         tc::smem_desc(bt + kb * kBSlabBytes + 32 * k4), idesc, k4 > 0);
          }
          tc::mma_commit(&aux.empty[stage]);  // the stage is free once these MMAs have read it
        }
        __syncwarp();
        if (++stage == S.nstages) {
          stage = 0;
          full_par ^= 1u;
        }
      }
      if (ok && lane == 0) tc::mma_commit(&aux.acc_full[ab]);
      __syncwarp();
    }
  } else if (warp < kWarpEpi) {
    // ================================================================ activation split
    const int ptid = tid - kWarpSplit * 32;
    if (!DOWN) {
      griddep_wait();
      griddep_launch();
      split_x(p, smem + S.b, aux, ptid);
      named_bar(kBarSelect, kThreads);
      named_bar(kBarTable, kThreads);
    } else {
      named_bar(kBarSelect, kThreads);
      named_bar(kBarTable, kThreads);
      griddep_wait();  // h comes from the up kernel
      griddep_launch();
      const int n_items = aux.n_slots * per_slot;
      for (int k = 0;; ++k) {
        const int idx = blockIdx.x + k * gridDim.x;
        if (idx >= n_items) break;
        const int bb = k & 1;
        // one thread waits; the outcome reaches both warps through shared memory and a barrier
        if (ptid == 0) {
          aux.split_ok = mbar_wait(&aux.b_free[bb], ((k >> 1) & 1) ^ 1u) ? 1 : 0;
          if (!aux.split_ok) flag_error(p, L, STATUS_TIMEOUT);
        }
        named_bar(kBarSplit, kSplitThreads);
        if (!aux.split_ok) break;
        split_h(p, L, smem + S.b + bb * S.b_bytes, aux.hmax[bb], idx / per_slot, ptid);
        mbar_arrive(&aux.b_ready[bb]);
      }
    }
  } else {
    // ================================================================ epilogue (+ route table)
    const int e = warp - kWarpEpi;  // TMEM lane quarter (warp % 4)
    if (!DOWN) {
      griddep_wait();
      griddep_launch();
    }
    if (p.mode == 1 && e < p.T) route_row(p, L, e, lane, tab, !DOWN && blockIdx.x == 0);
    named_bar(kBarSelect, kThreads);
    if (warp == kWarpEpi) {
      const int n = p.mode == 1 ? table_from_selection(p, lane, tab) : table_from_ids(p, L, lane, tab, !DOWN);
      if (lane == 0) aux.n_slots = n;
    }
    named_bar(kBarTable, kThreads);
    if (DOWN) {
      griddep_wait();
      griddep_launch();
      if (blockIdx.x == 0 && warp == kWarpEpi) {
        // the combine kernel reads the slot count and the shared gate of this call from the workspace
        if (lane == 0) ctrl(p, L)[CTRL_NSLOTS] = static_cast<uint32_t>(aux.n_slots);
        if (lane < p.T) reinterpret_cast<float*>(p.ws + L.coef)[lane] = tab.coef[lane];
      }
    }
    const int n_items = aux.n_slots * per_slot;
    for (int k = 0;; ++k) {
      const int idx = blockIdx.x + k * gridDim.x;
      if (idx >= n_items) break;
      const int ab = k % nacc, bb = k & 1;
      bool ready = true;
      if (lane == 0) {
        ready = mbar_wait(&aux.acc_full[ab], (k / nacc) & 1);
        if (ready && DOWN) ready = mbar_wait(&aux.b_ready[bb], (k >> 1) & 1);
      }
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) {
        if (lane == 0) flag_error(p, L, STATUS_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * e) << 16) + ab * acc_cols;
      if (!DOWN)
        epilogue_up(p, L, aux, taddr, &aux.acc_empty[ab], idx / per_slot, idx % per_slot, e, lane, k);
      else
        epilogue_down(p, L, aux, taddr, &aux.acc_empty[ab], &aux.b_free[bb], aux.hmax[bb], idx / per_slot,
                      idx % per_slot, e, lane);
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
  const int nb = n / kBlockRows, r = n % kBlockRows;
  const float* col = partial_block(p, L, nb, 0) + t * kBlockRows + r;
  const uint32_t n_slots = __ldcg(ctrl(p, L) + CTRL_NSLOTS);
  const float gate = sh ? __ldcg(reinterpret_cast<const float*>(p.ws + L.coef) + t) : 0.f;
  float v[kMaxSlots];
#pragma unroll
  for (int s = 0; s < kMaxSlots; ++s) v[s] = __ldcg(col + s * kMaxT * kBlockRows);
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
  if (p.mode == 1) {
    const int rows = p.n_router + (p.sh_w13 && p.sh_gate ? 1 : 0);
    if (int rc = launch_one(moe::route_kernel, (rows + moe::kRouteWarps - 1) / moe::kRouteWarps,
                            moe::kRouteWarps * 32, 0, stream, "moe route", p))
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
