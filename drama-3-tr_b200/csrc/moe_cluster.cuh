// Expert phase of the decode MoE layer as ONE kernel of thread-block clusters (included by
// moe_decode.cu inside namespace dm3::moe; it uses that file's Params, workspace layout, route
// helpers and epilogue helpers).
//
// After the route kernel (logits + x split), a cluster of kCl = 2 CTAs serves one quarter of one
// slot: 128 of the I columns of h (slot 0 is the shared expert, then the distinct routed experts
// ascending). With one CTA per SM a B200 co-schedules 74 clusters of 2 (but only 15 of 8), so the
// 17 slots x 4 quarters of a 2-row frame run as one wave on 136 SMs. CTA q of the cluster:
//
//   up    gate rows [c0 + 64q, c0 + 64q + 64) and the matching up rows over all of H (c0 = 128 x
//         the quarter; one M = 128 tile, 16 k blocks); SwiGLU in the epilogue, h rounded to bf16;
//   swap  its 64 columns of h, split exactly into e4m3 hi / lo with one power-of-two exponent, are
//         stored into both CTAs of the cluster with st.async (distributed shared memory) and
//         counted on each receiver's mbarrier: no global memory, no gpu-scope fence;
//   down  output rows [qH/2, qH/2 + H/2) against the quarter's 128 columns of h (split-K over the
//         quarters). These weights do not depend on h, so they stream through the same ring right
//         behind the up slabs and are already in shared memory when h arrives;
//   sum   every output element's contribution is added as a 64-bit fixed-point integer (units
//         of 2^-u per row, u from the row's magnitude) into the workspace with a reduction in L2:
//         integer addition is exact and
//         associative, so the sum does not depend on arrival order (deterministic). For each half
//         of the output rows, the CTA that counts last converts its sums to y with the reference's
//         rounding points and clears them.
//
// Warps 2-3 split x into the up MMAs' B operand themselves while warps 4-7 select the experts.
//
// Every CTA selects the experts itself from the route kernel's logits (one warp per row, the same
// code as the route kernel's tail), so no single-CTA step sits between the router and the first
// weight bytes. The shared-expert clusters issue their first weight stages before
// griddepcontrol.wait.
//
// TMEM (512 columns): the up accumulators in [0, 256) (one 16-column accumulator per 128-wide k
// block), the down blocks in [256, 512): 32 columns per 128-row block, one accumulator per source
// CTA's 64 columns of h (each has its own exponent).

constexpr int kCl = 2;                  // CTAs per cluster
constexpr int kFStages = 5;             // weight ring stages of 32 KB
constexpr int kFMaxTiles = kMaxH / 2 / kBlockRows;  // down blocks per CTA (H / 256)
constexpr uint32_t kFTmemCols = 512;
constexpr int kBarGate = 4;             // named barrier of the 64 gate-row threads (warps 4-5)
constexpr int kHxRows = 8;              // B rows of h sent: hi of rows 0-3, lo of rows 0-3
constexpr uint32_t kHxBytesPerSrc = kHxRows * kUpHalf + 16;  // h bytes + the exponent vector
// Fixed-point unit of row t: 2^-u_t with u_t = 22 + 2 e_t, e_t the row's split exponent (x * 2^e_t
// has its maximum in [128, 256)). A layer's output scales as |x|^2 (h = silu(gate x) * up x), so the
// sums keep about 30 significant bits whatever the rows' magnitude: u = 34 for RMS-normalised rows
// (maximum ~3.5), larger for tiny rows, smaller for rows with large outliers.
__device__ __forceinline__ int fix_exponent(float xmax) {
  const int u = 22 + 2 * split_exponent(xmax);
  return u < -60 ? -60 : (u > 100 ? 100 : u);
}
constexpr int kTableThreads = kThreads - 64;                  // the table barrier: all warps but 2-3

// Barriers and small state of the cluster kernel.
struct FAux {
  uint64_t full[kFStages], empty[kFStages];
  uint64_t xb_ready;                  // x image copied in
  uint64_t acc_full, acc_empty;       // up accumulator: MMAs done / epilogue read it
  uint64_t hx_full;                   // both CTAs' h bytes and exponents arrived (st.async tx)
  uint64_t dacc_full[kFMaxTiles];     // down blocks: MMAs done
  uint32_t tmem;
  int epi_ok[4];
  int n_slots;
  float xinv[kMaxT];
  float fixu[kMaxT];                  // 2^u_t: fixed-point units per 1.0 of row t
  float upv[kUpHalf][kMaxT];
  uint32_t hmax[2][kMaxT];            // |h| maxima of the two gate warps
  uint32_t xmax[kMaxT];               // |x| maxima (float bits) of the x split
  alignas(16) float hexp[kCl][kMaxT];             // 2^-e of each source CTA's columns of h, per row
  alignas(16) uint8_t hstage[kHxRows][kUpHalf];   // this CTA's h bytes before they are sent
  Table tab;
  RouteTail rt;
  // the fast selection (T <= 2): each row's candidates as (logit order, ~expert) keys in ascending
  // expert order, their count (kMaxCand + 1 = too many), the row's logit maximum and softmax sum
  uint64_t ckey[2][32];
  int ncand[2];
  float rmax[2], rz[2];
  int sel_e[2][kMaxTopK];
  float sel_v[2][kMaxTopK];
};

// Shared memory of the cluster kernel from a 1024-byte aligned base: the ring, the x image (16 rows
// x H, the up MMAs' B operand), the h image (16 rows x 128, the down MMAs' B operand), FAux.
struct FSmem {
  int stage, xb, xb_bytes, hb, aux, total;
};

__host__ __device__ inline FSmem fsmem_layout(int H, int I) {
  FSmem S;
  (void)I;
  S.stage = 0;
  S.xb = kFStages * kStageBytes;
  S.xb_bytes = H / 128 * kBSlabBytes;
  S.hb = S.xb + S.xb_bytes;
  S.aux = S.hb + kBSlabBytes;
  S.total = S.aux + static_cast<int>(align_up(sizeof(FAux), 128)) + 1024;  // + alignment slack
  return S;
}

// The cluster kernel handles I = 128 x quarters and H a multiple of 512 (each CTA's half of the
// output rows is a whole number of 32 KB ring stages).
__host__ __device__ inline bool cluster_shape_ok(int H, int I) {
  return I % 128 == 0 && I <= kMaxI && H % 512 == 0 && H <= kMaxH;
}

// ---------------------------------------------------------------- cluster PTX
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// All threads of all CTAs of the cluster; release / acquire at cluster scope.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// 16-byte store into another CTA's shared memory, counted as 16 transaction bytes on its mbarrier.
__device__ __forceinline__ void st_async16(uint32_t raddr, uint4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   raddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
               : "memory");
}
// Bounded wait on a local mbarrier whose phase other CTAs of the cluster complete.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (globaltimer() - t0 > wait_limit_ns()) return false;
  }
  return true;
}

// The slot table of the call in shared memory from the selections of route_row (one warp), as
// write_table lays it out: slot 0 is the shared expert when present, then the distinct selected
// experts ascending. Returns the slot count.
__device__ int table_smem(const Params& p, RouteTail& rt, int lane, Table& tab) {
  const int n = p.T * p.top_k;
  const bool valid = lane < n;
  const int e = valid ? rt.sel_e[lane] : 0;
  const int t = valid ? lane / p.top_k : 0;
  if (lane < kMaxRouter / 32) rt.bitmap[lane] = 0u;
  __syncwarp();
  if (valid) atomicOr(&rt.bitmap[e >> 5], 1u << (e & 31));
  __syncwarp();
  int srank = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kMaxRouter / 32; ++w) {
    const uint32_t word = rt.bitmap[w];
    total += __popc(word);
    if (w < (e >> 5)) srank += __popc(word);
  }
  srank += __popc(rt.bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
  const int base = p.sh_slot ? 1 : 0;
  for (int i = lane; i < kMaxSlots * kMaxT; i += 32) tab.coef[i] = 0.f;
  __syncwarp();
  if (valid) {
    tab.expert[base + srank] = e;  // rows that chose the same expert write the same value
    tab.coef[(base + srank) * kMaxT + t] = rt.sel_w[lane];
  }
  if (base && lane < p.T) tab.coef[lane] = rt.shared_coef[lane];
  if (base && lane == 0) tab.expert[0] = -1;
  __syncwarp();
  return base + total;
}

// Makes the loaded values of v live here, so that their loads are complete before a long wait
// rather than being sunk past it by the compiler.
template <int N>
__device__ __forceinline__ void hold(const float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" ::"f"(v[i]));
}

// Row t's candidates, found by an otherwise idle warp while another takes the row's softmax sum:
// every expert whose logit is at least theta, the top_k-th largest of the 32 lane maxima (each lane
// holds 8 logits). The top_k-th largest logit is at least theta, so the set holds every expert the
// row can select (usually a few more). Their (logit order, ~expert) keys go to shared memory in
// ascending expert order, with their count. (Asking L2 for the candidates' weights from here was
// measured and dropped: the bulk prefetches queue in the SM's copy engine ahead of the CTA's own
// weight copies and made the layer slower.)
__device__ void find_candidates(const Params& p, const RouteTail& rt, int t, int lane, uint64_t* ckey, int* ncand) {
  const int E = p.n_router, K = p.top_k;
  float lv[8];
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lv[i] = lane + 32 * i < E ? rt.logits[t][lane + 32 * i] : -FLT_MAX;
    m = fmaxf(m, lv[i]);
  }
  // rank of this lane's maximum among the 32 (ties to the lower lane): a permutation of 0..31
  int beats = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float o = __shfl_sync(0xffffffffu, m, j);
    beats += (o > m || (o == m && j < lane)) ? 1 : 0;
  }
  const unsigned who = __ballot_sync(0xffffffffu, beats == K - 1);
  const float theta = __shfl_sync(0xffffffffu, m, __ffs(who) - 1);
  // candidate index of (lane, i): the candidates of the columns before i, then of the lanes before
  int base = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool c = lane + 32 * i < E && lv[i] >= theta;
    const unsigned bal = __ballot_sync(0xffffffffu, c);
    const int k = base + __popc(bal & ((1u << lane) - 1u));
    if (c && k < 32)
      ckey[k] = (static_cast<uint64_t>(order_key(lv[i])) << 32) | static_cast<uint32_t>(~(lane + 32 * i));
    base += __popc(bal);
  }
  if (lane == 0) *ncand = base;
}

// Row t's logit maximum and softmax denominator, in the order route_row sums them (each lane its 8
// logits in index order, then the butterfly), so the routing weights come out identical.
__device__ void row_softmax_sum(const Params& p, const RouteTail& rt, int t, int lane, float& m_out, float& z_out) {
  const int E = p.n_router;
  float lv[8];
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lv[i] = lane + 32 * i < E ? rt.logits[t][lane + 32 * i] : -FLT_MAX;
    m = fmaxf(m, lv[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (lane + 32 * i < E) z += expf(lv[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  m_out = m;
  z_out = z;
}

// The top_k of row t from its candidates (every expert that can be selected, at most 32): lane c
// ranks candidate c by counting the larger keys, which gives the order of route_row's merge (logit
// descending, ties to the lower expert); then softmax weights and renormalisation as route_row.
__device__ void route_row_candidates(const Params& p, FAux& aux, int t, int lane, bool emit) {
  const int K = p.top_k, nc = aux.ncand[t];
  const uint64_t mine = lane < nc ? aux.ckey[t][lane] : 0ull;
  int rank = 0;
  for (int j = 0; j < nc; ++j) rank += aux.ckey[t][j] > mine ? 1 : 0;
  if (lane < nc && rank < K) {
    aux.sel_e[t][rank] = static_cast<int>(~static_cast<uint32_t>(mine));
    aux.sel_v[t][rank] = key_value(static_cast<uint32_t>(mine >> 32));
  }
  __syncwarp();
  const float m = aux.rmax[t], z = aux.rz[t];
  int my_e = 0;
  float my_v = 0.f;
  if (lane < K) {
    my_e = aux.sel_e[t][lane];
    my_v = aux.sel_v[t][lane];
  }
  const float my_p = expf(my_v - m) / z;
  float psum = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    const float pj = __shfl_sync(0xffffffffu, my_p, j);
    if (j < K) psum += pj;
  }
  RouteTail& rt = aux.rt;
  if (lane < K) {
    const __nv_bfloat16 wb = __float2bfloat16_rn(my_p / psum);
    rt.sel_e[t * K + lane] = my_e;
    rt.sel_w[t * K + lane] = __bfloat162float(wb);
    if (emit && p.ids_out) p.ids_out[t * K + lane] = my_e;
    if (emit && p.w_out) p.w_out[t * K + lane] = wb;
  }
  if (lane == 0) rt.shared_coef[t] = p.sh_gate ? bf16_round(1.f / (1.f + expf(-rt.logits[t][p.n_router]))) : 1.f;
}

// The four epilogue warps wait for one mbarrier phase (lane 0 of each, bounded) and continue only
// if all four waits succeeded: a uniform decision, so no warp is left alone at a named barrier.
__device__ __forceinline__ bool epi_wait_all(FAux& aux, uint64_t* bar, uint32_t parity, bool cluster_scope, int e,
                                             int lane) {
  bool ok = true;
  if (lane == 0) ok = cluster_scope ? mbar_wait_cluster(bar, parity) : mbar_wait(bar, parity);
  if (lane == 0) aux.epi_ok[e] = ok ? 1 : 0;
  named_bar(kBarEpi, kEpiThreads);
  ok = aux.epi_ok[0] && aux.epi_ok[1] && aux.epi_ok[2] && aux.epi_ok[3];
  named_bar(kBarEpi, kEpiThreads);  // epi_ok may be rewritten by the next wait
  return ok;
}

// ---------------------------------------------------------------- epilogues
// Up: as epilogue_up, thread r holds gate row c0 + 64q + r (r < 64) or the matching up row; the up
// values reach the gate threads through shared memory. The gate threads apply SwiGLU, round h to
// bf16 (the reference's activation dtype) and split it exactly into e4m3 hi + lo with one
// power-of-two exponent for the CTA's 64 columns. The bytes are staged in shared memory, then each
// gate thread stores one 16-byte chunk into one CTA of the cluster (rows hi 0-3 / lo 0-3 of the down
// MMAs' B operand, at the swizzled position of these columns) and thread 0 the exponent vector into
// both; each store counts its bytes on the receiver's hx_full.
__device__ void cl_epilogue_up(const Params& p, FAux& aux, uint8_t* hb, uint32_t taddr, bool shared_slot, int q,
                               int e, int lane, const float (&sc)[kMaxH / 128]) {
  const int r = 32 * e + lane;
  float acc[kMaxT];
  reduce_acc<kMaxH / 128>(taddr, p.H / 128, [&](int j, int) { return sc[j]; }, acc);
  tc::fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(&aux.acc_empty);
  if (r >= kUpHalf)
#pragma unroll
    for (int t = 0; t < kMaxT; ++t) aux.upv[r - kUpHalf][t] = acc[t] * aux.xinv[t];
  named_bar(kBarEpi, kEpiThreads);
  if (r >= kUpHalf) return;
  float hv[kMaxT];
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) {
    hv[t] = 0.f;
    if (t < p.T) {
      float gt = acc[t] * aux.xinv[t];
      float ut = aux.upv[r][t];
      if (shared_slot) {
        // the shared expert is a chain of bf16 modules: down(silu(gate(x)) * up(x))
        gt = bf16_round(gt);
        ut = bf16_round(ut);
        hv[t] = bf16_round(bf16_round(gt * __frcp_rn(1.f + __expf(-gt))) * ut);
      } else {
        hv[t] = bf16_round(gt * __frcp_rn(1.f + __expf(-gt)) * ut);
      }
    }
    const uint32_t am = t < p.T ? __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(hv[t]))) : 0u;
    if (lane == 0) aux.hmax[e][t] = am;
  }
  named_bar(kBarGate, 2 * 32);
  float ex[kMaxT];
#pragma unroll
  for (int t = 0; t < kMaxT; t += 2) {
    const int e0 = split_exponent(__uint_as_float(max(aux.hmax[0][t], aux.hmax[1][t])));
    const int e1 = split_exponent(__uint_as_float(max(aux.hmax[0][t + 1], aux.hmax[1][t + 1])));
    ex[t] = exp2i(-e0);
    ex[t + 1] = exp2i(-e1);
    uint16_t hi, lo;
    split2(hv[t] * exp2i(e0), hv[t + 1] * exp2i(e1), hi, lo);
    aux.hstage[t][r] = static_cast<uint8_t>(hi & 0xFF);
    aux.hstage[t + 1][r] = static_cast<uint8_t>(hi >> 8);
    aux.hstage[4 + t][r] = static_cast<uint8_t>(lo & 0xFF);
    aux.hstage[5 + t][r] = static_cast<uint8_t>(lo >> 8);
  }
  named_bar(kBarGate, 2 * 32);
  const uint32_t lbar = smem_u32(&aux.hx_full);
  {
    const int ch = r & 31, row = ch >> 2, c = ch & 3, d = r >> 5;
    const uint4 v = *reinterpret_cast<const uint4*>(&aux.hstage[row][16 * c]);
    const uint32_t laddr = smem_u32(hb + tc::swz_offset(row, kUpHalf * q + 16 * c, kN));
    st_async16(mapa_shared(laddr, d), v, mapa_shared(lbar, d));
  }
  if (r == 0) {
    const uint4 xv = make_uint4(__float_as_uint(ex[0]), __float_as_uint(ex[1]), __float_as_uint(ex[2]),
                                __float_as_uint(ex[3]));
    const uint32_t la = smem_u32(&aux.hexp[q][0]);
#pragma unroll
    for (int d = 0; d < kCl; ++d) st_async16(mapa_shared(la, d), xv, mapa_shared(lbar, d));
  }
}

// Down, for kB consecutive 128-row blocks (nb of them valid) of this CTA: thread r holds output row
// rows0 + 128 b + r of block b for the quarter's 128 k. A block's two accumulators (16 TMEM columns
// each) cover the 64 columns of h from CTA 0 and from CTA 1 of the cluster, each with its own 2^-e;
// sc[b] is the weight's 128-block scale. Every accumulator of the batch is read before the first
// wait. The contributions (times the routing weight; the shared expert's stay raw) are added to the
// fixed-point sums of their rows.
template <int kB>
__device__ __forceinline__ void cl_epilogue_down(const Params& p, const WsLayout& L, FAux& aux, uint32_t taddr,
                                                 int slot, bool shared_slot, int row0, const float* sc, int nb) {
  float v[kB][2][8];
#pragma unroll
  for (int b = 0; b < kB; ++b)
    if (b < nb) {
      tc::tmem_ld8(taddr + 32u * b, v[b][0]);
      tc::tmem_ld8(taddr + 32u * b + 16u, v[b][1]);
    }
  tc::tmem_wait_ld();
  unsigned long long* fa = reinterpret_cast<unsigned long long*>(p.ws + L.facc) +
                           static_cast<size_t>(shared_slot ? kMaxT : 0) * p.H + row0;
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) {
    if (t >= p.T) break;
    const float h0 = aux.hexp[0][t], h1 = aux.hexp[1][t];
    const float cf = shared_slot ? 1.f : aux.tab.coef[slot * kMaxT + t];
#pragma unroll
    for (int b = 0; b < kB; ++b)
      if (b < nb) {
        const float y = sc[b] * fmaf(h0, v[b][0][t] + v[b][0][4 + t], h1 * (v[b][1][t] + v[b][1][4 + t])) * cf;
        atomicAdd(fa + static_cast<size_t>(t) * p.H + kBlockRows * b,
                  static_cast<unsigned long long>(__float2ll_rn(y * aux.fixu[t])));
      }
  }
}

// The fixed-point sums to y, after the cluster kernel has completed: one thread per pair of output
// elements, with the rounding points of combine_kernel,
// y = bf16(bf16(bf16(routed) + bias) + bf16(sigmoid gate * bf16(shared))); the sums are cleared for
// the next call. A sum converts to fp32 with one rounding (int64 -> float, then an exact 2^-u).
// Kernel completion orders every CTA's reductions before these loads, so the cluster kernel needs
// no fence, counter or last-CTA step of its own; the bias is requested before griddepcontrol.wait.
// (Releasing the next layer's route kernel at this kernel's entry, so that it fetches its router
// rows during the cluster kernel, measured 1.8 µs per layer slower: its CTAs then sit on the
// cluster kernel's SMs.)
constexpr int kFinishThreads = 256;
__global__ void __launch_bounds__(kFinishThreads) finish_kernel(const __grid_constant__ Params p) {
  const WsLayout L = ws_layout(p.H, p.I);
  const int i = (blockIdx.x * kFinishThreads + threadIdx.x) * 2;  // first of two consecutive outputs
  const bool active = i < p.T * p.H;
  const int t = active ? i / p.H : 0, n = active ? i % p.H : 0;
  float b0 = 0.f, b1 = 0.f;
  if (active && p.out_bias) {
    b0 = __ldg(p.out_bias + n);
    b1 = __ldg(p.out_bias + n + 1);
  }
  griddep_wait();
  griddep_launch();
  if (!active) return;
  long long* fa = reinterpret_cast<long long*>(p.ws + L.facc);
  const size_t shared_off = static_cast<size_t>(kMaxT) * p.H;
  const size_t off = static_cast<size_t>(t) * p.H + n;
  const longlong2 R = __ldcg(reinterpret_cast<const longlong2*>(fa + off));
  const bool sh = p.sh_w13 != nullptr;
  longlong2 S = make_longlong2(0, 0);
  float g = 0.f;
  if (sh) {
    S = __ldcg(reinterpret_cast<const longlong2*>(fa + shared_off + off));
    g = __ldcg(reinterpret_cast<const float*>(p.ws + L.gate) + t);
  }
  const float unit = __ldcg(reinterpret_cast<const float*>(p.ws + L.xinv) + t);
  float y0 = bf16_round(__ll2float_rn(R.x) * unit), y1 = bf16_round(__ll2float_rn(R.y) * unit);
  if (p.out_bias) {
    y0 = bf16_round(y0 + b0);
    y1 = bf16_round(y1 + b1);
  }
  if (sh) {
    y0 += bf16_round(g * bf16_round(__ll2float_rn(S.x) * unit));
    y1 += bf16_round(g * bf16_round(__ll2float_rn(S.y) * unit));
  }
  *reinterpret_cast<__nv_bfloat162*>(p.y + off) = __floats2bfloat162_rn(y0, y1);
  __stcg(reinterpret_cast<longlong2*>(fa + off), make_longlong2(0, 0));
  if (sh) __stcg(reinterpret_cast<longlong2*>(fa + shared_off + off), make_longlong2(0, 0));
}

// x split into the up MMAs' B operand by the 64 threads of warps 2-3 (which are otherwise idle while
// the experts are selected): row t holds the e4m3 hi part of x[t] * 2^e_t (e_t maps the row's
// absolute maximum into [128, 256)), row 4 + t the lo remainder; rows of absent tokens and rows 8-15
// only feed accumulator columns that nothing reads. The threads fence their writes for the tensor
// core, then thread 0 arrives on xb_ready.
__device__ void cl_split_x(const Params& p, uint8_t* bt, FAux& aux, int sidx) {
  constexpr int kNT = 64;
  constexpr int kMaxTasks = kMaxT * (kMaxH / 16) / kNT;
  const int chunks = p.H / 16, n = p.T * chunks;
  if (sidx < kMaxT) aux.xmax[sidx] = 0u;
  named_bar(kBarSplit, kNT);
  uint4 v[kMaxTasks][2];
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = sidx + q * kNT;
    if (task < n) {
      const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(task / chunks) * p.H + (task % chunks) * 16);
      v[q][0] = src[0];
      v[q][1] = src[1];
    }
  }
  // this thread's maximum per row, then one warp reduction and one atomic per row
  float m[kMaxT] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = sidx + q * kNT;
    if (task < n) {
      const int t = task / chunks;
      const float a = abs_max16(v[q]);
#pragma unroll
      for (int u = 0; u < kMaxT; ++u)
        if (u == t) m[u] = fmaxf(m[u], a);
    }
  }
#pragma unroll
  for (int t = 0; t < kMaxT; ++t) {
    if (t >= p.T) break;
    const uint32_t wm = __reduce_max_sync(0xffffffffu, __float_as_uint(m[t]));
    if ((sidx & 31) == 0) atomicMax(&aux.xmax[t], wm);
  }
  named_bar(kBarSplit, kNT);
  if (sidx < kMaxT) {
    const float am = __uint_as_float(aux.xmax[sidx]);
    aux.xinv[sidx] = exp2i(-split_exponent(am));
    aux.fixu[sidx] = exp2i(fix_exponent(am));
    // the finish kernel converts the sums with the inverse unit (the x-split slot of the workspace is
    // free on this path)
    if (blockIdx.x == 0 && sidx < p.T)
      reinterpret_cast<float*>(p.ws + ws_layout(p.H, p.I).xinv)[sidx] = exp2i(-fix_exponent(am));
  }
#pragma unroll
  for (int q = 0; q < kMaxTasks; ++q) {
    const int task = sidx + q * kNT;
    if (task < n) {
      const int t = task / chunks, c = task % chunks;
      uint4 hi, lo;
      split16(v[q], exp2i(split_exponent(__uint_as_float(aux.xmax[t]))), hi, lo);
      *reinterpret_cast<uint4*>(bt + tc::swz_offset(t, c * 16, kN)) = hi;
      *reinterpret_cast<uint4*>(bt + tc::swz_offset(4 + t, c * 16, kN)) = lo;
    }
  }
  tc::fence_proxy_async_smem();
  named_bar(kBarSplit, kNT);
  if (sidx == 0) mbar_arrive(&aux.xb_ready);
}

// ---------------------------------------------------------------- the cluster kernel
// Grid: one cluster of kCl CTAs per (possible slot, quarter of I); clusters past the call's slot
// count leave after the selection. Warp roles as in expert_kernel: warp 0 lane 0 feeds the ring with
// TMA copies (the CTA's up slabs, then its down slabs), warp 1 lane 0 issues the MMAs, warps 4-7
// select the experts, then run the epilogues.
__global__ void __launch_bounds__(kThreads, 1)
    layer_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map13,
                 const __grid_constant__ CUtensorMap map2, const __grid_constant__ CUtensorMap msh13,
                 const __grid_constant__ CUtensorMap msh2) {
  extern __shared__ uint8_t smem_raw[];
  // the same offset in every CTA, so mapa of a local address names the same buffer in the peer
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const FSmem S = fsmem_layout(p.H, p.I);
  const WsLayout L = ws_layout(p.H, p.I);
  FAux& aux = *reinterpret_cast<FAux*>(smem + S.aux);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = static_cast<int>(cluster_ctarank());
  const int nq = p.I / 128;                            // quarters (128 columns of h each)
  const int slot = static_cast<int>(cluster_id_x()) / nq, quarter = static_cast<int>(cluster_id_x()) % nq;
  const int c0 = 128 * quarter;                        // first column of h of this cluster
  const bool shared_slot = p.sh_slot != 0 && slot == 0;
  const int nkb = p.H / 128;                           // up k blocks
  const int n_up = nkb / 2;                            // up ring stages (two slabs each)
  const int ntiles = p.H / 2 / kBlockRows;             // down blocks of this CTA
  const int n_total = n_up + ntiles / 2;               // + down ring stages (two blocks each)
  const int row_base = q * (p.H / 2);                  // first output row of this CTA

  if (tid == 0) {
    tc::prefetch_map(&map13);
    tc::prefetch_map(&map2);
    if (p.sh_slot) {
      tc::prefetch_map(&msh13);
      tc::prefetch_map(&msh2);
    }
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(&aux.full[s], 1);
      mbar_init(&aux.empty[s], 1);
    }
    mbar_init(&aux.xb_ready, 1);
    mbar_init(&aux.acc_full, 1);
    mbar_init(&aux.acc_empty, kEpiThreads / 32);
    mbar_init(&aux.hx_full, 1);
    for (int j = 0; j < kFMaxTiles; ++j) mbar_init(&aux.dacc_full[j], 1);
    fence_mbar_init();
    // armed before the cluster barrier below, so no peer's st.async can reach it earlier
    mbar_arrive_expect_tx(&aux.hx_full, kCl * kHxBytesPerSrc);
  }
  if (warp == kWarpMma) tc::tmem_alloc(&aux.tmem, kFTmemCols);
  tc::fence_before_sync();
  cluster_sync_all();
  tc::fence_after_sync();
  const uint32_t tmem = aux.tmem;

  if (warp == kWarpTma) {
    // ================================================================ TMA producer (lane 0 issues)
    int stage = 0, s_next = 0;
    uint32_t empty_par = 1;
    bool ok = true;
    auto issue = [&](int s, int ex, const CUtensorMap* m13, const CUtensorMap* m2) -> bool {
      if (!mbar_wait(&aux.empty[stage], empty_par)) {
        flag_error(p, L, STATUS_TIMEOUT);
        return false;
      }
      uint8_t* dst = smem + S.stage + stage * kStageBytes;
      mbar_arrive_expect_tx(&aux.full[stage], static_cast<uint32_t>(kStageBytes));
      if (s < n_up) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int kx = (2 * s + j) * 128;
          tc::tma_load_3d(dst + j * kSlabBytes, m13, kx, c0 + kUpHalf * q, ex, &aux.full[stage]);
          tc::tma_load_3d(dst + j * kSlabBytes + kSlabBytes / 2, m13, kx, p.I + c0 + kUpHalf * q, ex,
                          &aux.full[stage]);
        }
      } else {
        const int tile0 = 2 * (s - n_up);
#pragma unroll
        for (int j = 0; j < 2; ++j)
          tc::tma_load_3d(dst + j * kSlabBytes, m2, c0, row_base + kBlockRows * (tile0 + j), ex, &aux.full[stage]);
      }
      if (++stage == kFStages) {
        stage = 0;
        empty_par ^= 1u;
      }
      return true;
    };
    if (lane == 0) {
      // the shared expert needs no routing: its first ring of stages goes out before the wait
      if (shared_slot)
        for (; ok && s_next < kFStages && s_next < n_total; ++s_next) ok = issue(s_next, 0, &msh13, &msh2);
      griddep_wait();
      griddep_launch();
    }
    __syncwarp();
    named_bar(kBarTable, kTableThreads);
    if (lane == 0) {
      if (slot < aux.n_slots) {
        const int ex = shared_slot ? 0 : aux.tab.expert[slot];
        const CUtensorMap* m13 = shared_slot ? &msh13 : &map13;
        const CUtensorMap* m2 = shared_slot ? &msh2 : &map2;
        for (; ok && s_next < n_total; ++s_next) ok = issue(s_next, ex, m13, m2);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ================================================================ MMA issuer (lane 0 issues)
    named_bar(kBarTable, kTableThreads);
    if (lane == 0 && slot < aux.n_slots) {
      bool ok = mbar_wait(&aux.xb_ready, 0);
      const uint32_t idesc = tc::idesc_e4m3(kTileRows, kN);
      const uint32_t xb = smem_u32(smem + S.xb), hb = smem_u32(smem + S.hb);
      int stage = 0;
      uint32_t full_par = 0;
      auto advance = [&]() {
        if (++stage == kFStages) {
          stage = 0;
          full_par ^= 1u;
        }
      };
      // up: one accumulator per 128-wide k block
      for (int c = 0; ok && c < n_up; ++c) {
        ok = mbar_wait(&aux.full[stage], full_par);
        if (!ok) break;
        const uint32_t a = smem_u32(smem + S.stage + stage * kStageBytes);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int kb = 2 * c + j;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)
            tc::mma_f8(tmem + kb * 16, tc::smem_desc(a + j * kSlabBytes + 32 * k4),
                       tc::smem_desc(xb + kb * kBSlabBytes + 32 * k4), idesc, k4 > 0);
        }
        tc::mma_commit(&aux.empty[stage]);
        advance();
      }
      if (ok) tc::mma_commit(&aux.acc_full);
      if (ok) {
        // h from both CTAs of the cluster (st.async), made visible to the tensor core's proxy
        ok = mbar_wait_cluster(&aux.hx_full, 0);
        tc::fence_proxy_async_smem();
        tc::fence_after_sync();
      }
      // down: per 128-row block, one accumulator per source CTA's 64 columns of h
      for (int c = 0; ok && c < ntiles / 2; ++c) {
        ok = mbar_wait(&aux.full[stage], full_par);
        if (!ok) break;
        const uint32_t a = smem_u32(smem + S.stage + stage * kStageBytes);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int tile = 2 * c + j;
          const uint32_t d = tmem + 256u + 32u * tile;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)
            tc::mma_f8(d + (k4 >> 1) * 16, tc::smem_desc(a + j * kSlabBytes + 32 * k4), tc::smem_desc(hb + 32 * k4),
                       idesc, (k4 & 1) != 0);
          tc::mma_commit(&aux.dacc_full[tile]);
        }
        tc::mma_commit(&aux.empty[stage]);
        advance();
      }
      if (!ok) flag_error(p, L, STATUS_TIMEOUT);
    }
    __syncwarp();
  } else if (warp < kWarpEpi) {
    // ================================================================ warps 2-3: the x split
    griddep_wait();  // x comes from the preceding kernels
    cl_split_x(p, smem + S.xb, aux, tid - 64);
  } else {
    // ================================================================ selection, then epilogues
    const int e = warp - kWarpEpi, et = tid - kWarpEpi * 32;
    griddep_wait();
    griddep_launch();
    {
      // the logits of every row (the last column is the shared expert's gate), requested at once:
      // one L2 round trip
      const int rows = p.n_router + (p.sh_w13 != nullptr && p.sh_gate != nullptr ? 1 : 0);
      const float* lg = reinterpret_cast<const float*>(p.ws + L.logits);
      constexpr int kPer = (kMaxT * (kMaxRouter + 1) + kEpiThreads - 1) / kEpiThreads;
      float v[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int k = et + i * kEpiThreads;
        v[i] = k < p.T * (kMaxRouter + 1) && k % (kMaxRouter + 1) < rows ? __ldcg(lg + k) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int k = et + i * kEpiThreads;
        if (k < kMaxT * (kMaxRouter + 1)) (&aux.rt.logits[0][0])[k] = v[i];
      }
    }
    named_bar(kBarEpi, kEpiThreads);
    if (p.T <= 2) {
      // warps 4..4+T-1 take each row's maximum and softmax sum while warps 4+T.. find the row's
      // candidates; then the first warps rank the candidates
      if (e < p.T)
        row_softmax_sum(p, aux.rt, e, lane, aux.rmax[e], aux.rz[e]);
      else if (e < 2 * p.T)
        find_candidates(p, aux.rt, e - p.T, lane, aux.ckey[e - p.T], &aux.ncand[e - p.T]);
      named_bar(kBarEpi, kEpiThreads);
      if (e < p.T) {
        if (aux.ncand[e] <= 32)
          route_row_candidates(p, aux, e, lane, blockIdx.x == 0);
        else
          route_row(p, aux.rt, e, lane, blockIdx.x == 0);  // ties over more than 32 experts
      }
    } else if (e < p.T) {
      route_row(p, aux.rt, e, lane, blockIdx.x == 0);
    }
    named_bar(kBarEpi, kEpiThreads);
    if (blockIdx.x == 0 && et < p.T) reinterpret_cast<float*>(p.ws + L.gate)[et] = aux.rt.shared_coef[et];
    if (e == 0) {
      const int n = table_smem(p, aux.rt, lane, aux.tab);
      if (lane == 0) aux.n_slots = n;
    }
    named_bar(kBarTable, kTableThreads);
    if (slot < aux.n_slots) {
      const ExpertRef ex = expert_ref(p, slot, aux.tab.expert);
      const int r = 32 * e + lane;
      const uint32_t tlane = static_cast<uint32_t>(32 * e) << 16;
      // every block scale this thread needs, requested before the first accumulator wait
      float sc13[kMaxH / 128];
      const int wrow = r < kUpHalf ? c0 + kUpHalf * q + r : p.I + c0 + kUpHalf * q + (r - kUpHalf);
      load_scales(ex.s13 + static_cast<size_t>(wrow / ex.srows) * nkb, nkb, sc13, kMaxH / 128);
      float sc2[kFMaxTiles];
#pragma unroll
      for (int j = 0; j < kFMaxTiles; ++j) {
        const int row = row_base + kBlockRows * j + r;
        sc2[j] = j < ntiles ? __ldg(ex.s2 + static_cast<size_t>(row / ex.srows) * nq + quarter) : 0.f;
      }
      hold(sc13);
      hold(sc2);
      // xb_ready orders the split warps' xinv before this read; acc_full comes later anyway
      bool ok = epi_wait_all(aux, &aux.xb_ready, 0, false, e, lane);
      ok = ok && epi_wait_all(aux, &aux.acc_full, 0, false, e, lane);
      if (ok) {
        tc::fence_after_sync();
        cl_epilogue_up(p, aux, smem + S.hb, tmem + tlane, shared_slot, q, e, lane, sc13);
        ok = epi_wait_all(aux, &aux.hx_full, 0, true, e, lane);
      }
      // four blocks at a time: the MMAs are committed in order, so block j + 3's barrier covers the
      // batch, and the first batch is read while the MMAs of the second are issued
#pragma unroll
      for (int j = 0; j < kFMaxTiles; j += 4) {
        if (!ok || j >= ntiles) break;
        ok = epi_wait_all(aux, &aux.dacc_full[min(j + 3, ntiles - 1)], 0, false, e, lane);
        if (!ok) break;
        tc::fence_after_sync();
        cl_epilogue_down<4>(p, L, aux, tmem + tlane + 256u + 32u * j, slot, shared_slot, row_base + kBlockRows * j + r,
                            &sc2[j], min(4, ntiles - j));
      }
      if (!ok && et == 0) flag_error(p, L, STATUS_TIMEOUT);

    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kWarpMma) tc::tmem_dealloc(tmem, kFTmemCols);
}
