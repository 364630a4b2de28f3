// Block-FP8 GEMV on the tcgen05 tensor cores (sm_100a): y[M, N] = x[M, K] * dequant(q[N, K])^T,
// M <= 4 activation rows, for weights whose rows are contiguous (the dense FP8Linear layers).
//
// Work split: one 128-row tile of q per thread-block cluster and one K chunk per CTA of the
// cluster (split-K), so that every SM streams an equal share of the weights: 2048x4096 runs as 32
// tiles x 4 chunks of 512, 4096x2048 as 16 x 8 of 512, 2048x8192 as 64 x 2 of 1024.
//
// Per CTA (8 warps):
//   warp 0    lane 0 loads the whole chunk (at most 8 slabs of 128 rows x 128 bytes, 128-byte
//             swizzle) with TMA before griddepcontrol.wait: weights never come from the preceding
//             kernel, so in a chain of GEMVs the copies overlap the previous kernel's tail
//   warps 2-3 split the chunk of x exactly into e4m3 hi (rows 0-3) and lo (rows 4-7) with a
//             power-of-two prescale taken from the chunk's absolute maximum
//   warp 1    lane 0 issues tcgen05.mma kind::f8f6f4 (M = 128 weight rows, N = 16, K = 32), one
//             TMEM accumulator of 16 columns per 128-wide k block
//   warps 4-7 read TMEM (one weight row per thread), apply the fp32 block scales per k block and
//             the prescale, and leave the chunk's partial sums in shared memory
// Each CTA then owns 128 / split rows of the tile: every epilogue thread pushes its row's partial
// sums (16 bytes) into the owner's shared memory with st.async, counted on the owner's mbarrier;
// the owner sums the split partials in rank order (a fixed order, so the result does not depend on
// arrival order), adds the bias and writes y. No cluster-wide barrier sits on the path after the
// MMAs: one cluster barrier at kernel start (arrive early, wait just before the first push) makes
// every CTA's mbarrier initialisation visible to the others. The per-block scale multiplies each
// 128-wide k-block partial in fp32, as the reference Triton kernel does (fp8_linear.py:21-26).
// A bounded wait that runs out sets a bit in the library's GEMV status word (dm3_gemv_status).
#include <cooperative_groups.h>

#include "dm3_common.cuh"
#include "dm3_internal.h"
#include "dm3_tc.cuh"

namespace cg = cooperative_groups;

namespace dm3 {
namespace gemv_tc {

// Split cluster barrier: every thread arrives (release) after initialisation and waits (acquire)
// once, before it first touches another CTA's shared memory.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async16(uint32_t raddr, uint4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   raddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const uint64_t t0 = globaltimer();
  while (!try_once()) {
    if (globaltimer() - t0 > wait_limit_ns()) return false;
  }
  return true;
}

constexpr int kThreads = 256;
constexpr int kTileRows = 128;
constexpr int kN = 16;
constexpr int kSlabBytes = kTileRows * 128;
constexpr int kBSlabBytes = kN * 128;
constexpr int kMaxSlabs = 8;                  // slabs per CTA (K chunk <= 1024)
constexpr int kMaxSplit = 8;                  // CTAs per cluster (portable cluster size)
constexpr uint32_t kTmemCols = kMaxSlabs * 16;
constexpr int kSplitThreads = 64;

struct Params {
  const __nv_bfloat16* x;
  int M, K, N;
  const float* s;
  int64_t lds;
  int srows;
  const void* bias;
  int bias_kind;
  void* y;
  int64_t ldy;
  int y_fp32;
  int split;  // CTAs per cluster (K chunks)
  int nsl;    // slabs per CTA
};

// Sticky status of every tensor-core GEMV launch on this device (dm3_gemv_status reads and clears it).
static __device__ uint32_t g_status;

struct Aux {
  uint64_t full, done, rx_full;
  uint32_t tmem;
  uint32_t xmax[kMaxT];
  float xinv[kMaxT];
  // partial sums of the rows this CTA owns: [source rank][row within the owned block][token]
  alignas(16) float recv[kTileRows][kMaxT];
};

__host__ __device__ inline int smem_bytes(int nsl) {
  return nsl * kSlabBytes + nsl * kBSlabBytes + static_cast<int>((sizeof(Aux) + 127) / 128 * 128) + 1024;
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

__global__ void __launch_bounds__(kThreads, 1) gemv_tc_kernel(const __grid_constant__ Params p,
                                                             const __grid_constant__ CUtensorMap map_q) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int tile = blockIdx.x / p.split;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nsl = p.nsl, kchunk = nsl * 128, k0 = rank * kchunk;
  uint8_t* a_tiles = smem;
  uint8_t* b_tile = smem + nsl * kSlabBytes;
  Aux& aux = *reinterpret_cast<Aux*>(b_tile + nsl * kBSlabBytes);

  const int per = kTileRows / p.split;  // rows owned by each CTA of the cluster
  if (tid == 0) {
    tc::prefetch_map(&map_q);
    mbar_init(&aux.full, 1);
    mbar_init(&aux.done, 1);
    mbar_init(&aux.rx_full, 1);
    fence_mbar_init();
    // armed before the cluster barrier's arrival, so no peer's push can come first
    mbar_arrive_expect_tx(&aux.rx_full, static_cast<uint32_t>((p.split - 1) * per * 16));
  }
  if (tid < kMaxT) aux.xmax[tid] = 0u;
  if (warp == 1) tc::tmem_alloc(&aux.tmem, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  cluster_arrive();
  const uint32_t tmem = aux.tmem;

  if (warp == 0) {
    if (lane == 0) {
      // the next kernel may start as soon as every CTA of this one runs: in a chain of GEMVs its weight
      // copies then overlap this one (each kernel still waits for its predecessor's completion before
      // touching x or y, so the data order is unchanged)
      griddep_launch();
      mbar_arrive_expect_tx(&aux.full, static_cast<uint32_t>(nsl * kSlabBytes));
      for (int j = 0; j < nsl; ++j)
        tc::tma_load_3d(a_tiles + j * kSlabBytes, &map_q, k0 + j * 128, tile * kTileRows, 0, &aux.full);
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // x chunk -> activation tile (rows t: hi, 4 + t: lo; other rows only feed unread columns)
    const int sidx = tid - 64;
    griddep_wait();
    const int chunks = kchunk / 16, n = p.M * chunks;
    constexpr int kMaxTasks = kMaxT * (kMaxSlabs * 128 / 16) / kSplitThreads;
    uint4 v[kMaxTasks][2];
#pragma unroll
    for (int q = 0; q < kMaxTasks; ++q) {
      const int task = sidx + q * kSplitThreads;
      if (task < n) {
        const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(task / chunks) * p.K + k0 + (task % chunks) * 16);
        v[q][0] = src[0];
        v[q][1] = src[1];
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(v[q]);
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(__bfloat162float(e[i])));
        atomicMax(&aux.xmax[task / chunks], __float_as_uint(m));
      }
    }
    named_bar(2, kSplitThreads);
    if (sidx < kMaxT) aux.xinv[sidx] = exp2i(-split_exponent(__uint_as_float(aux.xmax[sidx])));
#pragma unroll
    for (int q = 0; q < kMaxTasks; ++q) {
      const int task = sidx + q * kSplitThreads;
      if (task < n) {
        const int t = task / chunks, c = task % chunks;
        uint4 hi, lo;
        split16(v[q], exp2i(split_exponent(__uint_as_float(aux.xmax[t]))), hi, lo);
        *reinterpret_cast<uint4*>(b_tile + tc::swz_offset(t, c * 16, kN)) = hi;
        *reinterpret_cast<uint4*>(b_tile + tc::swz_offset(4 + t, c * 16, kN)) = lo;
      }
    }
    tc::fence_proxy_async_smem();
  } else if (warp >= 4) {
    griddep_wait();  // y may be read by the preceding kernel's consumers until it completes
  }
  __syncthreads();  // activation tile written (and fenced for the tensor core), xinv set

  if (warp == 1 && lane == 0) {
    if (mbar_wait(&aux.full, 0)) {
      tc::fence_after_sync();
      const uint32_t idesc = tc::idesc_e4m3(kTileRows, kN);
      const uint32_t a = smem_u32(a_tiles), b = smem_u32(b_tile);
      // k step outer, slab inner: consecutive MMAs go to different accumulators
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4)
        for (int j = 0; j < nsl; ++j)
          tc::mma_f8(tmem + j * 16, tc::smem_desc(a + j * kSlabBytes + 32 * k4), tc::smem_desc(b + j * kBSlabBytes + 32 * k4),
                     idesc, k4 > 0);
      tc::mma_commit(&aux.done);
    } else {
      atomicOr(&g_status, STATUS_TIMEOUT);
    }
  }
  if (warp >= 4) {
    const int e = warp - 4;
    const int r = 32 * e + lane, n = tile * kTileRows + r;
    const int kb0 = k0 / 128;
    float sc[kMaxSlabs];
#pragma unroll
    for (int j = 0; j < kMaxSlabs; ++j)
      sc[j] = (j < nsl && n < p.N) ? __ldg(p.s + static_cast<size_t>(n / p.srows) * p.lds + kb0 + j) : 0.f;
    bool ready = true;
    if (lane == 0) ready = mbar_wait(&aux.done, 0);
    ready = __shfl_sync(0xffffffffu, ready, 0);
    if (!ready && lane == 0) atomicOr(&g_status, STATUS_TIMEOUT);
    tc::fence_after_sync();
    float acc[kMaxT] = {0.f, 0.f, 0.f, 0.f};
    float v[kMaxSlabs][8];
    const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * e) << 16);
#pragma unroll
    for (int j = 0; j < kMaxSlabs; ++j)
      if (j < nsl) tc::tmem_ld8(taddr + j * 16, v[j]);
    tc::tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < kMaxSlabs; ++j)
      if (j < nsl)
#pragma unroll
        for (int t = 0; t < kMaxT; ++t) acc[t] = fmaf(sc[j], v[j][t] + v[j][4 + t], acc[t]);
    const float4 v4 = ready ? make_float4(acc[0] * aux.xinv[0], acc[1] * aux.xinv[1], acc[2] * aux.xinv[2],
                                          acc[3] * aux.xinv[3])
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    tc::fence_before_sync();
    // this row's partials to the CTA owning it: slot [my rank][row within the owned block]
    const int owner = r / per;
    const uint32_t slot = smem_u32(&aux.recv[rank * per + r % per][0]);
    cluster_wait();  // every CTA's rx_full is initialised and armed
    if (owner == rank) {
      *reinterpret_cast<float4*>(&aux.recv[rank * per + r % per][0]) = v4;
    } else {
      const uint4 u = make_uint4(__float_as_uint(v4.x), __float_as_uint(v4.y), __float_as_uint(v4.z),
                                 __float_as_uint(v4.w));
      st_async16(mapa_shared(slot, static_cast<uint32_t>(owner)), u,
                 mapa_shared(smem_u32(&aux.rx_full), static_cast<uint32_t>(owner)));
    }
    named_bar(1, 128);  // the owned rows' own partials are in shared memory
    bool got = true;
    if (p.split > 1) {
      if (lane == 0) got = mbar_wait_cluster(&aux.rx_full, 0);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got && lane == 0) atomicOr(&g_status, STATUS_TIMEOUT);
    }
    // the owned rows [rank * per, (rank + 1) * per): sum over the source ranks in order, + bias
    const int et = tid - 128;
    for (int i = et; i < per * p.M; i += 128) {
      const int t = i / per, rr = i % per;
      const int n = tile * kTileRows + rank * per + rr;
      if (n < p.N && got) {
        float sum = 0.f;
        for (int q = 0; q < p.split; ++q) sum += aux.recv[q * per + rr][t];
        if (p.bias_kind == 1) sum += __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n]);
        if (p.bias_kind == 2) sum += static_cast<const float*>(p.bias)[n];
        if (p.y_fp32)
          static_cast<float*>(p.y)[t * p.ldy + n] = sum;
        else
          static_cast<__nv_bfloat16*>(p.y)[t * p.ldy + n] = __float2bfloat16_rn(sum);
      }
    }
  } else {
    __syncwarp();    // warp 1 reconverges after its lane 0 issued the MMAs
    cluster_wait();  // every thread that arrived waits once
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace gemv_tc

// Launches the tensor-core GEMV; returns -1 when the shape is outside what it covers (the caller
// then uses the CUDA-core kernel).
int launch_gemv_tc(const __nv_bfloat16* x, int M, int K, int N, const uint8_t* q, int64_t ldq, const float* s,
                   int64_t lds, int srows, const void* bias, int bias_kind, void* y, int64_t ldy, int y_fp32,
                   cudaStream_t stream) {
  using namespace gemv_tc;
  const int slabs = K / 128;
  const int tiles = (N + kTileRows - 1) / kTileRows;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_error("cudaGetDevice failed");
    return 2;
  }
  const int sms = sm_count(dev);
  // the largest power-of-two split <= 8 that divides the slabs and does not exceed the SM count by
  // more than a few percent, raised until a CTA holds at most 4 slabs (64 KB): two CTAs then fit an
  // SM, so a chain's next GEMV loads its weights beside this one (measured on a 40-call chain:
  // 2048 x 8192 takes 5.6 µs per call at split 4, 6.3 at split 2)
  int split = 1;
  while (split * 2 <= kMaxSplit && slabs % (split * 2) == 0 && tiles * split * 2 <= sms + sms / 16) split *= 2;
  while (slabs / split > 4 && split * 2 <= kMaxSplit && slabs % (split * 2) == 0) split *= 2;
  if (slabs / split > kMaxSlabs || slabs % split) return -1;
  Params p{};
  p.x = x;
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
  p.split = split;
  p.nsl = slabs / split;
  CUtensorMap mq;
  if (!tensor_map_3d(&mq, q, static_cast<uint64_t>(K), static_cast<uint64_t>(N), 1, static_cast<uint64_t>(ldq),
                     static_cast<uint64_t>(ldq) * static_cast<uint64_t>(N), kTileRows))
    return 2;
  const int smem = smem_bytes(p.nsl);
  static bool configured[64] = {false};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(gemv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
      set_error("cudaFuncSetAttribute(gemv_tc) failed");
      return 2;
    }
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles * split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = split;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemv_tc_kernel, p, mq);
  if (err != cudaSuccess) {
    set_error(std::string("gemv_tc launch: ") + cudaGetErrorString(err));
    return 2;
  }
  note_launches(1);
  return 0;
}

}  // namespace dm3

namespace dm3 {
// This file's copy of the device wait limit on the current device (dm3_set_wait_limit_ns).
int wait_limit_gemv_tc(uint64_t ns) { return static_cast<int>(set_wait_limit_here(ns)); }
}  // namespace dm3

extern "C" int dm3_gemv_status(uint32_t* status, void* stream) {
  if (!status) return dm3::set_error("null pointer argument"), 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0, v_cc = 0;
  const uint32_t zero = 0;
  if (dm3::gemv_status_async(&v_cc, s) != 0 ||
      cudaMemcpyFromSymbolAsync(&v, dm3::gemv_tc::g_status, 4, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(dm3::gemv_tc::g_status, &zero, 4, 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return dm3::set_error("reading the GEMV status word failed"), 2;
  v |= v_cc;
  *status = v;
  return (v & dm3::STATUS_TIMEOUT) ? 3 : 0;
}
