// The audio head of one CFG decode frame (sm_100a), fused after its block-FP8 GEMV:
//
//   logits  = (hidden[2, K] @ head[Nc, K]^T).float()          engine.py:423 (head = lm_head rows of
//                                                             the eos token and the semantic band,
//                                                             engine.py:409-410)
//   guided  = vocab.index_copy(1, candidates, l1 + s * (l0 - l1))   engine.py:424
//   score  += log_softmax(logits)[0, i] - log_softmax(logits)[1, i]  engine.py:476-479, i the sampled
//                                                             token's column (direction_score)
//
// The reference runs this as a GEMV and about five elementwise kernels per frame and builds a new
// vocabulary-wide tensor for index_copy. Here the GEMV (tensor-core kernel for a contiguous head,
// the gathering kernel for a row list) is followed by one finishing kernel: every CTA rounds its
// columns of the logits to the head's output dtype (bf16, as the bf16 matmul or the FP8 GEMV
// returns), applies the guidance with the reference's three fp32 roundings (no fused multiply-add),
// scatters the guided values into the caller's vocabulary buffer (whose other entries keep the
// -inf it was filled with once), and leaves its per-row (max, sum exp) partial; the CTA that
// finishes last combines the partials into each row's log-sum-exp. direction_score, which needs
// the token sampled afterwards, is a one-warp kernel reading that token from device memory, so the
// whole frame stays capturable in a CUDA graph.
#include <cstdint>
#include <string>

#include "dm3.h"
#include "dm3_common.cuh"
#include "dm3_internal.h"

namespace dm3 {
namespace head {

constexpr int kThreads = 256;
constexpr int kColsPerThread = 4;
constexpr int kColsPerCta = kThreads * kColsPerThread;

struct Params {
  float* logits;           // [2][Nc] fp32, written by the GEMV; rounded in place when round_bf16
  int Nc;
  int round_bf16;
  const float* strength;   // device scalar
  const int64_t* cols;     // [Nc] vocabulary column of each candidate
  float* vocab;            // [V]
  int64_t V;
  float* lse;              // [2]
  float* part;             // [ctas][2][2] (max, sum exp) per row
  uint32_t* ctrl;          // ctrl[0]: CTAs that have left their partials (zero between calls)
};


__device__ __forceinline__ void warp_combine(float& m, float& s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
}

__global__ void __launch_bounds__(kThreads) finish_kernel(const __grid_constant__ Params p) {
  __shared__ float sm[2][kThreads / 32], ss[2][kThreads / 32];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = blockIdx.x * kColsPerCta;
  // the dependents (direction_score, then the next frame's GEMV, whose weight copies need no input)
  // may start now; each waits for its own predecessor before reading
  griddep_launch();
  griddep_wait();
  const float st = __ldg(p.strength);
  float l[2][kColsPerThread];
  float m[2] = {-INFINITY, -INFINITY}, s[2] = {0.f, 0.f};
#pragma unroll
  for (int j = 0; j < kColsPerThread; ++j) {
    const int c = c0 + j * kThreads + tid;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float v = c < p.Nc ? __ldcg(p.logits + static_cast<size_t>(r) * p.Nc + c) : -INFINITY;
      if (p.round_bf16 && c < p.Nc) v = bf16_round(v);
      l[r][j] = v;
      m[r] = fmaxf(m[r], v);
    }
  }
#pragma unroll
  for (int j = 0; j < kColsPerThread; ++j) {
    const int c = c0 + j * kThreads + tid;
    if (c < p.Nc) {
      if (p.round_bf16) {
        p.logits[c] = l[0][j];
        p.logits[static_cast<size_t>(p.Nc) + c] = l[1][j];
      }
      // l1 + s * (l0 - l1), each operation rounded to fp32 as torch evaluates it
      const float g = __fadd_rn(l[1][j], __fmul_rn(st, __fsub_rn(l[0][j], l[1][j])));
      const int64_t col = __ldg(p.cols + c);
      if (col >= 0 && col < p.V) p.vocab[col] = g;
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
#pragma unroll
    for (int j = 0; j < kColsPerThread; ++j)
      if (l[r][j] != -INFINITY) s[r] += __expf(l[r][j] - m[r]);
    warp_combine(m[r], s[r]);
    if (lane == 0) {
      sm[r][warp] = m[r];
      ss[r][warp] = s[r];
    }
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mm = lane < kThreads / 32 ? sm[r][lane] : -INFINITY, sv = lane < kThreads / 32 ? ss[r][lane] : 0.f;
      warp_combine(mm, sv);
      if (lane == 0) {
        p.part[blockIdx.x * 4 + 2 * r] = mm;
        p.part[blockIdx.x * 4 + 2 * r + 1] = sv;
      }
    }
    if (lane == 0) {
      __threadfence();
      s_last = atomicAdd(p.ctrl, 1u) == gridDim.x - 1 ? 1 : 0;
    }
  }
  __syncthreads();
  if (!s_last) return;
  // the last CTA: every partial is visible (each CTA fenced before counting)
  __threadfence();
  if (warp < 2) {
    const int r = warp;
    float mm = -INFINITY, sv = 0.f;
    for (int b = lane; b < static_cast<int>(gridDim.x); b += 32) {
      const float m2 = __ldcg(p.part + b * 4 + 2 * r), s2 = __ldcg(p.part + b * 4 + 2 * r + 1);
      const float mx = fmaxf(mm, m2);
      sv = (mm == -INFINITY ? 0.f : sv * __expf(mm - mx)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mx));
      mm = mx;
    }
    warp_combine(mm, sv);
    if (lane == 0) p.lse[r] = mm + __logf(sv);
  }
  if (tid == 0) p.ctrl[0] = 0u;  // ready for the next call
}

// score += (logits[0, i] - lse[0]) - (logits[1, i] - lse[1]), i = 0 for the eos token, else
// token - semantic_begin + 1 (direction_score, engine.py:476-479).
__global__ void score_kernel(const float* logits, const float* lse, int Nc, const int64_t* token, int64_t eos_id,
                             int64_t sem_begin, float* score) {
  griddep_launch();  // as in finish_kernel: the next frame's GEMV may stage its weights meanwhile
  griddep_wait();
  if (threadIdx.x != 0) return;
  const int64_t t = *token;
  int64_t i = t == eos_id ? 0 : t - sem_begin + 1;
  if (i < 0 || i >= Nc) i = 0;  // a token outside the head's band scores as column 0 (never for a sampled one)
  const float a = __fsub_rn(logits[i], lse[0]);
  const float b = __fsub_rn(logits[static_cast<size_t>(Nc) + i], lse[1]);
  *score = __fadd_rn(*score, __fsub_rn(a, b));
}

}  // namespace head
}  // namespace dm3

// ------------------------------------------------------------------ C ABI
extern "C" size_t dm3_audio_head_workspace_bytes(int Nc) {
  if (Nc < 1) return 0;
  const size_t ctas = (static_cast<size_t>(Nc) + dm3::head::kColsPerCta - 1) / dm3::head::kColsPerCta;
  return 256 + ctas * 16;
}

extern "C" int dm3_audio_head(const void* x, int K, const void* q, int64_t ldq, const float* s, int64_t lds,
                              int srows, const int64_t* rows, int64_t n_rows_q, int Nc, const float* strength,
                              const int64_t* cols, float* vocab, int64_t V, float* logits, float* lse, int round_bf16,
                              void* workspace, size_t workspace_bytes, void* stream) {
  using dm3::set_error;
  dm3::note_launches(0);
  if (Nc < 1 || !strength || !cols || !vocab || V < 1 || !logits || !lse || !workspace)
    return set_error("audio head: null pointer or empty size"), 1;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return set_error("workspace must be 256-byte aligned"), 1;
  if (workspace_bytes < dm3_audio_head_workspace_bytes(Nc)) return set_error("workspace too small"), 4;
  int rc;
  if (rows)
    rc = dm3_fp8_gemv_gather(x, 2, K, Nc, q, ldq, n_rows_q, rows, s, lds, srows, logits, Nc, 1, stream);
  else
    rc = dm3_fp8_gemv(x, 2, K, Nc, q, ldq, s, lds, srows, nullptr, 0, logits, Nc, 1, stream);
  if (rc) return rc;
  const int gemv_launches = dm3_last_launch_count();
  dm3::head::Params p{};
  p.logits = logits;
  p.Nc = Nc;
  p.round_bf16 = round_bf16;
  p.strength = strength;
  p.cols = cols;
  p.vocab = vocab;
  p.V = V;
  p.lse = lse;
  p.ctrl = static_cast<uint32_t*>(workspace);
  p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = dm3::pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((Nc + dm3::head::kColsPerCta - 1) / dm3::head::kColsPerCta);
  cfg.blockDim = dim3(dm3::head::kThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, dm3::head::finish_kernel, p);
  if (err != cudaSuccess) return set_error(std::string("audio head launch: ") + cudaGetErrorString(err)), 2;
  dm3::note_launches(gemv_launches + 1);
  return 0;
}

extern "C" int dm3_direction_score(const float* logits, const float* lse, int Nc, const int64_t* token,
                                   int64_t eos_id, int64_t semantic_begin, float* score, void* stream) {
  using dm3::set_error;
  dm3::note_launches(0);
  if (!logits || !lse || !token || !score || Nc < 1) return set_error("direction score: bad arguments"), 1;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = dm3::pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err =
      cudaLaunchKernelEx(&cfg, dm3::head::score_kernel, logits, lse, Nc, token, eos_id, semantic_begin, score);
  if (err != cudaSuccess) return set_error(std::string("direction score launch: ") + cudaGetErrorString(err)), 2;
  dm3::note_launches(1);
  return 0;
}
