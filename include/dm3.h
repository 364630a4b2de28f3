/*
 * drama3-b200 C ABI: the drop-in boundary for the Drama-3 per-frame MoE feed-forward and the
 * block-FP8 GEMV, built for NVIDIA B200 (sm_100a).
 *
 * Every entry point takes raw device pointers, explicit sizes and strides, and a cudaStream_t
 * passed as `void*` (0 = legacy default stream). Nothing here allocates device memory except
 * where the caller hands in a workspace. All calls are asynchronous on the given stream and
 * contain no host synchronisation (dm3_moe_status excepted), so they can be captured into CUDA
 * graphs. The return value is DM3_OK or one of the DM3_E* codes below; dm3_last_error() gives a
 * one-line reason.
 *
 * Dtypes: activations and outputs bf16 (uint16 storage), weights float8_e4m3fn (uint8 storage),
 * scales fp32, expert ids int64, routing weights bf16.
 *
 * Scale layout ("srows"): an e4m3 weight [R, C] carries one fp32 scale per (srows x 128) block,
 * stored row-major as [ceil(R / srows), C / 128]. srows = 128 is the 128x128 block layout of
 * engine.fp8_block (engine.py:214-219, release/convert_weights.py:14-15); srows = 1 is the
 * per-row 1x128 layout of fp8_linear.quantize (fp8_linear.py:30-34). Dequantised weight =
 * float(q) * scale.
 */
#ifndef DM3_H
#define DM3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DM3_OK 0
#define DM3_EINVAL 1   /* bad argument (shape, stride, alignment, null pointer) */
#define DM3_ECUDA 2    /* a CUDA runtime call failed */
#define DM3_ETIMEOUT 3 /* reported by dm3_moe_status: a device-side bounded wait ran out */
#define DM3_ENOSPACE 4 /* workspace too small */

/* Scale-table layouts accepted by every weight operand. */
#define DM3_SCALE_1x128 1
#define DM3_SCALE_128x128 128

/* Router weight dtypes. */
#define DM3_ROUTER_F32 0
#define DM3_ROUTER_BF16 1

/* One-line description of the last error on the calling host thread ("" if none). */
const char* dm3_last_error(void);

/* Library version, e.g. "0.1.0". */
const char* dm3_version(void);

/*
 * Block-FP8 GEMV: y[m, n] = sum_k x[m, k] * float(q[n, k]) * s[n / srows, k / 128] (+ bias[n]),
 * fp32 accumulation, for M <= 4 activation rows.
 * Replaces the Triton `_gemv` kernel behind FP8Linear.forward for rows <= 2
 * (fp8_linear.py:10-27, :56-59) and the restricted audio-head projection (engine.py:423).
 *   x     bf16 [M, K], row stride K elements
 *   q     e4m3 [N, K], row stride ldq bytes (ldq >= K, ldq % 16 == 0, 16-byte aligned base)
 *   s     fp32 [ceil(N / srows), K / 128], row stride lds floats
 *   bias  optional [N] (bias_kind 0 none, 1 bf16, 2 fp32)
 *   y     [M, N] row stride ldy elements; y_fp32 = 0 writes bf16, 1 writes fp32
 * K % 128 == 0, K <= 8192, 1 <= M <= 4.
 */
int dm3_fp8_gemv(const void* x, int M, int K, int N, const void* q, int64_t ldq, const float* s, int64_t lds,
                 int srows, const void* bias, int bias_kind, void* y, int64_t ldy, int y_fp32, void* stream);

/*
 * Reads and clears the sticky status word of the tensor-core GEMV on the current device
 * (synchronises the stream): bit 0 = a bounded wait ran out in some launch since the last read.
 * Returns DM3_ETIMEOUT in that case, DM3_OK otherwise. The reference has no counterpart.
 */
int dm3_gemv_status(uint32_t* status, void* stream);

/*
 * Gathered block-FP8 GEMV: as dm3_fp8_gemv, but output row n reads weight row rows[n] of q
 * (and its scale row rows[n] / srows). Covers the audio head restricted to the eos token plus
 * the semantic band, `lm_head.weight[candidates]` (engine.py:409-411), without materialising
 * the gathered copy. rows: int64 [N] on the device, each in [0, n_rows_q).
 */
int dm3_fp8_gemv_gather(const void* x, int M, int K, int N, const void* q, int64_t ldq, int64_t n_rows_q,
                        const int64_t* rows, const float* s, int64_t lds, int srows, void* y, int64_t ldy,
                        int y_fp32, void* stream);

/* Workspace bytes of dm3_audio_head for Nc candidate rows. */
size_t dm3_audio_head_workspace_bytes(int Nc);

/*
 * The audio head of one CFG decode frame (engine.py:423-424, head of engine.py:409-410): the
 * block-FP8 GEMV logits[2, Nc] = hidden[2, K] @ head[Nc, K]^T (fp32, rounded to bf16 first when
 * round_bf16, the dtype the reference's bf16 head or FP8Linear returns), then
 * vocab[cols[j]] = l1[j] + strength * (l0[j] - l1[j]) with the reference's three fp32 roundings
 * (index_copy into the -inf buffer; entries outside cols are not touched), and lse[r] =
 * log-sum-exp of row r for direction_score. Two launches instead of a GEMV and about five
 * elementwise kernels, no vocabulary-wide allocation.
 *   x         bf16 [2, K] (row 0 conditional, row 1 unconditional)
 *   q, s      e4m3 head [Nc, K] (rows == null) or the full matrix [n_rows_q, K] with rows int64 [Nc]
 *             choosing the candidates; scale layout srows as dm3_fp8_gemv
 *   strength  device fp32 scalar (CfgGraphs keeps it as a device tensor)
 *   cols      device int64 [Nc]: vocabulary column of each candidate (the candidates tensor)
 *   vocab     fp32 [V], filled with -inf once by the caller
 *   logits    fp32 [2, Nc] out; lse fp32 [2] out
 *   workspace dm3_audio_head_workspace_bytes(Nc), zero-filled once, 256-byte aligned
 */
int dm3_audio_head(const void* x, int K, const void* q, int64_t ldq, const float* s, int64_t lds, int srows,
                   const int64_t* rows, int64_t n_rows_q, int Nc, const float* strength, const int64_t* cols,
                   float* vocab, int64_t V, float* logits, float* lse, int round_bf16, void* workspace,
                   size_t workspace_bytes, void* stream);

/*
 * direction_score (engine.py:476-479) accumulated on the device: *score += (logits[0, i] - lse[0])
 * - (logits[1, i] - lse[1]) with i = 0 when *token == eos_id, else *token - semantic_begin + 1;
 * logits / lse as dm3_audio_head wrote them, token a device int64 (the sampled frame's first code).
 */
int dm3_direction_score(const float* logits, const float* lse, int Nc, const int64_t* token, int64_t eos_id,
                        int64_t semantic_begin, float* score, void* stream);

/* Workspace bytes of dm3_fp8_gemm for M activation rows of K elements. */
size_t dm3_fp8_gemm_workspace_bytes(int M, int K);

/*
 * Block-FP8 GEMM for any number of activation rows: y[m, n] = sum_k x[m, k] * float(q[n, k]) *
 * s[n / srows, k / 128] (+ bias[n]) on the tensor cores, products exact and each 128-wide k block
 * scaled in fp32. Replaces FP8Linear.forward's path for more than 2 rows, which dequantises the
 * weight and calls F.linear (fp8_linear.py:60-61), as the prompt-reading chunks run it
 * (engine.py:283-288). Arguments as dm3_fp8_gemv, plus:
 *   M          1 <= M <= 2^20; K % 128 == 0, K <= 65536
 *   workspace  dm3_fp8_gemm_workspace_bytes(M, K) bytes, 256-byte aligned, zero-filled once before
 *              its first use (only its status word must start at zero; dm3_moe_status reads it);
 *              calls on one stream may share it
 */
int dm3_fp8_gemm(const void* x, int M, int K, int N, const void* q, int64_t ldq, const float* s, int64_t lds,
                 int srows, const void* bias, int bias_kind, void* y, int64_t ldy, int y_fp32, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * Workspace bytes needed by dm3_moe_forward / dm3_moe_layer for hidden H and expert intermediate
 * I (sized for the maximum of 4 rows, so T is ignored). The workspace must be zero-filled once
 * before its first use; every call leaves its counters at zero again, so it can be reused by
 * later calls on the same stream (calls that overlap on the GPU must not share one workspace).
 */
size_t dm3_moe_workspace_bytes(int T, int H, int I);

/*
 * Grouped SwiGLU over block-FP8 experts with routing given by the caller:
 *   y[t] = sum_j weights[t, j] * W2[e] ( silu(W1[e] x[t]) * W3[e] x[t] ),  e = ids[t, j]
 * where W13[e] = [gate (rows 0..I-1); up (rows I..2I-1)] is [2I, H] e4m3 and W2[e] is [H, I]
 * e4m3, each with its block scales; the SwiGLU activation is rounded to bf16 before the down
 * projection and y is written as bf16. Replaces fish-speech `fp8_moe_forward(x, ids, w, w13,
 * s13, w2, s2)` as called by OnDemandExperts.forward (engine.py:147) and Speaker.__call__
 * (engine.py:236). This fused decode kernel covers T <= 4 rows.
 *   x        bf16 [T, H]
 *   ids      int64 [T, top_k] expert indices into dim 0 of w13/w2 (an ExpertStore slot or a
 *            speaker expert); an id outside [0, n_experts) is skipped and flagged in the status
 *   weights  bf16 [T, top_k]
 *   w13      e4m3, expert e at w13 + e * w13_stride bytes, rows of H bytes
 *   s13      fp32, expert e at s13 + e * s13_stride floats, layout [2I / srows, H / 128]
 *   w2       e4m3, expert e at w2 + e * w2_stride bytes, rows of I bytes
 *   s2       fp32, expert e at s2 + e * s2_stride floats, layout [H / srows, I / 128]
 * ExpertStore slots (engine.py:32-34) have w13_stride = w2_stride = 3 * I * H.
 * H % 128 == 0, H <= 2048, I % 128 == 0, I <= 512, top_k <= 8.
 */
int dm3_moe_forward(const void* x, int T, int H, int I, const int64_t* ids, const void* weights, int top_k,
                    int n_experts, const void* w13, int64_t w13_stride, const float* s13, int64_t s13_stride,
                    const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride, int srows, void* y,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused decode MoE layer in one launch: router + top-k + grouped SwiGLU + shared expert +
 * combine. Covers Speaker.__call__ (engine.py:232-237: fp32 router over the distilled experts,
 * softmax, top-k, renormalise, bf16 weights, fp8_moe_forward, + bias) and speaker_forward
 * (engine.py:153-158: + sigmoid(shared_expert_gate(x)) * shared_expert(x)), and the same
 * block with the full bf16 router (the routed SparseMoeBlock decode row).
 *   router_w      [n_router, H], fp32 (router_dtype DM3_ROUTER_F32) or bf16
 *   logits_bf16   1: logits are rounded to bf16 before softmax (a bf16 nn.Linear router);
 *                 0: fp32 logits (the speaker's x.float() @ gate.T)
 *   logit_bias    optional fp32 [n_router] added to the logits before softmax
 *   experts       as dm3_moe_forward, n_experts = n_router
 *   sh_w13/sh_s13/sh_w2/sh_s2  optional shared expert (null sh_w13 = none), e4m3 with scale
 *                 layout sh_srows; sh_gate optional bf16 [H] (null: gate coefficient 1)
 *   out_bias      optional fp32 [H] added before the final bf16 rounding (the speaker bias)
 *   ids_out       optional int64 [T, top_k]: chosen experts, descending probability
 *   w_out         optional bf16 [T, top_k]: renormalised routing weights
 * Logits are accumulated exactly (fp64) and rounded once, so the chosen experts do not depend
 * on summation order; ties are broken towards the lower expert index.
 * n_router <= 256, top_k <= 8, T * top_k <= 32, other limits as dm3_moe_forward.
 */
int dm3_moe_layer(const void* x, int T, int H, int I, const void* router_w, int router_dtype, int n_router,
                  int top_k, int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride,
                  const float* s13, int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2,
                  int64_t s2_stride, int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2,
                  const float* sh_s2, int sh_srows, const void* sh_gate, const float* out_bias, void* y,
                  int64_t* ids_out, void* w_out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Reads and clears the sticky device status word of a MoE workspace (synchronises the
 * stream). *status receives the STATUS bits (0 = every bounded wait completed and every
 * expert id was valid; bit 0 = a wait timed out; bit 1 = an expert id was out of range).
 * Returns DM3_ETIMEOUT if a wait ran out, DM3_OK otherwise.
 */
int dm3_moe_status(void* workspace, uint32_t* status, void* stream);

/*
 * dm3_moe_layer without a workspace argument, for callers that cannot allocate device memory:
 * code running inside another runtime's memory pool, plugin hosts that only hand out their own
 * buffers, or paths where cudaMalloc is not allowed. It has no counterpart in the reference.
 * Arguments and results are those of dm3_moe_layer. The scratch is a 1.5 MiB array compiled
 * into the library, held by every GPU that loads it until the process exits; it holds the layer
 * of H <= 2048 and I <= 512, and larger H or I is rejected with DM3_ENOSPACE. The first call on a
 * device looks up the array's address and zeroes it, waiting for the clear before it returns, so
 * make that first call before any stream capture. All calls share the one array and each call
 * leaves it ready for the next, so calls that overlap on the GPU race. After a device-side
 * failure read dm3_moe_noalloc_status, which also clears the array. Allocates nothing.
 */
int dm3_moe_layer_noalloc(const void* x, int T, int H, int I, const void* router_w, int router_dtype, int n_router,
                          int top_k, int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride,
                          const float* s13, int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2,
                          int64_t s2_stride, int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2,
                          const float* sh_s2, int sh_srows, const void* sh_gate, const float* out_bias, void* y,
                          int64_t* ids_out, void* w_out, void* stream);

/*
 * The status word of the allocation-free layer's static scratch on the current device, as
 * dm3_moe_status reports it for a workspace (synchronises the stream). A call that stopped at a
 * bounded wait may leave counters and partial sums in the scratch, so when the word is non-zero
 * the whole array is zeroed before this returns; the next dm3_moe_layer_noalloc is then correct
 * again. It has no counterpart in the reference.
 */
int dm3_moe_noalloc_status(uint32_t* status, void* stream);

/*
 * Time limit of every bounded device-side wait (spins on flags, counters and mbarriers) on the
 * current device, in nanoseconds; 1 s by default. A wait that runs out sets STATUS_TIMEOUT in the
 * status word and the kernel stops its work uniformly. Call while no kernel of this library runs
 * on the device. The reference has no device-side waits; this exists for failure detection.
 */
int dm3_set_wait_limit_ns(uint64_t ns);

/*
 * Workspace bytes of dm3_moe_prefill / dm3_moe_grouped for T tokens, hidden H, intermediate I,
 * n_experts routed experts and top_k. Allocate it zero-filled once; every call rewrites what it
 * reads, so it can be reused by later calls on the same stream with the same or smaller sizes.
 */
size_t dm3_moe_prefill_workspace_bytes(int T, int H, int I, int n_experts, int top_k);

/*
 * Prompt-reading (prefill) MoE layer for T tokens, the routed path of SparseMoeBlock.forward
 * that speaker_forward falls back to when more rows than OnDemandExperts.batch arrive
 * (engine.py:153-157): a bf16 router over n_router experts (+ optional fp32 logit bias) with
 * softmax, top-k and renormalisation to bf16 (exp1_routing.py:59-60, engine.py:233-235), the
 * token-to-expert dispatch that OnDemandExperts.forward prepares with ids.unique() / slot_map
 * (engine.py:143-146), the grouped block-FP8 SwiGLU of fp8_moe_forward (engine.py:147), the
 * weighted combine and the sigmoid-gated shared expert (engine.py:158), and an optional fp32 bias.
 * Arguments as dm3_moe_layer (router_w bf16 [n_router, H], experts with their dim-0 strides), plus:
 *   perm_out     optional int64 [T * top_k]: the (token, k) pairs (index t * top_k + j) in dispatch
 *                order, i.e. stably sorted by expert (argsort(ids.flatten(), stable=True))
 *   offsets_out  optional int64 [n_router + 1]: first dispatch position of each expert
 * Router logits are those of exact sums rounded once (fp32, then bf16 for logits_bf16), so the
 * chosen experts match an exact reference; ties go to the lower expert index.
 * 1 <= T, H % 256 == 0, H <= 2048, I % 128 == 0, I <= 512, top_k <= n_router <= 256, top_k <= 8.
 */
int dm3_moe_prefill(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                    int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride, const float* s13,
                    int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride,
                    int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                    int sh_srows, const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out, void* w_out,
                    int64_t* perm_out, int64_t* offsets_out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * fp8_moe_forward(x, ids, weights, w13, s13, w2, s2) for any row count (engine.py:147, :236): the
 * dispatch, grouped SwiGLU and combine of dm3_moe_prefill with the caller's routing. Arguments as
 * dm3_moe_forward plus perm_out / offsets_out as dm3_moe_prefill; the workspace is
 * dm3_moe_prefill_workspace_bytes(T, H, I, n_experts, top_k). Out-of-range ids are skipped and
 * flagged in the status word (dm3_moe_status).
 */
int dm3_moe_grouped(const void* x, int T, int H, int I, const int64_t* ids, const void* weights, int top_k,
                    int n_experts, const void* w13, int64_t w13_stride, const float* s13, int64_t s13_stride,
                    const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride, int srows, void* y,
                    int64_t* perm_out, int64_t* offsets_out, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes of dm3_route for T tokens, hidden H, n_router experts and top_k. */
size_t dm3_route_workspace_bytes(int T, int H, int n_router, int top_k);

/*
 * The router alone for T tokens: logits = x @ router_w.T (bf16 [n_router, H], exact sums rounded
 * once; rounded to bf16 for logits_bf16) + optional fp32 logit_bias, softmax, top-k, renormalised
 * bf16 weights (exp1_routing.py:59-60, engine.py:233-235). ids_out int64 [T, top_k] in descending
 * probability, w_out bf16 [T, top_k]. Limits as dm3_moe_prefill.
 */
int dm3_route(const void* x, int T, int H, const void* router_w, int n_router, int top_k, int logits_bf16,
              const float* logit_bias, int64_t* ids_out, void* w_out, void* workspace, size_t workspace_bytes,
              void* stream);

/*
 * Expert-parallel prefill over `world` ranks (one process per GPU, 2 <= world <= 8): rank r owns
 * the experts [r * n_router / world, (r + 1) * n_router / world) and routes its own T <= tokens_per_rank
 * tokens over all n_router experts. Each rank allocates one arena (dm3_ep_alloc of
 * dm3_ep_arena_bytes), exports it (dm3_ep_ipc_handle, 64 bytes), and opens every other rank's handle
 * (dm3_ep_ipc_open); `arenas` is the host array of the world arena pointers as mapped in this
 * process (arenas[rank] its own). Pairs travel to their owner and output rows back over NVLink peer
 * stores from inside the kernels, with flags carrying a per-call epoch (bounded waits; a wait that
 * runs out sets the status word). Every rank must make the same sequence of calls.
 * These calls carry the token-to-expert dispatch of OnDemandExperts.forward (engine.py:138-147)
 * across GPUs.
 */
size_t dm3_ep_arena_bytes(int world, int tokens_per_rank, int top_k, int H);
int dm3_ep_alloc(size_t bytes, void** ptr);
int dm3_ep_free(void* ptr);
int dm3_ep_ipc_handle(void* ptr, void* handle_out);
int dm3_ep_ipc_open(const void* handle, void** ptr);
int dm3_ep_ipc_close(void* ptr);
size_t dm3_moe_prefill_ep_workspace_bytes(int world, int tokens_per_rank, int H, int I, int n_router, int top_k);

/*
 * The prefill layer of dm3_moe_prefill under expert parallelism: x, y, ids_out, w_out are this
 * rank's T tokens; w13 / s13 / w2 / s2 hold this rank's n_router / world experts (local index
 * order); the router weight, logit bias and shared expert are replicated. The result equals
 * dm3_moe_prefill on the concatenated tokens. owner: optional int32 [n_router] on the device,
 * (rank << 16) | local index of every expert, for a placement other than contiguous blocks (it
 * must give every rank n_router / world experts, and each rank's w13 / w2 must follow it); null
 * places expert e on rank e / (n_router / world).
 */
int dm3_moe_prefill_ep(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                       int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride, const float* s13,
                       int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2, int64_t s2_stride,
                       int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2, const float* sh_s2,
                       int sh_srows, const void* sh_gate, const float* out_bias, void* y, int64_t* ids_out, void* w_out,
                       int world, int rank, int tokens_per_rank, void* const* arenas, const int* owner,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * The two halves of dm3_moe_prefill_ep. dm3_ep_dispatch routes this rank's tokens and sends every
 * (token, k) pair's exact e4m3 hi / lo rows to the rank owning its expert. dm3_ep_combine takes
 * the pairs every rank sent here into expert tiles, runs this rank's experts, sends each output row
 * back to its source rank, and combines this rank's tokens (+ shared expert, + bias). Call them in
 * this order on the same stream with the same workspace; sh_gate must be given to both or neither.
 * owner as dm3_moe_prefill_ep (dm3_ep_combine takes this rank's experts in that placement).
 */
int dm3_ep_dispatch(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                    int logits_bf16, const float* logit_bias, const void* sh_gate, int64_t* ids_out, void* w_out,
                    int world, int rank, int tokens_per_rank, void* const* arenas, const int* owner, void* workspace,
                    size_t workspace_bytes, void* stream);
int dm3_ep_combine(const void* x, int T, int H, int I, const void* router_w, int n_router, int top_k,
                   const void* w13, int64_t w13_stride, const float* s13, int64_t s13_stride, const void* w2,
                   int64_t w2_stride, const float* s2, int64_t s2_stride, int srows, const void* sh_w13,
                   const float* sh_s13, const void* sh_w2, const float* sh_s2, int sh_srows, const void* sh_gate,
                   const float* out_bias, void* y, int world, int rank, int tokens_per_rank, void* const* arenas,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * dm3_moe_layer sharded over `world` ranks (2 <= world <= 8, one process per GPU): every rank holds
 * the same rows x and router and computes the same routing; rank r runs only its n_router / world
 * experts (w13 / s13 / w2 / s2 hold them, in local index order: expert e is local index
 * e - r * n_router / world) and rank 0 the shared expert; the partial sums meet in a one-shot
 * all-reduce over the expert-parallel arenas (stored over NVLink into every rank's arena, epoch
 * flags, bounded waits), after which every rank holds the full layer output y. arenas and
 * tokens_per_rank as dm3_moe_prefill_ep (one arena serves both paths). Other arguments and limits
 * as dm3_moe_layer; every rank must make the same sequence of calls.
 */
int dm3_moe_layer_ep(const void* x, int T, int H, int I, const void* router_w, int router_dtype, int n_router,
                     int top_k, int logits_bf16, const float* logit_bias, const void* w13, int64_t w13_stride,
                     const float* s13, int64_t s13_stride, const void* w2, int64_t w2_stride, const float* s2,
                     int64_t s2_stride, int srows, const void* sh_w13, const float* sh_s13, const void* sh_w2,
                     const float* sh_s2, int sh_srows, const void* sh_gate, const float* out_bias, void* y,
                     int64_t* ids_out, void* w_out, int world, int rank, int tokens_per_rank, void* const* arenas,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Number of kernels the last MoE / GEMV entry point launched on this host thread. */
int dm3_last_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* DM3_H */
