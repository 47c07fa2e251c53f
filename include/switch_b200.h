/* switch_b200.h -- C-ABI of the B200 (sm_100a) matrix-multiply hot path of
 * pkia/switch-l4t-gpu.
 *
 * Two boundaries are provided.
 *
 * 1. Module images (the reference's own boundary).  libswitch_b200.so ships
 *    four cubins whose `extern "C" __global__` kernels keep the reference's
 *    names and parameter lists, so a reference host that does
 *    cuModuleLoadData + cuModuleGetFunction + cuLaunchKernel (void** params,
 *    its hard-coded grids) works unchanged with them:
 *      switch_gpu.cubin  sgemm_tiled, sgemm_tiled4, sgemm_opt, sgemm_naive,
 *                        membw_read4                 (switch_gpu.cu:5-152)
 *      gemv.cubin        gemv, gemv4, gemv_warp      (gpu-llm/kernels/gemv.cu)
 *      gpt2.cubin        gemv_warp, gemv_warp_b, gemv_multi, layernorm, gelu,
 *                        add_bias, add2, attn_scores, attn_softmax, attn_mix
 *                                                    (gpt2_kernels.cu:38-268)
 *      qwen.cubin        gemv_h, rmsnorm, rope, swiglu, attn_scores_gqa,
 *                        attn_softmax, attn_mix_gqa, add2
 *                                                    (qwen_kernels.cu:34-189)
 *    sb_module_image() returns them for hosts that load from memory.
 *
 * 2. Host entry points (below): the launches the reference's C hosts make,
 *    as plain C functions with device pointers, sizes and a CUstream
 *    (passed as void*; NULL = the legacy default stream).  They use the
 *    CUDA driver API on the calling thread's current context; when none is
 *    current, device 0's primary context is retained and made current (the
 *    context the CUDA runtime, NCCL and PyTorch also use).
 *
 * Errors: every function returns 0 on success, else a nonzero CUresult (or
 * SB_ERR_* below) and records a message for sb_last_error().  Nothing
 * exits the process (the reference hosts' CHK macro does; cuda_drv.h:39-40).
 * Kernels never allocate; the caller owns every buffer, as in the reference.
 */
#ifndef SWITCH_B200_H
#define SWITCH_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_ERR_ARG 9001    /* invalid argument (size, alignment, null)    */
#define SB_ERR_FILE 9002   /* weight file missing or of the wrong size    */
#define SB_ERR_STATE 9003  /* engine not ready / misuse                   */

/* ---- runtime ------------------------------------------------------------ */
/* Make a context current (device `device`'s primary context if none is) and
 * load the module images into it.  Called implicitly by every entry point. */
int sb_init(int device);
/* Message of the last failure on this thread ("" if none). */
const char *sb_last_error(void);
/* Embedded module image by name ("switch_gpu", "gemv", "gpt2", "qwen"):
 * pointer/size of the sm_100a cubin, for cuModuleLoadData. */
int sb_module_image(const char *name, const void **image, size_t *size);
/* SM count of the current device. */
int sb_sm_count(void);

/* ---- SGEMM (replaces the launches of gpu_workload.c:90,135,142,160,168,186)
 * C[M][N] = A[M][K] . B[K][N], FP32 row-major, FP32 FFMA on CUDA cores.
 * Any M, N, K >= 0; 128-bit loads when K, N % 4 == 0 and pointers aligned.
 * Products with fewer 128x128 tiles than two per SM (M, N % 128 == 0,
 * aligned) split K over CTAs through a library-owned workspace and add the
 * partial tiles in split order (deterministic); split-K calls on different
 * streams of one context must not overlap. */
int sb_sgemm(const float *A, const float *B, float *C, int M, int N, int K, void *stream);
/* Rows [row0, row1) of C only: the row panel a rank computes when C is
 * sharded across GPUs (A, C point at the full matrices). */
int sb_sgemm_rows(const float *A, const float *B, float *C, int M, int N, int K, int row0, int row1,
                  void *stream);

/* The same CUDA-core SGEMM with its operand tiles staged by TMA
 * (cp.async.bulk.tensor into a 4-stage shared-memory ring, persistent CTAs,
 * a producer warp and eight compute warps): bit-identical to a one-CTA-
 * per-tile launch of sb_sgemm's kernel (each output one fma chain over k in
 * order).  With fewer 128 x 128 tiles than SMs (M, N % 128 == 0, K % 32 ==
 * 0) it runs stream-K -- each tile's k-slices split over CTAs, the pieces
 * added in CTA order through the context's workspace (deterministic, not
 * bit-identical to the single chain); sb_sgemm / sb_sgemm_rows take this
 * path for such products.  K % 4 == 0, N % 4 == 0, 16-byte aligned
 * pointers; any M, N.  No counterpart in the reference. */
int sb_sgemm_tma(const float *A, const float *B, float *C, int M, int N, int K, void *stream);

/* C[d] = A . B for d < nc (nc <= SB_SGEMM_MAX_DST): every finished 128 x 128
 * tile is stored into each output -- this device's memory or a peer's,
 * mapped into this process (sb_ipc_open or peer access) -- by the kernel
 * that computed it, so a row-panel product lands in every rank's C over
 * NVLink while the other tiles are still being multiplied, with no
 * separate all-gather.  Plain stores (no TMA); the kernel ends with a
 * system-scope fence, and the caller orders the peers' readers after it (a
 * collective or an event on their streams).  M, N % 128 == 0, K % 16 == 0,
 * 16-byte aligned pointers.  The same arithmetic as sb_sgemm's one-CTA-per-
 * tile kernel: every output one fma chain over k in order.  No counterpart
 * in the reference, which has no multi-GPU path. */
#define SB_SGEMM_MAX_DST 8
int sb_sgemm_multi(const float *A, const float *B, float *const *C, int nc, int M, int N, int K, void *stream);

/* Device memory shared with the other processes of one node (CUDA IPC):
 * sb_ipc_export writes the 64-byte handle of the allocation that holds
 * `ptr` and ptr's offset in it; sb_ipc_open maps a handle another process
 * exported into this process's current context and returns its base +
 * offset; sb_ipc_close unmaps it (pass the pointer and offset sb_ipc_open
 * took).  The exporting process must keep the memory allocated until every
 * importer has closed it.  No counterpart in the reference. */
int sb_ipc_export(const void *ptr, void *handle64, size_t *offset);
int sb_ipc_open(const void *handle64, size_t offset, void **ptr);
int sb_ipc_close(void *ptr, size_t offset);

/* ---- multi-GPU SGEMM (row panels + NCCL all-gather of C), one rank per GPU.
 * No counterpart in the reference, which runs on device 0 only
 * (gpu_workload.c:66-67).  NCCL is loaded at run time (libnccl.so.2).
 * Communicators are non-blocking: every wait polls ncclCommGetAsyncError
 * against `timeout_s` and aborts the communicator (ncclCommAbort) when a
 * peer never arrives or a collective never finishes, returning an error
 * instead of hanging.  Call them with the rank's device context current. */
/* A new NCCL unique id (ncclUniqueId, 128 bytes) for rank 0 to share. */
int sb_nccl_unique_id(void *id128);
/* ncclCommInitRankConfig (non-blocking) on the current context's device;
 * *comm receives the ncclComm_t. */
int sb_nccl_comm_init(void **comm, int world, const void *id128, int rank, double timeout_s);
/* Finalise and destroy (aborts on failure or timeout). */
int sb_nccl_comm_destroy(void *comm, double timeout_s);
int sb_nccl_abort(void *comm);
/* Rank `rank` of `world`: rows [rank R, min(M, rank R + R)) of C = A B
 * (R = ceil(M / world)) with sb_sgemm_rows, then -- when gather != 0 -- an
 * in-place ncclAllGather on `stream` so every rank holds all of C.  A and C
 * point at full-size matrices on this rank's device (only this rank's rows
 * of A are read); C must have room for world * R rows (the padding rows
 * past M are scratch).  Asynchronous: follow with sb_nccl_wait. */
int sb_sgemm_panel_allgather(const float *A, const float *B, float *C, int M, int N, int K, int rank, int world,
                             void *comm, int gather, void *stream);
/* Wait until `stream` is idle, watching `comm` (may be NULL) for errors;
 * on an error or after timeout_s the communicator is aborted. */
int sb_nccl_wait(void *comm, void *stream, double timeout_s);

/* ---- bandwidth probe (membw_read4, gpu_workload.c:197-220) ---------------
 * out[i] (i < min(n4, grid*block)) = sum of this thread's float4s, `iters`
 * passes over buf[n4]; grid = 0 picks 4 CTAs per SM. */
int sb_membw_read4(const void *buf, float *out, int n4, int iters, int grid, void *stream);
/* FP32 FMA probe: returns the FLOP count issued (grid*256*iters*256). */
int sb_fma_peak(float *out, int iters, int grid, void *stream, double *flops);

/* ---- GEMV ------------------------------------------------------------------
 * y[n] = sum_k W[n][k] x[k] (+ bias[n] if bias), W row-major [N][K].
 * FP32 weights: gemv / gemv4 / gemv_warp / gemv_warp_b (gemv.cu:3-71,
 * gpt2_kernels.cu:38-108).  K % 4 == 0.  Outputs shorter than 8 rows per
 * SM run split-K (K divided over a CTA's warps); longer ones stage x in
 * shared memory and need K <= 51200. */
int sb_gemv_f32(const float *W, const float *x, const float *bias, float *y, int K, int N, void *stream);
/* Y[t][n] = sum_k W[n][k] X[t][k] (+ bias[n]) for T token rows
 * (gemv_multi, gpt2_kernels.cu:115-155). */
int sb_gemv_multi_f32(const float *W, const float *X, const float *bias, float *Y, int K, int N, int T,
                      void *stream);
/* FP16 weights (raw IEEE half bits, exponent-0 values read as 0 as in the
 * reference's h2f), FP32 x, y, bias: gemv_h (qwen_kernels.cu:34-70).
 * K % 8 == 0.  Outputs shorter than 8 rows per SM run split-K; longer ones
 * stage x in shared memory and need K <= 51200. */
int sb_gemv_h(const uint16_t *W, const float *x, const float *bias, float *y, int K, int N, void *stream);
/* FP16 weights and FP16 activations, batch B in 1..8: Y[b][n] =
 * sum_k h2f(W[n][k]) h2f(X[b][k]), FP32 accumulate and output (the GEMV
 * sweep's y = W x with x FP16).  K % 8 == 0.  Outputs shorter than 8 rows
 * per SM run split-K (K divided over a CTA's warps). */
int sb_gemv_hh(const uint16_t *W, const uint16_t *X, float *Y, int K, int N, int B, void *stream);
/* The same product for B in 1..256 on the 5th-generation tensor cores
 * (tcgen05, TMA-fed, FP32 accumulation in tensor memory): the batched-decode
 * and prefill form of gemv_h.  fp16 subnormals are used as subnormals (the
 * tensor pipe does not flush them).  K % 8 == 0; W, X 16-byte aligned.
 * Short matrices are split along K through a library-owned workspace and
 * summed in split order, so results are deterministic; batches of up to 16
 * rows on short outputs (fewer than 16 rows per SM) run in one launch on
 * mma.sync tiles instead (fp16 in, FP32 accumulation, subnormals kept
 * likewise; K split over a CTA's warps, partials added in warp order).  No
 * counterpart in the reference (its prefill is gemv_multi,
 * gpt2_kernels.cu:115-155). */
int sb_gemm_hh(const uint16_t *W, const uint16_t *X, float *Y, int K, int N, int B, void *stream);
/* Opt-in SGEMM on the TF32 tensor pipe with the 3xTF32 split (big/small
 * parts of each operand, three products accumulated in FP32): the contract
 * of sb_sgemm (row-major C = A B) at FP32-level accuracy (relative Frobenius
 * error ~1e-6) and tensor-core speed.  K % 4 == 0, N % 4 == 0, 16-byte
 * aligned pointers.  No counterpart in the reference. */
int sb_sgemm_3xtf32(const float *A, const float *B, float *C, int M, int N, int K, void *stream);
/* The same product stored into every output C[d], d < nc <= SB_SGEMM_MAX_DST
 * (local or peer-mapped, as sb_sgemm_multi): each finished row of a tile
 * goes to all of them with plain stores, and the kernel ends with a
 * system-scope fence.  M, N % 128 == 0, K % 4 == 0, 16-byte aligned
 * pointers; no K split.  Bit-identical to sb_sgemm_3xtf32 whenever that
 * call runs without a K split (128 x 128 tiles at least as many as SMs).
 * No counterpart in the reference. */
int sb_sgemm_3xtf32_multi(const float *A, const float *B, float *const *C, int nc, int M, int N, int K,
                          void *stream);
/* The same product with the second operand given transposed: C = A Bt^T for
 * Bt [N][K] row-major (an [out][in] weight matrix), no transpose pass.  Same
 * alignment rules.  No counterpart in the reference. */
int sb_sgemm_nt_3xtf32(const float *A, const float *Bt, float *C, int M, int N, int K, void *stream);
/* Reads and clears the tensor-core kernels' device error flag (nonzero after
 * a bounded wait gave up); synchronises the context first. */
int sb_tc_error(int *err);
/* Failure-detection test hook (no counterpart in the reference): chunk >= 0
 * makes every later sb_gemm_hh launch's TMA producer stop before its K-chunk
 * `chunk` (64 k), so the MMA issuer's bounded wait for that stage runs out
 * (~2 s), the kernel drains what it issued, frees its tensor memory and
 * returns with the error flag set (sb_tc_error reports it); -1 turns it off.
 * Synchronises the context first. */
int sb_tc_set_test_skip(int chunk);

/* ---- decode-step pieces (Qwen2.5 FP16-weight path, qwen_engine.c:205-269)
 * Exposed for kernel-level parity tests; the engines below fuse them.      */
int sb_rmsnorm(const float *x, const uint16_t *w, float *y, int n, float eps, int rows, void *stream);
int sb_rope(float *x, const float *cosT, const float *sinT, int T, int H, int HD, int pos0, void *stream);
int sb_swiglu(const float *g, const float *u, float *y, int n, void *stream);
/* Decode attention of one query token over cached positions [0, T):
 * out[h*HD+d] = sum_t softmax_t(scale q_h.k_t) v_t[g*HD+d], g = h/(NH/NKV).
 * kc/vc rows have stride kv_stride floats.  HD must be 64, NH/NKV in {1,7}.
 * part: >= NKV*ceil(T/16)*(NH/NKV)*66 floats; counters: NKV zeroed uints
 * (left zeroed on return).  Replaces attn_scores_gqa/attn_softmax/
 * attn_mix_gqa (qwen_kernels.cu:130-180) and attn_scores/attn_softmax/
 * attn_mix (gpt2_kernels.cu:221-268). */
int sb_attn_decode(const float *q, const float *kc, const float *vc, float *out, int T, int NH, int NKV,
                   int HD, int kv_stride, float scale, float *part, unsigned *counters, void *stream);
/* The same decode attention for callers that cannot allocate device memory
 * (a fixed device budget sized at start-up, a host framework that owns every
 * allocation, an allocation-free token loop): the partials and tickets live
 * in a static array compiled into this library, at most T <= 2048 positions
 * and NH <= 16 heads (larger requests return SB_ERR_ARG).  The array exists
 * once per CUDA context (a device's primary context or one the host created);
 * the first call in a context resolves its address there (make it before any
 * stream capture begins); all calls in a context share the array, so calls
 * that overlap on the GPU race.
 * No counterpart in the reference, which has no scratch-using kernel. */
int sb_attn_decode_noalloc(const float *q, const float *kc, const float *vc, float *out, int T, int NH, int NKV,
                           int HD, int kv_stride, float scale, void *stream);
int sb_layernorm(const float *x, const float *w, const float *b, float *y, int n, float eps, int rows,
                 void *stream);
int sb_gelu(const float *x, float *y, int n, void *stream);

/* ---- engines ---------------------------------------------------------------
 * One process, one model, one GPU.  Weight files use the reference's exact
 * flat layouts (qwen_engine.c:8-16,60-75 / conv_qwen.py; gpt2_engine.c:10-13,
 * 50-70 / conv_gpt2.py).  The whole decode step runs on the device: token
 * embedding, all layers, final norm, LM head, argmax and the next-token
 * write, captured once as a CUDA graph and replayed per token. */
typedef struct sb_engine sb_engine;
#define SB_MODEL_QWEN 1
#define SB_MODEL_GPT2 2
#define SB_FLAG_NO_GRAPH 1u  /* launch kernels directly instead of graph replay */
#define SB_FLAG_NO_PDL 2u    /* no programmatic dependent launch            */
#define SB_FLAG_MULTI_KERNEL 4u /* one kernel per stage instead of the
                                 * persistent whole-step kernel (both models) */
#define SB_FLAG_NO_PREFILL 8u /* sb_engine_generate primes the prompt one token
                               * per step instead of sb_engine_prefill        */
#define SB_FLAG_MK_V1 16u     /* Qwen: the earlier persistent kernel (MLP down
                               * projection after a hand-off of the whole
                               * hidden vector) instead of the split-K one  */
#define SB_GEN_STOP_EOS 1u   /* stop at the model's end tokens (reference behaviour) */

/* max_ctx: KV-cache positions (<= 8192 Qwen, <= 1024 GPT-2). NULL on error. */
sb_engine *sb_engine_create(int model, const char *weights_path, int max_ctx, unsigned flags);
void sb_engine_destroy(sb_engine *e);
int sb_engine_reset(sb_engine *e); /* zero the KV cache */
/* One decode step with the reference's gpu_forward contract
 * (qwen_engine.c:205 / gpt2_engine.c:174): token at pos, cache gains pos;
 * when want_logits, the V logits are computed and, if logits_host != NULL,
 * copied there (synchronous). */
int sb_engine_forward(sb_engine *e, int token, int pos, int want_logits, float *logits_host);
/* Greedy generation: prompt ids from host memory, then n_gen+1 tokens are
 * produced exactly as the reference's prime-then-generate loop
 * (qwen_engine.c:523-548).  out_ids receives prompt + generated ids (room
 * for n_prompt+n_gen+1); returns the count in *n_out. */
int sb_engine_generate(sb_engine *e, const int *prompt, int n_prompt, int n_gen, int *out_ids, int *n_out,
                       unsigned gen_flags);
/* The same, split so a caller can time the phases on sb_engine_stream():
 * begin = upload prompt/state; steps = n graph replays (prefill steps use
 * with_logits=0); finish = synchronise and copy ids back. */
int sb_engine_begin(sb_engine *e, const int *prompt, int n_prompt, int n_gen, unsigned gen_flags);
int sb_engine_steps(sb_engine *e, int n, int with_logits);
/* Right after sb_engine_begin: the first n prompt tokens (n < n_prompt) run
 * through every layer together, filling the KV cache; the step position
 * becomes n.  Weight products are tensor-core GEMMs -- Qwen: fp16 GEMMs of
 * hi/lo fp16 activation rows (sb_gemm_hh); GPT-2: 3xTF32 GEMMs against the
 * FP32 weights (sb_sgemm_nt_3xtf32) -- and attention is causal per (token,
 * head).  The reference primes Qwen prompts one token at a time
 * (qwen_engine.c:529) and batches GPT-2's through gemv_multi (gpu_prefill,
 * gpt2_engine.c:269-326). */
int sb_engine_prefill(sb_engine *e, int n);
int sb_engine_finish(sb_engine *e, int *out_ids, int *n_out);
void *sb_engine_stream(sb_engine *e);
/* Device pointer of the logits buffer (V floats) and the vocabulary size. */
int sb_engine_logits(sb_engine *e, const float **dev_logits, int *vocab);
/* The engine's KV cache (the reference's kc / vc device buffers,
 * qwen_engine.c:83,180-181 and gpt2_engine.c:82,149-150, sized by max_ctx instead of
 * the file's CTX): FP32 [2][layers][max_ctx][width] -- keys for every layer,
 * then values -- with width 128 (Qwen, 2 KV heads x 64) or 768 (GPT-2).  A
 * host may read it, or write positions the next steps will attend to (a
 * cached prefix), between steps on sb_engine_stream(). */
int sb_engine_kv_cache(sb_engine *e, void **dev_kv, size_t *bytes, int *layers, int *max_ctx, int *width);
/* Kernel launches issued per decode step (with / without LM head). */
int sb_engine_launches_per_step(sb_engine *e, int with_logits);
/* 1 when the step runs as the persistent whole-step kernel (GPUs with >= 128
 * SMs: one cooperative launch per token, stages handed over through flagged
 * exchange words), 0 for one kernel per stage. */
int sb_engine_uses_persistent_kernel(sb_engine *e);
/* Name of the kernel that runs the decode step ("qwen_decode_mk2",
 * "qwen_decode_mk", "gpt2_decode_mk", or "<model> per-stage kernels"). */
const char *sb_engine_step_kernel(sb_engine *e);
/* Profiling aid for the persistent kernel: dev_buf (u64[SMs][256], or NULL
 * to stop) receives %globaltimer stamps per CTA: [cta][0] = kernel start,
 * [cta][1 + 2k] / [cta][2 + 2k] = inputs ready / outputs written of stage
 * k = layer * 5 + stage.  Graphs are re-captured on next use.  No
 * counterpart in the reference. */
int sb_engine_set_trace(sb_engine *e, void *dev_buf);
/* Failure-detection test hook for the persistent kernel (no counterpart in
 * the reference): cta >= 0 makes that CTA withhold its layer-0 outputs, so
 * every other CTA's bounded wait runs out (~1 s), the kernel returns early
 * and the step reports SB_ERR_STATE ("a wait inside the persistent kernel
 * timed out"); the engine clears its exchange words and stays usable.  -1
 * turns it off.  Graphs are re-captured on next use. */
int sb_engine_set_test_stall(sb_engine *e, int cta);
/* Bytes of weights a decode step streams (with LM head). */
double sb_engine_step_bytes(sb_engine *e);
/* Time `reps` standalone launches (CUDA events on the engine stream) of one
 * kernel of the step -- 1 QKV, 2 attention, 3 O-proj, 4 MLP up (gate|up or
 * fc), 5 MLP down, 6 LM head (layer 0 where it applies) -- each after an
 * optional streaming read of `flush` (a device buffer larger than L2; at
 * most 4*SMs*256 floats of the engine's logits buffer receive its sums) so
 * the weights come from HBM.  Reports the average ms and the kernel's algorithmic bytes. */
int sb_engine_profile(sb_engine *e, int which, int reps, void *flush, size_t flush_bytes, float *avg_ms,
                      double *bytes);

/* ---- token selection -------------------------------------------------------
 * Sampled next token with the reference Qwen engine's settings and step
 * order (qwen_engine.c:366-404; it passes temperature 0.7, top_k 20,
 * top_p 0.8, repetition penalty 1.1, xorshift state seeded 1234).  Given
 * the same logits, context and state it draws the same token.  top_k <= 64;
 * scratch (V floats) may be NULL.  Returns the id, or -1 on bad arguments. */
int sb_sample_token(const float *logits, int V, const int *ctx, int ctx_len, float temperature, int top_k,
                    float top_p, float rep_penalty, uint32_t *rng_state, float *scratch);
/* Steps 1-3 of that sampler on the GPU (device pointers): logits[V] FP32,
 * ctx[ctx_len] token ids.  Writes the top_k candidates -- ids and their
 * penalised, temperature-scaled values, ordered by value descending then
 * id ascending, which is the order of the reference's k first-index argmax
 * passes -- to idx_out / val_out (device).  Bit-identical to the host
 * steps (IEEE division and multiplication in the same order).  top_k in
 * 1..64, V <= 2^18, ceil(V / 1024) * top_k <= 16384; logits finite.  Uses the
 * context's workspace (calls on different streams must not overlap). */
int sb_topk_penalized(const float *logits, int V, const int *ctx, int ctx_len, float temperature, float rep_penalty,
                      int top_k, int *idx_out, float *val_out, void *stream);
/* Steps 4-6 on the host: softmax of the k candidate values (clamped exp),
 * top_p prefix, xorshift draw.  idx / val as sb_topk_penalized writes
 * them (host copies).  Returns the id, or -1 on bad arguments. */
int sb_sample_topk(const int *idx, const float *val, int top_k, float top_p, uint32_t *rng_state);
/* The engine's next token from its last step's logits (sb_engine_forward
 * with want_logits), the first ctx_len token ids it was fed as the
 * context: sb_topk_penalized on the device, 2 x top_k values copied back,
 * sb_sample_topk on the host -- the same token as sb_sample_token on the
 * full logits, without their 608 KB copy.  Returns the id or a negative
 * SB_ERR_* code. */
int sb_engine_sample(sb_engine *e, int ctx_len, float temperature, int top_k, float top_p, float rep_penalty,
                     uint32_t *rng_state);

/* ---- synthetic inputs in the reference layouts -----------------------------
 * Deterministic from `seed`: weights N(0, 0.02) (fp16 round-to-nearest for
 * Qwen), norm gains 1, LN betas 0, biases N(0, 0.02); Qwen RoPE tables
 * theta 1e6 as conv_qwen.py:75-80.  Returns bytes written. */
long sb_synth_weights(int model, const char *path, uint64_t seed);
/* n ids uniform in [0, vocab). */
void sb_synth_ids(int *ids, int n, int vocab, uint64_t seed);
/* n floats uniform in [lo, hi). */
void sb_synth_uniform(float *out, size_t n, float lo, float hi, uint64_t seed);
/* n fp16 values N(0, std), round-to-nearest-even. */
void sb_synth_normal_h(uint16_t *out, size_t n, float stdv, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
