/*
 * m1moe_cuda.h — C ABI of the B200 (sm_100a) int4 expert-FFN library.
 *
 * This is the drop-in boundary for M1MoE's MoE block.  In the reference the
 * block is private Swift in InferenceEngine (Sources/M1MoE/InferenceEngine.swift
 * :240-266 router + expert load + CMD3, :401-478 encoders, :490-519 router)
 * driving Metal pipelines built in MetalContext.swift:101-111 whose kernel ABI
 * is "buffer index + setBytes scalar" (Shaders.metal:29-51).  A SwiftPM C
 * module target exposing this header replaces those encoders one for one; the
 * comment on each entry point names the reference code it replaces.
 *
 * Conventions
 *  - Every entry point returns an m1moe_status (0 = success).  Nothing throws
 *    across the ABI and nothing calls exit().  m1moe_cuda_last_error() gives a
 *    thread-local message for the last failure on the calling thread.
 *  - Pointers named d_* are device pointers; h_* are host pointers.
 *  - `stream` is a cudaStream_t passed as void* (NULL = the legacy default
 *    stream).  Functions taking a stream are stream-ordered and do not
 *    synchronise; the *_host variants are synchronous like the reference's
 *    commitSync (InferenceEngine.swift:289-294).
 *  - Weights use the reference's on-disk format unchanged (scripts/
 *    extract_olmoe.py:20-38): per projection W uint32[rows][cols/8] with
 *    nibble b of word w = column 8w+b, then S and B as bf16[rows][cols/gs];
 *    dequant w = q*S + B.  One expert block is
 *    [gateW|gateS|gateB|upW|upS|upB|downW|downS|downB] (ModelSpec.swift:36-52).
 *  - Decode arithmetic (matvec and MoE block): activations are quantised to
 *    int16 per 32-column chunk of x (gate/up) or per group of SwiGLU
 *    activations (down), multiplied with the int4 nibbles by dp2a into
 *    int32 per chunk or group, and scaled in fp32 as s*s_x*Q + b*X (s, b the
 *    group's bf16 scale and bias, s_x the chunk's scale, X its exact fp32
 *    sum); sums over chunks, groups and experts are fp32.  Results agree with
 *    the reference's fp32 FMA loop within 1e-3 of the output's L2 norm.
 *    Activations may be passed as f32 or bf16 and outputs written as f32 or
 *    bf16.  The dense decode step (m1moe_dense_*) computes bf16 weights x
 *    f32 activations with fp32 FMA accumulation.
 */
#ifndef M1MOE_CUDA_H
#define M1MOE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define M1MOE_CUDA_ABI_VERSION 1

/* Exported symbols (the library is built with hidden default visibility). */
#if defined(__GNUC__)
#define M1MOE_API __attribute__((visibility("default")))
#else
#define M1MOE_API
#endif

typedef enum m1moe_status {
    M1MOE_OK = 0,
    M1MOE_ERR_INVALID_ARG = 1,   /* bad pointer, size, dtype or shape       */
    M1MOE_ERR_OUT_OF_MEMORY = 2, /* cudaMalloc / cudaHostAlloc failed        */
    M1MOE_ERR_CUDA = 3,          /* any other CUDA runtime error             */
    M1MOE_ERR_NOT_LOADED = 4,    /* layer weights or router not loaded yet   */
    M1MOE_ERR_DEVICE = 5,        /* a kernel raised the context's error word */
    M1MOE_ERR_UNSUPPORTED = 6    /* valid but unsupported shape (e.g. gs%32) */
} m1moe_status;

typedef enum m1moe_dtype {
    M1MOE_DTYPE_F32 = 0,
    M1MOE_DTYPE_BF16 = 1
} m1moe_dtype;

/* Dimensions of one MoE model; field meanings follow ModelSpec.swift
 * (hiddenDim, MoESpec.intermediateDim/numExperts/topK/normTopkProb,
 * QuantSpec.groupSize, numLayers).  hidden_dim is a multiple of 128,
 * intermediate_dim of 64, group_size a multiple of 32 dividing both. */
typedef struct m1moe_cuda_cfg {
    int32_t hidden_dim;
    int32_t intermediate_dim;
    int32_t num_experts;
    int32_t top_k;
    int32_t group_size;
    int32_t num_layers;
    int32_t norm_topk_prob;
    int32_t max_batch;     /* tokens per call, 1..8                              */
    int32_t device;        /* CUDA device ordinal                                */
    int32_t expert_begin;  /* expert-parallel shard: first expert held here      */
    int32_t expert_count;  /* experts held here; 0 = all num_experts             */
} m1moe_cuda_cfg;

typedef struct m1moe_cuda_ctx m1moe_cuda_ctx;

/* ABI version of the loaded library (M1MOE_CUDA_ABI_VERSION at build time). */
M1MOE_API int32_t m1moe_cuda_abi_version(void);

/* Thread-local message for the last failed call on this thread ("" if none). */
M1MOE_API const char *m1moe_cuda_last_error(void);

/* Bytes of one packed expert block.  Replaces ModelSpec.expertBytes4Bit
 * (ModelSpec.swift:36-52); 0 if the shape is invalid. */
M1MOE_API size_t m1moe_cuda_expert_bytes(int32_t hidden_dim, int32_t intermediate_dim,
                               int32_t group_size);

/* Create a context on cfg->device: allocates the HBM expert table for every
 * layer (the experts this shard holds), the router table and the per-call
 * scratch.  Replaces the expert-slot and MoE buffers of MetalContext.swift
 * :150-178 and the expert fds/offsets of InferenceEngine.init (:62-97). */
M1MOE_API m1moe_status m1moe_cuda_create(const m1moe_cuda_cfg *cfg, m1moe_cuda_ctx **out_ctx);

/* Free everything the context owns.  NULL is accepted. */
M1MOE_API m1moe_status m1moe_cuda_destroy(m1moe_cuda_ctx *ctx);

/* Fill one layer of the HBM expert table from the exact bytes of
 * packed_experts/layer_NN.bin (num_experts blocks back to back), copied through
 * pinned host staging.  Only this shard's experts are kept.  Replaces the
 * per-token pread of loadExpert (InferenceEngine.swift:271-280); the copy
 * happens once, at cold start.  nbytes must equal num_experts*expert_bytes. */
M1MOE_API m1moe_status m1moe_cuda_load_expert_layer(m1moe_cuda_ctx *ctx, int32_t layer,
                                          const void *h_layer_bytes, size_t nbytes);

/* Same as above from device memory (stream-ordered), for callers that already
 * hold the layer image in HBM. */
M1MOE_API m1moe_status m1moe_cuda_load_expert_layer_device(m1moe_cuda_ctx *ctx, int32_t layer,
                                                 const void *d_layer_bytes, size_t nbytes,
                                                 void *stream);

/* Load one layer's router (mlp.gate.weight / block_sparse_moe.gate.weight,
 * bf16 [num_experts][hidden_dim]).  Replaces the bf16->f32 router preconvert
 * of InferenceEngine.init (:99-113); the table stays bf16 in HBM and is
 * upcast exactly inside the kernel. */
M1MOE_API m1moe_status m1moe_cuda_load_router(m1moe_cuda_ctx *ctx, int32_t layer,
                                    const uint16_t *h_router_bf16, size_t count);

/* Stateless int4 group-quantised matvec for `batch` tokens (1..8):
 *   y[t][r] = sum_j (q[r][j]*S[r][j/gs] + B[r][j/gs]) * x[t][j]
 * x is [batch][in_dim] (x_dtype), y is [batch][out_dim] (y_dtype).
 * Replaces encode4BitMV + matvec4bit (InferenceEngine.swift:446-465,
 * Shaders.metal:39-92).  Requires in_dim % 64 == 0, gs % 32 == 0,
 * in_dim % gs == 0 and 16-byte-aligned d_w. */
M1MOE_API m1moe_status m1moe_cuda_matvec4(const uint32_t *d_w, const uint16_t *d_scales,
                                const uint16_t *d_biases, const void *d_x, int32_t x_dtype,
                                void *d_y, int32_t y_dtype, int32_t out_dim, int32_t in_dim,
                                int32_t group_size, int32_t batch, void *stream);

/* The same matvec over `num_mats` matrices that sit `mat_stride_bytes` apart
 * (e.g. the gate projection of every expert in a layer table), all applied to
 * the same x:  y[m][t][r].  The expert table's experts are such a strided set. */
M1MOE_API m1moe_status m1moe_cuda_matvec4_strided(const uint32_t *d_w, const uint16_t *d_scales,
                                        const uint16_t *d_biases, int64_t mat_stride_bytes,
                                        int32_t num_mats, const void *d_x, int32_t x_dtype,
                                        void *d_y, int32_t y_dtype, int32_t out_dim,
                                        int32_t in_dim, int32_t group_size, int32_t batch,
                                        void *stream);

/* Unpack nibbles to bytes: q[r][c] = (W[r][c/8] >> 4*(c%8)) & 0xF, the exact
 * unpack the matvec uses (Shaders.metal:73-74).  For bit-exact checks. */
M1MOE_API m1moe_status m1moe_cuda_unpack4(const uint32_t *d_w, uint8_t *d_q, int32_t rows,
                                int32_t cols, void *stream);

/* Router for `batch` tokens: scores = softmax(W_r x) and the top-K experts,
 * descending, ties to the lower index, renormalised if norm_topk_prob.
 * Replaces computeRouterScores + selectTopK (InferenceEngine.swift:490-519).
 * d_scores_out [batch][num_experts] may be NULL. */
M1MOE_API m1moe_status m1moe_cuda_router_topk(m1moe_cuda_ctx *ctx, int32_t layer, const void *d_x,
                                    int32_t x_dtype, int32_t batch, int32_t *d_topk_idx,
                                    float *d_topk_w, float *d_scores_out, void *stream);

/* Router top-K for callers that cannot allocate GPU memory (no counterpart in
 * the reference).  Bit-identical to m1moe_cuda_router_topk on the same router
 * and x (the same kernel variant per batch), but needs no context: the caller
 * passes the bf16 router [num_experts][hidden_dim] and x (16-byte aligned
 * device pointers) and the outputs; the kernel's scratch is a fixed
 * 49,152-byte array compiled into this library, present on every GPU that
 * loads it until the process exits.  It calls no cudaMalloc, cudaFree or
 * other allocating routine, for callers whose memory is allocated up front
 * or by someone else (a host runtime that owns the GPU heap, a plugin that
 * may not grow the process's footprint, code that runs where allocation is
 * not allowed).  Limits: num_experts <= 256, batch <= 8, top_k <= 16,
 * hidden_dim a multiple of 64 (any size: routing stages nothing in shared
 * memory that grows with it).
 * The first call on a device (with that device current) looks up and clears
 * the array and waits for the device; make it before any stream capture.
 * All calls on a device share the array: calls that overlap on the GPU race,
 * so issue them on one stream or otherwise one after another.  d_status
 * (int32 device word, required) is cleared on the stream and receives a
 * nonzero error bit if a bounded device wait gave up -- read it after the
 * stream to trust the outputs; NULL is rejected with M1MOE_ERR_INVALID_ARG.
 * d_topk_idx, d_topk_w ([batch][top_k]) and d_scores_out
 * ([batch][num_experts]) may be NULL. */
M1MOE_API m1moe_status m1moe_cuda_router_topk_noalloc(const uint16_t *d_router,
                                    int32_t num_experts, int32_t hidden_dim, int32_t top_k,
                                    int32_t norm_topk_prob, const void *d_x, int32_t x_dtype,
                                    int32_t batch, int32_t *d_topk_idx, float *d_topk_w,
                                    float *d_scores_out, int32_t *d_status, void *stream);

/* One MoE block for `batch` tokens (stream-ordered, device pointers):
 *   out[t] = residual[t] + sum_{k ascending} w[t][k] * Expert_{idx[t][k]}(x[t])
 * with Expert(x) = W_down (silu(W_gate x) * (W_up x)).  Replaces the MoE part of
 * runLayer (InferenceEngine.swift:240-266): router, loadExpert x K, CMD3
 * (encodeExpertForward x K, encodeMoECombine) and the copy-back.
 * d_residual may be NULL (treated as zero).  Expert-parallel shards sum only
 * the experts they hold; the caller reduces over shards.  d_topk_idx/d_topk_w
 * ([batch][top_k]) may be NULL. */
M1MOE_API m1moe_status m1moe_cuda_moe_layer(m1moe_cuda_ctx *ctx, int32_t layer, const void *d_x,
                                  int32_t x_dtype, const void *d_residual, int32_t res_dtype,
                                  void *d_out, int32_t out_dtype, int32_t batch,
                                  int32_t *d_topk_idx, float *d_topk_w, void *stream);

/* The same MoE block for `tokens` tokens at once (prefill, large batches) as
 * grouped int4 x bf16 GEMMs on the tensor cores (stream-ordered, device
 * pointers, the argument meanings of m1moe_cuda_moe_layer).  The reference
 * has no batched path: it runs runLayer token by token during prefill
 * (bench/main.swift:139-141, InferenceEngine.swift:240-266).  Weights,
 * tokens and SwiGLU activations enter the tensor cores as fp16 (fp32
 * accumulation), so results agree with m1moe_cuda_moe_layer within the FFN
 * tolerance, not bitwise; a value beyond the fp16 range (|v| > 65504) makes
 * the next m1moe_cuda_synchronize report M1MOE_ERR_DEVICE.  Needs group_size
 * 64 and intermediate_dim a multiple of 128.
 * Scratch for `tokens` is allocated on the first call that needs more
 * (synchronously, outside stream capture); out may alias x. */
M1MOE_API m1moe_status m1moe_cuda_moe_prefill(m1moe_cuda_ctx *ctx, int32_t layer, const void *d_x,
                                    int32_t x_dtype, const void *d_residual, int32_t res_dtype,
                                    void *d_out, int32_t out_dtype, int32_t tokens,
                                    int32_t *d_topk_idx, float *d_topk_w, void *stream);

/* Expert parallelism over NVLink peer memory (one process per GPU, all on one
 * node), the expert-parallel decode step: every rank owns tokens_per_rank
 * tokens and the experts of its shard (expert_begin/expert_count); one call
 * per layer gathers all ranks' tokens, applies the local experts and returns
 * each rank its own tokens' full MoE output, with no collective library in
 * between.  The reference runs on one GPU and has no counterpart; it is the
 * multi-GPU mode of runLayer's MoE part (InferenceEngine.swift:240-266).
 *
 * Setup, on every rank: m1moe_cuda_ep_region(ctx, world, tokens_per_rank,
 * handle) allocates this rank's exchange region and writes its 64-byte CUDA
 * IPC handle to `handle`; the caller gathers the handles of all ranks (any
 * host transport) into world x 64 bytes in rank order and calls
 * m1moe_cuda_ep_connect(ctx, rank, handles).  world * tokens_per_rank must
 * not exceed the context's max_batch; world is 2..8. */
M1MOE_API m1moe_status m1moe_cuda_ep_region(m1moe_cuda_ctx *ctx, int32_t world,
                                  int32_t tokens_per_rank, void *h_handle_out);
M1MOE_API m1moe_status m1moe_cuda_ep_connect(m1moe_cuda_ctx *ctx, int32_t rank,
                                   const void *h_handles);

/* One expert-parallel MoE step for this rank's tokens (stream-ordered):
 * d_x, d_residual and d_out hold this rank's tokens_per_rank tokens; out =
 * residual + sum over ALL ranks' experts.  Every rank must make the same
 * sequence of calls (a call waits, bounded, for the other ranks' inputs and
 * partial sums; a rank that stops calling makes the others time out with
 * M1MOE_ERR_DEVICE on m1moe_cuda_synchronize).  d_topk_idx/d_topk_w, if not
 * NULL, receive [world*tokens_per_rank][top_k] for all ranks' tokens in rank
 * order.  After an error the contexts of all ranks must be recreated. */
M1MOE_API m1moe_status m1moe_cuda_moe_layer_ep(m1moe_cuda_ctx *ctx, int32_t layer, const void *d_x,
                                     int32_t x_dtype, const void *d_residual,
                                     int32_t res_dtype, void *d_out, int32_t out_dtype,
                                     int32_t *d_topk_idx, float *d_topk_w, void *stream);

/* Synchronous host-buffer form of m1moe_cuda_moe_layer with the reference's
 * f32 buffers (buf_h_mid, buf_residual -> buf_moe_out, MetalContext.swift
 * :134-152): copies in, runs, copies out and waits.  h_topk_* may be NULL.
 * The copies go through one pinned buffer of the context, so calls on one
 * context must come from one thread at a time. */
M1MOE_API m1moe_status m1moe_cuda_moe_layer_host(m1moe_cuda_ctx *ctx, int32_t layer,
                                       const float *h_x, const float *h_residual,
                                       float *h_out, int32_t batch, int32_t *h_topk_idx,
                                       float *h_topk_w);

/* Wait for all work of the context and report (then clear) its device error
 * word: M1MOE_ERR_DEVICE if any kernel flagged an error since the last call. */
M1MOE_API m1moe_status m1moe_cuda_synchronize(m1moe_cuda_ctx *ctx);

/* Number of kernels this library has launched in the calling process. */
M1MOE_API int64_t m1moe_cuda_launch_count(void);

/* Phase tracing (the reference only has wall-clock timing, bench/main.swift
 * :51-54).  With a non-NULL device buffer of 160 x 24 uint64, every MoE call
 * made afterwards records, per CTA (first 160), the SM cycle counter at each
 * phase event (slots 0-13, 16-19, 22, 23) and the global nanosecond timer at
 * events 0 and 10 (slots 20 and 21); NULL turns tracing off (the default).
 * Events: 0 start, 1 output rows initialised, 2 this CTA's logits published,
 * 3 top-K ranked, 4 consumers released (routing and geometry known),
 * 5 first gate/up tile landed, 6 activations quantised, 7 every CTA's output
 * rows seen initialised, 8 down items done, 9 producer issued every tile,
 * 10 end, 11 producer issued its first tile, 12 every logit seen, 13 ranks
 * counted, 16 producer's geometry done, 17 gate/up items done, 18 first down
 * item started, 19 producer saw the routing, 22 first and 23 last down tile
 * seen landed.  Slots 14 and 15 hold values, not times: the CTA's gate/up
 * row range (first | end << 32) and its tile counts (gate/up | down << 32). */
M1MOE_API m1moe_status m1moe_cuda_set_trace(m1moe_cuda_ctx *ctx, uint64_t *d_trace);

#ifdef __cplusplus
}
#endif
#endif /* M1MOE_CUDA_H */
