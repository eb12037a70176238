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

/* Cold start from the converted model directory: every
 * <packed_experts_dir>/layer_NN.bin (NN = 00 .. num_layers-1) into the HBM
 * table, this shard's experts only.  All file sizes are checked first (each
 * must be num_experts * expert_bytes, the converter's check in
 * scripts/extract_olmoe.py:340-344); a missing or short file fails the call
 * with M1MOE_ERR_INVALID_ARG and names it, where the reference would zero the
 * expert and keep going (InferenceEngine.swift:274-279).  io_threads host
 * threads pread 32 MB chunks into a ring of pinned buffers while earlier
 * chunks are copied to the GPU and repacked, the concurrent-read shape of
 * ExpertCache.prefetch (ExpertCache.swift:126-196); synchronous. */
M1MOE_API m1moe_status m1moe_cuda_load_expert_files(m1moe_cuda_ctx *ctx, const char *packed_experts_dir,
                                          int32_t io_threads);

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

/* Single-process form of m1moe_cuda_ep_connect, for one process that drives
 * several GPUs (or, in tests, several contexts on one GPU): ctxs[r] is rank
 * r's context (ctxs[rank] == ctx), each with its exchange region already made
 * by m1moe_cuda_ep_region with the same world and tokens_per_rank; peer access
 * between different devices is enabled here. */
M1MOE_API m1moe_status m1moe_cuda_ep_connect_local(m1moe_cuda_ctx *ctx, int32_t rank,
                                         m1moe_cuda_ctx *const *ctxs);

/* How many polls an expert-parallel flag wait makes before it gives up, sets
 * the device error word and lets the call unwind (0 = the default, 2^22
 * polls with back-off, about a second).  A short limit lets failure drills
 * and tests see a missing rank within milliseconds. */
M1MOE_API m1moe_status m1moe_cuda_set_wait_limit(m1moe_cuda_ctx *ctx, uint32_t polls);

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
 * The copies go through one mapped pinned buffer of the context (kernels load
 * and store it; the calling thread polls a completion word there, and returns
 * M1MOE_ERR_DEVICE if the stream ends or a minute passes without it), so
 * calls on one context must come from one thread at a time. */
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
 * :51-54).  With a non-NULL device buffer of 160 x 32 uint64, every MoE call
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
 * seen landed; expert parallel calls add 24 this rank's tokens pushed (CTAs
 * 0..world-1), 25 every rank's tokens seen, 26 every CTA's sums seen (the
 * grid arrival), 27 this CTA's slices sent to the peers, 28 the peers'
 * slices of this rank's tokens seen.  Slots 14 and 15 hold values, not times: the CTA's gate/up
 * row range (first | end << 32) and its tile counts (gate/up | down << 32). */
M1MOE_API m1moe_status m1moe_cuda_set_trace(m1moe_cuda_ctx *ctx, uint64_t *d_trace);

/* ===================== the dense half of a decode step =====================
 * The reference runs the non-MoE part of a layer as two Metal command buffers
 * with CPU work between them (InferenceEngine.swift:167-238): CMD1 = input
 * RMSNorm + q/k/v matvecBF16 (Shaders.metal:97-134, :328-353), then on the CPU
 * QK-norm (OLMoE), RoPE and the KV store (:194-220, :521-548), then CMD2 =
 * attention scores/softmax/values, o_proj, residual add and the post-attention
 * RMSNorm (:222-238; Shaders.metal:153-163, :209-313); forward() ends with the
 * final RMSNorm, the LM head and greedy sampling (:140-155, :550-555).  The
 * entry points below replace those encoders and CPU steps; a dense context
 * owns the non-expert weights (WeightStore's mmap, WeightStore.swift:47-126),
 * the bf16 KV cache and the step buffers (MetalContext.swift:134-152). */

typedef struct m1moe_dense_cfg {
    int32_t hidden_dim;
    int32_t num_heads;      /* attention.numHeads                                  */
    int32_t num_kv_heads;   /* attention.numKvHeads (GQA when < num_heads)          */
    int32_t head_dim;       /* 128                                                 */
    int32_t num_layers;
    int32_t vocab_size;
    int32_t qk_norm;        /* per-head RMSNorm of q and k (architecture "olmoe")  */
    float rms_norm_eps;
    float rope_theta;
    int32_t max_batch;      /* sequences decoded together, 1..8                    */
    int32_t max_seq;        /* KV cache positions per sequence                    */
    int32_t device;
} m1moe_dense_cfg;

/* Tensor names of m1moe_cuda_dense_load (the reference's model_weights.json
 * keys, InferenceEngine.swift:577-598; bf16 in the model file). */
typedef enum m1moe_dense_tensor {
    M1MOE_W_EMBED = 0,       /* model.embed_tokens.weight [vocab][h]            */
    M1MOE_W_FINAL_NORM = 1,  /* model.norm.weight [h]                           */
    M1MOE_W_LM_HEAD = 2,     /* lm_head.weight [vocab][h]                       */
    M1MOE_W_INPUT_NORM = 3,  /* layers.L.input_layernorm.weight [h]             */
    M1MOE_W_POST_NORM = 4,   /* layers.L.post_attention_layernorm.weight [h]    */
    M1MOE_W_Q = 5,           /* layers.L.self_attn.q_proj.weight [nh*hd][h]     */
    M1MOE_W_K = 6,           /* layers.L.self_attn.k_proj.weight [nkv*hd][h]    */
    M1MOE_W_V = 7,           /* layers.L.self_attn.v_proj.weight [nkv*hd][h]    */
    M1MOE_W_O = 8,           /* layers.L.self_attn.o_proj.weight [h][nh*hd]     */
    M1MOE_W_Q_NORM = 9,      /* layers.L.self_attn.q_norm.weight [nh*hd] or [hd] */
    M1MOE_W_K_NORM = 10      /* layers.L.self_attn.k_norm.weight [nkv*hd] or [hd] */
} m1moe_dense_tensor;

typedef struct m1moe_dense_ctx m1moe_dense_ctx;

/* Create a dense context: weights, the bf16 KV cache [layers][max_batch]
 * [num_kv_heads][max_seq][head_dim] (zeroed), the step buffers and a device
 * position counter at 0.  Replaces MetalContext's dense buffers
 * (MetalContext.swift:134-152) and WeightStore's Metal buffer (:119-126). */
M1MOE_API m1moe_status m1moe_cuda_dense_create(const m1moe_dense_cfg *cfg, m1moe_dense_ctx **out_ctx);
M1MOE_API m1moe_status m1moe_cuda_dense_destroy(m1moe_dense_ctx *ctx);

/* Copy one bf16 tensor (host memory, e.g. WeightStore's mmap) into the
 * context; `layer` is ignored for the model-wide tensors.  QK-norm weights
 * may be given whole ([nh*hd] / [nkv*hd]) or as their first head_dim values:
 * the reference applies the first head_dim to every head
 * (InferenceEngine.swift:538-548). */
M1MOE_API m1moe_status m1moe_cuda_dense_load(m1moe_dense_ctx *ctx, int32_t tensor, int32_t layer,
                                   const uint16_t *h_bf16, size_t count);
/* The same from device memory (stream-ordered). */
M1MOE_API m1moe_status m1moe_cuda_dense_load_device(m1moe_dense_ctx *ctx, int32_t tensor, int32_t layer,
                                          const uint16_t *d_bf16, size_t count, void *stream);

/* Device pointers of one layer's K and V caches, bf16
 * [max_batch][num_kv_heads][max_seq][head_dim], for callers that prefill them. */
M1MOE_API m1moe_status m1moe_cuda_dense_kv_cache(m1moe_dense_ctx *ctx, int32_t layer, void **d_k,
                                       void **d_v);

/* The position of the next token (the reference's seqPos,
 * InferenceEngine.swift:23-24): set (synchronous), read (synchronous), and
 * reset() = zero the KV cache and the position (:159-163). */
M1MOE_API m1moe_status m1moe_cuda_dense_set_position(m1moe_dense_ctx *ctx, int32_t pos);
M1MOE_API m1moe_status m1moe_cuda_dense_get_position(m1moe_dense_ctx *ctx, int32_t *pos);
M1MOE_API m1moe_status m1moe_cuda_dense_reset(m1moe_dense_ctx *ctx);

/* Wait for the device and report (then clear) the dense context's error
 * word: M1MOE_ERR_DEVICE if a token id or the position was out of range. */
M1MOE_API m1moe_status m1moe_cuda_dense_synchronize(m1moe_dense_ctx *ctx);

/* y[t] = W . xn[t] (+ res[t]) for bf16 W [rows][in_dim] and `batch` tokens
 * (1..8), xn = x or, with d_norm_w, RMSNorm(x) * norm_w.  Replaces matvecBF16
 * (Shaders.metal:328-353), with the RMSNorm (:97-134) and residual add
 * (:153-163) fused.  in_dim a multiple of 256 (<= 8192); d_w and d_x 16-byte
 * aligned; d_res may alias d_y; y and res are f32 [batch][rows]. */
M1MOE_API m1moe_status m1moe_cuda_dense_gemv(const uint16_t *d_w, int32_t rows, int32_t in_dim,
                                   const void *d_x, int32_t x_dtype, const uint16_t *d_norm_w,
                                   float eps, const float *d_res, float *d_y, int32_t batch,
                                   void *stream);

/* y[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w (rmsNormSum + rmsNormApply,
 * Shaders.metal:97-134), f32 out, `batch` rows of `dim`. */
M1MOE_API m1moe_status m1moe_cuda_dense_rmsnorm(const void *d_x, int32_t x_dtype, const uint16_t *d_w,
                                      float eps, float *d_y, int32_t dim, int32_t batch,
                                      void *stream);

/* One layer's attention for `batch` sequences at the context's position:
 * from the q|k|v projections (f32 [batch][(nh + 2 nkv) * hd]) it applies the
 * QK-norm (if configured), RoPE, stores k and v (bf16) at the position and
 * attends over positions 0..pos (softmax(q.k / sqrt(hd)) . v, GQA groups of
 * nh / nkv heads), writing f32 [batch][nh * hd].  Replaces the CPU steps of
 * InferenceEngine.swift:194-220 and encodeAttention (:349-399,
 * Shaders.metal:209-313).  It does not advance the position. */
M1MOE_API m1moe_status m1moe_cuda_dense_attention(m1moe_dense_ctx *ctx, int32_t layer, const float *d_qkv,
                                        int32_t batch, float *d_out, void *stream);

/* Final RMSNorm + LM head + greedy sample (InferenceEngine.swift:140-155,
 * :550-555: the first maximum wins): d_tokens[t] = argmax_v logits[t][v].
 * d_logits (f32 [batch][vocab]) may be NULL. */
M1MOE_API m1moe_status m1moe_cuda_dense_lm_head(m1moe_dense_ctx *ctx, const float *d_x, int32_t batch,
                                      int32_t *d_tokens, float *d_logits, void *stream);

/* One whole decode step for `batch` sequences (stream-ordered, capturable in a
 * CUDA graph): embed d_tokens, then per layer the input RMSNorm + q/k/v,
 * QK-norm + RoPE + KV store + attention, o_proj + residual + post-attention
 * RMSNorm, and the MoE block of `moe` (m1moe_cuda_moe_layer on this layer);
 * then the final norm, the LM head and the greedy next tokens
 * (d_next_tokens [batch]; d_logits [batch][vocab] may be NULL), and the
 * device position advances by one.  Replaces InferenceEngine.forward
 * (:124-156) at temperature 0.  `moe` must have the same hidden size, layer
 * count and device, and max_batch >= batch. */
M1MOE_API m1moe_status m1moe_cuda_decode_step(m1moe_dense_ctx *ctx, m1moe_cuda_ctx *moe,
                                    const int32_t *d_tokens, int32_t batch, int32_t *d_next_tokens,
                                    float *d_logits, void *stream);

/* Token-parallel prefill of one sequence (sequence slot 0): the T prompt
 * tokens d_tokens [T] at positions pos .. pos+T-1 (pos = the context's
 * device position) go through every layer together -- embedding, input
 * RMSNorm and the q|k|v projection as one bf16 GEMM (cuBLAS, fp32
 * accumulation), QK-norm + RoPE + the KV store of all T positions, causal
 * attention, the o projection added to the residual, the post-attention
 * RMSNorm and the MoE block on the tensor cores (m1moe_cuda_moe_prefill) --
 * then the last token's final norm, LM head and greedy next token
 * (d_next_token [1]; d_logits [vocab] may be NULL); the position advances by
 * T.  The reference runs the prompt token by token through forward()
 * (bench/main.swift:139-141); this gives the same cache and next token
 * within the tolerance of its bf16/fp16 GEMM operands.  Buffers for T tokens
 * are allocated on the first call that needs them (synchronously). */
M1MOE_API m1moe_status m1moe_cuda_prefill_step(m1moe_dense_ctx *ctx, m1moe_cuda_ctx *moe,
                                     const int32_t *d_tokens, int32_t tokens,
                                     int32_t *d_next_token, float *d_logits, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* M1MOE_CUDA_H */
