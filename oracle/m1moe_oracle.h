/*
 * m1moe_oracle.h — CPU restatement of M1MoE's int4 expert-FFN arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the m1moe_b200 product links, loads or
 * calls this code.  It is the parity checker for the CUDA path (tests/,
 * __graft_entry__.smoke()) and the timed CPU baseline (bench.py's
 * cpu_baseline leg and `--impl reference`).
 *
 * Parity pin: the weight format, the nibble order and the dequant rule
 * w = q*scale + bias are pinned against the reference's own Python quantiser
 * (scripts/extract_olmoe.py:116-159, run end to end through its extract()
 * to produce tests/golden fixtures).  The kernel arithmetic (64-lane strided
 * partial sums, the FMA rearrangement, the tree reduction, SwiGLU, combine,
 * router softmax and top-K) is restated from the reference's Metal and Swift
 * sources, which cannot execute here (no Metal stack, no Swift toolchain);
 * for those steps parity is pinned by source semantics only.
 *
 * All sizes are element counts unless named *_bytes.
 */
#ifndef M1MOE_ORACLE_H
#define M1MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Shaders.metal:11-14 (bf16_to_f32) and InferenceEngine.swift:603-606. */
float orc_bf16_to_f32(uint16_t b);
/* scripts/extract_olmoe.py:104-111 (f32_to_bf16: round to nearest even). */
uint16_t orc_f32_to_bf16(float f);

/* ModelSpec.swift:36-52 (expertBytes4Bit) / extract_olmoe.py:162-169. */
size_t orc_expert_bytes(int hidden, int inter, int gs);
/* InferenceEngine.swift:79-97: byte offsets of
 * gateW, gateS, gateB, upW, upS, upB, downW, downS, downB in one expert block. */
void orc_expert_offsets(int hidden, int inter, int gs, size_t off[9]);

/* Shaders.metal:39-92 (matvec4bit), rows [row0,row1) of y = W x.
 * W uint32[out][in/8], S/B bf16[out][in/gs], x f32[in], y f32[out].
 * Emulates the 64-thread threadgroup: lane lid sums words lid, lid+64, ...
 * with acc = fma(nibble, scale*x, fma(bias, x, acc)), then the shared-memory
 * tree reduction s = 32, 16, ..., 1. */
void orc_matvec4bit_rows(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                         const float *x, float *y, int out_dim, int in_dim, int gs,
                         int row0, int row1);
/* The same rows with the 64 lanes innermost (vectorisable), bit-identical to
 * orc_matvec4bit_rows; orc_matvec4bit and orc_matvec4bit_mt use it. */
void orc_matvec4bit_rows_lanes(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                               const float *x, float *y, int out_dim, int in_dim, int gs,
                               int row0, int row1);
void orc_matvec4bit(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                    const float *x, float *y, int out_dim, int in_dim, int gs);

/* Shaders.metal:138-149: act = g / (1 + exp(-g)) * up. */
void orc_swiglu(const float *gate, const float *up, float *act, int n);

/* Shaders.metal:360-376: out[i] = residual[i] + sum_{k=0..K-1} w[k]*E[k*h+i]. */
void orc_moe_combine(const float *expert_outs, const float *w, const float *residual,
                     float *out, int K, int h);

/* InferenceEngine.swift:490-508: scores[e] = sum_d W[e,d]*x[d] (d ascending,
 * W upcast from bf16 exactly as at :99-113), then max-subtracted softmax with
 * expf and multiplication by 1/sum. */
void orc_router_scores(const uint16_t *router_bf16, const float *x, int E, int h,
                       float *scores);

/* InferenceEngine.swift:510-519: sort descending, keep K, renormalise over the
 * kept K when norm != 0.  The reference's sort is not stable; this restatement
 * breaks ties by the lower expert index. */
void orc_select_topk(const float *scores, int E, int K, int norm, int32_t *idx, float *w);

/* InferenceEngine.swift:401-444 for one expert block:
 * gate = W_g x, up = W_u x, act = swiGLU(gate, up), y = W_d act.
 * scratch holds 3*inter floats. */
void orc_expert_forward(const uint8_t *block, const float *x, int hidden, int inter,
                        int gs, float *y, float *scratch);

/* The MoE part of InferenceEngine.runLayer (:240-266) for B tokens:
 * router -> top-K -> K expert forwards -> combine with the residual.
 * table: E expert blocks of expert_bytes each (one layer_NN.bin image).
 * h_mid, residual, out: f32[B][hidden].  idx/w: [B][K].
 * nthreads > 1 splits every matvec's rows over that many threads. */
int orc_moe_layer(const uint8_t *table, const uint16_t *router_bf16, const float *h_mid,
                  const float *residual, float *out, int B, int hidden, int inter, int E,
                  int K, int gs, int norm, int32_t *idx, float *w, int nthreads);

/* Multi-threaded matvec for the CPU baseline: rows split over nthreads of a
 * persistent thread pool (threads are created once per process). */
void orc_matvec4bit_mt(const uint32_t *W, const uint16_t *S, const uint16_t *B,
                       const float *x, float *y, int out_dim, int in_dim, int gs,
                       int nthreads);

/* ---- the dense half of a decode step ---- */

/* Shaders.metal:97-134: 256-lane sum of squares with tree reduction, then
 * y = x * (1/sqrt(ss/dim + eps)) * w. */
void orc_rmsnorm(const float *x, const uint16_t *w, float eps, float *y, int dim);

/* Shaders.metal:328-353 (matvecBF16): y = W x, bf16 W [out][in], f32 x;
 * 64 lanes strided over `in`, tree reduction; rows over nthreads threads. */
void orc_matvec_bf16(const uint16_t *W, const float *x, float *y, int out_dim, int in_dim,
                     int nthreads);

/* InferenceEngine.swift:538-548 (per-head RMSNorm, first head_dim weights). */
void orc_head_rmsnorm(float *buf, int num_heads, int head_dim, const uint16_t *w, float eps);

/* InferenceEngine.swift:521-536 (RoPE, half-split pairs). */
void orc_rope(float *buf, int num_heads, int head_dim, float theta, int pos);

/* Shaders.metal:209-313 for one sequence over positions [0, seq_len) of a
 * bf16 cache laid out [num_kv_heads][max_seq][head_dim]; out [num_heads*hd]. */
void orc_attention(const float *q, const uint16_t *kc, const uint16_t *vc, int num_heads,
                   int num_kv_heads, int head_dim, int max_seq, int seq_len, float *out);

/* InferenceEngine.swift:552-555: index of the first maximum. */
int orc_argmax(const float *logits, int n);

#ifdef __cplusplus
}
#endif
#endif
