// dense.cuh — the dense half of a decode step (sm_100a): BF16 GEMV with fused
// RMSNorm / residual / argmax, and decode attention over a BF16 KV cache with
// the QK-norm, RoPE and KV store fused in.
//
// Replaces the reference's per-layer CMD1/CMD2 Metal work and its CPU steps
// (InferenceEngine.swift:167-238, 521-548; Shaders.metal:97-134 rmsNorm,
// :153-163 residualAdd, :209-313 attention, :328-353 matvecBF16) and the LM
// head + greedy sampling of forward() (:141-155, :550-555).
//
// GEMV (k_dense_gemv).  y[t][r] = W[r] . xn[t] for bf16 W [rows][K] and up to 8
// tokens.  The reference gives every row a 64-thread threadgroup that walks
// the row (Shaders.metal:340-352), reading x again per row.  Here the K
// columns are split over the warps of a CTA, 256 per warp (8 bf16 = one
// 16-byte load per lane per row), so every lane keeps its 8 columns of x --
// RMS-normalised in the prologue when asked -- in registers for all rows,
// and a CTA walks a contiguous block of rows U at a time (U 16-byte weight
// loads in flight per lane; the first round is issued before waiting on the
// previous kernel, since weights do not depend on it).  Per round the lanes'
// U*NT partial dot products are reduced with one multi-value butterfly; per
// 64-row chunk the warps' partials are added in shared memory in warp order.
// Epilogues: store (+ residual, which may alias y); store + RMSNorm of the
// finished rows into a second buffer by the last CTA (the post-attention
// norm feeding the MoE block); argmax over the rows (the LM head's greedy
// sample, ties to the lower index), where the last CTA also writes the next
// step's embedding.  Accumulation is fp32 FMA on exact bf16->f32 upcasts.
//
// Attention (k_attn_decode).  One CTA per (token, KV head, position split):
// its q heads (the GQA group) are loaded, head-RMS-normalised (OLMoE's QK-norm,
// with the first head_dim weights as the reference does) and rotated (RoPE,
// half-split pairs, pos * theta^(-2i/hd)); the CTA whose split holds `pos`
// also normalises and rotates k and writes k and v, as bf16, into the cache.
// Four warps stream the split's K and V rows (8 positions per warp round, all
// loads in flight), score them (q.k * scale), and keep an online softmax
// (running max, sum and weighted V); the last CTA of a (token, KV head)
// merges the splits' partials into the attention output.  The position is
// read from device memory, so a captured step can be replayed while the
// position advances (the LM head's last CTA adds one).
#pragma once

#include <math.h>

#include "common.cuh"
#include "pipeline.cuh"

namespace m1 {

constexpr int kGemvColsPerWarp = 256;  // 32 lanes x 8 bf16
constexpr int kGemvChunkRows = 64;     // rows per shared-memory reduction round
constexpr int kGemvMaxWarps = 16;      // K <= 4096 (512 threads: up to 128 registers)
constexpr int kDenseMaxTok = 8;

enum GemvEpi { kEpiStore = 0, kEpiPostNorm = 1, kEpiArgmax = 2 };

struct GemvParams {
    const uint16_t *w;  // bf16 [rows][K]
    int rows, K;
    const void *x;      // [ntok][K], f32 or bf16
    int x_bf16;
    const uint16_t *norm_w;  // RMS-normalise x first with this bf16 [K] weight, or null
    float eps;
    float *y;           // [ntok][rows] f32 (argmax: may be null)
    const float *res;   // added to y, [ntok][rows] (may alias y), or null
    int ntok;
    // kEpiPostNorm: the last CTA writes post_out[t] = rmsnorm(y[t]) * post_w
    const uint16_t *post_w;
    float *post_out;
    float *ss_acc;      // [kDenseMaxTok] sums of squares of y (zero between calls)
    unsigned *done;     // CTAs finished (zero between calls)
    // kEpiArgmax: keys[t] = max over rows of {ordered logit, ~row}; the last
    // CTA writes tokens[t] and, with embed, embed_out[t] = embed[tokens[t]]
    unsigned long long *keys;  // [kDenseMaxTok] (zero between calls)
    int32_t *tokens;
    const uint16_t *embed;     // bf16 [vocab][embed_dim], or null
    float *embed_out;
    int embed_dim;
    int *pos;           // device position, advanced by pos_add by the argmax's last CTA (or null)
    int pos_add;
    int *err;           // device error word (a bounded ring wait gave up)
    // ring geometry (gemv_plan)
    int stage_rows, nstages, off_bars, off_part;
};

__device__ __forceinline__ float dot8_bf16(const uint4 w, const float (&x)[8], float acc) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc = fmaf(__uint_as_float(ws[i] << 16), x[2 * i], acc);
        acc = fmaf(__uint_as_float(ws[i] & 0xFFFF0000u), x[2 * i + 1], acc);
    }
    return acc;
}

// Ordered key of a logit for a max-reduction: larger value first, then the
// lower row (the reference's `if logits[i] > bestV` keeps the first maximum,
// InferenceEngine.swift:552-555); NaN lowest, -0 equal to +0.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
    uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    if (v != v) ord = 0u;
    return ((unsigned long long)ord << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)row);
}

// This lane's 8 columns of token t's x, as f32.
__device__ __forceinline__ void load_x8(const void *x, int x_bf16, size_t off, float (&v)[8]) {
    if (x_bf16) {
        const uint4 r = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + off);
        const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] = __uint_as_float(rr[j] << 16);
            v[2 * j + 1] = __uint_as_float(rr[j] & 0xFFFF0000u);
        }
    } else {
        const float4 *f = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + off);
        const float4 a = f[0], b = f[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

// Rows per round for NT tokens: U*NT values per warp reduction (<= 32).
template <int NT>
struct GemvRound {
    static constexpr int U = NT <= 4 ? 8 : 4;
};

// Shared-memory map of k_dense_gemv (host-planned, gemv_plan): the weight
// ring [nstages][stage_rows][K] bf16, its full/empty barriers, the warps'
// partials of one 64-row chunk [nw][kGemvChunkRows][NT] f32.
struct GemvPlan {
    int stage_rows, nstages, off_bars, off_part, smem;
};

__host__ __device__ inline GemvPlan gemv_plan(int K, int nt, int rows_per_cta, size_t smem_cap) {
    GemvPlan g{};
    const int nw = K / kGemvColsPerWarp;
    g.stage_rows = K <= 2048 ? 16 : 8;  // 64 KB stages
    const size_t stage = (size_t)g.stage_rows * K * 2;
    const size_t part = (size_t)nw * kGemvChunkRows * nt * 4;
    const int need = (rows_per_cta + g.stage_rows - 1) / g.stage_rows;
    int nst = (int)((smem_cap - part - 256) / stage);
    nst = nst < need ? nst : need;
    g.nstages = nst < 1 ? 1 : (nst > 4 ? 4 : nst);
    g.off_bars = (int)(g.nstages * stage);
    g.off_part = g.off_bars + 2 * 8 * 4;  // room for 4 full + 4 empty barriers
    g.smem = g.off_part + (int)part;
    return g;
}

// One CTA per SM: warps 0..nw-1 own 256 columns each (x in registers), warp
// nw is the producer.  The CTA's rows are one contiguous block of W, copied
// stage by stage into the ring with bulk copies; the first stages are
// requested before waiting on the previous kernel (weights are constants),
// so the whole block can be in flight while that kernel finishes.
template <int NT, int EPI>
__global__ void __launch_bounds__((kGemvMaxWarps + 1) * 32) k_dense_gemv(const GemvParams p) {
    constexpr int U = GemvRound<NT>::U, NV = U * NT, kS = 32 / NV;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[kGemvMaxWarps][NT];
    __shared__ unsigned long long kred[NT];
    __shared__ int is_last;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nw = (int)(blockDim.x >> 5) - 1, nct = nw * 32;  // consumer warps / threads
    const int G = gridDim.x, K = p.K, SR = p.stage_rows, NST = p.nstages;
    const size_t stage_bytes = (size_t)SR * K * 2;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.off_bars);
    uint64_t *empty = full + 4;
    float *part = reinterpret_cast<float *>(smem + p.off_part);
    const int r0 = (int)((long long)p.rows * blockIdx.x / G);
    const int r1 = (int)((long long)p.rows * (blockIdx.x + 1) / G);
    const int nstg = (r1 - r0 + SR - 1) / SR;  // stages of this CTA
    if (tid == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], nw);
        }
        abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_trigger();
    if (warp == nw) {
        // ================= producer =================
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int n = 0;
            for (; n < nstg; ++n) {
                const int s = n % NST;
                if (n >= NST && !mbar_wait(&empty[s], ((n / NST) - 1) & 1, &abort_flag, p.err)) break;
                const int rs = r0 + n * SR, nr = min(SR, r1 - rs);
                const uint32_t bytes = (uint32_t)nr * K * 2;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(ring + (size_t)s * stage_bytes, p.w + (size_t)rs * K, bytes, &full[s], pol);
            }
            // the last stages' copies land before this warp exits (a consumer
            // that gave up may not be waiting for them)
            volatile int never = 0;
            for (int m = n > NST ? n - NST : 0; m < n; ++m)
                mbar_wait(&full[m % NST], (m / NST) & 1, &never, nullptr);
        }
        return;
    }
    // ================= consumers =================
    pdl_wait();
    const int c0 = warp * kGemvColsPerWarp + lane * 8;
    float xr[NT][8];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if (t < p.ntok) {
            load_x8(p.x, p.x_bf16, (size_t)t * K + c0, xr[t]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) xr[t][j] = 0.f;
        }
    }
    if (p.norm_w) {
        // RMSNorm (Shaders.metal:97-134): x * rsqrt(mean(x^2) + eps) * w
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float s2 = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) s2 = fmaf(xr[t][j], xr[t][j], s2);
            s2 = warp_sum(s2);
            if (lane == 0) red[warp][t] = s2;
        }
        named_sync(1, nct);
        float nwv[8];
        {
            const uint4 r = *reinterpret_cast<const uint4 *>(p.norm_w + c0);
            const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                nwv[2 * j] = __uint_as_float(rr[j] << 16);
                nwv[2 * j + 1] = __uint_as_float(rr[j] & 0xFFFF0000u);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float ss = 0.f;
            for (int w = 0; w < nw; ++w) ss += red[w][t];
            const float rms = rsqrtf(ss / (float)K + p.eps);
#pragma unroll
            for (int j = 0; j < 8; ++j) xr[t][j] = (xr[t][j] * rms) * nwv[j];
        }
    }
    float ssl[NT];  // post-norm: sums of squares of this thread's outputs
    unsigned long long kmax[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        ssl[t] = 0.f;
        kmax[t] = 0ull;
    }
    bool ok = true;
    for (int cr = r0; cr < r1; cr += kGemvChunkRows) {
        const int ce = min(cr + kGemvChunkRows, r1);
        // the chunk's stages (SR divides the chunk's 64 rows)
        for (int rs = cr; ok && rs < ce; rs += SR) {
            const int n = (rs - r0) / SR, s = n % NST, nr = min(SR, r1 - rs);
            ok = mbar_wait(&full[s], (n / NST) & 1, &abort_flag, p.err);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const uint8_t *st = ring + (size_t)s * stage_bytes + (size_t)c0 * 2;
            for (int r = 0; r < nr; r += U) {
                float acc[NV];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const uint4 wv = (r + u < nr) ? *reinterpret_cast<const uint4 *>(st + (size_t)(r + u) * K * 2)
                                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int t = 0; t < NT; ++t) acc[u * NT + t] = dot8_bf16(wv, xr[t], 0.f);
                }
                const float tot = warp_reduce_multi(acc);
                if (lane % kS == 0) {
                    const int v = lane / kS, u = v / NT, t = v - u * NT;
                    if (r + u < nr)
                        part[((size_t)warp * kGemvChunkRows + (rs + r + u - cr)) * NT + t] = tot;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        named_sync(1, nct);
        if (abort_flag) break;
        const int nrow = ce - cr;
        for (int i = tid; i < nrow * NT; i += nct) {
            const int rr = i / NT, t = i - rr * NT, row = cr + rr;
            float v = 0.f;
            for (int w = 0; w < nw; ++w) v += part[((size_t)w * kGemvChunkRows + rr) * NT + t];
            if (t >= p.ntok) continue;
            const size_t o = (size_t)t * p.rows + row;
            if (p.res) v += p.res[o];
            if (p.y) p.y[o] = v;
            if constexpr (EPI == kEpiPostNorm) ssl[t] = fmaf(v, v, ssl[t]);
            if constexpr (EPI == kEpiArgmax) {
                const unsigned long long k = argmax_key(v, row);
                kmax[t] = k > kmax[t] ? k : kmax[t];
            }
        }
        named_sync(1, nct);
    }
    if (abort_flag) return;  // the producer drains its copies; the error word is set
    if constexpr (EPI == kEpiStore) return;
    // ---- the CTA's contribution, then the last CTA finishes the call ----
    if constexpr (EPI == kEpiPostNorm) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float s2 = warp_sum(ssl[t]);
            if (lane == 0) red[warp][t] = s2;
        }
        named_sync(1, nct);
        if (tid < p.ntok) {
            float s2 = 0.f;
            for (int w = 0; w < nw; ++w) s2 += red[w][tid];
            atomicAdd(p.ss_acc + tid, s2);
        }
    } else {
        if (tid < NT) kred[tid] = 0ull;
        named_sync(1, nct);
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (kmax[t]) atomicMax(&kred[t], kmax[t]);
        named_sync(1, nct);
        if (tid < p.ntok) atomicMax(p.keys + tid, kred[tid]);
    }
    named_sync(1, nct);
    if (tid == 0) {
        __threadfence();
        is_last = atomicAdd(p.done, 1u) == (unsigned)G - 1u;
    }
    named_sync(1, nct);
    if (!is_last) return;
    __threadfence();
    if constexpr (EPI == kEpiPostNorm) {
        __shared__ float rms_s[kDenseMaxTok];
        const int n = p.rows, total = p.ntok * n;
        if (tid < p.ntok) rms_s[tid] = rsqrtf(__ldcg(p.ss_acc + tid) / (float)n + p.eps);
        named_sync(1, nct);
        // eight independent loads in flight per thread and round (a loop of
        // dependent L2 round trips would dominate this tail)
        for (int base = tid; base < total; base += 8 * nct) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * nct;
                v[j] = i < total ? __ldcg(p.y + i) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * nct;
                if (i < total) {
                    const int t = i / n, c = i - t * n;
                    p.post_out[i] = (v[j] * rms_s[t]) * bf16_bits(p.post_w[c]);
                }
            }
        }
        named_sync(1, nct);
        if (tid < kDenseMaxTok) p.ss_acc[tid] = 0.f;
    } else {
        __shared__ int tok[kDenseMaxTok];
        if (tid < p.ntok) {
            const unsigned long long k = __ldcg(p.keys + tid);
            tok[tid] = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
            if (p.tokens) p.tokens[tid] = tok[tid];
        }
        named_sync(1, nct);
        if (p.embed)
            for (int i = tid; i < p.ntok * p.embed_dim; i += nct) {
                const int t = i / p.embed_dim, c = i - t * p.embed_dim;
                p.embed_out[i] = bf16_bits(p.embed[(size_t)tok[t] * p.embed_dim + c]);
            }
        named_sync(1, nct);
        if (tid < kDenseMaxTok) p.keys[tid] = 0ull;
        if (tid == 0 && p.pos) *p.pos += p.pos_add;
    }
    if (tid == 0) *p.done = 0u;
}

// ---------------------------------------------------------------- embed ----
// residual[t] = embed[token[t]] (InferenceEngine.swift:482-488); an id
// outside the vocabulary sets the error word and reads row 0.
__global__ void k_embed(const uint16_t *embed, const int32_t *tokens, int vocab, int h, float *out,
                        int ntok, int *err) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    if (t >= ntok) return;
    int tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && err) atomicOr(err, kErrBadIndex);
        tok = 0;
    }
    for (int i = threadIdx.x; i < h; i += blockDim.x)
        out[(size_t)t * h + i] = bf16_bits(embed[(size_t)tok * h + i]);
}

// ------------------------------------------------------------- rmsnorm ----
// y[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w, one CTA per token (the
// stand-alone form of the GEMV prologue; Shaders.metal:97-134).
__global__ void k_rmsnorm(const void *x, int x_bf16, const uint16_t *w, float eps, float *y, int dim) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t base = (size_t)t * dim;
    float s = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = load_act(x, x_bf16, base + i);
        s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float ss = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) ss += red[i];
    const float rms = rsqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        y[base + i] = (load_act(x, x_bf16, base + i) * rms) * bf16_bits(w[i]);
}

// ------------------------------------------------------------ attention ----
constexpr int kHeadDim = 128;   // dims per head (32 lanes x 4)
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnStage = 128;     // positions per shared-memory stage (K and V: 64 KB)
constexpr int kAttnMaxSplit = 128;  // position splits per (token, KV head)

struct AttnParams {
    const float *qkv;   // [ntok][qkv_stride]: q [nh*hd] | k [nkv*hd] | v [nkv*hd]
    int qkv_stride;
    int nh, nkv, ntok;
    const int *pos;     // device position of this step (the new token's index)
    int max_seq;
    const uint16_t *qn_w, *kn_w;  // QK-norm weights (bf16, first hd used), or null
    float eps, theta, scale;
    uint16_t *kc, *vc;  // this layer's caches, bf16 [max_batch][nkv][max_seq][hd]
    int nsplit;         // position splits (gridDim.x)
    float *part;        // [ntok][nh][nsplit][hd + 2]: unnormalised o, max, sum
    unsigned *cnt;      // [kDenseMaxTok][nkv] splits finished (zero between calls)
    float *out;         // [ntok][nh*hd]
    int *err;
};

// Per-head RMSNorm of a 128-dim head held 4 per lane (InferenceEngine.swift
// :538-548: the first hd weights of the norm apply to every head).
__device__ __forceinline__ void head_rmsnorm(float (&v)[4], const uint16_t *w, float eps) {
    const int lane = threadIdx.x & 31;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) s = fmaf(v[i], v[i], s);
    s = warp_sum(s);
    const float rms = 1.0f / sqrtf(s / (float)kHeadDim + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] *= rms * bf16_bits(w[4 * lane + i]);
}

// The rotation of pair i at position pos (InferenceEngine.swift:521-536):
// angle = pos * theta^(-2i/hd); rc/rs[i] = cos/sin of it, for the hd/2 pairs.
__device__ __forceinline__ void rope_table(float *rc, float *rs, int pos, float theta) {
    for (int i = threadIdx.x; i < kHeadDim / 2; i += blockDim.x) {
        const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)kHeadDim);
        const float ang = (float)pos * freq;
        rc[i] = cosf(ang);
        rs[i] = sinf(ang);
    }
}

// RoPE on a head held 4 per lane: pairs (i, i + hd/2) -- lanes l and l ^ 16
// -- rotate by the table's angle of pair i.
__device__ __forceinline__ void head_rope(float (&v)[4], const float *rc, const float *rs) {
    const int lane = threadIdx.x & 31;
    const bool lo = lane < 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float other = __shfl_xor_sync(0xffffffffu, v[i], 16);
        const int pair = 4 * (lane & 15) + i;
        const float c = rc[pair], s = rs[pair];
        // lo: x0' = x0 c - x1 s; hi: x1' = x0 s + x1 c
        v[i] = lo ? (v[i] * c - other * s) : (other * s + v[i] * c);
    }
}

__device__ __forceinline__ void load4(const float *p, float (&v)[4]) {
    const float4 a = *reinterpret_cast<const float4 *>(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}

__device__ __forceinline__ uint2 pack4_bf16(const float (&v)[4]) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 r;
    r.x = *reinterpret_cast<const uint32_t *>(&a);
    r.y = *reinterpret_cast<const uint32_t *>(&b);
    return r;
}

// Dynamic shared memory of k_attn_decode: two stages of K and V rows.
__host__ __device__ constexpr size_t attn_smem() {
    return 2 * 2 * (size_t)kAttnStage * kHeadDim * 2 + 64;
}

// HP: q heads per KV head (the GQA group size), 1..8.  One CTA per (split,
// KV head, token); about one CTA per SM in all.  Thread 0 bulk-copies the
// split's cached K and V rows (positions before `pos`) stage by stage into a
// two-stage shared-memory ring; 8 warps score 16 positions of a stage each
// from shared memory; the new token's own k and v (position `pos`) come from
// registers.
template <int HP>
__global__ void __launch_bounds__(kAttnThreads, 1) k_attn_decode(const AttnParams p) {
    constexpr int P = HP <= 4 ? 8 : 4;  // positions per warp round (P*HP <= 32)
    constexpr int NV = P * HP, kS = 32 / NV;
    constexpr int kPerWarp = kAttnStage / kAttnWarps;  // positions of a stage per warp
    extern __shared__ __align__(128) uint8_t smem[];
    const int split = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hd = kHeadDim;
    uint16_t *sk = reinterpret_cast<uint16_t *>(smem);                 // [2][kAttnStage][hd]
    uint16_t *sv = sk + 2 * (size_t)kAttnStage * hd;                    // [2][kAttnStage][hd]
    uint64_t *full = reinterpret_cast<uint64_t *>(sv + 2 * (size_t)kAttnStage * hd);
    __shared__ float sm_m[kAttnWarps][HP], sm_l[kAttnWarps][HP];
    __shared__ __align__(16) float sm_o[kAttnWarps][HP][kHeadDim];
    __shared__ int is_last, abort_flag;
    __shared__ float rope_c[kHeadDim / 2], rope_s[kHeadDim / 2];
    if (threadIdx.x == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        abort_flag = 0;
        mbar_fence_init();
    }
    pdl_trigger();
    {
        // warm L2 with this split's cached rows while the previous kernel
        // finishes: the position read here may be a step old, which only
        // makes the hint less exact (a prefetch consumes no data)
        const int pq = *reinterpret_cast<const volatile int *>(p.pos);
        if (threadIdx.x == 0 && pq > 0 && pq < p.max_seq) {
            const int sl = (pq + p.nsplit) / p.nsplit, a = min(pq, split * sl), e = min(pq, a + sl);
            if (e > a) {
                const size_t off = (((size_t)t * p.nkv + g) * p.max_seq + a) * kHeadDim;
                const uint32_t bytes = (uint32_t)(e - a) * kHeadDim * 2;
                bulk_prefetch_l2(p.kc + off, bytes);
                bulk_prefetch_l2(p.vc + off, bytes);
            }
        }
    }
    pdl_wait();
    // a position outside the cache sets the error word; the call then runs on
    // position 0 without storing, so that every CTA still takes part in the
    // split merge below (its output is not to be used)
    const int pos_in = *p.pos;
    const bool bad = pos_in < 0 || pos_in >= p.max_seq;
    if (bad && threadIdx.x == 0 && split == 0 && g == 0 && t == 0) atomicOr(p.err, kErrBadIndex);
    const int pos = bad ? 0 : pos_in;
    const int seq = pos + 1;
    const int qd = p.nh * hd, kvd = p.nkv * hd;
    const int slen = (seq + p.nsplit - 1) / p.nsplit;
    const int p0 = min(seq, split * slen), p1 = min(seq, p0 + slen);
    const int c1 = min(p1, pos);             // cached rows [p0, c1)
    const int nst = c1 > p0 ? (c1 - p0 + kAttnStage - 1) / kAttnStage : 0;
    const bool has_pos = p0 <= pos && pos < p1;
    const size_t slab = ((size_t)t * p.nkv + g) * p.max_seq * hd;
    uint16_t *kb = p.kc + slab, *vb = p.vc + slab;
    auto issue = [&](int j) {  // stage j -> buffer j & 1
        const int a = p0 + j * kAttnStage, n = min(kAttnStage, c1 - a);
        const uint32_t bytes = (uint32_t)n * hd * 2;
        const int b = j & 1;
        mbar_arrive_expect_tx(&full[b], 2 * bytes);
        bulk_g2s(sk + (size_t)b * kAttnStage * hd, kb + (size_t)a * hd, bytes, &full[b], 0ull);
        bulk_g2s(sv + (size_t)b * kAttnStage * hd, vb + (size_t)a * hd, bytes, &full[b], 0ull);
    };
    int issued = 0;  // stages issued (thread 0's count)
    rope_table(rope_c, rope_s, pos, p.theta);
    __syncthreads();  // barriers initialised, rotation table written
    if (threadIdx.x == 0)
        for (; issued < nst && issued < 2; ++issued) issue(issued);
    const float *qt = p.qkv + (size_t)t * p.qkv_stride;
    float q[HP][4];
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
        load4(qt + (size_t)(g * HP + hh) * hd + 4 * lane, q[hh]);
        if (p.qn_w) head_rmsnorm(q[hh], p.qn_w, p.eps);
        head_rope(q[hh], rope_c, rope_s);
    }
    float kp[4], vp[4];  // the new token's k and v (warp 0 of the split holding pos)
    if (warp == 0 && has_pos) {
        load4(qt + qd + (size_t)g * hd + 4 * lane, kp);
        load4(qt + qd + kvd + (size_t)g * hd + 4 * lane, vp);
        if (p.kn_w) head_rmsnorm(kp, p.kn_w, p.eps);
        head_rope(kp, rope_c, rope_s);
        // the cache keeps them as bf16; this step uses the same rounded values
        const uint2 kq = pack4_bf16(kp), vq = pack4_bf16(vp);
        if (!bad) {
            *reinterpret_cast<uint2 *>(kb + (size_t)pos * hd + 4 * lane) = kq;
            *reinterpret_cast<uint2 *>(vb + (size_t)pos * hd + 4 * lane) = vq;
        }
        kp[0] = __uint_as_float(kq.x << 16), kp[1] = __uint_as_float(kq.x & 0xFFFF0000u);
        kp[2] = __uint_as_float(kq.y << 16), kp[3] = __uint_as_float(kq.y & 0xFFFF0000u);
        vp[0] = __uint_as_float(vq.x << 16), vp[1] = __uint_as_float(vq.x & 0xFFFF0000u);
        vp[2] = __uint_as_float(vq.y << 16), vp[3] = __uint_as_float(vq.y & 0xFFFF0000u);
    }
    float m[HP], l[HP], o[HP][4];
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
        m[hh] = -INFINITY;
        l[hh] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[hh][i] = 0.f;
    }
    // online softmax over P positions whose K/V rows (4 dims per lane) are in kw/vw
    auto consume = [&](const uint2 (&kw)[P], const uint2 (&vw)[P], int nvalid) {
        float acc[NV];
#pragma unroll
        for (int j = 0; j < P; ++j) {
            const float k0 = __uint_as_float(kw[j].x << 16), k1 = __uint_as_float(kw[j].x & 0xFFFF0000u);
            const float k2 = __uint_as_float(kw[j].y << 16), k3 = __uint_as_float(kw[j].y & 0xFFFF0000u);
#pragma unroll
            for (int hh = 0; hh < HP; ++hh)
                acc[j * HP + hh] = fmaf(q[hh][3], k3, fmaf(q[hh][2], k2, fmaf(q[hh][1], k1, q[hh][0] * k0)));
        }
        const float tot = warp_reduce_multi(acc);  // lane holds value lane / kS
#pragma unroll
        for (int hh = 0; hh < HP; ++hh) {
            float sc[P];
            float mx = m[hh];
#pragma unroll
            for (int j = 0; j < P; ++j) {
                sc[j] = __shfl_sync(0xffffffffu, tot, (j * HP + hh) * kS) * p.scale;
                if (j >= nvalid) sc[j] = -INFINITY;
                mx = fmaxf(mx, sc[j]);
            }
            const float corr = expf(m[hh] - mx);  // 0 on the first round (m = -inf)
            l[hh] *= corr;
#pragma unroll
            for (int i = 0; i < 4; ++i) o[hh][i] *= corr;
#pragma unroll
            for (int j = 0; j < P; ++j) {
                const float e = expf(sc[j] - mx);
                l[hh] += e;
                const float v0 = __uint_as_float(vw[j].x << 16), v1 = __uint_as_float(vw[j].x & 0xFFFF0000u);
                const float v2 = __uint_as_float(vw[j].y << 16), v3 = __uint_as_float(vw[j].y & 0xFFFF0000u);
                o[hh][0] = fmaf(e, v0, o[hh][0]);
                o[hh][1] = fmaf(e, v1, o[hh][1]);
                o[hh][2] = fmaf(e, v2, o[hh][2]);
                o[hh][3] = fmaf(e, v3, o[hh][3]);
            }
            m[hh] = mx;
        }
    };
    for (int j = 0; j < nst; ++j) {
        const int b = j & 1, a = p0 + j * kAttnStage, n = min(kAttnStage, c1 - a);
        bool ok = mbar_wait(&full[b], (j >> 1) & 1, &abort_flag, p.err);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            const uint16_t *kst = sk + (size_t)b * kAttnStage * hd, *vst = sv + (size_t)b * kAttnStage * hd;
            for (int i0 = warp * kPerWarp; i0 < min(n, (warp + 1) * kPerWarp); i0 += P) {
                uint2 kw[P], vw[P];
                const int nv = min(P, n - i0);
#pragma unroll
                for (int jj = 0; jj < P; ++jj) {
                    const int i = i0 + (jj < nv ? jj : 0);
                    kw[jj] = *reinterpret_cast<const uint2 *>(kst + (size_t)i * hd + 4 * lane);
                    vw[jj] = *reinterpret_cast<const uint2 *>(vst + (size_t)i * hd + 4 * lane);
                }
                consume(kw, vw, nv);
            }
        }
        __syncthreads();  // every warp is done with buffer b (and saw the abort flag)
        if (abort_flag) {
            // a wait gave up: the copies still in flight land before the CTA exits
            if (threadIdx.x == 0)
                for (int k = j + 1; k < issued; ++k)
                    for (uint32_t it = 0; it < kWaitLimit; ++it)
                        if (mbar_try_wait(&full[k & 1], (k >> 1) & 1)) break;
            break;
        }
        if (threadIdx.x == 0 && j + 2 < nst) issue(issued++);
    }
    if (warp == 0 && has_pos) {
        uint2 kw[P], vw[P];
        const uint2 kq = pack4_bf16(kp), vq = pack4_bf16(vp);
#pragma unroll
        for (int jj = 0; jj < P; ++jj) {
            kw[jj] = kq;
            vw[jj] = vq;
        }
        consume(kw, vw, 1);
    }
    // merge the warps, then write this split's partial
#pragma unroll
    for (int hh = 0; hh < HP; ++hh) {
        if (lane == 0) {
            sm_m[warp][hh] = m[hh];
            sm_l[warp][hh] = l[hh];
        }
        *reinterpret_cast<float4 *>(&sm_o[warp][hh][4 * lane]) = make_float4(o[hh][0], o[hh][1], o[hh][2], o[hh][3]);
    }
    __syncthreads();
    const int hd2 = hd + 2;
    for (int i = threadIdx.x; i < HP * hd; i += kAttnThreads) {
        const int hh = i / hd, d = i - hh * hd;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w][hh]);
        float L = 0.f, O = 0.f;
        if (M > -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float f = expf(sm_m[w][hh] - M);
                L = fmaf(sm_l[w][hh], f, L);
                O = fmaf(sm_o[w][hh][d], f, O);
            }
        }
        float *dst = p.part + (((size_t)t * p.nh + g * HP + hh) * p.nsplit + split) * hd2;
        dst[d] = O;
        if (d == 0) {
            dst[hd] = M;
            dst[hd + 1] = L;
        }
    }
    // the last split of (t, g) merges all splits into the output
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned *c = p.cnt + (size_t)t * p.nkv + g;
        is_last = atomicAdd(c, 1u) == (unsigned)p.nsplit - 1u;
        if (is_last) *c = 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // every split's max into shared memory (one load per thread), per head
    // the global max, the splits' factors and the total, then each output
    // dimension sums its splits with eight loads in flight
    __shared__ float sm_f[HP][kAttnMaxSplit];
    __shared__ float sm_L[HP];
    const int ns = p.nsplit;
    const float *base = p.part + ((size_t)t * p.nh + g * HP) * ns * hd2;
    for (int i = threadIdx.x; i < HP * ns; i += kAttnThreads) {
        const int hh = i / ns, s2 = i - hh * ns;
        sm_f[hh][s2] = __ldcg(base + ((size_t)hh * ns + s2) * hd2 + hd);
    }
    __syncthreads();
    for (int hh = warp; hh < HP; hh += kAttnWarps) {
        float M = -INFINITY;
        for (int s2 = lane; s2 < ns; s2 += 32) M = fmaxf(M, sm_f[hh][s2]);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        float L = 0.f;
        for (int s2 = lane; s2 < ns; s2 += 32) {
            const float ms = sm_f[hh][s2];
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            L = fmaf(__ldcg(base + ((size_t)hh * ns + s2) * hd2 + hd + 1), f, L);
            sm_f[hh][s2] = f;
        }
        L = warp_sum(L);
        if (lane == 0) sm_L[hh] = L;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < HP * hd; i += kAttnThreads) {
        const int hh = i / hd, d = i - hh * hd;
        const float *src = base + (size_t)hh * ns * hd2 + d;
        float O = 0.f;
        for (int s0 = 0; s0 < ns; s0 += 8) {
            float v[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) v[jj] = s0 + jj < ns ? __ldcg(src + (size_t)(s0 + jj) * hd2) : 0.f;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
                if (s0 + jj < ns) O = fmaf(v[jj], sm_f[hh][s0 + jj], O);
        }
        p.out[(size_t)t * p.nh * hd + (size_t)(g * HP + hh) * hd + d] = O / sm_L[hh];
    }
}

// --------------------------------------------------- prefill (T tokens) ----
// Token-parallel prefill of one sequence: T prompt tokens at positions
// pos0 .. pos0+T-1 go through each layer together.

// y[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * w): the GEMM operand of the
// next projection, one CTA per token.
__global__ void k_rmsnorm_bf16(const float *x, const uint16_t *w, float eps, __nv_bfloat16 *y, int dim) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t base = (size_t)t * dim;
    float s = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(x[base + i], x[base + i], s);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float ss = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) ss += red[i];
    const float rms = rsqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        y[base + i] = __float2bfloat16_rn((x[base + i] * rms) * bf16_bits(w[i]));
}

// Per (token, head): QK-norm and RoPE of q in place, and for the KV heads
// k (norm, RoPE) and v stored as bf16 in the cache at the token's position.
// grid (T, nh + nkv), one warp (hd = 128, 4 dims per lane).
__global__ void k_qk_rope_store(float *qkv, int qkv_stride, int nh, int nkv, const int *pos0p, int max_seq,
                                const uint16_t *qn_w, const uint16_t *kn_w, float eps, float theta,
                                uint16_t *kc, uint16_t *vc, int *err) {
    __shared__ float rc[kHeadDim / 2], rs[kHeadDim / 2];
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, hh = blockIdx.y, lane = threadIdx.x;
    const int pos = *pos0p + t;
    if (pos < 0 || pos >= max_seq) {
        if (lane == 0 && hh == 0) atomicOr(err, kErrBadIndex);
        return;
    }
    rope_table(rc, rs, pos, theta);
    __syncwarp();
    const int hd = kHeadDim, qd = nh * hd, kvd = nkv * hd;
    float *row = qkv + (size_t)t * qkv_stride;
    float v4[4];
    if (hh < nh) {
        load4(row + (size_t)hh * hd + 4 * lane, v4);
        if (qn_w) head_rmsnorm(v4, qn_w, eps);
        head_rope(v4, rc, rs);
        *reinterpret_cast<float4 *>(row + (size_t)hh * hd + 4 * lane) = make_float4(v4[0], v4[1], v4[2], v4[3]);
    } else {
        const int g = hh - nh;
        load4(row + qd + (size_t)g * hd + 4 * lane, v4);
        if (kn_w) head_rmsnorm(v4, kn_w, eps);
        head_rope(v4, rc, rs);
        const size_t at = ((size_t)g * max_seq + pos) * hd + 4 * lane;  // sequence slot 0
        *reinterpret_cast<uint2 *>(kc + at) = pack4_bf16(v4);
        load4(row + qd + kvd + (size_t)g * hd + 4 * lane, v4);
        *reinterpret_cast<uint2 *>(vc + at) = pack4_bf16(v4);
    }
}

// Tiled causal attention for a prompt (token-parallel prefill): one CTA per
// (block of kPfQ consecutive tokens, q head), 8 warps of kPfQ / 8 tokens each.
// The block's K and V rows come into shared memory once per tile of kPfKT
// positions and serve all its tokens (a per-token kernel reads a token's whole
// causal prefix from L2 on its own: ~1 GB per layer for 512 tokens).  Scores:
// lane j takes positions j and j + 32 of the tile for the warp's tokens (K rows
// padded by one word, so the lanes' rows fall in different banks; the tokens'
// q rows are broadcast from shared memory).  Online softmax per token in fp32;
// P.V with lane = 4 dimensions.  Token t (position pos0 + t) attends positions
// 0 .. pos0 + t; bf16 output (the o-projection GEMM's operand).
constexpr int kPfQ = 32, kPfKT = 64, kPfQW = kPfQ / 8;
static_assert(kPfQW == 4, "P.V reads one float4 of probabilities per position");
constexpr int kPfKRow = kHeadDim / 2 + 1;  // words per padded K row
__host__ __device__ constexpr size_t attn_prefill_smem() {
    return (size_t)kPfQ * kHeadDim * 4 + (size_t)kPfKT * kPfKRow * 4 + (size_t)kPfKT * kHeadDim * 2 +
           (size_t)8 * kPfKT * kPfQW * 4;
}
__global__ void __launch_bounds__(256) k_attn_prefill_tiled(const float *qkv, int qkv_stride, int nh, int nkv,
                                                            int T, const int *pos0p, int max_seq, float scale,
                                                            const uint16_t *kc, const uint16_t *vc,
                                                            __nv_bfloat16 *out) {
    extern __shared__ __align__(16) uint8_t pf_att_smem[];
    float *sq = reinterpret_cast<float *>(pf_att_smem);                       // [kPfQ][hd]
    uint32_t *sk = reinterpret_cast<uint32_t *>(sq + kPfQ * kHeadDim);         // [kPfKT][kPfKRow]
    uint32_t *sv = sk + kPfKT * kPfKRow;                                        // [kPfKT][hd/2]
    float *sp = reinterpret_cast<float *>(sv + kPfKT * (kHeadDim / 2));         // [8][kPfKT][kPfQW]
    pdl_trigger();
    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the last blocks attend the longest prefixes: they start first
    const int t0 = (gridDim.x - 1 - blockIdx.x) * kPfQ, head = blockIdx.y, g = head / (nh / nkv);
    const int pos0 = *pos0p;
    const int tlast = min(T, t0 + kPfQ) - 1;
    const int kmax = max(1, min(pos0 + tlast + 1, max_seq));  // positions the block reads
    // the block's q rows (rows past T are zero)
    for (int i = tid; i < kPfQ * kHeadDim / 4; i += 256) {
        const int r = i / (kHeadDim / 4), c4 = i - r * (kHeadDim / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + r < T)
            v = *reinterpret_cast<const float4 *>(qkv + (size_t)(t0 + r) * qkv_stride + (size_t)head * kHeadDim + 4 * c4);
        *reinterpret_cast<float4 *>(sq + r * kHeadDim + 4 * c4) = v;
    }
    const uint16_t *kb = kc + (size_t)g * max_seq * kHeadDim, *vb = vc + (size_t)g * max_seq * kHeadDim;
    int seq[kPfQW];  // positions each of the warp's tokens attends
    float m[kPfQW], l[kPfQW], o[kPfQW][4];
#pragma unroll
    for (int qi = 0; qi < kPfQW; ++qi) {
        const int t = t0 + warp * kPfQW + qi;
        seq[qi] = t < T ? max(1, min(pos0 + t + 1, max_seq)) : 0;
        m[qi] = -INFINITY;
        l[qi] = 0.f;
        o[qi][0] = o[qi][1] = o[qi][2] = o[qi][3] = 0.f;
    }
    float *spw = sp + warp * kPfKT * kPfQW;
    for (int k0 = 0; k0 < kmax; k0 += kPfKT) {
        __syncthreads();  // the previous tile is consumed (and sq is written, first time)
        for (int i = tid; i < kPfKT * (kHeadDim / 8); i += 256) {
            const int r = i / (kHeadDim / 8), c8 = i - r * (kHeadDim / 8);
            const int pp = min(k0 + r, kmax - 1);  // rows past the block's range repeat the last one
            const uint4 kw = __ldcg(reinterpret_cast<const uint4 *>(kb + (size_t)pp * kHeadDim) + c8);
            const uint4 vw = __ldcg(reinterpret_cast<const uint4 *>(vb + (size_t)pp * kHeadDim) + c8);
            uint32_t *kr = sk + r * kPfKRow + 4 * c8;
            kr[0] = kw.x;
            kr[1] = kw.y;
            kr[2] = kw.z;
            kr[3] = kw.w;
            *reinterpret_cast<uint4 *>(sv + r * (kHeadDim / 2) + 4 * c8) = vw;
        }
        __syncthreads();
        // scores of positions k0 + lane and k0 + lane + 32 for the warp's tokens
        float s[kPfQW][2];
#pragma unroll
        for (int qi = 0; qi < kPfQW; ++qi) s[qi][0] = s[qi][1] = 0.f;
        const uint32_t *k_a = sk + lane * kPfKRow, *k_b = sk + (lane + 32) * kPfKRow;
        const float *qw = sq + warp * kPfQW * kHeadDim;
#pragma unroll 4
        for (int d2 = 0; d2 < kHeadDim / 2; ++d2) {
            const uint32_t ka = k_a[d2], kbw = k_b[d2];
            const float a0 = __uint_as_float(ka << 16), a1 = __uint_as_float(ka & 0xFFFF0000u);
            const float b0 = __uint_as_float(kbw << 16), b1 = __uint_as_float(kbw & 0xFFFF0000u);
#pragma unroll
            for (int qi = 0; qi < kPfQW; ++qi) {
                const float2 qv = *reinterpret_cast<const float2 *>(qw + qi * kHeadDim + 2 * d2);
                s[qi][0] = fmaf(qv.y, a1, fmaf(qv.x, a0, s[qi][0]));
                s[qi][1] = fmaf(qv.y, b1, fmaf(qv.x, b0, s[qi][1]));
            }
        }
        // online softmax per token; the probabilities go to shared memory as
        // [position][token] so that P.V reads one float4 per position
#pragma unroll
        for (int qi = 0; qi < kPfQW; ++qi) {
            const float sa = (k0 + lane < seq[qi]) ? s[qi][0] * scale : -INFINITY;
            const float sb = (k0 + lane + 32 < seq[qi]) ? s[qi][1] * scale : -INFINITY;
            float mx = fmaxf(sa, sb);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[qi], mx);
            float pa = 0.f, pb = 0.f, corr = 1.f;
            if (mn != -INFINITY) {
                pa = expf(sa - mn);
                pb = expf(sb - mn);
                corr = expf(m[qi] - mn);
            }
            float ps = pa + pb;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l[qi] = l[qi] * corr + ps;
            m[qi] = mn;
#pragma unroll
            for (int i = 0; i < 4; ++i) o[qi][i] *= corr;
            spw[lane * kPfQW + qi] = pa;
            spw[(lane + 32) * kPfQW + qi] = pb;
        }
        __syncwarp();
        const int jn = min(kPfKT, kmax - k0);
        for (int j = 0; j < jn; ++j) {
            const uint2 vw = *reinterpret_cast<const uint2 *>(sv + j * (kHeadDim / 2) + 2 * lane);
            const float v0 = __uint_as_float(vw.x << 16), v1 = __uint_as_float(vw.x & 0xFFFF0000u);
            const float v2 = __uint_as_float(vw.y << 16), v3 = __uint_as_float(vw.y & 0xFFFF0000u);
            const float4 pj = *reinterpret_cast<const float4 *>(spw + j * kPfQW);
            const float pq[4] = {pj.x, pj.y, pj.z, pj.w};
#pragma unroll
            for (int qi = 0; qi < kPfQW; ++qi) {
                o[qi][0] = fmaf(pq[qi], v0, o[qi][0]);
                o[qi][1] = fmaf(pq[qi], v1, o[qi][1]);
                o[qi][2] = fmaf(pq[qi], v2, o[qi][2]);
                o[qi][3] = fmaf(pq[qi], v3, o[qi][3]);
            }
        }
        __syncwarp();
    }
#pragma unroll
    for (int qi = 0; qi < kPfQW; ++qi) {
        const int t = t0 + warp * kPfQW + qi;
        if (t < T) {
            const float inv = 1.0f / l[qi];
            const float v[4] = {o[qi][0] * inv, o[qi][1] * inv, o[qi][2] * inv, o[qi][3] * inv};
            *reinterpret_cast<uint2 *>(out + (size_t)t * nh * kHeadDim + (size_t)head * kHeadDim + 4 * lane) =
                pack4_bf16(v);
        }
    }
}


}  // namespace m1
