// moe_decode.cuh — one MoE block for a decode batch of 1..8 tokens.
//
// Replaces the MoE part of InferenceEngine.runLayer (InferenceEngine.swift
// :240-266): the CPU router (:490-519), loadExpert x K (:271-280) and CMD3 =
// K x (gate matvec4bit, up matvec4bit, swiGLU, down matvec4bit) + moeCombine
// (:401-478; Shaders.metal:39-92, 138-149, 360-376).  Three kernels:
//
//  1. k_router_logits  one warp per expert row: logits[t][e] = W_r[e] . x[t]
//                      (bf16 router upcast exactly, fp32 FMA).
//  2. k_moe_gateup     every CTA recomputes softmax + top-K for all tokens from
//                      the logits (deterministic, identical in every CTA), builds
//                      the list of DISTINCT selected experts, then streams each
//                      distinct expert's gate and up rows once for all tokens
//                      routed to it; the SwiGLU epilogue writes act[t*K+k][I].
//  3. k_moe_down       each warp owns R output rows; for every (token, k) pair
//                      in k-ascending order it computes the down row dot with
//                      act[t*K+k] and accumulates w[t][k] * y onto the residual,
//                      which is moeCombine's order (residual first, k ascending).
//
// Experts outside this shard's [e0, e0+ne) are skipped (expert parallelism:
// the caller sums the shards' partial outputs).
#pragma once

#include <math.h>

#include "common.cuh"
#include "matvec4.cuh"

namespace m1 {

constexpr int kMaxTok = 8;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxPairs = kMaxTok * kMaxTopK;

struct MoeParams {
    const uint8_t *table;  // this layer's blocks for experts [e0, e0+ne)
    long long expert_bytes;
    long long off[9];      // gateW gateS gateB upW upS upB downW downS downB
    const uint16_t *router;  // bf16 [E][h]
    int E, K, h, I, gs, norm;
    int e0, ne;
    int ntok;
    const void *x;
    int x_bf16;
    const void *res;  // may be null
    int res_bf16;
    void *out;
    int out_bf16;
    float *logits;    // [ntok][E]
    int *route_idx;   // [ntok][K]
    float *route_w;   // [ntok][K]
    float *act;       // [ntok*K][I]
    int *user_idx;    // optional [ntok][K]
    float *user_w;    // optional [ntok][K]
    float *user_scores;  // optional [ntok][E]
};

__device__ __forceinline__ void load_x8(const void *xbase, int is_bf16, int col, float (&x)[8]) {
    if (is_bf16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(
            reinterpret_cast<const uint16_t *>(xbase) + col));
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[2 * j] = __uint_as_float(vv[j] << 16);
            x[2 * j + 1] = __uint_as_float(vv[j] & 0xFFFF0000u);
        }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(
            reinterpret_cast<const float *>(xbase) + col);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
}

// ---------------------------------------------------------------- router ----
// grid = ceil(E/8) CTAs of 8 warps; warp e computes logits[:, e].
template <int NT>
__global__ void __launch_bounds__(256) k_router_logits(const MoeParams p) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= p.E) return;
    const uint16_t *row = p.router + (size_t)e * p.h;
    const size_t xtok = (size_t)p.h * (p.x_bf16 ? 2 : 4);
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
#pragma unroll 4
    for (int c = lane * 8; c < p.h; c += 256) {
        const uint4 wv = ld_stream16(row + c);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        float wf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wf[2 * j] = __uint_as_float(ww[j] << 16);
            wf[2 * j + 1] = __uint_as_float(ww[j] & 0xFFFF0000u);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < p.ntok) {
                float xv[8];
                load_x8(reinterpret_cast<const uint8_t *>(p.x) + (size_t)t * xtok, p.x_bf16, c, xv);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[t] = fmaf(wf[j], xv[j], acc[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0 && t < p.ntok) p.logits[(size_t)t * p.E + e] = v;
    }
}

// ------------------------------------------------------ softmax + top-K ----
struct RouteSmem {
    int idx[kMaxTok][kMaxTopK];
    float w[kMaxTok][kMaxTopK];
    int uid[kMaxExperts];          // expert -> distinct slot (or -1)
    int ulist[kMaxPairs];          // distinct slot -> expert (ascending)
    unsigned umask[kMaxPairs];     // distinct slot -> token bitmask
    unsigned char uk[kMaxPairs][kMaxTok];  // distinct slot, token -> k
    int nU;
};

// One warp: softmax over E logits (max-subtracted, expf, times 1/sum —
// InferenceEngine.swift:502-507) and top-K selection, descending, ties to the
// lower expert index (:510-519), optional renormalisation in k order.
__device__ __forceinline__ void route_token(const MoeParams &p, int t, RouteSmem &rs,
                                            bool write_scores) {
    const int lane = threadIdx.x & 31;
    constexpr int J = kMaxExperts / 32;
    const float *lg = p.logits + (size_t)t * p.E;
    float v[J];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        v[j] = (e < p.E) ? __ldcg(lg + e) : -INFINITY;
        m = fmaxf(m, v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        v[j] = (e < p.E) ? expf(v[j] - m) : 0.f;
        s += v[j];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        v[j] *= inv;
        const int e = lane + 32 * j;
        if (write_scores && e < p.E) p.user_scores[(size_t)t * p.E + e] = v[j];
    }
    unsigned taken = 0;
    float wsum = 0.f;
    for (int k = 0; k < p.K; ++k) {
        unsigned bestkey = 0;
        int bestj = -1;
        float bestp = 0.f;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int e = lane + 32 * j;
            if (e < p.E && !((taken >> j) & 1u)) {
                // probabilities are >= 0, so their bit patterns order like the
                // values; +1 keeps every candidate above "no candidate" (0) and
                // NaN ranks lowest.
                const unsigned key = (v[j] != v[j]) ? 1u : __float_as_uint(v[j]) + 1u;
                if (key > bestkey) {
                    bestkey = key;
                    bestj = j;
                    bestp = v[j];
                }
            }
        }
        const unsigned mk = __reduce_max_sync(0xffffffffu, bestkey);
        const unsigned mine =
            (bestj >= 0 && bestkey == mk) ? (unsigned)(lane + 32 * bestj) : 0xFFFFFFFFu;
        const unsigned win = __reduce_min_sync(0xffffffffu, mine);
        const int owner = (int)(win & 31u);
        const float wp = __shfl_sync(0xffffffffu, bestp, owner);
        if (lane == owner) taken |= 1u << (win >> 5);
        if (lane == 0) {
            rs.idx[t][k] = (int)win;
            rs.w[t][k] = wp;
        }
        wsum += wp;
    }
    if (p.norm) {
        __syncwarp();
        if (lane == 0)
            for (int k = 0; k < p.K; ++k) rs.w[t][k] = rs.w[t][k] / wsum;
    }
}

__device__ __forceinline__ bool is_local(const MoeParams &p, int e) {
    return e >= p.e0 && e < p.e0 + p.ne;
}

// Distinct local experts (ascending) and, per distinct expert, its tokens.
__device__ __forceinline__ void build_unique(const MoeParams &p, RouteSmem &rs) {
    const int tid = threadIdx.x;
    for (int e = tid; e < p.E; e += blockDim.x) rs.uid[e] = 0;
    for (int i = tid; i < kMaxPairs; i += blockDim.x) rs.umask[i] = 0u;
    __syncthreads();
    const int npair = p.ntok * p.K;
    for (int i = tid; i < npair; i += blockDim.x) {
        const int e = rs.idx[i / p.K][i % p.K];
        if (is_local(p, e)) rs.uid[e] = 1;
    }
    __syncthreads();
    if (tid < 32) {
        int base = 0;
        for (int eb = 0; eb < p.E; eb += 32) {
            const int e = eb + tid;
            const bool mk = e < p.E && rs.uid[e] != 0;
            const unsigned bal = __ballot_sync(0xffffffffu, mk);
            const int pos = base + __popc(bal & ((1u << tid) - 1u));
            if (e < p.E) rs.uid[e] = mk ? pos : -1;
            if (mk) rs.ulist[pos] = e;
            base += __popc(bal);
        }
        if (tid == 0) rs.nU = base;
    }
    __syncthreads();
    for (int i = tid; i < npair; i += blockDim.x) {
        const int t = i / p.K, k = i % p.K;
        const int e = rs.idx[t][k];
        if (is_local(p, e)) {
            const int u = rs.uid[e];
            atomicOr(&rs.umask[u], 1u << t);
            rs.uk[u][t] = (unsigned char)k;
        }
    }
    __syncthreads();
}

// ------------------------------------------------------- gate/up + SwiGLU ----
template <int NT, int R>
__global__ void __launch_bounds__(256) k_moe_gateup(const MoeParams p) {
    __shared__ RouteSmem rs;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    if (warp < p.ntok) route_token(p, warp, rs, blockIdx.x == 0 && p.user_scores != nullptr);
    __syncthreads();
    build_unique(p, rs);
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < p.ntok * p.K; i += blockDim.x) {
            const int t = i / p.K, k = i % p.K;
            p.route_idx[i] = rs.idx[t][k];
            p.route_w[i] = rs.w[t][k];
            if (p.user_idx) p.user_idx[i] = rs.idx[t][k];
            if (p.user_w) p.user_w[i] = rs.w[t][k];
        }
    }
    const int gpe = p.I / R;  // row groups per expert (I % R == 0)
    long long gb, ge;
    split_range((long long)rs.nU * gpe, gridDim.x, blockIdx.x, gb, ge);
    const int nch = p.h / kChunkCols;
    const size_t wrow = (size_t)p.h / 2;
    const size_t srow = (size_t)(p.h / p.gs) * 2;
    const size_t xtok = (size_t)p.h * (p.x_bf16 ? 2 : 4);

    for (long long g = gb + warp; g < ge; g += nwarps) {
        const int u = (int)(g / gpe);
        const int r0 = (int)(g % gpe) * R;
        const int e = rs.ulist[u];
        const unsigned mask = rs.umask[u];
        const uint8_t *blk = p.table + (size_t)(e - p.e0) * p.expert_bytes;
        const uint8_t *gw = blk + p.off[0], *gs_ = blk + p.off[1], *gb_ = blk + p.off[2];
        const uint8_t *uw = blk + p.off[3], *us_ = blk + p.off[4], *ub_ = blk + p.off[5];
        float ga[R][NT], ua[R][NT];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) ga[r][t] = ua[r][t] = 0.f;

        int ch = lane;
        ChunkW<R> cg, cu;
        if (ch < nch) {
            load_chunk_rows<R>(cg, gw, gs_, gb_, r0, p.I, wrow, srow, ch, p.gs);
            load_chunk_rows<R>(cu, uw, us_, ub_, r0, p.I, wrow, srow, ch, p.gs);
        }
        while (ch < nch) {
            const int nxt = ch + kWarp;
            ChunkW<R> ng, nu;
            if (nxt < nch) {
                load_chunk_rows<R>(ng, gw, gs_, gb_, r0, p.I, wrow, srow, nxt, p.gs);
                load_chunk_rows<R>(nu, uw, us_, ub_, r0, p.I, wrow, srow, nxt, p.gs);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if ((mask >> t) & 1u) {
                    float xv[32];
                    const float X = load_x32(
                        reinterpret_cast<const uint8_t *>(p.x) + (size_t)t * xtok, p.x_bf16,
                        ch * kChunkCols, xv);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float Qg = dot_chunk(cg.w[r], xv);
                        ga[r][t] = fmaf(cg.s[r], Qg, fmaf(cg.b[r], X, ga[r][t]));
                        const float Qu = dot_chunk(cu.w[r], xv);
                        ua[r][t] = fmaf(cu.s[r], Qu, fmaf(cu.b[r], X, ua[r][t]));
                    }
                }
            }
            if (nxt < nch) {
                cg = ng;
                cu = nu;
            }
            ch = nxt;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if ((mask >> t) & 1u) {
                const int k = rs.uk[u][t];
                float *arow = p.act + ((size_t)t * p.K + k) * p.I;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float gv = warp_sum(ga[r][t]);
                    const float uv = warp_sum(ua[r][t]);
                    // Shaders.metal:147-148: SiLU(gate) * up
                    if (lane == 0) arow[r0 + r] = (gv / (1.0f + expf(-gv))) * uv;
                }
            }
        }
    }
}

// ------------------------------------------------------- down + combine ----
template <int NT, int R>
__global__ void __launch_bounds__(256) k_moe_down(const MoeParams p) {
    __shared__ int s_e[kMaxPairs];
    __shared__ float s_w[kMaxPairs];
    __shared__ int s_pair[kMaxPairs];  // act row index t*K+k of local pairs, t-major, k ascending
    __shared__ int s_np;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int npair = p.ntok * p.K;
    for (int i = threadIdx.x; i < npair; i += blockDim.x) {
        s_e[i] = __ldcg(p.route_idx + i);
        s_w[i] = __ldcg(p.route_w + i);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int n = 0;
        for (int i = 0; i < npair; ++i)
            if (is_local(p, s_e[i])) s_pair[n++] = i;
        s_np = n;
    }
    __syncthreads();
    const int np = s_np;
    const int nch = p.I / kChunkCols;
    const int npass = (nch + kWarp - 1) / kWarp;
    const size_t wrow = (size_t)p.I / 2;
    const size_t srow = (size_t)(p.I / p.gs) * 2;
    long long gb, ge;
    split_range((long long)((p.h + R - 1) / R), gridDim.x, blockIdx.x, gb, ge);

    for (long long g = gb + warp; g < ge; g += nwarps) {
        const int r0 = (int)g * R;
        float acc[R][NT];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int row = r0 + r;
                acc[r][t] = (p.res != nullptr && t < p.ntok && row < p.h)
                                ? load_act(p.res, p.res_bf16, (size_t)t * p.h + row)
                                : 0.f;
            }
        // Steps = (pair, pass), flattened so the next step's weights are in
        // flight while the current step computes.
        const int nsteps = np * npass;
        auto load_step = [&](int st, ChunkW<R> &c) {
            const int pi = st / npass, ps = st % npass;
            const int ch = ps * kWarp + lane;
            if (ch < nch) {
                const int ai = s_pair[pi];
                const uint8_t *blk = p.table + (size_t)(s_e[ai] - p.e0) * p.expert_bytes;
                load_chunk_rows<R>(c, blk + p.off[6], blk + p.off[7], blk + p.off[8], r0, p.h,
                                   wrow, srow, ch, p.gs);
            }
        };
        ChunkW<R> cur;
        if (nsteps > 0) load_step(0, cur);
        float y[R];
#pragma unroll
        for (int r = 0; r < R; ++r) y[r] = 0.f;
        for (int st = 0; st < nsteps; ++st) {
            ChunkW<R> nb;
            if (st + 1 < nsteps) load_step(st + 1, nb);
            const int pi = st / npass, ps = st % npass;
            const int ch = ps * kWarp + lane;
            const int ai = s_pair[pi];
            if (ch < nch) {
                float xv[32];
                const float X =
                    load_x32(p.act + (size_t)ai * p.I, 0, ch * kChunkCols, xv);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float Q = dot_chunk(cur.w[r], xv);
                    y[r] = fmaf(cur.s[r], Q, fmaf(cur.b[r], X, y[r]));
                }
            }
            if (ps == npass - 1) {
                const int t = ai / p.K;
                const float wk = s_w[ai];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float v = warp_sum(y[r]);
                    y[r] = 0.f;
#pragma unroll
                    for (int tt = 0; tt < NT; ++tt)
                        if (tt == t) acc[r][tt] = fmaf(wk, v, acc[r][tt]);
                }
            }
            if (st + 1 < nsteps) cur = nb;
        }
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const int row = r0 + r;
                    if (t < p.ntok && row < p.h)
                        store_act(p.out, p.out_bf16, (size_t)t * p.h + row, acc[r][t]);
                }
        }
    }
}

}  // namespace m1
