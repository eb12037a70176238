// moe_decode.cuh — one MoE block for a decode batch of 1..8 tokens (sm_100a).
//
// Replaces the MoE part of InferenceEngine.runLayer (InferenceEngine.swift
// :240-266): the CPU router (:490-519), loadExpert x K (:271-280) and CMD3 =
// K x (gate matvec4bit, up matvec4bit, swiGLU, down matvec4bit) + moeCombine
// (:401-478; Shaders.metal:39-92, 138-149, 360-376).
//
// Three kernels chained with Programmatic Dependent Launch:
//
//  k_router       bulk-copies its router rows into shared memory BEFORE waiting
//                 on the previous grid, then computes logits[t][e] = W_r[e].x[t]
//                 (bf16 router upcast exactly, fp32 FMA, fixed reduction order)
//                 and writes x as bf16 pair-permuted chunks (common.cuh) with
//                 fp32 chunk sums.  The last CTA to finish (atomic ticket)
//                 computes softmax + top-K for every token and the list of
//                 DISTINCT selected experts with their tokens (RouteInfo).
//  k_moe_gateup   one CTA per SM: a producer warp streams the CTA's slice of
//                 the (distinct expert, row) space through a ring of shared-
//                 memory stages (cp.async.bulk, mbarrier completion); 24
//                 consumer warps grab (tile, column-slice) work items
//                 dynamically and compute gate and up rows for every token
//                 routed to the expert; the SwiGLU epilogue writes act[t*K+k]
//                 (bf16, pair-permuted).
//  k_moe_down     launched while gate/up still runs: reads the route, and its
//                 producer prefetches the down rows of its h-row slice for every
//                 distinct expert; consumers wait for gate/up (griddepcontrol),
//                 compute y for each (token, k) and combine per output row in
//                 moeCombine's order: residual first, k ascending.
//
// Activations (x and the SwiGLU output) are kept as bf16 in the pair-permuted,
// chunk-transposed layout of common.cuh (ppos): the 32 values a lane needs for
// one 16-byte weight chunk are 4 uint4 loads, coalesced across the warp, and
// the inner loop is one LOP3 + two fma.rn.f32.bf16 per nibble pair (exact
// products, fp32 accumulation).  x given as bf16 is used exactly; f32 inputs
// and the SwiGLU activation are rounded to bf16 (round to nearest even).
//
// Experts outside this shard's [e0, e0+ne) are skipped (expert parallelism:
// the caller sums the shards' partial outputs).
#pragma once

#include <math.h>

#include "common.cuh"
#include "pipeline.cuh"

namespace m1 {

constexpr int kMaxTok = 8;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxPairs = kMaxTok * kMaxTopK;
constexpr int kConsumerWarps = 24;
constexpr int kPipeThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kRouterThreads = 256;
constexpr int kMaxStages = 64;

// The routing decision of one call, computed once by the router kernel.
struct RouteInfo {
    int idx[kMaxTok][kMaxTopK];    // top-K experts per token, descending
    float w[kMaxTok][kMaxTopK];    // their weights (renormalised if asked)
    int ulist[kMaxPairs];          // distinct LOCAL experts, ascending
    unsigned umask[kMaxPairs];     // tokens routed to each distinct expert
    unsigned char uk[kMaxPairs][kMaxTok];  // k of (distinct expert, token)
    int nU;                        // number of distinct local experts
    int pad_[3];
};

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
    uint16_t *xT;     // [ntok][h] bf16, pair-permuted chunk-transposed (common.cuh ppos)
    float *xsum;      // [ntok][h/32] fp32 chunk sums of the bf16 x
    uint16_t *actT;   // [ntok*K][I] bf16, pair-permuted chunk-transposed
    RouteInfo *route;
    int *ticket;      // router CTAs done (reset to 0 by the last one)
    int *user_idx;    // optional [ntok][K]
    float *user_w;    // optional [ntok][K]
    float *user_scores;  // optional [ntok][E]
    int *err;         // device error word
    // pipeline geometry, chosen by the host
    int gu_stage_bytes, gu_nstages, gu_nslices, gu_rows_max;
    int dn_stage_bytes, dn_nstages, dn_nslices, dn_rows_max;
    int x_smem;       // gate/up stages x pairs + chunk sums in shared memory
    unsigned long long *trace;  // optional phase timestamps (pipeline.cuh trace_event)
};

// Rows per tile held in registers by each consumer thread (accumulators are
// rows x tokens): the host plans tiles of exactly these row counts.
template <int NT>
struct TileRows {
    static constexpr int gu = NT == 1 ? 4 : (NT == 2 ? 2 : 1);
    static constexpr int dn = NT <= 2 ? 4 : 2;
};

__device__ __forceinline__ bool is_local(const MoeParams &p, int e) {
    return e >= p.e0 && e < p.e0 + p.ne;
}

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

// ------------------------------------------------------ softmax + top-K ----
// One warp: softmax over E logits (max-subtracted, expf, times 1/sum —
// InferenceEngine.swift:502-507) and top-K selection, descending, ties to the
// lower expert index (:510-519), optional renormalisation in k order.
__device__ __forceinline__ void route_token(const MoeParams &p, int t, RouteInfo &rs,
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
                // values; +1 keeps every candidate above "none" (0); NaN ranks lowest.
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
    __syncwarp();
}

// Route every token and build the distinct local expert list (all threads of
// the CTA participate; `mark` has kMaxExperts ints of scratch).
__device__ __forceinline__ void route_all(const MoeParams &p, RouteInfo &rs, int *mark,
                                          bool write_scores) {
    const int tid = threadIdx.x, warp = tid >> 5;
    if (warp < p.ntok) route_token(p, warp, rs, write_scores);
    for (int e = tid; e < p.E; e += blockDim.x) mark[e] = 0;
    for (int i = tid; i < kMaxPairs; i += blockDim.x) rs.umask[i] = 0u;
    __syncthreads();
    const int npair = p.ntok * p.K;
    for (int i = tid; i < npair; i += blockDim.x) {
        const int e = rs.idx[i / p.K][i % p.K];
        if (is_local(p, e)) mark[e] = 1;
    }
    __syncthreads();
    if (tid < 32) {
        int base = 0;
        for (int eb = 0; eb < p.E; eb += 32) {
            const int e = eb + tid;
            const bool mk = e < p.E && mark[e] != 0;
            const unsigned bal = __ballot_sync(0xffffffffu, mk);
            const int pos = base + __popc(bal & ((1u << tid) - 1u));
            if (e < p.E) mark[e] = mk ? pos : -1;
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
            const int u = mark[e];
            atomicOr(&rs.umask[u], 1u << t);
            rs.uk[u][t] = (unsigned char)k;
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------- router ----
// grid G <= #SMs; CTA c owns experts e = c, c+G, ... (bulk-copied to shared
// memory) and x chunks q = c*8+warp, ...; the last CTA to finish routes.
template <int NT>
__global__ void __launch_bounds__(kRouterThreads) k_router(const MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ RouteInfo s_route;
    __shared__ int s_mark[kMaxExperts];
    __shared__ int s_abort, s_last;
    pdl_trigger();
    const int G = gridDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nmine = (p.E > (int)blockIdx.x) ? (p.E - (int)blockIdx.x + G - 1) / G : 0;
    const size_t rowb = (size_t)p.h * 2;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + (size_t)nmine * rowb);
    float *part = reinterpret_cast<float *>(bar + 1);  // [8 warps][NT]
    if (tid == 0) {
        s_abort = 0;
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0 && nmine > 0) {
        const uint64_t pol = l2_evict_first_policy();
        mbar_arrive_expect_tx(bar, (uint32_t)(nmine * rowb));
        for (int k = 0; k < nmine; ++k)
            bulk_g2s(smem + k * rowb, p.router + (size_t)(blockIdx.x + k * G) * p.h,
                     (uint32_t)rowb, bar, pol);
    }
    if (tid == 0) trace_event(p.trace, 0, 0);
    pdl_wait();  // x is produced by the preceding grid
    if (tid == 0) trace_event(p.trace, 0, 1);

    // x -> bf16 pair-permuted chunk-transposed + fp32 chunk sums of the bf16
    // values (one warp per 32-column chunk).
    const int nch = p.h / kChunkCols;
    const size_t xtok = (size_t)p.h * (p.x_bf16 ? 2 : 4);
    for (int q = blockIdx.x * (kRouterThreads / 32) + warp; q < p.ntok * nch;
         q += G * (kRouterThreads / 32)) {
        const int t = q / nch, c = q % nch, j = c * kChunkCols + lane;
        const uint16_t vb = f32_to_bf16_rn(
            load_act(reinterpret_cast<const uint8_t *>(p.x) + t * xtok, p.x_bf16, j));
        p.xT[(size_t)t * p.h + ppos(j, nch)] = vb;
        const float s = warp_sum(bf16_bits(vb));
        if (lane == 0) p.xsum[(size_t)t * nch + c] = s;
    }

    if (nmine > 0 && mbar_wait(bar, 0, &s_abort, p.err)) {
        if (tid == 0) trace_event(p.trace, 0, 2);
        for (int k = 0; k < nmine; ++k) {
            const int e = blockIdx.x + k * G;
            const uint8_t *row = smem + k * rowb;
            float acc[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.f;
            for (int g8 = tid; g8 < p.h / 8; g8 += kRouterThreads) {
                const uint4 wv = *reinterpret_cast<const uint4 *>(row + g8 * 16);
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
                        load_x8(reinterpret_cast<const uint8_t *>(p.x) + t * xtok, p.x_bf16,
                                g8 * 8, xv);
#pragma unroll
                        for (int j = 0; j < 8; ++j) acc[t] = fmaf(wf[j], xv[j], acc[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(acc[t]);
                if (lane == 0) part[warp * NT + t] = v;
            }
            __syncthreads();
            if (tid < p.ntok) {
                float s = 0.f;
                for (int w = 0; w < kRouterThreads / 32; ++w) s += part[w * NT + tid];
                p.logits[(size_t)tid * p.E + e] = s;
            }
            __syncthreads();
        }
    }

    // The last CTA to arrive routes every token (threadFenceReduction pattern).
    __syncthreads();
    if (tid == 0) trace_event(p.trace, 0, 3);
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(p.ticket, 1) == G - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    route_all(p, s_route, s_mark, p.user_scores != nullptr);
    const int npair = p.ntok * p.K;
    for (int i = tid; i < npair; i += kRouterThreads) {
        const int t = i / p.K, k = i % p.K;
        if (p.user_idx) p.user_idx[i] = s_route.idx[t][k];
        if (p.user_w) p.user_w[i] = s_route.w[t][k];
    }
    const int *src = reinterpret_cast<const int *>(&s_route);
    int *dst = reinterpret_cast<int *>(p.route);
    for (int i = tid; i < (int)(sizeof(RouteInfo) / 4); i += kRouterThreads) dst[i] = src[i];
    if (tid == 0) *p.ticket = 0;
    if (tid == 0) trace_event(p.trace, 0, 4);
}

// --------------------------------------------------------------- tiling ----
struct Tile {
    int u, r0, nr;
};

// Shared-memory image of one tile of a projection: W rows, then the S and B
// row ranges each rounded out to 16 bytes.
struct ProjTile {
    const uint8_t *w;  // global
    Span16 s, b;
    uint32_t wbytes;
};

__device__ __forceinline__ ProjTile proj_tile(const uint8_t *blk, long long ow, long long os,
                                              long long ob, int r0, int nr, size_t wrb,
                                              size_t srb) {
    ProjTile pt;
    pt.w = blk + ow + (size_t)r0 * wrb;
    pt.wbytes = (uint32_t)(nr * wrb);
    pt.s = span16(blk + os + (size_t)r0 * srb, (size_t)nr * srb);
    pt.b = span16(blk + ob + (size_t)r0 * srb, (size_t)nr * srb);
    return pt;
}

__device__ __forceinline__ uint32_t proj_bytes(const ProjTile &t) {
    return t.wbytes + t.s.bytes + t.b.bytes;
}

// Issue the three copies of a projection tile at `dst`; returns bytes used.
__device__ __forceinline__ uint32_t proj_issue(const ProjTile &t, uint8_t *dst, uint64_t *bar,
                                               uint64_t pol) {
    bulk_g2s(dst, t.w, t.wbytes, bar, pol);
    bulk_g2s(dst + t.wbytes, t.s.src, t.s.bytes, bar, pol);
    bulk_g2s(dst + t.wbytes + t.s.bytes, t.b.src, t.b.bytes, bar, pol);
    return proj_bytes(t);
}

// Gate/up tiles: the CTA's contiguous slice [ua, ub) of "units" of RT rows of
// the (distinct expert, row) space; I % RT == 0 so a unit never crosses experts.
__device__ __forceinline__ Tile gu_tile(long long ua, int n, int I, int rt) {
    const long long row = (ua + n) * rt;
    return Tile{(int)(row / I), (int)(row % I), rt};
}

// Down tiles: for each distinct expert u, the CTA's rows [i0, i1) cut in
// pieces of rt rows; tile n = u * mt + m.
__device__ __forceinline__ Tile dn_tile(int n, int mt, int i0, int i1, int rt) {
    const int u = n / mt, m = n % mt;
    const int r0 = i0 + m * rt;
    return Tile{u, r0, min(rt, i1 - r0)};
}

// Shared-memory layout of the pipelined kernels:
//   [ring: nstages x stage_bytes][full[nstages]][empty[nstages]][Ctl][extra]
struct Ctl {
    RouteInfo route;
    int abort;
    int next_item;                 // dynamic work-item counter
    int issued;                    // tiles the producer issued
    int pad_;
    int stage_tile[kMaxStages];    // tile whose copies were last issued into each stage
};

struct PipeSmem {
    uint8_t *ring;
    uint64_t *full, *empty;
    Ctl *ctl;
    uint8_t *extra;
};

__device__ __forceinline__ PipeSmem pipe_smem(uint8_t *smem, int stage_bytes, int nstages) {
    PipeSmem s;
    s.ring = smem;
    s.full = reinterpret_cast<uint64_t *>(smem + (size_t)stage_bytes * nstages);
    s.empty = s.full + nstages;
    s.ctl = reinterpret_cast<Ctl *>(s.empty + nstages);
    s.extra = reinterpret_cast<uint8_t *>(s.ctl + 1);
    return s;
}

// Initialise barriers and control words (thread 0); callers __syncthreads().
// A stage is released by the `consumers` work items that read it.
__device__ __forceinline__ void pipe_init(const PipeSmem &s, int nstages, int consumers) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < nstages; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], consumers);
            s.ctl->stage_tile[i] = -1;
        }
        s.ctl->abort = 0;
        s.ctl->next_item = 0;
        s.ctl->issued = 0;
        mbar_fence_init();
    }
}

// Copy the route (written by the router grid, which has completed) to shared memory.
__device__ __forceinline__ void load_route(const MoeParams &p, RouteInfo &dst) {
    const int *src = reinterpret_cast<const int *>(p.route);
    int *d = reinterpret_cast<int *>(&dst);
    for (int i = threadIdx.x; i < (int)(sizeof(RouteInfo) / 4); i += blockDim.x)
        d[i] = __ldcg(src + i);
}

// Producer side: publish that tile n's copies were issued into stage s.
__device__ __forceinline__ void publish_stage(Ctl &ctl, int s, int n) {
    *reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) = n;
}

// Consumer side: wait until tile n occupies stage s and its bytes have landed.
// The stage_tile check comes first because mbarrier.try_wait.parity(P) also
// succeeds while the barrier is still in the phase BEFORE the awaited one (the
// previous tile of this stage, not yet landed).  Once stage_tile[s] == n, the
// previous phase of full[s] has completed (its consumers released the stage),
// so the parity wait targets exactly tile n's phase.  Warp-uniform result.
__device__ __forceinline__ bool wait_tile(const PipeSmem &S, int s, int n, int nstages, int *err) {
    Ctl &ctl = *S.ctl;
    bool ok = false;
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (*reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) == n) {
            ok = true;
            break;
        }
        if (*reinterpret_cast<volatile int *>(&ctl.abort)) break;
        __nanosleep(32);
    }
    if (!ok && !*reinterpret_cast<volatile int *>(&ctl.abort)) {
        ctl.abort = 1;
        if (err) atomicOr(err, kErrWaitTimeout);
    }
    if (ok) ok = mbar_wait(&S.full[s], (n / nstages) & 1, &ctl.abort, err);
    return __all_sync(0xffffffffu, ok);
}

// Before a CTA exits after an abort, wait (bounded) for copies still in flight
// into its shared memory.  `issued` = number of tiles the producer issued.
__device__ __forceinline__ void pipe_drain(const PipeSmem &s, int nstages, int issued) {
    for (int n = issued - nstages; n < issued; ++n) {
        if (n < 0) continue;
        for (uint32_t i = 0; i < kWaitLimit; ++i)
            if (mbar_try_wait(&s.full[n % nstages], (n / nstages) & 1)) break;
    }
}

// Next work item for the calling warp (warp-uniform).
__device__ __forceinline__ int grab_item(Ctl &ctl) {
    int q = 0;
    if ((threadIdx.x & 31) == 0) q = atomicAdd(&ctl.next_item, 1);
    return __shfl_sync(0xffffffffu, q, 0);
}

// Work items: a tile (RT rows of one projection, all columns, one ring stage)
// is split into `nsl` column slices of 32 chunks; item q = tile q/nsl, slice
// q%nsl is done by ONE warp, lane L owning chunks slice*32 + L (+ 32*nsl*m).
// Per-slice row totals go to shared memory and are summed in slice order once
// every item is done, so the result does not depend on which warp did what.

// ------------------------------------------------------- gate/up + SwiGLU ----
template <int NT>
__global__ void __launch_bounds__(kPipeThreads, 1) k_moe_gateup(const MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RT = TileRows<NT>::gu;
    const PipeSmem S = pipe_smem(smem, p.gu_stage_bytes, p.gu_nstages);
    Ctl &ctl = *S.ctl;
    const RouteInfo &rs = ctl.route;
    const int nsl = p.gu_nslices, NST = p.gu_nstages;
    const int nch = p.h / kChunkCols, nchI = p.I / kChunkCols;
    // extra: [x pairs NT*h bf16 (x_smem)][x chunk sums NT*nch][partials]
    uint16_t *xs = reinterpret_cast<uint16_t *>(S.extra);
    float *xss = reinterpret_cast<float *>(xs + (p.x_smem ? (size_t)NT * p.h : 0));
    float *part = xss + (p.x_smem ? (size_t)NT * nch : 0);  // [rows][nsl][NT][2]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pipe_init(S, NST, nsl);
    if (threadIdx.x == 0) trace_event(p.trace, 1, 0);
    pdl_wait();     // router grid done: route, xT, xsum are complete
    pdl_trigger();  // the down kernel may start (it reads the route early)
    if (threadIdx.x == 0) trace_event(p.trace, 1, 1);
    load_route(p, ctl.route);
    if (p.x_smem) {
        const int nx = p.ntok * p.h / 8;  // uint4 of bf16
        for (int i = threadIdx.x; i < nx; i += blockDim.x)
            reinterpret_cast<uint4 *>(xs)[i] = __ldg(reinterpret_cast<const uint4 *>(p.xT) + i);
        for (int i = threadIdx.x; i < p.ntok * nch; i += blockDim.x) xss[i] = __ldg(p.xsum + i);
    }
    __syncthreads();
    if (threadIdx.x == 0) trace_event(p.trace, 1, 2);
    const uint16_t *xsrc = p.x_smem ? xs : p.xT;
    const float *xsumsrc = p.x_smem ? xss : p.xsum;
    long long ua, ub;
    split_range((long long)rs.nU * (p.I / RT), gridDim.x, blockIdx.x, ua, ub);
    const int ntiles = (int)(ub - ua);
    const int nitems = ntiles * nsl;
    const size_t wrb = (size_t)p.h / 2, srb = (size_t)(p.h / p.gs) * 2;

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int n = 0;
            for (; n < ntiles; ++n) {
                const int s = n % NST;
                if (n >= NST && !mbar_wait(&S.empty[s], ((n / NST) - 1) & 1, &ctl.abort, p.err))
                    break;
                const Tile t = gu_tile(ua, n, p.I, RT);
                const uint8_t *blk = p.table + (size_t)(rs.ulist[t.u] - p.e0) * p.expert_bytes;
                const ProjTile g = proj_tile(blk, p.off[0], p.off[1], p.off[2], t.r0, t.nr, wrb, srb);
                const ProjTile u = proj_tile(blk, p.off[3], p.off[4], p.off[5], t.r0, t.nr, wrb, srb);
                uint8_t *st = S.ring + (size_t)s * p.gu_stage_bytes;
                mbar_arrive_expect_tx(&S.full[s], proj_bytes(g) + proj_bytes(u));
                const uint32_t gb = proj_issue(g, st, &S.full[s], pol);
                proj_issue(u, st + gb, &S.full[s], pol);
                publish_stage(ctl, s, n);
            }
            ctl.issued = n;
            trace_event(p.trace, 1, 3);
        }
    } else {
        // ---------------- consumer warps ----------------
        constexpr int kN = 2 * RT * NT, kStride = 32 / kN;
        for (;;) {
            const int q = grab_item(ctl);
            if (q >= nitems) break;
            const int n = q / nsl, j = q % nsl, s = n % NST;
            if (!wait_tile(S, s, n, NST, p.err)) break;
            if (q == 0 && lane == 0) trace_event(p.trace, 1, 4);
            const Tile t = gu_tile(ua, n, p.I, RT);
            const uint8_t *st = S.ring + (size_t)s * p.gu_stage_bytes;
            const uint8_t *blk = p.table + (size_t)(rs.ulist[t.u] - p.e0) * p.expert_bytes;
            const ProjTile g = proj_tile(blk, p.off[0], p.off[1], p.off[2], t.r0, RT, wrb, srb);
            const ProjTile u = proj_tile(blk, p.off[3], p.off[4], p.off[5], t.r0, RT, wrb, srb);
            const uint8_t *gst = st, *ust = st + proj_bytes(g);
            const uint8_t *gsp = gst + g.wbytes + g.s.skew, *gbp = gst + g.wbytes + g.s.bytes + g.b.skew;
            const uint8_t *usp = ust + u.wbytes + u.s.skew, *ubp = ust + u.wbytes + u.s.bytes + u.b.skew;
            const unsigned mask = rs.umask[t.u];
            float acc[kN];  // [(row * NT + token) * 2 + gate0/up1]
#pragma unroll
            for (int i = 0; i < kN; ++i) acc[i] = 0.f;
            for (int ch = j * 32 + lane; ch < nch; ch += 32 * nsl) {
                const int gi = (ch * kChunkCols) / p.gs;
#pragma unroll
                for (int k = 0; k < NT; ++k) {
                    if (!((mask >> k) & 1u)) continue;
                    uint32_t xp[16];
                    load_pairs_any(xsrc + (size_t)k * p.h, nch, ch, xp);
                    const float X = xsumsrc[(size_t)k * nch + ch];
#pragma unroll
                    for (int r = 0; r < RT; ++r) {
                        const uint4 wg = *reinterpret_cast<const uint4 *>(gst + r * wrb + ch * 16);
                        const uint4 wu = *reinterpret_cast<const uint4 *>(ust + r * wrb + ch * 16);
                        const float sg = bf16_bits(*reinterpret_cast<const uint16_t *>(gsp + r * srb + gi * 2));
                        const float bg = bf16_bits(*reinterpret_cast<const uint16_t *>(gbp + r * srb + gi * 2));
                        const float su = bf16_bits(*reinterpret_cast<const uint16_t *>(usp + r * srb + gi * 2));
                        const float bu = bf16_bits(*reinterpret_cast<const uint16_t *>(ubp + r * srb + gi * 2));
                        float &ag = acc[(r * NT + k) * 2 + 0];
                        float &au = acc[(r * NT + k) * 2 + 1];
                        // s*(A - 128X) + b*X with A = sum (128+q) x
                        ag = fmaf(sg, dot_chunk_bf16(wg, xp), fmaf(fmaf(-128.f, sg, bg), X, ag));
                        au = fmaf(su, dot_chunk_bf16(wu, xp), fmaf(fmaf(-128.f, su, bu), X, au));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);  // stage data no longer needed by this item
            // lane holds value lane/kStride = (r*NT + k)*2 + m
            const float tot = warp_reduce_multi(acc);
            if (nsl == 1) {
                // the up value of (r, k) sits kStride lanes above its gate value
                const float upv = __shfl_down_sync(0xffffffffu, tot, kStride);
                if (lane % (2 * kStride) == 0) {
                    const int jj = lane / (2 * kStride), r = jj / NT, k = jj % NT;
                    if ((mask >> k) & 1u) {
                        // Shaders.metal:147-148: SiLU(gate) * up
                        uint16_t *arow = p.actT + ((size_t)k * p.K + rs.uk[t.u][k]) * p.I;
                        arow[ppos(t.r0 + r, nchI)] = f32_to_bf16_rn((tot / (1.0f + expf(-tot))) * upv);
                    }
                }
            } else if (lane % kStride == 0) {
                const int v = lane / kStride, r = v / (2 * NT), km = v % (2 * NT);
                part[((size_t)(n * RT + r) * nsl + j) * (2 * NT) + km] = tot;
            }
        }
        if (nsl > 1) {
            // Every item of this CTA is done: sum the slices in order, SwiGLU.
            named_sync(1, kConsumerWarps * 32);
            if (threadIdx.x == 0) trace_event(p.trace, 1, 5);
            if (!ctl.abort) {
                for (int i = threadIdx.x; i < ntiles * RT * NT; i += kConsumerWarps * 32) {
                    const int lr = i / NT, k = i % NT;
                    const long long row = ua * RT + lr;
                    const int u = (int)(row / p.I), r = (int)(row % p.I);
                    if (!((rs.umask[u] >> k) & 1u)) continue;
                    float gv = 0.f, uv = 0.f;
                    for (int jj = 0; jj < nsl; ++jj) {
                        gv += part[((size_t)lr * nsl + jj) * (2 * NT) + 2 * k + 0];
                        uv += part[((size_t)lr * nsl + jj) * (2 * NT) + 2 * k + 1];
                    }
                    uint16_t *arow = p.actT + ((size_t)k * p.K + rs.uk[u][k]) * p.I;
                    arow[ppos(r, nchI)] = f32_to_bf16_rn((gv / (1.0f + expf(-gv))) * uv);
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) trace_event(p.trace, 1, 6);
    if (ctl.abort && threadIdx.x == 0) pipe_drain(S, NST, ctl.issued);
}

// ------------------------------------------------------- down + combine ----
template <int NT>
__global__ void __launch_bounds__(kPipeThreads, 1) k_moe_down(const MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RT = TileRows<NT>::dn;
    const PipeSmem S = pipe_smem(smem, p.dn_stage_bytes, p.dn_nstages);
    Ctl &ctl = *S.ctl;
    const RouteInfo &rs = ctl.route;
    const int nsl = p.dn_nslices, NST = p.dn_nstages, rmax = p.dn_rows_max;
    float *part = reinterpret_cast<float *>(S.extra);  // [ntok*K pairs][rows_max][nsl]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pipe_init(S, NST, nsl);
    if (threadIdx.x == 0) trace_event(p.trace, 2, 0);
    pdl_trigger();
    // The route is final: the gate/up grid only let this grid launch after its
    // own griddepcontrol.wait on the router grid returned.
    load_route(p, ctl.route);
    __syncthreads();
    int i0, i1;
    {
        long long lb, le;
        split_range(p.h, gridDim.x, blockIdx.x, lb, le);
        i0 = (int)lb;
        i1 = (int)le;
    }
    if (threadIdx.x == 0) trace_event(p.trace, 2, 1);
    const int mt = (i1 - i0 + RT - 1) / RT;  // row pieces per distinct expert
    const int ntiles = rs.nU * mt;
    const int nitems = ntiles * nsl;
    const size_t wrb = (size_t)p.I / 2, srb = (size_t)(p.I / p.gs) * 2;

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int n = 0;
            for (; n < ntiles; ++n) {
                const int s = n % NST;
                if (n >= NST && !mbar_wait(&S.empty[s], ((n / NST) - 1) & 1, &ctl.abort, p.err))
                    break;
                const Tile t = dn_tile(n, mt, i0, i1, RT);
                const uint8_t *blk = p.table + (size_t)(rs.ulist[t.u] - p.e0) * p.expert_bytes;
                const ProjTile d = proj_tile(blk, p.off[6], p.off[7], p.off[8], t.r0, t.nr, wrb, srb);
                mbar_arrive_expect_tx(&S.full[s], proj_bytes(d));
                proj_issue(d, S.ring + (size_t)s * p.dn_stage_bytes, &S.full[s], pol);
                publish_stage(ctl, s, n);
            }
            ctl.issued = n;
            trace_event(p.trace, 2, 2);
        }
    } else {
        pdl_wait();  // gate/up grid done: act is complete
        if (threadIdx.x == 0) trace_event(p.trace, 2, 3);
        const int nchI = p.I / kChunkCols;
        constexpr int kStride = 32 / RT;
        for (;;) {
            const int q = grab_item(ctl);
            if (q >= nitems) break;
            const int n = q / nsl, j = q % nsl, s = n % NST;
            if (!wait_tile(S, s, n, NST, p.err)) break;
            const Tile t = dn_tile(n, mt, i0, i1, RT);
            const uint8_t *st = S.ring + (size_t)s * p.dn_stage_bytes;
            const uint8_t *blk = p.table + (size_t)(rs.ulist[t.u] - p.e0) * p.expert_bytes;
            const ProjTile d = proj_tile(blk, p.off[6], p.off[7], p.off[8], t.r0, t.nr, wrb, srb);
            const uint8_t *sp = st + d.wbytes + d.s.skew, *bp = st + d.wbytes + d.s.bytes + d.b.skew;
            const unsigned mask = rs.umask[t.u];
            for (int k = 0; k < NT; ++k) {
                if (!((mask >> k) & 1u)) continue;
                const int pair = k * p.K + rs.uk[t.u][k];
                const uint16_t *aT = p.actT + (size_t)pair * p.I;
                float y[RT];
#pragma unroll
                for (int r = 0; r < RT; ++r) y[r] = 0.f;
                for (int ch = j * 32 + lane; ch < nchI; ch += 32 * nsl) {
                    const int gi = (ch * kChunkCols) / p.gs;
                    uint32_t xp[16];
                    load_pairs(aT, nchI, ch, xp);
                    const float X = pair_sum(xp);
#pragma unroll
                    for (int r = 0; r < RT; ++r) {
                        if (r < t.nr) {
                            const uint4 w = *reinterpret_cast<const uint4 *>(st + r * wrb + ch * 16);
                            const float sc = bf16_bits(*reinterpret_cast<const uint16_t *>(sp + r * srb + gi * 2));
                            const float bi = bf16_bits(*reinterpret_cast<const uint16_t *>(bp + r * srb + gi * 2));
                            y[r] = fmaf(sc, dot_chunk_bf16(w, xp), fmaf(fmaf(-128.f, sc, bi), X, y[r]));
                        }
                    }
                }
                const float tot = warp_reduce_multi(y);
                if (lane % kStride == 0) {
                    const int r = lane / kStride;
                    if (r < t.nr)
                        part[((size_t)pair * rmax + (t.r0 - i0) + r) * nsl + j] = tot;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
        }
        named_sync(1, kConsumerWarps * 32);
        if (threadIdx.x == 0) trace_event(p.trace, 2, 4);
        // moeCombine (Shaders.metal:360-376): residual first, then k ascending;
        // each expert output is its slices summed in order.
        const int nrows = i1 - i0;
        if (!ctl.abort) {
            for (int qq = threadIdx.x; qq < p.ntok * nrows; qq += kConsumerWarps * 32) {
                const int t = qq / nrows, i = i0 + qq % nrows;
                float acc = p.res ? load_act(p.res, p.res_bf16, (size_t)t * p.h + i) : 0.f;
                for (int k = 0; k < p.K; ++k) {
                    if (!is_local(p, rs.idx[t][k])) continue;
                    const float *pp = part + ((size_t)(t * p.K + k) * rmax + (i - i0)) * nsl;
                    float y = 0.f;
                    for (int jj = 0; jj < nsl; ++jj) y += pp[jj];
                    acc = fmaf(rs.w[t][k], y, acc);
                }
                store_act(p.out, p.out_bf16, (size_t)t * p.h + i, acc);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) trace_event(p.trace, 2, 5);
    if (ctl.abort && threadIdx.x == 0) pipe_drain(S, NST, ctl.issued);
}

}  // namespace m1
