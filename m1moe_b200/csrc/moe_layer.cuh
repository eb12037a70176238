// moe_layer.cuh — one MoE block for a decode batch of 1..8 tokens in ONE
// kernel (sm_100a).
//
// Replaces the MoE part of InferenceEngine.runLayer (InferenceEngine.swift
// :240-266): the CPU router (:490-519), loadExpert x K (:271-280) and CMD3 =
// K x (gate matvec4bit, up matvec4bit, swiGLU, down matvec4bit) + moeCombine
// (:401-478; Shaders.metal:39-92, 138-149, 360-376).
//
// One CTA per SM (cooperative launch: every CTA is resident, which the
// cross-CTA waits below need).  Phases:
//   1. stage x in shared memory as bf16 pair-permuted chunks with fp32 chunk
//      sums (common.cuh); prefetch this CTA's router rows (bulk copy);
//   2. logits[t][e] = W_r[e] . x[t] for this CTA's experts (bf16 router
//      upcast exactly, the caller's x, fp32 FMA, fixed reduction order),
//      published as TAGGED words (below);
//   3. every CTA routes every token from the logits (identical,
//      deterministic): softmax, top-K by rank (descending, ties to the lower
//      index), optional renormalisation, distinct local experts;
//   4. a producer warp streams this CTA's gate/up tiles and then its down
//      tiles through a ring of shared-memory stages, one bulk copy per tile;
//      24 consumer warps take (tile, row pairs, column slice) work items and
//      write the SwiGLU activations (bf16) to global memory; the CTA then
//      publishes them;
//   5. the consumers compute the down rows of this CTA's h-slice for every
//      (token, k) from tiles prefetched during phase 4, each 32-row chunk of
//      an activation as soon as the CTAs that wrote it have published, and
//      combine per output row in moeCombine's order: residual first, k
//      ascending.
//
// Cross-CTA exchange without grid barriers.  Every CTA keeps a call counter
// in its own epoch word (one 128-byte line per CTA); all CTAs start a call
// with the same value, so tag = epoch + 1 names the call everywhere without
// communication.  A logit travels as one 64-bit word {tag, f32} (relaxed
// gpu-scope 64-bit accesses are single-copy atomic), so a reader that sees the
// tag sees the value.  Activations are plain bf16; a CTA release-stores the
// tag into its epoch word once all of its activations are written, and a
// reader acquire-loads the epoch words of the one or two CTAs that wrote the
// chunk it needs (remembered in a shared-memory bit mask).  Loads that poll
// touch one word per writer, not the data, which keeps the L2 free for the
// weight stream.  All waits are bounded; on timeout the CTA sets the device
// error word and unwinds.
//
// Expert weights use the TILED table layout (tiled_layout.cuh): gate/up
// "pair-rows" [gateW|gateS|gateB|upW|upS|upB] and down rows [W|S|B], so a run
// of rows is one contiguous bulk copy.  The bytes are the reference's bytes,
// reordered once at load time.
//
// Experts outside this shard's [e0, e0+ne) are skipped (expert parallelism:
// the caller sums the shards' partial outputs).
#pragma once

#include <math.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "tiled_layout.cuh"

namespace m1 {

constexpr int kMaxTok = 8;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxPairs = kMaxTok * kMaxTopK;
constexpr int kConsumerWarps = 24;
constexpr int kLayerThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kMaxStages = 32;
constexpr int kMaxCtas = 1024;
constexpr int kEpochStride = 32;  // words between two CTAs' epoch words (own 128-byte line)
constexpr int kLogitsPerLane = kMaxExperts / 32;

// Work-item shapes for NT tokens.  A gate/up item covers PG "row pairs"
// (rows R and R+4 of an expert, R % 8 < 4: the two rows whose activations
// share one pair-permuted word), computing RG rows at a time in NPASS passes.
// A down item covers up to DN rows.
template <int NT>
struct ItemRows {
    static constexpr int gu = NT == 1 ? 4 : (NT == 2 ? 2 : 1);  // RG
    static constexpr int pairs = gu >= 2 ? gu / 2 : 1;          // PG
    static constexpr int passes = gu >= 2 ? 1 : 2;              // NPASS
    static constexpr int dn = NT == 1 ? 8 : 4;  // DN
};

// The routing decision of one call.
struct RouteInfo {
    int idx[kMaxTok][kMaxTopK];    // top-K experts per token, descending
    float w[kMaxTok][kMaxTopK];    // their weights (renormalised if asked)
    unsigned emask[kMaxExperts / 32];        // routed local experts (bit e)
    unsigned tmask[kMaxExperts];             // tokens routed to expert e
    unsigned char kof[kMaxExperts][kMaxTok];  // k of (expert e, token t)
    int ulist[kMaxPairs];          // distinct local experts, ascending
    int nU;                        // number of distinct local experts
    int pad_[3];
};

struct LayerParams {
    const uint8_t *table;  // this layer's tiled blocks, experts [e0, e0+ne)
    TiledLayout tl;
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
    unsigned long long *xlog;  // [kMaxTok][E] tagged logits {tag, f32}
    uint32_t *actT;            // [ntok*K][I/2] bf16 activation pairs, pair-permuted
    unsigned *epochs;          // [kMaxCtas * kEpochStride] per-CTA call counters
    int *user_idx;    // optional [ntok][K]
    float *user_w;    // optional [ntok][K]
    float *user_scores;  // optional [ntok][E]
    int *err;         // device error word
    unsigned long long *trace;  // optional phase timestamps
    // geometry (host-planned)
    int stage_bytes, nstages;
    int gu_tile_rows, gu_nslices, gu_rows_max;  // pair-rows per tile (multiple of 8, divides I)
    int dn_tile_rows, dn_nslices, dn_rows_max, dn_group;
    int router_rows;  // router rows per CTA (max)
    int route_only;   // stop after routing (m1moe_cuda_router_topk)
    // shared-memory offsets (bytes, 16-aligned)
    int off_bars, off_ctl, off_xs, off_xsum, off_rrows, off_gup, off_dnp, off_keys, off_lpart,
        off_res;
};

// Geometry of the tile in a ring stage: distinct expert u, first row r0
// (pair-row of the expert for gate/up, row of h for down) and row count nr.
struct StageGeo {
    int u, r0, nr, pad_;
};

struct Ctl {
    RouteInfo route;
    uint64_t rbar;      // router rows landed
    unsigned tag;       // this call's tag (epoch + 1, never 0)
    int abort;
    int next_gu, next_dn;  // work-item counters
    int issued;            // tiles issued by the producer
    int a, b;              // this CTA's gate/up rows [a, b) of the distinct-expert row space
    int ntg, ntd;          // gate/up and down tiles of this CTA
    int stage_tile[kMaxStages];  // tile whose copy was last issued into each stage
    int stage_done[kMaxStages];  // work items finished on each stage's current tile
    StageGeo geo[kMaxStages];
    unsigned published[kMaxCtas / 32];  // CTAs seen to have published their activations
};

__device__ __forceinline__ bool is_local(const LayerParams &p, int e) {
    return e >= p.e0 && e < p.e0 + p.ne;
}

// ------------------------------------------------------- tagged words ----
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u32(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void ld_relaxed_2u64(const unsigned long long *p, unsigned long long &a,
                                                unsigned long long &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];"
                 : "=l"(a), "=l"(b)
                 : "l"(p)
                 : "memory");
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long tagged(unsigned tag, uint32_t payload) {
    return ((unsigned long long)tag << 32) | payload;
}

__device__ __forceinline__ void set_abort(Ctl &ctl, int *err) {
    *reinterpret_cast<volatile int *>(&ctl.abort) = 1;
    if (err) atomicOr(err, kErrWaitTimeout);
}

// Word index, inside one activation vector of I values, of the pair word
// holding rows R and R+4 (R % 8 < 4) in the pair-permuted chunk-transposed
// order of common.cuh (ppos / 2).
__device__ __forceinline__ int act_word(int R, int nchI) {
    return ((((R >> 3) & 3) * nchI + (R >> 5)) << 2) + (R & 3);
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_cta_shared(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
    return v;
}

__device__ __forceinline__ void or_release_cta_shared(unsigned *p, unsigned bits) {
    asm volatile("red.release.cta.shared::cta.or.b32 [%0], %1;" ::"r"(smem_addr(p)), "r"(bits)
                 : "memory");
}

// The 16 pairs of chunk c of an activation vector written by other CTAs in
// this call (L2-coherent loads).
__device__ __forceinline__ void load_pairs_cg(const uint32_t *vT, int nchI, int c, uint32_t (&xp)[16]) {
    const uint4 *p = reinterpret_cast<const uint4 *>(vT);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = __ldcg(p + (size_t)i * nchI + c);
        xp[4 * i + 0] = v.x;
        xp[4 * i + 1] = v.y;
        xp[4 * i + 2] = v.z;
        xp[4 * i + 3] = v.w;
    }
}

// Have all CTAs that wrote rows [R, R+32) of the distinct-expert row space
// published this call's activations?  Gate/up rows are split over the G CTAs
// in 8-row units, CTA w owning units [units*w/G, units*(w+1)/G), so unit U
// belongs to CTA ((U+1)*G - 1) / units.
__device__ __forceinline__ bool writers_published(const unsigned *epochs, unsigned *published, int R,
                                                  int units, int G, unsigned tag) {
    const int U0 = R >> 3;
    const int w0 = ((U0 + 1) * G - 1) / units;
    const int w1 = (min(U0 + 4, units) * G - 1) / units;
    for (int w = w0; w <= w1; ++w) {
        const unsigned bit = 1u << (w & 31);
        if (ld_acquire_cta_shared(&published[w >> 5]) & bit) continue;
        if (ld_acquire_u32(epochs + (size_t)w * kEpochStride) != tag) return false;
        or_release_cta_shared(&published[w >> 5], bit);
    }
    return true;
}

// ------------------------------------------------------------------ route ----
// Warp t routes token t: polls the E tagged logits, softmax (max-subtracted,
// expf, times 1/sum — InferenceEngine.swift:502-507), top-K by rank
// (descending, ties to the lower index, NaN lowest — :510-519),
// renormalisation in k order, then marks its local experts.  Returns false if
// the logits did not arrive in time.
__device__ bool route_token(const LayerParams &p, RouteInfo &rs, unsigned long long *keys, int t,
                            unsigned tag, const volatile int *abort, bool write_user) {
    const int lane = threadIdx.x & 31, E = p.E, K = p.K;
    float v[kLogitsPerLane];
    bool ok = false;
    const unsigned long long *lw = p.xlog + (size_t)t * E;
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        bool all = true;
#pragma unroll
        for (int j = 0; j < kLogitsPerLane; ++j) {
            const int e = lane + 32 * j;
            if (e < E) {
                const unsigned long long w = ld_relaxed_u64(lw + e);
                v[j] = __uint_as_float((uint32_t)w);
                all = all && (unsigned)(w >> 32) == tag;
            }
        }
        if (all) {
            ok = true;
            break;
        }
        if (*abort) break;
        __nanosleep(32);
    }
    if (!__all_sync(0xffffffffu, ok)) return false;
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kLogitsPerLane; ++j)
        if (lane + 32 * j < E) m = fmaxf(m, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kLogitsPerLane; ++j) {
        if (lane + 32 * j < E) {
            v[j] = expf(v[j] - m);
            s += v[j];
        }
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    unsigned long long *kt = keys + (size_t)t * E;
#pragma unroll
    for (int j = 0; j < kLogitsPerLane; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
            v[j] *= inv;
            if (write_user && p.user_scores) p.user_scores[(size_t)t * E + e] = v[j];
            // Probabilities are >= 0, so their bit patterns order like the
            // values; +1 leaves 0 for NaN (lowest).  The low half breaks ties
            // in favour of the lower index.  All keys are distinct.
            const uint32_t hi = (v[j] != v[j]) ? 0u : __float_as_uint(v[j]) + 1u;
            kt[e] = ((unsigned long long)hi << 32) | (uint32_t)(0xFFFF - e);
        }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kLogitsPerLane; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
            const unsigned long long ke = kt[e];
            int rank = 0;
#pragma unroll 8
            for (int f = 0; f < E; ++f) rank += kt[f] > ke ? 1 : 0;
            if (rank < K) {
                rs.idx[t][rank] = e;
                rs.w[t][rank] = v[j];
            }
        }
    }
    __syncwarp();
    if (p.norm) {
        float sum = 0.f;
        if (lane == 0)
            for (int k = 0; k < K; ++k) sum += rs.w[t][k];  // reduce(0) in k order
        sum = __shfl_sync(0xffffffffu, sum, 0);
        if (lane < K) rs.w[t][lane] = rs.w[t][lane] / sum;
        __syncwarp();
    }
    if (lane < K) {
        const int e = rs.idx[t][lane];
        if (write_user) {
            if (p.user_idx) p.user_idx[t * K + lane] = e;
            if (p.user_w) p.user_w[t * K + lane] = rs.w[t][lane];
        }
        if (is_local(p, e)) {
            atomicOr(&rs.tmask[e], 1u << t);
            rs.kof[e][t] = (unsigned char)lane;
            atomicOr(&rs.emask[e >> 5], 1u << (e & 31));
        }
    }
    return true;
}

// ------------------------------------------------------------ pipeline ----
// Wait until tile n occupies stage s and its bytes have landed (warp-uniform).
// The stage_tile check comes first because mbarrier.try_wait.parity(P) also
// succeeds while the barrier is still in the phase BEFORE the awaited one.
// Once stage_tile[s] == n, the previous phase of full[s] has completed (its
// consumers released the stage), so the parity wait targets tile n's phase.
__device__ __forceinline__ bool wait_tile(uint64_t *full, Ctl &ctl, int s, int n, int nstages,
                                          int *err) {
    bool ok = false;
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (*reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) == n) {
            ok = true;
            break;
        }
        if (*reinterpret_cast<volatile int *>(&ctl.abort)) break;
        __nanosleep(20);
    }
    if (!ok && !*reinterpret_cast<volatile int *>(&ctl.abort)) set_abort(ctl, err);
    if (ok) ok = mbar_wait(&full[s], (n / nstages) & 1, &ctl.abort, err);
    return __all_sync(0xffffffffu, ok);
}

// A work item finished reading stage s; the last of the tile's `items` items
// releases the stage to the producer.
__device__ __forceinline__ void release_item(uint64_t *empty, Ctl &ctl, int s, int items) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
        if (atomicAdd(&ctl.stage_done[s], 1) == items - 1) {
            ctl.stage_done[s] = 0;
            mbar_arrive(&empty[s]);
        }
    }
}

__device__ __forceinline__ int grab(int *counter) {
    int q = 0;
    if ((threadIdx.x & 31) == 0) q = atomicAdd(counter, 1);
    return __shfl_sync(0xffffffffu, q, 0);
}

__device__ __forceinline__ float swiglu(float g, float u) {
    return (g / (1.0f + expf(-g))) * u;  // Shaders.metal:147-148: SiLU(gate) * up
}

// Store the activations of rows R and R+4 of pair `pair` (R % 8 < 4).
__device__ __forceinline__ void put_act_pair(const LayerParams &p, int pair, int R, float lo,
                                             float hi) {
    const int nchI = p.I / kChunkCols;
    const uint32_t word = (uint32_t)f32_to_bf16_rn(lo) | ((uint32_t)f32_to_bf16_rn(hi) << 16);
    p.actT[(size_t)pair * (p.I / 2) + act_word(R, nchI)] = word;
}

// ---------------------------------------------------------------- kernel ----
template <int NT>
__global__ void __launch_bounds__(kLayerThreads, 1) k_moe_layer(const LayerParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RG = ItemRows<NT>::gu, PG = ItemRows<NT>::pairs, NPASS = ItemRows<NT>::passes;
    constexpr int RD = ItemRows<NT>::dn;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = (int)gridDim.x, blk = (int)blockIdx.x;
    const int NST = p.nstages, STG = p.stage_bytes;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.off_bars);
    uint64_t *empty = full + NST;
    Ctl &ctl = *reinterpret_cast<Ctl *>(smem + p.off_ctl);
    RouteInfo &rs = ctl.route;
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem + p.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + p.off_xsum);
    uint8_t *rrows = smem + p.off_rrows;
    float *gup = reinterpret_cast<float *>(smem + p.off_gup);
    float *dnp = reinterpret_cast<float *>(smem + p.off_dnp);
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smem + p.off_keys);
    float *lpart = reinterpret_cast<float *>(smem + p.off_lpart);
    float *resid = reinterpret_cast<float *>(smem + p.off_res);  // [ntok][rows] residual
    const volatile int *vabort = &ctl.abort;
    const int h = p.h, I = p.I, nch = h / kChunkCols, nchI = I / kChunkCols;
    const TiledLayout &tl = p.tl;
    unsigned *my_epoch = p.epochs + (size_t)blk * kEpochStride;

    if (tid == 0) trace_event(p.trace, 0, 0);
    // ---- phase 1: barriers, router-row prefetch, x staging ----
    const int nmine = (p.E > blk) ? (p.E - blk + G - 1) / G : 0;
    const int rowb = h * 2;
    if (tid == kConsumerThreads) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
            ctl.stage_tile[i] = -1;
            ctl.stage_done[i] = 0;
        }
        mbar_init(&ctl.rbar, 1);
        ctl.abort = 0;
        ctl.next_gu = ctl.next_dn = 0;
        ctl.issued = 0;
        mbar_fence_init();
        if (nmine > 0) {
            const uint64_t pol = l2_evict_first_policy();
            mbar_arrive_expect_tx(&ctl.rbar, (uint32_t)(nmine * rowb));
            for (int m = 0; m < nmine; ++m)
                bulk_g2s(rrows + m * rowb, p.router + (size_t)(blk + m * G) * h, (uint32_t)rowb,
                         &ctl.rbar, pol);
        }
    } else if (tid == kLayerThreads - 1) {
        const unsigned t1 = ld_relaxed_u32(my_epoch) + 1u;
        ctl.tag = t1 ? t1 : 1u;
    }
    // this CTA's rows of h (down projection, combine)
    const int i0 = (int)((long long)h * blk / G), i1 = (int)((long long)h * (blk + 1) / G);
    const int nrows = i1 - i0;
    for (int e = tid; e < p.E; e += kLayerThreads) rs.tmask[e] = 0u;
    if (tid < kMaxExperts / 32) rs.emask[tid] = 0u;
    for (int i = tid; i < kMaxCtas / 32; i += kLayerThreads) ctl.published[i] = 0u;
    // x: 4 consecutive values per thread, every load in flight at once
    {
        const int nx4 = p.ntok * h / 4;
#pragma unroll 4
        for (int q = tid; q < nx4; q += kLayerThreads) {
            const int t = (q * 4) / h, j = (q * 4) % h;
            float v[4];
            if (p.x_bf16) {
                const uint2 r = __ldg(reinterpret_cast<const uint2 *>(
                    reinterpret_cast<const uint16_t *>(p.x) + (size_t)t * h + j));
                v[0] = __uint_as_float(r.x << 16);
                v[1] = __uint_as_float(r.x & 0xFFFF0000u);
                v[2] = __uint_as_float(r.y << 16);
                v[3] = __uint_as_float(r.y & 0xFFFF0000u);
            } else {
                const float4 r = __ldg(reinterpret_cast<const float4 *>(
                    reinterpret_cast<const float *>(p.x) + (size_t)t * h + j));
                v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) xs[(size_t)t * h + ppos(j + u, nch)] = f32_to_bf16_rn(v[u]);
        }
        if (tid == 0) trace_event(p.trace, 0, 15);
        if (p.res) {
            for (int q = tid; q < p.ntok * nrows; q += kLayerThreads) {
                const int t = q / nrows, i = i0 + q % nrows;
                resid[q] = load_act(p.res, p.res_bf16, (size_t)t * h + i);
            }
        }
    }
    __syncthreads();
    if (tid == 0) trace_event(p.trace, 0, 1);
    const unsigned tag = ctl.tag;

    if (warp < 8) {
        // ---- phase 2: logits of this CTA's experts (warps 0..7) ----
        if (nmine > 0) {
            const bool landed = mbar_wait(&ctl.rbar, 0, &ctl.abort, p.err);
            if (named_sync_and(2, 256, landed)) {
                const size_t xtok = (size_t)h * (p.x_bf16 ? 2 : 4);
                for (int m = 0; m < nmine; ++m) {
                    const int e = blk + m * G;
                    const uint8_t *row = rrows + m * rowb;
                    float acc[NT];
#pragma unroll
                    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
                    for (int g8 = tid; g8 < h / 8; g8 += 256) {
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
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    acc[t] = fmaf(wf[j],
                                                  load_act(reinterpret_cast<const uint8_t *>(p.x) + t * xtok,
                                                           p.x_bf16, g8 * 8 + j),
                                                  acc[t]);
                            }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const float v = warp_sum(acc[t]);
                        if (lane == 0) lpart[warp * kMaxTok + t] = v;
                    }
                    named_sync(2, 256);
                    if (tid < p.ntok) {
                        float s = 0.f;
                        for (int w = 0; w < 8; ++w) s += lpart[w * kMaxTok + tid];
                        st_relaxed_u64(p.xlog + (size_t)tid * p.E + e, tagged(tag, __float_as_uint(s)));
                    }
                    named_sync(2, 256);
                }
            }
        }
        if (tid == 0) trace_event(p.trace, 0, 2);
        // ---- phase 3: route (warps 0..NT-1 of every CTA) ----
        if (warp < NT) {
            bool ok = true;
            if (warp < p.ntok && !*vabort) ok = route_token(p, rs, keys, warp, tag, vabort, blk == 0);
            if (!ok && lane == 0) set_abort(ctl, p.err);
            if (tid == 0) trace_event(p.trace, 0, 3);
            named_sync(3, NT * 32);
            if (warp == 0) {
                // distinct local experts, ascending, from the expert bit mask
                unsigned m = lane < kMaxExperts / 32 ? rs.emask[lane] : 0u;
                const int c = __popc(m);
                int incl = c;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                int pos = incl - c;
                while (m) {
                    rs.ulist[pos++] = lane * 32 + __ffs(m) - 1;
                    m &= m - 1;
                }
                const int nU = __shfl_sync(0xffffffffu, incl, 31);
                if (lane == 0) {
                    rs.nU = nU;
                    // gate/up rows [a, b) of the distinct-expert row space
                    // (expert u's rows are u*I .. u*I+I-1), cut in units of 8
                    // rows so that row pairs (R, R+4) stay together.
                    const int units = nU * (I / 8);
                    const int a = (int)((long long)units * blk / G) * 8;
                    const int b = (int)((long long)units * (blk + 1) / G) * 8;
                    const int GT = p.gu_tile_rows, DT = p.dn_tile_rows;
                    ctl.a = a;
                    ctl.b = b;
                    ctl.ntg = (b > a) ? (b - 1) / GT - a / GT + 1 : 0;
                    ctl.ntd = nrows > 0 ? nU * ((nrows + DT - 1) / DT) : 0;
                }
            }
        }
    }
    // xsum: the other warps, meanwhile
    if (tid >= 256) {
        for (int q = tid - 256; q < p.ntok * nch; q += kLayerThreads - 256) {
            const int t = q / nch, c = q % nch;
            uint32_t xp[16];
            load_pairs_any(xs + (size_t)t * h, nch, c, xp);
            xsum[q] = pair_sum(xp);
        }
    }
    __syncthreads();
    if (tid == 0) trace_event(p.trace, 0, 4);
    if (p.route_only || ctl.abort) {
        // uniform; no copies were issued
        if (tid == 0) st_relaxed_u32(my_epoch, tag);
        return;
    }

    // ---- phase 4/5 geometry ----
    const int GT = p.gu_tile_rows, DT = p.dn_tile_rows, DG = p.dn_group;
    const int a = ctl.a, b = ctl.b, ntg = ctl.ntg, ntd = ctl.ntd, nU = rs.nU;
    const int nslg = p.gu_nslices, nsld = p.dn_nslices;
    const int ipt_g = (GT / 2 / PG) * nslg;          // work items per gate/up tile
    const int ipt_d = ((DT + DG - 1) / DG) * nsld;  // work items per down tile

    if (warp == kConsumerWarps) {
        // ================= producer =================
        if (lane == 0) {
            trace_event(p.trace, 0, 19);
            const uint64_t pol = l2_evict_first_policy();
            int n = 0, s = 0, wrap = 0;
            bool ok = true;
            // Wait for stage s to be free, record its tile, copy.
            auto issue = [&](int u, int r0, int nr, const uint8_t *src, uint32_t bytes) {
                if (n >= NST && !mbar_wait(&empty[s], (wrap - 1) & 1, &ctl.abort, p.err)) return false;
                ctl.geo[s] = StageGeo{u, r0, nr, 0};
                __threadfence_block();
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(ring + (size_t)s * STG, src, bytes, &full[s], pol);
                *reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) = n;
                if (n == 0) trace_event(p.trace, 0, 11);
                ++n;
                if (++s == NST) {
                    s = 0;
                    ++wrap;
                }
                return true;
            };
            // gate/up tiles: [a, b) cut at multiples of GT (GT | I, so a tile
            // never crosses experts)
            int R = a, u = ntg ? a / I : 0, bound = (a / GT + 1) * GT;
            for (int k = 0; k < ntg && ok; ++k) {
                const int hi = min(bound, b), r0 = R - u * I;
                ok = issue(u, r0, hi - R,
                           p.table + (size_t)(rs.ulist[u] - p.e0) * tl.block + (size_t)r0 * tl.pr,
                           (uint32_t)((hi - R) * tl.pr));
                R = hi;
                bound += GT;
                if (R == (u + 1) * I) ++u;
            }
            // down tiles: expert by expert, this CTA's rows [i0, i1) in runs of DT
            for (int uu = 0; uu < nU && ok && ntd > 0; ++uu) {
                const uint8_t *blkp = p.table + (size_t)(rs.ulist[uu] - p.e0) * tl.block + tl.down_off;
                for (int r0 = i0; r0 < i1 && ok; r0 += DT) {
                    const int nr = min(DT, i1 - r0);
                    ok = issue(uu, r0, nr, blkp + (size_t)r0 * tl.dr, (uint32_t)(nr * tl.dr));
                }
            }
            ctl.issued = n;
            trace_event(p.trace, 0, 9);
        }
    } else {
        // ================= consumers: gate/up =================
        constexpr int kNg = 2 * RG * NT, kSg = 32 / kNg;
        const size_t wo_u = (size_t)h / 2 + 2 * tl.sbh;  // up part offset in a pair-row
        const int ng_items = ntg * ipt_g;
        for (;;) {
            const int q = grab(&ctl.next_gu);
            if (q >= ng_items) break;
            const int n = q / ipt_g, rem = q - n * ipt_g, pg = rem / nslg, j = rem - pg * nslg;
            const int s = n % NST;
            if (!wait_tile(full, ctl, s, n, NST, p.err)) break;
            if (q == 0 && lane == 0) trace_event(p.trace, 0, 5);
            const StageGeo g = ctl.geo[s];
            if (pg * PG < g.nr / 2) {
                const uint8_t *st = ring + (size_t)s * STG;
                const int e = rs.ulist[g.u];
                const unsigned mask = rs.tmask[e];
                float act_prev = 0.f;
#pragma unroll
                for (int pass = 0; pass < NPASS; ++pass) {
                    // tile-relative rows of this pass
                    int trow[RG];
#pragma unroll
                    for (int r = 0; r < RG; ++r) {
                        const int pu = NPASS == 1 ? pg * PG + (r >> 1) : pg;
                        const int half = NPASS == 1 ? (r & 1) : pass;
                        trow[r] = 8 * (pu >> 2) + (pu & 3) + 4 * half;
                    }
                    float acc[kNg];  // [(row * NT + token) * 2 + gate0/up1]
#pragma unroll
                    for (int i = 0; i < kNg; ++i) acc[i] = 0.f;
                    for (int ch = j * 32 + lane; ch < nch; ch += 32 * nslg) {
                        const int gi = (ch * kChunkCols) / p.gs;
#pragma unroll
                        for (int k = 0; k < NT; ++k) {
                            if (!((mask >> k) & 1u)) continue;
                            uint32_t xp[16];
                            load_pairs_any(xs + (size_t)k * h, nch, ch, xp);
                            const float X = xsum[k * nch + ch];
#pragma unroll
                            for (int r = 0; r < RG; ++r) {
                                const uint8_t *pr = st + (size_t)trow[r] * tl.pr;
                                const uint4 wg = *reinterpret_cast<const uint4 *>(pr + ch * 16);
                                const uint4 wu = *reinterpret_cast<const uint4 *>(pr + wo_u + ch * 16);
                                const uint16_t *sgp = reinterpret_cast<const uint16_t *>(pr + h / 2);
                                const uint16_t *sup = reinterpret_cast<const uint16_t *>(pr + wo_u + h / 2);
                                const float sg = bf16_bits(sgp[gi]);
                                const float bg = bf16_bits(sgp[tl.sbh / 2 + gi]);
                                const float su = bf16_bits(sup[gi]);
                                const float bu = bf16_bits(sup[tl.sbh / 2 + gi]);
                                float &ag = acc[(r * NT + k) * 2 + 0];
                                float &au = acc[(r * NT + k) * 2 + 1];
                                // s*(A - 128X) + b*X with A = sum (128+q) x
                                ag = fmaf(sg, dot_chunk_bf16(wg, xp), fmaf(fmaf(-128.f, sg, bg), X, ag));
                                au = fmaf(su, dot_chunk_bf16(wu, xp), fmaf(fmaf(-128.f, su, bu), X, au));
                            }
                        }
                    }
                    // lane holds value lane / kSg = (r*NT + k)*2 + m
                    const float tot = warp_reduce_multi(acc);
                    if (nslg == 1) {
                        const float upv = __shfl_down_sync(0xffffffffu, tot, kSg);
                        const float act = swiglu(tot, upv);  // meaningful where lane % (2kSg) == 0
                        const int jj = lane / (2 * kSg), r = jj / NT, k = jj % NT;
                        const bool lead = (lane % (2 * kSg)) == 0 && ((mask >> k) & 1u);
                        if (NPASS == 1) {
                            // slot r+1 (row R+4) is 2*kSg*NT lanes further on
                            const float other = __shfl_down_sync(0xffffffffu, act, 2 * kSg * NT);
                            if (lead && (r & 1) == 0) {
                                const int pu = pg * PG + (r >> 1);
                                put_act_pair(p, k * p.K + rs.kof[e][k],
                                             g.r0 + 8 * (pu >> 2) + (pu & 3), act, other);
                            }
                        } else if (pass == 0) {
                            act_prev = act;
                        } else if (lead) {
                            put_act_pair(p, k * p.K + rs.kof[e][k],
                                         g.r0 + 8 * (pg >> 2) + (pg & 3), act_prev, act);
                        }
                    } else if (lane % kSg == 0) {
                        const int v = lane / kSg, r = v / (2 * NT), km = v % (2 * NT);
                        const int lr = g.u * I + g.r0 + trow[r] - a;
                        gup[((size_t)lr * nslg + j) * (2 * NT) + km] = tot;
                    }
                }
            }
            release_item(empty, ctl, s, ipt_g);
        }
        if (tid == 0) trace_event(p.trace, 0, 17);
        named_sync(1, kConsumerThreads);  // every gate/up item of this CTA is done
        if (nslg > 1) {
            // sum the column slices in order, SwiGLU
            if (!ctl.abort) {
                for (int i = tid; i < (b - a) / 2 * NT; i += kConsumerThreads) {
                    const int slot = i / NT, k = i % NT;
                    const int lr = 8 * (slot >> 2) + (slot & 3);  // row R - a; R+4 is lr + 4
                    const int Ru = a + lr, u = Ru / I;
                    const int e = rs.ulist[u];
                    if (!((rs.tmask[e] >> k) & 1u)) continue;
                    float gv[2] = {0.f, 0.f}, uv[2] = {0.f, 0.f};
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh)
                        for (int jj = 0; jj < nslg; ++jj) {
                            const float *gp = gup + ((size_t)(lr + 4 * hh) * nslg + jj) * (2 * NT) + 2 * k;
                            gv[hh] += gp[0];
                            uv[hh] += gp[1];
                        }
                    put_act_pair(p, k * p.K + rs.kof[e][k], Ru - u * I, swiglu(gv[0], uv[0]),
                                 swiglu(gv[1], uv[1]));
                }
            }
            named_sync(1, kConsumerThreads);
        }
        if (tid == 0) {
            // publish this CTA's activations (also after an abort, so that no
            // other CTA waits for them until its own time limit)
            __threadfence();
            st_release_u32(my_epoch, tag);
            trace_event(p.trace, 0, 6);
        }

        // ================= consumers: down =================
        // An item is (tile, 32-chunk column slice, DG rows): each lane loads
        // one 32-value chunk of each routed token's activation once and uses
        // it for all the item's rows, RD at a time.
        constexpr int kSd = 32 / RD;
        const int rmax = p.dn_rows_max, units = nU * (I / 8);
        const int nd_items = ctl.abort ? 0 : ntd * ipt_d;
        for (;;) {
            const int q = grab(&ctl.next_dn);
            if (q >= nd_items) break;
            const int n = q / ipt_d, rem = q - n * ipt_d, grp = rem / nsld, j = rem - grp * nsld;
            const int s = (ntg + n) % NST;
            if (!wait_tile(full, ctl, s, ntg + n, NST, p.err)) break;
            if (q == 0 && lane == 0) trace_event(p.trace, 0, 18);
            const StageGeo g = ctl.geo[s];
            const int rg0 = grp * DG, nr = min(DG, g.nr - rg0);
            const int ch = j * 32 + lane;
            const bool have = ch < nchI && nr > 0;
            // this lane's 32 activation rows were written by one or two CTAs
            bool ok = !have;
            if (have) {
                for (uint32_t it = 0; it < kWaitLimit; ++it) {
                    if (writers_published(p.epochs, ctl.published, g.u * I + ch * kChunkCols, units,
                                          G, tag)) {
                        ok = true;
                        break;
                    }
                    if (*vabort) break;
                    __nanosleep(64);
                }
            }
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0 && !*vabort) set_abort(ctl, p.err);
                break;
            }
            if (lane == 0 && q == 0) trace_event(p.trace, 0, 12);
            if (nr > 0) {
                const uint8_t *st = ring + (size_t)s * STG + (size_t)rg0 * tl.dr;
                const int e = rs.ulist[g.u];
                const unsigned mask = rs.tmask[e];
                const int gi = have ? (ch * kChunkCols) / p.gs : 0;
                for (int k = 0; k < NT; ++k) {
                    if (!((mask >> k) & 1u)) continue;
                    const int pair = k * p.K + rs.kof[e][k];
                    uint32_t xp[16];
                    if (have) {
                        load_pairs_cg(p.actT + (size_t)pair * (I / 2), nchI, ch, xp);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) xp[i] = 0u;
                    }
                    const float X = pair_sum(xp);
                    if (lane == 0 && q == 0) {
                        asm volatile("" ::"f"(X));
                        trace_event(p.trace, 0, 14);
                    }
                    for (int r0 = 0; r0 < nr; r0 += RD) {
                        float y[RD];
#pragma unroll
                        for (int r = 0; r < RD; ++r) {
                            y[r] = 0.f;
                            if (have && r0 + r < nr) {
                                const uint8_t *pr = st + (size_t)(r0 + r) * tl.dr;
                                const uint4 w = *reinterpret_cast<const uint4 *>(pr + ch * 16);
                                const uint16_t *sp = reinterpret_cast<const uint16_t *>(pr + I / 2);
                                const float sc = bf16_bits(sp[gi]);
                                const float bi = bf16_bits(sp[tl.sbi / 2 + gi]);
                                y[r] = fmaf(sc, dot_chunk_bf16(w, xp), fmaf(fmaf(-128.f, sc, bi), X, 0.f));
                            }
                        }
                        const float tot = warp_reduce_multi(y);
                        if (lane % kSd == 0) {
                            const int r = lane / kSd;
                            if (r0 + r < nr)
                                dnp[((size_t)pair * rmax + (g.r0 + rg0 + r0 + r - i0)) * nsld + j] = tot;
                        }
                    }
                }
            }
            if (lane == 0 && q == 0) trace_event(p.trace, 0, 13);
            if (lane == 0 && q == 1) trace_event(p.trace, 0, 16);
            release_item(empty, ctl, s, ipt_d);
        }
        named_sync(1, kConsumerThreads);
        if (tid == 0) trace_event(p.trace, 0, 8);
        // moeCombine (Shaders.metal:360-376): residual first, then k ascending;
        // each expert output is its slices summed in order.  resid[qq] is
        // token qq / nrows, row i0 + qq % nrows (prefetched at kernel start).
        if (!ctl.abort) {
            for (int qq = tid; qq < p.ntok * nrows; qq += kConsumerThreads) {
                const int t = qq / nrows, i = i0 + qq % nrows;
                float acc = p.res ? resid[qq] : 0.f;
                for (int k = 0; k < p.K; ++k) {
                    if (!is_local(p, rs.idx[t][k])) continue;
                    const float *pp = dnp + ((size_t)(t * p.K + k) * rmax + (i - i0)) * nsld;
                    float y = 0.f;
                    for (int jj = 0; jj < nsld; ++jj) y += pp[jj];
                    acc = fmaf(rs.w[t][k], y, acc);
                }
                store_act(p.out, p.out_bf16, (size_t)t * h + i, acc);
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        trace_event(p.trace, 0, 10);
        st_relaxed_u32(my_epoch, tag);
    }
    if (ctl.abort && tid == 0) {
        // wait (bounded) for copies still in flight into this CTA's shared memory
        for (int n = ctl.issued - NST; n < ctl.issued; ++n) {
            if (n < 0) continue;
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(&full[n % NST], (n / NST) & 1)) break;
        }
    }
}

}  // namespace m1
