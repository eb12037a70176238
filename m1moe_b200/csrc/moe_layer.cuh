// moe_layer.cuh — one MoE block for a decode batch of 1..8 tokens in ONE
// kernel (sm_100a).
//
// Replaces the MoE part of InferenceEngine.runLayer (InferenceEngine.swift
// :240-266): the CPU router (:490-519), loadExpert x K (:271-280) and CMD3 =
// K x (gate matvec4bit, up matvec4bit, swiGLU, down matvec4bit) + moeCombine
// (:401-478; Shaders.metal:39-92, 138-149, 360-376).
//
// One CTA per SM (cooperative launch: every CTA is resident, which the waits
// on other CTAs need).  Phases:
//   1. warps 8..24 initialise this CTA's rows of the output with the
//      residual (or zero) and, once this CTA's logits are out, stage x in
//      shared memory as int16 chunks with per-chunk scales and exact fp32
//      sums (common.cuh); meanwhile
//   2. warps 0..7 compute logits[t][e] = W_r[e] . x[t] for this CTA's experts
//      straight from global memory (bf16 router upcast exactly, the caller's
//      x, fp32 FMA, fixed reduction order), publish them as TAGGED words
//      (below) and
//   3. route every token from all logits (identical in every CTA,
//      deterministic): top-K by rank (descending, ties to the lower index),
//      the distinct local experts, their token slots and this CTA's share of
//      the rows; the softmax weights (with optional renormalisation) are
//      computed while the first copies are in flight;
//   4. the routed experts' gate/up rows, concatenated, are split over the CTAs
//      in runs of 8 rows (evenly for one token, else by the cost beta + tokens
//      of each expert's rows).  A producer warp streams this CTA's gate/up tiles and
//      then the matching COLUMNS of the down matrices (split-K; the table
//      stores them column-block major, tiled_layout.cuh) through a ring of
//      shared-memory stages, one or two bulk copies per tile.  24 consumer
//      warps compute SwiGLU activations for the CTA's rows into shared memory
//      (fp32, then int16 per group of gs rows with the group's scale), then
//      each row of h's partial sum over those columns, and add
//      weight_k * partial into the output with fp32 atomics.  Both
//      projections multiply nibbles with int16 activations by dp2a into int32
//      per chunk or group, scaled in fp32 (common.cuh).
//
// There is no grid-wide barrier.  Every CTA keeps a call counter in its own
// epoch word (one 128-byte line per CTA); all CTAs start a call with the same
// value, so tag = epoch + 1 names the call everywhere without communication.
// A logit travels as one 64-bit word {tag, f32} (relaxed gpu-scope 64-bit
// accesses are single-copy atomic), so a reader that sees the tag sees the
// value.  A CTA release-stores the tag into its epoch word once its output
// rows are initialised; before its first atomic a CTA waits (acquire) until
// every epoch word carries the tag, which normally holds long before.
// Expert contributions are summed by atomics in no fixed order: the output is
// within rounding of the reference's moeCombine order, not bitwise repeatable.
// For bf16 output the sums go to an fp32 accumulator and the last CTA to
// finish converts it.  All waits are bounded; on timeout the CTA sets the
// device error word and unwinds.
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
constexpr int kLayerSlots = 32;  // tiles in flight per CTA at most (a power of two)
constexpr int kMaxCtas = 1024;
constexpr int kEpochStride = 32;  // words between two CTAs' epoch words (own 128-byte line)
constexpr int kMaxRanks = 8;      // expert-parallel ranks joined over peer memory

// Expert parallelism over NVLink peer memory: every rank owns one exchange
// region (its own device memory, mapped into the other ranks' address space)
// laid out the same way on all ranks, for `world` ranks of `b` tokens:
//   [0]                   x-ready flags, one 128-byte line per source rank
//   [world*128]           done flags, one 128-byte line per source rank
//   [2*world*128]         the call counter (one line)
//   [xs_off]              gathered x, f32 [2][world*b][h] (by call parity)
//   [rt_off]              gathered routing: idx int32 [2][world*b][kMaxTopK], then
//                         weights f32 [2][world*b][kMaxTopK]
//   [recv_off]            partial sums received, tagged words {call tag, f32}
//                         [2][world][b][h]: each value carries its call's tag, so
//                         a receiver polls the values themselves (no flag, no
//                         system-scope fence on the sender's side)
struct EpLayout {
    long long xs_off, rt_off, recv_off, bytes;
};

__host__ __device__ inline EpLayout ep_layout(int world, int b, int h) {
    EpLayout l;
    l.xs_off = (2LL * world + 1) * 128;
    l.rt_off = l.xs_off + 2LL * world * b * h * 4;
    l.recv_off = l.rt_off + 2LL * 2 * world * b * 16 * 4;
    l.bytes = l.recv_off + 2LL * world * b * h * 8;
    return l;
}

// Gate/up work items for NT tokens: an item covers PG "row pairs" (rows R and
// R+4 of an expert, R % 8 < 4: the two rows whose activations share one
// pair-permuted word), computing RG rows at a time in NPASS passes.
template <int NT>
struct ItemRows {
    static constexpr int gu = NT == 1 ? 4 : (NT == 2 ? 2 : 1);  // RG
    static constexpr int pairs = gu >= 2 ? gu / 2 : 1;          // PG
    static constexpr int passes = gu >= 2 ? 1 : 2;              // NPASS
};

// Batches of 4 and 8 work in token SLOTS: slot j of distinct expert u is the
// j-th token (ascending) routed to it, and the inner loops are instantiated
// for the expert's token count, so no lane tests token bits or multiplies
// for a token the expert does not see.  A gate/up item is then ONE row of a
// tile for all of the expert's tokens; smaller batches keep the row-group
// items above (with column slices for 1 and 2 tokens).
// The host takes the slot path for 4 and 8 tokens, and for 2 tokens when rows
// are long (h >= 4096: the row-group items would hold a quarter of a row).
__host__ __device__ constexpr bool slot_path(int nt, int h) { return nt >= 4 || (nt == 2 && h >= 4096); }

__host__ __device__ constexpr int gu_items_per_tile(bool slot, int nt, int gt, int nslices) {
    return slot ? gt : (gt / 2 / (nt == 1 ? 2 : 1)) * nslices;  // rows, or row groups x slices
}

// Relative cost of a unit of 8 gate/up rows of an expert with t tokens
// (the same rows of the down matrices included): beta + t.  beta weighs the
// bytes, which do not depend on t, against the per-token arithmetic; the
// rows are split so that every CTA gets the same total cost.
#ifndef M1_BAL_BETA
#define M1_BAL_BETA 2
#endif
constexpr int kBalBeta = M1_BAL_BETA;

// The routing decision of one call.
struct RouteInfo {
    int idx[kMaxTok][kMaxTopK];    // top-K experts per token, descending
    float w[kMaxTok][kMaxTopK];    // their weights (renormalised if asked)
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
    void *out;        // must not overlap x
    int out_bf16;
    int out_acc;      // sums go to acc, the last CTA writes out (bf16, or f32 not 16-byte aligned)
    float *acc;       // [ntok][h] fp32 sums for bf16 output
    int *done;        // CTAs finished with their atomics (bf16 output)
    unsigned long long *xlog;  // [nbox][box_words] tagged logits {tag, f32}, box = [ntok][E][lparts]
    int nbox, box_words;       // logit boxes (CTA c reads box c % nbox) and their stride
    int lparts;                // partial sums per logit (h cut into lparts column ranges)
    unsigned *epochs;          // [kMaxCtas * kEpochStride] per-CTA call counters
    int *user_idx;    // optional [ntok][K]
    float *user_w;    // optional [ntok][K]
    float *user_scores;  // optional [ntok][E]
    int *err;         // device error word
    uint32_t ep_wait_limit;     // polls before an expert-parallel flag wait gives up
    unsigned long long *trace;  // optional phase timestamps
    // expert parallelism (ep_world > 1): tokens [ep_rank*ep_b, +ep_b) of the
    // ntok = ep_world*ep_b are this rank's (x, residual and out point at them);
    // ep_base[r] is rank r's exchange region as mapped here
    int ep_world, ep_rank, ep_b;
    uint8_t *ep_base[kMaxRanks];
    // routing made at each token's owner (ep_pre): this rank's own tokens'
    // top-K [ep_b][K] (a route-only call just before), pushed with the tokens
    int ep_pre;
    const int *ep_own_idx;
    const float *ep_own_w;
    // geometry (host-planned)
    int stage_bytes;       // largest tile (bytes)
    int ring_bytes;        // bytes of the tile ring
    int gu_tile_rows, gu_nslices, gu_rows_max;  // pair-rows per tile (multiple of 8, divides I)
    int dn_max_cb;    // column blocks per down tile (a multiple of gs/8)
    int act_cb;       // activation capacity, column blocks per token (gu_rows_max / 8)
    int xseg_max;     // activation groups per token (scale and sum)
    int route_only;   // stop after routing (m1moe_cuda_router_topk)
    int bal_beta;     // 0: rows split evenly; else cost-weighted split (kBalBeta)
    int nic;          // row chunks of the down matrices (h / tl.rc)
    // divisors known on the host: grid, gate/up tile rows, I, column blocks
    // per expert and per group, group size, items per gate/up tile, column
    // slices, items per down tile
    FastDiv fd_G, fd_GT, fd_I, fd_ncbE, fd_gcb, fd_gs, fd_iptg, fd_nslg, fd_iptd;
    // shared-memory offsets (bytes, 16-aligned)
    int off_bars, off_ctl, off_xs, off_xsum, off_gup, off_actf, off_act, off_xseg, off_blk, off_keys,
        off_rlog,
        off_lpart, off_slots;
};

// The tile in a ring slot.  Gate/up: distinct expert u, first pair-row r0 of
// the expert, row count nr (ic = -1).  Down: distinct expert u, first column
// block cb0 (in the concatenated row space, 8 rows per block), ncb blocks,
// row chunk ic.  off: its first byte in the ring.
struct StageGeo {
    int u, r0, nr, ic, off;
};

// A tile's bulk copies: b0 bytes from src0, then b1 bytes from src1.
struct TileCopy {
    const uint8_t *src0, *src1;
    uint32_t b0, b1;
    StageGeo g;
};

struct Ctl {
    RouteInfo route;
    unsigned tag;       // this call's tag (epoch + 1, never 0)
    int abort;
    int route_ok;       // warps 0..7 routed this call (written before barrier 3)
    int next_gu, next_dn;  // work-item counters
    int issued;            // tiles issued by the producer
    int a, b;              // this CTA's gate/up rows [a, b) of the distinct-expert row space
    int range[2];          // cost-weighted split: this CTA's units [range[0], range[1])
    int ntg, ntd;          // gate/up and down tiles of this CTA
    int nsub;              // down tiles per row chunk (ntd = nsub * nic)
    int last;              // this CTA finished last (bf16 output)
    int epochs_seen;       // every CTA's output rows are initialised (1)
    int stage_tile[kMaxStages];  // tile whose copy was last issued into each slot
    int stage_done[kMaxStages];  // work items finished on each slot's current tile
    int vstart[kMaxStages];      // producer: running byte position of each slot's tile
    StageGeo geo[kMaxStages];
    TileCopy copy[32];           // producer: the next (up to) 32 tiles' copies
};

// Token slots of the distinct experts (slot path only; a shared-memory
// region of its own, so that smaller batches keep the bytes for tiles).
struct Slots {
    unsigned char ute[kMaxExperts];            // tokens of expert e
    unsigned char utok[kMaxExperts][kMaxTok];  // its token slots: j-th token, ascending
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

__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Two adjacent tagged words in one 16-byte store (each 64-bit element is
// single-copy atomic on its own, which is all a reader relies on).
__device__ __forceinline__ void st_relaxed_v2_u64(unsigned long long *p, unsigned long long a,
                                                  unsigned long long b) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu_s32(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long tagged(unsigned tag, uint32_t payload) {
    return ((unsigned long long)tag << 32) | payload;
}

__device__ __forceinline__ int ld_acquire_cta_shared(const int *p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];"
                 : "=r"(v)
                 : "r"((unsigned)__cvta_generic_to_shared(p))
                 : "memory");
    return v;
}

__device__ __forceinline__ void st_release_cta_shared(int *p, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(p)),
                 "r"(v)
                 : "memory");
}

__device__ __forceinline__ void set_abort(Ctl &ctl, int *err) {
    *reinterpret_cast<volatile int *>(&ctl.abort) = 1;
    if (err) atomicOr(err, kErrWaitTimeout);
}

// One warp: wait until every CTA's epoch word carries `tag` (all output rows
// initialised for this call), then fence (acquire).  Loads of a round are all
// in flight at once; rounds back off.  Returns false on timeout or abort.
__device__ bool wait_all_epochs(const unsigned *epochs, int G, unsigned tag,
                                const volatile int *abort) {
    const int lane = threadIdx.x & 31;
    for (int w0 = 0; w0 < G; w0 += 256) {
        bool ok = false;
        for (uint32_t it = 0, nap = 64; it < kWaitLimit; ++it) {
            unsigned v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int w = w0 + 32 * k + lane;
                v[k] = w < G ? ld_relaxed_u32(epochs + (size_t)w * kEpochStride) : tag;
            }
            bool mine = true;
#pragma unroll
            for (int k = 0; k < 8; ++k) mine = mine && v[k] == tag;
            if (__all_sync(0xffffffffu, mine)) {
                ok = true;
                break;
            }
            if (*abort) break;
            __nanosleep(nap);
            nap = min(nap * 2, 512u);
        }
        if (!ok) return false;
    }
    __threadfence();
    return true;
}

// ------------------------------------------------------------------ route ----
// Top-K (descending, ties to the lower index — InferenceEngine.swift:510-519)
// by the 256 threads of warps 0..7, then the local-expert marks.  The ranking
// is taken on the logits, which order like the softmax probabilities (softmax
// is monotonic), so the softmax itself (route_weights) is off the path to the
// first weight copy; NaN ranks lowest and -0 equals +0.  rlog/keys: shared
// [ntok][E].  Returns false if the logits did not arrive in time (uniform
// over the 256 threads).
__device__ __forceinline__ unsigned long long logit_key(float v, int e) {
    const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
    uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    if (v != v) ord = 0u;
    return ((unsigned long long)ord << 32) | (uint32_t)(0xFFFF - e);
}

template <int NT, bool SL>
__device__ bool route_cta(const LayerParams &p, RouteInfo &rs, Slots &sl, int *range, float *rlog,
                          unsigned long long *keys, float *parts, unsigned tag, const volatile int *abort,
                          bool pre = false) {
    const int tid = threadIdx.x;
    const int E = p.E, K = p.K, ntok = p.ntok, nel = ntok * E;
    // marks of token t's k-th expert: the caller's index output, and for a
    // local expert its token mask and the token's k
    auto mark = [&](int t, int k) {
        const int e = rs.idx[t][k];
        if (p.user_idx && blockIdx.x == 0) p.user_idx[t * K + k] = e;
        if (is_local(p, e)) {
            atomicOr(&rs.tmask[e], 1u << t);
            rs.kof[e][t] = (unsigned char)k;
        }
    };
    if (!pre) {
    // a. collect the tagged (partial) logits: all of this thread's loads in
    //    flight at once.  Slot path: word (e, part, t) at (e*LP + part)*NT + t,
    //    t < ntok; otherwise word (t, e) at t*E + e.  nw <= kMaxTok * kMaxExperts.
    const int LP = SL ? p.lparts : 1, nw = SL ? E * LP * NT : nel;
    constexpr int kPer = kMaxTok * kMaxExperts / 256;
    const unsigned long long *box = p.xlog + (size_t)(blockIdx.x % p.nbox) * p.box_words;
    auto used = [&](int i) { return i < nw && (!SL || (i & (NT - 1)) < ntok); };
    bool ok = false;
    unsigned long long w[kPer];
    for (uint32_t it = 0, nap = 32; it < kWaitLimit; ++it) {
        bool all = true;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = tid + 256 * j;
            if (used(i)) w[j] = ld_relaxed_u64(box + i);
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j)
            if (used(tid + 256 * j)) all = all && (unsigned)(w[j] >> 32) == tag;
        if (all) {
            ok = true;
            break;
        }
        if (*abort) break;
        __nanosleep(nap);
        nap = min(nap * 2, 64u);  // the wait is short: keep the wake-up lag small
    }
    // b. the logit of (token, expert) element t*E + e (its parts summed in
    //    order) and its ranking key
    auto put = [&](int t, int e, float v) {
        rlog[t * E + e] = v;
        keys[t * E + e] = logit_key(v, e);
    };
    if constexpr (SL) {
        if (LP > 1) {
#pragma unroll
            for (int j = 0; j < kPer; ++j)
                if (used(tid + 256 * j)) parts[tid + 256 * j] = __uint_as_float((uint32_t)w[j]);
            named_sync(2, 256);
            for (int i = tid; i < nel; i += 256) {
                int t = 0, e = i;
                while (e >= E) {
                    e -= E;
                    ++t;
                }
                float v = 0.f;
                for (int q = 0; q < LP; ++q) v += parts[(e * LP + q) * NT + t];
                put(t, e, v);
            }
        } else {
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int i = tid + 256 * j;
                if (used(i)) put(i & (NT - 1), i / NT, __uint_as_float((uint32_t)w[j]));
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = tid + 256 * j;
            if (i < nel) {
                int e = i;
                while (e >= E) e -= E;
                const float v = __uint_as_float((uint32_t)w[j]);
                rlog[i] = v;
                keys[i] = logit_key(v, e);
            }
        }
    }
    if (!named_sync_and(2, 256, ok)) return false;
    if (tid == 0) trace_event(p.trace, 0, 12);
    // b. rank of every (token, expert).  Many tokens over at most 64 experts
    //    (slot path, more than 256 elements): a warp per token holds its keys
    //    in registers, two per lane, and counts the larger ones over 32
    //    shuffle rounds.  Otherwise P threads per element, each counting the
    //    keys above it in one slice of the token's E keys.
    if (SL && E <= 64 && nel > 256) {
        const int lane = tid & 31;
        for (int t = tid >> 5; t < ntok; t += 8) {
            const unsigned long long *kt = keys + (size_t)t * E;
            // absent slots hold 0, below every key (a key's low bits hold 0xFFFF - e)
            const unsigned long long k0 = lane < E ? kt[lane] : 0ull, k1 = lane + 32 < E ? kt[lane + 32] : 0ull;
            int c0 = 0, c1 = 0;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) {
                const unsigned long long a = __shfl_sync(0xffffffffu, k0, j), b = __shfl_sync(0xffffffffu, k1, j);
                c0 += (a > k0 ? 1 : 0) + (b > k0 ? 1 : 0);
                c1 += (a > k1 ? 1 : 0) + (b > k1 ? 1 : 0);
            }
            if (lane < E && c0 < K) rs.idx[t][c0] = lane;
            if (lane + 32 < E && c1 < K) rs.idx[t][c1] = lane + 32;
        }
    } else {
        int lp = 0;
        while (lp < 5 && (nel << (lp + 1)) <= 256) ++lp;
        const int P = 1 << lp;
        for (int base = 0; base < (nel << lp); base += 256) {
            const int gidx = base + tid, i = gidx >> lp, part = gidx & (P - 1);
            int cnt = 0, t = 0, e = i;
            if (i < nel) {
                while (e >= E) {
                    e -= E;
                    ++t;
                }
                const unsigned long long *kt = keys + (size_t)t * E;
                const unsigned long long ki = kt[e];
                // four independent loads in flight per round (a plain loop waits
                // out each shared-memory load in turn)
                int f = part;
                for (; f + 3 * P < E; f += 4 * P) {
                    const unsigned long long k0 = kt[f], k1 = kt[f + P], k2 = kt[f + 2 * P], k3 = kt[f + 3 * P];
                    cnt += (k0 > ki ? 1 : 0) + (k1 > ki ? 1 : 0) + (k2 > ki ? 1 : 0) + (k3 > ki ? 1 : 0);
                }
                for (; f < E; f += P) cnt += kt[f] > ki ? 1 : 0;
            }
            for (int o = 1; o < P; o <<= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
            if (i < nel && part == 0 && cnt < K) rs.idx[t][cnt] = e;
        }
    }
    named_sync(2, 256);
    if (tid == 0) trace_event(p.trace, 0, 13);
    }  // !pre (with pre, rs.idx holds the owners' routing and tmask is zero)
    // c. local-expert marks
    for (int i = tid; i < ntok * K; i += 256) {
        int t = 0, k = i;
        while (k >= K) {
            k -= K;
            ++t;
        }
        mark(t, k);
    }
    named_sync(2, 256);
    // d. one thread per expert e (E <= 256): on the slot path its token slots;
    //    with the cost-weighted split (route_geometry), this CTA's range of
    //    units -- a block scan of the costs beta + t of the routed local
    //    experts in ascending order, and the thread whose expert holds a
    //    cost target writes the unit there.  Done here by 256 threads rather
    //    than by the producer warp alone, whose path leads to the first copy.
    const int e = tid;
    const unsigned tm = e < E ? rs.tmask[e] : 0u;
    const int te = __popc(tm);
    if constexpr (SL) {
        if (te) {
            unsigned m = tm;
            int j = 0;
            while (m) {
                sl.utok[e][j++] = (unsigned char)(__ffs(m) - 1);
                m &= m - 1;
            }
            sl.ute[e] = (unsigned char)te;
        }
    }
    // the distinct local experts in ascending order (ulist, nU) and, with
    // the cost-weighted split, this CTA's range: block scans of one per
    // routed expert and of its cost
    const int lane = tid & 31, warp = tid >> 5, n8 = p.I >> 3;
    const int c = (p.bal_beta > 0 && te) ? p.bal_beta + te : 0, one = te ? 1 : 0;
    int ci = c, ui = one;  // inclusive prefixes within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int yc = __shfl_up_sync(0xffffffffu, ci, o), yu = __shfl_up_sync(0xffffffffu, ui, o);
        if (lane >= o) {
            ci += yc;
            ui += yu;
        }
    }
    int *wt = reinterpret_cast<int *>(parts);  // warp totals (the ring is idle until routing ends)
    if (lane == 31) {
        wt[2 * warp] = ci;
        wt[2 * warp + 1] = ui;
    }
    named_sync(2, 256);
    int cpre = ci - c, upre = ui - one, ctot = 0, utot = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const int wc = wt[2 * w], wu = wt[2 * w + 1];
        if (w < warp) {
            cpre += wc;
            upre += wu;
        }
        ctot += wc;
        utot += wu;
    }
    if (te) rs.ulist[upre] = e;
    if (tid == 0) rs.nU = utot;
    if (p.bal_beta > 0) {
        // costs are ints: total * G < 2^31 (checked on the host)
        const int total = ctot * n8, blk = blockIdx.x;
        const int T[2] = {fdiv(total * blk, p.fd_G), fdiv(total * (blk + 1), p.fd_G)};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            if (te && T[q] >= cpre * n8 && T[q] < (cpre + c) * n8)
                range[q] = upre * n8 + (T[q] - cpre * n8 + c - 1) / c;
            if (tid == 0 && T[q] >= total) range[q] = utot * n8;
        }
    }
    return true;
}

// The weights of token t's selected experts (one warp): softmax statistics
// over all E logits, w_k = exp(l_k - max) * (1/sum), optional renormalisation
// (reduce(0) in k order); CTA 0 also writes the caller's outputs.  Only the
// final combine reads the weights.
__device__ void route_weights(const LayerParams &p, RouteInfo &rs, const float *rlog, int t) {
    const int lane = threadIdx.x & 31, E = p.E, K = p.K;
    const float *lt = rlog + (size_t)t * E;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, lt[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int e = lane; e < E; e += 32) s += expf(lt[e] - m);
    s = warp_sum(s);
    const float inv = 1.0f / s;
    const bool user = blockIdx.x == 0;
    if (user && p.user_scores)
        for (int e = lane; e < E; e += 32) p.user_scores[(size_t)t * E + e] = expf(lt[e] - m) * inv;
    if (lane < K) rs.w[t][lane] = expf(lt[rs.idx[t][lane]] - m) * inv;
    __syncwarp();
    if (p.norm) {
        float sum = 0.f;
        if (lane == 0)
            for (int k = 0; k < K; ++k) sum += rs.w[t][k];
        sum = __shfl_sync(0xffffffffu, sum, 0);
        if (lane < K) rs.w[t][lane] = rs.w[t][lane] / sum;
    }
    if (user && p.user_w && lane < K) p.user_w[t * K + lane] = rs.w[t][lane];
}

// ------------------------------------------------------------ pipeline ----
// ------------------------------------------------------------ pipeline ----
// Wait until tile n occupies slot s and its bytes have landed (warp-uniform).
// The stage_tile check comes first because mbarrier.try_wait.parity(P) also
// succeeds while the barrier is still in the phase BEFORE the awaited one.
// Once stage_tile[s] == n, the previous phase of full[s] has completed (its
// consumers released the stage), so the parity wait targets tile n's phase.
__device__ __forceinline__ bool wait_tile(uint64_t *full, Ctl &ctl, int s, int n, int nstages,
                                          int *err) {
    bool ok = false;
    // Spinning warps take issue slots from the working ones: back off.
    for (uint32_t i = 0, nap = 64; i < kWaitLimit; ++i) {
        if (*reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) == n) {
            ok = true;
            break;
        }
        if (*reinterpret_cast<volatile int *>(&ctl.abort)) break;
        __nanosleep(nap);
        nap = min(nap * 2, 512u);
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

// End of the down-tile run that starts at column block cb (this CTA's blocks
// end at b8; ncbE blocks per expert, gcb per group): a run stays inside one
// expert, ends on a group boundary unless it ends the CTA's range (a group's
// bias term b*X uses the CTA's whole part of the group, so a group must not
// be split between two tiles), and spans at most mcb blocks from the start
// of cb's group, so it touches at most mcb/gcb groups (the stage holds mcb
// weight blocks and mcb/gcb scale/bias rows).
__device__ __forceinline__ int dn_run_end(const LayerParams &p, int cb, int b8) {
    const int ncbE = p.I >> 3, gcb = p.gs >> 3;
    const int uend = (fdiv(cb, p.fd_ncbE) + 1) * ncbE;
    return min(min(b8, uend), fdiv(cb, p.fd_gcb) * gcb + p.dn_max_cb);
}

// Rows of h per lane in a down item: several adjacent rows give one vector
// load per column block and one vector atomic per token, and independent
// dot-product chains; fewer for larger batches (registers: LR*NT of each of
// Q, y and the totals).
__host__ __device__ constexpr int dn_lane_rows(bool slot, int nt) {
    return nt <= 2 ? (slot ? 2 : 4) : (nt == 4 ? 2 : 1);  // the slot path keeps two Q chains per row
}


// LR consecutive 32-bit words from shared memory (4*LR-byte aligned).
template <int LR>
__device__ __forceinline__ void load_words(const uint32_t *p, uint32_t (&w)[LR]) {
    if constexpr (LR == 4) {
        const uint4 v = *reinterpret_cast<const uint4 *>(p);
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
    } else if constexpr (LR == 2) {
        const uint2 v = *reinterpret_cast<const uint2 *>(p);
        w[0] = v.x, w[1] = v.y;
    } else {
        w[0] = *p;
    }
}

// Add token t's LR row totals to LR consecutive floats of global memory
// (4*LR-byte aligned) with one vector atomic.
template <int LR, int NT>
__device__ __forceinline__ void add_words(float *dst, const float (&tot)[LR][NT], int t) {
    if constexpr (LR == 4) {
        atomicAdd(reinterpret_cast<float4 *>(dst), make_float4(tot[0][t], tot[1][t], tot[2][t], tot[3][t]));
    } else if constexpr (LR == 2) {
        atomicAdd(reinterpret_cast<float2 *>(dst), make_float2(tot[0][t], tot[1][t]));
    } else {
        atomicAdd(dst, tot[0][t]);
    }
}

// ------------------------------------------------------------ producer ----
// One warp, right after routing: this CTA's share of the work.  Gate/up rows [a, b)
// of the distinct-expert row space (expert u's rows are u*I .. u*I+I-1), cut
// in units of 8 rows so that row pairs (R, R+4) stay together; ntg gate/up
// tiles (cut at multiples of GT, so a tile never crosses experts) and ntd =
// nsub * nic down tiles (column-block runs, dn_run_end, per row chunk).
__device__ void route_geometry(const LayerParams &p, Ctl &ctl, int blk) {
    RouteInfo &rs = ctl.route;
    const int lane = threadIdx.x & 31;
    const int nU = rs.nU;  // the distinct local experts are in ulist (route_cta)
    const int n8 = p.I >> 3;  // units of 8 rows per expert
    int ua, ub;               // this CTA's units [ua, ub)
    if (p.bal_beta == 0) {
        const int units = nU * n8;  // units * G < 2^31 (kMaxPairs, I, kMaxCtas)
        ua = fdiv(units * blk, p.fd_G);
        ub = fdiv(units * (blk + 1), p.fd_G);
    } else {
        // cost-weighted: unit i of expert u costs c_u = beta + t_u, and the
        // boundary for a cost target T is the first unit whose preceding
        // cost reaches T, so that neighbouring CTAs agree on it (computed by
        // the router warps, route_cta)
        ua = ctl.range[0];
        ub = ctl.range[1];
    }
    if (lane == 0) {
        int a = ua * 8, b = ub * 8;
        if (b - a > p.gu_rows_max) {  // cannot happen (host bound); never overrun the buffers
            set_abort(ctl, p.err);
            b = a;
        }
        ctl.a = a;
        ctl.b = b;
        ctl.ntg = (b > a) ? fdiv(b - 1, p.fd_GT) - fdiv(a, p.fd_GT) + 1 : 0;
        int nsub = 0;
        for (int cb = a >> 3; cb < (b >> 3); cb = dn_run_end(p, cb, b >> 3)) ++nsub;
        ctl.nsub = nsub;
        ctl.ntd = nsub * p.nic;
    }
    __syncwarp();
}

// Producer state; lane 0 of the producer warp holds the authoritative copy
// (batch is kept by every lane).
struct Producer {
    int n = 0;        // next tile to issue
    int tail = 0;     // oldest tile whose release has not been seen
    int head = 0;     // running byte position of the next tile
    int pos = 0;      // head within the ring
    int batch = -1;   // tiles 32*batch .. +31 are described in ctl.copy
    bool ok = true;
};

// The copies of tile k.  Tile order: gate/up tiles, then the down tiles row
// chunk by row chunk, runs within a chunk in column order.
__device__ void describe_tile(const LayerParams &p, const Ctl &ctl, int k, TileCopy &c) {
    const TiledLayout &tl = p.tl;
    const RouteInfo &rs = ctl.route;
    const int a = ctl.a, b = ctl.b, ntg = ctl.ntg, ntd = ctl.ntd, nsub = ctl.nsub;
    const int GT = p.gu_tile_rows, RC = tl.rc, ncbE = p.I >> 3;
    if (k < ntg) {
        // gate/up: [a, b) cut at multiples of GT (GT | I, so a tile never
        // crosses experts)
        const int g0 = fdiv(a, p.fd_GT) + k;
        const int R = k == 0 ? a : g0 * GT, hi = min((g0 + 1) * GT, b);
        const int u = fdiv(R, p.fd_I), r0 = R - u * p.I;
        c.src0 = p.table + (size_t)(rs.ulist[u] - p.e0) * tl.block + (size_t)r0 * tl.pr;
        c.b0 = (uint32_t)((hi - R) * tl.pr);
        c.src1 = nullptr;
        c.b1 = 0;
        c.g = StageGeo{u, r0, hi - R, -1, 0};
    } else if (k < ntg + ntd) {
        // down: the same rows as columns of the down matrices, in runs
        // (dn_run_end)
        int j = k - ntg, ic = 0;
        while (j >= nsub) {
            j -= nsub;
            ++ic;
        }
        int cb = a >> 3;
        for (int q = 0; q < j; ++q) cb = dn_run_end(p, cb, b >> 3);
        const int cend = dn_run_end(p, cb, b >> 3);
        const int u = fdiv(cb, p.fd_ncbE), lcb = cb - u * ncbE, ncb = cend - cb;
        const int lg0 = fdiv(lcb, p.fd_gcb), lg1 = fdiv(lcb + ncb - 1, p.fd_gcb);
        const uint8_t *blkp = p.table + (size_t)(rs.ulist[u] - p.e0) * tl.block;
        c.src0 = blkp + tl.dn_w + ((size_t)ic * tl.ncbI + lcb) * RC * 4;
        c.b0 = (uint32_t)(ncb * RC * 4);
        c.src1 = blkp + tl.dn_sb + ((size_t)ic * tl.ngI + lg0) * RC * 4;
        c.b1 = (uint32_t)((lg1 - lg0 + 1) * RC * 4);
        c.g = StageGeo{u, cb, ncb, ic, 0};
    }
}

// Lane l describes tile 32*batch + l into ctl.copy[l] (the lanes work in
// parallel).
__device__ __forceinline__ void describe_tiles(const LayerParams &p, Ctl &ctl, int batch) {
    const int lane = threadIdx.x & 31;
    describe_tile(p, ctl, batch * 32 + lane, ctl.copy[lane]);
}

// Lane 0: issue the described tiles of the current batch in order.  Tile n
// takes slot n % kLayerSlots and the next bytes of the ring (tiles back to
// back; one that would run past the end starts at 0).  Slots and bytes come
// free in tile order, so this waits, oldest tile first, for as many releases
// as the new tile needs -- unless may_wait is false (the consumers have not
// started yet): then it stops before such a tile and returns false.
__device__ bool issue_batch(const LayerParams &p, Ctl &ctl, uint8_t *ring, uint64_t *full,
                            uint64_t *empty, Producer &ps, bool may_wait, uint64_t pol,
                            int ntiles) {
    constexpr int NSL = kLayerSlots;
    const int RB = p.ring_bytes, end = min(ntiles, (ps.batch + 1) * 32);
    while (ps.ok && ps.n < end) {
        const TileCopy c = ctl.copy[ps.n & 31];
        const int len = (int)((c.b0 + c.b1 + 127u) & ~127u);
        if (ps.pos + len > RB) {
            ps.head += RB - ps.pos;
            ps.pos = 0;
        }
        const bool slot_busy = ps.tail <= ps.n - NSL;
        const bool bytes_busy = ps.tail < ps.n && ps.head + len - ctl.vstart[ps.tail % NSL] > RB;
        if (!may_wait && (slot_busy || bytes_busy)) return false;
        while (ps.ok && ps.tail <= ps.n - NSL) {
            ps.ok = mbar_wait(&empty[ps.tail % NSL], (ps.tail / NSL) & 1, &ctl.abort, p.err);
            ps.tail += ps.ok;
        }
        while (ps.ok && ps.tail < ps.n && ps.head + len - ctl.vstart[ps.tail % NSL] > RB) {
            ps.ok = mbar_wait(&empty[ps.tail % NSL], (ps.tail / NSL) & 1, &ctl.abort, p.err);
            ps.tail += ps.ok;
        }
        if (!ps.ok) break;
        const int s = ps.n % NSL;
        ctl.vstart[s] = ps.head;
        StageGeo g = c.g;
        g.off = ps.pos;
        ctl.geo[s] = g;
        __threadfence_block();
        mbar_arrive_expect_tx(&full[s], c.b0 + c.b1);
        bulk_g2s(ring + ps.pos, c.src0, c.b0, &full[s], pol);
        if (c.b1) bulk_g2s(ring + ps.pos + c.b0, c.src1, c.b1, &full[s], pol);
        *reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) = ps.n;
        if (ps.n == 0) trace_event(p.trace, 0, 11);
        ++ps.n;
        ps.head += len;
        ps.pos += len;
    }
    return true;
}

// The producer warp: describe and issue tiles until `limit` tiles (or all)
// are issued, an error stops it, or (may_wait false) a tile would have to
// wait.
__device__ void produce(const LayerParams &p, Ctl &ctl, uint8_t *ring, uint64_t *full,
                        uint64_t *empty, Producer &ps, bool may_wait, uint64_t pol, int limit) {
    const int lane = threadIdx.x & 31;
    const int ntiles = min(ctl.ntg + ctl.ntd, limit);
    for (;;) {
        const int n = __shfl_sync(0xffffffffu, ps.n, 0);
        const bool ok = __shfl_sync(0xffffffffu, ps.ok, 0);
        if (!ok || n >= ntiles) break;
        if ((n >> 5) != ps.batch) {
            ps.batch = n >> 5;
            describe_tiles(p, ctl, ps.batch);
            __syncwarp();
        }
        bool more = true;
        if (lane == 0) more = issue_batch(p, ctl, ring, full, empty, ps, may_wait, pol, ntiles);
        more = __shfl_sync(0xffffffffu, more, 0);
        __syncwarp();  // ctl.copy may be rewritten next round
        if (!more) break;
    }
}

__device__ __forceinline__ float swiglu(float g, float u) {
    return (g / (1.0f + expf(-g))) * u;  // Shaders.metal:147-148: SiLU(gate) * up
}

// ------------------------------------------------------------ slot path ----
// One gate/up row (pair-row pr in the ring) for the TE token slots of its
// expert: lane = chunk of 32 columns; the chunk's weights are split into
// nibble planes once and shared by the tokens; per chunk and token
// acc += s*sx*Q + b*X for gate and up (common.cuh).  The SwiGLU activation
// of slot j lands in actf[j][lr].
template <int TE>
__device__ __forceinline__ void gu_row_te(const LayerParams &p, const uint8_t *pr, const unsigned char *tk,
                                          const uint32_t *xq, const float *xsc, const float *xsum,
                                          float *actf, int arows, int lr) {
    const int lane = threadIdx.x & 31, h = p.h, nch = h / kChunkCols;
    const size_t wo_u = (size_t)h / 2 + 2 * p.tl.sbh;  // up part of the pair-row
    const uint16_t *sgp = reinterpret_cast<const uint16_t *>(pr + h / 2);
    const uint16_t *sup = reinterpret_cast<const uint16_t *>(pr + wo_u + h / 2);
    const int bo = p.tl.sbh / 2;  // biases follow the scales
    int tok[TE];
#pragma unroll
    for (int j = 0; j < TE; ++j) tok[j] = tk[j];
    constexpr int NV = TE <= 1 ? 2 : (TE <= 2 ? 4 : (TE <= 4 ? 8 : 16));
    float acc[NV];  // [2*slot + gate0/up1], zero-padded to a power of two
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = 0.f;
    for (int ch = lane; ch < nch; ch += 32) {
        const int gi = fdiv(ch * kChunkCols, p.fd_gs);
        const uint4 wg = *reinterpret_cast<const uint4 *>(pr + ch * 16);
        const uint4 wu = *reinterpret_cast<const uint4 *>(pr + wo_u + ch * 16);
        const float sg = bf16_bits(sgp[gi]), bg = bf16_bits(sgp[bo + gi]);
        const float su = bf16_bits(sup[gi]), bu = bf16_bits(sup[bo + gi]);
        // up to 4 slots the split planes stay in registers across the slots;
        // beyond, registers go to the accumulators and the planes are split
        // again per slot
        uint32_t glo[4], ghi[4], ulo[4], uhi[4];
        if constexpr (TE <= 4) {
            split_nibbles(wg, glo, ghi);
            split_nibbles(wu, ulo, uhi);
        }
#pragma unroll
        for (int j = 0; j < TE; ++j) {
            uint32_t xp[16];
            load_pairs_any(reinterpret_cast<const uint16_t *>(xq + (size_t)tok[j] * (h / 2)), nch, ch, xp);
            const float X = xsum[tok[j] * nch + ch], sx = xsc[tok[j] * nch + ch];
            int Qg, Qu;
            if constexpr (TE <= 4) {
                Qg = dot_split_i16(glo, ghi, xp);
                Qu = dot_split_i16(ulo, uhi, xp);
            } else {
                Qg = dot_chunk_i16(wg, xp);
                Qu = dot_chunk_i16(wu, xp);
            }
            acc[2 * j] = fmaf(sg * sx, (float)Qg, fmaf(bg, X, acc[2 * j]));
            acc[2 * j + 1] = fmaf(su * sx, (float)Qu, fmaf(bu, X, acc[2 * j + 1]));
        }
    }
    // lane l holds value l / kS; the up value sits kS lanes above its gate
    const float tot = warp_reduce_multi(acc);
    constexpr int kS = 32 / NV;
    const float upv = __shfl_down_sync(0xffffffffu, tot, kS);
    const int j = lane / (2 * kS);
    if ((lane % (2 * kS)) == 0 && j < TE) actf[(size_t)j * arows + lr] = swiglu(tot, upv);
}

template <int NT>
__device__ __forceinline__ void gu_row_slots(int te, const LayerParams &p, const uint8_t *pr,
                                             const unsigned char *tk, const uint32_t *xq, const float *xsc,
                                             const float *xsum, float *actf, int arows, int lr) {
    switch (te) {
    case 1: gu_row_te<1>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
    case 2: gu_row_te<2>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
    case 3: gu_row_te<3>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
    case 4: gu_row_te<4>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
    default:
        if constexpr (NT > 4) {
            switch (te) {
            case 5: gu_row_te<5>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
            case 6: gu_row_te<6>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
            case 7: gu_row_te<7>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
            default: gu_row_te<8>(p, pr, tk, xq, xsc, xsum, actf, arows, lr); break;
            }
        }
    }
}

// One down tile (column blocks [r0, r0+nr) of one expert, this lane's LR rows
// of the row chunk) for the TE slots: per column block the LR weight words
// are split once and shared by the slots, whose activation blocks (int16
// pairs, slot-major) feed two dp2a chains each; per group
// y += s*sa*Q + b*X (common.cuh).
template <int TE, int LR, int NT>
__device__ __forceinline__ void dn_tile_te(const LayerParams &p, float (&y)[LR][NT], const uint32_t *Wt,
                                           const uint32_t *SBt, const StageGeo &g, const uint32_t *act,
                                           const float *xseg, int a8, int ag) {
    const int RC = p.tl.rc, gcb = p.gs >> 3;
    const int gfirst = fdiv(g.r0, p.fd_gcb);
    const uint4 *av = reinterpret_cast<const uint4 *>(act) + (g.r0 - a8);
    int Qa[LR][TE], Qb[LR][TE];
#pragma unroll
    for (int r = 0; r < LR; ++r)
#pragma unroll
        for (int j = 0; j < TE; ++j) Qa[r][j] = Qb[r][j] = 0;
    int gcur = gfirst, c = 0;
    int left = gcb - (g.r0 - gfirst * gcb);  // blocks of the first group in this tile
    while (c < g.nr) {
        const int cend = min(g.nr, c + left);
#pragma unroll 2
        for (; c < cend; ++c) {
            uint32_t wd[LR];
            load_words<LR>(Wt + (size_t)c * RC, wd);
            uint32_t lo[LR], hi[LR];
#pragma unroll
            for (int r = 0; r < LR; ++r) {
                lo[r] = wd[r] & 0x0F0F0F0Fu;
                hi[r] = wd[r] & 0xF0F0F0F0u;  // 16 * q: Qb is 16 times its sum
            }
#pragma unroll
            for (int j = 0; j < TE; ++j) {
                const uint4 v = av[c + (size_t)j * p.act_cb];
#pragma unroll
                for (int r = 0; r < LR; ++r) {
                    Qa[r][j] = dp2a_hi(v.y, lo[r], dp2a_lo(v.x, lo[r], Qa[r][j]));
                    Qb[r][j] = dp2a_hi(v.w, hi[r], dp2a_lo(v.z, hi[r], Qb[r][j]));
                }
            }
        }
        // the group ends here (or the tile does): fold its scale and bias
        uint32_t sb[LR];
        load_words<LR>(SBt + (size_t)(gcur - gfirst) * RC, sb);
        const float *xg = xseg + (size_t)(gcur - ag) * NT * 2;
#pragma unroll
        for (int r = 0; r < LR; ++r) {
            const float sc = bf16_bits(sb[r] & 0xFFFFu), bi = bf16_bits(sb[r] >> 16);
#pragma unroll
            for (int j = 0; j < TE; ++j) {
                y[r][j] = fmaf(sc * xg[2 * j + 1], (float)(Qa[r][j] + (Qb[r][j] >> 4)), fmaf(bi, xg[2 * j], y[r][j]));
                Qa[r][j] = Qb[r][j] = 0;
            }
        }
        ++gcur;
        left = gcb;
    }
}

template <int LR, int NT>
__device__ __forceinline__ void dn_tile_slots(int te, const LayerParams &p, float (&y)[LR][NT],
                                              const uint32_t *Wt, const uint32_t *SBt, const StageGeo &g,
                                              const uint32_t *act, const float *xseg, int a8, int ag) {
    switch (te) {
    case 1: dn_tile_te<1, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
    case 2: dn_tile_te<2, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
    case 3: dn_tile_te<3, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
    case 4: dn_tile_te<4, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
    default:
        if constexpr (NT > 4) {
            switch (te) {
            case 5: dn_tile_te<5, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
            case 6: dn_tile_te<6, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
            case 7: dn_tile_te<7, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
            default: dn_tile_te<8, LR, NT>(p, y, Wt, SBt, g, act, xseg, a8, ag); break;
            }
        }
    }
}

// Activations of token t for rows R and R+4 (concatenated row space), fp32,
// at row - a of this CTA's range.
__device__ __forceinline__ void put_act(float *actf, int act_rows, int a, int t, int R, float lo,
                                        float hi) {
    float *f = actf + (size_t)t * act_rows + (R - a);
    f[0] = lo;
    f[4] = hi;
}

// ---------------------------------------------------------------- kernel ----
template <int NT, bool SL>
__global__ void __launch_bounds__(kLayerThreads, 1) k_moe_layer(const LayerParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RG = ItemRows<NT>::gu, PG = ItemRows<NT>::pairs, NPASS = ItemRows<NT>::passes;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = (int)gridDim.x, blk = (int)blockIdx.x;
    constexpr int NSL = kLayerSlots;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.off_bars);
    uint64_t *empty = full + NSL;
    Ctl &ctl = *reinterpret_cast<Ctl *>(smem + p.off_ctl);
    Slots &sl = *reinterpret_cast<Slots *>(smem + p.off_slots);  // valid on the slot path
    RouteInfo &rs = ctl.route;
    uint32_t *xq = reinterpret_cast<uint32_t *>(smem + p.off_xs);       // [ntok][h/2] int16 pairs
    float *xsc = reinterpret_cast<float *>(smem + p.off_xsum);          // [ntok][nch] chunk scales
    float *xsum = xsc + NT * (p.h / kChunkCols);                        // [ntok][nch] chunk sums
    float *actf = reinterpret_cast<float *>(smem + p.off_actf);         // [ntok][act_cb*8]
    float *gup = reinterpret_cast<float *>(smem + p.off_gup);
    uint32_t *act = reinterpret_cast<uint32_t *>(smem + p.off_act);   // [ntok][act_cb][4] int16 pairs
    float *xseg = reinterpret_cast<float *>(smem + p.off_xseg);        // [seg][ntok] sums, then scales
    float *bst = reinterpret_cast<float *>(smem + p.off_blk);          // [cb][ntok] block max, sum
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smem + p.off_keys);
    float *rlog = reinterpret_cast<float *>(smem + p.off_rlog);
    float *lpart = reinterpret_cast<float *>(smem + p.off_lpart);
    const volatile int *vabort = &ctl.abort;
    const int h = p.h, I = p.I, nch = h / kChunkCols;
    const TiledLayout &tl = p.tl;
    unsigned *my_epoch = p.epochs + (size_t)blk * kEpochStride;

    // programmatic dependent launch: let the next launch in the stream be
    // scheduled now, and touch nothing until the previous grid has completed
    // and its memory is visible (no-ops without a dependent launch)
    pdl_trigger();
    // The router is a constant: warps 0..7 load their first block of it
    // before waiting on the previous kernel, so that the logits need only x
    // (one L2 round trip) once the wait returns.
    uint4 wpre = make_uint4(0u, 0u, 0u, 0u);
    if (warp < 8) {
        if constexpr (SL) {
            const int P = p.lparts, n8 = h / 8;
            constexpr int LT0 = NT == 1 ? 0 : (NT == 2 ? 1 : (NT == 4 ? 2 : 3));
            if (blk < p.E * P) {
                const int e = blk / P, part = blk - e * P;
                const int g8 = n8 * part / P + (tid >> LT0);
                if (g8 < n8 * (part + 1) / P)
                    wpre = __ldg(reinterpret_cast<const uint4 *>(p.router + (size_t)e * h) + g8);
            }
        } else {
            if (blk < p.E && tid < h / 8)
                wpre = __ldg(reinterpret_cast<const uint4 *>(p.router + (size_t)blk * h) + tid);
        }
    }
    pdl_wait();
    if (tid == 0) {
        trace_event(p.trace, 0, 0);
        ctl.abort = 0;
        ctl.route_ok = 0;
        ctl.epochs_seen = 0;
        const unsigned t1 = ld_relaxed_u32(my_epoch) + 1u;
        ctl.tag = t1 ? t1 : 1u;
    }
    __syncthreads();
    const unsigned tag = ctl.tag;
    // this CTA's rows of h (output initialisation)
    Producer ps;       // the producer warp's state (warp 24)
    uint64_t pol = 0;  // its L2 policy for the streamed weights
    const int i0 = (int)((long long)h * blk / G), i1 = (int)((long long)h * (blk + 1) / G);
    // ---- expert parallelism: gather x from every rank over peer memory ----
    const bool ep = p.ep_world > 1;
    const void *X = p.x;
    int Xbf16 = p.x_bf16;
    unsigned ep_tag = 0;
    int ep_par = 0;
    if (ep) {
        const EpLayout el = ep_layout(p.ep_world, p.ep_b, h);
        uint8_t *mine = p.ep_base[p.ep_rank];
        // every rank makes the same sequence of EP calls: the call counter
        // (advanced by the last CTA at the end of a call) names the call
        ep_tag = ld_acquire_sys_u32(reinterpret_cast<const unsigned *>(mine + 2LL * p.ep_world * 128)) + 1u;
        ep_par = ep_tag & 1;
        // CTA o writes this rank's tokens (and, with ep_pre, their routing)
        // into rank o's gathered slots for this call's parity, then raises
        // one tagged flag there (148 CTAs adding to one counter over NVLink
        // serialise for ~10 us; one CTA per destination runs in parallel)
        const int nb = p.ep_b;
        if (blk < p.ep_world) {
            const int o = blk;
            float *xs = reinterpret_cast<float *>(p.ep_base[o] + el.xs_off) +
                        ((size_t)ep_par * p.ep_world + p.ep_rank) * nb * h;
            for (int q = tid; q < nb * h; q += kLayerThreads) xs[q] = load_act(p.x, p.x_bf16, q);
            if (p.ep_pre) {
                const size_t slot = ((size_t)ep_par * p.ep_world + p.ep_rank) * nb * kMaxTopK;
                int *ri = reinterpret_cast<int *>(p.ep_base[o] + el.rt_off) + slot;
                float *rw = reinterpret_cast<float *>(p.ep_base[o] + el.rt_off) +
                            2LL * p.ep_world * nb * kMaxTopK + slot;
                for (int q = tid; q < nb * p.K; q += kLayerThreads) {
                    const int j = q / p.K, k = q - j * p.K;
                    ri[j * kMaxTopK + k] = p.ep_own_idx[q];
                    rw[j * kMaxTopK + k] = p.ep_own_w[q];
                }
            }
            // the barrier orders every thread's stores before the release
            // store of the flag (release is cumulative): one system-scope
            // release instead of a system fence in every thread
            __syncthreads();
            if (tid == 0) {
                st_release_sys_u32(reinterpret_cast<unsigned *>(p.ep_base[o]) + p.ep_rank * 32, ep_tag);
                trace_event(p.trace, 0, 24);
            }
        }
        // every rank's tokens have arrived
        if (tid < p.ep_world) {
            const unsigned *fl = reinterpret_cast<const unsigned *>(mine) + tid * 32;
            bool ok = false;
            for (uint32_t it = 0, nap = 32; it < p.ep_wait_limit; ++it) {
                if (ld_acquire_sys_u32(fl) == ep_tag) {
                    ok = true;
                    break;
                }
                __nanosleep(nap);
                nap = min(nap * 2, 256u);
            }
            if (!ok) set_abort(ctl, p.err);
        }
        __syncthreads();
        if (tid == 0) trace_event(p.trace, 0, 25);
        X = reinterpret_cast<const float *>(mine + el.xs_off) + (size_t)ep_par * p.ep_world * nb * h;
        Xbf16 = 0;
    }
    const int nrows = i1 - i0;
    const bool pre = ep && p.ep_pre;
    if (warp < 8 && pre) {
        // ---- phases 2-3 with the owners' routing (made by their route-only
        // calls, gathered with the tokens): no logits, no exchange ----
        const EpLayout el = ep_layout(p.ep_world, p.ep_b, h);
        const uint8_t *mine = p.ep_base[p.ep_rank];
        const int *gi = reinterpret_cast<const int *>(mine + el.rt_off) + (size_t)ep_par * p.ntok * kMaxTopK;
        const float *gw = reinterpret_cast<const float *>(mine + el.rt_off) +
                          2LL * p.ntok * kMaxTopK + (size_t)ep_par * p.ntok * kMaxTopK;
        for (int e = tid; e < p.E; e += 256) rs.tmask[e] = 0u;
        for (int q = tid; q < p.ntok * p.K; q += 256) {
            const int t = q / p.K, k = q - t * p.K;
            int e = __ldcv(gi + t * kMaxTopK + k);
            if (e < 0 || e >= p.E) {  // cannot happen; never index out of the tables
                set_abort(ctl, p.err);
                e = 0;
            }
            rs.idx[t][k] = e;
            const float wk = __ldcv(gw + t * kMaxTopK + k);
            rs.w[t][k] = wk;
            if (p.user_w && blk == 0) p.user_w[q] = wk;
        }
        named_sync(2, 256);
        named_arrive(6, kLayerThreads);
        const bool ok = route_cta<NT, SL>(p, rs, sl, ctl.range, rlog, keys, reinterpret_cast<float *>(ring), tag,
                                          vabort, true);
        if (tid == 0) {
            if (ok) ctl.route_ok = 1;
            else set_abort(ctl, p.err);
        }
        named_arrive(3, 256 + 32);
    } else if (warp < 8) {
        if constexpr (SL) {
            // ---- phase 2: partial logits, straight from global memory ----
            // Work item (e, part): W_r[e] . x[t] over the part's 8-column blocks
            // [n8*part/P, n8*(part+1)/P) for every token; a thread takes token
            // tid % NT of blocks tid / NT, +256/NT, ...  Fixed order throughout:
            // lanes of one token by xor shuffles, then the 8 warps in order.
            for (int e = tid; e < p.E; e += 256) rs.tmask[e] = 0u;
            const int P = p.lparts, nitems = p.E * P, n8 = h / 8;
            constexpr int LT = NT == 1 ? 0 : (NT == 2 ? 1 : (NT == 4 ? 2 : 3));
            const int tt = tid & (NT - 1);
            const int nmine = (nitems > blk) ? (nitems - blk + G - 1) / G : 0;
            for (int m = 0; m < nmine; ++m) {
                const int item = blk + m * G, e = item / P, part = item - e * P;
                const int g0 = n8 * part / P, g1 = n8 * (part + 1) / P;
                const uint4 *row = reinterpret_cast<const uint4 *>(p.router + (size_t)e * h);
                float acc = 0.f;
                if (tt < p.ntok) {
                    for (int g8 = g0 + (tid >> LT); g8 < g1; g8 += 256 >> LT) {
                        const uint4 wv = (m == 0 && g8 == g0 + (tid >> LT)) ? wpre : __ldg(row + g8);
                        float xv[8];
                        if (Xbf16) {
                            const uint4 r = *(reinterpret_cast<const uint4 *>(
                                reinterpret_cast<const uint16_t *>(X) + (size_t)tt * h) + g8);
                            const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
    #pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                xv[2 * j] = __uint_as_float(rr[j] << 16);
                                xv[2 * j + 1] = __uint_as_float(rr[j] & 0xFFFF0000u);
                            }
                        } else {
                            const float4 *xf = reinterpret_cast<const float4 *>(
                                reinterpret_cast<const float *>(X) + (size_t)tt * h) + 2 * g8;
                            const float4 a0 = xf[0], a1 = xf[1];  // plain loads (load_x32_any)
                            xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
                            xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
                        }
                        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    #pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            acc = fmaf(__uint_as_float(ww[j] << 16), xv[2 * j], acc);
                            acc = fmaf(__uint_as_float(ww[j] & 0xFFFF0000u), xv[2 * j + 1], acc);
                        }
                    }
                }
    #pragma unroll
                for (int o = NT; o < 32; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane < NT) lpart[warp * kMaxTok + lane] = acc;
                named_sync(2, 256);
                // publish into every CTA's box (each box is polled by its CTAs only)
                uint32_t sv[NT];
    #pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float s = 0.f;
                    if (t < p.ntok)
                        for (int w = 0; w < 8; ++w) s += lpart[w * kMaxTok + t];
                    sv[t] = __float_as_uint(s);
                }
                // box layout [e][part][t], t padded to NT: an item's tokens
                // are NT adjacent words, written with 16-byte stores
                for (int bx = tid; bx < p.nbox; bx += 256) {
                    unsigned long long *box = p.xlog + (size_t)bx * p.box_words + (size_t)item * NT;
    #pragma unroll
                    for (int t = 0; t < NT; t += 2)
                        st_relaxed_v2_u64(box + t, tagged(tag, sv[t]), tagged(tag, sv[t + 1]));
                }
                named_sync(2, 256);
            }
        } else {
            // ---- phase 2: logits of this CTA's experts, straight from global memory ----
            // (batches of 1 and 2: one part per logit, a CTA per expert)
            for (int e = tid; e < p.E; e += 256) rs.tmask[e] = 0u;
            const int nmine = (p.E > blk) ? (p.E - blk + G - 1) / G : 0;
            for (int m = 0; m < nmine; ++m) {
                const int e = blk + m * G;
                const uint4 *row = reinterpret_cast<const uint4 *>(p.router + (size_t)e * h);
                float acc[NT];
    #pragma unroll
                for (int t = 0; t < NT; ++t) acc[t] = 0.f;
                for (int g8 = tid; g8 < h / 8; g8 += 256) {
                    const uint4 wv = (m == 0 && g8 == tid) ? wpre : __ldg(row + g8);
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
                            if (Xbf16) {
                                const uint4 r = *(reinterpret_cast<const uint4 *>(
                                    reinterpret_cast<const uint16_t *>(X) + (size_t)t * h) + g8);
                                const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
    #pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    xv[2 * j] = __uint_as_float(rr[j] << 16);
                                    xv[2 * j + 1] = __uint_as_float(rr[j] & 0xFFFF0000u);
                                }
                            } else {
                                const float4 *xf = reinterpret_cast<const float4 *>(
                                    reinterpret_cast<const float *>(X) + (size_t)t * h) + 2 * g8;
                                const float4 a0 = xf[0], a1 = xf[1];  // plain loads (load_x32_any)
                                xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
                                xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
                            }
    #pragma unroll
                            for (int j = 0; j < 8; ++j) acc[t] = fmaf(wf[j], xv[j], acc[t]);
                        }
                    }
                }
    #pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const float v = warp_sum(acc[t]);
                    if (lane == 0) lpart[warp * kMaxTok + t] = v;
                }
                named_sync(2, 256);
                // publish into every CTA's box (each box is polled by its CTAs only)
                uint32_t sv[NT];
    #pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float s = 0.f;
                    if (t < p.ntok)
                        for (int w = 0; w < 8; ++w) s += lpart[w * kMaxTok + t];
                    sv[t] = __float_as_uint(s);
                }
                for (int bx = tid; bx < p.nbox; bx += 256) {
                    unsigned long long *box = p.xlog + (size_t)bx * p.box_words + e;
    #pragma unroll
                    for (int t = 0; t < NT; ++t)
                        if (t < p.ntok) st_relaxed_u64(box + (size_t)t * p.E, tagged(tag, sv[t]));
                }
                named_sync(2, 256);
            }
        }
        if (tid == 0) trace_event(p.trace, 0, 2);
        named_arrive(6, kLayerThreads);  // this CTA's logits are out: x staging may start
        // ---- phase 3: route (warps 0..7 of every CTA) ----
        // partial logits are summed in the tile ring, idle until routing is done
        const bool ok = route_cta<NT, SL>(p, rs, sl, ctl.range, rlog, keys, reinterpret_cast<float *>(ring), tag, vabort);
        if (tid == 0) trace_event(p.trace, 0, 3);
        if (tid == 0) {
            if (ok) ctl.route_ok = 1;
            else set_abort(ctl, p.err);
        }
        named_arrive(3, 256 + 32);  // routing (or its failure) is in shared memory
    } else {
        // ---- phase 1 (warps 8..24): pipeline set-up, x staging, output rows ----
        const int st = tid - 256, nst = kLayerThreads - 256;
        if (tid == kConsumerThreads) {
            for (int i = 0; i < NSL; ++i) {
                mbar_init(&full[i], 1);
                mbar_init(&empty[i], 1);
                ctl.stage_tile[i] = -1;
                ctl.stage_done[i] = 0;
            }
            ctl.next_gu = ctl.next_dn = 0;
            ctl.issued = 0;
            mbar_fence_init();
        }
        // this CTA's output rows start as the residual (moeCombine adds it
        // first, Shaders.metal:368) or zero
        if (!p.route_only) {
            float *dst = p.out_acc ? p.acc : reinterpret_cast<float *>(p.out);
            for (int q = st; q < p.ntok * nrows; q += nst) {
                const int t = q / nrows, i = i0 + q % nrows;
                // (expert parallel: the residual is added once, by the owner, at the end)
                dst[(size_t)t * h + i] = (p.res && !ep) ? load_act(p.res, p.res_bf16, (size_t)t * h + i) : 0.f;
            }
        }
        named_sync(4, nst);
        if (tid == 256) {
            trace_event(p.trace, 0, 1);
            __threadfence();
            st_release_u32(my_epoch, tag);
        }
        // The router warps' loads of x and of the router rows go first: x
        // staging (every CTA reading all of x at once) waits until this CTA's
        // logits are published (barrier 6), overlapping the logit exchange.
        named_sync(6, kLayerThreads);
        // x as int16 chunks (dp2a layout, common.cuh) with scales and exact
        // sums (a routing-only call has no use for it, nor room: the host
        // plans no x staging then)
        for (int q = st; !p.route_only && q < p.ntok * nch; q += nst) {
            const int t = q / nch, c = q - t * nch;
            float v[32];
            load_x32_any(X, Xbf16, (size_t)t * h + (size_t)c * kChunkCols, v);
            xsc[q] = quant_chunk_i16(v, xq + (size_t)t * (h / 2), nch, c, &xsum[q]);
        }
        if (warp == kConsumerWarps) {
            // the producer starts as soon as warps 0..7 have routed: the
            // geometry and the first tile, then it lets the others go
            // (barrier 5, without waiting) and keeps issuing
            pol = l2_evict_first_policy();
            named_sync(3, 256 + 32);
            if (lane == 0) trace_event(p.trace, 0, 19);
            if (!p.route_only && ctl.route_ok) {
                route_geometry(p, ctl, blk);
                if (lane == 0) {
                    trace_event(p.trace, 0, 16);
                    if (ctl.ntg + ctl.ntd > 0) {
                        // the first tile, described by lane 0 alone; the
                        // whole first batch is described again later
                        describe_tile(p, ctl, 0, ctl.copy[0]);
                        ps.batch = 0;
                        issue_batch(p, ctl, ring, full, empty, ps, false, pol, 1);
                        ps.batch = -1;
                    }
                }
            }
            named_arrive(5, kLayerThreads);
        }
    }
    if (warp != kConsumerWarps) named_sync(5, kLayerThreads);
    const bool go = !p.route_only && ctl.route_ok;  // uniform: fixed before barrier 5
    if (tid == 0) {
        trace_event(p.trace, 0, 4);
        trace_value(p.trace, 0, 14, (unsigned)ctl.a | ((unsigned long long)(unsigned)ctl.b << 32));
        trace_value(p.trace, 0, 15, (unsigned)ctl.ntg | ((unsigned long long)(unsigned)ctl.ntd << 32));
    }
    // the routing weights: needed only by the caller's outputs and the final
    // atomics, so warps 1..7 compute them while the first copies are in flight
    if (warp >= 1 && warp < 8 && ctl.route_ok && !pre)
        for (int t = warp - 1; t < p.ntok; t += 7) route_weights(p, rs, rlog, t);
    if (!go) {
        if (p.route_only) __syncthreads();  // user outputs complete before the epoch advances
        return;  // uniform; no copies were issued
    }
    // Every CTA's output rows must be initialised before this CTA's first
    // atomic, long after this point: warp 8 checks the epoch words here, off
    // the path to the first weight copy, and the down items wait for its flag.
    if (warp == 8) {
        if (wait_all_epochs(p.epochs, G, tag, vabort)) {
            if (lane == 0) st_release_cta_shared(&ctl.epochs_seen, 1);
        } else if (lane == 0) {
            set_abort(ctl, p.err);
        }
        if (lane == 0) trace_event(p.trace, 0, 7);
    }

    // ---- phase 4 geometry ----
    const int GT = p.gu_tile_rows, RC = tl.rc, nic = p.nic;
    const int a = ctl.a, b = ctl.b, ntg = ctl.ntg, ntd = ctl.ntd;
    const int a8 = a >> 3, ag = fdiv(a, p.fd_gs), gcb = p.gs >> 3;
    const int nslg = p.gu_nslices;
    const int ipt_g = gu_items_per_tile(SL, NT, GT, nslg);  // work items per gate/up tile
    const int ipt_d = RC / (32 * dn_lane_rows(SL, NT));  // work items per down tile

    if (warp == kConsumerWarps) {
        // ================= producer (warp 24) =================
        // the rest of the tiles, waiting for releases as needed
        produce(p, ctl, ring, full, empty, ps, true, pol, 1 << 30);
        if (lane == 0) {
            ctl.issued = ps.n;
            trace_event(p.trace, 0, 9);
        }
    } else {
        // ================= consumers: gate/up =================
        const int ng_items = ntg * ipt_g;
        if constexpr (SL) {
            // item = one row of a tile, for all of its expert's token slots
            for (;;) {
                const int q = grab(&ctl.next_gu);
                if (q >= ng_items) break;
                const int n = fdiv(q, p.fd_iptg), rr = q - n * ipt_g;
                const int s = n % NSL;
                if (!wait_tile(full, ctl, s, n, NSL, p.err)) break;
                if (q == 0 && lane == 0) trace_event(p.trace, 0, 5);
                const StageGeo g = ctl.geo[s];
                if (rr < g.nr)
                    gu_row_slots<NT>(sl.ute[rs.ulist[g.u]], p, ring + g.off + (size_t)rr * tl.pr, sl.utok[rs.ulist[g.u]], xq, xsc,
                                     xsum, actf, p.act_cb * 8, g.u * I + g.r0 + rr - a);
                release_item(empty, ctl, s, ipt_g);
            }
        } else {
            constexpr int kNg = 2 * RG * NT, kSg = 32 / kNg;
            const size_t wo_u = (size_t)h / 2 + 2 * tl.sbh;  // up part offset in a pair-row
            for (;;) {
                const int q = grab(&ctl.next_gu);
                if (q >= ng_items) break;
                const int n = fdiv(q, p.fd_iptg), rem = q - n * ipt_g, pg = fdiv(rem, p.fd_nslg),
                          j = rem - pg * nslg;
                const int s = n % NSL;
                if (!wait_tile(full, ctl, s, n, NSL, p.err)) break;
                if (q == 0 && lane == 0) trace_event(p.trace, 0, 5);
                const StageGeo g = ctl.geo[s];
                if (pg * PG < g.nr / 2) {
                    const uint8_t *st = ring + g.off;
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
                        float accg[kNg];  // [(row * NT + token) * 2 + gate0/up1]
    #pragma unroll
                        for (int i = 0; i < kNg; ++i) accg[i] = 0.f;
                        for (int ch = j * 32 + lane; ch < nch; ch += 32 * nslg) {
                            const int gi = fdiv(ch * kChunkCols, p.fd_gs);
    #pragma unroll
                            for (int k = 0; k < NT; ++k) {
                                if (!((mask >> k) & 1u)) continue;
                                uint32_t xp[16];
                                load_pairs_any(reinterpret_cast<const uint16_t *>(xq + (size_t)k * (h / 2)), nch, ch, xp);
                                const float X = xsum[k * nch + ch], sx = xsc[k * nch + ch];
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
                                    float &ag = accg[(r * NT + k) * 2 + 0];
                                    float &au = accg[(r * NT + k) * 2 + 1];
                                    // s*sx*Q + b*X per chunk (Q exact, common.cuh)
                                    ag = fmaf(sg * sx, (float)dot_chunk_i16(wg, xp), fmaf(bg, X, ag));
                                    au = fmaf(su * sx, (float)dot_chunk_i16(wu, xp), fmaf(bu, X, au));
                                }
                            }
                        }
                        // lane holds value lane / kSg = (r*NT + k)*2 + m
                        const float tot = warp_reduce_multi(accg);
                        if (nslg == 1) {
                            const float upv = __shfl_down_sync(0xffffffffu, tot, kSg);
                            const float av = swiglu(tot, upv);  // meaningful where lane % (2kSg) == 0
                            const int jj = lane / (2 * kSg), r = jj / NT, k = jj % NT;
                            const bool lead = (lane % (2 * kSg)) == 0 && ((mask >> k) & 1u);
                            if (NPASS == 1) {
                                // slot r+1 (row R+4) is 2*kSg*NT lanes further on
                                const float other = __shfl_down_sync(0xffffffffu, av, 2 * kSg * NT);
                                if (lead && (r & 1) == 0) {
                                    const int pu = pg * PG + (r >> 1);
                                    put_act(actf, p.act_cb * 8, a, k, g.u * I + g.r0 + 8 * (pu >> 2) + (pu & 3),
                                            av, other);
                                }
                            } else if (pass == 0) {
                                act_prev = av;
                            } else if (lead) {
                                put_act(actf, p.act_cb * 8, a, k, g.u * I + g.r0 + 8 * (pg >> 2) + (pg & 3),
                                        act_prev, av);
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
        }
        if (tid == 0) trace_event(p.trace, 0, 17);
        named_sync(1, kConsumerThreads);  // every gate/up item of this CTA is done
        // Activations of this CTA's rows.  Other group sizes than 64 take two
        // short passes: (1) one thread
        // per (row, token) sums the column slices in order and applies SwiGLU
        // where items left partial sums, and the 8 lanes of a column block
        // reduce its max |a| and sum; (2) one per (block, token): the group's
        // (gs rows) max from its blocks, the block as int16 pairs in the dp2a
        // layout (4 words, as for x), and per group the scale and fp32 sum.
        const int ncb_cta = (b - a) >> 3, arows = p.act_cb * 8;
        if (p.gs == 64) {
            // Groups of 64 rows (every shipped model): one warp per (group of
            // this CTA's range, token), lane l holding rows 2l and 2l+1 of the
            // group -- SwiGLU where items left partial sums, the group's max
            // |a| and fp32 sum by warp reductions, the int16 quantisation, and
            // the dp2a packing (lanes 4c+j hold rows 8c+2j, 8c+2j+1 of column
            // block c) by one shuffle: no block-wide pass in between
            const int ngr = b > a ? fdiv(b - 1, p.fd_gs) - ag + 1 : 0;
            for (int wi = warp; wi < ngr * NT; wi += kConsumerWarps) {
                const int gi = wi / NT, k = wi - gi * NT, gg = ag + gi;
                const int r_lo = max(gg * 64, a), r_hi = min(gg * 64 + 64, b);
                const int u = fdiv(r_lo, p.fd_I);  // 64 | I: a group lies in one expert
                // k: a token (row groups) or a token slot of expert u (slot path)
                if (ctl.abort || (SL ? k >= sl.ute[rs.ulist[u]] : !((rs.tmask[rs.ulist[u]] >> k) & 1u))) continue;
                float v[2] = {0.f, 0.f};
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    const int R = gg * 64 + 2 * lane + h2;
                    if (R >= r_lo && R < r_hi) {
                        const int lr = R - a;
                        if (nslg > 1) {
                            float gv = 0.f, uv = 0.f;
                            const float *gp = gup + (size_t)lr * nslg * (2 * NT) + 2 * k;
                            for (int jj = 0; jj < nslg; ++jj) {
                                gv += gp[jj * 2 * NT];
                                uv += gp[jj * 2 * NT + 1];
                            }
                            v[h2] = swiglu(gv, uv);
                        } else {
                            v[h2] = actf[(size_t)k * arows + lr];
                        }
                    }
                }
                float m = fmaxf(fabsf(v[0]), fabsf(v[1])), sm = v[0] + v[1];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                    sm += __shfl_xor_sync(0xffffffffu, sm, o);
                }
                const float inv = m > 0.f ? 32767.0f / m : 0.f;
                const uint32_t q0 = (uint32_t)(__float2int_rn(v[0] * inv) & 0xFFFF);
                const uint32_t q1 = (uint32_t)(__float2int_rn(v[1] * inv) & 0xFFFF);
                const uint32_t n0 = __shfl_down_sync(0xffffffffu, q0, 1), n1 = __shfl_down_sync(0xffffffffu, q1, 1);
                const int R0 = gg * 64 + 8 * (lane >> 2);  // first row of this lane's column block
                if ((lane & 1) == 0 && R0 >= r_lo && R0 < r_hi) {
                    // words 0/1: rows (0,2) / (4,6) of the block; 2/3: rows (1,3) / (5,7)
                    const int w = (lane & 3) >> 1;
                    uint32_t *o = act + (((size_t)k * p.act_cb + ((R0 - a) >> 3)) << 2);
                    o[w] = q0 | (n0 << 16);
                    o[2 + w] = q1 | (n1 << 16);
                }
                if (lane == 0) {
                    float *xg = xseg + ((size_t)(gg - ag) * NT + k) * 2;
                    xg[0] = sm;
                    xg[1] = m * (1.0f / 32767.0f);
                }
            }
        } else {
            {
                // passes 1 and 2 together: thread (token k, row lr), rows inner, so
                // the 8 rows of a column block are 8 consecutive lanes and the
                // block's max |a| and sum come from shuffles
                const int nrows = b - a, total = nrows * NT;
                for (int base = warp * 32; base < total; base += kConsumerThreads) {
                    const int i = base + lane, k = i / max(nrows, 1), lr = i - k * nrows;
                    float v = 0.f;
                    if (i < total) {
                        float *af = actf + (size_t)k * arows + lr;
                        if (nslg > 1) {
                            const int e = rs.ulist[fdiv(a + lr, p.fd_I)];
                            if (!ctl.abort && ((rs.tmask[e] >> k) & 1u)) {
                                float gv = 0.f, uv = 0.f;
                                const float *gp = gup + (size_t)lr * nslg * (2 * NT) + 2 * k;
                                for (int jj = 0; jj < nslg; ++jj) {
                                    gv += gp[jj * 2 * NT];
                                    uv += gp[jj * 2 * NT + 1];
                                }
                                v = swiglu(gv, uv);
                                *af = v;
                            }
                        } else {
                            v = *af;
                        }
                    }
                    float m = fabsf(v), sm = v;
    #pragma unroll
                    for (int o = 1; o < 8; o <<= 1) {
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                        sm += __shfl_xor_sync(0xffffffffu, sm, o);
                    }
                    if (i < total && (lane & 7) == 0) {
                        const int bi = (lr >> 3) * NT + k;
                        bst[2 * bi] = m;
                        bst[2 * bi + 1] = sm;
                    }
                }
            }
            named_sync(1, kConsumerThreads);
            for (int i = tid; i < ncb_cta * NT; i += kConsumerThreads) {
                const int cb = i / NT, k = i % NT;
                const int R0 = a + 8 * cb, u = fdiv(R0, p.fd_I);
                // k: a token (row groups) or a token slot of expert u (slot path)
                if (ctl.abort || (SL ? k >= sl.ute[rs.ulist[u]] : !((rs.tmask[rs.ulist[u]] >> k) & 1u))) continue;
                const int gg = fdiv(a8 + cb, p.fd_gcb);
                const int c_lo = max(gg * gcb, a8) - a8, c_hi = min((gg + 1) * gcb, b >> 3) - a8;
                float m = 0.f;
                for (int c = c_lo; c < c_hi; ++c) m = fmaxf(m, bst[2 * (c * NT + k)]);
                const float inv = m > 0.f ? 32767.0f / m : 0.f;
                const float *x = actf + (size_t)k * arows + 8 * cb;
                auto qz = [&](float v) { return (uint32_t)(__float2int_rn(v * inv) & 0xFFFF); };
                uint32_t *o = act + (((size_t)k * p.act_cb + cb) << 2);
                o[0] = qz(x[0]) | (qz(x[2]) << 16);
                o[1] = qz(x[4]) | (qz(x[6]) << 16);
                o[2] = qz(x[1]) | (qz(x[3]) << 16);
                o[3] = qz(x[5]) | (qz(x[7]) << 16);
                if (cb == c_lo) {  // the group's first block of this range: scale and sum
                    float sum = 0.f;
                    for (int c = c_lo; c < c_hi; ++c) sum += bst[2 * (c * NT + k) + 1];
                    float *xg = xseg + ((size_t)(gg - ag) * NT + k) * 2;
                    xg[0] = sum;
                    xg[1] = m * (1.0f / 32767.0f);
                }
            }
        }
        named_sync(1, kConsumerThreads);
        if (tid == 0) trace_event(p.trace, 0, 6);

        // ================= consumers: down (split-K) =================
        // Item = 32*LR consecutive rows of one row chunk (lane: LR adjacent
        // rows of h), over all of this CTA's down tiles of that chunk in ring
        // order.  Per column block: LR weight words (one vector load), the
        // nibble pairs of each shared by the tokens; per group:
        // y += s*sa*Q + b*X; per tile (one expert): total += w_k * y.  One
        // LR-wide atomic per lane and token at the end.
        constexpr int LR = dn_lane_rows(SL, NT);
        const int nsub = ctl.nsub;  // down tiles per row chunk
        const int nd_items = (ctl.abort || ntd == 0) ? 0 : nic * ipt_d;
        float *dst = p.out_acc ? p.acc : reinterpret_cast<float *>(p.out);
        bool seen = false;  // epochs_seen observed (acquire) by this warp
        // (acquire) every CTA's output rows are initialised: needed once per
        // warp, before its first atomic
        auto see_epochs = [&]() -> bool {
            if (!seen) {
                if (lane == 0) {
                    for (uint32_t it = 0; it < kWaitLimit && !seen; ++it) {
                        seen = ld_acquire_cta_shared(&ctl.epochs_seen) != 0;
                        if (!seen) {
                            if (*vabort) break;
                            __nanosleep(64);
                        }
                    }
                    if (!seen && !*vabort) set_abort(ctl, p.err);
                }
                seen = __shfl_sync(0xffffffffu, seen, 0);
            }
            return seen;
        };
        if constexpr (SL) {
            // Item as above; the chunk's tiles come expert by expert (a tile
            // never spans two), and each expert's run of tiles is summed per
            // token slot and added to the output once, weighted by the
            // slot's routing weight.
            for (;;) {
                const int q = grab(&ctl.next_dn);
                if (q >= nd_items) break;
                const int ic = fdiv(q, p.fd_iptd), wi = q - ic * ipt_d;
                const int ri = (wi * 32 + lane) * LR;  // first row (in the chunk) of this lane
                const int i = ic * RC + ri;
                if (q == 0 && lane == 0) trace_event(p.trace, 0, 18);
                float y[LR][NT];
#pragma unroll
                for (int r = 0; r < LR; ++r)
#pragma unroll
                    for (int t = 0; t < NT; ++t) y[r][t] = 0.f;
                int cur = -1;  // distinct expert whose sums y holds
                auto flush_expert = [&]() -> bool {
                    if (!see_epochs()) return false;
                    const int e = rs.ulist[cur], te = sl.ute[e];
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        if (j < te) {
                            const int t = sl.utok[e][j];
                            const float wk = rs.w[t][rs.kof[e][t]];
                            float v[LR][1];
#pragma unroll
                            for (int r = 0; r < LR; ++r) v[r][0] = wk * y[r][j];
                            add_words<LR>(dst + (size_t)t * h + i, v, 0);
                        }
#pragma unroll
                        for (int r = 0; r < LR; ++r) y[r][j] = 0.f;
                    }
                    return true;
                };
                bool ok = true;
                for (int jt = 0; jt < nsub; ++jt) {
                    const int n = ntg + ic * nsub + jt, s = n % NSL;
                    if (!wait_tile(full, ctl, s, n, NSL, p.err)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0 && wi == 0 && n == ntg) trace_event(p.trace, 0, 22);
                    if (lane == 0 && wi == 0 && n == ntg + ntd - 1) trace_event(p.trace, 0, 23);
                    const StageGeo g = ctl.geo[s];
                    if (g.u != cur) {
                        if (cur >= 0 && !flush_expert()) {
                            ok = false;
                            break;
                        }
                        cur = g.u;
                    }
                    const uint32_t *Wt = reinterpret_cast<const uint32_t *>(ring + g.off) + ri;
                    dn_tile_slots<LR, NT>(sl.ute[rs.ulist[g.u]], p, y, Wt, Wt + (size_t)g.nr * RC, g, act, xseg, a8, ag);
                    release_item(empty, ctl, s, ipt_d);
                }
                if (ok && cur >= 0) ok = flush_expert();
                if (!ok) break;
            }
        } else {
            for (;;) {
                const int q = grab(&ctl.next_dn);
                if (q >= nd_items) break;
                const int ic = fdiv(q, p.fd_iptd), wi = q - ic * ipt_d;
                const int ri = (wi * 32 + lane) * LR;  // first row (in the chunk) of this lane
                if (q == 0 && lane == 0) trace_event(p.trace, 0, 18);
                float tot[LR][NT];
    #pragma unroll
                for (int r = 0; r < LR; ++r)
    #pragma unroll
                    for (int t = 0; t < NT; ++t) tot[r][t] = 0.f;
                unsigned any = 0u;
                bool ok = true;
                for (int jt = 0; jt < nsub; ++jt) {
                    const int n = ntg + ic * nsub + jt, s = n % NSL;
                    if (!wait_tile(full, ctl, s, n, NSL, p.err)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0 && wi == 0 && n == ntg) trace_event(p.trace, 0, 22);
                    if (lane == 0 && wi == 0 && n == ntg + ntd - 1) trace_event(p.trace, 0, 23);
                    const StageGeo g = ctl.geo[s];
                    const int e = rs.ulist[g.u];
                    const unsigned mask = rs.tmask[e];
                    const uint32_t *Wt = reinterpret_cast<const uint32_t *>(ring + g.off) + ri;
                    const uint32_t *SBt = Wt + (size_t)g.nr * RC;
                    const int gfirst = fdiv(g.r0, p.fd_gcb);  // first group (concatenated space)
                    float y[LR][NT];
                    int Q[LR][NT];
    #pragma unroll
                    for (int r = 0; r < LR; ++r)
    #pragma unroll
                        for (int t = 0; t < NT; ++t) {
                            y[r][t] = 0.f;
                            Q[r][t] = 0;
                        }
                    int gcur = gfirst, left = gcb - (g.r0 - gfirst * gcb);  // blocks left in gcur
                    auto flush = [&](int gg) {
                        uint32_t sb[LR];
                        load_words<LR>(SBt + (size_t)(gg - gfirst) * RC, sb);
                        const float *xg = xseg + (size_t)(gg - ag) * NT * 2;
    #pragma unroll
                        for (int r = 0; r < LR; ++r) {
                            const float sc = bf16_bits(sb[r] & 0xFFFFu), bi = bf16_bits(sb[r] >> 16);
    #pragma unroll
                            for (int t = 0; t < NT; ++t) {
                                // s * sa * Q + b * X over the group's columns in this range
                                if ((mask >> t) & 1u)
                                    y[r][t] = fmaf(sc * xg[2 * t + 1], (float)Q[r][t],
                                                   fmaf(bi, xg[2 * t], y[r][t]));
                                Q[r][t] = 0;
                            }
                        }
                    };
                    for (int c = 0; c < g.nr; ++c) {
                        uint32_t wd[LR];
                        load_words<LR>(Wt + (size_t)c * RC, wd);
                        const uint4 *av = reinterpret_cast<const uint4 *>(act) + (g.r0 + c - a8);
    #pragma unroll
                        for (int t = 0; t < NT; ++t) {
                            if ((mask >> t) & 1u) {
                                const uint4 v = av[(size_t)t * p.act_cb];
    #pragma unroll
                                for (int r = 0; r < LR; ++r) {
                                    const uint32_t lo = wd[r] & 0x0F0F0F0Fu, hi = (wd[r] >> 4) & 0x0F0F0F0Fu;
                                    Q[r][t] = dp2a_hi(v.w, hi, dp2a_lo(v.z, hi, dp2a_hi(v.y, lo,
                                                                                      dp2a_lo(v.x, lo, Q[r][t]))));
                                }
                            }
                        }
                        if (--left == 0) {
                            flush(gcur);
                            ++gcur;
                            left = gcb;
                        }
                    }
                    if (left != gcb) flush(gcur);
    #pragma unroll
                    for (int t = 0; t < NT; ++t)
                        if ((mask >> t) & 1u) {
                            const float wk = rs.w[t][rs.kof[e][t]];
    #pragma unroll
                            for (int r = 0; r < LR; ++r) tot[r][t] = fmaf(wk, y[r][t], tot[r][t]);
                        }
                    any |= mask;
                    release_item(empty, ctl, s, ipt_d);
                }
                if (!ok) break;
                if (!see_epochs()) break;
                const int i = ic * RC + ri;
    #pragma unroll
                for (int t = 0; t < NT; ++t)
                    if ((any >> t) & 1u) add_words<LR>(dst + (size_t)t * h + i, tot, t);
            }
        }
        if (tid == 0) trace_event(p.trace, 0, 8);
        if (p.out_acc) {
            // the last CTA to finish writes the fp32 sums out
            named_sync(1, kConsumerThreads);
            if (tid == 0) {
                __threadfence();
                ctl.last = atomicAdd(p.done, 1) == G - 1;
            }
            named_sync(1, kConsumerThreads);
            if (ep) {
                // expert parallel, spread over every CTA: once all CTAs' sums
                // are in the accumulator (a grid-wide arrival count: the
                // launch is cooperative), CTA c sends each peer its slice
                // [i0, i1) of h for that peer's tokens as tagged words {call
                // tag, value} (one 8-byte store each: no flag, no fence),
                // polls (bounded) its slice of this rank's tokens from every
                // peer until the words carry this call's tag, and writes
                // residual + the ranks' sums in rank order
                const EpLayout el = ep_layout(p.ep_world, p.ep_b, h);
                const int W = p.ep_world, nb = p.ep_b, me = p.ep_rank;
                uint8_t *mine = p.ep_base[me];
                if (tid == 0) {
                    bool ok = ctl.abort == 0;
                    for (uint32_t it = 0, nap = 32; ok && it < kWaitLimit; ++it) {
                        if (ld_acquire_gpu_s32(p.done) >= G) break;
                        if (it + 1 == kWaitLimit || *vabort) ok = false;
                        __nanosleep(nap);
                        nap = min(nap * 2, 64u);
                    }
                    if (!ok && !*vabort) set_abort(ctl, p.err);
                    trace_event(p.trace, 0, 26);
                }
                named_sync(1, kConsumerThreads);
                const int sr = i1 - i0;
                if (!ctl.abort) {
                    for (int q = tid; q < W * nb * sr; q += kConsumerThreads) {
                        const int o = q / (nb * sr);
                        if (o == me) continue;
                        const int rem = q - o * nb * sr, t = rem / sr, i = i0 + (rem - t * sr);
                        unsigned long long *rv = reinterpret_cast<unsigned long long *>(p.ep_base[o] + el.recv_off) +
                                                 ((size_t)ep_par * W + me) * nb * h;
                        st_relaxed_sys_u64(rv + (size_t)t * h + i,
                                           tagged(ep_tag, __float_as_uint(__ldcg(p.acc + ((size_t)o * nb + t) * h + i))));
                    }
                }
                if (tid == 0) trace_event(p.trace, 0, 27);
                const unsigned long long *rv =
                    reinterpret_cast<const unsigned long long *>(mine + el.recv_off) + (size_t)ep_par * W * nb * h;
                bool got = ctl.abort == 0;
                for (int q = tid; got && q < nb * sr; q += kConsumerThreads) {
                    const int t = q / sr, i = i0 + (q - t * sr);
                    const size_t oi = (size_t)t * h + i;
                    float v = p.res ? load_act(p.res, p.res_bf16, oi) : 0.f;
                    for (int o = 0; got && o < W; ++o) {
                        if (o == me) {
                            v += __ldcg(p.acc + (size_t)me * nb * h + oi);
                            continue;
                        }
                        unsigned long long wd = 0;
                        for (uint32_t it = 0, nap = 32;; ++it) {
                            wd = ld_relaxed_sys_u64(rv + (size_t)o * nb * h + oi);
                            if ((unsigned)(wd >> 32) == ep_tag) break;
                            if (it >= p.ep_wait_limit || *vabort) {
                                got = false;
                                break;
                            }
                            __nanosleep(nap);
                            nap = min(nap * 2, 64u);
                        }
                        v += __uint_as_float((unsigned)wd);
                    }
                    if (!got) break;
                    if (p.out_bf16)
                        reinterpret_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(v);
                    else
                        reinterpret_cast<float *>(p.out)[oi] = v;
                }
                if (!got && !*vabort) set_abort(ctl, p.err);
                named_sync(1, kConsumerThreads);
                if (tid == 0) trace_event(p.trace, 0, 28);
                // the last CTA through resets the counts and advances the
                // region's call counter, which names the next call
                named_sync(1, kConsumerThreads);
                if (tid == 0 && atomicAdd(p.done + 1, 1) == G - 1) {
                    p.done[0] = 0;
                    p.done[1] = 0;
                    st_release_sys_u32(reinterpret_cast<unsigned *>(mine + 2LL * W * 128), ep_tag);
                }
            } else if (ctl.last) {
                __threadfence();
                if (p.out_bf16) {
                    __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(p.out);
                    for (int i = tid; i < p.ntok * h; i += kConsumerThreads)
                        o[i] = __float2bfloat16_rn(__ldcg(p.acc + i));
                } else {
                    float *o = reinterpret_cast<float *>(p.out);
                    for (int i = tid; i < p.ntok * h; i += kConsumerThreads) o[i] = __ldcg(p.acc + i);
                }
                if (tid == 0) *p.done = 0;
            }
        }
    }
    __syncthreads();
    if (tid == 0) trace_event(p.trace, 0, 10);
    if (ctl.abort && tid == 0) {
        // wait (bounded) for copies still in flight into this CTA's shared memory
        for (int n = ctl.issued - NSL; n < ctl.issued; ++n) {
            if (n < 0) continue;
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(&full[n % NSL], (n / NSL) & 1)) break;
        }
    }
}

}  // namespace m1
