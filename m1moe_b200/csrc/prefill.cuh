// prefill.cuh — the MoE block for many tokens at once (prefill, large
// batches) as grouped GEMMs on the tcgen05 tensor cores.
//
// Same result as T decode calls of k_moe_layer (the reference runs the MoE
// block token by token: InferenceEngine.runLayer :240-266, bench/main.swift
// :139-141), organised as a dense contraction per expert:
//   1. k_prefill_route: per token, router logits (fp32, d ascending per
//      lane), top-K by rank (ties to the lower index, InferenceEngine.swift
//      :510-519), softmax weights with optional renormalisation (:490-508);
//   2. k_prefill_plan: a stable counting sort of the (token, k) pairs by
//      expert (local experts only) into slots; each expert's slots are cut
//      into token tiles of at most kPfTileTok;
//   3. k_prefill_gather: each tile's tokens as fp16 in the tensor-core
//      operand layout (K-major, 128B-swizzled, the nibble K order of
//      umma.cuh), one contiguous block per 64 columns, so a plain bulk copy
//      fills a shared-memory operand;
//   4. k_prefill_gemm<kGateUp>: per (tile, 128 rows of I) the gate and up
//      products in TMEM (weights dequantised to fp16 on the fly from the
//      int4 table), SwiGLU in the epilogue, written as fp16 in the same
//      operand layout for the down product;
//   5. k_prefill_gemm<kDown>: per (tile, 128 rows of h, K split) the down
//      product, fp32 partial sums per slot;
//   6. k_prefill_combine: out = residual + sum_k w_k * expert_k (k ascending,
//      residual first: moeCombine, Shaders.metal:360-376).
// The tensor cores take fp16 (11 significant bits; bf16's 8 would put the
// error at the 1e-3 bar for small h): weights are rounded once (q*s + b in
// one fma), tokens and SwiGLU activations once; the accumulation is fp32.
// A value beyond the fp16 range sets the error word (kErrRange) rather than
// leaking an infinity.  The output is deterministic (no atomics).
#pragma once

#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "tiled_layout.cuh"
#include "umma.cuh"

namespace m1 {

constexpr int kPfTileTok = 256;   // tokens per tile (the MMA's N, at most 256)
constexpr int kPfRows = 128;      // weight rows per unit (the MMA's M)
constexpr int kPfMaxExperts = 256;
constexpr int kPfMaxTopK = 16;

// A token tile: expert e (global index), its tokens are slots slot0 ..
// slot0+ntok-1; npad = ntok rounded up to 16 (the MMA's N); xoff / aoff:
// byte offsets of its blocks in the gathered-token and activation buffers.
struct PfTile {
    int e, ntok, npad, slot0;
    long long xoff, aoff;
};

struct PrefillParams {
    // model
    const uint8_t *table;     // this layer's tiled expert blocks, experts [e0, e0+ne)
    TiledLayout tl;
    const uint16_t *router;   // bf16 [E][h]
    int E, K, h, I, gs, norm, e0, ne;
    int zblock;               // index of this layer's first block in the table maps
    // call
    int T;
    const void *x;
    int x_bf16;
    const void *res;          // may be null
    int res_bf16;
    void *out;
    int out_bf16;
    int *user_idx;            // optional [T][K]
    float *user_w;            // optional [T][K]
    // scratch
    int *idx;                 // [T][K]
    float *w;                 // [T][K]
    int *tok_slot;            // [T][K] slot of (t, k), or -1 (expert not in this shard)
    int *slot_tok;            // [T*K] token of each slot
    PfTile *tiles;            // [max_tiles]
    int *ntiles;              // device count of tiles
    int max_tiles;
    uint8_t *xg;              // gathered tokens (operand blocks)
    uint8_t *act;             // SwiGLU activations (operand blocks)
    float *ypart;             // [nsplit][T*K][h] down partial sums
    int nsplit;
    int *err;
};

// ------------------------------------------------------------------ route ----
// One CTA (256 threads) per token; dynamic shared memory: x as fp32 [h].
__global__ void __launch_bounds__(256) k_prefill_route(const PrefillParams p) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float lg[kPfMaxExperts];
    __shared__ int sel[kPfMaxTopK];
    __shared__ float wsel[kPfMaxTopK];
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, K = p.K, h = p.h;
    for (int d = tid; d < h; d += 256) xs[d] = load_act(p.x, p.x_bf16, (size_t)t * h + d);
    __syncthreads();
    for (int e = warp; e < E; e += 8) {
        const uint4 *row = reinterpret_cast<const uint4 *>(p.router + (size_t)e * h);
        float acc = 0.f;
        for (int g8 = lane; g8 < h / 8; g8 += 32) {
            const uint4 wv = __ldg(row + g8);
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc = fmaf(__uint_as_float(ww[j] << 16), xs[8 * g8 + 2 * j], acc);
                acc = fmaf(__uint_as_float(ww[j] & 0xFFFF0000u), xs[8 * g8 + 2 * j + 1], acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) lg[e] = acc;
    }
    __syncthreads();
    // rank on the logits (the softmax is monotonic): NaN lowest, -0 == +0,
    // ties to the lower index
    if (tid < E) {
        auto key = [](float v, int e) {
            const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
            uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
            if (v != v) ord = 0u;
            return ((unsigned long long)ord << 32) | (uint32_t)(0xFFFF - e);
        };
        const unsigned long long ki = key(lg[tid], tid);
        int cnt = 0;
        for (int f = 0; f < E; ++f) cnt += key(lg[f], f) > ki ? 1 : 0;
        if (cnt < K) sel[cnt] = tid;
    }
    __syncthreads();
    if (warp == 0) {
        float m = -INFINITY;
        for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float s = 0.f;
        for (int e = lane; e < E; e += 32) s += expf(lg[e] - m);
        s = warp_sum(s);
        const float inv = 1.0f / s;
        if (lane < K) wsel[lane] = expf(lg[sel[lane]] - m) * inv;
        __syncwarp();
        if (p.norm) {
            float sum = 0.f;
            if (lane == 0)
                for (int k = 0; k < K; ++k) sum += wsel[k];
            sum = __shfl_sync(0xffffffffu, sum, 0);
            if (lane < K) wsel[lane] = wsel[lane] / sum;
        }
        __syncwarp();
        if (lane < K) {
            p.idx[t * K + lane] = sel[lane];
            p.w[t * K + lane] = wsel[lane];
            if (p.user_idx) p.user_idx[t * K + lane] = sel[lane];
            if (p.user_w) p.user_w[t * K + lane] = wsel[lane];
        }
    }
}

// ------------------------------------------------------------------- plan ----
// One CTA of 1024 threads: a stable counting sort of the T*K (token, k)
// pairs by local expert, in (t, k) order within an expert, then the token
// tiles.  Per chunk of 1024 pairs: each warp counts its pairs per expert
// (match_any), a scan over the warps gives every pair its rank.
__global__ void __launch_bounds__(1024) k_prefill_plan(const PrefillParams p) {
    __shared__ int cnt[32][kPfMaxExperts];  // per-warp counts, then their running bases
    __shared__ int base[kPfMaxExperts];     // pairs of expert e seen so far / its first slot
    __shared__ int nloc[kPfMaxExperts];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NE = p.ne, n = p.T * p.K;
    // pass 1: pairs per local expert
    for (int e = tid; e < NE; e += 1024) nloc[e] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += 1024) {
        const int e = p.idx[i] - p.e0;
        if (e >= 0 && e < NE) atomicAdd(&nloc[e], 1);
    }
    __syncthreads();
    // slot bases (expert order) and tiles; one thread
    if (tid == 0) {
        int slot = 0, nt = 0;
        long long xo = 0, ao = 0;
        for (int e = 0; e < NE; ++e) {
            base[e] = slot;
            for (int s0 = 0; s0 < nloc[e]; s0 += kPfTileTok) {
                const int nk = min(kPfTileTok, nloc[e] - s0), np = (nk + 15) & ~15;
                if (nt < p.max_tiles)
                    p.tiles[nt] = PfTile{p.e0 + e, nk, np, slot + s0, xo, ao};
                ++nt;
                xo += (long long)np * p.h * 2;
                ao += (long long)np * p.I * 2;
            }
            slot += nloc[e];
        }
        *p.ntiles = nt <= p.max_tiles ? nt : 0;
        if (nt > p.max_tiles) atomicOr(p.err, kErrWaitTimeout);
    }
    __syncthreads();
    // pass 2: stable slots
    for (int c0 = 0; c0 < n; c0 += 1024) {
        for (int k = tid; k < 32 * NE; k += 1024) cnt[k / NE][k % NE] = 0;
        __syncthreads();
        const int i = c0 + tid;
        int e = -1;
        if (i < n) {
            e = p.idx[i] - p.e0;
            if (e < 0 || e >= NE) e = -1;
        }
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int before = __popc(same & ((1u << lane) - 1u));
        if (e >= 0 && before == 0) cnt[warp][e] = __popc(same);
        __syncthreads();
        for (int ee = tid; ee < NE; ee += 1024) {
            int run = base[ee];
            for (int w = 0; w < 32; ++w) {
                const int c = cnt[w][ee];
                cnt[w][ee] = run;
                run += c;
            }
            base[ee] = run;
        }
        __syncthreads();
        if (i < n) {
            const int slot = e >= 0 ? cnt[warp][e] + before : -1;
            p.tok_slot[i] = slot;
            if (slot >= 0) p.slot_tok[slot] = i / p.K;
        }
        __syncthreads();
    }
}

// ----------------------------------------------------------------- gather ----
// Tile rows as tensor-core operand blocks: for 64 columns kb, the tile's npad
// rows (128 bytes each, 128B-swizzled, nibble K order) are one contiguous
// block at off + kb * npad * 128.  Rows beyond ntok are zero.
__device__ __forceinline__ void put_operand_chunk(uint8_t *blk, int npad, int n, int k8,
                                                  const float (&v)[8], int *err) {
    uint32_t o[4];
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 pr = __floats2half2_rn(v[j], v[j + 4]);  // (k = j, k = j + 4)
        o[j] = *reinterpret_cast<const uint32_t *>(&pr);
        bad |= (isinf(__low2float(pr)) && !isinf(v[j])) || (isinf(__high2float(pr)) && !isinf(v[j + 4]));
    }
    if (bad) atomicOr(err, kErrRange);
    const int kb = k8 >> 3, c = k8 & 7;
    *reinterpret_cast<uint4 *>(blk + (size_t)kb * npad * 128 + sw128_offset(n, c)) =
        make_uint4(o[0], o[1], o[2], o[3]);
}

// grid (max_tiles, kPfTileTok / 8), 256 threads: warp = one row of the tile,
// lanes over its h/8 chunks.
__global__ void __launch_bounds__(256) k_prefill_gather(const PrefillParams p) {
    const int ti = blockIdx.x;
    if (ti >= *p.ntiles) return;
    const PfTile tl = p.tiles[ti];
    const int n = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (n >= tl.npad) return;
    const int t = n < tl.ntok ? p.slot_tok[tl.slot0 + n] : -1;
    uint8_t *blk = p.xg + tl.xoff;
    for (int k8 = lane; k8 < p.h / 8; k8 += 32) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = t >= 0 ? load_act(p.x, p.x_bf16, (size_t)t * p.h + 8 * k8 + j) : 0.f;
        put_operand_chunk(blk, tl.npad, n, k8, v, p.err);
    }
}

// ---------------------------------------------------------------- combine ----
// out[t][i] = residual[t][i] + sum_k w[t][k] * y(t, k)[i], k ascending, where
// y(t, k) sums the down product's K splits in order.  grid (T, ceil(h/256)).
__global__ void __launch_bounds__(256) k_prefill_combine(const PrefillParams p) {
    const int t = blockIdx.x, i = blockIdx.y * 256 + threadIdx.x;
    if (i >= p.h) return;
    float acc = p.res ? load_act(p.res, p.res_bf16, (size_t)t * p.h + i) : 0.f;
    const size_t plane = (size_t)p.T * p.K * p.h;
    for (int k = 0; k < p.K; ++k) {
        const int slot = p.tok_slot[t * p.K + k];
        if (slot < 0) continue;
        float y = 0.f;
        for (int s = 0; s < p.nsplit; ++s) y += p.ypart[s * plane + (size_t)slot * p.h + i];
        acc = fmaf(p.w[t * p.K + k], y, acc);
    }
    if (p.out_bf16)
        reinterpret_cast<__nv_bfloat16 *>(p.out)[(size_t)t * p.h + i] = __float2bfloat16_rn(acc);
    else
        reinterpret_cast<float *>(p.out)[(size_t)t * p.h + i] = acc;
}

// ------------------------------------------------------------------- GEMM ----
enum PfKind { kGateUp = 0, kDown = 1 };

// Shared-memory stage: the fp16 A operand(s) (gate and up, or down: 128 rows
// x 64 columns, 16 KB each), the B operand (npad tokens x 64 columns, up to
// 32 KB), and the raw int4 rows the A operands come from (4 KB each).
template <int KIND>
struct PfStage {
    static constexpr int na = KIND == kGateUp ? 2 : 1;
    static constexpr int a_bytes = 16384, b_bytes = 32768, raw_bytes = 4096;
    static constexpr int bytes = na * a_bytes + b_bytes + na * raw_bytes;  // multiple of 1024
    static constexpr int count = KIND == kGateUp ? 3 : 4;
    static constexpr int tmem_cols = KIND == kGateUp ? 512 : 256;
    static constexpr int smem = count * bytes + 2048;  // + alignment slack, barriers, control
};

struct PfCtl {
    uint64_t full[4], deq[4], empty[4], accf, acce, fin;
    uint32_t taddr;
    int abort;
};

// warp 0 copies, 1 issues MMAs, 2 owns TMEM, 4..11 dequantise + epilogue: two
// threads per weight row, each converting 4 of the step's 8 words (with one
// thread per row, one warp per scheduler could not hide the conversion's
// latency: 465 -> 500 TFLOP/s on 512 Mixtral tokens)
constexpr int kPfThreads = 384;

// The units of this kernel: gate/up (tile, 128 rows of I); down (tile, 128
// rows of h, K split), split fastest.
template <int KIND>
__device__ __forceinline__ void pf_unit(const PrefillParams &p, int u, int &tile, int &rb, int &kb0,
                                        int &kb1) {
    const int KB = (KIND == kGateUp ? p.h : p.I) / 64;
    if (KIND == kGateUp) {
        const int nrb = p.I / kPfRows;
        tile = u / nrb;
        rb = u - tile * nrb;
        kb0 = 0;
        kb1 = KB;
    } else {
        const int nrb = p.h / kPfRows, s = u % p.nsplit, r = u / p.nsplit;
        tile = r / nrb;
        rb = r - tile * nrb;
        kb0 = KB * s / p.nsplit;
        kb1 = KB * (s + 1) / p.nsplit;
    }
}

template <int KIND>
__device__ __forceinline__ int pf_units(const PrefillParams &p, int ntiles) {
    return KIND == kGateUp ? ntiles * (p.I / kPfRows) : ntiles * (p.h / kPfRows) * p.nsplit;
}

// The 16-bit value g (0..7) of v, by selects (a dynamic index into a register
// array would go through local memory).
__device__ __forceinline__ uint32_t pick16(const uint4 &v, int g) {
    const uint32_t w01 = (g & 2) ? v.y : v.x, w23 = (g & 2) ? v.w : v.z;
    const uint32_t w = (g & 4) ? w23 : w01;
    return (g & 1) ? (w >> 16) : (w & 0xFFFFu);
}

__device__ __forceinline__ uint32_t pick32(const uint32_t (&v)[8], int g) {
    uint32_t r = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) r = g == j ? v[j] : r;
    return r;
}

// Linear bulk copy without a cache hint.
__device__ __forceinline__ void bulk_g2s_plain(void *dst, const void *src, uint32_t bytes,
                                               uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            (uint32_t)__cvta_generic_to_shared(dst)),
        "l"(src), "r"(bytes), "r"((uint32_t)__cvta_generic_to_shared(bar))
        : "memory");
}

// One CTA per SM (persistent over the units, assigned round-robin).  The
// copy warp loads each 64-column step's raw int4 rows (tensor-map TMA) and
// the B operand (bulk copy) into a stage; the eight dequant warps turn the
// raw rows into the fp16 A operand (two threads per row) and, after a unit's
// last step, read the accumulators from TMEM for the epilogue; one thread
// issues the MMAs (4 per A operand per step, K = 16 each) and commits them
// to the stage's empty barrier and, per unit, to the accumulator barrier.
// All waits are bounded; on timeout the CTA flags the error word and unwinds.
template <int KIND>
__global__ void __launch_bounds__(kPfThreads, 1)
    k_prefill_gemm(const PrefillParams p, const __grid_constant__ CUtensorMap wmap) {
    using St = PfStage<KIND>;
    constexpr int S = St::count, NA = St::na;
    extern __shared__ __align__(128) uint8_t pf_smem_raw[];
    // the operand tiles need 1024-byte alignment (128B-swizzle atoms)
    uint8_t *smem = pf_smem_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(pf_smem_raw) & 1023u)) & 1023u);
    PfCtl &ctl = *reinterpret_cast<PfCtl *>(smem + S * St::bytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const volatile int *vabort = &ctl.abort;
    auto stage_a = [&](int s, int m) { return smem + s * St::bytes + m * St::a_bytes; };
    auto stage_b = [&](int s) { return smem + s * St::bytes + NA * St::a_bytes; };
    auto stage_raw = [&](int s, int m) {
        return smem + s * St::bytes + NA * St::a_bytes + St::b_bytes + m * St::raw_bytes;
    };

    if (tid == 0) {
        ctl.abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&ctl.full[s], 1);
            mbar_init(&ctl.deq[s], 256);
            mbar_init(&ctl.empty[s], 1);
        }
        mbar_init(&ctl.accf, 1);
        mbar_init(&ctl.acce, 256);
        mbar_init(&ctl.fin, 1);
        mbar_fence_init();
    }
    if (warp == 2) {
        tmem_alloc(&ctl.taddr, St::tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t taddr = ctl.taddr;
    const int ntiles = *p.ntiles, nunits = pf_units<KIND>(p, ntiles);
    const int G = gridDim.x;
    const TiledLayout &tl = p.tl;

    if (warp == 0) {
        // ================= copies =================
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += G) {
                int ti, rb, kb0, kb1;
                pf_unit<KIND>(p, u, ti, rb, kb0, kb1);
                const PfTile t = p.tiles[ti];
                const int z = p.zblock + (t.e - p.e0);
                const uint8_t *bsrc = (KIND == kGateUp ? p.xg + t.xoff : p.act + t.aoff);
                const uint32_t bbytes = (uint32_t)t.npad * 128;
                for (int kb = kb0; kb < kb1 && ok; ++kb, ++it) {
                    const int s = it % S;
                    if (it >= S) ok = mbar_wait(&ctl.empty[s], ((it / S) + 1) & 1, &ctl.abort, p.err);
                    if (!ok) break;
                    mbar_arrive_expect_tx(&ctl.full[s], NA * St::raw_bytes + bbytes);
                    if (KIND == kGateUp) {
                        const int wo_u = p.h / 2 + 2 * tl.sbh;  // the up half of a pair-row
                        tma_load_3d(stage_raw(s, 0), &wmap, kb * 32, rb * kPfRows, z, &ctl.full[s]);
                        tma_load_3d(stage_raw(s, 1), &wmap, wo_u + kb * 32, rb * kPfRows, z, &ctl.full[s]);
                    } else {
                        const int i0 = rb * kPfRows, ic = i0 / tl.rc;
                        tma_load_3d(stage_raw(s, 0), &wmap, i0 - ic * tl.rc, ic * tl.ncbI + kb * 8, z,
                                    &ctl.full[s]);
                    }
                    bulk_g2s_plain(stage_b(s), bsrc + (size_t)kb * bbytes, bbytes, &ctl.full[s]);
                }
            }
            // copies still in flight land before the CTA may exit
            for (int k = 0; k < S && ok == false; ++k) {
                const int j = it - 1 - k;
                if (j < 0) break;
                for (uint32_t i = 0; i < kWaitLimit; ++i)
                    if (mbar_try_wait(&ctl.full[j % S], (j / S) & 1)) break;
            }
        }
    } else if (warp == 1) {
        // ================= MMA issue =================
        if (lane == 0) {
            int it = 0, ui = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += G, ++ui) {
                int ti, rb, kb0, kb1;
                pf_unit<KIND>(p, u, ti, rb, kb0, kb1);
                const int npad = p.tiles[ti].npad;
                const uint32_t idesc = umma_idesc_f16(kPfRows, npad);
                if (ui > 0) ok = mbar_wait(&ctl.acce, (ui - 1) & 1, &ctl.abort, p.err);
                tc_fence_after_sync();
                for (int kb = kb0; kb < kb1 && ok; ++kb, ++it) {
                    const int s = it % S;
                    ok = mbar_wait(&ctl.deq[s], (it / S) & 1, &ctl.abort, p.err);
                    if (!ok) break;
                    tc_fence_after_sync();
                    const uint32_t b0 = (uint32_t)__cvta_generic_to_shared(stage_b(s));
#pragma unroll
                    for (int m = 0; m < NA; ++m) {
                        const uint32_t a0 = (uint32_t)__cvta_generic_to_shared(stage_a(s, m));
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            umma_f16(taddr + m * 256, umma_desc_sw128(a0 + 32 * k),
                                      umma_desc_sw128(b0 + 32 * k), idesc, kb > kb0 || k > 0);
                    }
                    umma_commit(&ctl.empty[s]);
                }
                if (ok) umma_commit(&ctl.accf);
            }
            // every MMA issued has completed before TMEM is released
            umma_commit(&ctl.fin);
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(&ctl.fin, 0)) break;
        }
    } else if (warp >= 4) {
        // ========== dequant + epilogue (two threads per row: halves hf 0/1) ==========
        // row r (TMEM lane r: warps 4+q and 8+q both read lanes 32q .. 32q+31);
        // half hf converts words 4hf .. 4hf+3 and reads every other 16 columns
        const int dq = tid - 128, r = dq & 127, hf = dq >> 7, q = warp & 3;
        int it = 0, ui = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok; u += G, ++ui) {
            int ti, rb, kb0, kb1;
            pf_unit<KIND>(p, u, ti, rb, kb0, kb1);
            const PfTile t = p.tiles[ti];
            const uint8_t *blk = p.table + (size_t)(t.e - p.e0) * tl.block;
            const int R = rb * kPfRows + r;  // this thread's weight row
            // scales and biases, 8 groups (= 8 steps) at a time
            uint4 sc[4];
            uint32_t dsb[8];
            for (int kb = kb0; kb < kb1 && ok; ++kb, ++it) {
                if (kb == kb0 || (kb & 7) == 0) {
                    const int g0 = kb & ~7;
                    if (KIND == kGateUp) {
                        const uint8_t *row = blk + (size_t)R * tl.pr + p.h / 2 + 2 * g0;
                        const size_t up = (size_t)p.h / 2 + 2 * tl.sbh;
                        sc[0] = __ldg(reinterpret_cast<const uint4 *>(row));
                        sc[1] = __ldg(reinterpret_cast<const uint4 *>(row + tl.sbh));
                        sc[2] = __ldg(reinterpret_cast<const uint4 *>(row + up));
                        sc[3] = __ldg(reinterpret_cast<const uint4 *>(row + up + tl.sbh));
                    } else {
                        const int ic = R / tl.rc, ri = R - ic * tl.rc;
                        const uint32_t *sbw = reinterpret_cast<const uint32_t *>(blk + tl.dn_sb);
                        for (int j = 0; j < 8; ++j)
                            dsb[j] = g0 + j < tl.ngI ? __ldg(sbw + ((size_t)ic * tl.ngI + g0 + j) * tl.rc + ri) : 0u;
                    }
                }
                const int s = it % S, gj = kb & 7;
                ok = mbar_wait(&ctl.full[s], (it / S) & 1, &ctl.abort, p.err);
                if (!ok) break;
#pragma unroll
                for (int m = 0; m < NA; ++m) {
                    uint32_t w[8];
                    uint32_t s2, b2;
                    if (KIND == kGateUp) {
                        const uint4 *rw = reinterpret_cast<const uint4 *>(stage_raw(s, m) + r * 32);
                        const uint4 w0 = rw[hf];
                        w[0] = w0.x, w[1] = w0.y, w[2] = w0.z, w[3] = w0.w;
                        s2 = bf16_to_f16_pair(pick16(sc[2 * m], gj));
                        b2 = bf16_to_f16_pair(pick16(sc[2 * m + 1], gj));
                    } else {
                        const uint32_t *rw = reinterpret_cast<const uint32_t *>(stage_raw(s, 0));
#pragma unroll
                        for (int c = 0; c < 4; ++c) w[c] = rw[(4 * hf + c) * 128 + r];
                        const uint32_t sb = pick32(dsb, gj);
                        s2 = bf16_to_f16_pair(sb);
                        b2 = bf16_to_f16_pair(sb >> 16);
                    }
                    uint8_t *a = stage_a(s, m);
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4 *>(a + sw128_offset(r, 4 * hf + c)) = dequant_word_f16(w[c], s2, b2);
                }
                fence_proxy_async_smem();
                mbar_arrive(&ctl.deq[s]);
            }
            if (!ok) break;
            // ---- epilogue: the unit's accumulators ----
            ok = mbar_wait(&ctl.accf, ui & 1, &ctl.abort, p.err);
            if (!ok) break;
            tc_fence_after_sync();
            const uint32_t tl_row = taddr + ((uint32_t)(32 * q) << 16);
            for (int n0 = 16 * hf; n0 < t.npad; n0 += 32) {
                uint32_t g[16], v[16];
                tmem_ld16(tl_row + n0, g);
                if (KIND == kGateUp) tmem_ld16(tl_row + 256 + n0, v);
                tmem_wait_ld();
                if (KIND == kGateUp) {
                    // SwiGLU (Shaders.metal:147-148) -> fp16 at (token n, column R)
                    // of the down product's B operand
                    uint8_t *ab = p.act + t.aoff + (size_t)(R >> 6) * t.npad * 128;
                    const int c = (R & 63) >> 3, pos = kperm_pos(R & 7);
                    bool bad = false;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = n0 + j;
                        const float gv = __uint_as_float(g[j]), uv = __uint_as_float(v[j]);
                        const float av = n < t.ntok ? (gv / (1.0f + expf(-gv))) * uv : 0.f;
                        const __half hv = __float2half_rn(av);
                        bad |= isinf(__half2float(hv)) && !isinf(av);
                        *reinterpret_cast<__half *>(ab + sw128_offset(n, c) + 2 * pos) = hv;
                    }
                    if (bad) atomicOr(p.err, kErrRange);
                } else {
                    const int split = u % p.nsplit;
                    float *yp = p.ypart + (size_t)split * p.T * p.K * p.h;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = n0 + j;
                        if (n < t.ntok) yp[(size_t)(t.slot0 + n) * p.h + R] = __uint_as_float(g[j]);
                    }
                }
            }
            tc_fence_before_sync();
            mbar_arrive(&ctl.acce);
        }
        (void)vabort;
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    if (warp == 2) tmem_dealloc(taddr, St::tmem_cols);
}

}  // namespace m1
