// matvec4.cuh — decode-time int4 group-quantised matvec (batch 1..8).
//
// Replaces matvec4bit (Shaders.metal:39-92) on the reference's own layout
// (W uint32 [out][in/8], S/B bf16 [out][in/gs]), for one matrix or a run of
// matrices `mat_stride` bytes apart that share x.  The reference gives each
// output row a 64-thread threadgroup that walks 4-byte words; here:
//   * each CTA stages x once in shared memory, quantised per 32-value chunk
//     to int16 (dp2a layout, common.cuh) with the chunk's scale and exact sum;
//   * a warp owns R consecutive rows; lane L streams 16-byte chunks (32
//     columns) L, L+32, ... with read-only no-L1-allocate loads, the next
//     round's R loads in flight while the current round is computed
//     (register double buffering; three CTAs of 8 warps per SM);
//   * the inner loop is two masks and four dp2a per weight word (int32
//     partial sum per chunk, exact), then s*sx*Q + b*X per chunk in fp32,
//     then one multi-value butterfly reduction per warp.
#pragma once

#include "common.cuh"
#include "pipeline.cuh"

namespace m1 {

struct MatvecParams {
    const uint8_t *w;
    const uint8_t *s;
    const uint8_t *b;
    long long mat_stride;  // bytes between consecutive matrices (W, S, B alike)
    int num_mats;
    const void *x;         // [ntok][in_dim]
    int x_bf16;
    void *y;               // [num_mats][y_ntok][out_dim]; this launch writes tokens y_t0..
    int y_bf16;
    int out_dim, in_dim, gs, ntok;
    int y_ntok, y_t0;      // token count of y's layout, first token of this launch
};

constexpr int kMatvecThreads = 256;

// Rows per warp for NT tokens.
template <int NT>
struct MatvecRows {
    static constexpr int R = NT <= 2 ? 4 : 2;
};

// Dynamic shared memory: xq [NT][in/2] int16 pairs + scale and sum f32 [NT][in/32].
__host__ __device__ inline size_t matvec_smem(int nt, int in_dim) {
    return (size_t)nt * in_dim * 2 + (size_t)nt * (in_dim / kChunkCols) * 8;
}

// Stage x (ntok tokens) as int16 chunks: one thread per chunk.
__device__ __forceinline__ void stage_x_i16(const MatvecParams &p, uint32_t *xq, float *xsc,
                                            float *xsum, int tid, int nthreads) {
    const int in = p.in_dim, nch = in / kChunkCols;
    for (int q = tid; q < p.ntok * nch; q += nthreads) {
        const int t = q / nch, c = q - t * nch;
        float v[32];
        load_x32_any(p.x, p.x_bf16, (size_t)t * in + (size_t)c * kChunkCols, v);
        xsc[q] = quant_chunk_i16(v, xq + (size_t)t * (in / 2), nch, c, &xsum[q]);
    }
}

template <int NT>
__global__ void __launch_bounds__(kMatvecThreads, 3) k_matvec4(const MatvecParams p) {
    constexpr int R = MatvecRows<NT>::R;
    constexpr int kNv = R * NT;  // values reduced per warp: [row][token]
    extern __shared__ __align__(128) uint8_t smem[];
    const int in = p.in_dim, nch = in / kChunkCols;
    uint32_t *xq = reinterpret_cast<uint32_t *>(smem);
    float *xsc = reinterpret_cast<float *>(smem + (size_t)NT * in * 2);
    float *xsum = xsc + NT * nch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    stage_x_i16(p, xq, xsc, xsum, tid, kMatvecThreads);
    __syncthreads();

    // ---- rows: warp-strided units of R rows, one 32-chunk round per step ----
    // Register double buffering: the loads of step n+1 are in flight while
    // step n is reduced.
    const int gpm = (p.out_dim + R - 1) / R;
    const long long units = (long long)p.num_mats * gpm;
    const size_t wrow = (size_t)in / 2, srow = (size_t)(in / p.gs) * 2;
    const int nwarps = gridDim.x * (kMatvecThreads / 32);
    const int rounds = (nch + 31) / 32;
    struct Step {
        uint4 w[R];
        uint32_t sb[R];  // scale (low half) and bias (high half), bf16
    };
    auto load_step = [&](Step &st, long long u, int k) {
        const int m = (int)(u / gpm), r0 = (int)(u % gpm) * R;
        const int ch = 32 * k + lane, gi = (ch * kChunkCols) / p.gs;
        const size_t mo = (size_t)m * p.mat_stride;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = r0 + r;
            if (ch < nch && row < p.out_dim) {
                st.w[r] = ld_stream16(p.w + mo + (size_t)row * wrow + (size_t)ch * 16);
                st.sb[r] = (uint32_t)ld_u16(p.s + mo + (size_t)row * srow + (size_t)gi * 2) |
                           ((uint32_t)ld_u16(p.b + mo + (size_t)row * srow + (size_t)gi * 2) << 16);
            } else {
                st.w[r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
                st.sb[r] = 0u;
            }
        }
    };
    long long u = (long long)blockIdx.x * (kMatvecThreads / 32) + warp;
    int k = 0;
    Step cur, nxt;
    if (u < units) load_step(cur, u, 0);
    float acc[kNv];
#pragma unroll
    for (int i = 0; i < kNv; ++i) acc[i] = 0.f;
    while (u < units) {
        long long un = u;
        int kn = k + 1;
        if (kn == rounds) {
            kn = 0;
            un = u + nwarps;
        }
        if (un < units) load_step(nxt, un, kn);
        const int ch = 32 * k + lane;
        if (ch < nch) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t >= p.ntok) continue;
                uint32_t xp[16];
                load_pairs_any(reinterpret_cast<const uint16_t *>(xq + (size_t)t * (in / 2)), nch, ch, xp);
                const float X = xsum[t * nch + ch], sx = xsc[t * nch + ch];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float sc = bf16_bits(cur.sb[r] & 0xFFFFu);
                    const float bi = bf16_bits(cur.sb[r] >> 16);
                    float &a = acc[r * NT + t];
                    a = fmaf(sc * sx, (float)dot_chunk_i16(cur.w[r], xp), fmaf(bi, X, a));
                }
            }
        }
        if (kn == 0) {
            // lane holds value lane / (32/kNv) = r*NT + t
            const float tot = warp_reduce_multi(acc);
            constexpr int kS = 32 / kNv;
            const int m = (int)(u / gpm), r0 = (int)(u % gpm) * R;
            if (lane % kS == 0) {
                const int v = lane / kS, r = v / NT, t = v % NT, row = r0 + r;
                if (t < p.ntok && row < p.out_dim)
                    store_act(p.y, p.y_bf16, ((size_t)m * p.y_ntok + p.y_t0 + t) * p.out_dim + row, tot);
            }
#pragma unroll
            for (int i = 0; i < kNv; ++i) acc[i] = 0.f;
        }
        cur = nxt;
        u = un;
        k = kn;
    }
}

// ---------------------------------------------------------------------------
// Ring variant for streams of matrices: one CTA per SM; a producer warp copies
// tiles of TR rows ([W rows | S rows | B rows], three bulk copies into one
// shared-memory stage) through a ring of NST stages; 16 consumer warps take
// (tile, 4 rows) items and reduce from shared memory.  Bytes in flight are the
// ring (up to ~200 KB per SM), not registers, so the stream runs at HBM speed.
// Needs 16-byte aligned rows: in/2 and (in/gs)*2 bytes, and W/S/B bases.
// ---------------------------------------------------------------------------
constexpr int kRingConsumers = 16;
constexpr int kRingThreads = (kRingConsumers + 1) * 32;
constexpr int kRingRows = 4;  // the tile's row count is a multiple of this
constexpr int kRingMaxStages = 16;

// Rows per work item for NT tokens (R * NT accumulators per lane).
template <int NT>
struct RingRows {
    static constexpr int R = NT <= 2 ? 4 : 2;
};

struct MatvecRing {
    int tile_rows, nstages, stage_bytes, off_bars, off_ctl, off_xs, off_xsum;
};

struct RingCtl {
    int abort;
    int next;
    int issued;
    int stage_tile[kRingMaxStages];
    int stage_done[kRingMaxStages];
};

__device__ __forceinline__ bool ring_wait_tile(uint64_t *full, RingCtl &ctl, int s, int n,
                                               int nstages, int *err) {
    bool ok = false;
    for (uint32_t i = 0, nap = 64; i < kWaitLimit; ++i) {
        if (*reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) == n) {
            ok = true;
            break;
        }
        if (*reinterpret_cast<volatile int *>(&ctl.abort)) break;
        __nanosleep(nap);
        nap = min(nap * 2, 512u);
    }
    if (!ok && !*reinterpret_cast<volatile int *>(&ctl.abort)) {
        *reinterpret_cast<volatile int *>(&ctl.abort) = 1;
        if (err) atomicOr(err, kErrWaitTimeout);
    }
    if (ok) ok = mbar_wait(&full[s], (n / nstages) & 1, &ctl.abort, err);
    return __all_sync(0xffffffffu, ok);
}

template <int NT>
__global__ void __launch_bounds__(kRingThreads, 1) k_matvec4_ring(const MatvecParams p,
                                                                  const MatvecRing g, int *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int in = p.in_dim, nch = in / kChunkCols, TR = g.tile_rows, NST = g.nstages;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + g.off_bars);
    uint64_t *empty = full + NST;
    RingCtl &ctl = *reinterpret_cast<RingCtl *>(smem + g.off_ctl);
    uint32_t *xq = reinterpret_cast<uint32_t *>(smem + g.off_xs);
    float *xsc = reinterpret_cast<float *>(smem + g.off_xsum);
    float *xsum = xsc + NT * nch;
    const size_t wrow = (size_t)in / 2, srow = (size_t)(in / p.gs) * 2;
    const int tpm = (p.out_dim + TR - 1) / TR;  // tiles per matrix
    const long long ntiles_all = (long long)p.num_mats * tpm;
    // this CTA's tiles: blockIdx.x, blockIdx.x + G, ...
    const int ntiles = ntiles_all > blockIdx.x
                           ? (int)((ntiles_all - blockIdx.x + gridDim.x - 1) / gridDim.x) : 0;
    if (tid == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
            ctl.stage_tile[i] = -1;
            ctl.stage_done[i] = 0;
        }
        ctl.abort = 0;
        ctl.next = 0;
        ctl.issued = 0;
        mbar_fence_init();
    }
    // stage x (consumers; the producer starts copying at once)
    if (warp < kRingConsumers) stage_x_i16(p, xq, xsc, xsum, tid, kRingConsumers * 32);
    __syncthreads();
    if (warp == kRingConsumers) {
        // ================= producer =================
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int n = 0;
            for (; n < ntiles; ++n) {
                const int s = n % NST;
                if (n >= NST && !mbar_wait(&empty[s], ((n / NST) - 1) & 1, &ctl.abort, err)) break;
                const long long tg = blockIdx.x + (long long)n * gridDim.x;
                const int m = (int)(tg / tpm), r0 = (int)(tg % tpm) * TR;
                const int nr = min(TR, p.out_dim - r0);
                const size_t mo = (size_t)m * p.mat_stride;
                const uint32_t bw = (uint32_t)(nr * wrow), bs = (uint32_t)(nr * srow);
                uint8_t *dst = ring + (size_t)s * g.stage_bytes;
                mbar_arrive_expect_tx(&full[s], bw + 2 * bs);
                bulk_g2s(dst, p.w + mo + (size_t)r0 * wrow, bw, &full[s], pol);
                bulk_g2s(dst + (size_t)TR * wrow, p.s + mo + (size_t)r0 * srow, bs, &full[s], pol);
                bulk_g2s(dst + (size_t)TR * (wrow + srow), p.b + mo + (size_t)r0 * srow, bs, &full[s], pol);
                *reinterpret_cast<volatile int *>(&ctl.stage_tile[s]) = n;
            }
            ctl.issued = n;
        }
    } else {
        // ================= consumers =================
        constexpr int R = RingRows<NT>::R, kNv = R * NT, kS = 32 / kNv;
        const int ipt = TR / R;  // items per tile
        // chunk -> group: a shift when gs/32 is a power of two
        const int cpg = p.gs / kChunkCols;
        const int gshift = (cpg & (cpg - 1)) == 0 ? __ffs(cpg) - 1 : -1;
        const int nitems = ntiles * ipt;
        for (;;) {
            int q = 0;
            if (lane == 0) q = atomicAdd(&ctl.next, 1);
            q = __shfl_sync(0xffffffffu, q, 0);
            if (q >= nitems) break;
            const int n = q / ipt, grp = q - n * ipt, s = n % NST;
            if (!ring_wait_tile(full, ctl, s, n, NST, err)) break;
            const long long tg = blockIdx.x + (long long)n * gridDim.x;
            const int m = (int)(tg / tpm), r0 = (int)(tg % tpm) * TR;
            const uint8_t *st = ring + (size_t)s * g.stage_bytes;
            const uint8_t *sS = st + (size_t)TR * wrow, *sB = sS + (size_t)TR * srow;
            float acc[kNv];
#pragma unroll
            for (int i = 0; i < kNv; ++i) acc[i] = 0.f;
            const uint8_t *wr = st + (size_t)grp * R * wrow;
            const uint16_t *sr = reinterpret_cast<const uint16_t *>(sS + (size_t)grp * R * srow);
            const uint16_t *br = reinterpret_cast<const uint16_t *>(sB + (size_t)grp * R * srow);
            const int sstep = (int)(srow / 2);
            for (int ch = lane; ch < nch; ch += 32) {
                const int gi = gshift >= 0 ? ch >> gshift : ch / cpg;
                float sc[R], bi[R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    sc[r] = bf16_bits(sr[r * sstep + gi]);
                    bi[r] = bf16_bits(br[r * sstep + gi]);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t >= p.ntok) continue;
                    uint32_t xp[16];
                    load_pairs_any(reinterpret_cast<const uint16_t *>(xq + (size_t)t * (in / 2)), nch, ch, xp);
                    const float X = xsum[t * nch + ch], sx = xsc[t * nch + ch];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint4 w = *reinterpret_cast<const uint4 *>(wr + (size_t)r * wrow + ch * 16);
                        float &a = acc[r * NT + t];
                        a = fmaf(sc[r] * sx, (float)dot_chunk_i16(w, xp), fmaf(bi[r], X, a));
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && atomicAdd(&ctl.stage_done[s], 1) == ipt - 1) {
                ctl.stage_done[s] = 0;
                mbar_arrive(&empty[s]);
            }
            const float tot = warp_reduce_multi(acc);
            if (lane % kS == 0) {
                const int v = lane / kS, r = v / NT, t = v % NT, row = r0 + grp * R + r;
                if (t < p.ntok && row < p.out_dim)
                    store_act(p.y, p.y_bf16, ((size_t)m * p.y_ntok + p.y_t0 + t) * p.out_dim + row, tot);
            }
        }
    }
    __syncthreads();
    if (ctl.abort && tid == 0) {
        for (int n = ctl.issued - NST; n < ctl.issued; ++n) {
            if (n < 0) continue;
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(&full[n % NST], (n / NST) & 1)) break;
        }
    }
}

// q[r][c] = (W[r][c/8] >> 4*(c%8)) & 0xF — one thread per 32-bit word.
__global__ void k_unpack4(const uint32_t *__restrict__ w, uint8_t *__restrict__ q,
                          long long nwords) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nwords;
         i += (long long)gridDim.x * blockDim.x) {
        const uint32_t u = w[i];
        uint2 o;
        o.x = (u & 0xFu) | ((u >> 4 & 0xFu) << 8) | ((u >> 8 & 0xFu) << 16) | ((u >> 12 & 0xFu) << 24);
        o.y = (u >> 16 & 0xFu) | ((u >> 20 & 0xFu) << 8) | ((u >> 24 & 0xFu) << 16) |
              ((u >> 28 & 0xFu) << 24);
        reinterpret_cast<uint2 *>(q)[i] = o;
    }
}

}  // namespace m1
