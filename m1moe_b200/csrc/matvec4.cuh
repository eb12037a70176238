// matvec4.cuh — decode-time int4 group-quantised matvec (batch 1..8).
//
// Replaces matvec4bit (Shaders.metal:39-92).  The reference gives each output
// row a 64-thread threadgroup that walks 4-byte words; here a warp owns R
// consecutive rows and each lane streams 16-byte chunks (32 columns) with
// read-only, no-L1-allocate loads, so one warp-wide load moves 512 contiguous
// bytes.  The next chunk's weights are fetched before the current chunk is
// reduced (register double buffering) to keep >= 2R loads in flight per lane.
// Accumulation is fp32 FMA with a butterfly warp reduction.
#pragma once

#include "common.cuh"

namespace m1 {

struct MatvecParams {
    const uint8_t *w;
    const uint8_t *s;
    const uint8_t *b;
    long long mat_stride;  // bytes between consecutive matrices (W, S, B alike)
    int num_mats;
    const void *x;         // [ntok][in_dim]
    int x_bf16;
    void *y;               // [num_mats][ntok][out_dim]
    int y_bf16;
    int out_dim, in_dim, gs, ntok;
};

template <int R>
struct ChunkW {
    uint4 w[R];
    float s[R], b[R];
};

template <int R>
__device__ __forceinline__ void load_chunk_rows(ChunkW<R> &c, const uint8_t *wm, const uint8_t *sm,
                                                const uint8_t *bm, int r0, int out_dim,
                                                size_t wrow, size_t srow, int ch, int gs) {
    const int gi = (ch * kChunkCols) / gs;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int row = r0 + r;
        if (row < out_dim) {
            c.w[r] = ld_stream16(wm + (size_t)row * wrow + (size_t)ch * 16);
            c.s[r] = bf16_bits(ld_u16(sm + (size_t)row * srow + (size_t)gi * 2));
            c.b[r] = bf16_bits(ld_u16(bm + (size_t)row * srow + (size_t)gi * 2));
        } else {
            c.w[r] = make_uint4(0, 0, 0, 0);
            c.s[r] = 0.f;
            c.b[r] = 0.f;
        }
    }
}

// grid: any size (work split evenly over CTAs); block: 256 threads.
template <int NT, int R>
__global__ void __launch_bounds__(256) k_matvec4(const MatvecParams p) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int gpm = (p.out_dim + R - 1) / R;  // row groups per matrix
    long long gb, ge;
    split_range((long long)p.num_mats * gpm, gridDim.x, blockIdx.x, gb, ge);
    const int nch = p.in_dim / kChunkCols;
    const size_t wrow = (size_t)p.in_dim / 2;
    const size_t srow = (size_t)(p.in_dim / p.gs) * 2;
    const size_t xtok = (size_t)p.in_dim * (p.x_bf16 ? 2 : 4);

    for (long long g = gb + warp; g < ge; g += nwarps) {
        const int m = (int)(g / gpm);
        const int r0 = (int)(g % gpm) * R;
        const uint8_t *wm = p.w + (size_t)m * p.mat_stride;
        const uint8_t *sm = p.s + (size_t)m * p.mat_stride;
        const uint8_t *bm = p.b + (size_t)m * p.mat_stride;
        float acc[R][NT];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;

        int ch = lane;
        ChunkW<R> cur;
        if (ch < nch) load_chunk_rows<R>(cur, wm, sm, bm, r0, p.out_dim, wrow, srow, ch, p.gs);
        while (ch < nch) {
            const int nxt = ch + kWarp;
            ChunkW<R> nb;
            if (nxt < nch) load_chunk_rows<R>(nb, wm, sm, bm, r0, p.out_dim, wrow, srow, nxt, p.gs);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < p.ntok) {
                    float xv[32];
                    const float X = load_x32(
                        reinterpret_cast<const uint8_t *>(p.x) + (size_t)t * xtok, p.x_bf16,
                        ch * kChunkCols, xv);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float Q = dot_chunk(cur.w[r], xv);
                        acc[r][t] = fmaf(cur.s[r], Q, fmaf(cur.b[r], X, acc[r][t]));
                    }
                }
            }
            if (nxt < nch) cur = nb;
            ch = nxt;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(acc[r][t]);
                const int row = r0 + r;
                if (lane == 0 && t < p.ntok && row < p.out_dim)
                    store_act(p.y, p.y_bf16, ((size_t)m * p.ntok + t) * p.out_dim + row, v);
            }
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
