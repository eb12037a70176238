// common.cuh — device helpers shared by the int4 expert-FFN kernels (sm_100a).
//
// Weight format (the reference's, unchanged; scripts/extract_olmoe.py:20-38,
// :145-150): a projection with `rows` outputs and `cols` inputs is
//   W  uint32[rows][cols/8]   nibble b of word w is column 8w+b (low nibble first)
//   S  bf16  [rows][cols/gs]  per-group scale
//   B  bf16  [rows][cols/gs]  per-group bias
// and dequantises as w = q*S + B (Shaders.metal:73-77).
//
// Arithmetic: a lane owns one 16-byte "chunk" = 4 words = 32 consecutive
// columns, which lie inside one group because gs % 32 == 0.  Per chunk
//   sum_j (q_j*s + b)*x_j = s * sum_j q_j*x_j + b * sum_j x_j
// so the inner loop is one exact nibble->float conversion and one fp32 FMA
// per weight; the scale/bias terms are applied once per chunk.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace m1 {

constexpr int kWarp = 32;
constexpr int kChunkCols = 32;  // columns per 16-byte weight chunk

__device__ __forceinline__ float bf16_bits(uint32_t b16) { return __uint_as_float(b16 << 16); }

// 16-byte streaming load of weights: read-only path, no L1 allocation
// (each weight byte is used exactly once per call).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ld_u16(const void *p) {
    return __ldg(reinterpret_cast<const unsigned short *>(p));
}

// Exact nibble -> float: 2^23 + q has q in its low mantissa bits; subtracting
// 2^23 is exact.  (A float with exponent 150 has ulp 1.)
__device__ __forceinline__ float nib_to_f32(uint32_t word, int b) {
    return __uint_as_float(0x4B000000u | ((word >> (4 * b)) & 0xFu)) - 8388608.0f;
}

// Q = sum_{j<32} q_j * x_j for one 16-byte chunk (exact q, fp32 FMA).
__device__ __forceinline__ float dot_chunk(const uint4 w, const float (&x)[32]) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t u = ws[i];
        a0 = fmaf(nib_to_f32(u, 0), x[8 * i + 0], a0);
        a1 = fmaf(nib_to_f32(u, 1), x[8 * i + 1], a1);
        a2 = fmaf(nib_to_f32(u, 2), x[8 * i + 2], a2);
        a3 = fmaf(nib_to_f32(u, 3), x[8 * i + 3], a3);
        a0 = fmaf(nib_to_f32(u, 4), x[8 * i + 4], a0);
        a1 = fmaf(nib_to_f32(u, 5), x[8 * i + 5], a1);
        a2 = fmaf(nib_to_f32(u, 6), x[8 * i + 6], a2);
        a3 = fmaf(nib_to_f32(u, 7), x[8 * i + 7], a3);
    }
    return (a0 + a1) + (a2 + a3);
}

// Load 32 consecutive activations (f32 or bf16, selected at run time) into
// registers as f32, and return their sum.
__device__ __forceinline__ float load_x32(const void *xbase, int is_bf16, int col,
                                          float (&x)[32]) {
    if (is_bf16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(
            reinterpret_cast<const uint16_t *>(xbase) + col);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldg(p + i);
            const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                x[8 * i + 2 * j] = __uint_as_float(vv[j] << 16);
                x[8 * i + 2 * j + 1] = __uint_as_float(vv[j] & 0xFFFF0000u);
            }
        }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(
            reinterpret_cast<const float *>(xbase) + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = __ldg(p + i);
            x[4 * i + 0] = v.x;
            x[4 * i + 1] = v.y;
            x[4 * i + 2] = v.z;
            x[4 * i + 3] = v.w;
        }
    }
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        s0 += x[j];
        s1 += x[j + 1];
    }
    return s0 + s1;
}

__device__ __forceinline__ float load_act(const void *base, int is_bf16, size_t i) {
    if (is_bf16) return bf16_bits(ld_u16(reinterpret_cast<const uint16_t *>(base) + i));
    return __ldg(reinterpret_cast<const float *>(base) + i);
}

__device__ __forceinline__ void store_act(void *base, int is_bf16, size_t i, float v) {
    if (is_bf16)
        reinterpret_cast<__nv_bfloat16 *>(base)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float *>(base)[i] = v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Reduce N values (N a power of two, 1..32) over the lanes of a warp with
// N-1 + log2(32/N) shuffles instead of 5N: each stage exchanges half of the
// remaining values.  Afterwards lane l holds, in v[0], the warp total of value
// l / (32/N).
template <int N>
__device__ __forceinline__ float warp_reduce_multi(float (&v)[N]) {
    static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N must be a power of two <= 32");
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int st = 0; st < 5; ++st) {
        const int o = 16 >> st;
        if ((N >> st) > 1) {
            const int half = N >> (st + 1);
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < half) {
                    const float send = up ? v[i] : v[i + half];
                    const float keep = up ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

// ---------------------------------------------------------------------------
// bf16 inner loop (the decode hot path).
//
// Weights: one 32-bit word holds 8 nibbles q0..q7 (columns 8w..8w+7).  A single
// LOP3 turns nibbles k and k+4 into the bf16 pair (128+q_k, 128+q_{k+4}):
// 0x4300 is bf16 128.0, whose mantissa ulp is 1, so OR-ing q into the low
// mantissa bits is exact.  Activations are bf16 pairs (x_k, x_{k+4}) in the
// same order ("pair-permuted").  fma.rn.f32.bf16 multiplies two bf16 values
// exactly into fp32 and accumulates in fp32, so per chunk
//     A = sum_j (128 + q_j) * x_j = 128*X + Q,   X = sum_j x_j,
// and the projection row accumulates  s*A + (b - 128*s)*X.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t q_pair(uint32_t word, int k) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;"  // (a & b) | c
        : "=r"(d)
        : "r"(word >> (4 * k)), "r"(0x000F000Fu), "r"(0x43004300u));
    return d;
}

// acc + a.lo*b.lo + a.hi*b.hi, exact bf16 products, fp32 accumulation.
__device__ __forceinline__ float fma_pair(uint32_t a, uint32_t b, float acc) {
    float d;
    asm("{ .reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %3;\n\t"
        "fma.rn.f32.bf16 %0, ah, bh, %0; }"
        : "=f"(d)
        : "r"(a), "r"(b), "f"(acc));
    return d;
}

// A = sum_j (128 + q_j) x_j over one 16-byte weight chunk; xp holds the
// chunk's 16 pair-permuted bf16 pairs (word i, pair k at xp[4*i + k]).
__device__ __forceinline__ float dot_chunk_bf16(const uint4 w, const uint32_t (&xp)[16]) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        a0 = fma_pair(q_pair(w.x, k), xp[0 + k], a0);
        a1 = fma_pair(q_pair(w.y, k), xp[4 + k], a1);
        a2 = fma_pair(q_pair(w.z, k), xp[8 + k], a2);
        a3 = fma_pair(q_pair(w.w, k), xp[12 + k], a3);
    }
    return (a0 + a1) + (a2 + a3);
}

// A over two chunks (64 columns) with shared partial accumulators.
__device__ __forceinline__ float dot_chunk2_bf16(const uint4 w0, const uint32_t (&x0)[16],
                                                 const uint4 w1, const uint32_t (&x1)[16]) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        a0 = fma_pair(q_pair(w0.x, k), x0[0 + k], a0);
        a1 = fma_pair(q_pair(w0.y, k), x0[4 + k], a1);
        a2 = fma_pair(q_pair(w0.z, k), x0[8 + k], a2);
        a3 = fma_pair(q_pair(w0.w, k), x0[12 + k], a3);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        a0 = fma_pair(q_pair(w1.x, k), x1[0 + k], a0);
        a1 = fma_pair(q_pair(w1.y, k), x1[4 + k], a1);
        a2 = fma_pair(q_pair(w1.z, k), x1[8 + k], a2);
        a3 = fma_pair(q_pair(w1.w, k), x1[12 + k], a3);
    }
    return (a0 + a1) + (a2 + a3);
}

// Pair-permuted chunk-transposed bf16 activation layout.  A vector of
// n = 32*nch values is stored as nch chunks of 32; chunk c holds 4 words x 4
// pairs; pair (i, k) of chunk c is the 32-bit element (i*nch + c)*4 + k and
// holds (v[32c+8i+k], v[32c+8i+k+4]).  A warp whose lane L reads chunk L for
// fixed i loads 512 contiguous bytes.  Returns the bf16 element index of v[j].
__device__ __forceinline__ int ppos(int j, int nch) {
    const int c = j >> 5, rem = j & 31, i = rem >> 3, r8 = rem & 7;
    return ((((i * nch + c) << 2) + (r8 & 3)) << 1) + (r8 >> 2);
}

// The 16 pairs of chunk c (read-only cached loads).
__device__ __forceinline__ void load_pairs(const uint16_t *vT, int nch, int c, uint32_t (&xp)[16]) {
    const uint4 *p = reinterpret_cast<const uint4 *>(vT);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = __ldg(p + (size_t)i * nch + c);
        xp[4 * i + 0] = v.x;
        xp[4 * i + 1] = v.y;
        xp[4 * i + 2] = v.z;
        xp[4 * i + 3] = v.w;
    }
}

// As load_pairs, through a generic pointer (shared or global memory).
__device__ __forceinline__ void load_pairs_any(const uint16_t *vT, int nch, int c,
                                               uint32_t (&xp)[16]) {
    const uint4 *p = reinterpret_cast<const uint4 *>(vT);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = p[(size_t)i * nch + c];
        xp[4 * i + 0] = v.x;
        xp[4 * i + 1] = v.y;
        xp[4 * i + 2] = v.z;
        xp[4 * i + 3] = v.w;
    }
}

// Sum of the 32 bf16 values of a chunk, in fp32.
__device__ __forceinline__ float pair_sum(const uint32_t (&xp)[16]) {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        s0 += __uint_as_float(xp[i] << 16);
        s1 += __uint_as_float(xp[i] & 0xFFFF0000u);
    }
    return s0 + s1;
}

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// ---------------------------------------------------------------------------
// Integer inner loop (dp2a).  x is quantised per 32-value chunk to int16 with
// scale sx = max|x| / 32767 (round to nearest; the error is below 2^-16 of
// the chunk's largest value, far inside the 1e-3 parity bar), and stored as
// 16 words per chunk whose int16 pairs line up with the nibbles that two
// masks pull out of a weight word:
//   lo = w & 0x0F0F0F0F holds nibbles (0, 2, 4, 6) in its four bytes,
//   hi = (w >> 4) & 0x0F0F0F0F holds nibbles (1, 3, 5, 7),
// and dp2a.lo / dp2a.hi multiply bytes (0, 1) / (2, 3) of b with the two
// int16 halves of a and add to an int32.  Word (i, k) of chunk c (i = weight
// word of the chunk, k = 0..3) holds the x pair
//   k=0: (x[8i], x[8i+2])  k=1: (x[8i+4], x[8i+6])
//   k=2: (x[8i+1], x[8i+3])  k=3: (x[8i+5], x[8i+7])
// at element ((i*nch + c)*4 + k), so a lane reading chunk c for fixed i loads
// 16 contiguous bytes (load_pairs_any).  Per chunk Q = sum q_j * x16_j is
// exact (|Q| < 2^24), and the row accumulates s*sx*Q + b*X with X the exact
// fp32 sum of the chunk's x.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Q = sum_j q_j * x16_j over one 16-byte weight chunk.  The odd nibbles stay
// in the high half of each byte (one AND, no shift: 16 * q), summed in their
// own chain and scaled down once at the end -- exact, since that chain is a
// multiple of 16 and |chain| <= 16 * 240 * 32767 < 2^31.
__device__ __forceinline__ int dot_chunk_i16(const uint4 w, const uint32_t (&xq)[16]) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    int a0 = 0, a1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = ws[i] & 0x0F0F0F0Fu, hi = ws[i] & 0xF0F0F0F0u;
        a0 = dp2a_lo(xq[4 * i + 0], lo, a0);
        a0 = dp2a_hi(xq[4 * i + 1], lo, a0);
        a1 = dp2a_lo(xq[4 * i + 2], hi, a1);
        a1 = dp2a_hi(xq[4 * i + 3], hi, a1);
    }
    return a0 + (a1 >> 4);
}

// The chunk's nibble planes, for reuse by several token vectors: lo[i] holds
// nibbles 0,2,4,6 of word i as bytes; hi[i] nibbles 1,3,5,7 left in the high
// half of each byte (16*q: one AND instead of a shift and an AND).
__device__ __forceinline__ void split_nibbles(const uint4 w, uint32_t (&lo)[4], uint32_t (&hi)[4]) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo[i] = ws[i] & 0x0F0F0F0Fu;
        hi[i] = ws[i] & 0xF0F0F0F0u;
    }
}

// dot_chunk_i16 on split planes: the low nibbles and the high ones (times
// 16) in two chains; Q = lo + hi/16, exact (hi is a multiple of 16 and
// |hi| <= 16 * 16 * 15 * 32767 < 2^31).
__device__ __forceinline__ int dot_split_i16(const uint32_t (&lo)[4], const uint32_t (&hi)[4],
                                             const uint32_t (&xq)[16]) {
    int a0 = 0, a1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        a0 = dp2a_lo(xq[4 * i + 0], lo[i], a0);
        a0 = dp2a_hi(xq[4 * i + 1], lo[i], a0);
        a1 = dp2a_lo(xq[4 * i + 2], hi[i], a1);
        a1 = dp2a_hi(xq[4 * i + 3], hi[i], a1);
    }
    return a0 + (a1 >> 4);
}

// Quantise one 32-value chunk (v) into its 16 words (strided by nch*4 words
// per i), returning the scale; *sum receives the exact fp32 sum.
__device__ __forceinline__ float quant_chunk_i16(const float (&v)[32], uint32_t *xq, int nch, int c,
                                                 float *sum) {
    float m = 0.f, s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        m = fmaxf(m, fmaxf(fabsf(v[j]), fabsf(v[j + 1])));
        s0 += v[j];
        s1 += v[j + 1];
    }
    *sum = s0 + s1;
    const float inv = m > 0.f ? 32767.0f / m : 0.f;
    auto q = [&](float f) { return (uint32_t)(__float2int_rn(f * inv) & 0xFFFF); };
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float *x = v + 8 * i;
        uint32_t *o = xq + (((size_t)i * nch + c) << 2);
        o[0] = q(x[0]) | (q(x[2]) << 16);
        o[1] = q(x[4]) | (q(x[6]) << 16);
        o[2] = q(x[1]) | (q(x[3]) << 16);
        o[3] = q(x[5]) | (q(x[7]) << 16);
    }
    return m * (1.0f / 32767.0f);
}

// Load 32 consecutive activations (f32 or bf16) of x as f32.
__device__ __forceinline__ void load_x32_any(const void *x, int is_bf16, size_t at, float (&v)[32]) {
    if (is_bf16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + at);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 r = __ldg(p + i);
            const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[8 * i + 2 * j] = __uint_as_float(rr[j] << 16);
                v[8 * i + 2 * j + 1] = __uint_as_float(rr[j] & 0xFFFF0000u);
            }
        }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(x) + at);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // a plain (weak, L1-cached) load: x may come from peers during the
            // launch, which the caller orders before this load by an acquire
            // and a barrier (the non-coherent __ldg path would not be covered);
            // L1 merges the chunk's 8 loads into one line fill (__ldcg made 8
            // L2 requests per line, from every SM at once)
            const float4 r = p[i];
            v[4 * i] = r.x;
            v[4 * i + 1] = r.y;
            v[4 * i + 2] = r.z;
            v[4 * i + 3] = r.w;
        }
    }
}

// Balanced contiguous split of `total` items over `parts`: [begin, end) of part p.
__device__ __forceinline__ void split_range(long long total, int parts, int p, long long &b,
                                            long long &e) {
    b = total * p / parts;
    e = total * (p + 1) / parts;
}

}  // namespace m1
