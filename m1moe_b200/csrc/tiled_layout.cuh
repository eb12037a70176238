// tiled_layout.cuh — the HBM expert table's layout and its load-time repack.
//
// The reference's expert block (ModelSpec.swift:36-52, extract_olmoe.py:20-38)
// is [gateW|gateS|gateB|upW|upS|upB|downW|downS|downB], each a full matrix.
// A decode tile needs a run of ROWS of all of W, S and B, which in that layout
// is three (or six) separate copies, and the bulk-copy engine pays a fixed
// cost per copy (about 0.2 us; copies below ~16 KB cannot keep up with HBM).
// The table therefore stores each expert once, reordered by row:
//
//   gate/up pair-row r (r < I):  [gateW_r | gateS_r | gateB_r | upW_r | upS_r | upB_r]
//   down row i (i < h):          [downW_i | downS_i | downB_i]
//
// with every S/B row padded to a multiple of 16 bytes (no padding for group 64
// and dims that are multiples of 512, e.g. OLMoE and Mixtral).  A run of rows is
// one contiguous copy.  The stored bytes are the reference's bytes.
#pragma once

#include <stdint.h>

namespace m1 {

struct TiledLayout {
    long long pr;        // gate/up pair-row bytes: 2 * (h/2 + 2*sbh)
    long long dr;        // down row bytes: I/2 + 2*sbi
    int sbh, sbi;        // one S (or B) row of gate/up resp. down, padded to 16 bytes
    long long down_off;  // I * pr
    long long block;     // expert block stride (multiple of 128)
};

__host__ __device__ inline long long round_up_ll(long long v, long long m) {
    return (v + m - 1) / m * m;
}

__host__ __device__ inline TiledLayout make_tiled_layout(int h, int I, int gs) {
    TiledLayout t;
    t.sbh = (int)round_up_ll((long long)(h / gs) * 2, 16);
    t.sbi = (int)round_up_ll((long long)(I / gs) * 2, 16);
    t.pr = 2LL * (h / 2 + 2LL * t.sbh);
    t.dr = (long long)I / 2 + 2LL * t.sbi;
    t.down_off = (long long)I * t.pr;
    t.block = round_up_ll(t.down_off + (long long)h * t.dr, 128);
    return t;
}

// Byte offsets of the nine arrays inside a reference expert block
// (InferenceEngine.swift:79-97).
struct RefOffsets {
    long long off[9];
};

__device__ __forceinline__ void copy16(uint8_t *d, const uint8_t *s, int bytes) {
    for (int k = threadIdx.x; k < bytes / 16; k += blockDim.x)
        reinterpret_cast<uint4 *>(d)[k] = reinterpret_cast<const uint4 *>(s)[k];
}

__device__ __forceinline__ void copy_sb(uint8_t *d, const uint8_t *s, int bytes, int padded) {
    for (int k = threadIdx.x; k < padded / 2; k += blockDim.x)
        reinterpret_cast<uint16_t *>(d)[k] =
            k < bytes / 2 ? reinterpret_cast<const uint16_t *>(s)[k] : (uint16_t)0;
}

// Reference-layout blocks (src, `ne` experts, src_block bytes apart) -> tiled
// blocks (dst).  One CTA per (expert, row).
__global__ void k_repack_tiled(const uint8_t *__restrict__ src, long long src_block,
                               uint8_t *__restrict__ dst, TiledLayout tl, RefOffsets ro, int ne,
                               int h, int I, int gs) {
    const long long rows_per_e = (long long)I + h;
    const int sbh = (h / gs) * 2, sbi = (I / gs) * 2;
    for (long long rid = blockIdx.x; rid < ne * rows_per_e; rid += gridDim.x) {
        const int e = (int)(rid / rows_per_e), r = (int)(rid % rows_per_e);
        const uint8_t *sb = src + (size_t)e * src_block;
        uint8_t *db = dst + (size_t)e * tl.block;
        if (r < I) {
            uint8_t *d = db + (size_t)r * tl.pr;
            const size_t half = (size_t)h / 2 + 2 * tl.sbh;
            for (int m = 0; m < 2; ++m) {  // gate, up
                const long long *o = ro.off + 3 * m;
                copy16(d + m * half, sb + o[0] + (size_t)r * (h / 2), h / 2);
                copy_sb(d + m * half + h / 2, sb + o[1] + (size_t)r * sbh, sbh, tl.sbh);
                copy_sb(d + m * half + h / 2 + tl.sbh, sb + o[2] + (size_t)r * sbh, sbh, tl.sbh);
            }
        } else {
            const int i = r - I;
            uint8_t *d = db + tl.down_off + (size_t)i * tl.dr;
            copy16(d, sb + ro.off[6] + (size_t)i * (I / 2), I / 2);
            copy_sb(d + I / 2, sb + ro.off[7] + (size_t)i * sbi, sbi, tl.sbi);
            copy_sb(d + I / 2 + tl.sbi, sb + ro.off[8] + (size_t)i * sbi, sbi, tl.sbi);
        }
    }
}

}  // namespace m1
