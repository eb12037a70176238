// tiled_layout.cuh — the HBM expert table's layout and its load-time repack.
//
// The reference's expert block (ModelSpec.swift:36-52, extract_olmoe.py:20-38)
// is [gateW|gateS|gateB|upW|upS|upB|downW|downS|downB], each a full matrix in
// row-major order.  The decode kernel (moe_layer.cuh) wants different runs of
// bytes to be contiguous, because the bulk-copy engine pays a fixed cost per
// copy (about 0.2 us; copies below ~16 KB cannot keep up with HBM):
//
//   gate/up: a CTA computes a run of rows of gate AND up, so the table stores
//     pair-row r (r < I) as [gateW_r | gateS_r | gateB_r | upW_r | upS_r | upB_r]
//     with every S/B row padded to a multiple of 16 bytes (no padding for
//     group 64 and dims that are multiples of 512, e.g. OLMoE and Mixtral);
//   down: the same CTA then needs the down matrix's COLUMNS for its rows of
//     the activation (split-K), so the down weights are stored column-block
//     major: a column block is 8 columns = one packed uint32 per row of h.
//     Rows of h are cut into chunks of `rc`:
//       W:  uint32 [h/rc][I/8][rc]       word (ic, cb, r) = downW[ic*rc + r][cb]
//       SB: uint32 [h/rc][I/gs][rc]      word (ic, g, r)  = downS[i][g] | downB[i][g] << 16
//     so a run of column blocks of one row chunk is one contiguous copy, and so
//     is the run of groups that covers it.
//
// The stored bytes are the reference's bytes (bf16 scales and biases, packed
// nibbles), reordered once at load time.
#pragma once

#include <stdint.h>

namespace m1 {

struct TiledLayout {
    long long pr;        // gate/up pair-row bytes: 2 * (h/2 + 2*sbh)
    int sbh;             // one gate/up S (or B) row, padded to 16 bytes
    int rc;              // rows of h per down row chunk
    int ncbI, ngI;       // column blocks (I/8) and groups (I/gs) of the down matrix
    long long dn_w;      // offset of the down weight words: I * pr
    long long dn_sb;     // offset of the down scale/bias words
    long long block;     // expert block stride (multiple of 128)
};

__host__ __device__ inline long long round_up_ll(long long v, long long m) {
    return (v + m - 1) / m * m;
}

// Rows of h per down chunk: the largest of 512, 256, 128, 64 dividing h (h is
// a multiple of 64).  The decode kernel gives each 32 rows of a chunk to one
// warp, and all of a chunk's warps must be able to run at once (16 <= its 24
// consumer warps): a tile's stage is freed only when every one of them has
// read it.
__host__ __device__ inline int down_row_chunk(int h) {
    int rc = 512;
    while (rc > 64 && h % rc) rc >>= 1;
    return rc;
}

__host__ __device__ inline TiledLayout make_tiled_layout(int h, int I, int gs) {
    TiledLayout t;
    t.sbh = (int)round_up_ll((long long)(h / gs) * 2, 16);
    t.pr = 2LL * (h / 2 + 2LL * t.sbh);
    t.rc = down_row_chunk(h);
    t.ncbI = I / 8;
    t.ngI = I / gs;
    t.dn_w = (long long)I * t.pr;
    t.dn_sb = t.dn_w + (long long)h * (I / 2);
    t.block = round_up_ll(t.dn_sb + (long long)h * t.ngI * 4, 128);
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
// blocks (dst).  One CTA per (expert, gate/up pair-row) and per (expert, row
// of h) of the down matrix; the down rows scatter into the column-block-major
// words (a one-time load cost).
__global__ void k_repack_tiled(const uint8_t *__restrict__ src, long long src_block,
                               uint8_t *__restrict__ dst, TiledLayout tl, RefOffsets ro, int ne,
                               int h, int I, int gs) {
    const long long rows_per_e = (long long)I + h;
    const int sbh = (h / gs) * 2;
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
            const int i = r - I, ic = i / tl.rc, ri = i % tl.rc;
            const uint32_t *w = reinterpret_cast<const uint32_t *>(sb + ro.off[6]) + (size_t)i * tl.ncbI;
            const uint16_t *s = reinterpret_cast<const uint16_t *>(sb + ro.off[7]) + (size_t)i * tl.ngI;
            const uint16_t *b = reinterpret_cast<const uint16_t *>(sb + ro.off[8]) + (size_t)i * tl.ngI;
            uint32_t *dw = reinterpret_cast<uint32_t *>(db + tl.dn_w);
            uint32_t *dsb = reinterpret_cast<uint32_t *>(db + tl.dn_sb);
            for (int cb = threadIdx.x; cb < tl.ncbI; cb += blockDim.x)
                dw[((size_t)ic * tl.ncbI + cb) * tl.rc + ri] = w[cb];
            for (int g = threadIdx.x; g < tl.ngI; g += blockDim.x)
                dsb[((size_t)ic * tl.ngI + g) * tl.rc + ri] = (uint32_t)s[g] | ((uint32_t)b[g] << 16);
        }
    }
}

}  // namespace m1
