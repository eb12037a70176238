// umma.cuh — the sm_100a tensor-core pieces of the prefill GEMM: tensor
// memory (TMEM) allocation, tcgen05.mma of kind::f16 (fp16 x fp16 -> fp32,
// both operands K-major in shared memory, 128B-swizzled), its commit to an
// mbarrier, TMEM -> register loads, and the 3-D tiled TMA load.
//
// Shared-memory operand layout (K-major, SWIZZLE_128B): a tile of R rows x
// 64 fp16 (128 bytes per row) is stored in 8-row atoms of 1024 bytes; row r
// lives at (r/8)*1024 + (r%8)*128 and its 16-byte chunk c at chunk (c ^ r%8).
// The matrix descriptor names the tile by its start address, the stride
// between 8-row atoms (SBO = 1024) and the swizzle mode; stepping along K
// by 16 elements (one MMA) adds 32 bytes to the start address.  Field
// positions follow the PTX ISA's tcgen05 shared-memory descriptor and
// instruction descriptor tables.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace m1 {

// ------------------------------------------------------------ descriptors ----
// Shared-memory matrix descriptor: start address >> 4 in bits 0-13, leading
// byte offset >> 4 in 16-29 (16 bytes; unused by swizzled K-major), stride
// byte offset >> 4 in 32-45, the descriptor version (1) in 46-47, base
// offset 0 (atoms 1024-byte aligned), layout type 2 (128-byte swizzle) in
// 61-63.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) |
           ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor for kind::f16: fp32 accumulator (bits 4-5 = 1),
// A and B fp16 (bits 7-9 = 0, 10-12 = 0: the same type for both), both
// K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------- TMEM ----
// One warp: allocate ncols columns (a power of two >= 32) of this SM's
// tensor memory; the address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Writes by this thread to shared memory become visible to the tensor cores
// (the async proxy) after this fence and a synchronisation.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------------------------------------------- MMA ----
// D[tmem] (+)= A[smem] . B[smem]^T, M x N x 16, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, bool accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// The mbarrier receives one arrival once every MMA issued so far by this
// thread has completed (its shared-memory operands may be reused).
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(bar))
                 : "memory");
}

// ------------------------------------------------------------ TMEM loads ----
// Warp w%4 of a warpgroup reads lanes 32*(w%4) .. +31: thread i gets 16
// consecutive 32-bit columns of lane (taddr lane + i), starting at the
// address's column.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// -------------------------------------------------------------------- TMA ----
// 3-D tiled load of the map's box at element coordinates (x, y, z) into this
// CTA's shared memory; completes the box's bytes on `bar`.  x * element size
// must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
        "r"((uint32_t)__cvta_generic_to_shared(bar))
        : "memory");
}

// ---------------------------------------------------------- fp16 helpers ----
// Swizzled byte offset of 16-byte chunk c (0..7) of row r in a K-major
// 128B-swizzled tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((c ^ (r & 7u)) << 4);
}

// Position, within its chunk of 8, of element k (0..7) of a nibble word in
// the tensor-core K order: the pair (k, k+4) is one half2, so a chunk holds
// k = 0, 4, 1, 5, 2, 6, 3, 7.
__host__ __device__ __forceinline__ int kperm_pos(int k) { return k < 4 ? 2 * k : 2 * (k - 4) + 1; }

// The 8 nibbles of w (nibble j = element j) as 8 fp16 values q*s + b in the
// tensor-core K order (4 half2 words): (w >> 4j) & 0x000F000F | 0x6400
// gives 1024 + q exactly for the pair (j, j+4); subtracting 1024 is exact,
// and the fma rounds once (fp16: 11 significant bits).  s2, b2: the group's
// scale and bias as fp16 in both halves.
__device__ __forceinline__ uint4 dequant_word_f16(uint32_t w, uint32_t s2, uint32_t b2) {
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t v = ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
        uint32_t q;
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(v), "r"(0x64006400u));
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[j]) : "r"(q), "r"(s2), "r"(b2));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// A bf16 value (low 16 bits) as an fp16 pair, rounded to nearest.
__device__ __forceinline__ uint32_t bf16_to_f16_pair(uint32_t b16) {
    const __half hv = __float2half_rn(__uint_as_float((b16 & 0xFFFFu) << 16));
    const uint32_t u = __half_as_ushort(hv);
    return u | (u << 16);
}

}  // namespace m1
