// Pieces of the block-scaled (kind::mxf8f6f4, UE8M0 scales per 32 values along K) tcgen05 kernels: the scale atom's
// shared-memory descriptor, its copy into TMEM, the block-scaled MMA and its instruction descriptor, and the untiled
// bulk copy the atoms arrive by.
//
// Scale atom (128 rows x 4 scales of one 128-wide k-block, 512 bytes): byte (r % 32) * 16 + (r / 32) * 4 + j holds
// row r's scale of K values [32 j, 32 j + 32). tcgen05.cp 32x128b.warpx4 copies its 32 rows of 16 bytes to 4 TMEM
// columns of every lane quarter; the MMA reads row r's scale word in lane r, column r / 32, and the byte named by the
// two top bits of the scale address (the idesc's scale-factor id).
#pragma once
#include <stdint.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace xt {

// Shared-memory descriptor of a scale atom as the source of tcgen05.cp 32x128b: K-major, no swizzle, 8-row core
// matrices of 16-byte rows, 128 bytes apart
XT_DEV uint64_t sf_atom_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFF);
    d |= uint64_t(128 >> 4) << 32;   // stride byte offset: the next 8 rows
    d |= uint64_t(1) << 46;          // version
    return d;                        // layout type 0: no swizzle
}

// Untiled bulk copy global -> shared, completing `bytes` on `bar` (both addresses 16-byte aligned, bytes % 16 == 0)
XT_DEV void mx_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

XT_DEV void sf_copy(uint32_t taddr, uint64_t desc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n" ::"r"(taddr), "l"(desc) : "memory");
}

XT_DEV void mma_mx(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                   uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
        : "memory");
}

constexpr uint32_t MX_FMT_E4M3 = 0, MX_FMT_E2M1 = 5;   // operand formats of kind::mxf8f6f4

// Instruction descriptor of kind::mxf8f6f4 block-scaled: E4M3 A (format 0), B of format b_fmt (E4M3 0, E2M1 5), both
// K-major, UE8M0 scales, M x N, scale bytes sf_id of A and B
__host__ __device__ constexpr uint32_t idesc_mx(int M, int N, uint32_t sf_id, uint32_t b_fmt) {
    return (sf_id << 4)                 // B scale factor id
           | (b_fmt << 10)              // B format
           | (uint32_t(N >> 3) << 17)   // N / 8
           | (1u << 23)                 // scale format E8M0
           | (uint32_t(M >> 4) << 24)   // M / 16
           | (sf_id << 29);             // A scale factor id
}

}  // namespace xt
