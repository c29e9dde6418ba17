// tc.cuh — tcgen05 / TMEM helpers (sm_100a) for the tensor-core kernels.
//
// Shared-memory operand descriptors and instruction descriptors follow the
// sm_100 UMMA formats; the operand tiles used here are K-major with the
// 128-byte swizzle: atoms of 8 rows x 128 bytes (1024-byte aligned), the
// 16-byte granule g of row r stored at granule g ^ (r % 8).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace leap {
namespace tc {

// 64-bit shared-memory matrix descriptor, K-major, SWIZZLE_128B.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major: 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 49-51 base offset (0: atoms 1024-byte aligned)
//   bits 61-63 layout (2 = 128-byte swizzle)
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_byte_addr) {
    uint64_t d = 0;
    d |= uint64_t((smem_byte_addr >> 4) & 0x3FFFu);
    d |= uint64_t(1u) << 16;
    d |= uint64_t((1024u >> 4) & 0x3FFFu) << 32;
    d |= uint64_t(1u) << 46;
    d |= uint64_t(2u) << 61;
    return d;
}

// The start-address field is the low 14 bits and every shared-memory
// address is below 256 KB, so desc(addr + off) == desc(addr) + (off >> 4):
// descriptors of one tile are a base plus compile-time constants.

// One lane of a converged warp (elect.sync): the MMA issuer.  Issuing from
// a warp-uniform branch with descriptors precomputed keeps the issue cost
// per tcgen05.mma near the tensor core's own time even for small N.
__device__ __forceinline__ bool elect_one_sync() {
    uint32_t p = 0;
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}"
        : "=r"(p));
    return p != 0;
}

// 32-bit instruction descriptor for kind::tf32, F32 accumulate, both
// operands K-major, dense.
//   bits 4-5 D format (1 = F32); 7-9 A format, 10-12 B format (2 = TF32);
//   15/16 A/B major (0 = K); 17-22 N >> 3; 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] . B[smem desc]^T
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem desc]^T
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
        :
        : "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Allocate `ncols` TMEM columns (warp-wide); the base address is written
// to *dst_smem.
__device__ __forceinline__ void alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Thread i of the warp reads 32 consecutive 32-bit columns of TMEM lane
// (warp's lane base + i), starting at column `taddr & 0xffff`.
__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// Thread i of the warp writes 16 consecutive 32-bit columns of TMEM lane
// (warp's lane base + i), starting at column `taddr & 0xffff`.
__device__ __forceinline__ void st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}

// 32-bit instruction descriptor for kind::f16 with BF16 A and B (format 1),
// F32 accumulate, both K-major, dense (the layout of idesc_tf32).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] . B[smem desc]^T, BF16 operands (K = 16 per product;
// A in TMEM holds two BF16 values of consecutive k per 32-bit column).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        :
        : "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Two floats rounded to BF16 (nearest even) in one 32-bit word: `a` in the
// low half (the lower k), `b` in the high half.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Byte offset of 16-bit element (row, k) in a K-major SW128 operand made of
// 64-element K chunks of `rows` rows each (chunk = rows*128 bytes).
__device__ __forceinline__ uint32_t sw128_offset_b16(int row, int k, int rows) {
    const int chunk = k >> 6;
    const int gran = (k & 63) >> 3;
    return uint32_t(chunk * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 +
                    ((gran ^ (row & 7)) << 4) + ((k & 7) << 1));
}

// TF32 split: hi keeps the top 10 explicit mantissa bits (the rest cleared),
// lo = x - hi exactly.  hi*hi + hi*lo + lo*hi reproduces an FP32 product to
// about 2^-21 relative (3xTF32).
__device__ __forceinline__ float tf32_hi(float x) {
    return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Byte offset of element (row, k) in a K-major SW128 operand made of
// 32-element K chunks of `rows` rows each (chunk = rows*128 bytes).
__device__ __forceinline__ uint32_t sw128_offset(int row, int k, int rows) {
    const int chunk = k >> 5;
    const int gran = (k & 31) >> 2;
    return uint32_t(chunk * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 +
                    ((gran ^ (row & 7)) << 4) + ((k & 3) << 2));
}

}  // namespace tc
}  // namespace leap
