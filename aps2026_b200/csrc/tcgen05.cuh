// sm_100a tensor-core (tcgen05) primitives for the kernels of this library:
// tensor-memory allocation, shared-memory operand descriptors, the TF32 MMA
// with its accumulator in tensor memory, commits to an mbarrier, and
// tensor-memory loads / stores. Inline PTX; the encodings follow the PTX ISA
// descriptors for sm_100 (bit positions cross-checked against CUTLASS's
// cute/arch/mma_sm100_desc.hpp).
#pragma once

#include "common.cuh"

namespace b2 {
namespace tc {

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzle layout: rows of 128 bytes (32 fp32 / tf32 values of K), 8-row
// atoms of 1024 bytes stacked along M/N, the 16-byte chunks of row r stored at
// chunk ^ (r % 8). `p` is the first byte of the K slice the MMA reads (atom
// base + 32 bytes per 8-value k-step); atom bases are 1024-byte aligned.
__device__ __forceinline__ std::uint64_t sw128_desc(const void* p) {
    const std::uint32_t a = smem_addr(p);
    std::uint64_t d = static_cast<std::uint64_t>((a >> 4) & 0x3FFFu);  // start address, 16-byte units
    d |= static_cast<std::uint64_t>(1) << 16;                            // leading byte offset (unused: 1)
    d |= static_cast<std::uint64_t>(1024 >> 4) << 32;                    // stride byte offset: one 8-row atom
    d |= static_cast<std::uint64_t>(1) << 46;                            // descriptor version (sm_100)
    d |= static_cast<std::uint64_t>(2) << 61;                            // layout: 128-byte swizzle
    return d;
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `r` inside an
// 8-row-atom stack of the 128-byte swizzle layout.
__device__ __forceinline__ int sw128_offset(int r, int chunk) {
    return (r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4);
}

// Instruction descriptor of kind::tf32 with an fp32 accumulator, both
// operands K-major, M x N.
__host__ __device__ constexpr std::uint32_t tf32_idesc(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<std::uint32_t>(n >> 3) << 17) |
           (static_cast<std::uint32_t>(m >> 4) << 24);
}

// TF32 value of a finite x rounded to nearest, ties away from zero (what
// cvt.rna.tf32.f32 gives): half a TF32 unit (bit 12) added to the magnitude
// bits, the 13 bits below the TF32 mantissa cleared; a carry moves into the
// exponent as rounding up should. Integer operations, so the conversions of a
// 3 x TF32 split do not queue on the SM's conversion / transcendental unit
// beside expf. (NaN inputs may come out as infinities.)
__device__ __forceinline__ float tf32_round(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// One warp: allocate / free `cols` tensor-memory columns (a power of two >= 32).
__device__ __forceinline__ void tmem_alloc(std::uint32_t* dst_smem, std::uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
                 "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_free(std::uint32_t taddr, std::uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A . B^T, A from tensor memory (rows in lanes, K along
// columns), B a shared-memory descriptor; issued by one thread.
__device__ __forceinline__ void mma_tf32_ts(std::uint32_t d, std::uint32_t a, std::uint64_t b, std::uint32_t idesc,
                                            bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(static_cast<std::uint32_t>(accumulate)), "r"(0u)
        : "memory");
}

// Arrives on the mbarrier once every MMA this thread issued has completed.
__device__ __forceinline__ void commit(std::uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// The warp's 32 lanes (lane base 32 * (warp % 4)) x 32 columns from `taddr`:
// thread t gets its lane's 32 consecutive 32-bit columns.
__device__ __forceinline__ void ld32(std::uint32_t taddr, float (&v)[32]) {
    std::uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void st32(std::uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
        "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
        "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
        "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16-column forms of ld32 / st32 (ld16 waits for its load).
__device__ __forceinline__ void ld16(std::uint32_t taddr, float (&v)[16]) {
    std::uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void st16(std::uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}

}  // namespace tc
}  // namespace b2
