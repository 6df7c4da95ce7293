// Device helpers shared by the quantized GEMV kernels (gemv_quant.cu,
// gemv_tma.cu): code-to-f16 conversion without multiplies, the mma.sync
// m16n8k16 wrapper, and the permuted activation layout in shared memory.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace slc {
namespace k {

template <int FMT>
struct Fmt;
template <>
struct Fmt<0> {  // INT4: 32 codes per 16-byte lane chunk, 128 k per warp-step
    static constexpr int kStep = 128;
};
template <>
struct Fmt<1> {  // INT8: 16 codes per chunk, 64 k per warp-step
    static constexpr int kStep = 64;
};

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;  // (a & b) ^ c
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Four f16x2 pairs (nibble i, nibble i + 4), i = 0..3, of a word of eight
// two's-complement INT4 codes, as exact f16 integers. Even pairs: the nibble
// under the mantissa of 1024 with its sign bit flipped gives 1032 + c, minus
// 1032. Odd pairs are masked in place (bits 4..7): 1152 + 16 c, times 1/16
// minus 72. Every step is exact in f16.
__device__ __forceinline__ void int4_pairs(uint32_t w, uint32_t (&p)[4]) {
    const uint32_t w8 = w >> 8;
    p[0] = hsub2(lop3_and_xor(w, 0x000F000Fu, 0x64086408u), 0x64086408u);
    p[1] = hfma2(lop3_and_xor(w, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);
    p[2] = hsub2(lop3_and_xor(w8, 0x000F000Fu, 0x64086408u), 0x64086408u);
    p[3] = hfma2(lop3_and_xor(w8, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(const void *p) {
    uint4 r;
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(a));
    return r;
}

__device__ __forceinline__ float ld_cg(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// Position of k (relative to the slice) inside the staged activation plane:
// a 16-byte unit index (swizzled for conflict-free 128-bit reads) and the
// f16 slot inside the unit (INT4 interleaves nibbles i and i+4).
template <int FMT>
__device__ __forceinline__ int stage_slot(int kr, int S, int col) {
    int unit = kr >> 3, e = kr & 7;
    if (FMT == 0) {
        unit ^= (unit >> 3) & 1;
        e = e < 4 ? 2 * e : 2 * (e - 4) + 1;
    }
    return (col * S + unit) * 8 + e;
}

}  // namespace k
}  // namespace slc
