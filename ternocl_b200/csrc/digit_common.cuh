// Integer-MMA pieces shared by the int2 GEMVs on int8 weights and fixed-point activation
// digits (gemv_i2d.cu, moe_decode.cu):
//
//  * weights: the 2-bit code of row j of a packed word sits in bits 2j..2j+1 of its byte,
//    so (x << (6 - 2j)) & 0xC0C0C0C0 ("class j") leaves the codes of rows j, j+4, j+8, j+12
//    in the top bits of the four bytes, which read as int8 are 64 * code_to_value(code)
//    (int2_fp16_upcvt/main.cpp:76);
//  * activations: with 2^e chosen so that |A| * 2^e < 2^22, fma(A, 2^e, 1.5 * 2^23) leaves
//    i + 2^22 (i = round(A * 2^e)) in the low 23 bits; its three bytes are unsigned digit
//    planes, and a plane of ones gives sum W, so sum W*i = d0 + 256 d1 + 65536 d2 - 2^22 ones;
//  * mma.sync m16n8k32 s8 x u8 -> s32 with the accumulator started at the bit pattern of
//    1.5 * 2^23, so that an exact dot |d| < 2^22 reads back as the float 1.5 * 2^23 + d.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ternocl {
namespace digit {

constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

// class j of a packed int2 word: int8 weights of rows j, j+4, j+8, j+12
__device__ __forceinline__ uint32_t cls(uint32_t x, int j) {
    return j == 3 ? (x & 0xC0C0C0C0u) : ((x << (6 - 2 * j)) & 0xC0C0C0C0u);
}

__device__ __forceinline__ void imma(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// max |value| of 8 packed 16-bit values, as magnitude bits (fp16 and bf16 order like
// their values); per half-word maxima first (a plain 32-bit max would drop the low half)
__device__ __forceinline__ uint32_t absmax_bits(const uint32_t (&h2)[8]) {
    uint32_t mx = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) mx = __vmaxu2(mx, h2[k] & 0x7FFF7FFFu);
    return max(mx & 0xFFFFu, mx >> 16);
}

// fixed-point exponent e for a maximum |A| (as DT bits): |A| * 2^e < 2^22
template <class DT>
__device__ __forceinline__ int exponent_for(uint32_t mx_bits) {
    const float amax = DT::tof((uint16_t)mx_bits);
    int e = 0;
    if (amax > 0.0f) {
        int E;
        frexpf(amax, &E);  // amax = f * 2^E, f in [0.5, 1)
        e = min(max(22 - E, -126), 120);
    }
    return e;
}

// 2^-e / 64 (the weights are 64 x code); NaN when the maximum is Inf or NaN
template <class DT>
__device__ __forceinline__ float inverse_scale(uint32_t mx_bits, int e) {
    const bool bad = DT::kBF16 ? mx_bits >= 0x7F80u : mx_bits >= 0x7C00u;
    return bad ? __int_as_float(0x7FC00000) : __int_as_float((127 - e - 6) << 23);
}

// 16 activations of one word row (h2 = 8 packed pairs, rows in order) -> the three digit
// planes, each as 4 registers: register j = class j (rows j, j+4, j+8, j+12, byte i =
// row 4i + j), the MMA's K order within the word
template <class DT>
__device__ __forceinline__ void word_digits(const uint32_t (&h2)[8], int e, uint32_t (&d0)[4], uint32_t (&d1)[4],
                                            uint32_t (&d2)[4]) {
    const float up = __int_as_float((127 + e) << 23);  // 2^e
    uint32_t x[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        x[2 * k] = __float_as_uint(fmaf(DT::tof((uint16_t)(h2[k] & 0xFFFFu)), up, kMagic));
        x[2 * k + 1] = __float_as_uint(fmaf(DT::tof((uint16_t)(h2[k] >> 16)), up, kMagic));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t p01 = __byte_perm(x[j], x[j + 4], 0x5140);
        const uint32_t p23 = __byte_perm(x[j + 8], x[j + 12], 0x5140);
        d0[j] = __byte_perm(p01, p23, 0x5410);
        d1[j] = __byte_perm(p01, p23, 0x7632);
        const uint32_t q01 = __byte_perm(x[j], x[j + 4], 0x7362);
        const uint32_t q23 = __byte_perm(x[j + 8], x[j + 12], 0x7362);
        d2[j] = __byte_perm(q01, q23, 0x5410);
    }
}

}  // namespace digit
}  // namespace ternocl
