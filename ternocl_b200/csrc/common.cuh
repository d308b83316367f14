// Shared device code of the ternary GEMM/GEMV library: 16-bit dtype traits, the
// fused epilogues, the int2 -> fp16/bf16 register decode and the mma wrappers.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ternocl.h"

namespace ternocl {

constexpr int kGS = 128;  // scale group size along K (reference: kGS / GS = 128)

// ---------------------------------------------------------------------------------
// dtype traits.  DT is the activation / scale / output type: fp16 or bf16 (raw bits
// in memory, as the reference's `dt` = ushort).
struct F16 {
    using h2 = __half2;
    static constexpr bool kBF16 = false;
    __device__ static float tof(uint16_t h) { return __half2float(__ushort_as_half(h)); }
    // round to nearest even (the reference host cast (_Float16)f, common/dt16.hpp:38)
    __device__ static uint16_t fromf(float f) { return __half_as_ushort(__float2half_rn(f)); }
};
struct BF16 {
    using h2 = __nv_bfloat162;
    static constexpr bool kBF16 = true;
    __device__ static float tof(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
    // round to nearest even with NaN quieting, bit-identical to common/dt16.hpp:30-37
    __device__ static uint16_t fromf(float f) {
        uint32_t u = __float_as_uint(f);
        if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
        u += 0x7fffu + ((u >> 16) & 1u);
        return (uint16_t)(u >> 16);
    }
};

// ---------------------------------------------------------------------------------
// Fused epilogues on the fp32 accumulator (common/epilogue.clh:1-37, host gold
// common/epilogue.hpp:50-67):
//   0 none, 1 v*sigmoid(v)*other, 2 v+other, 3 v+bias[n], 4 sigmoid(v);
// sigmoid(x) = 0 for x <= -10 else 1/(exp(-x)+1)  (xetla_sigmoid).
__device__ __forceinline__ float sigmoid_x(float x) {
    // __expf (the hardware exp2 path, ~2 ulp) and __fdividef (the hardware reciprocal,
    // ~2 ulp; the denominator stays in [1, e^10 + 1]): within a few fp32 ulp of the
    // reference's 1/(exp(-x)+1), far inside the output tolerance
    return x <= -10.0f ? 0.0f : __fdividef(1.0f, __expf(-x) + 1.0f);
}

template <int POSTOP>
__device__ __forceinline__ float epi(float v, float e) {
    if constexpr (POSTOP == 1) return v * sigmoid_x(v) * e;
    else if constexpr (POSTOP == 2 || POSTOP == 3) return v + e;
    else if constexpr (POSTOP == 4) return sigmoid_x(v);
    else return v;
}

// Epilogue operand of element (m, n): Other[m, n] (DT) for POSTOP 1/2, Bias[n]
// (fp32 when OUT_F32 else DT) for POSTOP 3.
template <class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ float epi_in(const uint16_t *__restrict__ other,
                                        const void *__restrict__ bias, size_t i, int n) {
    if constexpr (POSTOP == 1 || POSTOP == 2) return DT::tof(other[i]);
    else if constexpr (POSTOP == 3) {
        if constexpr (OUT_F32) return reinterpret_cast<const float *>(bias)[n];
        else return DT::tof(reinterpret_cast<const uint16_t *>(bias)[n]);
    } else return 0.0f;
}

// Apply the epilogue to element (m, n) of C and store it (DT or fp32).
template <class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ void epi_store(void *__restrict__ C, const uint16_t *__restrict__ other,
                                          const void *__restrict__ bias, int N, int m, int n,
                                          float v) {
    const size_t i = (size_t)m * N + n;
    v = epi<POSTOP>(v, epi_in<DT, POSTOP, OUT_F32>(other, bias, i, n));
    if constexpr (OUT_F32) reinterpret_cast<float *>(C)[i] = v;
    else reinterpret_cast<uint16_t *>(C)[i] = DT::fromf(v);
}

// Two adjacent columns (n, n+1) of row m: one 32-bit (DT) or 64-bit (fp32) store.
template <class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ void epi_store2(void *__restrict__ C, const uint16_t *__restrict__ other,
                                           const void *__restrict__ bias, int N, int m, int n,
                                           float v0, float v1) {
    const size_t i = (size_t)m * N + n;
    if constexpr (POSTOP == 1 || POSTOP == 2) {
        const uint32_t o = *reinterpret_cast<const uint32_t *>(other + i);
        v0 = epi<POSTOP>(v0, DT::tof((uint16_t)(o & 0xffffu)));
        v1 = epi<POSTOP>(v1, DT::tof((uint16_t)(o >> 16)));
    } else if constexpr (POSTOP == 3) {
        v0 = epi<POSTOP>(v0, epi_in<DT, POSTOP, OUT_F32>(other, bias, i, n));
        v1 = epi<POSTOP>(v1, epi_in<DT, POSTOP, OUT_F32>(other, bias, i + 1, n + 1));
    } else {
        v0 = epi<POSTOP>(v0, 0.0f);
        v1 = epi<POSTOP>(v1, 0.0f);
    }
    if constexpr (OUT_F32) {
        *reinterpret_cast<float2 *>(reinterpret_cast<float *>(C) + i) = make_float2(v0, v1);
    } else {
        const uint32_t w = (uint32_t)DT::fromf(v0) | ((uint32_t)DT::fromf(v1) << 16);
        *reinterpret_cast<uint32_t *>(reinterpret_cast<uint16_t *>(C) + i) = w;
    }
}

// A warp's 32 x 32 block of results, lane = row (v: 32 consecutive columns of its row, as
// a TMEM lane holds them), stored along rows through the warp's shared tile t[32][33]
// (conflict-free both ways): lanes 0-15 and 16-31 store column pairs of two rows at a
// time, so a store instruction writes two contiguous row segments.  Rows from m_end on
// and columns from ncols on (ncols even) are skipped.  For POSTOP 1/2 the block's 16 Other
// pairs are loaded first (epi_load_rows32), all in flight together.
template <int POSTOP>
__device__ __forceinline__ void epi_load_rows32(uint32_t (&o)[16], const uint16_t *__restrict__ other, int N,
                                                int mrow, int m_end, int n, int ncols, int lane) {
    if constexpr (POSTOP == 1 || POSTOP == 2) {
        const int rsub = lane >> 4, c2 = 2 * (lane & 15);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int r = 2 * i + rsub;
            o[i] = (c2 < ncols && mrow + r < m_end)
                       ? *reinterpret_cast<const uint32_t *>(other + (size_t)(mrow + r) * N + n + c2)
                       : 0u;
        }
    }
}

template <class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ void epi_store_rows32(float *t, const float (&v)[32], const uint32_t (&o)[16],
                                                 void *__restrict__ C, const void *__restrict__ bias, int N, int mrow,
                                                 int m_end, int n, int ncols, int lane) {
#pragma unroll
    for (int j = 0; j < 32; ++j) t[lane * 33 + j] = v[j];
    __syncwarp();
    const int rsub = lane >> 4, c2 = 2 * (lane & 15);
    if (c2 < ncols) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int r = 2 * i + rsub;
            if (mrow + r < m_end) {
                float v0 = t[r * 33 + c2], v1 = t[r * 33 + c2 + 1];
                const size_t idx = (size_t)(mrow + r) * N + n + c2;
                if constexpr (POSTOP == 1 || POSTOP == 2) {
                    v0 = epi<POSTOP>(v0, DT::tof((uint16_t)(o[i] & 0xffffu)));
                    v1 = epi<POSTOP>(v1, DT::tof((uint16_t)(o[i] >> 16)));
                } else if constexpr (POSTOP == 3) {
                    v0 = epi<POSTOP>(v0, epi_in<DT, POSTOP, OUT_F32>(nullptr, bias, idx, n + c2));
                    v1 = epi<POSTOP>(v1, epi_in<DT, POSTOP, OUT_F32>(nullptr, bias, idx + 1, n + c2 + 1));
                } else {
                    v0 = epi<POSTOP>(v0, 0.0f);
                    v1 = epi<POSTOP>(v1, 0.0f);
                }
                if constexpr (OUT_F32) *reinterpret_cast<float2 *>(reinterpret_cast<float *>(C) + idx) = make_float2(v0, v1);
                else *reinterpret_cast<uint32_t *>(reinterpret_cast<uint16_t *>(C) + idx) =
                    (uint32_t)DT::fromf(v0) | ((uint32_t)DT::fromf(v1) << 16);
            }
        }
    }
    __syncwarp();
}

// The 16 Other pairs of a 32 x 32 block from a shared copy os[32 rows][32 columns] (DT)
__device__ __forceinline__ void epi_load_rows32_smem(uint32_t (&o)[16], const uint16_t *os, int lane) {
    const int rsub = lane >> 4, c2 = 2 * (lane & 15);
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = *reinterpret_cast<const uint32_t *>(os + (2 * i + rsub) * 32 + c2);
}

// both steps at once
template <class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ void epi_store_rows32(float *t, const float (&v)[32], void *__restrict__ C,
                                                 const uint16_t *__restrict__ other, const void *__restrict__ bias,
                                                 int N, int mrow, int m_end, int n, int ncols, int lane) {
    uint32_t o[16];
    epi_load_rows32<POSTOP>(o, other, N, mrow, m_end, n, ncols, lane);
    epi_store_rows32<DT, POSTOP, OUT_F32>(t, v, o, C, bias, N, mrow, m_end, n, ncols, lane);
}
constexpr int kEpiTileBytes = 32 * 33 * 4;

// ---------------------------------------------------------------------------------
// int2 weight decode in registers.
//
// A packed word holds 16 codes of one column (code of row 16kp+j at bits 2j..2j+1;
// int2_fp16_upcvt.cl:6-9).  Codes {0,1,3} mean {0,+1,-1}; bit 0 = non-zero, bit 1 =
// sign.  decode_pair(x, p) returns the f16x2 / bf16x2 register (lo, hi) = (value of
// row j, value of row j+8) for pair p = j in 0..7 -- the two codes that sit at the
// same bit offset of the word's two halves, so one LOP3 serves both halves.
//
// Magic-number decode: with c = (~nz, sign) copied into the mantissa at the bits
// where one ulp of the constant M = 2^(mantissa_bits - 2j') is 1, the register
// reads M + d with d = (c ^ 1) in {1, 0, 2} for codes {0, 1, 3}; the weight is
// (M + 1) - (M + d) = 1 - d in {0, +1, -1}, exactly.  Per register: one LOP3
// ((x & both_bits) ^ (nz_bit | M)) and one HSUB2.  fp16 has 10 mantissa bits, so
// pairs 0..4 decode in place and 5..7 after one shift by 10; bf16 has 7, so pairs
// 0..2 in place, 3..5 after >>6 and 6..7 after >>12.  Code 2 (never produced by the
// packers) decodes to -2, as the reference host gold's code_to_value.
template <class DT>
struct Int2Decode;

template <>
struct Int2Decode<F16> {
    // fp16 magic for in-half position j' (bits 2j'..2j'+1): 2^(10-2j')
    __device__ __forceinline__ static uint32_t magic(int jp) { return (uint32_t)(25 - 2 * jp) << 10; }
    __device__ __forceinline__ static __half2 pair(uint32_t x, int jp) {
        const uint32_t both = (3u << (2 * jp)) * 0x00010001u;
        // M + 1 in both halves (M + one ulp at bit 2j'); also the LOP3 constant
        const uint32_t k1 = (magic(jp) | (1u << (2 * jp))) * 0x00010001u;
        const uint32_t r = (x & both) ^ k1;
        return __hsub2(*reinterpret_cast<const __half2 *>(&k1), *reinterpret_cast<const __half2 *>(&r));
    }
    // all 8 pairs of a word: out[p] = (row p, row p+8)
    __device__ __forceinline__ static void word(uint32_t x, uint32_t out[8]) {
        const uint32_t y = x >> 10;
#pragma unroll
        for (int p = 0; p < 5; ++p) {
            __half2 v = pair(x, p);
            out[p] = *reinterpret_cast<uint32_t *>(&v);
        }
#pragma unroll
        for (int p = 5; p < 8; ++p) {
            __half2 v = pair(y, p - 5);
            out[p] = *reinterpret_cast<uint32_t *>(&v);
        }
    }
};

template <>
struct Int2Decode<BF16> {
    // bf16 magic for in-half position j' (bits 2j'..2j'+1): 2^(7-2j')
    __device__ __forceinline__ static uint32_t magic(int jp) { return (uint32_t)(134 - 2 * jp) << 7; }
    __device__ __forceinline__ static __nv_bfloat162 pair(uint32_t x, int jp) {
        const uint32_t both = (3u << (2 * jp)) * 0x00010001u;
        const uint32_t k1 = (magic(jp) | (1u << (2 * jp))) * 0x00010001u;
        const uint32_t r = (x & both) ^ k1;
        return __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&k1),
                       *reinterpret_cast<const __nv_bfloat162 *>(&r));
    }
    __device__ __forceinline__ static void word(uint32_t x, uint32_t out[8]) {
        const uint32_t y1 = x >> 6, y2 = x >> 12;
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            __nv_bfloat162 v = pair(x, p);
            out[p] = *reinterpret_cast<uint32_t *>(&v);
        }
#pragma unroll
        for (int p = 3; p < 6; ++p) {
            __nv_bfloat162 v = pair(y1, p - 3);
            out[p] = *reinterpret_cast<uint32_t *>(&v);
        }
#pragma unroll
        for (int p = 6; p < 8; ++p) {
            __nv_bfloat162 v = pair(y2, p - 6);
            out[p] = *reinterpret_cast<uint32_t *>(&v);
        }
    }
};

// ---------------------------------------------------------------------------------
// Warp-level tensor-core MMA m16n8k16, fp32 accumulate in place (A row-major 16x16,
// B column-major 16x8).  Used by the decode GEMVs, whose operands are built in
// registers (the weights are the 16-row operand, activation rows the 8 columns).
template <class DT>
__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    if constexpr (DT::kBF16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    }
}

// Streaming 128-bit global load that does not allocate in L1 (weights are read
// exactly once).
__device__ __forceinline__ uint4 ldg_stream128(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream64(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue (weight prefetch) while this one drains; wait for the previous kernel's
// results before reading activations.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

}  // namespace ternocl
