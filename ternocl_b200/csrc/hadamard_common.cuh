// Pieces of the blockwise Walsh-Hadamard transform shared by the standalone kernel
// (hadamard.cu) and the BITCOS GEMVs that transform their staged activations
// (gemv_bitcos.cu, gemv_bitcos_p.cu).  Every radix-2 stage is the exact fp32 pair (a + b, a - b) and the
// stages run in increasing stride order, as in hadamard_fwht (hadamard/hadamard_fwht.cl),
// so any grouping of the stages gives bit-identical results.
#pragma once
#include <cuda_runtime.h>

namespace ternocl {
namespace fwht {

// fp32 scratch index with one pad word per 16 (bank-conflict-free strided access)
__device__ __forceinline__ int pad16(int i) { return i + (i >> 4); }

// the four radix-2 stages over the bits of j, in increasing order
__device__ __forceinline__ void wht16(float v[16]) {
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if ((j & h) == 0) {
                const float a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
}

// Sign flip + FWHT, in place, of HB = 32 E-wide blocks of a CTA's staged activation rows
// [rows x krange] (16-byte unit u of a row at u ^ (((u >> 3) & 1) << 1); sgn = the range's
// signs, in shared or global memory, or null): warps warp, warp + nwarps, ... one block each, lane l holding elements E l .. E l + E - 1, the stages of stride
// 1 .. E/2 in registers and those of stride E .. HB/2 across lanes (__shfl_xor), every
// stage the fp32 pair (a + b, a - b), in increasing stride order as hadamard_fwht, then
// the scale and the DT rounding of the standalone kernel.
template <class DT, int E>
__device__ void staged_rows(char *act, int act_stride, const int8_t *sgn, int rows, int krange, float scale,
                            int warp, int nwarps, int lane) {
    constexpr int HB = 32 * E;
    const int nb = krange / HB, total = rows * nb;
    for (int blk = warp; blk < total; blk += nwarps) {
        const int m = blk / nb, k0 = (blk % nb) * HB + lane * E;  // within the range
        char *row = act + (size_t)m * act_stride;
        float v[E];
#pragma unroll
        for (int q = 0; q < E / 8; ++q) {
            const int u = k0 / 8 + q;
            const uint4 w4 = *reinterpret_cast<const uint4 *>(row + (size_t)(u ^ (((u >> 3) & 1) << 1)) * 16);
            const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                v[8 * q + 2 * j] = DT::tof((uint16_t)(w[j] & 0xffffu));
                v[8 * q + 2 * j + 1] = DT::tof((uint16_t)(w[j] >> 16));
            }
        }
        if (sgn) {
#pragma unroll
            for (int q = 0; q < E / 8; ++q) {  // 8 signs per 8-byte read
                const uint2 sv = *reinterpret_cast<const uint2 *>(sgn + k0 + 8 * q);
                const uint32_t sw[2] = {sv.x, sv.y};
#pragma unroll
                for (int j = 0; j < 8; ++j) v[8 * q + j] *= (float)(int8_t)((sw[j >> 2] >> (8 * (j & 3))) & 0xffu);
            }
        }
#pragma unroll
        for (int h = 1; h < E; h <<= 1)
#pragma unroll
            for (int j = 0; j < E; ++j)
                if ((j & h) == 0) {
                    const float a = v[j], b = v[j + h];
                    v[j] = a + b;
                    v[j + h] = a - b;
                }
#pragma unroll
        for (int c = 0; c < 5; ++c) {  // stride E << c: lane bit c
            const bool upper = (lane >> c) & 1;
#pragma unroll
            for (int j = 0; j < E; ++j) {
                const float o = __shfl_xor_sync(0xffffffffu, v[j], 1 << c);
                v[j] = upper ? o - v[j] : v[j] + o;
            }
        }
#pragma unroll
        for (int q = 0; q < E / 8; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[j] = (uint32_t)DT::fromf(v[8 * q + 2 * j] * scale) |
                       ((uint32_t)DT::fromf(v[8 * q + 2 * j + 1] * scale) << 16);
            const int u = k0 / 8 + q;
            *reinterpret_cast<uint4 *>(row + (size_t)(u ^ (((u >> 3) & 1) << 1)) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

}  // namespace fwht
}  // namespace ternocl
