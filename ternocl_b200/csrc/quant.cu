// s8 x s2 support kernels:
//  * quant_a   -- replaces quant_a (int2_via_int2_x_int8_dpas/int2_int8_dpas.cl:103-123):
//      SA[g, m] = DT(127 / max(FLT_EPSILON, absmax of A[m, 128g .. 128g+127]))
//      Aq[m, k] = sat_int8(rint(A[m, k] * SA[g, m]))   (round to nearest even)
//    Host gold: compute_scale_a / compute_gold (int2_via_int2_x_int8_dpas/main.cpp:82-103).
//    The division is correctly rounded (the reference builds with
//    -cl-fp32-correctly-rounded-divide-sqrt) and A * SA is exact in fp32 (a product of
//    two 11- or 8-bit significands), so SA and Aq are bit-identical to the gold.
//  * group_dots -- int32 Dots[m, g, n] = sum_{k in g} Aq[m, k] * code(B[k, n]), the
//    exact integer partial sums of the s8 x s2 contraction, for verification.
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"

namespace ternocl {
namespace {

constexpr float kFltEpsilon = 1.1920928955078125e-07f;

// One warp per (row m, group g): lane l holds A[m, 128g + 4l .. 4l+3].  SCALE: compute
// SA[g, m] from the group's absmax and write it (quant_a); otherwise read the caller's SA
// and only quantise (the QMODE 1 scheme's in-GEMM quantisation, int2_int8_dpas.cl:128-160,
// run once per row block instead of once per column tile).
template <class DT, bool SCALE>
__global__ void __launch_bounds__(256) quant_a_kernel(const uint16_t *__restrict__ A, uint16_t *__restrict__ SA,
                                                     int8_t *__restrict__ Aq, int M, int K, int ldsa) {
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int G = K / kGS;
    if (warp >= M * G) return;
    const int m = warp / G, g = warp - m * G;
    const size_t off = (size_t)m * K + (size_t)g * kGS + 4 * lane;
    const uint2 raw = *reinterpret_cast<const uint2 *>(A + off);
    float a[4] = {DT::tof((uint16_t)(raw.x & 0xffffu)), DT::tof((uint16_t)(raw.x >> 16)),
                  DT::tof((uint16_t)(raw.y & 0xffffu)), DT::tof((uint16_t)(raw.y >> 16))};
    uint16_t sh;
    if (SCALE) {
        float mx = fmaxf(fmaxf(fabsf(a[0]), fabsf(a[1])), fmaxf(fabsf(a[2]), fabsf(a[3])));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // max(FLT_EPSILON, absmax), then the correctly rounded quotient, then RNE to DT
        sh = DT::fromf(__fdiv_rn(127.0f, fmaxf(mx, kFltEpsilon)));
        if (lane == 0) SA[(size_t)g * ldsa + m] = sh;
    } else {
        sh = SA[(size_t)g * ldsa + m];
    }
    if (Aq) {
        const float sa = DT::tof(sh);
        uint32_t packed = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int v = __float2int_rn(a[i] * sa);
            v = v < -128 ? -128 : (v > 127 ? 127 : v);
            packed |= ((uint32_t)v & 0xffu) << (8 * i);
        }
        *reinterpret_cast<uint32_t *>(Aq + off) = packed;
    }
    pdl_launch_dependents();
}

// One thread per (m, n, g); 2-bit two's complement codes (int2_fp16_upcvt/main.cpp:76).
__global__ void group_dots_kernel(const int8_t *__restrict__ Aq, const uint32_t *__restrict__ B,
                                  int32_t *__restrict__ D, int M, int N, int K) {
    const int G = K / kGS;
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)M * G * N) return;
    const int n = (int)(t % N);
    const int g = (int)((t / N) % G);
    const int m = (int)(t / ((long long)N * G));
    int32_t dot = 0;
    for (int w = 0; w < 8; ++w) {
        const uint32_t word = B[(size_t)(g * 8 + w) * N + n];
        for (int j = 0; j < 16; ++j) {
            const int code = (int)((word >> (2 * j)) & 3u);
            const int v = (code & 1) - (code & 2);
            dot += (int)Aq[(size_t)m * K + g * kGS + w * 16 + j] * v;
        }
    }
    D[((size_t)m * G + g) * N + n] = dot;
}

}  // namespace

cudaError_t quant_a_launch(const void *A, void *SA, int8_t *Aq, int M, int K, int dtype, cudaStream_t s) {
    const int warps = M * (K / kGS);
    dim3 grid((warps + 7) / 8);
    const int ldsa = (M + 31) & ~31;
    if (dtype == TERNOCL_BF16)
        return launch_kernel(quant_a_kernel<BF16, true>, grid, dim3(256), 0, s, (const uint16_t *)A, (uint16_t *)SA,
                             Aq, M, K, ldsa);
    return launch_kernel(quant_a_kernel<F16, true>, grid, dim3(256), 0, s, (const uint16_t *)A, (uint16_t *)SA, Aq,
                         M, K, ldsa);
}

cudaError_t quant_apply_launch(const void *A, const void *SA, int8_t *Aq, int M, int K, int dtype, cudaStream_t s) {
    const int warps = M * (K / kGS);
    dim3 grid((warps + 7) / 8);
    const int ldsa = (M + 31) & ~31;
    uint16_t *sa = (uint16_t *)const_cast<void *>(SA);  // read only (SCALE = false)
    if (dtype == TERNOCL_BF16)
        return launch_kernel(quant_a_kernel<BF16, false>, grid, dim3(256), 0, s, (const uint16_t *)A, sa, Aq, M, K,
                             ldsa);
    return launch_kernel(quant_a_kernel<F16, false>, grid, dim3(256), 0, s, (const uint16_t *)A, sa, Aq, M, K, ldsa);
}

cudaError_t group_dots_launch(const int8_t *Aq, const uint32_t *B, int32_t *D, int M, int N, int K,
                              cudaStream_t s) {
    const long long total = (long long)M * (K / kGS) * N;
    group_dots_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(Aq, B, D, M, N, K);
    return cudaGetLastError();
}

}  // namespace ternocl
