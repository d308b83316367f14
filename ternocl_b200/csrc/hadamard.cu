// Fused sign flip + blockwise normalised Walsh-Hadamard transform, replaces
// hadamard_fwht (hadamard/hadamard_fwht.cl:62-115):
//
//   y[r, b*HB + i] = DT( (H_HB (s (.) x[r, b*HB : (b+1)*HB]))[i] * (1/sqrt(HB)) )
//
// fp32 butterflies, DT rounding at the store only.  The radix-2 stages run in
// increasing stride order (h = 1, 2, 4, ..., HB/2), as in the reference kernel, and a
// stage is the exact pair (a + b, a - b), so every output is the same sequence of fp32
// operations and the results are bit-identical to it, whatever the grouping of stages.
//
// Here the stages are grouped four at a time: a thread holds 16 elements whose index
// differs in four bits and runs those four stages in registers; between groups the
// block goes through shared memory (fp32, one pad word per 16 so that every access
// pattern below is free of bank conflicts or nearly so):
//   pass 1: bits 0-3   thread t holds i = 16t + j                (loaded from global)
//   pass 2: bits 4-7   thread t holds i = (t & 15) + 16j + 256(t >> 4)
//   pass 3: bits 8..L-1 (HB > 256) thread t holds 16 / 2^r groups of 2^r elements,
//           i = (t 2^(4-r) + jg) + 256 jr,  r = L - 8
// then the block is read back as i = 16t + j, scaled, rounded and stored with 16-byte
// stores.  A CTA of 256 threads holds 4096 elements: 4096 / HB blocks.
#include <cuda_runtime.h>

#include <cmath>

#include "common.cuh"
#include "hadamard_common.cuh"
#include "launch.h"

namespace ternocl {
namespace {

constexpr int kFwhtThreads = 256;
constexpr int kFwhtElems = kFwhtThreads * 16;

using fwht::pad16;
using fwht::wht16;

template <class DT, int L>
__global__ void __launch_bounds__(kFwhtThreads) fwht_kernel(const uint16_t *x,  // may alias y
                                                          const int8_t *__restrict__ signs, uint16_t *y,
                                                          int K, long long nblocks, int use_signs, float scale) {
    constexpr int HB = 1 << L;
    constexpr int TPB = HB / 16;  // threads per block
    constexpr int BPC = kFwhtThreads / TPB;
    __shared__ float sm[kFwhtElems + kFwhtElems / 16];
    const int t = threadIdx.x % TPB, b = threadIdx.x / TPB;
    const long long blk = (long long)blockIdx.x * BPC + b;
    const bool ok = blk < nblocks;
    const int bpr = K / HB;
    const size_t off = ok ? (size_t)(blk / bpr) * K + (size_t)(blk % bpr) * HB : 0;
    float *s = sm + b * (HB + HB / 16);

    pdl_wait();
    float v[16];
    if (ok) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + off + 16 * t);
        const uint4 lo = src[0], hi = src[1];
        const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[2 * j] = DT::tof((uint16_t)(w[j] & 0xffffu));
            v[2 * j + 1] = DT::tof((uint16_t)(w[j] >> 16));
        }
        if (use_signs) {
            const uint4 sv = *reinterpret_cast<const uint4 *>(signs + (size_t)(blk % bpr) * HB + 16 * t);
            const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] *= (float)(int8_t)((sw[j >> 2] >> (8 * (j & 3))) & 0xffu);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.0f;
    }
    wht16(v);  // h = 1 .. 8
#pragma unroll
    for (int j = 0; j < 16; ++j) s[pad16(16 * t + j)] = v[j];
    __syncthreads();
    const int i2 = (t & 15) + 256 * (t >> 4);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = s[pad16(i2 + 16 * j)];
    wht16(v);  // h = 16 .. 128
#pragma unroll
    for (int j = 0; j < 16; ++j) s[pad16(i2 + 16 * j)] = v[j];
    __syncthreads();
    if constexpr (L > 8) {
        constexpr int r = L - 8, R = 1 << r, NG = 16 / R;
#pragma unroll
        for (int jg = 0; jg < NG; ++jg) {
            const int lo = t * NG + jg;
            float u[R];
#pragma unroll
            for (int jr = 0; jr < R; ++jr) u[jr] = s[pad16(lo + 256 * jr)];
#pragma unroll
            for (int h = 1; h < R; h <<= 1)  // h * 256 = 256 .. HB/2
#pragma unroll
                for (int jr = 0; jr < R; ++jr)
                    if ((jr & h) == 0) {
                        const float a = u[jr], c = u[jr + h];
                        u[jr] = a + c;
                        u[jr + h] = a - c;
                    }
#pragma unroll
            for (int jr = 0; jr < R; ++jr) s[pad16(lo + 256 * jr)] = u[jr];
        }
        __syncthreads();
    }
    if (ok) {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t a = DT::fromf(s[pad16(16 * t + 2 * j)] * scale);
            const uint32_t c = DT::fromf(s[pad16(16 * t + 2 * j + 1)] * scale);
            w[j] = a | (c << 16);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(y + off + 16 * t);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
    pdl_launch_dependents();
}

template <class DT>
cudaError_t launch_dt(const void *x, const int8_t *signs, void *y, int rows, int K, int hb, int use_signs,
                      cudaStream_t st) {
    const long long nblocks = (long long)rows * (K / hb);
    const int bpc = kFwhtElems / hb;
    const dim3 grid((unsigned)((nblocks + bpc - 1) / bpc));
    const float scale = (float)(1.0 / std::sqrt((double)hb));  // hadamard_fwht.cl:17-31
    const uint16_t *xs = (const uint16_t *)x;
    uint16_t *ys = (uint16_t *)y;
    switch (hb) {
    case 256: return launch_kernel(fwht_kernel<DT, 8>, grid, dim3(kFwhtThreads), 0, st, xs, signs, ys, K, nblocks, use_signs, scale);
    case 512: return launch_kernel(fwht_kernel<DT, 9>, grid, dim3(kFwhtThreads), 0, st, xs, signs, ys, K, nblocks, use_signs, scale);
    case 1024: return launch_kernel(fwht_kernel<DT, 10>, grid, dim3(kFwhtThreads), 0, st, xs, signs, ys, K, nblocks, use_signs, scale);
    case 2048: return launch_kernel(fwht_kernel<DT, 11>, grid, dim3(kFwhtThreads), 0, st, xs, signs, ys, K, nblocks, use_signs, scale);
    default: return launch_kernel(fwht_kernel<DT, 12>, grid, dim3(kFwhtThreads), 0, st, xs, signs, ys, K, nblocks, use_signs, scale);
    }
}

}  // namespace

cudaError_t hadamard_launch(const void *x, const int8_t *signs, void *y, int rows, int K, int hb, int use_signs,
                            int dtype, cudaStream_t st) {
    if (dtype == TERNOCL_BF16) return launch_dt<BF16>(x, signs, y, rows, K, hb, use_signs, st);
    return launch_dt<F16>(x, signs, y, rows, K, hb, use_signs, st);
}

}  // namespace ternocl
