// s8 x s2 decode GEMV (small M), replaces int2_int8_gemv
// (int2_via_int2_x_int8_dpas/int2_int8_dpas.cl:210-281):
//
//   C[m,n] = DT(epi( sum_g float(dot_g[m,n]) * (SB[g,n] * (1 / SA[g,m])) ))
//   dot_g[m,n] = sum_{k in g} q[m,k] * code(B[k,n])      (exact int32)
//   q[m,k] = Aq[m,k] (qmode 0) or sat_int8(rint(A[m,k] * SA[g,m])) (qmode 1)
//
// Host gold: int2_via_int2_x_int8_dpas/main.cpp:94-121 (1/SA is the IEEE quotient,
// as in the gold; the reference kernel uses native_recip).
//
// Same skeleton as the int2 upconvert GEMV (gemv_common.cuh): per 128-row group each
// thread streams the words of rows kp = 8g + 4r + q, columns n0+4g .. n0+4g+3.  A word
// becomes 4 registers of int8 weights with 2-bit sign extension in 3-4 integer ops:
// register j holds rows {j, j+4, j+8, j+12} (byte i = row 4i+j):
//     t = (x >> 2j) & 0x03030303;  r = t + (t & 0x02020202) * 0x7E
// (per byte b - 4*bit1: codes {0,1,2,3} -> {0,1,-2,-1}, the 2-bit two's complement
// of code_to_value, int2_via_int2_x_int8_dpas/main.cpp:77).  They feed
// mma.sync m16n8k32 s8 x s8 -> s32, one int32 accumulator per 128-row group, so the
// dots are exact; the int8 activations are staged per CTA in the same permuted K
// order (a 4x4 byte transpose per 16-row word), quantised from A when qmode == 1.
#include <cuda_runtime.h>

#include "gemv_common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

__device__ __forceinline__ void mma_s8(int d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// int8 weights of a word: out[j] = rows {j, j+4, j+8, j+12}
__device__ __forceinline__ void s8_word(uint32_t x, uint32_t out[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t t = (x >> (2 * j)) & 0x03030303u;
        out[j] = t + (t & 0x02020202u) * 0x7Eu;
    }
}

// 4x4 byte transpose: out[j] byte i = in[i] byte j
__device__ __forceinline__ void transpose4x4(const uint32_t in[4], uint32_t out[4]) {
    const uint32_t t0 = __byte_perm(in[0], in[1], 0x5140), t1 = __byte_perm(in[0], in[1], 0x7362);
    const uint32_t t2 = __byte_perm(in[2], in[3], 0x5140), t3 = __byte_perm(in[2], in[3], 0x7362);
    // t0 = (i0b0, i1b0, i0b1, i1b1), t1 = (i0b2, i1b2, i0b3, i1b3) and likewise t2, t3
    out[0] = __byte_perm(t0, t2, 0x5410);
    out[1] = __byte_perm(t0, t2, 0x7632);
    out[2] = __byte_perm(t1, t3, 0x5410);
    out[3] = __byte_perm(t1, t3, 0x7632);
}

struct Int8Policy {
    static constexpr int kWords16 = 2;
    static constexpr int kWordRegs = kWords16;
    static constexpr bool kSharedSlots = false;
    __device__ static void read_words(const char *stage, int tid, int nthreads, uint4 *w) {
#pragma unroll
        for (int c = 0; c < kWords16; ++c) w[c] = reinterpret_cast<const uint4 *>(stage)[c * nthreads + tid];
    }
    static constexpr bool kContiguousCols = true;
    static constexpr int kActGroupBytes = 8 * 16;   // 8 words x 16 int8
    static constexpr int kExtraGroupBytes = 8 * 4;  // 1/SA of 8 activation rows
    __device__ static int thread_col0(int g) { return 4 * g; }
    __device__ static bool copy_ok(int N, int n0, int g) { return n0 + 4 * g < N; }
    __device__ static int thread_col(int g, int i) { return 4 * g + i; }
    __device__ static const uint32_t *word_ptr(const gemv::Params &p, int grp, int g, int q, int n0) {
        return p.B + (size_t)(grp * 8 + q) * p.N + n0 + 4 * g;
    }
    __device__ static size_t group_stride(const gemv::Params &p) { return (size_t)8 * p.N; }
    __device__ static size_t chunk_stride(const gemv::Params &p) { return (size_t)4 * p.N; }
    __host__ __device__ static size_t extra_smem(int, int krange) { return (size_t)(krange / kGS) * kExtraGroupBytes; }
    static constexpr int kActBytesPerK = 1;  // int8 activations
    static constexpr int kActPadBytes = 64;  // row stride = 64 mod 128: 16-byte reads conflict-free

    template <class DT>
    __device__ static void stage(const gemv::Params &p, char *act, int stride, char *extra, int mb, int rows,
                                 int cg0, int ng) {
        const int nw = ng * 8;
        for (int it = threadIdx.x; it < rows * nw; it += blockDim.x) {
            const int m = it / nw, w = it - m * nw;
            const int grp = cg0 + w / 8;
            const size_t k0 = (size_t)(cg0 * 8 + w) * 16;
            uint32_t in[4];
            if (p.qmode == 0) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p.Aq + (size_t)(mb + m) * p.K + k0));
                in[0] = v.x; in[1] = v.y; in[2] = v.z; in[3] = v.w;
            } else {
                const float sa = DT::tof(p.SA[(size_t)grp * p.ldsa + mb + m]);
                const uint16_t *src = p.A + (size_t)(mb + m) * p.K + k0;
                const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(src));
                const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(src + 8));
                const uint32_t h[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint32_t packed = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const uint32_t hw = h[(4 * i + b) >> 1];
                        const uint16_t raw = (uint16_t)(((4 * i + b) & 1) ? (hw >> 16) : (hw & 0xffffu));
                        int v = __float2int_rn(DT::tof(raw) * sa);
                        v = v < -128 ? -128 : (v > 127 ? 127 : v);
                        packed |= ((uint32_t)v & 0xffu) << (8 * b);
                    }
                    in[i] = packed;
                }
            }
            uint32_t o[4];
            transpose4x4(in, o);
            *reinterpret_cast<uint4 *>(act + (size_t)m * stride + (size_t)w * 16) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        float *inv = reinterpret_cast<float *>(extra);
        for (int it = threadIdx.x; it < ng * 8; it += blockDim.x) {
            const int g = it >> 3, m = it & 7;
            float v = 0.0f;
            if (m < rows) {
                const float sa = DT::tof(p.SA[(size_t)(cg0 + g) * p.ldsa + mb + m]);
                v = sa == 0.0f ? 0.0f : __frcp_rn(sa);  // the gold's IEEE 1 / sa
            }
            inv[g * 8 + m] = v;
        }
    }

    template <class DT>
    __device__ static void compute(const uint4 w[2], uint2 sc, const char *arow, bool rowok, int q,
                                   const char *xg, float acc[2][4], int) {
        int part[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            uint32_t b[4] = {0u, 0u, 0u, 0u};
            if (rowok) {
                const uint4 v = *reinterpret_cast<const uint4 *>(arow + (4 * r + q) * 16);
                b[0] = v.x; b[1] = v.y; b[2] = v.z; b[3] = v.w;
            }
            uint32_t d0[4], d1[4], d2[4], d3[4];
            s8_word(w[r].x, d0);
            s8_word(w[r].y, d1);
            s8_word(w[r].z, d2);
            s8_word(w[r].w, d3);
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                const uint32_t bb[2] = {b[2 * s], b[2 * s + 1]};
                const uint32_t a0[4] = {d0[2 * s], d1[2 * s], d0[2 * s + 1], d1[2 * s + 1]};
                const uint32_t a1[4] = {d2[2 * s], d3[2 * s], d2[2 * s + 1], d3[2 * s + 1]};
                mma_s8(part[0], a0, bb);
                mma_s8(part[1], a1, bb);
            }
        }
        const float2 inv = *reinterpret_cast<const float2 *>(xg + 8 * q);  // rows 2q, 2q+1
        const float s0 = DT::tof((uint16_t)(sc.x & 0xffffu)), s1 = DT::tof((uint16_t)(sc.x >> 16));
        const float s2 = DT::tof((uint16_t)(sc.y & 0xffffu)), s3 = DT::tof((uint16_t)(sc.y >> 16));
        // acc += float(dot) * (SB * inv)   (int2_via_int2_x_int8_dpas/main.cpp:117)
        acc[0][0] += (float)part[0][0] * (s0 * inv.x);
        acc[0][1] += (float)part[0][1] * (s0 * inv.y);
        acc[0][2] += (float)part[0][2] * (s1 * inv.x);
        acc[0][3] += (float)part[0][3] * (s1 * inv.y);
        acc[1][0] += (float)part[1][0] * (s2 * inv.x);
        acc[1][1] += (float)part[1][1] * (s2 * inv.y);
        acc[1][2] += (float)part[1][2] * (s3 * inv.x);
        acc[1][3] += (float)part[1][3] * (s3 * inv.y);
    }

    __device__ static void thread_values(const float acc[2][4], float v[8]) {
        v[0] = acc[0][0]; v[1] = acc[0][2]; v[2] = acc[1][0]; v[3] = acc[1][2];
        v[4] = acc[0][1]; v[5] = acc[0][3]; v[6] = acc[1][1]; v[7] = acc[1][3];
    }
};

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a) {
    gemv::Params p = gemv::gemv_params_impl(a);
    const int G = a.K / kGS;
    const int max_ng = (G + a.SK - 1) / a.SK;
    const int rows = a.M < 8 ? a.M : 8;
    const size_t smem = gemv::smem_bytes<Int8Policy, gemv::kWarps>(rows, max_ng * kGS);
    auto kern = gemv::gemv_kernel<Int8Policy, gemv::kWarps, DT, POSTOP, OUT_F32>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((a.N + 31) / 32, a.SK, (a.M + 7) / 8);
    return launch_kernel_cluster(kern, grid, dim3(gemv::kThreads), smem, a.stream,
                                 dim3(1, a.cluster ? a.SK : 1, 1), p);
}

}  // namespace

size_t int8_gemv_smem(int M, int K, int SK) {
    const int G = K / kGS;
    const int max_ng = (G + SK - 1) / SK;
    return gemv::smem_bytes<Int8Policy, gemv::kWarps>(M < 8 ? M : 8, max_ng * kGS);
}

cudaError_t int8_gemv_launch(const GemvArgs &a) {
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_t<DT, decltype(po)::value, decltype(of)::value>(a);
    });
}

}  // namespace ternocl
