// int2 upconvert decode GEMV (small M), replaces int2_fp16_upcvt_gemm
// (int2_fp16_upcvt.cl:193-290):
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(B[k,n]) ))
//
// Weight layout B uint32 [K/16, N] (code of row 16kp+j at bits 2j..2j+1).  Thread
// (g, q) streams, per 128-row group, the words of rows kp = 8grp + 4r + q (r = 0, 1)
// and columns n0+4g .. n0+4g+3 (one 16-byte chunk per r; a warp reads 4 rows x 128
// contiguous bytes per chunk) plus the 4 scales of those columns.
//
// Each word is decoded in registers (one LOP3 + one HSUB2 per pair of weights, see
// Int2Decode in common.cuh) straight into the A operand of mma.sync m16n8k16: the
// 16 weight columns of a block are the MMA rows (row g = column 4g+{0,2}, row g+8 =
// 4g+{1,3}), the <= 8 activation rows its 8 columns.  Decoded pair p of a word holds
// rows p and p+8, so the MMA's K runs over a fixed permutation of each 16-row word;
// the activations are staged in shared memory in that permuted order.  After the
// group's 8 MMAs the exact fp32 partial is scaled by S[g,n] and accumulated (the host
// gold's `acc += partial * S`, int2_fp16_upcvt/main.cpp:94).
//
// (A variant that feeds the raw LOP3 result to the MMA and subtracts the magic
// constant once per group through an activation-sum correction was measured slower
// on B200 -- the integer pipe is already the busiest -- and less accurate.)
#include <cuda_runtime.h>

#include "gemv_common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

// decoded pair at in-half position JP of x: LOP3 ((x & both) ^ k1) then k1 - r, see
// Int2Decode (common.cuh) for the derivation
template <class DT, int JP>
__device__ __forceinline__ uint32_t dec_pair(uint32_t x) {
    constexpr uint32_t both = (3u << (2 * JP)) * 0x00010001u;
    constexpr uint32_t magic = DT::kBF16 ? ((uint32_t)(134 - 2 * JP) << 7) : ((uint32_t)(25 - 2 * JP) << 10);
    constexpr uint32_t k1 = (magic | (1u << (2 * JP))) * 0x00010001u;
    uint32_t r, v;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;\n" : "=r"(r) : "r"(x), "n"(both), "r"(k1));
    if constexpr (DT::kBF16) asm("sub.rn.bf16x2 %0, %1, %2;\n" : "=r"(v) : "r"(k1), "r"(r));
    else asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(v) : "r"(k1), "r"(r));
    return v;
}

// all 8 pairs of a word: out[p] = (row p, row p+8)
template <class DT>
__device__ __forceinline__ void dec_word(uint32_t x, uint32_t out[8]) {
    if constexpr (DT::kBF16) {
        const uint32_t y1 = x >> 6, y2 = x >> 12;
        out[0] = dec_pair<DT, 0>(x); out[1] = dec_pair<DT, 1>(x); out[2] = dec_pair<DT, 2>(x);
        out[3] = dec_pair<DT, 0>(y1); out[4] = dec_pair<DT, 1>(y1); out[5] = dec_pair<DT, 2>(y1);
        out[6] = dec_pair<DT, 0>(y2); out[7] = dec_pair<DT, 1>(y2);
    } else {
        const uint32_t y = x >> 10;
        out[0] = dec_pair<DT, 0>(x); out[1] = dec_pair<DT, 1>(x); out[2] = dec_pair<DT, 2>(x);
        out[3] = dec_pair<DT, 3>(x); out[4] = dec_pair<DT, 4>(x);
        out[5] = dec_pair<DT, 0>(y); out[6] = dec_pair<DT, 1>(y); out[7] = dec_pair<DT, 2>(y);
    }
}

struct Int2Policy {
    static constexpr int kWords16 = 2;
    static constexpr int kWordRegs = kWords16;
    static constexpr bool kSharedSlots = false;
    __device__ static void read_words(const char *stage, int tid, int nthreads, uint4 *w) {
#pragma unroll
        for (int c = 0; c < kWords16; ++c) w[c] = reinterpret_cast<const uint4 *>(stage)[c * nthreads + tid];
    }
    static constexpr bool kContiguousCols = true;
    static constexpr int kActGroupBytes = 8 * 32;   // 8 words x 8 slot registers
    static constexpr int kExtraGroupBytes = 0;
    static constexpr int kActBytesPerK = 2;  // DT activations
    static constexpr int kActPadBytes = 16;  // row stride = 16 mod 128: 32-byte reads conflict-free
    __device__ static int thread_col0(int g) { return 4 * g; }
    __device__ static bool copy_ok(int N, int n0, int g) { return n0 + 4 * g < N; }
    __device__ static int thread_col(int g, int i) { return 4 * g + i; }
    // chunk c of group grp: word row kp = 8grp + 4c + q, columns n0+4g .. n0+4g+3
    __device__ static const uint32_t *word_ptr(const gemv::Params &p, int grp, int g, int q, int n0) {
        return p.B + (size_t)(grp * 8 + q) * p.N + n0 + 4 * g;
    }
    __device__ static size_t group_stride(const gemv::Params &p) { return (size_t)8 * p.N; }
    __device__ static size_t chunk_stride(const gemv::Params &p) { return (size_t)4 * p.N; }
    __host__ __device__ static size_t extra_smem(int, int) { return 0; }

    // Stage rows [mb, mb+rows) x words [8cg0, 8(cg0+ng)) as 8 pairs (j, j+8) per word.
    template <class DT>
    __device__ static void stage(const gemv::Params &p, char *act, int stride, char *, int mb, int rows, int cg0,
                                 int ng) {
        const int nw = ng * 8;
        for (int it = threadIdx.x; it < rows * nw; it += blockDim.x) {
            const int m = it / nw, w = it - m * nw;
            const uint16_t *src = p.A + (size_t)(mb + m) * p.K + (size_t)(cg0 * 8 + w) * 16;
            const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(src));
            const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(src + 8));
            uint4 o0, o1;
            o0.x = __byte_perm(lo.x, hi.x, 0x5410);
            o0.y = __byte_perm(lo.x, hi.x, 0x7632);
            o0.z = __byte_perm(lo.y, hi.y, 0x5410);
            o0.w = __byte_perm(lo.y, hi.y, 0x7632);
            o1.x = __byte_perm(lo.z, hi.z, 0x5410);
            o1.y = __byte_perm(lo.z, hi.z, 0x7632);
            o1.z = __byte_perm(lo.w, hi.w, 0x5410);
            o1.w = __byte_perm(lo.w, hi.w, 0x7632);
            uint4 *dst = reinterpret_cast<uint4 *>(act + (size_t)m * stride + (size_t)w * 32);
            dst[0] = o0;
            dst[1] = o1;
        }
    }

    template <class DT>
    __device__ static void compute(const uint4 w[2], uint2 sc, const char *arow, bool rowok, int q,
                                   const char *xg, float acc[2][4], int) {
        float part[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            uint32_t b[8];
            if (rowok) {
                const uint4 *src = reinterpret_cast<const uint4 *>(arow + (4 * r + q) * 32);
                const uint4 b0 = src[0], b1 = src[1];
                b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
                b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) b[i] = 0u;
            }
            uint32_t d0[8], d1[8], d2[8], d3[8];
            dec_word<DT>(w[r].x, d0);
            dec_word<DT>(w[r].y, d1);
            dec_word<DT>(w[r].z, d2);
            dec_word<DT>(w[r].w, d3);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t bb[2] = {b[2 * s], b[2 * s + 1]};
                const uint32_t a0[4] = {d0[2 * s], d1[2 * s], d0[2 * s + 1], d1[2 * s + 1]};
                const uint32_t a1[4] = {d2[2 * s], d3[2 * s], d2[2 * s + 1], d3[2 * s + 1]};
                mma16816<DT>(part[0], a0, bb);
                mma16816<DT>(part[1], a1, bb);
            }
        }
        const float s0 = DT::tof((uint16_t)(sc.x & 0xffffu)), s1 = DT::tof((uint16_t)(sc.x >> 16));
        const float s2 = DT::tof((uint16_t)(sc.y & 0xffffu)), s3 = DT::tof((uint16_t)(sc.y >> 16));
        acc[0][0] += part[0][0] * s0;
        acc[0][1] += part[0][1] * s0;
        acc[0][2] += part[0][2] * s1;
        acc[0][3] += part[0][3] * s1;
        acc[1][0] += part[1][0] * s2;
        acc[1][1] += part[1][1] * s2;
        acc[1][2] += part[1][2] * s3;
        acc[1][3] += part[1][3] * s3;
    }

    // C fragment: block b, c0/c1 = (row g -> column 4g+2b, activation rows 2q, 2q+1),
    // c2/c3 = (row g+8 -> column 4g+2b+1)
    __device__ static void thread_values(const float acc[2][4], float v[8]) {
        v[0] = acc[0][0]; v[1] = acc[0][2]; v[2] = acc[1][0]; v[3] = acc[1][2];
        v[4] = acc[0][1]; v[5] = acc[0][3]; v[6] = acc[1][1]; v[7] = acc[1][3];
    }
};

template <int W, class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_w(const GemvArgs &a) {
    gemv::Params p = gemv::gemv_params_impl(a);
    const int G = a.K / kGS;
    const int max_ng = (G + a.SK - 1) / a.SK;
    const int rows = a.M < 8 ? a.M : 8;
    const size_t smem = gemv::smem_bytes<Int2Policy, W>(rows, max_ng * kGS);
    auto kern = gemv::gemv_kernel<Int2Policy, W, DT, POSTOP, OUT_F32>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((a.N + 31) / 32, a.SK, (a.M + 7) / 8);
    return launch_kernel_cluster(kern, grid, dim3(W * 32), smem, a.stream, dim3(1, a.cluster ? a.SK : 1, 1), p);
}

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a) {
    if (a.warps >= 16) return launch_w<16, DT, POSTOP, OUT_F32>(a);
    if (a.warps >= 8) return launch_w<8, DT, POSTOP, OUT_F32>(a);
    return launch_w<4, DT, POSTOP, OUT_F32>(a);
}

}  // namespace

size_t int2_gemv_smem(int M, int K, int SK, int warps) {
    const int G = K / kGS;
    const int max_ng = (G + SK - 1) / SK;
    return gemv::smem_bytes_w<Int2Policy>(warps, M < 8 ? M : 8, max_ng * kGS);
}

cudaError_t int2_gemv_launch(const GemvArgs &a) {
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_t<DT, decltype(po)::value, decltype(of)::value>(a);
    });
}

}  // namespace ternocl
