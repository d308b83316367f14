// int1 ({+1,-1} x per-group scale) upconvert decode GEMV (small M), replaces
// int1_fp16_upcvt_gemm (int1_fp16_upcvt.cl:166-170):
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * sgn(B[k,n]) )),  bit 1 -> -1
//
// B is the reference's select layout, uint32 [K/32, N]: within K32 row kp and
// 16-column block n0, word (kp, n0+p) bit j = (row 32kp + 2p + (j&1), column n0 + j/2)
// (int1_fp16_upcvt/main.cpp:78-92).  Host gold: compute_gold, main.cpp:95-114.
//
// Ring and reads.  Per 128-row group a warp's 32 lanes copy the group's 4 x 32 words
// of the CTA's 32-column strip (lane t: K32 row t/8, block (t/4)&1, words 4(t&3)..+3),
// one 16-byte cp.async each.  A sel word holds 2 rows x 16 columns, so every word is
// needed by 4 lanes: lane (g, q) reads, for each K32 row j, the 16 bytes of words
// p = 4q..4q+3 of block g/4 (a broadcast read; the 8 distinct chunks of a warp read
// are one contiguous 128 bytes), i.e. rows 32j + 8q .. 32j + 8q + 7.
//
// Decode.  Byte g&3 of a word holds the thread's columns 4g..4g+3 for the word's
// row pair (bit 2c + r: column 4g + c, row 2p + r).  One PRMT isolates it (t), then
// per column one IMAD moves bits 2c and 2c+1 onto the two sign bits (15 and 31) --
// t * (2^(15-2c) + 2^(30-2c)) puts the 16 bits of t at distinct positions, so there
// are no carries -- and one LOP3 keeps the sign bits and ORs in DT(1.0): a half2 of
// +-1 for rows (2p, 2p+1) of the column, the A operand register of mma.sync
// m16n8k16 (weights = MMA rows: row g -> column 4g+2b, row g+8 -> 4g+2b+1).  That
// is 9 instructions per 8 weights.  The MMA's K order is the natural row order
// within the thread's 8 rows, so the activations are staged unpermuted.
#include <cuda_runtime.h>

#include "gemv_common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

template <class DT>
__device__ __forceinline__ uint32_t sign_pair(uint32_t t, uint32_t mul) {
    constexpr uint32_t one = DT::kBF16 ? 0x3F803F80u : 0x3C003C00u;
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(t * mul), "n"(0x80008000u), "n"(one));
    return r;
}

struct Int1Policy {
    static constexpr int kWords16 = 1;     // one 16-byte chunk copied per lane per group
    static constexpr int kWordRegs = 4;    // four 16-byte chunks read per lane per group
    static constexpr bool kSharedSlots = true;
    static constexpr bool kContiguousCols = true;
    static constexpr int kActGroupBytes = 128 * 2;
    static constexpr int kExtraGroupBytes = 0;
    static constexpr int kActBytesPerK = 2;
    static constexpr int kActPadBytes = 64;  // row stride = 64 mod 128: 16-byte reads conflict-free
    __device__ static int thread_col0(int g) { return 4 * g; }
    // a strip's second 16-column block exists only when N - n0 > 16 (N % 16 == 0)
    __device__ static bool copy_ok(int N, int n0, int g) { return n0 + 16 * (g & 1) < N; }
    __device__ static int thread_col(int g, int i) { return 4 * g + i; }
    // the chunk this lane copies: K32 row g/2 of the group, block g&1, words 4q..4q+3
    __device__ static const uint32_t *word_ptr(const gemv::Params &p, int grp, int g, int q, int n0) {
        return p.B + (size_t)(grp * 4 + (g >> 1)) * p.N + n0 + 16 * (g & 1) + 4 * q;
    }
    __device__ static size_t group_stride(const gemv::Params &p) { return (size_t)4 * p.N; }
    __device__ static size_t chunk_stride(const gemv::Params &) { return 0; }
    __host__ __device__ static size_t extra_smem(int, int) { return 0; }

    __device__ static void read_words(const char *stage, int tid, int, uint4 *w) {
        const int lane = tid & 31, g = lane >> 2, q = lane & 3;
        const uint4 *base = reinterpret_cast<const uint4 *>(stage) + (tid & ~31) + (g >> 2) * 4 + q;
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = base[j * 8];
    }

    // plain copy of rows [mb, mb+rows) x K [128 cg0, 128 (cg0+ng))
    template <class DT>
    __device__ static void stage(const gemv::Params &p, char *act, int stride, char *, int mb, int rows, int cg0,
                                 int ng) {
        const int nc = ng * (kGS / 8);  // 16-byte chunks per row
        for (int it = threadIdx.x; it < rows * nc; it += blockDim.x) {
            const int m = it / nc, c = it - m * nc;
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p.A + (size_t)(mb + m) * p.K + (size_t)cg0 * kGS) + c);
            *reinterpret_cast<uint4 *>(act + (size_t)m * stride + (size_t)c * 16) = v;
        }
    }

    template <class DT>
    __device__ static void compute(const uint4 w[4], uint2 sc, const char *arow, bool rowok, int q, const char *,
                                   float acc[2][4], int g) {
        constexpr uint32_t K1 = (1u << 15) + (1u << 30), K2 = (1u << 13) + (1u << 28);
        constexpr uint32_t K3 = (1u << 11) + (1u << 26), K4 = (1u << 9) + (1u << 24);
        const uint32_t sel = 0x4440u | (uint32_t)(g & 3);
        float part[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (rowok) v = *reinterpret_cast<const uint4 *>(arow + (32 * j + 8 * q) * 2);
            const uint32_t words[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
            const uint32_t acts[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t t0 = __byte_perm(words[2 * h], 0u, sel);
                const uint32_t t1 = __byte_perm(words[2 * h + 1], 0u, sel);
                const uint32_t bb[2] = {acts[2 * h], acts[2 * h + 1]};
                const uint32_t a0[4] = {sign_pair<DT>(t0, K1), sign_pair<DT>(t0, K2), sign_pair<DT>(t1, K1),
                                        sign_pair<DT>(t1, K2)};
                const uint32_t a1[4] = {sign_pair<DT>(t0, K3), sign_pair<DT>(t0, K4), sign_pair<DT>(t1, K3),
                                        sign_pair<DT>(t1, K4)};
                mma16816<DT>(part[0], a0, bb);
                mma16816<DT>(part[1], a1, bb);
            }
        }
        const float s0 = DT::tof((uint16_t)(sc.x & 0xffffu)), s1 = DT::tof((uint16_t)(sc.x >> 16));
        const float s2 = DT::tof((uint16_t)(sc.y & 0xffffu)), s3 = DT::tof((uint16_t)(sc.y >> 16));
        // acc += partial * S  (main.cpp:111)
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

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a) {
    gemv::Params p = gemv::gemv_params_impl(a);
    const int G = a.K / kGS;
    const int max_ng = (G + a.SK - 1) / a.SK;
    const int rows = a.M < 8 ? a.M : 8;
    const size_t smem = gemv::smem_bytes<Int1Policy, gemv::kWarps>(rows, max_ng * kGS);
    auto kern = gemv::gemv_kernel<Int1Policy, gemv::kWarps, DT, POSTOP, OUT_F32>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((a.N + 31) / 32, a.SK, (a.M + 7) / 8);
    return launch_kernel_cluster(kern, grid, dim3(gemv::kThreads), smem, a.stream,
                                 dim3(1, a.cluster ? a.SK : 1, 1), p);
}

}  // namespace

size_t int1_gemv_smem(int M, int K, int SK) {
    const int G = K / kGS;
    const int max_ng = (G + SK - 1) / SK;
    return gemv::smem_bytes<Int1Policy, gemv::kWarps>(M < 8 ? M : 8, max_ng * kGS);
}

cudaError_t int1_gemv_launch(const GemvArgs &a) {
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_t<DT, decltype(po)::value, decltype(of)::value>(a);
    });
}

}  // namespace ternocl
