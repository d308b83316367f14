// int2 upconvert decode GEMV (small M), replaces int2_fp16_upcvt_gemm
// (int2_fp16_upcvt.cl:193-290).
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(B[k,n]) ))
//
// Design (memory-bound; the weight stream is the roofline):
//  * A warp owns a strip of 32 columns and a contiguous range of 128-row scale
//    groups.  Thread (g = lane/4, q = lane%4) loads, per 64-row round, the four
//    adjacent packed words (kp = 4*round + q, columns n0+4g .. n0+4g+3) with one
//    streaming 128-bit load: a warp reads 4 rows x 128 contiguous bytes.
//  * Words are decoded in registers (Int2Decode: one LOP3 + one HSUB2 per pair of
//    weights) straight into the A operand of mma.sync m16n8k16 -- the weights are
//    the 16-row operand (rows g / g+8 = columns n0+4g+{0,1} and n0+4g+{2,3} of the
//    two 16-column blocks), the <= 8 activation rows the 8 MMA columns.  Each MMA's
//    K is a permutation of 16 physical rows (decoded pair p holds rows p and p+8);
//    the activation fragment is permuted the same way with two PRMTs per register.
//  * Per 128-row group the MMA partial (fp32) is scaled by S[g, n] and added to the
//    running fp32 accumulator (the host gold's `acc += partial * S`).
//  * K is split over the 4 warps of a CTA (fixed-order shared-memory reduction) and
//    over SK CTAs (grid.y); with SK > 1 the CTAs write fp32 partials to a workspace
//    and the last CTA to arrive for a column strip sums them in split order and runs
//    the epilogue, so results are bitwise reproducible.
//  * Rows beyond 8 use more CTAs along grid.z (8 activation rows each).
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kU = 2;  // groups whose loads are in flight ahead of the compute

struct GroupLoads {
    uint4 w[2];  // two 64-row rounds: 4 words (4 columns) each
    uint2 s;     // 4 scales (4 columns)
};

__device__ __forceinline__ void load_group(const uint32_t *__restrict__ B,
                                           const uint16_t *__restrict__ S, int N, int grp, int q,
                                           int col, bool ok, GroupLoads &L) {
    if (ok) {
        L.w[0] = ldg_stream128(B + (size_t)(grp * 8 + q) * N + col);
        L.w[1] = ldg_stream128(B + (size_t)(grp * 8 + 4 + q) * N + col);
        L.s = ldg_stream64(S + (size_t)grp * N + col);
    } else {
        L.w[0] = L.w[1] = make_uint4(0, 0, 0, 0);
        L.s = make_uint2(0, 0);
    }
}

// Activation fragment of one 64-row round for activation row m (lane group g):
// b[p] = (A[m, 16kp + p], A[m, 16kp + p + 8]), kp = this thread's word row.
__device__ __forceinline__ void load_act(const uint16_t *__restrict__ A, int K, int m, bool ok,
                                         int kp, uint32_t b[8]) {
    if (ok) {
        const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(A + (size_t)m * K + kp * 16));
        const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(A + (size_t)m * K + kp * 16 + 8));
        const uint32_t l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            b[2 * i] = __byte_perm(l[i], h[i], 0x5410);
            b[2 * i + 1] = __byte_perm(l[i], h[i], 0x7632);
        }
    } else {
#pragma unroll
        for (int p = 0; p < 8; ++p) b[p] = 0u;
    }
}

template <class DT>
__device__ __forceinline__ void compute_group(const GroupLoads &L, const uint32_t b[2][8],
                                              float acc[2][4]) {
    float part[2][4];
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        uint32_t d[4][8];
        Int2Decode<DT>::word(L.w[r].x, d[0]);
        Int2Decode<DT>::word(L.w[r].y, d[1]);
        Int2Decode<DT>::word(L.w[r].z, d[2]);
        Int2Decode<DT>::word(L.w[r].w, d[3]);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const uint32_t bb[2] = {b[r][2 * s], b[r][2 * s + 1]};
            const uint32_t a0[4] = {d[0][2 * s], d[1][2 * s], d[0][2 * s + 1], d[1][2 * s + 1]};
            const uint32_t a1[4] = {d[2][2 * s], d[3][2 * s], d[2][2 * s + 1], d[3][2 * s + 1]};
            if (r == 0 && s == 0) {
                mma16816<DT>(part[0], a0, bb, zero);
                mma16816<DT>(part[1], a1, bb, zero);
            } else {
                mma16816<DT>(part[0], a0, bb, part[0]);
                mma16816<DT>(part[1], a1, bb, part[1]);
            }
        }
    }
    const float s0 = DT::tof((uint16_t)(L.s.x & 0xffffu)), s1 = DT::tof((uint16_t)(L.s.x >> 16));
    const float s2 = DT::tof((uint16_t)(L.s.y & 0xffffu)), s3 = DT::tof((uint16_t)(L.s.y >> 16));
    acc[0][0] += part[0][0] * s0;
    acc[0][1] += part[0][1] * s0;
    acc[0][2] += part[0][2] * s1;
    acc[0][3] += part[0][3] * s1;
    acc[1][0] += part[1][0] * s2;
    acc[1][1] += part[1][1] * s2;
    acc[1][2] += part[1][2] * s3;
    acc[1][3] += part[1][3] * s3;
}

// Epilogue + store of the 8 accumulator values of one thread: rows mb+2q, mb+2q+1,
// columns col..col+3.
template <class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ void store_thread(void *C, const uint16_t *Other, const void *Bias,
                                             int M, int N, int mb, int q, int col,
                                             const float v[8]) {
    // v: row0 cols 0..3 = v[0..3], row1 cols 0..3 = v[4..7]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int m = mb + 2 * q + h;
        if (m < M) {
            epi_store2<DT, POSTOP, OUT_F32>(C, Other, Bias, N, m, col, v[4 * h + 0], v[4 * h + 1]);
            epi_store2<DT, POSTOP, OUT_F32>(C, Other, Bias, N, m, col + 2, v[4 * h + 2], v[4 * h + 3]);
        }
    }
}

template <class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kThreads) int2_gemv_kernel(
    const uint16_t *__restrict__ A, const uint32_t *__restrict__ B, const uint16_t *__restrict__ S,
    void *__restrict__ C, const uint16_t *__restrict__ Other, const void *__restrict__ Bias, int M,
    int N, int K, int SK, float *__restrict__ ws_part, unsigned *__restrict__ ws_cnt) {
    __shared__ float red[kWarps - 1][32][8];
    __shared__ unsigned s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int n0 = blockIdx.x * 32;
    const int mb = blockIdx.z * 8;
    const int G = K / kGS;
    const int sk = blockIdx.y;
    const int cg0 = (int)((long long)G * sk / SK), cg1 = (int)((long long)G * (sk + 1) / SK);
    const int ng = cg1 - cg0;
    const int wg0 = cg0 + ng * warp / kWarps, wg1 = cg0 + ng * (warp + 1) / kWarps;

    const int col = n0 + 4 * g;
    const bool colok = col < N;  // N % 16 == 0: the 4 columns are all valid or all not
    const int am = mb + g;       // activation row of this thread's B fragment
    const bool rowok = am < M;

    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    // Weight loads of the first kU groups are issued before waiting on the previous
    // kernel in the stream (programmatic dependent launch); activations after.
    GroupLoads cur[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) load_group(B, S, N, wg0 + u, q, col, colok && wg0 + u < wg1, cur[u]);
    pdl_wait();

    for (int grp = wg0; grp < wg1; grp += kU) {
        GroupLoads nxt[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
            load_group(B, S, N, grp + kU + u, q, col, colok && grp + kU + u < wg1, nxt[u]);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (grp + u < wg1) {
                uint32_t b[2][8];
                load_act(A, K, am, rowok, (grp + u) * 8 + q, b[0]);
                load_act(A, K, am, rowok, (grp + u) * 8 + 4 + q, b[1]);
                compute_group<DT>(cur[u], b, acc);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) cur[u] = nxt[u];
    }
    pdl_launch_dependents();

    // in-CTA reduction over the K-split warps, in warp order
    float v[8] = {acc[0][0], acc[0][2], acc[1][0], acc[1][2], acc[0][1], acc[0][3], acc[1][1], acc[1][3]};
    if (warp > 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) red[warp - 1][lane][i] = v[i];
    }
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int w = 0; w < kWarps - 1; ++w)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] += red[w][lane][i];

    if (SK == 1) {
        if (colok) store_thread<DT, POSTOP, OUT_F32>(C, Other, Bias, M, N, mb, q, col, v);
        return;
    }

    // cross-CTA split: partial -> workspace [SK][M][N]; the last CTA reduces in order
    if (colok) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = mb + 2 * q + h;
            if (m < M) {
                float *p = ws_part + ((size_t)sk * M + m) * N + col;
                __stcg(reinterpret_cast<float4 *>(p), make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]));
            }
        }
    }
    __threadfence();
    __syncwarp();
    const unsigned tile = blockIdx.z * gridDim.x + blockIdx.x;
    if (lane == 0) s_last = (atomicAdd(&ws_cnt[tile], 1u) == (unsigned)(SK - 1)) ? 1u : 0u;
    __syncwarp();
    if (!s_last) return;
    __threadfence();
    if (colok) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = mb + 2 * q + h;
            if (m < M) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int s = 0; s < SK; ++s) {
                    const float4 x = __ldcg(reinterpret_cast<const float4 *>(ws_part + ((size_t)s * M + m) * N + col));
                    t.x += x.x;
                    t.y += x.y;
                    t.z += x.z;
                    t.w += x.w;
                }
                v[4 * h] = t.x;
                v[4 * h + 1] = t.y;
                v[4 * h + 2] = t.z;
                v[4 * h + 3] = t.w;
            }
        }
        store_thread<DT, POSTOP, OUT_F32>(C, Other, Bias, M, N, mb, q, col, v);
    }
    if (lane == 0) ws_cnt[tile] = 0u;  // ready for the next call
}

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a) {
    dim3 grid((a.N + 31) / 32, a.SK, (a.M + 7) / 8);
    return launch_kernel(int2_gemv_kernel<DT, POSTOP, OUT_F32>, grid, dim3(kThreads), 0, a.stream,
                         (const uint16_t *)a.A, a.B, (const uint16_t *)a.S, a.C,
                         (const uint16_t *)a.Other, a.Bias, a.M, a.N, a.K, a.SK, a.ws_part,
                         a.ws_cnt);
}

}  // namespace

cudaError_t int2_gemv_launch(const GemvArgs &a) {
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_t<DT, decltype(po)::value, decltype(of)::value>(a);
    });
}

}  // namespace ternocl
