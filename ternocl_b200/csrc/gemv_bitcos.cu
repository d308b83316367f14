// BITCOS ternary decode GEMV (small M), replaces bitcos_fp16_upcvt_gemv
// (bitcos_fp16_upcvt.cl:177-277):
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(k,n) )),  code in {-1,0,+1}
//
// B is one uint32 buffer (common/bitcos.hpp:1-8): bitmap [K/32][N] (bit c of word
// (kp,n) = weight(32kp+c, n) != 0) | offsets [N] (first sign word of column n) |
// signs (one bit per non-zero, column-major in k, 1 -> -1) | 4 pad words.  SR =
// slice_ranks [ls-1][N]: non-zeros of column n above row s*K/ls.  Host gold:
// compute_gold + bitcos_decode_col (bitcos_fp16_upcvt/main.cpp:64-86,
// common/bitcos.hpp:97-106).
//
// The sign stream of a column is addressed by its rank (non-zeros above a row), so a
// CTA (32 columns x a range of 128-row groups x <= 8 activation rows) first stages its
// whole slice in shared memory:
//   1. the bitmap words of its K range (coalesced rows of 32 columns) and the scales;
//   2. the rank of each column at the range start: SR at the reference slice that
//      contains it, plus the popcount of the bitmap words between that slice boundary
//      and the range start (read straight from global memory / L2);
//   3. per warp the popcount of its sub-range -> every warp's starting rank;
//   4. the sign words that cover [start rank, end rank] of each column (plus one word
//      for the 64-bit window), which are contiguous in the stream;
//   5. (after griddepcontrol.wait) the activation rows, 16-byte units swizzled so the
//      main loop's reads are conflict-free.  With the fused Hadamard transform (had_L > 0,
//      the reference's hadamard_fwht -> BITCOS GEMV pipeline in one launch) each HB-wide
//      block of the CTA's K range (K split on HB boundaries) is then sign-flipped and
//      transformed in place by one warp, as hadamard_fwht does it (same fp32 stages in the
//      same order, the same DT rounding): the result equals the two-kernel pipeline's.
// Main loop (per warp, per group): lane (g, q) takes bitmap word q (rows 32q..32q+31)
// of columns 4g..4g+3.  The four q lanes of a column scan their popcounts (packed
// 4 columns x 8 bits, two shuffles) to get each word's rank, and funnel-shift a
// 32-bit sign window out of the staged stream.  Each 4-row nibble then indexes a
// 256-entry shared table (presence nibble, next 4 sign bits) -> 4 DT codes as two
// half2 (the reference's table, bitcos_fp16_upcvt.cl:109-123), and the window shifts
// by the nibble's popcount.  The codes are the A operand of mma.sync m16n8k16
// (row g -> column 4g+2b, row g+8 -> 4g+2b+1; nibble s of lane q = MMA k-step s), the
// group's fp32 partial is scaled by S (the gold's `acc += partial * S`).  K split and
// reduction as the other GEMVs (gemv::finish).
#include <cuda_runtime.h>

#include "gemv_common.cuh"
#include "hadamard_common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

constexpr int kThreads = gemv::kThreads;
constexpr int kMetaBytes = 2048;  // ranks and per-column sign-window bookkeeping
constexpr int kRedBytes = gemv::kWarps * 32 * 8 * 4;  // gemv::finish's reduction area (>= the 2 KB table)

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(gemv::smem_u32(dst)), "l"(src));
}

struct BitcosCols {
    static constexpr bool kContiguousCols = true;
    __device__ static int thread_col(int g, int i) { return 4 * g + i; }
};

__host__ __device__ inline int sign_cap(int ng) { return 4 * ng + 3; }  // staged sign words per column

__host__ __device__ inline size_t bitcos_smem_bytes(int rows, int ng, bool had = false) {
    return (size_t)kRedBytes + kMetaBytes + (size_t)ng * 32 * 2 + (size_t)ng * 4 * 32 * 4 +
           (size_t)32 * sign_cap(ng) * 4 + (size_t)rows * ((size_t)ng * kGS * 2 + 16) + (had ? (size_t)ng * kGS : 0);
}

template <class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kThreads) bitcos_gemv_kernel(const gemv::Params p) {
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q = lane & 3;
    const int n0 = blockIdx.x * 32;
    const int mb = blockIdx.z * 8;
    const int N = p.N, K = p.K;
    const int G = K / kGS;
    const int sk = blockIdx.y;
    // K split in units of gran groups (the fused transform's blocks stay within one CTA)
    const int gran = p.had_L ? (1 << p.had_L) / kGS : 1, U = G / gran;
    const int cg0 = gran * (int)((long long)U * sk / p.SK), cg1 = gran * (int)((long long)U * (sk + 1) / p.SK);
    const int ng = cg1 - cg0;
    const int wg0 = cg0 + ng * warp / gemv::kWarps, wg1 = cg0 + ng * (warp + 1) / gemv::kWarps;
    const int rows = min(8, p.M - mb);
    const int krange = ng * kGS;
    const bool colok = n0 + 4 * g < N;  // N % 16 == 0

    uint2 *lut = reinterpret_cast<uint2 *>(smem);  // 256 entries; the reduction reuses it
    uint32_t *meta = reinterpret_cast<uint32_t *>(smem + kRedBytes);
    uint32_t *rk = meta;           // [5][32]: rank of each warp's first row, then the end rank
    uint32_t *pre = meta + 160;    // [4][32]: popcount partials before the range
    uint32_t *seg = meta + 288;    // [4][32]: popcount of each warp's sub-range
    uint32_t *soff = meta + 416;   // [32]: column's first sign word (offsets plane)
    uint32_t *swlo = meta + 448;   // [32]: first staged sign word (relative to soff)
    uint32_t *scnt = meta + 480;   // [32]: staged sign words
    uint16_t *ssc = reinterpret_cast<uint16_t *>(smem + kRedBytes + kMetaBytes);  // [ng][32]
    uint32_t *sbm = reinterpret_cast<uint32_t *>(ssc + ng * 32);                     // [4ng][32]
    const int cap = sign_cap(ng);
    uint32_t *ssg = sbm + 4 * ng * 32;  // [32][cap]
    char *act = reinterpret_cast<char *>(ssg + 32 * cap);
    const int act_stride = krange * 2 + 16;

    // (presence nibble m, 4 sign bits s) -> DT codes of 4 rows, in row order
    constexpr uint32_t kPos = DT::kBF16 ? 0x3F80u : 0x3C00u, kNeg = kPos | 0x8000u;
    for (int idx = tid; idx < 256; idx += kThreads) {
        const uint32_t m = (uint32_t)idx >> 4, s = (uint32_t)idx & 15u;
        uint32_t c[4], r = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t pr = (m >> i) & 1u;
            c[i] = pr ? (((s >> r) & 1u) ? kNeg : kPos) : 0u;
            r += pr;
        }
        lut[idx] = make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
    }

    // 1. bitmap words and scales of the range (weights: staged before the PDL wait),
    //    16-byte cp.async chunks: a bitmap row of 32 columns is 8 chunks, a scale row 4
    const uint32_t *B = p.B;
    const int nkp = 4 * ng;
    const int ncol = min(32, N - n0);  // 16 or 32 (N % 16 == 0)
    for (int idx = tid; idx < nkp * 8; idx += kThreads) {
        const int kp = idx >> 3, ch = idx & 7;
        if (ch * 4 < ncol) gemv::cp_async16(sbm + kp * 32 + ch * 4, B + (size_t)(cg0 * 4 + kp) * N + n0 + ch * 4);
    }
    for (int idx = tid; idx < ng * 4; idx += kThreads) {
        const int gi = idx >> 2, ch = idx & 3;
        if (ch * 8 < ncol) gemv::cp_async16(ssc + gi * 32 + ch * 8, p.S + (size_t)(cg0 + gi) * N + n0 + ch * 8);
    }
    gemv::cp_async_commit();
    // 2. popcount between the enclosing reference slice's boundary and the range start
    const int slice_rows = K / p.ls;
    const int s0 = (cg0 * kGS) / slice_rows;
    {
        const int kp_from = s0 * slice_rows / 32, kp_to = cg0 * 4;
        uint32_t cnt = 0;
        if (lane < ncol) {
#pragma unroll 8
            for (int kp = kp_from + warp; kp < kp_to; kp += gemv::kWarps)
                cnt += __popc(__ldg(B + (size_t)kp * N + n0 + lane));
        }
        pre[warp * 32 + lane] = cnt;
    }
    gemv::cp_async_wait<0>();
    __syncthreads();
    // 3. popcount of each warp's sub-range (columns >= N hold stale words: not used)
    {
        uint32_t cnt = 0;
        for (int kp = (wg0 - cg0) * 4; kp < (wg1 - cg0) * 4; ++kp) cnt += __popc(sbm[kp * 32 + lane]);
        seg[warp * 32 + lane] = lane < ncol ? cnt : 0u;
    }
    __syncthreads();
    const size_t bw = (size_t)(K / 32) * N;
    if (tid < 32) {
        const int c = tid;
        const bool ok = c < ncol;
        uint32_t r = (ok && s0 > 0) ? __ldg(p.SR + (size_t)(s0 - 1) * N + n0 + c) : 0u;
        r += pre[c] + pre[32 + c] + pre[64 + c] + pre[96 + c];
#pragma unroll
        for (int w = 0; w < gemv::kWarps; ++w) {
            rk[w * 32 + c] = r;
            r += seg[w * 32 + c];
        }
        rk[128 + c] = r;
        const uint32_t wlo = rk[c] >> 5;
        soff[c] = ok ? __ldg(B + bw + n0 + c) : 0u;
        swlo[c] = wlo;
        scnt[c] = ok ? (r >> 5) + 2 - wlo : 0u;  // windows read words rank/32 and rank/32 + 1
    }
    __syncthreads();
    // 4. the sign words of each column's range, contiguous in the stream: warp w copies
    //    columns w, w + 4, ..., its lanes consecutive words (4-byte copies: a column's
    //    first word has no alignment)
    const uint32_t *signs = B + bw + N;
    for (int c = warp; c < 32; c += gemv::kWarps) {
        const uint32_t cnt = scnt[c];
        const uint32_t *src = signs + soff[c] + swlo[c];
        uint32_t *dst = ssg + c * cap;
        for (uint32_t i = lane; i < cnt; i += 32) cp_async4(dst + i, src + i);
    }
    // 5. activations, 16-byte unit u stored at u ^ (((u >> 3) & 1) << 1)
    pdl_wait();
    const int nu = krange / 8;
    for (int it = tid; it < rows * nu; it += kThreads) {
        const int m = it / nu, u = it - m * nu;
        const int pu = u ^ (((u >> 3) & 1) << 1);
        gemv::cp_async16(act + (size_t)m * act_stride + (size_t)pu * 16,
                         p.A + (size_t)(mb + m) * K + (size_t)cg0 * kGS + (size_t)u * 8);
    }
    // the fused transform's signs of the range follow the rows
    int8_t *sgn = reinterpret_cast<int8_t *>(act + (size_t)rows * act_stride);
    if (p.had_L && p.had_signs)
        for (int u = tid; u < krange / 16; u += kThreads) gemv::cp_async16(sgn + 16 * u, p.had_signs + cg0 * kGS + 16 * u);
    gemv::cp_async_commit();
    gemv::cp_async_wait<0>();
    __syncthreads();
    if (p.had_L) {
        const int8_t *sg = p.had_signs ? sgn : nullptr;
        if (p.had_L == 8) fwht::staged_rows<DT, 8>(act, act_stride, sg, rows, krange, p.had_scale, warp, gemv::kWarps, lane);
        else if (p.had_L == 9) fwht::staged_rows<DT, 16>(act, act_stride, sg, rows, krange, p.had_scale, warp, gemv::kWarps, lane);
        else fwht::staged_rows<DT, 32>(act, act_stride, sg, rows, krange, p.had_scale, warp, gemv::kWarps, lane);
        __syncthreads();
    }

    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    const bool rowok = g < rows;
    const char *arow = act + (size_t)(rowok ? g : 0) * act_stride;
    uint32_t rcur[4], wbase[4];
    const uint32_t *sgc[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        rcur[c] = rk[warp * 32 + 4 * g + c];
        wbase[c] = swlo[4 * g + c];
        sgc[c] = ssg + (4 * g + c) * cap;
    }

    for (int grp = wg0; grp < wg1; ++grp) {
        const int gl = grp - cg0;
        const uint4 P4 = *reinterpret_cast<const uint4 *>(sbm + (gl * 4 + q) * 32 + 4 * g);
        const uint32_t P[4] = {P4.x, P4.y, P4.z, P4.w};
        // rank of word q within the group: exclusive scan over the 4 q lanes, 4 columns
        // packed in bytes (sums <= 128)
        const uint32_t cnt = __popc(P[0]) | (__popc(P[1]) << 8) | (__popc(P[2]) << 16) | (__popc(P[3]) << 24);
        uint32_t x = cnt;
        uint32_t y = __shfl_up_sync(0xffffffffu, x, 1, 4);
        if (q >= 1) x += y;
        y = __shfl_up_sync(0xffffffffu, x, 2, 4);
        if (q >= 2) x += y;
        const uint32_t excl = x - cnt;
        const uint32_t tot = __shfl_sync(0xffffffffu, x, 3, 4);
        uint32_t W[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t r = rcur[c] + ((excl >> (8 * c)) & 0xffu);
            const uint32_t l = (r >> 5) - wbase[c];
            W[c] = __funnelshift_r(sgc[c][l], sgc[c][l + 1], r & 31u);
            rcur[c] += (tot >> (8 * c)) & 0xffu;
        }

        float part[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) {
            uint4 av = make_uint4(0u, 0u, 0u, 0u);
            if (rowok) {
                const int u = gl * 16 + 4 * q + s2;  // rows 32q + 8 s2 .. +7 of the group
                av = *reinterpret_cast<const uint4 *>(arow + (size_t)(u ^ (((u >> 3) & 1) << 1)) * 16);
            }
            const uint32_t acts[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int hs = 0; hs < 2; ++hs) {
                const int s = 2 * s2 + hs;  // nibble s: rows 32q + 4s .. 32q + 4s + 3
                uint2 e[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t nib4 = s == 0 ? (P[c] << 4) & 0xf0u : (P[c] >> (4 * s - 4)) & 0xf0u;
                    e[c] = lut[nib4 | (W[c] & 0xfu)];
                    W[c] >>= __popc(nib4);
                }
                const uint32_t bb[2] = {acts[2 * hs], acts[2 * hs + 1]};
                const uint32_t a0[4] = {e[0].x, e[1].x, e[0].y, e[1].y};
                const uint32_t a1[4] = {e[2].x, e[3].x, e[2].y, e[3].y};
                mma16816<DT>(part[0], a0, bb);
                mma16816<DT>(part[1], a1, bb);
            }
        }
        const uint2 sc = *reinterpret_cast<const uint2 *>(ssc + gl * 32 + 4 * g);
        const float s0f = DT::tof((uint16_t)(sc.x & 0xffffu)), s1f = DT::tof((uint16_t)(sc.x >> 16));
        const float s2f = DT::tof((uint16_t)(sc.y & 0xffffu)), s3f = DT::tof((uint16_t)(sc.y >> 16));
        // acc += partial * S  (bitcos_fp16_upcvt/main.cpp:80)
        acc[0][0] += part[0][0] * s0f;
        acc[0][1] += part[0][1] * s0f;
        acc[0][2] += part[0][2] * s1f;
        acc[0][3] += part[0][3] * s1f;
        acc[1][0] += part[1][0] * s2f;
        acc[1][1] += part[1][1] * s2f;
        acc[1][2] += part[1][2] * s3f;
        acc[1][3] += part[1][3] * s3f;
    }
    pdl_launch_dependents();

    float v[8];
    v[0] = acc[0][0]; v[1] = acc[0][2]; v[2] = acc[1][0]; v[3] = acc[1][2];
    v[4] = acc[0][1]; v[5] = acc[0][3]; v[6] = acc[1][1]; v[7] = acc[1][3];
    __syncthreads();  // the table and staging area are reused for the reduction
    gemv::finish<BitcosCols, gemv::kWarps, DT, POSTOP, OUT_F32>(p, smem, v, colok);
}

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a) {
    gemv::Params p = gemv::gemv_params_impl(a);
    const int G = a.K / kGS, gran = a.had_hb ? a.had_hb / kGS : 1;
    const int max_ng = gran * ((G / gran + a.SK - 1) / a.SK);
    const int rows = a.M < 8 ? a.M : 8;
    const size_t smem = bitcos_smem_bytes(rows, max_ng, a.had_hb != 0);
    auto kern = bitcos_gemv_kernel<DT, POSTOP, OUT_F32>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((a.N + 31) / 32, a.SK, (a.M + 7) / 8);
    return launch_kernel_cluster(kern, grid, dim3(kThreads), smem, a.stream, dim3(1, a.cluster ? a.SK : 1, 1), p);
}

}  // namespace

size_t bitcos_gemv_smem(int M, int K, int SK, int had_hb) {
    const int G = K / kGS, gran = had_hb ? had_hb / kGS : 1;
    return bitcos_smem_bytes(M < 8 ? M : 8, gran * ((G / gran + SK - 1) / SK), had_hb != 0);
}

cudaError_t bitcos_gemv_launch(const GemvArgs &a) {
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_t<DT, decltype(po)::value, decltype(of)::value>(a);
    });
}

}  // namespace ternocl
