// int2 decode GEMV on integer MMAs (small M), the default M <= 4 implementation of
// int2_fp16_upcvt_gemm (int2_fp16_upcvt.cl:193-290):
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(B[k,n]) ))
//
// At M = 1 a GEMV is bound by the instructions that turn packed weights into MMA operands.
// Here one LOP3 turns a word into four MMA weights: the 2-bit code of a row sits in bits
// 2j..2j+1 of its byte, so (x << (6 - 2j)) & 0xC0C0C0C0 leaves the codes of rows
// j, j+4, j+8, j+12 in the top bits of the four bytes, which read as int8 are exactly
// 64 * code_to_value(code): 0 -> 0, 1 -> +64, 3 -> -64, 2 -> -128 (the host gold's
// int2_fp16_upcvt/main.cpp:76).  These feed mma.sync m16n8k32 s8 x u8 -> s32.
//
// The activations become exact integers: per warp and activation row m, with E_m the
// exponent of max |A[m, k]| over the warp's K range, i = round(A * 2^(22-E_m)) lies in
// (-2^22, 2^22) and is A exactly for every element within 2^11 of the row maximum (fp16
// keeps 11 significant bits); fma(A, 2^(22-E_m), 1.5 * 2^23) leaves i + 2^22 in the low
// 23 bits of the result.  Its three bytes are three unsigned activation "digit planes",
// which occupy three of the MMA's eight n-columns per row; a fourth column of ones
// gives sum_k W[k, n], which removes the 2^22 offset:
//
//   sum_k W * i = d0 + 256 d1 + 65536 d2 - 2^22 ones       (d_j = sum_k W * byte_j(i + 2^22))
//
// Every per-group dot product is exact in int32; the accumulator starts at the bit pattern
// of 1.5 * 2^23 so that, read as a float, it is 1.5 * 2^23 + dot (|dot| < 2^22) and one
// FADD recovers dot.  Per group and column the float dots are scaled by S (the gold's
// `acc += partial * S`), summed in fp32, and the planes are combined and scaled by
// 2^-(22-E_m) / 64 once at the end.  Error: only elements more than 2^11 below their row's
// maximum are rounded (by at most 2^-23 of that maximum), far inside the fp16 output.
// Rows whose maximum is Inf or NaN produce NaN.
//
// CTA: 32 columns x a K range of 128-row groups, W warps splitting the range by groups.
// Per group a warp's lanes copy the 8 x 32 weight words (two 16-byte cp.async each, rows
// of 128 bytes, the 64-byte halves of odd rows swapped so the reads below are
// conflict-free) and the 32 scales into the warp's ring stage.  Lane (g, t) of the MMA
// owns columns 2g, 2g+1 of each 16-column block (MMA rows g, g+8) and word rows t and
// 4+t (MMA k-blocks t and 4+t): one 8-byte read per block and word row gives the two
// words, and class j of the four words is MMA j's A operand.  The MMA's K order is a fixed
// permutation of the group's rows, and the activation planes are staged in that order
// (word row, class, byte) so that one 16-byte read gives a lane its B operand for all
// four classes.  The split-K reduction and the epilogue are gemv::finish.
#include <cuda_runtime.h>

#include "digit_common.cuh"
#include "gemv_common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

constexpr int kCols = 32;                        // CTA columns
constexpr int kRowBytes = kCols * 4;             // one word row of the strip
constexpr int kWordBytes = 8 * kRowBytes;        // a group's words (1 KB)
constexpr int kScaleBytes = kCols * 2;
constexpr int kStageBytes = kWordBytes + kScaleBytes;  // per warp
constexpr int kRingBytes = gemv::kStages * kStageBytes;
constexpr int kMaxRows = 4;                      // activation rows per CTA (13 n-columns)

__host__ __device__ constexpr int nmma_for(int rows) { return (1 + 3 * rows + 7) / 8; }

// plane stride in bytes for a warp's ngw groups: 16 bytes per word row, padded to 64 mod 128
__host__ __device__ inline int plane_stride(int ngw) { return ngw * 128 + 64; }

__host__ __device__ inline size_t i2d_smem(int W, int rows, int ngw) {
    // ring (reused by finish: W * 1 KB) | digit planes | per-warp row scales
    return (size_t)W * kRingBytes + (size_t)W * 3 * rows * plane_stride(ngw) + (size_t)W * kMaxRows * 4;
}

struct I2DCols {
    static constexpr bool kContiguousCols = true;
    __device__ static int thread_col(int g, int i) { return 4 * g + i; }
};

using digit::cls;
using digit::imma;
using digit::kMagic;
using digit::kMagicBits;

template <int W, int NMMA, class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(W * 32) gemv_i2d_kernel(const gemv::Params p) {
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * kCols;
    const int mb = blockIdx.z * kMaxRows;
    const int G = p.K / kGS;
    const int sk = blockIdx.y;
    const int cg0 = (int)((long long)G * sk / p.SK), cg1 = (int)((long long)G * (sk + 1) / p.SK);
    const int ng = cg1 - cg0;
    const int wg0 = cg0 + ng * warp / W, wg1 = cg0 + ng * (warp + 1) / W;
    const int nwg = wg1 - wg0;
    const int ngw_max = (ng + W - 1) / W;
    const int rows = min(kMaxRows, p.M - mb);
    const int pstride = plane_stride(ngw_max);

    char *ring = smem + warp * kRingBytes;
    char *planes = smem + W * kRingBytes + (size_t)warp * 3 * rows * pstride;
    float *rscale = reinterpret_cast<float *>(smem + W * kRingBytes + (size_t)W * 3 * rows * pstride) +
                    warp * kMaxRows;

    // ---- weight stream of this warp's groups -------------------------------------------
    // chunk x = c * 32 + lane: word row x / 8, 16-byte column chunk x % 8
    int kp_c[2], ch_c[2];
    bool ok_c[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const int x = c * 32 + lane;
        kp_c[c] = x >> 3;
        ch_c[c] = x & 7;
        ok_c[c] = n0 + 4 * ch_c[c] < p.N;  // N % 16 == 0: 4-column chunks are whole
    }
    const bool sok = lane < 4 && n0 + 8 * lane < p.N;
    int issued = 0;
    auto issue = [&]() {
        if (issued < nwg) {
            char *st = ring + (issued & (gemv::kStages - 1)) * kStageBytes;
            const int grp = wg0 + issued;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                if (ok_c[c])
                    gemv::cp_async16(st + kp_c[c] * kRowBytes + ((16 * ch_c[c]) ^ ((kp_c[c] & 1) * 64)),
                                     p.B + (size_t)(grp * 8 + kp_c[c]) * p.N + n0 + 4 * ch_c[c]);
            }
            if (sok) gemv::cp_async16(st + kWordBytes + 16 * lane, p.S + (size_t)grp * p.N + n0 + 8 * lane);
        }
        gemv::cp_async_commit();
        ++issued;
    };
#pragma unroll
    for (int i = 0; i < gemv::kStages - 1; ++i) issue();

    // ---- activation digit planes of this warp's K range ------------------------------
    pdl_wait();
    const int k0 = wg0 * kGS, klen = nwg * kGS;
    for (int m = 0; m < rows; ++m) {
        const uint16_t *arow = p.A + (size_t)(mb + m) * p.K + k0;
        // row maximum of |A| over the warp's range -> fixed-point exponent
        uint32_t mx = 0;
        for (int u = lane; u < klen / 8; u += 32) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(arow) + u);
            const uint32_t h2[8] = {v.x, v.y, v.z, v.w, 0u, 0u, 0u, 0u};
            mx = max(mx, digit::absmax_bits(h2));
        }
        mx = __reduce_max_sync(0xffffffffu, mx);
        const int e = digit::exponent_for<DT>(mx);
        if (lane == 0) rscale[m] = digit::inverse_scale<DT>(mx, e);
        // digits: one word row (16 activations) per lane iteration
        char *pl0 = planes + (size_t)(3 * m) * pstride;
        for (int w = lane; w < klen / 16; w += 32) {
            const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(arow + 16 * w));
            const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(arow + 16 * w + 8));
            const uint32_t h2[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            uint32_t d0[4], d1[4], d2[4];
            digit::word_digits<DT>(h2, e, d0, d1, d2);
            *reinterpret_cast<uint4 *>(pl0 + 16 * w) = make_uint4(d0[0], d0[1], d0[2], d0[3]);
            *reinterpret_cast<uint4 *>(pl0 + pstride + 16 * w) = make_uint4(d1[0], d1[1], d1[2], d1[3]);
            *reinterpret_cast<uint4 *>(pl0 + 2 * pstride + 16 * w) = make_uint4(d2[0], d2[1], d2[2], d2[3]);
        }
    }
    __syncwarp();

    // B operand source of this lane's n-columns: n = 8 tt + g; n = 0 -> ones, n = 1 + 3m + d
    // -> plane 3m + d, beyond -> zero
    const char *bsrc[NMMA];
    uint32_t bconst[NMMA];
#pragma unroll
    for (int tt = 0; tt < NMMA; ++tt) {
        const int n = 8 * tt + g;
        bsrc[tt] = nullptr;
        bconst[tt] = n == 0 ? 0x01010101u : 0u;
        if (n >= 1 && n <= 3 * rows) bsrc[tt] = planes + (size_t)(n - 1) * pstride;
    }

    float acc[2][NMMA][4];
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int tt = 0; tt < NMMA; ++tt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[b][tt][c] = 0.0f;

    const int swz = (t & 1) * 64;  // word rows t and 4 + t have the same parity
    for (int i = 0; i < nwg; ++i) {
        gemv::cp_async_wait<gemv::kStages - 2>();
        __syncwarp();  // the lanes' copies of this stage are visible to the whole warp
        const char *st = ring + (i & (gemv::kStages - 1)) * kStageBytes;
        uint2 wa[2], wb[2];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            wa[b] = *reinterpret_cast<const uint2 *>(st + t * kRowBytes + ((64 * b + 8 * g) ^ swz));
            wb[b] = *reinterpret_cast<const uint2 *>(st + (4 + t) * kRowBytes + ((64 * b + 8 * g) ^ swz));
        }
        uint4 ba[NMMA], bb[NMMA];
#pragma unroll
        for (int tt = 0; tt < NMMA; ++tt) {
            if (bsrc[tt]) {
                ba[tt] = *reinterpret_cast<const uint4 *>(bsrc[tt] + (8 * i + t) * 16);
                bb[tt] = *reinterpret_cast<const uint4 *>(bsrc[tt] + (8 * i + 4 + t) * 16);
            } else {
                ba[tt] = make_uint4(bconst[tt], bconst[tt], bconst[tt], bconst[tt]);
                bb[tt] = ba[tt];
            }
        }
        int32_t d[2][NMMA][4];
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int tt = 0; tt < NMMA; ++tt)
#pragma unroll
                for (int c = 0; c < 4; ++c) d[b][tt][c] = (int32_t)kMagicBits;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const uint32_t a0 = cls(wa[b].x, j), a1 = cls(wa[b].y, j), a2 = cls(wb[b].x, j),
                               a3 = cls(wb[b].y, j);
#pragma unroll
                for (int tt = 0; tt < NMMA; ++tt) {
                    const uint32_t b0 = j == 0 ? ba[tt].x : j == 1 ? ba[tt].y : j == 2 ? ba[tt].z : ba[tt].w;
                    const uint32_t b1 = j == 0 ? bb[tt].x : j == 1 ? bb[tt].y : j == 2 ? bb[tt].z : bb[tt].w;
                    imma(d[b][tt], a0, a1, a2, a3, b0, b1);
                }
            }
        }
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const uint32_t s2 = *reinterpret_cast<const uint32_t *>(st + kWordBytes + (16 * b + 2 * g) * 2);
            const float s_lo = DT::tof((uint16_t)(s2 & 0xFFFFu)), s_hi = DT::tof((uint16_t)(s2 >> 16));
#pragma unroll
            for (int tt = 0; tt < NMMA; ++tt) {
                acc[b][tt][0] = fmaf(__int_as_float(d[b][tt][0]) - kMagic, s_lo, acc[b][tt][0]);
                acc[b][tt][1] = fmaf(__int_as_float(d[b][tt][1]) - kMagic, s_lo, acc[b][tt][1]);
                acc[b][tt][2] = fmaf(__int_as_float(d[b][tt][2]) - kMagic, s_hi, acc[b][tt][2]);
                acc[b][tt][3] = fmaf(__int_as_float(d[b][tt][3]) - kMagic, s_hi, acc[b][tt][3]);
            }
        }
        __syncwarp();  // every lane is done with this stage before it is refilled
        issue();
    }
    gemv::cp_async_wait<0>();
    pdl_launch_dependents();
    __syncwarp();

    // ---- planes -> rows: acc[b][tt][c] = (column 16b + 2g + (c >> 1), n = 8tt + 2t + (c & 1))
    float(*tb)[kCols] = reinterpret_cast<float(*)[kCols]>(ring);  // [8 NMMA][32], this warp's ring
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int tt = 0; tt < NMMA; ++tt)
#pragma unroll
            for (int c = 0; c < 4; ++c) tb[8 * tt + 2 * t + (c & 1)][16 * b + 2 * g + (c >> 1)] = acc[b][tt][c];
    __syncwarp();
    float v[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int m = 2 * t + h;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float r = 0.0f;
            if (m < rows) {
                const int col = 4 * g + i;
                const float s = tb[1 + 3 * m][col] + 256.0f * tb[2 + 3 * m][col];
                r = (s + (65536.0f * tb[3 + 3 * m][col] - 4194304.0f * tb[0][col])) * rscale[m];
            }
            v[4 * h + i] = r;
        }
    }
    __syncthreads();  // the rings are reused for the reduction
    gemv::finish<I2DCols, W, DT, POSTOP, OUT_F32>(p, smem, v, n0 + 4 * g < p.N);
    if (p.world > 0) gemv::peer_complete(p, p.err, OUT_F32 ? 4 : 2);
}

template <int W, int NMMA, class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_w(const GemvArgs &a) {
    gemv::Params p = gemv::gemv_params_impl(a);
    const int G = a.K / kGS;
    const int ng = (G + a.SK - 1) / a.SK;
    const int ngw = (ng + W - 1) / W;
    const int rows = a.M < kMaxRows ? a.M : kMaxRows;
    const size_t smem = i2d_smem(W, rows, ngw);
    auto kern = gemv_i2d_kernel<W, NMMA, DT, POSTOP, OUT_F32>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((a.N + kCols - 1) / kCols, a.SK, (a.M + kMaxRows - 1) / kMaxRows);
    return launch_kernel_cluster(kern, grid, dim3(W * 32), smem, a.stream, dim3(1, a.cluster ? a.SK : 1, 1), p);
}

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a) {
    const int rows = a.M < kMaxRows ? a.M : kMaxRows;
    const bool two = nmma_for(rows) > 1;
    if (a.warps >= 16) return two ? launch_w<16, 2, DT, POSTOP, OUT_F32>(a) : launch_w<16, 1, DT, POSTOP, OUT_F32>(a);
    if (a.warps >= 8) return two ? launch_w<8, 2, DT, POSTOP, OUT_F32>(a) : launch_w<8, 1, DT, POSTOP, OUT_F32>(a);
    return two ? launch_w<4, 2, DT, POSTOP, OUT_F32>(a) : launch_w<4, 1, DT, POSTOP, OUT_F32>(a);
}

}  // namespace

size_t int2_gemv_d_smem(int M, int K, int SK, int warps) {
    const int G = K / kGS;
    const int ng = (G + SK - 1) / SK;
    const int W = warps >= 16 ? 16 : warps >= 8 ? 8 : 4;
    return i2d_smem(W, M < kMaxRows ? M : kMaxRows, (ng + W - 1) / W);
}

cudaError_t int2_gemv_d_launch(const GemvArgs &a) {
    if (a.M > kMaxRows) return cudaErrorInvalidValue;  // the planner sends larger M elsewhere
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_t<DT, decltype(po)::value, decltype(of)::value>(a);
    });
}

}  // namespace ternocl
