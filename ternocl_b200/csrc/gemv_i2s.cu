// Stream-K int2 decode GEMV on integer MMAs (M <= 4): the default implementation of
// int2_fp16_upcvt_gemm (int2_fp16_upcvt.cl:193-290) when a workspace is available.
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(B[k,n]) ))
//
// The arithmetic is the integer-MMA GEMV's (gemv_i2d.cu, digit_common.cuh): one
// shift-and-mask per four weights gives int8 64 * code, the activations become three
// exact unsigned digit planes of a fixed-point integer plus a plane of ones, and
// mma.sync m16n8k32 s8 x u8 gives exact int32 dots per 128-row group, scaled by S in
// fp32.  What differs is how the weight stream is spread over the GPU.
//
// Work split.  A unit is one 128-row group of one 32-column strip (1 KB of packed
// weights + 64 B of scales); units are ordered strip by strip, K fastest.  The grid is
// one wave of at most one CTA per SM, and warp w of the PW warps takes the contiguous
// units [U w / PW, U (w+1) / PW): every SM streams the same number of bytes, whatever
// the shape (a grid of whole strips or K slices cannot divide evenly over 148 SMs).  A
// CTA is small (8 warps, about 100 KB of shared memory at M = 1), so that with
// programmatic dependent launch the next GEMV of the stream fits beside it on every
// SM and starts streaming its weights while this one drains.
//
// Memory pipeline.  Each lane copies with cp.async exactly the bytes it later reads:
// per unit two 16-byte chunks (word rows t and 4+t of its columns 4gl..4gl+3), laid
// out so that a warp's reads are contiguous 512-byte runs; lanes with t == 0 also copy
// the 8 bytes of scales of their four columns.  A warp's ring holds D units.
//
// Activations.  The CTA turns all of A (M <= 4 rows) into digit planes once, in the
// MMA's K order, with one fixed-point exponent per row and 128-row group (from max |A|
// over the group), so every element within 2^11 of its group's maximum is exact.  The
// group's exponent is folded into its scale (S * 2^-e / 64, an exact power-of-two
// factor), which needs a plane of ones per row: MMA column 4m is row m's ones, 4m + 1..3
// its digit planes -- 8 columns (one MMA per class) for M <= 2, 16 for M <= 4.
//
// Reduction.  A warp keeps fp32 accumulators per (column, plane) while it stays in
// one strip.  A strip it covers whole is finished and stored directly.  A strip split
// between consecutive warps: each piece writes its 32 x M partial to the workspace
// (two slots per warp: its first and its last strip), and the warp that completes the
// strip's arrival counter sums the pieces in warp order -- a fixed order, so the result
// is bitwise reproducible -- applies the epilogue, stores and resets the counter.
#include <cuda_runtime.h>

#include "digit_common.cuh"
#include "gemv_common.cuh"
#include "launch.h"

namespace ternocl {

namespace {

constexpr int kCols = 32;         // columns of a strip
constexpr int kUnitWords = 1024;  // packed weight bytes of a unit (8 word rows x 32 columns)
constexpr int kStageBytes = kUnitWords + 64;
constexpr int kMaxRows = 4;

struct I2SParams {
    const uint16_t *A;
    const uint32_t *B;
    const uint16_t *S;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K;
    float *part;    // [PW][2][M][32] fp32 partials of split strips
    unsigned *cnt;  // [strips] arrival counters (zero between calls)
    // column-sharded mode (world > 0): these are columns [n_off, n_off + N) of an output of
    // N_out columns; each finished strip is stored into this rank's C_peer[rank] (Other and
    // Bias are full width), then gemv::peer_complete copies the slice to the other ranks
    // and runs their flag handshake
    int world, rank, n_off, N_out;
    unsigned epoch;
    unsigned long long peer_timeout_ns;
    unsigned *done_cnt;
    unsigned *err;
    void *C_peer[gemv::kMaxPeers];
    unsigned *flag_peer[gemv::kMaxPeers];
};

__host__ __device__ constexpr int nmma_for(int rows) { return (4 * rows + 7) / 8; }

// bytes of one digit plane of K activations: K/16 word rows x 16 bytes, + 64 to stagger banks
__host__ __device__ inline int plane_stride(int K) { return K + 64; }

__host__ __device__ inline size_t i2s_smem(int W, int D, int rows, int K) {
    const int nmma = nmma_for(rows);
    return (size_t)W * D * kStageBytes                      // rings
           + (size_t)3 * rows * plane_stride(K)              // digit planes
           + (size_t)W * 8 * nmma * 33 * sizeof(float)       // per-warp transpose tile
           + (size_t)rows * (K / kGS) * 8;                    // per (row, group): exponent, 2^-e / 64
}

// Balanced split of U units over PW warps in 32-bit arithmetic (U < 2^31, PW <= U):
// warp w holds q + (w < r) units starting at w q + min(w, r), U = q PW + r.
struct UnitSplit {
    int q, r;
    __device__ __forceinline__ UnitSplit(int U, int PW) : q(U / PW), r(U - (U / PW) * PW) {}
    __device__ __forceinline__ int start(int w) const { return w * q + min(w, r); }
    __device__ __forceinline__ int warp_of(int u) const {
        const int b = r * (q + 1);
        return u < b ? u / (q + 1) : r + (u - b) / q;
    }
};

using digit::cls;
using digit::imma;
using digit::kMagic;
using digit::kMagicBits;

template <int W, int D, int NMMA, class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(W * 32, 2) gemv_i2s_kernel(const I2SParams p) {
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int gl = lane >> 2, t = lane & 3;
    const int G = p.K / kGS;
    const int strips = (p.N + kCols - 1) / kCols;
    const int U = strips * G;
    const int PW = gridDim.x * W;
    const int wid = blockIdx.x * W + warp;
    const UnitSplit split(U, PW);
    const int u0 = split.start(wid), u1 = split.start(wid + 1);
    const int rows = p.M;
    const int pstride = plane_stride(p.K);

    char *ring = smem + (size_t)warp * D * kStageBytes;
    char *planes = smem + (size_t)W * D * kStageBytes;
    float *tb = reinterpret_cast<float *>(planes + (size_t)3 * rows * pstride) + warp * (8 * NMMA * 33);
    // [rows][G]: the fixed-point exponent of each group and its factor 2^-e / 64
    int *gexp = reinterpret_cast<int *>(planes + (size_t)3 * rows * pstride +
                                        (size_t)W * 8 * NMMA * 33 * sizeof(float));
    float *gfac = reinterpret_cast<float *>(gexp + rows * G);

    // ---- weight stream: unit u -> stage (u - u0) mod D -------------------------------
    int ld_u = u0;
    int ld_s = u0 / G, ld_g = u0 - ld_s * G, ld_stage = 0;
    auto issue = [&]() {
        if (ld_u < u1) {
            char *st = ring + ld_stage * kStageBytes;
            const int col = ld_s * kCols + 4 * gl;
            if (col < p.N) {  // N % 16 == 0: a lane's four columns exist together
                const uint32_t *src = p.B + (size_t)(ld_g * 8 + t) * p.N + col;
                gemv::cp_async16(st + lane * 16, src);
                gemv::cp_async16(st + 512 + lane * 16, src + (size_t)4 * p.N);
                if (t == 0) gemv::cp_async8(st + kUnitWords + gl * 8, p.S + (size_t)ld_g * p.N + col);
            }
            if (++ld_g == G) {
                ld_g = 0;
                ++ld_s;
            }
            if (++ld_stage == D) ld_stage = 0;
        }
        gemv::cp_async_commit();
        ++ld_u;
    };
#pragma unroll
    for (int i = 0; i < D - 1; ++i) issue();
    // the rest of this warp's units into L2: per unit its 8 word rows and its scale row
    for (int ub = u0 + D - 1; ub < u1; ub += 4) {
        const int u = ub + (lane >> 3);
        if (u < u1) {
            const int s = u / G, g = u - s * G, col = s * kCols;
            gemv::prefetch_l2(p.B + (size_t)(g * 8 + (lane & 7)) * p.N + col);
            if ((lane & 7) == 0) gemv::prefetch_l2(p.S + (size_t)g * p.N + col);
        }
    }
    // The weights never depend on the previous kernel: their first D - 1 units are in
    // flight already.  Let the next kernel of the stream be scheduled (its own
    // griddepcontrol.wait still covers this whole grid), then wait for ours.
    pdl_launch_dependents();
    pdl_wait();

    // ---- activations: per-(row, group) exponents, then the digit planes -------------
    // 16 consecutive threads cover a group's 128 activations (16 x 16 bytes)
    for (int m = 0; m < rows; ++m) {
        const uint4 *arow = reinterpret_cast<const uint4 *>(p.A + (size_t)m * p.K);
        for (int u0g = 0; u0g < p.K / 8; u0g += W * 32) {  // uniform trip count: every lane shuffles
            const int u = u0g + tid;  // K / 8 is a multiple of 16: a half-warp is all in or all out
            uint32_t mx = 0;
            if (u < p.K / 8) {
                const uint4 v = __ldg(arow + u);
                const uint32_t h2[8] = {v.x, v.y, v.z, v.w, 0u, 0u, 0u, 0u};
                mx = digit::absmax_bits(h2);
            }
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o, 16));
            if (u < p.K / 8) {
                if ((lane & 15) == 0) {
                    const int e = digit::exponent_for<DT>(mx);
                    gexp[m * G + u / 16] = e;
                    gfac[m * G + u / 16] = digit::inverse_scale<DT>(mx, e);
                }
            }
        }
    }
    __syncthreads();
    for (int m = 0; m < rows; ++m) {
        const uint16_t *arow = p.A + (size_t)m * p.K;
        char *pl = planes + (size_t)(3 * m) * pstride;
        for (int wr = tid; wr < p.K / 16; wr += W * 32) {
            const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(arow + 16 * wr));
            const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(arow + 16 * wr + 8));
            const uint32_t h2[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            uint32_t d0[4], d1[4], d2[4];
            digit::word_digits<DT>(h2, gexp[m * G + wr / 8], d0, d1, d2);
            *reinterpret_cast<uint4 *>(pl + 16 * wr) = make_uint4(d0[0], d0[1], d0[2], d0[3]);
            *reinterpret_cast<uint4 *>(pl + pstride + 16 * wr) = make_uint4(d1[0], d1[1], d1[2], d1[3]);
            *reinterpret_cast<uint4 *>(pl + 2 * pstride + 16 * wr) = make_uint4(d2[0], d2[1], d2[2], d2[3]);
        }
    }
    __syncthreads();

    // B operand of this lane's MMA column n = 8 tt + gl: row n / 4; n % 4 == 0 -> ones,
    // n % 4 = 1 + d -> that row's plane d; rows >= M -> zero.  The accumulators of
    // column pair (8 tt + 2t, 8 tt + 2t + 1) belong to row 2 tt + t / 2 (fac[tt]).
    const char *bsrc[NMMA];
    uint32_t bconst[NMMA];
    const float *fac[NMMA];
#pragma unroll
    for (int tt = 0; tt < NMMA; ++tt) {
        const int n = 8 * tt + gl, m = n >> 2, d = n & 3;
        bsrc[tt] = nullptr;
        bconst[tt] = (m < rows && d == 0) ? 0x01010101u : 0u;
        if (m < rows && d > 0) bsrc[tt] = planes + (size_t)(3 * m + d - 1) * pstride + 16 * t;
        const int mr = 2 * tt + (t >> 1);
        fac[tt] = gfac + (mr < rows ? mr : 0) * G;
    }

    float acc[2][NMMA][4];
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int tt = 0; tt < NMMA; ++tt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[b][tt][c] = 0.0f;

    // ---- finish a strip: planes -> values, then store or hand over as a partial -------
    const int first_strip = u0 / G;
    auto flush = [&](int cs, bool whole) {
        __syncwarp();
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int tt = 0; tt < NMMA; ++tt)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    tb[(8 * tt + 2 * t + (c & 1)) * 33 + 4 * gl + 2 * b + (c >> 1)] = acc[b][tt][c];
                    acc[b][tt][c] = 0.0f;
                }
        __syncwarp();
        const int col = cs * kCols + lane;
        const bool colok = col < p.N;
        float v[kMaxRows];
#pragma unroll
        for (int m = 0; m < kMaxRows; ++m) {
            v[m] = 0.0f;
            if (m < rows) {
                const float *c4 = tb + 4 * m * 33 + lane;
                v[m] = (c4[33] + 256.0f * c4[66]) + (65536.0f * c4[99] - 4194304.0f * c4[0]);
            }
        }
        if (!whole) {
            const int slot = cs == first_strip ? 0 : 1;
            float *mine = p.part + ((size_t)(wid * 2 + slot) * rows) * kCols + lane;
#pragma unroll
            for (int m = 0; m < kMaxRows; ++m)
                if (m < rows) __stcg(mine + m * kCols, v[m]);
            __threadfence();
            __syncwarp();
            const int su = cs * G;
            const int wf = split.warp_of(su), wl = split.warp_of(su + G - 1);
            unsigned last = 0;
            if (lane == 0) last = atomicAdd(p.cnt + cs, 1u) == (unsigned)(wl - wf) ? 1u : 0u;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) return;
            __threadfence();
#pragma unroll
            for (int m = 0; m < kMaxRows; ++m) v[m] = 0.0f;
            for (int w2 = wf; w2 <= wl; ++w2) {
                const int slot2 = split.start(w2) >= su ? 0 : 1;  // strip cs is w2's first or last
                const float *pp = p.part + ((size_t)(w2 * 2 + slot2) * rows) * kCols + lane;
#pragma unroll
                for (int m = 0; m < kMaxRows; ++m)
                    if (m < rows) v[m] += __ldcg(pp + m * kCols);
            }
            if (lane == 0) p.cnt[cs] = 0u;  // ready for the next call
        }
        if (colok) {
            if (p.world > 0) {  // column-sharded: this rank's columns into its own copy of C
#pragma unroll
                for (int m = 0; m < kMaxRows; ++m)
                    if (m < rows)
                        epi_store<DT, POSTOP, OUT_F32>(p.C_peer[p.rank], p.Other, p.Bias, p.N_out, m, p.n_off + col,
                                                       v[m]);
            } else {
#pragma unroll
                for (int m = 0; m < kMaxRows; ++m)
                    if (m < rows) epi_store<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, m, col, v[m]);
            }
        }
    };

    // ---- main loop over this warp's units ---------------------------------------------
    int cs = first_strip, cg = u0 - first_strip * G, seg_g0 = cg, stage = 0;
    for (int u = u0; u < u1; ++u) {
        gemv::cp_async_wait<D - 2>();
        __syncwarp();  // the scale copies of lanes t == 0 are visible to the whole warp
        const char *st = ring + stage * kStageBytes;
        const uint4 w0 = *reinterpret_cast<const uint4 *>(st + lane * 16);
        const uint4 w1 = *reinterpret_cast<const uint4 *>(st + 512 + lane * 16);
        const uint2 sc = *reinterpret_cast<const uint2 *>(st + kUnitWords + gl * 8);
        uint4 ba[NMMA], bb[NMMA];
#pragma unroll
        for (int tt = 0; tt < NMMA; ++tt) {
            if (bsrc[tt]) {
                ba[tt] = *reinterpret_cast<const uint4 *>(bsrc[tt] + cg * 128);
                bb[tt] = *reinterpret_cast<const uint4 *>(bsrc[tt] + cg * 128 + 64);
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
                const uint32_t x0 = b ? w0.z : w0.x, x1 = b ? w0.w : w0.y;
                const uint32_t x2 = b ? w1.z : w1.x, x3 = b ? w1.w : w1.y;
                const uint32_t a0 = cls(x0, j), a1 = cls(x1, j), a2 = cls(x2, j), a3 = cls(x3, j);
#pragma unroll
                for (int tt = 0; tt < NMMA; ++tt) {
                    const uint32_t b0 = j == 0 ? ba[tt].x : j == 1 ? ba[tt].y : j == 2 ? ba[tt].z : ba[tt].w;
                    const uint32_t b1 = j == 0 ? bb[tt].x : j == 1 ? bb[tt].y : j == 2 ? bb[tt].z : bb[tt].w;
                    imma(d[b][tt], a0, a1, a2, a3, b0, b1);
                }
            }
        }
        float f[NMMA];
#pragma unroll
        for (int tt = 0; tt < NMMA; ++tt) f[tt] = fac[tt][cg];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const uint32_t s2 = b ? sc.y : sc.x;
            const float s_lo0 = DT::tof((uint16_t)(s2 & 0xFFFFu)), s_hi0 = DT::tof((uint16_t)(s2 >> 16));
#pragma unroll
            for (int tt = 0; tt < NMMA; ++tt) {
                const float s_lo = s_lo0 * f[tt], s_hi = s_hi0 * f[tt];
                acc[b][tt][0] = fmaf(__int_as_float(d[b][tt][0]) - kMagic, s_lo, acc[b][tt][0]);
                acc[b][tt][1] = fmaf(__int_as_float(d[b][tt][1]) - kMagic, s_lo, acc[b][tt][1]);
                acc[b][tt][2] = fmaf(__int_as_float(d[b][tt][2]) - kMagic, s_hi, acc[b][tt][2]);
                acc[b][tt][3] = fmaf(__int_as_float(d[b][tt][3]) - kMagic, s_hi, acc[b][tt][3]);
            }
        }
        // refill the stage read in the previous iteration (every lane passed this
        // iteration's __syncwarp after its reads of it)
        issue();
        if (++stage == D) stage = 0;
        if (cg == G - 1 || u == u1 - 1) {
            flush(cs, seg_g0 == 0 && cg == G - 1);
            ++cs;
            cg = 0;
            seg_g0 = 0;
        } else {
            ++cg;
        }
    }
    if (p.world > 0) gemv::peer_complete(p, p.err, OUT_F32 ? 4 : 2);
}

template <int W, int D, int NMMA, class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_i2s(const GemvArgs &a, int ctas) {
    I2SParams p;
    p.A = (const uint16_t *)a.A;
    p.B = a.B;
    p.S = (const uint16_t *)a.S;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.cnt = a.ws_cnt;
    p.part = a.ws_part;
    p.world = a.world;
    p.rank = a.rank;
    p.n_off = a.n_off;
    p.N_out = a.N_out;
    p.epoch = a.epoch;
    p.peer_timeout_ns = (unsigned long long)options().peer_timeout_ms * 1000000ull;
    p.done_cnt = a.done_cnt;
    p.err = a.err;
    for (int r = 0; r < gemv::kMaxPeers; ++r) {
        p.C_peer[r] = r < a.world ? a.C_peer[r] : nullptr;
        p.flag_peer[r] = r < a.world ? a.flag_peer[r] : nullptr;
    }
    const size_t smem = i2s_smem(W, D, a.M, a.K);
    auto kern = gemv_i2s_kernel<W, D, NMMA, DT, POSTOP, OUT_F32>;
    cudaError_t e = ensure_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3(ctas), dim3(W * 32), smem, a.stream, p);
}

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_i2s_t(const GemvArgs &a, int ctas, int depth) {
    if (a.M <= 2) {
        if (depth >= 8) return launch_i2s<8, 8, 1, DT, POSTOP, OUT_F32>(a, ctas);
        if (depth >= 6) return launch_i2s<8, 6, 1, DT, POSTOP, OUT_F32>(a, ctas);
        return launch_i2s<8, 4, 1, DT, POSTOP, OUT_F32>(a, ctas);
    }
    if (depth >= 6) return launch_i2s<8, 6, 2, DT, POSTOP, OUT_F32>(a, ctas);
    return launch_i2s<8, 4, 2, DT, POSTOP, OUT_F32>(a, ctas);
}

}  // namespace

constexpr int kI2SWarps = 8;

size_t int2_gemv_s_smem(int M, int K, int depth) { return i2s_smem(kI2SWarps, depth, M, K); }

int int2_gemv_s_ctas(int M, int N, int K, int sms) {
    if (M < 1 || M > kMaxRows) return 0;
    const long long U = (long long)((N + kCols - 1) / kCols) * (K / kGS);
    if (U >= (1ll << 31)) return 0;  // the kernel splits units in 32-bit arithmetic
    long long ctas = U / kI2SWarps;  // every warp gets at least one unit
    if (ctas > sms) ctas = sms;
    return (int)ctas;
}

size_t int2_gemv_s_cnt_bytes(int N) { return ((size_t)((N + kCols - 1) / kCols) * 4 + 255) / 256 * 256; }

size_t int2_gemv_s_workspace(int M, int N, int ctas) {
    return int2_gemv_s_cnt_bytes(N) + (size_t)ctas * kI2SWarps * 2 * M * kCols * sizeof(float);
}

cudaError_t int2_gemv_s_launch(const GemvArgs &a, int ctas, int depth) {
    if (a.M > kMaxRows || ctas < 1 || !a.ws_cnt || !a.ws_part) return cudaErrorInvalidValue;
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return launch_i2s_t<DT, decltype(po)::value, decltype(of)::value>(a, ctas, depth);
    });
}

}  // namespace ternocl
