// int2 MoE decode GEMVs, replace int2_moe.cl's kernels (int2_moe/int2_moe.cl:63-174):
//
//   gate_up   H[g, n] = DT(silu(x_t . gate_e[:, n]) * (x_t . up_e[:, n])),  x_t = X[g / topk]
//   down      Y[g, n] = RW[g] * (H[g] . down_e[:, n])                        (fp32)
//   reduce    O[t, n] = DT(sum_j Y[t*topk + j, n])                           (j ascending)
//   down_sum  O[t, n] = DT(sum_j RW[g] * (H[g] . down_e[:, n])),  g = t*topk + j
//
// with e = ids[g] (row g of the routed token-expert pairs, g = t*topk + j) and the int2
// weights of every expert stacked: B [E, K/16, N], S [E, K/128, N].  The dots are the
// integer-MMA GEMV of gemv_i2d.cu (int8 weights, exact fixed-point activation digits,
// mma.sync m16n8k32 s8 x u8, per-group float partials scaled by S) at one activation row
// per CTA, with the weight matrix chosen per row (gate_up, down) or per K segment
// (down_sum, whose K runs over the topk experts of the token: H viewed as [T, topk*K]).
// gate_up walks the gate and the up matrix as one range of 2 K/128 groups with two sets
// of accumulators, so both dots of a column meet in the CTA for the SwiGLU.  No split-K:
// a CTA owns 32 columns of one row over the whole K, its W warps split the groups and
// reduce in warp order through shared memory (deterministic).  An expert id outside
// [0, E) contributes zero and sets bit 1 of the device error word.
#include <cuda_runtime.h>

#include "common.cuh"
#include "digit_common.cuh"
#include "gemv_common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {

namespace {

constexpr int kCols = 32;
constexpr int kRowBytes = kCols * 4;
constexpr int kWordBytes = 8 * kRowBytes;
constexpr int kScaleBytes = kCols * 2;
constexpr int kStageBytes = kWordBytes + kScaleBytes;
constexpr int kRingBytes = gemv::kStages * kStageBytes;

enum Mode { kGateUp = 0, kDown = 1, kDownSum = 2 };

struct MParams {
    const int *ids;
    const uint16_t *A;                 // X [T, K] (gate_up) or H [G, K] (down, down_sum)
    const uint32_t *B0, *B1;           // gate / up (gate_up) or down
    const uint16_t *S0, *S1;
    const uint16_t *RW;                // [G]
    void *out;                         // H DT [G, N] | Y fp32 [G, N] | O DT [T, N]
    int N, K, G, topk, E;              // K, G = K / 128 of one expert matrix
};

__host__ __device__ inline int plane_stride(int ngw) { return ngw * 128 + 64; }

template <int MODE>
__host__ __device__ constexpr int mats() { return MODE == kGateUp ? 2 : 1; }
template <int MODE>
__host__ __device__ inline int total_groups(int G, int topk) {
    return MODE == kGateUp ? 2 * G : MODE == kDown ? G : topk * G;
}

__host__ __device__ inline size_t md_smem(int W, int ngw, int nmats) {
    return (size_t)W * kRingBytes + (size_t)W * 3 * plane_stride(ngw) + (size_t)W * 4 + (size_t)W * nmats * kCols * 4;
}

template <int W, int MODE, class DT>
__global__ void __launch_bounds__(W * 32) moe_decode_kernel(const MParams p) {
    constexpr int kMats = mats<MODE>();
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * kCols;
    const int z = blockIdx.y;  // routed row (gate_up, down) or token (down_sum)
    const int ng = total_groups<MODE>(p.G, p.topk);
    const int wg0 = ng * warp / W, wg1 = ng * (warp + 1) / W, nwg = wg1 - wg0;
    const int ngw_max = (ng + W - 1) / W;
    const int pstride = plane_stride(ngw_max);
    char *ring = smem + warp * kRingBytes;
    char *planes = smem + W * kRingBytes + (size_t)warp * 3 * pstride;
    float *rscale = reinterpret_cast<float *>(smem + W * kRingBytes + (size_t)W * 3 * pstride);
    float *red = rscale + W;  // [W][kMats][32]

    // the router's ids (and H) come from the previous kernels
    pdl_wait();

    // group -> (matrix, expert row of ids, local group)
    auto locate = [&](int grp, int &mat, int &gid, int &lg) {
        if (MODE == kGateUp) {
            mat = grp >= p.G;
            lg = grp - (mat ? p.G : 0);
            gid = z;
        } else if (MODE == kDown) {
            mat = 0;
            lg = grp;
            gid = z;
        } else {
            mat = 0;
            const int j = grp / p.G;
            lg = grp - j * p.G;
            gid = z * p.topk + j;
        }
    };
    auto expert = [&](int gid, bool &ok) {
        const int e = p.ids[gid];
        ok = e >= 0 && e < p.E;
        return ok ? e : 0;
    };
    // activations of group grp
    auto act = [&](int grp) -> const uint16_t * {
        if (MODE == kGateUp) return p.A + (size_t)(z / p.topk) * p.K + (size_t)(grp % p.G) * kGS;
        if (MODE == kDown) return p.A + (size_t)z * p.K + (size_t)grp * kGS;
        return p.A + (size_t)z * p.topk * p.K + (size_t)grp * kGS;
    };

    // ---- weight stream of this warp's groups (as gemv_i2d.cu) ----
    int kp_c[2], ch_c[2];
    bool ok_c[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const int x = c * 32 + lane;
        kp_c[c] = x >> 3;
        ch_c[c] = x & 7;
        ok_c[c] = n0 + 4 * ch_c[c] < p.N;
    }
    const bool sok = lane < 4 && n0 + 8 * lane < p.N;
    int issued = 0;
    auto issue = [&]() {
        if (issued < nwg) {
            char *st = ring + (issued & (gemv::kStages - 1)) * kStageBytes;
            int mat, gid, lg;
            locate(wg0 + issued, mat, gid, lg);
            bool ok;
            const size_t e = (size_t)expert(gid, ok);
            const uint32_t *B = (mat ? p.B1 : p.B0) + e * (size_t)(p.K / 16) * p.N;
            const uint16_t *S = (mat ? p.S1 : p.S0) + e * (size_t)p.G * p.N;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                if (ok_c[c])
                    gemv::cp_async16(st + kp_c[c] * kRowBytes + ((16 * ch_c[c]) ^ ((kp_c[c] & 1) * 64)),
                                     B + (size_t)(lg * 8 + kp_c[c]) * p.N + n0 + 4 * ch_c[c]);
            }
            if (sok) gemv::cp_async16(st + kWordBytes + 16 * lane, S + (size_t)lg * p.N + n0 + 8 * lane);
        }
        gemv::cp_async_commit();
        ++issued;
    };
#pragma unroll
    for (int i = 0; i < gemv::kStages - 1; ++i) issue();

    // ---- activation digits of the warp's groups (one exponent per warp) ----
    {
        uint32_t mx = 0;
        for (int u = lane; u < nwg * 8; u += 32) {  // 8 word rows of 16 activations per group
            const uint4 *src = reinterpret_cast<const uint4 *>(act(wg0 + u / 8) + 16 * (u % 8));
            const uint4 lo = __ldg(src), hi = __ldg(src + 1);
            const uint32_t h2[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            mx = max(mx, digit::absmax_bits(h2));
        }
        mx = __reduce_max_sync(0xffffffffu, mx);
        const int e = digit::exponent_for<DT>(mx);
        if (lane == 0) rscale[warp] = digit::inverse_scale<DT>(mx, e);
        for (int u = lane; u < nwg * 8; u += 32) {
            const uint4 *src = reinterpret_cast<const uint4 *>(act(wg0 + u / 8) + 16 * (u % 8));
            const uint4 lo = __ldg(src), hi = __ldg(src + 1);
            const uint32_t h2[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
            uint32_t d0[4], d1[4], d2[4];
            digit::word_digits<DT>(h2, e, d0, d1, d2);
            *reinterpret_cast<uint4 *>(planes + 16 * u) = make_uint4(d0[0], d0[1], d0[2], d0[3]);
            *reinterpret_cast<uint4 *>(planes + pstride + 16 * u) = make_uint4(d1[0], d1[1], d1[2], d1[3]);
            *reinterpret_cast<uint4 *>(planes + 2 * pstride + 16 * u) = make_uint4(d2[0], d2[1], d2[2], d2[3]);
        }
    }
    __syncwarp();

    // B operand of this lane's n-column: 0 ones, 1..3 the digit planes, beyond zero
    const char *bsrc = g >= 1 && g <= 3 ? planes + (size_t)(g - 1) * pstride : nullptr;
    const uint32_t bconst = g == 0 ? 0x01010101u : 0u;

    float acc[kMats][2][4];
#pragma unroll
    for (int m = 0; m < kMats; ++m)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[m][b][c] = 0.0f;

    bool bad_id = false;
    const int swz = (t & 1) * 64;
    for (int i = 0; i < nwg; ++i) {
        gemv::cp_async_wait<gemv::kStages - 2>();
        __syncwarp();
        const char *st = ring + (i & (gemv::kStages - 1)) * kStageBytes;
        int mat, gid, lg;
        locate(wg0 + i, mat, gid, lg);
        bool ok;
        expert(gid, ok);
        bad_id |= !ok;
        // per-group factor: the routing weight inside down_sum, 0 for a bad expert id
        float gf = ok ? 1.0f : 0.0f;
        if (MODE == kDownSum && ok) gf = DT::tof(p.RW[gid]);
        uint2 wa[2], wb[2];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            wa[b] = *reinterpret_cast<const uint2 *>(st + t * kRowBytes + ((64 * b + 8 * g) ^ swz));
            wb[b] = *reinterpret_cast<const uint2 *>(st + (4 + t) * kRowBytes + ((64 * b + 8 * g) ^ swz));
        }
        uint4 ba, bb;
        if (bsrc) {
            ba = *reinterpret_cast<const uint4 *>(bsrc + (8 * i + t) * 16);
            bb = *reinterpret_cast<const uint4 *>(bsrc + (8 * i + 4 + t) * 16);
        } else {
            ba = make_uint4(bconst, bconst, bconst, bconst);
            bb = ba;
        }
        const uint32_t bA[4] = {ba.x, ba.y, ba.z, ba.w}, bB[4] = {bb.x, bb.y, bb.z, bb.w};
        int32_t d[2][4];
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) d[b][c] = (int32_t)digit::kMagicBits;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int b = 0; b < 2; ++b)
                digit::imma(d[b], digit::cls(wa[b].x, j), digit::cls(wa[b].y, j), digit::cls(wb[b].x, j),
                            digit::cls(wb[b].y, j), bA[j], bB[j]);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const uint32_t s2 = *reinterpret_cast<const uint32_t *>(st + kWordBytes + (16 * b + 2 * g) * 2);
            const float s_lo = DT::tof((uint16_t)(s2 & 0xFFFFu)) * gf, s_hi = DT::tof((uint16_t)(s2 >> 16)) * gf;
#pragma unroll
            for (int m = 0; m < kMats; ++m) {
                if (m != mat) continue;
                acc[m][b][0] = fmaf(__int_as_float(d[b][0]) - digit::kMagic, s_lo, acc[m][b][0]);
                acc[m][b][1] = fmaf(__int_as_float(d[b][1]) - digit::kMagic, s_lo, acc[m][b][1]);
                acc[m][b][2] = fmaf(__int_as_float(d[b][2]) - digit::kMagic, s_hi, acc[m][b][2]);
                acc[m][b][3] = fmaf(__int_as_float(d[b][3]) - digit::kMagic, s_hi, acc[m][b][3]);
            }
        }
        __syncwarp();
        issue();
    }
    gemv::cp_async_wait<0>();
    if (bad_id && lane == 0) atomicOr(&tc::g_device_error, 2u);
    pdl_launch_dependents();
    __syncwarp();

    // ---- planes -> column values of this warp: tb[mat][n][col] in the warp's ring ----
    float(*tb)[8][kCols] = reinterpret_cast<float(*)[8][kCols]>(ring);
#pragma unroll
    for (int m = 0; m < kMats; ++m)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) tb[m][2 * t + (c & 1)][16 * b + 2 * g + (c >> 1)] = acc[m][b][c];
    __syncwarp();
    const float rs = nwg > 0 ? rscale[warp] : 0.0f;
#pragma unroll
    for (int m = 0; m < kMats; ++m) {
        const float s = tb[m][1][lane] + 256.0f * tb[m][2][lane];
        red[(warp * kMats + m) * kCols + lane] = (s + (65536.0f * tb[m][3][lane] - 4194304.0f * tb[m][0][lane])) * rs;
    }
    __syncthreads();
    if (warp != 0) return;
    float v[kMats];
#pragma unroll
    for (int m = 0; m < kMats; ++m) {
        v[m] = 0.0f;
        for (int w = 0; w < W; ++w) v[m] += red[(w * kMats + m) * kCols + lane];
    }
    const int n = n0 + lane;
    if (n >= p.N) return;
    if (MODE == kGateUp) {
        reinterpret_cast<uint16_t *>(p.out)[(size_t)z * p.N + n] = DT::fromf(epi<1>(v[0], v[kMats - 1]));
    } else if (MODE == kDown) {
        bool ok;
        expert(z, ok);
        reinterpret_cast<float *>(p.out)[(size_t)z * p.N + n] = ok ? v[0] * DT::tof(p.RW[z]) : 0.0f;
    } else {
        reinterpret_cast<uint16_t *>(p.out)[(size_t)z * p.N + n] = DT::fromf(v[0]);
    }
}

// O[t, n] = DT(sum_j Y[t*topk + j, n]), thread per (t, 4 columns)
template <class DT>
__global__ void __launch_bounds__(256) moe_decode_reduce_kernel(const float *__restrict__ Y, uint16_t *__restrict__ O,
                                                                int T, int N, int topk) {
    pdl_wait();
    const int n4 = N / 4;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < (long long)T * n4) {
        const int tt = (int)(idx / n4), c = (int)(idx % n4) * 4;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int j = 0; j < topk; ++j) {
            const float4 y = *reinterpret_cast<const float4 *>(Y + ((size_t)tt * topk + j) * N + c);
            s0 += y.x;
            s1 += y.y;
            s2 += y.z;
            s3 += y.w;
        }
        uint2 o;
        o.x = (uint32_t)DT::fromf(s0) | ((uint32_t)DT::fromf(s1) << 16);
        o.y = (uint32_t)DT::fromf(s2) | ((uint32_t)DT::fromf(s3) << 16);
        *reinterpret_cast<uint2 *>(O + (size_t)tt * N + c) = o;
    }
    pdl_launch_dependents();
}

template <int W, int MODE, class DT>
cudaError_t launch_mode(const MParams &p, int rows, cudaStream_t st) {
    const int ng = total_groups<MODE>(p.G, p.topk);
    const size_t smem = md_smem(W, (ng + W - 1) / W, mats<MODE>());
    auto kern = moe_decode_kernel<W, MODE, DT>;
    cudaError_t e = ensure_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3((p.N + kCols - 1) / kCols, rows), dim3(W * 32), smem, st, p);
}

template <int MODE>
cudaError_t launch(const MParams &p, int rows, int dtype, cudaStream_t st) {
    const int ng = total_groups<MODE>(p.G, p.topk);
    if (dtype == TERNOCL_BF16)
        return ng >= 16 ? launch_mode<8, MODE, BF16>(p, rows, st) : launch_mode<4, MODE, BF16>(p, rows, st);
    return ng >= 16 ? launch_mode<8, MODE, F16>(p, rows, st) : launch_mode<4, MODE, F16>(p, rows, st);
}

}  // namespace

size_t moe_decode_smem(int G, int topk, int mode) {
    const int ng = mode == kGateUp ? 2 * G : mode == kDown ? G : topk * G;
    const int W = ng >= 16 ? 8 : 4;
    return md_smem(W, (ng + W - 1) / W, mode == kGateUp ? 2 : 1);
}

cudaError_t moe_decode_gate_up_launch(const int *ids, const void *X, const uint32_t *Bg, const void *Sg,
                                      const uint32_t *Bu, const void *Su, void *H, int G, int N, int K, int topk,
                                      int E, int dtype, cudaStream_t st) {
    MParams p{ids, (const uint16_t *)X, Bg, Bu, (const uint16_t *)Sg, (const uint16_t *)Su, nullptr, H, N, K,
              K / kGS, topk, E};
    return launch<kGateUp>(p, G, dtype, st);
}

cudaError_t moe_decode_down_launch(const int *ids, const void *H, const void *RW, const uint32_t *B, const void *S,
                                   float *Y, int G, int N, int K, int E, int dtype, cudaStream_t st) {
    MParams p{ids, (const uint16_t *)H, B, B, (const uint16_t *)S, (const uint16_t *)S, (const uint16_t *)RW, Y, N, K,
              K / kGS, 1, E};
    return launch<kDown>(p, G, dtype, st);
}

cudaError_t moe_decode_down_sum_launch(const int *ids, const void *H, const void *RW, const uint32_t *B,
                                       const void *S, void *O, int T, int N, int K, int topk, int E, int dtype,
                                       cudaStream_t st) {
    MParams p{ids, (const uint16_t *)H, B, B, (const uint16_t *)S, (const uint16_t *)S, (const uint16_t *)RW, O, N, K,
              K / kGS, topk, E};
    return launch<kDownSum>(p, T, dtype, st);
}

cudaError_t moe_decode_reduce_launch(const float *Y, void *O, int T, int N, int topk, int dtype, cudaStream_t st) {
    const long long n = (long long)T * (N / 4);
    const dim3 grid((unsigned)((n + 255) / 256));
    if (dtype == TERNOCL_BF16)
        return launch_kernel(moe_decode_reduce_kernel<BF16>, grid, dim3(256), 0, st, Y, (uint16_t *)O, T, N, topk);
    return launch_kernel(moe_decode_reduce_kernel<F16>, grid, dim3(256), 0, st, Y, (uint16_t *)O, T, N, topk);
}

cudaError_t read_device_error_moe_decode(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
