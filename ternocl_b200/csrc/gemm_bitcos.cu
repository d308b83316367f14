// BITCOS prefill GEMM on the 5th-generation tensor cores, replaces the M-tiled
// bitcos_fp16_upcvt_gemm_mt (bitcos_fp16_upcvt.cl:279-368):
//
//   C[m,n] = DT(epi( sum_k A[m,k] * W[k,n] )),   W[k,n] = code(k,n) * S[k/128, n]
//
// B is the BITCOS buffer (common/bitcos.hpp:17-114): bitmap [K/32][N] (bit c of word
// (kp, n) = weight(32kp + c, n) != 0) | offsets [N] (first sign word of column n) |
// signs (one bit per non-zero, column-major in k, 1 -> -1) | 4 pad words.  As in the
// reference's M-tiled kernel a tile walks all of K (no K split), so the rank of a
// column's next non-zero is a running popcount and needs no slice ranks.
//
// CTA tile 256 (M; 128 for small M) x 256 (N), K in steps of 64, 320 threads:
//   warp 0      TMA producer: A [rows x 64] in the 128-byte swizzle layout, the two
//               bitmap word rows of the stage and the scale row through 1-D bulk
//               copies, one mbarrier per stage;
//   warp 1      TMEM allocation and MMA issue: per stage and 128-row half four
//               tcgen05.mma.kind::f16 (M=128, N=256, K=16), accumulators in TMEM;
//   warps 2-9   decode, one column per thread: the weights of a column are its bitmap
//               bits and its own contiguous sign stream, so the decoded B is written
//               K-major (a core-matrix row = 8 consecutive K rows of one column, one
//               16-byte store) and needs no transpose.  Per stage a thread funnel-shifts
//               two 32-bit sign windows (rows 0-31, 32-63) out of three sign words and
//               turns every 4-row nibble into 4 DT values with a 256-entry table
//               (presence nibble, next 4 sign bits) -> +-1 / 0 (the reference's table,
//               bitcos_fp16_upcvt.cl:109-123), scaled by HMUL2 (exact: +-s or 0).  The
//               sign words of stage kb+2 are requested while stage kb is decoded (their
//               position needs the popcounts of stages kb and kb+1, read from the
//               staged bitmap rows).  After the K loop the same warps drain TMEM through
//               the fused epilogue.
// Every mbarrier wait is bounded; on a timeout the roles skip ahead and flag the device
// error word.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {
namespace gemm_bc {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kDecStages = 3;
constexpr int kDecWarps = 8;  // 256 threads = one column each
constexpr int kThreads = (2 + kDecWarps) * 32;
// decoded B, K-major, no swizzle: core matrix (kc, nb) = K rows 8kc..8kc+7 of columns
// 8nb..8nb+7 at nb * kDecSBO + kc * kDecLBO
constexpr int kDecLBO = 128, kDecSBO = BK / 8 * 128;  // 1024
constexpr int kDecStageBytes = (BN / 8) * kDecSBO;    // 32768
constexpr int kPackStageBytes = 2 * BN * 4;           // bitmap word rows 2kb, 2kb+1
constexpr int kScaleStageBytes = BN * 2;
constexpr int kLutBytes = 256 * 8;

template <int HALVES>
struct Cfg {
    static constexpr int kRows = BM * HALVES;
    static constexpr int kLoadStages = HALVES == 2 ? 3 : 4;
    static constexpr int kAStageBytes = kRows * BK * 2;
    static constexpr int kTmemCols = BN * HALVES;
    static constexpr int dec = 0;
    static constexpr int a = kDecStages * kDecStageBytes;  // 1024-aligned
    static constexpr int pack = a + kLoadStages * kAStageBytes;
    static constexpr int scale = pack + kLoadStages * kPackStageBytes;
    static constexpr int lut = scale + kLoadStages * kScaleStageBytes;
    static constexpr int bars = lut + kLutBytes;
    static constexpr int total = bars + 256 + 1024;  // + alignment slack
    static_assert(a % 1024 == 0, "A stages on 1024-byte boundaries");
    static_assert(total <= 227 * 1024, "shared memory");
};

struct Params {
    const uint32_t *B;  // BITCOS buffer
    const uint16_t *S;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K;
};

template <class DT>
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT::kBF16) asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
    else asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

template <int HALVES, class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1) bitcos_gemm_kernel(const Params p, const __grid_constant__ CUtensorMap tmA) {
    using C = Cfg<HALVES>;
    constexpr int kLoadStages = C::kLoadStages;
    extern __shared__ __align__(1024) char smem_raw[];
    char *smem = smem_raw + ((1024u - (tc::smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * C::kRows;
    const int nk = p.K / BK;
    const int ncols = min(BN, p.N - n0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::bars);
    uint64_t *load_empty = full + kLoadStages;
    uint64_t *dec_full = load_empty + kLoadStages;
    uint64_t *dec_empty = dec_full + kDecStages;
    uint64_t *acc_full = dec_empty + kDecStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    uint2 *lut = reinterpret_cast<uint2 *>(smem + C::lut);

    if (tid == 0) {
        for (int s = 0; s < kLoadStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&load_empty[s], 1 + kDecWarps);
        }
        for (int d = 0; d < kDecStages; ++d) {
            tc::mbar_init(&dec_full[d], kDecWarps);
            tc::mbar_init(&dec_empty[d], 1);
        }
        tc::mbar_init(acc_full, 1);
        tc::fence_mbar_init();
    }
    if (tid >= 64) {
        // (presence nibble m, 4 sign bits s) -> DT +-1 / 0 of the nibble's 4 rows in row order
        constexpr uint32_t kPos = DT::kBF16 ? 0x3F80u : 0x3C00u, kNeg = kPos | 0x8000u;
        const uint32_t idx = (uint32_t)(tid - 64), m = idx >> 4, s = idx & 15u;
        uint32_t c[4], r = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t pr = (m >> i) & 1u;
            c[i] = pr ? (((s >> r) & 1u) ? kNeg : kPos) : 0u;
            r += pr;
        }
        lut[idx] = make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, C::kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            pdl_wait();
            const uint32_t row_bytes = ncols * 4, scale_bytes = ncols * 2;
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kLoadStages;
                if (kb >= kLoadStages && !tc::mbar_wait(&load_empty[s], ((kb / kLoadStages) - 1) & 1)) break;
                tc::mbar_expect_tx(&full[s], C::kAStageBytes + 2 * row_bytes + scale_bytes);
                tc::tma_load_2d(smem + C::a + s * C::kAStageBytes, &tmA, kb * BK, m0, &full[s]);
                char *pk = smem + C::pack + s * kPackStageBytes;
                for (int r = 0; r < 2; ++r)
                    tc::bulk_g2s(pk + r * (BN * 4), p.B + (size_t)(2 * kb + r) * p.N + n0, row_bytes, &full[s]);
                tc::bulk_g2s(smem + C::scale + s * kScaleStageBytes, p.S + (size_t)(kb * BK / kGS) * p.N + n0,
                             scale_bytes, &full[s]);
                ++issued;
            }
            for (int kb = issued - kLoadStages < 0 ? 0 : issued - kLoadStages; kb < issued; ++kb)
                tc::mbar_wait(&full[kb % kLoadStages], (kb / kLoadStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_f16(DT::kBF16, BM, BN);  // A and B K-major
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kLoadStages, d = kb % kDecStages;
                if (!tc::mbar_wait(&full[s], (kb / kLoadStages) & 1)) break;
                if (!tc::mbar_wait(&dec_full[d], (kb / kDecStages) & 1)) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_addr(smem + C::a + s * C::kAStageBytes);
                const uint32_t b = tc::smem_addr(smem + C::dec + d * kDecStageBytes);
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t bd = tc::sdesc_kmajor_noswz(b + kk * 2 * kDecLBO, kDecLBO, kDecSBO);
#pragma unroll
                    for (int h = 0; h < HALVES; ++h) {
                        const uint64_t ad = tc::sdesc_kmajor_sw128(a + h * BM * 128 + kk * 32);
                        tc::mma_ss_f16(tmem + h * BN, ad, bd, idesc, (kb | kk) != 0);
                    }
                }
                tc::mma_commit(&load_empty[s]);
                tc::mma_commit(&dec_empty[d]);
            }
            tc::mma_commit(acc_full);
        }
    } else {
        // ---------------- decode (one column per thread), then epilogue ----------------
        const int t = tid - 64;
        const bool ok = t < ncols;
        const size_t bw = (size_t)(p.K / 32) * p.N;
        pdl_wait();
        const uint32_t *sg = p.B + bw + p.N + (ok ? __ldg(p.B + bw + n0 + t) : 0u);
        const uint32_t *pk0 = reinterpret_cast<const uint32_t *>(smem + C::pack) + t;
        const uint16_t *sc0 = reinterpret_cast<const uint16_t *>(smem + C::scale) + t;
        // three sign words from word rank/32: the windows of a 64-row stage
        auto fetch = [&](uint32_t rank, uint32_t (&x)[3]) {
            if (ok) {
                const uint32_t *q = sg + (rank >> 5);
                x[0] = __ldg(q);
                x[1] = __ldg(q + 1);
                x[2] = __ldg(q + 2);
            } else {
                x[0] = x[1] = x[2] = 0u;
            }
        };
        auto stage_pop = [&](int s) {
            return ok ? (uint32_t)(__popc(pk0[s * (kPackStageBytes / 4)]) +
                                   __popc(pk0[s * (kPackStageBytes / 4) + BN]))
                      : 0u;
        };
        uint32_t r0 = 0, r1 = 0;  // ranks at stages kb, kb+1
        uint32_t x0[3], x1[3];    // their sign words
        bool alive = tc::mbar_wait(&full[0], 0);
        fetch(0, x0);
        if (alive && nk > 1) {
            r1 = stage_pop(0);
            fetch(r1, x1);
        }
        char *dst0 = smem + C::dec + (t >> 3) * kDecSBO + (t & 7) * 16;
        for (int kb = 0; kb < nk && alive; ++kb) {
            const int s = kb % kLoadStages, d = kb % kDecStages;
            // look ahead: stage kb+1's bitmap rows give the rank at stage kb+2
            uint32_t r2 = 0, x2[3] = {0u, 0u, 0u};
            if (kb + 1 < nk) {
                const int s1 = (kb + 1) % kLoadStages;
                if (!tc::mbar_wait(&full[s1], ((kb + 1) / kLoadStages) & 1)) break;
                if (kb + 2 < nk) {
                    r2 = r1 + stage_pop(s1);
                    fetch(r2, x2);
                }
            }
            if (kb >= kDecStages && !tc::mbar_wait(&dec_empty[d], ((kb / kDecStages) - 1) & 1)) break;
            const uint32_t w0 = ok ? pk0[s * (kPackStageBytes / 4)] : 0u;
            const uint32_t w1 = ok ? pk0[s * (kPackStageBytes / 4) + BN] : 0u;
            const uint32_t sc = sc0[s * (kScaleStageBytes / 2)];
            const uint32_t s2 = sc | (sc << 16);
            const uint32_t sh = r0 & 31u;
            const uint32_t o1 = sh + __popc(w0);  // <= 63
            uint32_t win[2];
            win[0] = __funnelshift_r(x0[0], x0[1], sh);
            win[1] = o1 < 32u ? __funnelshift_r(x0[0], x0[1], o1) : __funnelshift_r(x0[1], x0[2], o1 - 32u);
            const uint32_t wd[2] = {w0, w1};
            char *dst = dst0 + d * kDecStageBytes;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t W = win[h];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t nb0 = (wd[h] >> (8 * j)) & 15u, nb1 = (wd[h] >> (8 * j + 4)) & 15u;
                    const uint2 e0 = lut[(nb0 << 4) | (W & 15u)];
                    W >>= __popc(nb0);
                    const uint2 e1 = lut[(nb1 << 4) | (W & 15u)];
                    W >>= __popc(nb1);
                    *reinterpret_cast<uint4 *>(dst + (4 * h + j) * kDecLBO) =
                        make_uint4(hmul2<DT>(e0.x, s2), hmul2<DT>(e0.y, s2), hmul2<DT>(e1.x, s2),
                                   hmul2<DT>(e1.y, s2));
                }
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&dec_full[d]);
                tc::mbar_arrive(&load_empty[s]);
            }
            r0 = r1;
            r1 = r2;
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                x0[i] = x1[i];
                x1[i] = x2[i];
            }
        }
        if (tc::mbar_wait(acc_full, 0)) {
            tc::fence_after_sync();
            // through a 32 x 32 tile per warp in the (now free) decode stages: stores along rows
            const int quad = warp & 3, half = (warp - 2) >> 2;
            float *t = reinterpret_cast<float *>(smem + C::dec + (warp - 2) * kEpiTileBytes);
#pragma unroll 1
            for (int c = 0; c < HALVES * BN / 2 / 32; ++c) {
                const int h = c / (BN / 2 / 32);
                const int col = half * (BN / 2) + 32 * (c % (BN / 2 / 32));
                float v[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)(h * BN + col);
                tc::tmem_ld<16>(taddr, *reinterpret_cast<float(*)[16]>(&v[0]));
                tc::tmem_ld<16>(taddr + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
                tc::tmem_wait_ld();
                epi_store_rows32<DT, POSTOP, OUT_F32>(t, v, p.C, p.Other, p.Bias, p.N, m0 + h * BM + 32 * quad, p.M,
                                                      n0 + col, ncols - col, lane);
            }
        }
        pdl_launch_dependents();
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, C::kTmemCols);
    }
}

template <int HALVES>
cudaError_t launch_h(const GemvArgs &a) {
    CUtensorMap map;
    cudaError_t e = tc::make_map_sw128(&map, a.A,
                                       a.dtype == TERNOCL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                       2, a.M, a.K, Cfg<HALVES>::kRows);
    if (e != cudaSuccess) return e;
    Params p;
    p.B = a.B;
    p.S = (const uint16_t *)a.S;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) -> cudaError_t {
        using DT = typename decltype(dt)::type;
        auto kern = bitcos_gemm_kernel<HALVES, DT, decltype(po)::value, decltype(of)::value>;
        cudaError_t err = ensure_smem(kern, Cfg<HALVES>::total);
        if (err != cudaSuccess) return err;
        const int rows = Cfg<HALVES>::kRows;
        const dim3 grid((a.N + BN - 1) / BN, (a.M + rows - 1) / rows);
        return launch_kernel(kern, grid, dim3(kThreads), (size_t)Cfg<HALVES>::total, a.stream, p, map);
    });
}

}  // namespace gemm_bc

cudaError_t bitcos_gemm_tc_launch(const GemvArgs &a) {
    return gemm_use_256_rows(a.M, a.N) ? gemm_bc::launch_h<2>(a) : gemm_bc::launch_h<1>(a);
}

cudaError_t read_device_error_gemm_bitcos(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
