// s8 x s2 prefill GEMM on tcgen05 .kind::i8, replaces int2_int8_gemm_mt
// (int2_via_int2_x_int8_dpas/int2_int8_dpas.cl:283-385):
//
//   C[m,n] = DT(epi( sum_g float(dot_g[m,n]) * (SB[g,n] * (1 / SA[g,m])) ))
//   dot_g[m,n] = sum_{k in group g} Aq[m,k] * code(B[k,n])          (exact int32)
//
// with the int8 activations Aq and scales SA of ternocl_int8_quant_a (host gold:
// compute_gold, int2_via_int2_x_int8_dpas/main.cpp:94-121).
//
// CTA tile 128 (M) x 128 (N); one stage = one 128-row group (K = 128).  448 threads:
//   warp 0      producer: Aq [128 x 128] through a 2-D tensor map (one box of 128 rows x
//               128 bytes in the 128-byte swizzle layout), the group's 8 packed word rows, the SB row
//               and the tile's SA entries through 1-D bulk copies (3 stages);
//   warp 1      TMEM (2 x 128 int32 columns) and the MMA issuer: per group four
//               tcgen05.mma.cta_group::1.kind::i8 (M=128, N=128, K=32, s8 x s8 -> s32)
//               into accumulator buffer g % 2, started fresh each group;
//   warps 2-5   decode: thread n turns the 8 words of column n into 8 core-matrix rows of
//               the K-major int8 B tile (2-bit two's complement = code_to_value, main.cpp:77;
//               16 bytes in row order per word);
//   warps 6-13  promotion: after each group, tcgen05.ld of the int32 accumulator (warp w
//               owns TMEM lanes 32(w%4).., half the columns), then
//               acc += float(dot) * (SB[g,n] * (1/SA[g,m])) in registers (the gold's
//               formula; 1/SA is the IEEE quotient); after the last group, the fused
//               epilogue store.
// The int32 dots are exact (|dot| <= 128 * 128 * 2 < 2^22, converted to float exactly).
// Every mbarrier wait is bounded (tc::mbar_wait).
//
// Grouped (MoE) mode, int2_moe_gemm_mt_i8 (int2_moe/int2_moe_prefill_int8.cl:73-172): with
// `meta` set, blockIdx.y is a row tile of the expert found by binary search over meta's
// tile offsets, B and SB are that expert's [E, ...] slices, rows run from its first row
// (any offset) to the next expert's, and SA [K/128, LDSA(G)] is read at the tile's rows.
// The SA copy starts at the 8-element boundary below the tile's first row (bulk copies
// start on 16 bytes), so a stage holds BM + 8 scales.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {
namespace gemm8 {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int kStages = 3, kDecStages = 2;
constexpr int kDecWarps = 4, kEpiWarps = 8;
constexpr int kThreads = (2 + kDecWarps + kEpiWarps) * 32;
constexpr int kAStageBytes = BM * BK;  // int8 A: one 128-byte-swizzled box of 128 rows x 128 B
constexpr int kDecLBO = 128, kDecSBO = BK / 16 * 128 + 16;            // 1040
constexpr int kDecStageBytes = (BN / 8) * kDecSBO;                     // 16640
constexpr int kPackStageBytes = (BK / 16) * BN * 4;                    // 4096
constexpr int kSbBytes = BN * 2, kSaBytes = (BM + 8) * 2 + 16;  // 16-byte multiple
constexpr int kTmemCols = 2 * BN;

struct Smem {
    static constexpr int dec = 0;
    static constexpr int a = (kDecStages * kDecStageBytes + 1023) / 1024 * 1024;
    static constexpr int pack = a + kStages * kAStageBytes;
    static constexpr int sb = pack + kStages * kPackStageBytes;
    static constexpr int sa = sb + kStages * kSbBytes;
    static constexpr int bars = sa + kStages * kSaBytes;
    static constexpr int total = bars + 256 + 1024;  // + alignment slack
};

struct Params {
    const uint32_t *B;
    const uint16_t *SB;
    const uint16_t *SA;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K, ldsa;
    // grouped mode: [E+1 row offsets | E+1 row-tile offsets] of the expert-sorted rows
    const int *meta;
    int E;
};

__device__ __forceinline__ void mma_ss_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Instruction descriptor, kind::i8: [4,6) D format (2 = s32), [7,10) A format and
// [10,13) B format (1 = signed 8-bit), both K-major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 4x4 byte transpose: out[j] byte i = in[i] byte j
__device__ __forceinline__ void transpose4x4(const uint32_t in[4], uint32_t out[4]) {
    const uint32_t t0 = __byte_perm(in[0], in[1], 0x5140), t1 = __byte_perm(in[0], in[1], 0x7362);
    const uint32_t t2 = __byte_perm(in[2], in[3], 0x5140), t3 = __byte_perm(in[2], in[3], 0x7362);
    out[0] = __byte_perm(t0, t2, 0x5410);
    out[1] = __byte_perm(t0, t2, 0x7632);
    out[2] = __byte_perm(t1, t3, 0x5410);
    out[3] = __byte_perm(t1, t3, 0x7632);
}

// int2 word (16 rows of one column) -> 16 int8 codes in row order
__device__ __forceinline__ uint4 s8_row(uint32_t x) {
    uint32_t r[4], o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t t = (x >> (2 * j)) & 0x03030303u;  // byte i: code of row 4i + j
        r[j] = t + (t & 0x02020202u) * 0x7Eu;             // sign-extend 2 -> 8 bits
    }
    transpose4x4(r, o);  // o[q] byte i: row 4q + i
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// int32 -> fp32 for |d| < 2^22 in two full-rate instructions
__device__ __forceinline__ float i2f_small(uint32_t d) {
    return __int_as_float((int)(d + 0x4B400000u)) - 12582912.0f;
}

template <class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1) gemm_i8_kernel(const Params p, const __grid_constant__ CUtensorMap tmA) {
    extern __shared__ __align__(1024) char smem_raw[];
    // 1024-byte aligned base (the 128-byte swizzle pattern is anchored at 1024 B)
    char *smem = smem_raw + ((1024u - (tc::smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN;
    const int nk = p.K / BK;
    const int ncols = min(BN, p.N - n0);
    int m0 = blockIdx.y * BM, m_end = p.M;
    const uint32_t *Bw = p.B;
    const uint16_t *SBw = p.SB;
    if (p.meta) {
        pdl_wait();  // meta comes from the routing kernel
        const int E = p.E, tile = blockIdx.y;
        if (tile >= p.meta[2 * E + 1]) return;  // uniform over the CTA, before any barrier
        int lo = 0, hi = E - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.meta[E + 1 + mid] <= tile) lo = mid;
            else hi = mid - 1;
        }
        m0 = p.meta[lo] + (tile - p.meta[E + 1 + lo]) * BM;
        m_end = p.meta[lo + 1];
        Bw += (size_t)lo * (p.K / 16) * p.N;
        SBw += (size_t)lo * (p.K / BK) * p.N;
    }
    // SA columns sa0 .. sa0 + nsa of each group row: sa0 on a 16-byte boundary, within the
    // padded pitch (ldsa % 32 == 0, so nsa * 2 is a multiple of 16)
    const int sa0 = m0 & ~7, sa_off = m0 - sa0;
    const int nsa = min(BM + 8, p.ldsa - sa0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars);
    uint64_t *load_empty = full + kStages;
    uint64_t *dec_full = load_empty + kStages;
    uint64_t *dec_empty = dec_full + kDecStages;
    uint64_t *acc_full = dec_empty + kDecStages;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&load_empty[s], 1 + kDecWarps + kEpiWarps);
        }
        for (int d = 0; d < kDecStages; ++d) {
            tc::mbar_init(&dec_full[d], kDecWarps);
            tc::mbar_init(&dec_empty[d], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], kEpiWarps);
        }
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();
            const uint32_t pack_bytes = (BK / 16) * ncols * 4, sb_bytes = ncols * 2, sa_bytes = nsa * 2;
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                if (kb >= kStages && !tc::mbar_wait(&load_empty[s], ((kb / kStages) - 1) & 1)) break;
                tc::mbar_expect_tx(&full[s], kAStageBytes + pack_bytes + sb_bytes + sa_bytes);
                char *a = smem + Smem::a + s * kAStageBytes;
                tc::tma_load_2d(a, &tmA, kb * BK, m0, &full[s]);
                char *pk = smem + Smem::pack + s * kPackStageBytes;
                for (int r = 0; r < BK / 16; ++r)
                    tc::bulk_g2s(pk + r * (BN * 4), Bw + (size_t)(kb * (BK / 16) + r) * p.N + n0, ncols * 4, &full[s]);
                tc::bulk_g2s(smem + Smem::sb + s * kSbBytes, SBw + (size_t)kb * p.N + n0, sb_bytes, &full[s]);
                tc::bulk_g2s(smem + Smem::sa + s * kSaBytes, p.SA + (size_t)kb * p.ldsa + sa0, sa_bytes, &full[s]);
                ++issued;
            }
            for (int kb = issued - kStages < 0 ? 0 : issued - kStages; kb < issued; ++kb)
                tc::mbar_wait(&full[kb % kStages], (kb / kStages) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(BM, BN);
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages, d = kb % kDecStages, b = kb & 1;
                if (!tc::mbar_wait(&full[s], (kb / kStages) & 1)) break;
                if (!tc::mbar_wait(&dec_full[d], (kb / kDecStages) & 1)) break;
                if (kb >= 2 && !tc::mbar_wait(&acc_empty[b], ((kb >> 1) - 1) & 1)) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_addr(smem + Smem::a + s * kAStageBytes);
                const uint32_t bb = tc::smem_addr(smem + Smem::dec + d * kDecStageBytes);
#pragma unroll
                for (int kk = 0; kk < BK / 32; ++kk) {
                    const uint64_t ad = tc::sdesc_kmajor_sw128(a + kk * 32);
                    const uint64_t bd = tc::sdesc_kmajor_noswz(bb + kk * 2 * kDecLBO, kDecLBO, kDecSBO);
                    mma_ss_i8(tmem + b * BN, ad, bd, idesc, kk != 0);
                }
                tc::mma_commit(&load_empty[s]);
                tc::mma_commit(&dec_empty[d]);
                tc::mma_commit(&acc_full[b]);
            }
        }
    } else if (warp < 2 + kDecWarps) {
        // decode: thread n = column n of the tile, 8 word rows of the stage
        const int n = tid - 64;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kStages, d = kb % kDecStages;
            if (!tc::mbar_wait(&full[s], (kb / kStages) & 1)) break;
            if (kb >= kDecStages && !tc::mbar_wait(&dec_empty[d], ((kb / kDecStages) - 1) & 1)) break;
            const uint32_t *pk = reinterpret_cast<const uint32_t *>(smem + Smem::pack + s * kPackStageBytes);
            char *dst = smem + Smem::dec + d * kDecStageBytes + (n >> 3) * kDecSBO + (n & 7) * 16;
#pragma unroll
            for (int kc = 0; kc < BK / 16; ++kc) *reinterpret_cast<uint4 *>(dst + kc * 128) = s8_row(pk[kc * BN + n]);
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&dec_full[d]);
                tc::mbar_arrive(&load_empty[s]);
            }
        }
    } else {
        // promotion + epilogue: warp w owns TMEM lanes 32(w%4)..+31 and columns half*64..+63
        const int ew = warp - 2 - kDecWarps;
        const int quad = warp & 3, half = ew >> 2;
        const int row = 32 * quad + lane, m = m0 + row;
        float acc[BN / 2];
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) acc[i] = 0.0f;
        bool ok = true;
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int s = kb % kStages, b = kb & 1;
            ok = tc::mbar_wait(&acc_full[b], (kb >> 1) & 1) && tc::mbar_wait(&full[s], (kb / kStages) & 1);
            if (!ok) break;
            tc::fence_after_sync();
            // (float)dot * (SB * inv), inv = 1/SA: the gold's formula (main.cpp:115-117)
            const uint16_t *sbs = reinterpret_cast<const uint16_t *>(smem + Smem::sb + s * kSbBytes) + half * (BN / 2);
            const float sa = sa_off + row < nsa
                                 ? DT::tof(reinterpret_cast<const uint16_t *>(smem + Smem::sa + s * kSaBytes)[sa_off + row])
                                 : 0.0f;
            const float inv = sa == 0.0f ? 0.0f : __frcp_rn(sa);
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // two chunks of 32 columns keep the register count down
                uint32_t d[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)(b * BN + half * (BN / 2) + 32 * h);
                tc::tmem_ld_u32x16(taddr, &d[0]);
                tc::tmem_ld_u32x16(taddr + 16, &d[16]);
                tc::tmem_wait_ld();
                if (h == 1) {
                    tc::fence_before_sync();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
                }
#pragma unroll
                for (int c = 0; c < 32; c += 8) {
                    const uint4 sv = *reinterpret_cast<const uint4 *>(sbs + 32 * h + c);
                    const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float s0 = DT::tof((uint16_t)(w[i] & 0xffffu)), s1 = DT::tof((uint16_t)(w[i] >> 16));
                        float &a0 = acc[32 * h + c + 2 * i], &a1 = acc[32 * h + c + 2 * i + 1];
                        a0 = fmaf(i2f_small(d[c + 2 * i]), s0 * inv, a0);
                        a1 = fmaf(i2f_small(d[c + 2 * i + 1]), s1 * inv, a1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&load_empty[s]);
        }
        if (ok && m < m_end) {
            const int col0 = half * (BN / 2);
#pragma unroll
            for (int c = 0; c < BN / 2; c += 2)
                if (col0 + c < ncols)
                    epi_store2<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, m, n0 + col0 + c, acc[c], acc[c + 1]);
        }
        pdl_launch_dependents();
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace gemm8

// Aq [M, K] int8 row-major, SA [K/128, ldsa]; grouped (meta != null): M = G rows sorted by
// expert, B and SB [E, ...]
cudaError_t int8_gemm_tc_launch(const GemvArgs &a, const int *meta, int E) {
    using namespace gemm8;
    CUtensorMap map;
    const cudaError_t me = tc::make_map_sw128(&map, a.Aq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.M, a.K, BM);
    if (me != cudaSuccess) return me;
    Params p;
    p.B = a.B;
    p.SB = (const uint16_t *)a.S;
    p.SA = (const uint16_t *)a.SA;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.ldsa = (a.M + 31) & ~31;
    p.meta = meta;
    p.E = meta ? E : 0;
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) -> cudaError_t {
        using DT = typename decltype(dt)::type;
        auto kern = gemm_i8_kernel<DT, decltype(po)::value, decltype(of)::value>;
        cudaError_t err = ensure_smem(kern, Smem::total);
        if (err != cudaSuccess) return err;
        // grouped: every expert adds at most one partial row tile
        const dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM + (meta ? E : 0));
        return launch_kernel(kern, grid, dim3(kThreads), (size_t)Smem::total, a.stream, p, map);
    });
}

cudaError_t read_device_error_gemm_i8(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
