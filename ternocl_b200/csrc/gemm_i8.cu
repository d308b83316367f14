// s8 x s2 prefill GEMM on tcgen05 .kind::i8, replaces int2_int8_gemm_mt
// (int2_via_int2_x_int8_dpas/int2_int8_dpas.cl:283-385):
//
//   C[m,n] = DT(epi( sum_g float(dot_g[m,n]) * (SB[g,n] * (1 / SA[g,m])) ))
//   dot_g[m,n] = sum_{k in group g} Aq[m,k] * code(B[k,n])          (exact int32)
//
// with the int8 activations Aq and scales SA of ternocl_int8_quant_a (host gold:
// compute_gold, int2_via_int2_x_int8_dpas/main.cpp:94-121).
//
// CTA tile 128 (M) x 128 (N); one stage = one 128-row group (K = 128).  576 threads:
//   warp 0      producer: Aq [128 x 128] through a 2-D tensor map (one box of 128 rows x
//               128 bytes in the 128-byte swizzle layout), the group's 8 packed word rows, the SB row
//               and the tile's SA entries through 1-D bulk copies (5 stages);
//   warp 1      TMEM (4 x 128 int32 columns) and the MMA issuer: per group four
//               tcgen05.mma.cta_group::1.kind::i8 (M=128, N=128, K=32, s8 x s8 -> s32)
//               into accumulator buffer g % 4;
//   warps 2-9   decode (4 stages ahead of the MMA): two threads per column n each turn 4
//               of the column's 8 words into core-matrix rows of the K-major int8 B tile, 64 x the code value (code_to_value, main.cpp:77):
//               one shift-and-mask per four rows leaves each code in the top two bits of
//               a byte, then a 4x4 byte transpose puts the 16 rows of the word in order;
//               and the group's SB row (fp32) and 1/SA of the tile's rows into a ring of
//               its own, so that a load stage is free as soon as it is decoded;
//   warps 10-17 promotion: after each group, tcgen05.ld of the int32 accumulator (warp w
//               owns TMEM lanes 32(w%4).. and 64 of the columns), then
//               acc += float(dot) * (SB[g,n] * (1/SA[g,m])) in registers (the gold's
//               formula; 1/SA is the IEEE quotient) on packed f32x2 arithmetic, and the
//               buffer's columns are set back to the bit pattern of 1.5 * 2^23 for its
//               next group.
// The accumulator buffers start every group at 0x4B400000 (1.5 * 2^23 as fp32), so after
// the group's MMAs they hold the bits of the fp32 1.5 * 2^23 + 64 * dot (|64 * dot| <=
// 64 * 128 * 127 * 2 < 2^22): one f32 subtraction gives 64 * dot exactly, and the 1/64 is
// folded into 1/SA (a power of two: the products are the gold's, bit for bit).  After the
// last group, the fused epilogue, each warp's 32 x 32 block turned through shared memory so
// that a warp stores along rows.  Every mbarrier wait is bounded (tc::mbar_wait).
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
#include "digit_common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {
namespace gemm8 {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int kStages = 5, kDecStages = 4, kSclStages = 8;
constexpr int kDecWarps = 8, kEpiWarps = 8;
constexpr int kDecPerCol = kDecWarps * 32 / BN;         // decode threads per column (2)
constexpr int kWordsPerThread = BK / 16 / kDecPerCol;   // word rows each decodes (4)
constexpr int kEpiCols = BN * 4 / kEpiWarps;            // accumulator columns per promotion warp (64)
constexpr int kThreads = (2 + kDecWarps + kEpiWarps) * 32;
constexpr int kAStageBytes = BM * BK;  // int8 A: one 128-byte-swizzled box of 128 rows x 128 B
constexpr int kDecLBO = 128, kDecSBO = BK / 16 * 128 + 16;            // 1040
constexpr int kDecStageBytes = (BN / 8) * kDecSBO;                     // 16640
constexpr int kPackStageBytes = (BK / 16) * BN * 4;                    // 4096
constexpr int kSbBytes = BN * 2, kSaBytes = (BM + 8) * 2 + 16;  // 16-byte multiple
constexpr int kAccBufs = 4;  // accumulator buffers: the MMA runs up to 3 groups ahead of the promotion
constexpr int kTmemCols = kAccBufs * BN;  // all 512 columns: one CTA per SM (576 threads, > 65536/2 registers)

struct Smem {
    static constexpr int dec = 0;
    static constexpr int a = (kDecStages * kDecStageBytes + 1023) / 1024 * 1024;
    static constexpr int pack = a + kStages * kAStageBytes;
    static constexpr int sb = pack + kStages * kPackStageBytes;
    static constexpr int sa = sb + kStages * kSbBytes;
    // per group, written by the decode warps for the promotion warps: the SB row as fp32
    // [BN] and 1/SA / 64 of the tile's rows [BM]
    static constexpr int scl = sa + kStages * kSaBytes;
    static constexpr int kSclBytes = (BN + BM) * 4;
    static constexpr int bars = scl + kSclStages * kSclBytes;
    static constexpr int total = bars + 256 + 1024;  // + alignment slack
};

static_assert(kStages * kAStageBytes >= kEpiWarps * kEpiTileBytes, "epilogue tiles reuse the A stages");

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

// int2 word (16 rows of one column) -> 16 int8 values 64 * code in row order
__device__ __forceinline__ uint4 s8x64_row(uint32_t x) {
    uint32_t r[4], o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = digit::cls(x, j);  // byte i: 64 * code of row 4i + j
    transpose4x4(r, o);                                   // o[q] byte i: row 4q + i
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// packed fp32 pairs (f32x2 arithmetic of sm_100)
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// ncols (a multiple of 8) columns of this warp's lane quadrant set to v (x8 stores: 8
// registers carry v)
__device__ __forceinline__ void tmem_fill(uint32_t taddr, uint32_t v, int ncols) {
#pragma unroll
    for (int c = 0; c < ncols; c += 8)
        asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};\n" ::"r"(taddr + c),
                     "r"(v));
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
    uint64_t *acc_empty = acc_full + kAccBufs;
    uint64_t *scl_full = acc_empty + kAccBufs;
    uint64_t *scl_empty = scl_full + kSclStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(scl_empty + kSclStages);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&load_empty[s], 1 + kDecWarps);  // the MMA (A) and the decode warps
        }
        for (int d = 0; d < kDecStages; ++d) {
            tc::mbar_init(&dec_full[d], kDecWarps);
            tc::mbar_init(&dec_empty[d], 1);
        }
        for (int b = 0; b < kAccBufs; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], kEpiWarps);
        }
        for (int r = 0; r < kSclStages; ++r) {
            tc::mbar_init(&scl_full[r], kDecWarps);
            tc::mbar_init(&scl_empty[r], kEpiWarps);
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
                const int s = kb % kStages, d = kb % kDecStages, b = kb % kAccBufs;
                if (!tc::mbar_wait(&full[s], (kb / kStages) & 1)) break;
                if (!tc::mbar_wait(&dec_full[d], (kb / kDecStages) & 1)) break;
                // phase 0 of acc_empty is the promotion warps' initial fill of the buffer
                if (!tc::mbar_wait(&acc_empty[b], (kb / kAccBufs) & 1)) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_addr(smem + Smem::a + s * kAStageBytes);
                const uint32_t bb = tc::smem_addr(smem + Smem::dec + d * kDecStageBytes);
#pragma unroll
                for (int kk = 0; kk < BK / 32; ++kk) {
                    const uint64_t ad = tc::sdesc_kmajor_sw128(a + kk * 32);
                    const uint64_t bd = tc::sdesc_kmajor_noswz(bb + kk * 2 * kDecLBO, kDecLBO, kDecSBO);
                    mma_ss_i8(tmem + b * BN, ad, bd, idesc, 1);  // onto the 1.5 * 2^23 fill
                }
                tc::mma_commit(&load_empty[s]);
                tc::mma_commit(&dec_empty[d]);
                tc::mma_commit(&acc_full[b]);
            }
        }
    } else if (warp < 2 + kDecWarps) {
        // decode: thread (part, n) = word rows part * kWordsPerThread .. of column n of the
        // tile; part 0 also converts SB[n], the last part row n's scale
        const int n = (tid - 64) % BN, part = (tid - 64) / BN;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kStages, d = kb % kDecStages, r = kb % kSclStages;
            if (!tc::mbar_wait(&full[s], (kb / kStages) & 1)) break;
            if (kb >= kDecStages && !tc::mbar_wait(&dec_empty[d], ((kb / kDecStages) - 1) & 1)) break;
            if (kb >= kSclStages && !tc::mbar_wait(&scl_empty[r], ((kb / kSclStages) - 1) & 1)) break;
            const uint32_t *pk = reinterpret_cast<const uint32_t *>(smem + Smem::pack + s * kPackStageBytes);
            char *dst = smem + Smem::dec + d * kDecStageBytes + (n >> 3) * kDecSBO + (n & 7) * 16;
#pragma unroll
            for (int i = 0; i < kWordsPerThread; ++i) {
                const int kc = part * kWordsPerThread + i;
                *reinterpret_cast<uint4 *>(dst + kc * 128) = s8x64_row(pk[kc * BN + n]);
            }
            // the SB row as fp32 (columns past the matrix hold stale values; never stored) and
            // row n's 1/SA (the IEEE quotient, as the gold) / 64 (exact: 64 * dot comes back)
            float *scl = reinterpret_cast<float *>(smem + Smem::scl + r * Smem::kSclBytes);
            if (part == 0) scl[n] = DT::tof(reinterpret_cast<const uint16_t *>(smem + Smem::sb + s * kSbBytes)[n]);
            if (part == kDecPerCol - 1) {
                const float sa = sa_off + n < nsa
                                     ? DT::tof(reinterpret_cast<const uint16_t *>(smem + Smem::sa + s * kSaBytes)[sa_off + n])
                                     : 0.0f;
                scl[BN + n] = (sa == 0.0f ? 0.0f : __frcp_rn(sa)) * 0.015625f;
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&dec_full[d]);
                tc::mbar_arrive(&scl_full[r]);
                tc::mbar_arrive(&load_empty[s]);
            }
        }
    } else {
        // promotion + epilogue: warp w owns TMEM lanes 32(w%4)..+31 and kEpiCols columns
        const int ew = warp - 2 - kDecWarps;
        const int quad = warp & 3, col0 = (ew >> 2) * kEpiCols;
        const int row = 32 * quad + lane;
        const uint32_t tl = tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)col0;
        // every accumulator buffer starts at the 1.5 * 2^23 pattern (phase 0 of acc_empty)
#pragma unroll
        for (int b = 0; b < kAccBufs; ++b) tmem_fill(tl + b * BN, digit::kMagicBits, kEpiCols);
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < kAccBufs; ++b) tc::mbar_arrive(&acc_empty[b]);
        uint64_t acc[kEpiCols / 2];  // column pairs (2i, 2i + 1) of this warp's columns
#pragma unroll
        for (int i = 0; i < kEpiCols / 2; ++i) acc[i] = 0;
        const uint64_t neg_magic = f2(-digit::kMagic, -digit::kMagic);
        bool ok = true;
        for (int kb = 0; kb < nk && ok; ++kb) {
            const int r = kb % kSclStages, b = kb % kAccBufs;
            ok = tc::mbar_wait(&acc_full[b], (kb / kAccBufs) & 1) && tc::mbar_wait(&scl_full[r], (kb / kSclStages) & 1);
            if (!ok) break;
            tc::fence_after_sync();
            // (float)dot * (SB * inv), inv = 1/SA: the gold's formula (main.cpp:115-117), with
            // 64 * dot from the accumulator and inv / 64 (exact)
            const float *scl = reinterpret_cast<const float *>(smem + Smem::scl + r * Smem::kSclBytes);
            const float *sbf = scl + col0;
            const float inv = scl[BN + row];
            const uint64_t inv2 = f2(inv, inv);
            const uint32_t taddr = tl + b * BN;
#pragma unroll
            for (int h = 0; h < kEpiCols; h += 16) {  // chunks of 16 columns
                uint32_t d[16];
                tc::tmem_ld_u32x16(taddr + h, &d[0]);
                tc::tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; c += 4) {
                    const float4 sv = *reinterpret_cast<const float4 *>(sbf + h + c);
                    const uint64_t s01 = f2_mul(f2(sv.x, sv.y), inv2), s23 = f2_mul(f2(sv.z, sv.w), inv2);
                    const uint64_t x01 = f2_add(f2(__uint_as_float(d[c]), __uint_as_float(d[c + 1])), neg_magic);
                    const uint64_t x23 = f2_add(f2(__uint_as_float(d[c + 2]), __uint_as_float(d[c + 3])), neg_magic);
                    uint64_t &a01 = acc[(h + c) / 2], &a23 = acc[(h + c) / 2 + 1];
                    a01 = f2_fma(x01, s01, a01);
                    a23 = f2_fma(x23, s23, a23);
                }
                // the columns back to 1.5 * 2^23 for group kb + 2 (d is dead: its registers
                // can carry the fill); then the buffer goes to the MMA warp
                tmem_fill(taddr + h, digit::kMagicBits, 16);
            }
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&acc_empty[b]);
                tc::mbar_arrive(&scl_empty[r]);
            }
        }
        if (ok) {
            // 32 x 32 blocks through a tile of this warp (the load stages are free: every
            // MMA is done), stored along rows
            float *t = reinterpret_cast<float *>(smem + Smem::a + ew * kEpiTileBytes);
#pragma unroll
            for (int hc = 0; hc < kEpiCols; hc += 32) {
                float v[32];
#pragma unroll
                for (int c = 0; c < 32; c += 2) f2_split(acc[(hc + c) / 2], v[c], v[c + 1]);
                epi_store_rows32<DT, POSTOP, OUT_F32>(t, v, p.C, p.Other, p.Bias, p.N, m0 + 32 * quad, m_end,
                                                      n0 + col0 + hc, ncols - col0 - hc, lane);
            }
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
