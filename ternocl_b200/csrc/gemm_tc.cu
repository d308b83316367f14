// Prefill GEMM on the 5th-generation tensor cores (tcgen05), replaces the M-tiled
// upconvert kernels int2_fp16_upcvt_gemm_mt (int2_fp16_upcvt.cl:338-396) and
// int1_fp16_upcvt_gemm_mt (int1_fp16_upcvt.cl:302-352):
//
//   C[m,n] = DT(epi( sum_k A[m,k] * W[k,n] )),   W[k,n] = code(k,n) * S[k/128, n]
//
// As in the reference's GEMM the weights are upconverted to DT +-s (or 0) before the
// MMA (exact: s is a DT value), and the products are accumulated in fp32.
//
// CTA tile 256 (M; 128 for M <= 128 and for MoE row tiles) x 256 (N), K in steps of
// 64; 320 threads in three roles:
//   warp 0      TMA producer: A [rows x 64] through a 2-D tensor map (one box in the
//               128-byte swizzle layout), the packed weight rows and the scale row
//               through 1-D bulk copies, all completing on one mbarrier per stage (3-4
//               load stages);
//   warp 1      TMEM allocation (256 fp32 columns per 128-row half) and the MMA
//               issuer: per stage and half four tcgen05.mma.cta_group::1.kind::f16
//               (M=128, N=256, K=16), A and B from shared-memory descriptors (both
//               halves read the same decoded B), accumulators in TMEM;
//               tcgen05.commit frees the stage and the decoded buffer;
//   warps 2-9   decode: warp kc, lane nb turns the packed words of 8 columns
//               (8nb..8nb+7) and 8 K rows (8kc..8kc+7 of the stage) into one 8x8
//               core matrix of the B operand, MN-major (a core-matrix row = one K row,
//               8 consecutive columns, 16 bytes), 3 decode buffers; after the K loop
//               the same warps read the accumulator (tcgen05.ld, warp w owns TMEM lanes
//               32(w%4)..+31) and run the fused epilogue store.
// Every mbarrier wait is bounded (tc::mbar_wait); on a timeout the roles skip ahead,
// the producer waits (bounded) for its copies in flight, and TMEM is freed.
//
// The decode of a layout is a policy:
//   Int2Gemm  word (kp,n) = 16 rows; columns n, n+1 of the same 8 rows are paired with
//             one PRMT, decoded as a half2 (row r of column n, row r of column n+1) by
//             the same LOP3 + HSUB2 as the GEMV (Int2Decode), then scaled by HMUL2;
//   Int1Gemm  sel layout: word (kp, blk+p) = rows (2p, 2p+1) of 16 columns; one IMAD
//             puts the sign bits of columns (2i, 2i+1) of a row at bits 15 and 31 and
//             one LOP3 applies them to the scale pair: +-s exactly.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;  // BM: rows of one MMA (cta_group::1)
constexpr int kDecStages = 3;
constexpr int kDecWarps = 8;
constexpr int kThreads = (2 + kDecWarps) * 32;
// decoded B (MN-major, no swizzle): core matrix (kc, nb) at nb * kDecSBO + kc * 128;
// the 16-byte pad in kDecSBO spreads the decode warps' stores over all banks
constexpr int kDecLBO = 128, kDecSBO = BK / 8 * 128 + 16;  // 1040
constexpr int kDecStageBytes = (BN / 8) * kDecSBO;         // 33280
constexpr int kPackStageBytes = 4096;  // int2: 4 word rows x 256 columns; int1: 2 x 256
constexpr int kScaleStageBytes = BN * 2;

// A CTA tile is HALVES x 128 rows: with two halves the decoded B tile of a stage feeds
// two MMAs (one per 128-row half, accumulators side by side in TMEM), which halves the
// decode work and the shared-memory traffic of B per multiply-add.
template <int HALVES>
struct Cfg {
    static constexpr int kRows = BM * HALVES;
    static constexpr int kLoadStages = HALVES == 2 ? 3 : 4;
    // A (K-major, 128-byte swizzle): one TMA box of kRows rows x 64 elements per stage;
    // the 128-row half h starts at h * 16 KB
    static constexpr int kAStageBytes = kRows * BK * 2;
    static constexpr int kTmemCols = BN * HALVES;
    // decoded buffers first: every descriptor-derived address stays inside the block
    static constexpr int dec = 0;
    static constexpr int a = (kDecStages * kDecStageBytes + 1023) / 1024 * 1024;
    static constexpr int pack = a + kLoadStages * kAStageBytes;
    static constexpr int scale = pack + kLoadStages * kPackStageBytes;
    static constexpr int bars = scale + kLoadStages * kScaleStageBytes;
    static constexpr int total = bars + 256 + 1024;  // + alignment slack
    static_assert(total <= 227 * 1024, "shared memory");
    // the epilogue's Other ring (8 warps x 4 blocks of 32 x 32 DT) reuses the A stages
    static_assert(kLoadStages * kAStageBytes >= 8 * 4 * 32 * 32 * 2, "Other ring");
};

struct Params {
    const uint32_t *B;
    const uint16_t *S;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K;
    // grouped (MoE) mode: meta = [E+1 row offsets | E+1 row-tile offsets] of the rows
    // sorted by expert; blockIdx.y is a row tile of some expert, B and S are [E, ...]
    const int *meta;
    int E;
};

template <class DT>
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT::kBF16) asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
    else asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// ---- int2: [K/16, N] words, 4 word rows per stage --------------------------------
struct Int2Gemm {
    static constexpr int kRowsPerStage = BK / 16;  // packed word rows per stage
    static constexpr int kKPerWordRow = 16;
    __device__ static const uint32_t *row_ptr(const Params &p, int kb, int r, int n0) {
        return p.B + (size_t)(kb * kRowsPerStage + r) * p.N + n0;
    }
    // core matrix rows out[r] (K row 8kc + r; columns 8nb .. 8nb+7 as 4 half2)
    template <class DT>
    __device__ static void decode(const char *pack, const uint16_t *scale, int kc, int nb, uint4 out[8]) {
        const uint4 *src = reinterpret_cast<const uint4 *>(pack + (kc >> 1) * (BN * 4) + nb * 32);
        // lanes 4..7 of each quarter-warp read their two 16-byte chunks in the other
        // order, so that both loads touch 8 distinct 16-byte bank groups
        const int sw = (nb >> 2) & 1;
        const uint4 c0 = src[sw], c1 = src[sw ^ 1];
        const uint4 w0 = sw ? c1 : c0, w1 = sw ? c0 : c1;
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint4 sv = *reinterpret_cast<const uint4 *>(scale + nb * 8);
        const uint32_t s2[4] = {sv.x, sv.y, sv.z, sv.w};  // (s_{2i}, s_{2i+1})
        const uint32_t sel = (kc & 1) ? 0x7632u : 0x5410u;  // rows 8..15 or 0..7 of the words
        uint32_t d[4][8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t z = __byte_perm(w[2 * i], w[2 * i + 1], sel);  // (column 2i | column 2i+1)
            Int2Decode<DT>::word(z, d[i]);                                   // d[i][r] = (row r of both)
#pragma unroll
            for (int r = 0; r < 8; ++r) d[i][r] = hmul2<DT>(d[i][r], s2[i]);
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) out[r] = make_uint4(d[0][r], d[1][r], d[2][r], d[3][r]);
    }
};

// ---- int1: sel layout [K/32, N], 2 word rows per stage --------------------------
struct Int1Gemm {
    static constexpr int kRowsPerStage = BK / 32;
    static constexpr int kKPerWordRow = 32;
    __device__ static const uint32_t *row_ptr(const Params &p, int kb, int r, int n0) {
        return p.B + (size_t)(kb * kRowsPerStage + r) * p.N + n0;
    }
    template <class DT>
    __device__ static void decode(const char *pack, const uint16_t *scale, int kc, int nb, uint4 out[8]) {
        // K rows 8kc..8kc+7 of the stage = K32 row kc/4, row pairs p = 4(kc%4) .. +3;
        // columns 8nb..8nb+7 = half (nb & 1) of the words of 16-column block nb/2
        const uint4 wv = *reinterpret_cast<const uint4 *>(pack + (kc >> 2) * (BN * 4) + (nb >> 1) * 64 +
                                                          (kc & 3) * 16);
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint4 sv = *reinterpret_cast<const uint4 *>(scale + nb * 8);
        const uint32_t s2[4] = {sv.x, sv.y, sv.z, sv.w};
        const int sh = 16 * (nb & 1);
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
            const uint32_t h = w[pp] >> sh;  // bit 2c + r: column 8nb + c, row 2p + r
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                uint32_t o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    // bits 4i + r (column 2i) -> 15, 4i + 2 + r (column 2i+1) -> 31
                    const uint32_t t = (h >> (4 * i + r)) & 5u;
                    uint32_t v;
                    asm("lop3.b32 %0, %1, %2, %3, 0x6A;\n" : "=r"(v) : "r"(t * 0x20008000u), "n"(0x80008000u), "r"(s2[i]));
                    o[i] = v;  // (t*K & 0x80008000) ^ s2: the sign bits applied to (s_2i, s_2i+1)
                }
                out[2 * pp + r] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
};

template <class Policy, int HALVES, class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const Params pin, const __grid_constant__ CUtensorMap tmA) {
    using C = Cfg<HALVES>;
    constexpr int kLoadStages = C::kLoadStages;
    extern __shared__ __align__(1024) char smem_raw[];
    // 1024-byte aligned base (the 128-byte swizzle pattern is anchored at 1024 B)
    char *smem = smem_raw + ((1024u - (tc::smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN;
    Params p = pin;
    int m0 = blockIdx.y * C::kRows;  // first A / C row of the tile
    int m_end = p.M;           // rows >= m_end are not stored
    if (p.meta) {
        // the tile's expert: the last one whose first row tile is <= this tile
        // (int2_moe_prefill.cl:80-88); meta comes from the routing kernel
        pdl_wait();
        const int tile = blockIdx.y, E = p.E;
        if (tile >= p.meta[2 * E + 1]) return;
        int lo = 0, hi = E - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.meta[E + 1 + mid] <= tile) lo = mid;
            else hi = mid - 1;
        }
        const int local = tile - p.meta[E + 1 + lo];
        // 256-row CTAs: the CTA of an expert's even 128-row tile covers the odd one too
        if (HALVES == 2 && (local & 1)) return;
        m0 = p.meta[lo] + local * BM;
        m_end = p.meta[lo + 1];
        p.B += (size_t)lo * (p.K / Policy::kKPerWordRow) * p.N;
        p.S += (size_t)lo * (p.K / kGS) * p.N;
    }
    const int nk = p.K / BK;
    const int ncols = min(BN, p.N - n0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::bars);
    uint64_t *load_empty = full + kLoadStages;
    uint64_t *dec_full = load_empty + kLoadStages;
    uint64_t *dec_empty = dec_full + kDecStages;
    uint64_t *acc_full = dec_empty + kDecStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

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
    if (warp == 1) tc::tmem_alloc(tmem_slot, C::kTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            pdl_wait();
            const uint32_t pack_bytes = Policy::kRowsPerStage * ncols * 4, scale_bytes = ncols * 2;
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kLoadStages;
                if (kb >= kLoadStages && !tc::mbar_wait(&load_empty[s], ((kb / kLoadStages) - 1) & 1)) break;
                tc::mbar_expect_tx(&full[s], C::kAStageBytes + pack_bytes + scale_bytes);
                char *a = smem + C::a + s * C::kAStageBytes;
                tc::tma_load_2d(a, &tmA, kb * BK, m0, &full[s]);
                char *pk = smem + C::pack + s * kPackStageBytes;
                for (int r = 0; r < Policy::kRowsPerStage; ++r)
                    tc::bulk_g2s(pk + r * (BN * 4), Policy::row_ptr(p, kb, r, n0), pack_bytes / Policy::kRowsPerStage,
                                 &full[s]);
                tc::bulk_g2s(smem + C::scale + s * kScaleStageBytes, p.S + (size_t)(kb * BK / kGS) * p.N + n0,
                             scale_bytes, &full[s]);
                ++issued;
            }
            // copies still in flight must land before the block can exit
            for (int kb = issued - kLoadStages < 0 ? 0 : issued - kLoadStages; kb < issued; ++kb)
                tc::mbar_wait(&full[kb % kLoadStages], (kb / kLoadStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_f16(DT::kBF16, BM, BN) | (1u << 16);  // B MN-major
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
                        // rows 128h .. 128h+127 of the A stage: 16 core matrices from h * 2048
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
        // ---------------- decode, then epilogue ----------------
        const int kc = warp - 2, nb = lane;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kLoadStages, d = kb % kDecStages;
            if (!tc::mbar_wait(&full[s], (kb / kLoadStages) & 1)) break;
            if (kb >= kDecStages && !tc::mbar_wait(&dec_empty[d], ((kb / kDecStages) - 1) & 1)) break;
            uint4 rows[8];
            Policy::template decode<DT>(smem + C::pack + s * kPackStageBytes,
                                        reinterpret_cast<const uint16_t *>(smem + C::scale + s * kScaleStageBytes),
                                        kc, nb, rows);
            char *dst = smem + C::dec + d * kDecStageBytes + nb * kDecSBO + kc * 128;
#pragma unroll
            for (int r = 0; r < 8; ++r) *reinterpret_cast<uint4 *>(dst + r * 16) = rows[r];
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&dec_full[d]);
                tc::mbar_arrive(&load_empty[s]);
            }
        }
        if (tc::mbar_wait(acc_full, 0)) {
            tc::fence_after_sync();
            // 32 x 32 blocks through a tile of this warp (the decode stages are free: every
            // MMA is done), so that a warp's stores run along rows: lanes 0-15 and 16-31
            // take column pairs of two rows
            const int quad = warp & 3, half = kc >> 2;
            float *t = reinterpret_cast<float *>(smem + C::dec + kc * kEpiTileBytes);
            constexpr int kChunks = HALVES * BN / 2 / 32;
            auto chunk_row = [&](int c) { return m0 + (c / (BN / 2 / 32)) * BM + 32 * quad; };  // 128-row half
            auto chunk_col = [&](int c) { return half * (BN / 2) + 32 * (c % (BN / 2 / 32)); };
            // POSTOP 1/2: the Other blocks of the next kOtherRing chunks stream into a ring of
            // this warp in the freed A stages (lane = row, 16-byte copies), so their latency
            // overlaps the previous chunks' work (needs a 16-byte-aligned Other)
            constexpr bool kOther = POSTOP == 1 || POSTOP == 2;
            constexpr int kOtherRing = 4, kOtherBlock = 32 * 32;  // elements
            const bool ring_ok = kOther && (reinterpret_cast<uintptr_t>(p.Other) & 15u) == 0;
            uint16_t *oring = reinterpret_cast<uint16_t *>(smem + C::a) + kc * kOtherRing * kOtherBlock;
            auto fetch = [&](int c) {
                if (ring_ok && c < kChunks) {
                    const int r = chunk_row(c) + lane, col = chunk_col(c);
                    uint16_t *dst = oring + (c % kOtherRing) * kOtherBlock + lane * 32;
                    if (r < m_end)
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            if (col + 8 * q < ncols)
                                tc::cp_async16(dst + 8 * q, p.Other + (size_t)r * p.N + n0 + col + 8 * q);
                }
                tc::cp_async_commit();
            };
            if (ring_ok)
                for (int c = 0; c < kOtherRing; ++c) fetch(c);
#pragma unroll 1
            for (int c = 0; c < kChunks; ++c) {
                const int h = c / (BN / 2 / 32);
                const int col = chunk_col(c);
                float v[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)(h * BN + col);
                tc::tmem_ld<16>(taddr, *reinterpret_cast<float(*)[16]>(&v[0]));
                tc::tmem_ld<16>(taddr + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
                tc::tmem_wait_ld();
                if (ring_ok) {
                    uint32_t o[16];
                    tc::cp_async_wait<kOtherRing - 1>();  // chunk c's block has landed
                    __syncwarp();
                    epi_load_rows32_smem(o, oring + (c % kOtherRing) * kOtherBlock, lane);
                    epi_store_rows32<DT, POSTOP, OUT_F32>(t, v, o, p.C, p.Bias, p.N, chunk_row(c), m_end, n0 + col,
                                                          ncols - col, lane);
                    fetch(c + kOtherRing);  // after the warp's reads of that slot (synced above)
                } else {
                    epi_store_rows32<DT, POSTOP, OUT_F32>(t, v, p.C, p.Other, p.Bias, p.N, chunk_row(c), m_end,
                                                          n0 + col, ncols - col, lane);
                }
            }
            if (ring_ok) tc::cp_async_wait<0>();
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

// ---- persistent variant ---------------------------------------------------------
// One CTA per SM walks the tiles (column block fastest); 128-row tiles with two TMEM
// accumulators (2 x 256 columns) so that four dedicated epilogue warps drain tile i
// while the producer, decode and MMA warps already run tile i+1.  The pipeline's stage
// and phase counters simply continue across tiles.  Used for the MoE grouped GEMMs
// (many short tiles) and wherever the per-launch tile count leaves a ragged last wave.
constexpr int kPEpiWarps = 4;
constexpr int kPThreads = (2 + kDecWarps + kPEpiWarps) * 32;  // 448
// Cfg<1>'s layout plus the epilogue warps' staging tiles (the next tile's mainloop owns
// the decode stages while the epilogue runs)
struct PSmem {
    static constexpr int epi = Cfg<1>::bars + 256;
    static constexpr int total = epi + kPEpiWarps * kEpiTileBytes + 1024;
    static_assert(total <= 227 * 1024, "shared memory");
};

struct TileInfo {
    int m0, m_end, n0;
    const uint32_t *B;
    const uint16_t *S;
};

// tile t of the launch -> rows, columns and (grouped mode) the expert's weights
template <class Policy>
__device__ __forceinline__ bool tile_info(const Params &p, int t, int nN, TileInfo &ti) {
    const int tm = t / nN, tn = t - tm * nN;
    ti.n0 = tn * BN;
    ti.B = p.B;
    ti.S = p.S;
    if (!p.meta) {
        ti.m0 = tm * BM;
        ti.m_end = p.M;
        return true;
    }
    const int E = p.E;
    int lo = 0, hi = E - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.meta[E + 1 + mid] <= tm) lo = mid;
        else hi = mid - 1;
    }
    ti.m0 = p.meta[lo] + (tm - p.meta[E + 1 + lo]) * BM;
    ti.m_end = p.meta[lo + 1];
    ti.B = p.B + (size_t)lo * (p.K / Policy::kKPerWordRow) * p.N;
    ti.S = p.S + (size_t)lo * (p.K / kGS) * p.N;
    return true;
}

template <class Policy, class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kPThreads, 1) gemm_persistent_kernel(const Params p,
                                                                       const __grid_constant__ CUtensorMap tmA) {
    using C = Cfg<1>;
    constexpr int kLoadStages = C::kLoadStages;
    extern __shared__ __align__(1024) char smem_raw[];
    // 1024-byte aligned base (the 128-byte swizzle pattern is anchored at 1024 B)
    char *smem = smem_raw + ((1024u - (tc::smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nk = p.K / BK;
    const int nN = (p.N + BN - 1) / BN;
    if (p.meta) pdl_wait();  // the tile count comes from the routing kernel
    const int ntiles = (p.meta ? p.meta[2 * p.E + 1] : (p.M + BM - 1) / BM) * nN;
    if ((int)blockIdx.x >= ntiles) return;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::bars);
    uint64_t *load_empty = full + kLoadStages;
    uint64_t *dec_full = load_empty + kLoadStages;
    uint64_t *dec_empty = dec_full + kDecStages;
    uint64_t *acc_full = dec_empty + kDecStages;  // [2]
    uint64_t *acc_empty = acc_full + 2;           // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

    if (tid == 0) {
        for (int s = 0; s < kLoadStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&load_empty[s], 1 + kDecWarps);
        }
        for (int d = 0; d < kDecStages; ++d) {
            tc::mbar_init(&dec_full[d], kDecWarps);
            tc::mbar_init(&dec_empty[d], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], kPEpiWarps);
        }
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, 2 * BN);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            if (!p.meta) pdl_wait();
            int g = 0;  // stages issued so far, across tiles
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                TileInfo ti;
                tile_info<Policy>(p, t, nN, ti);
                const int ncols = min(BN, p.N - ti.n0);
                const uint32_t pack_bytes = Policy::kRowsPerStage * ncols * 4, scale_bytes = ncols * 2;
                Params q = p;
                q.B = ti.B;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % kLoadStages;
                    if (g >= kLoadStages && !tc::mbar_wait(&load_empty[s], ((g / kLoadStages) - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_expect_tx(&full[s], C::kAStageBytes + pack_bytes + scale_bytes);
                    char *a = smem + C::a + s * C::kAStageBytes;
                    tc::tma_load_2d(a, &tmA, kb * BK, ti.m0, &full[s]);
                    char *pk = smem + C::pack + s * kPackStageBytes;
                    for (int r = 0; r < Policy::kRowsPerStage; ++r)
                        tc::bulk_g2s(pk + r * (BN * 4), Policy::row_ptr(q, kb, r, ti.n0),
                                     pack_bytes / Policy::kRowsPerStage, &full[s]);
                    tc::bulk_g2s(smem + C::scale + s * kScaleStageBytes,
                                 ti.S + (size_t)(kb * BK / kGS) * p.N + ti.n0, scale_bytes, &full[s]);
                }
            }
            for (int x = g - kLoadStages < 0 ? 0 : g - kLoadStages; x < g; ++x)
                tc::mbar_wait(&full[x % kLoadStages], (x / kLoadStages) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_f16(DT::kBF16, BM, BN) | (1u << 16);
            int g = 0, it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
                const int b = it & 1;
                if (it >= 2 && !tc::mbar_wait(&acc_empty[b], ((it >> 1) - 1) & 1)) break;
                tc::fence_after_sync();
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int s = g % kLoadStages, d = g % kDecStages;
                    if (!tc::mbar_wait(&full[s], (g / kLoadStages) & 1) ||
                        !tc::mbar_wait(&dec_full[d], (g / kDecStages) & 1)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t a = tc::smem_addr(smem + C::a + s * C::kAStageBytes);
                    const uint32_t bb = tc::smem_addr(smem + C::dec + d * kDecStageBytes);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t bd = tc::sdesc_kmajor_noswz(bb + kk * 2 * kDecLBO, kDecLBO, kDecSBO);
                        const uint64_t ad = tc::sdesc_kmajor_sw128(a + kk * 32);
                        tc::mma_ss_f16(tmem + b * BN, ad, bd, idesc, (kb | kk) != 0);
                    }
                    tc::mma_commit(&load_empty[s]);
                    tc::mma_commit(&dec_empty[d]);
                }
                if (ok) tc::mma_commit(&acc_full[b]);
            }
        }
    } else if (warp < 2 + kDecWarps) {
        const int kc = warp - 2, nb = lane;
        int g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = g % kLoadStages, d = g % kDecStages;
                if (!tc::mbar_wait(&full[s], (g / kLoadStages) & 1) ||
                    (g >= kDecStages && !tc::mbar_wait(&dec_empty[d], ((g / kDecStages) - 1) & 1))) {
                    ok = false;
                    break;
                }
                uint4 rows[8];
                Policy::template decode<DT>(smem + C::pack + s * kPackStageBytes,
                                            reinterpret_cast<const uint16_t *>(smem + C::scale + s * kScaleStageBytes),
                                            kc, nb, rows);
                char *dst = smem + C::dec + d * kDecStageBytes + nb * kDecSBO + kc * 128;
#pragma unroll
                for (int r = 0; r < 8; ++r) *reinterpret_cast<uint4 *>(dst + r * 16) = rows[r];
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&dec_full[d]);
                    tc::mbar_arrive(&load_empty[s]);
                }
            }
        }
    } else {
        // epilogue: warp w owns TMEM lanes 32(w%4)..+31, all 256 columns of the tile
        const int quad = warp & 3;
        int it = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
            const int b = it & 1;
            if (!tc::mbar_wait(&acc_full[b], (it >> 1) & 1)) break;
            tc::fence_after_sync();
            TileInfo ti;
            tile_info<Policy>(p, t, nN, ti);
            const int ncols = min(BN, p.N - ti.n0);
            float *tt = reinterpret_cast<float *>(smem + PSmem::epi + quad * kEpiTileBytes);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                float v[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)(b * BN + 32 * c);
                tc::tmem_ld<16>(taddr, *reinterpret_cast<float(*)[16]>(&v[0]));
                tc::tmem_ld<16>(taddr + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
                tc::tmem_wait_ld();
                epi_store_rows32<DT, POSTOP, OUT_F32>(tt, v, p.C, p.Other, p.Bias, p.N, ti.m0 + 32 * quad, ti.m_end,
                                                      ti.n0 + 32 * c, ncols - 32 * c, lane);
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&acc_empty[b]);
        }
        pdl_launch_dependents();
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 2 * BN);
    }
}

// A [M, K] DT row-major; boxes of box_rows rows x 64 elements in the 128-byte swizzle
// layout, rows past M read as zero
static cudaError_t make_map_a(CUtensorMap *map, const void *A, int M, int K, bool bf16, int box_rows) {
    return tc::make_map_sw128(map, A, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                              M, K, box_rows);
}

template <class Policy>
cudaError_t launch_persistent(const GemvArgs &a, const int *meta = nullptr, int E = 0) {
    CUtensorMap map;
    cudaError_t e = make_map_a(&map, a.A, a.M, a.K, a.dtype == TERNOCL_BF16, BM);
    if (e != cudaSuccess) return e;
    Params p;
    p.meta = meta;
    p.E = E;
    p.B = a.B;
    p.S = (const uint16_t *)a.S;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // upper bound of the tile count (grouped: every expert adds at most one partial tile);
    // CTAs beyond the actual count return at once
    const long long tiles = ((long long)(a.M + BM - 1) / BM + (meta ? E : 0)) * ((a.N + BN - 1) / BN);
    const int grid = (int)(tiles < sms ? tiles : sms);
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) -> cudaError_t {
        using DT = typename decltype(dt)::type;
        auto kern = gemm_persistent_kernel<Policy, DT, decltype(po)::value, decltype(of)::value>;
        cudaError_t err = ensure_smem(kern, PSmem::total);
        if (err != cudaSuccess) return err;
        return launch_kernel(kern, dim3(grid), dim3(kPThreads), (size_t)PSmem::total, a.stream, p, map);
    });
}

template <class Policy, int HALVES>
cudaError_t launch_policy(const GemvArgs &a, const int *meta = nullptr, int E = 0) {
    CUtensorMap map;
    cudaError_t e = make_map_a(&map, a.A, a.M, a.K, a.dtype == TERNOCL_BF16, Cfg<HALVES>::kRows);
    if (e != cudaSuccess) return e;
    Params p;
    p.meta = meta;
    p.E = E;
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
        auto kern = gemm_kernel<Policy, HALVES, DT, decltype(po)::value, decltype(of)::value>;
        cudaError_t err = ensure_smem(kern, Cfg<HALVES>::total);
        if (err != cudaSuccess) return err;
        // grouped: one CTA per 128-row tile of meta (every expert adds at most one partial
        // tile); dense: one per kRows rows
        const int rows = meta ? BM : Cfg<HALVES>::kRows;
        const int tiles = (a.M + rows - 1) / rows + (meta ? E : 0);
        const dim3 grid((a.N + BN - 1) / BN, tiles);
        return launch_kernel(kern, grid, dim3(kThreads), (size_t)Cfg<HALVES>::total, a.stream, p, map);
    });
}

}  // namespace gemm

namespace gemm {
// 128- or 256-row tiles: one CTA per SM, so a grid runs in ceil(tiles / SMs) waves; a
// 256-row tile does twice the work of a 128-row one in ~1.6x the time (measured on
// B200), so pick the shape with fewer wave-weighted units.
bool use_256_rows(int M, int N) {
    if (const int tile_m = options().gemm_tile_m) return tile_m == 256;
    if (M <= BM) return false;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long nt = (N + BN - 1) / BN;
    const long long w1 = ((M + BM - 1) / BM * nt + sms - 1) / sms;
    const long long w2 = ((M + 2 * BM - 1) / (2 * BM) * nt + sms - 1) / sms;
    // a 256-row tile costs ~1.45x a 128-row one (the B decode is shared by two MMAs)
    return w2 * 16 < w1 * 11;
}
}  // namespace gemm

bool gemm_use_256_rows(int M, int N) { return gemm::use_256_rows(M, N); }

cudaError_t int2_gemm_tc_launch(const GemvArgs &a) {
    if (options().gemm_persistent == 2) return gemm::launch_persistent<gemm::Int2Gemm>(a);
    return gemm::use_256_rows(a.M, a.N) ? gemm::launch_policy<gemm::Int2Gemm, 2>(a)
                                        : gemm::launch_policy<gemm::Int2Gemm, 1>(a);
}
cudaError_t int1_gemm_tc_launch(const GemvArgs &a) {
    if (options().gemm_persistent == 2) return gemm::launch_persistent<gemm::Int1Gemm>(a);
    return gemm::use_256_rows(a.M, a.N) ? gemm::launch_policy<gemm::Int1Gemm, 2>(a)
                                        : gemm::launch_policy<gemm::Int1Gemm, 1>(a);
}
// MoE: 256-row CTAs (two MMAs share each decoded B tile) once the experts average two
// 128-row tiles, else 128-row ones (OPT_GEMM_TILE_M overrides)
cudaError_t moe_gemm_tc_launch(const GemvArgs &a, const int *meta, int E) {
    const int pers = options().gemm_persistent;
    if (pers == 1 || pers == 2 || (pers == 3 && a.K <= 1024))
        return gemm::launch_persistent<gemm::Int2Gemm>(a, meta, E);
    const int tile_m = options().gemm_tile_m;
    const bool rows256 = tile_m ? tile_m == 256 : a.M >= 2 * gemm::BM * E;
    return rows256 ? gemm::launch_policy<gemm::Int2Gemm, 2>(a, meta, E)
                   : gemm::launch_policy<gemm::Int2Gemm, 1>(a, meta, E);
}
cudaError_t read_device_error_gemm_tc(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
