// BITCOS ternary decode GEMV for M <= 8, persistent strip pipeline; replaces
// bitcos_fp16_upcvt_gemv (bitcos_fp16_upcvt.cl:177-277) on its decode shapes:
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(k,n) )),  code in {-1,0,+1}
//
// B is one uint32 buffer (common/bitcos.hpp:1-8, packed by bitcos_random :31-62):
// bitmap [K/32][N] | offsets [N] | signs | 4 pad words, where column n's signs are the
// words off[n] .. off[n] + ceil(nnz_n / 32) - 1, so the next column's offset ends them.
// Host gold: compute_gold + bitcos_decode_col (bitcos_fp16_upcvt/main.cpp:64-86,
// common/bitcos.hpp:97-106).
//
// One CTA per SM walks strips of 32 columns (strip s = blockIdx.x + i * gridDim.x), each
// over ALL of K, so a column's sign rank starts at 0 and no slice ranks are needed (LS
// and SR only serve the reference's K-sliced work split).  Everything a strip reads is
// known from the offsets plane alone, so one producer warp issues the whole strip at
// once (one mbarrier per stage, 2-3 stages in flight):
//   * the bitmap rows (K/32 rows of 32 words) and the scale rows (K/128 rows of 32 DT),
//     each as one or a few 2-D TMA boxes (a bulk copy per 128-byte row measured 1.5x
//     slower than the K-sliced kernel: the copy engine's cost is per request),
//   * per column the sign words [off[n], off[n+1]] (one word past the run: the 64-bit
//     window) as one 1-D bulk copy widened to 16-byte boundaries; the word offset inside
//     the slot is written beside the stage.
// The activation rows are staged once per CTA (after griddepcontrol.wait), with the
// 16-byte units swizzled as in the other GEMVs; with the fused Hadamard transform (the
// reference's hadamard_fwht -> BITCOS GEMV pipeline) the compute warps sign-flip and
// transform them in place, the stages of hadamard_fwht in its order (bit-identical to
// the standalone kernel), while the first strips load.
//
// nw compute warps (one per group up to 16, else 16) take contiguous group ranges of the
// strip, sized so that the SM's four schedulers get equal shares.  Per strip: each warp
// popcounts its bitmap rows (lane = column), a named barrier, and the warp's start rank
// per column is the sum of the earlier warps' counts.  The main loop per group is the nibble decode of the
// K-sliced kernel (gemv_bitcos.cu): lane (g, q) takes bitmap word q of columns
// 4g..4g+3, a 4-lane scan gives each word's rank, a 32-bit sign window comes out of the
// staged stream with one funnel shift, and each 4-row nibble indexes the 256-entry
// (presence nibble, 4 sign bits) -> 4 DT codes table (bitcos_fp16_upcvt.cl:109-123)
// feeding mma.sync m16n8k16 as the A operand (row g -> column 4g + 2b, row g + 8 -> column
// 4g + 2b + 1, the activation rows the 8 MMA columns).  (The codes as the B operand, with
// the activation row as A, need no register moves but twice the MMAs, and measured 5%
// slower.)  The table is replicated so that a lane reads its own copy:
// 16 copies (lane & 15) put every half-warp's 64-bit reads in distinct bank pairs; 8
// copies when shared memory is short.  The warps' partials are summed in warp order
// through shared memory (deterministic) and warp 0 stores the strip with the fused
// epilogue.  Every mbarrier wait is bounded (tc::mbar_wait); a timeout flags the device
// error word, and the compute warps leave together through a shared abort flag checked
// after a named barrier.
#include <cmath>
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv_common.cuh"
#include "hadamard_common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {
namespace bitcos_p {

constexpr int kMaxNW = 16;     // compute warps
constexpr int kMaxStages = 3;  // strips in flight
constexpr int kMaxRows = 8;    // activation rows (one MMA n-block)

struct Params {
    const uint16_t *A;
    const uint32_t *B;
    const uint16_t *S;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K;
    int nw, stages, lut_sh;  // compute warps, stages, log2 of the table copies
    int KW, G, cap;          // bitmap rows, scale groups, sign words per column slot
    int act_stride;          // bytes per staged activation row
    int box_b, box_s;        // rows per TMA box of the bitmap / scale plane (divide KW / G)
    int wg[kMaxNW + 1];      // compute warp w owns groups wg[w] .. wg[w+1] - 1 of a strip
    // the reference's hadamard_fwht -> BITCOS GEMV pipeline in one launch: log2 of the
    // FWHT block (0: none), its sign vector [K] (global, or null) and 1/sqrt(HB)
    int had_L;
    const int8_t *had_signs;
    float had_scale;
    // shared-memory layout (byte offsets)
    int o_red, o_seg, o_meta, o_bars, o_act, o_stage, stage_bytes, o_sc, o_sg, total;
};

__host__ __device__ inline int align128(int x) { return (x + 127) & ~127; }

// Layout of the shared memory for (M, K) with nw compute warps, `stages` stages and
// 2^lut_sh table copies; returns the total bytes.
__host__ __device__ inline int layout(Params &p, int M, int K, int nw, int stages, int lut_sh) {
    p.nw = nw;
    p.stages = stages;
    p.lut_sh = lut_sh;
    p.KW = K / 32;
    p.G = K / kGS;
    // a column's worst case (every weight non-zero) + window + alignment, rounded to 32
    // words; slot_base() skews the slots of columns 4g.. by 4g words so that the 8 columns
    // one warp-wide read touches (4g + c, g = 0..7) start in 8 different banks
    p.cap = (p.KW + 8 + 31) & ~31;
    p.act_stride = K * 2 + 16;
    const int rows = M < kMaxRows ? M : kMaxRows;
    int o = align128((256 << lut_sh) * 8);
    p.o_red = o;
    o = align128(o + nw * 32 * 8 * 4);
    p.o_seg = o;
    o = align128(o + nw * 32 * 4);
    p.o_meta = o;
    o = align128(o + kMaxStages * 32 * 4);
    p.o_bars = o;
    o = align128(o + 2 * kMaxStages * 8 + 16);
    p.o_act = o;
    o = align128(o + rows * p.act_stride);
    p.o_sc = p.KW * 128;
    p.o_sg = p.o_sc + p.G * 64;
    p.stage_bytes = align128(p.o_sg + (32 * p.cap + 4 * 8) * 4);
    p.o_stage = o;
    p.total = o + stages * p.stage_bytes;
    return p.total;
}

__host__ __device__ inline int slot_base(int cap, int col) { return col * cap + 4 * (col >> 2); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// A strip's sign runs, lane = column: first word o and one past the last word e (0, 0
// past the matrix).  The matrix's last column has no offset after it: its run length
// comes from its bitmap column, counted by the whole warp (independent loads).  Loaded
// ahead of the strip's issue so that the producer does not wait on them.
struct Runs {
    uint32_t o, e;
};
__device__ __forceinline__ Runs load_runs(const Params &p, int s, int lane) {
    const int N = p.N, KW = p.KW;
    const int n0 = s * 32, ncol = min(32, N - n0);
    const uint32_t *offs = p.B + (size_t)KW * N;
    uint32_t last_nnz = 0;
    if (n0 + ncol == N) {
        for (int kp = lane; kp < KW; kp += 32) last_nnz += __popc(__ldg(p.B + (size_t)kp * N + N - 1));
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) last_nnz += __shfl_xor_sync(0xffffffffu, last_nnz, d);
    }
    Runs r = {0u, 0u};
    if (lane < ncol) {
        const int n = n0 + lane;
        r.o = __ldg(offs + n);
        r.e = n + 1 < N ? __ldg(offs + n + 1) : r.o + (last_nnz + 31) / 32;
    }
    return r;
}

// Producer: strip s (columns n0 .. n0 + ncol - 1) into stage st, all copies completing on
// full[st].  Whole warp; lane = column for the sign copies.
__device__ __forceinline__ void issue_strip(const Params &p, const CUtensorMap *tmB, const CUtensorMap *tmS,
                                            char *smem, uint64_t *full, int s, int st, int lane, Runs r) {
    const int N = p.N, KW = p.KW, G = p.G;
    const int n0 = s * 32, ncol = min(32, N - n0);
    const uint32_t *signs = p.B + (size_t)KW * N + N;
    char *sp = smem + p.o_stage + st * p.stage_bytes;
    uint32_t *sh = reinterpret_cast<uint32_t *>(smem + p.o_meta) + st * 32;
    uint32_t a = 0, words = 0, shv = 0;  // shv: the run's first word within the slot
    if (lane < ncol) {
        a = r.o & ~3u;
        words = ((r.e + 4) & ~3u) - a;  // through word e (the window's second word), 16-byte units
        if (words > (uint32_t)p.cap) words = (uint32_t)p.cap;
        shv = r.o - a;
    }
    sh[lane] = shv;  // 0 for the columns past the matrix: their windows stay inside the slot
    uint32_t bytes = words * 4;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, d);
    bytes += (uint32_t)(KW * 128 + G * 64);  // whole boxes (columns past N read as 0)
    __syncwarp();  // sh[] before the arrive (release) that publishes the stage
    if (lane == 0) {
        tc::mbar_expect_tx(&full[st], bytes);
        for (int y = 0; y < KW; y += p.box_b) tc::tma_load_2d(sp + y * 128, tmB, n0, y, &full[st]);
        for (int y = 0; y < G; y += p.box_s) tc::tma_load_2d(sp + p.o_sc + y * 64, tmS, n0, y, &full[st]);
    }
    __syncwarp();
    if (words) tc::bulk_g2s(sp + p.o_sg + slot_base(p.cap, lane) * 4, signs + a, words * 4, &full[st]);
}

template <class DT, int POSTOP, bool OUT_F32, int LUT_SH>
__global__ void __launch_bounds__((kMaxNW + 1) * 32, 1)
    bitcos_gemv_p_kernel(const Params p, const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmS) {
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nw = p.nw, nthreads = (nw + 1) * 32;
    const int N = p.N, K = p.K;
    const int nstrips = (N + 31) / 32;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.o_bars);
    uint64_t *empty = full + kMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kMaxStages);
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], nw);
        }
        *abort_flag = 0;
        tc::fence_mbar_init();
    }
    __syncthreads();

    // the first strip: weights only, so before the wait on the previous kernel; the runs of
    // every first stage are loaded together (one latency), the other first stages are
    // issued after the CTA-wide barrier below, which they would otherwise hold up (the
    // copy engine takes ~2 us to accept a strip)
    Runs r[kMaxStages];
    if (warp == nw) {
#pragma unroll
        for (int j = 0; j < kMaxStages; ++j) {
            const int s = blockIdx.x + j * gridDim.x;
            r[j] = (j < p.stages && s < nstrips) ? load_runs(p, s, lane) : Runs{0u, 0u};
        }
        if ((int)blockIdx.x < nstrips) issue_strip(p, &tmB, &tmS, smem, full, blockIdx.x, 0, lane, r[0]);
    }

    // (presence nibble m, 4 sign bits s) -> DT codes of 4 rows in row order; entry e of
    // copy j at 8-byte slot e * 2^lut_sh + j
    uint2 *lut = reinterpret_cast<uint2 *>(smem);
    constexpr uint32_t kPos = DT::kBF16 ? 0x3F80u : 0x3C00u, kNeg = kPos | 0x8000u;
    for (int i = tid; i < (256 << LUT_SH); i += nthreads) {
        const uint32_t idx = (uint32_t)i >> LUT_SH;
        const uint32_t m = idx >> 4, s = idx & 15u;
        uint32_t c[4], r = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t pr = (m >> k) & 1u;
            c[k] = pr ? (((s >> r) & 1u) ? kNeg : kPos) : 0u;
            r += pr;
        }
        lut[i] = make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
    }

    // activation rows, 16-byte unit u of a row stored at u ^ (((u >> 3) & 1) << 1)
    pdl_wait();
    const int rows = min(kMaxRows, p.M);
    char *act = smem + p.o_act;
    const int nu = K / 8;
    for (int i = tid; i < rows * nu; i += nthreads) {
        const int m = i / nu, u = i - m * nu;
        const int pu = u ^ (((u >> 3) & 1) << 1);
        gemv::cp_async16(act + (size_t)m * p.act_stride + (size_t)pu * 16, p.A + (size_t)m * K + (size_t)u * 8);
    }
    gemv::cp_async_commit();
    gemv::cp_async_wait<0>();
    __syncthreads();

    if (warp == nw) {
#pragma unroll
        for (int j = 1; j < kMaxStages; ++j) {
            const int s = blockIdx.x + j * gridDim.x;
            if (j < p.stages && s < nstrips) issue_strip(p, &tmB, &tmS, smem, full, s, j, lane, r[j]);
        }
        // producer: the remaining strips, each into the stage its strip - stages freed
        int it = 0, issued = 0;
        const int s_first = blockIdx.x + p.stages * gridDim.x;  // the first strip issued here
        Runs nxt = s_first < nstrips ? load_runs(p, s_first, lane) : Runs{0u, 0u};
        for (int s = blockIdx.x; s < nstrips; s += gridDim.x, ++it) {
            if (it < p.stages) {
                ++issued;
                continue;
            }
            const int st = it % p.stages;
            if (!tc::mbar_wait(&empty[st], ((it / p.stages) - 1) & 1)) break;
            const Runs cur = nxt;
            if (s + gridDim.x < nstrips) nxt = load_runs(p, s + gridDim.x, lane);  // in flight meanwhile
            issue_strip(p, &tmB, &tmS, smem, full, s, st, lane, cur);
            ++issued;
        }
        // the copies in flight land before the CTA may exit (bounded waits)
        for (int j = issued - p.stages < 0 ? 0 : issued - p.stages; j < issued; ++j)
            tc::mbar_wait(&full[j % p.stages], (j / p.stages) & 1);
        pdl_launch_dependents();
        return;
    }

    // compute warps: warp w owns groups wg0 .. wg1 - 1 of every strip; lane (g, q)
    const int w = warp, g = lane >> 2, q = lane & 3;
    // the fused transform: every CTA turns its staged rows once, while the first strips
    // are still in flight (visible to all compute warps after the first named barrier)
    if (p.had_L == 8) fwht::staged_rows<DT, 8>(act, p.act_stride, p.had_signs, rows, K, p.had_scale, w, nw, lane);
    else if (p.had_L == 9) fwht::staged_rows<DT, 16>(act, p.act_stride, p.had_signs, rows, K, p.had_scale, w, nw, lane);
    else if (p.had_L == 10) fwht::staged_rows<DT, 32>(act, p.act_stride, p.had_signs, rows, K, p.had_scale, w, nw, lane);
    const int wg0 = p.wg[w], wg1 = p.wg[w + 1];
    const uint2 *lut_lane = lut + (lane & ((1 << LUT_SH) - 1));
    uint32_t *seg = reinterpret_cast<uint32_t *>(smem + p.o_seg);  // [nw][32]
    float *red = reinterpret_cast<float *>(smem + p.o_red);         // [nw][8][32]
    const bool rowok = g < rows;
    const char *arow = act + (size_t)(rowok ? g : 0) * p.act_stride;
    const int cw = nw * 32;
    int it = 0;
    for (int s = blockIdx.x; s < nstrips; s += gridDim.x, ++it) {
        const int st = it % p.stages;
        const bool ok = tc::mbar_wait(&full[st], (it / p.stages) & 1);
        if (!ok) *abort_flag = 1;
        const int n0 = s * 32, ncol = min(32, N - n0);
        const char *sp = smem + p.o_stage + st * p.stage_bytes;
        const uint32_t *sbm = reinterpret_cast<const uint32_t *>(sp);
        const uint16_t *ssc = reinterpret_cast<const uint16_t *>(sp + p.o_sc);
        const uint32_t *ssg = reinterpret_cast<const uint32_t *>(sp + p.o_sg);
        const uint32_t *sh = reinterpret_cast<const uint32_t *>(smem + p.o_meta) + st * 32;
        // non-zeros of this warp's rows per column (lane = column)
        uint32_t cnt = 0;
        if (ok && lane < ncol)
            for (int kp = wg0 * 4; kp < wg1 * 4; ++kp) cnt += __popc(sbm[kp * 32 + lane]);
        seg[w * 32 + lane] = cnt;
        named_bar_sync(1, cw);
        if (*abort_flag) break;  // uniform: read by every compute warp after the same barrier
        uint32_t r0 = 0;
        for (int v = 0; v < w; ++v) r0 += seg[v * 32 + lane];
        const bool colok = 4 * g < ncol;  // ncol is 16 or 32
        uint32_t rcur[4], wb[4];
        const uint32_t *sgc[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            rcur[c] = __shfl_sync(0xffffffffu, r0, 4 * g + c);
            wb[c] = sh[4 * g + c];
            sgc[c] = ssg + slot_base(p.cap, 4 * g + c);
        }

        float acc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
        for (int grp = wg0; grp < wg1; ++grp) {
            uint4 P4 = *reinterpret_cast<const uint4 *>(sbm + (grp * 4 + q) * 32 + 4 * g);
            if (!colok) P4 = make_uint4(0u, 0u, 0u, 0u);
            const uint32_t P[4] = {P4.x, P4.y, P4.z, P4.w};
            // rank of word q within the group: exclusive scan over the 4 q lanes, 4 columns
            // packed in bytes (sums <= 128)
            const uint32_t cnt4 = __popc(P[0]) | (__popc(P[1]) << 8) | (__popc(P[2]) << 16) | (__popc(P[3]) << 24);
            uint32_t x = cnt4;
            uint32_t y = __shfl_up_sync(0xffffffffu, x, 1, 4);
            if (q >= 1) x += y;
            y = __shfl_up_sync(0xffffffffu, x, 2, 4);
            if (q >= 2) x += y;
            const uint32_t excl = x - cnt4;
            const uint32_t tot = __shfl_sync(0xffffffffu, x, 3, 4);
            uint32_t W[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t r = rcur[c] + ((excl >> (8 * c)) & 0xffu);
                const uint32_t l = (r >> 5) + wb[c];
                W[c] = __funnelshift_r(sgc[c][l], sgc[c][l + 1], r & 31u);
                rcur[c] += (tot >> (8 * c)) & 0xffu;
            }

            float part[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int s2 = 0; s2 < 4; ++s2) {
                uint4 av = make_uint4(0u, 0u, 0u, 0u);
                if (rowok) {
                    const int u = grp * 16 + 4 * q + s2;  // rows 32q + 8 s2 .. +7 of the group
                    av = *reinterpret_cast<const uint4 *>(arow + (size_t)(u ^ (((u >> 3) & 1) << 1)) * 16);
                }
                const uint32_t acts[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                for (int hs = 0; hs < 2; ++hs) {
                    const int sn = 2 * s2 + hs;  // nibble sn: rows 32q + 4sn .. 32q + 4sn + 3
                    uint2 e[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t nib4 = sn == 0 ? (P[c] << 4) & 0xf0u : (P[c] >> (4 * sn - 4)) & 0xf0u;
                        e[c] = lut_lane[(nib4 | (W[c] & 0xfu)) << LUT_SH];
                        W[c] >>= __popc(nib4);
                    }
                    const uint32_t bb[2] = {acts[2 * hs], acts[2 * hs + 1]};
                    const uint32_t a0[4] = {e[0].x, e[1].x, e[0].y, e[1].y};
                    const uint32_t a1[4] = {e[2].x, e[3].x, e[2].y, e[3].y};
                    mma16816<DT>(part[0], a0, bb);
                    mma16816<DT>(part[1], a1, bb);
                }
            }
            const uint2 sc = *reinterpret_cast<const uint2 *>(ssc + grp * 32 + 4 * g);
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
        // the stage is read: back to the producer
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[st]);

        // v[h * 4 + i]: activation row 2q + h, column n0 + 4g + i, kept as red[w][h*4+i][lane];
        // warp j < 4 (warp 0 takes the rest when nw < 4) sums column pair j (values 2j,
        // 2j + 1) over the warps in warp order and stores it
        const float v[8] = {acc[0][0], acc[0][2], acc[1][0], acc[1][2], acc[0][1], acc[0][3], acc[1][1], acc[1][3]};
#pragma unroll
        for (int i = 0; i < 8; ++i) red[(w * 8 + i) * 32 + lane] = v[i];
        named_bar_sync(1, cw);
        for (int j = w; j < 4; j += nw) {
            float v0 = 0.0f, v1 = 0.0f;
            for (int v2 = 0; v2 < nw; ++v2) {
                v0 += red[(v2 * 8 + 2 * j) * 32 + lane];
                v1 += red[(v2 * 8 + 2 * j + 1) * 32 + lane];
            }
            const int m = 2 * q + (j >> 1);
            if (colok && m < p.M)
                epi_store2<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, N, m, n0 + 4 * g + 2 * (j & 1), v0, v1);
        }
        named_bar_sync(1, cw);  // red and seg free for the next strip
    }
    pdl_launch_dependents();
}

template <class DT, int POSTOP, bool OUT_F32>
cudaError_t launch_t(const GemvArgs &a, const Params &p, const CUtensorMap &tmB, const CUtensorMap &tmS,
                     int grid) {
    auto kern = p.lut_sh == 4 ? bitcos_gemv_p_kernel<DT, POSTOP, OUT_F32, 4> : bitcos_gemv_p_kernel<DT, POSTOP, OUT_F32, 3>;
    cudaError_t e = ensure_smem(kern, (size_t)p.total);
    if (e != cudaSuccess) return e;
    return launch_kernel(kern, dim3(grid), dim3((p.nw + 1) * 32), (size_t)p.total, a.stream, p, tmB, tmS);
}

// the largest divisor of x (x % 4 == 0 or x <= 256) that is at most 256: TMA box rows
static int box_rows(int x) {
    for (int d = x < 256 ? x : 256; d > 1; --d)
        if (x % d == 0) return d;
    return 1;
}

// Compute warps for G groups: one per group up to 16, else 16 (four per scheduler).
static int pick_nw(int G) { return G < kMaxNW ? G : kMaxNW; }

// Contiguous group ranges of the nw compute warps, sized so that each of the SM's four
// schedulers (warp w issues on scheduler w % 4) gets G/4 groups of a strip (one more for
// the first G % 4): the warps of one strip meet at named barriers, so the strip takes as
// long as the busiest scheduler's share.  (14 warps of 3 groups at G = 42 gave schedulers
// 12, 12, 9 and 9 groups; 16 warps split this way give 11, 11, 10, 10.)
static void split_groups(int G, int nw, int wg[kMaxNW + 1]) {
    int size[kMaxNW] = {};
    for (int sch = 0; sch < 4; ++sch) {
        const int total = G / 4 + (sch < G % 4 ? 1 : 0);
        int cnt = 0;
        for (int w = sch; w < nw; w += 4) ++cnt;
        int j = 0;
        for (int w = sch; w < nw; w += 4, ++j) size[w] = total / cnt + (j < total % cnt ? 1 : 0);
    }
    wg[0] = 0;
    for (int w = 0; w < nw; ++w) wg[w + 1] = wg[w] + size[w];
}

}  // namespace bitcos_p

// The plan for (M, K): 0 when this kernel does not apply (M > 8, or the stages do not fit
// in shared memory even with 2 stages and 8 table copies).
size_t bitcos_gemv_p_smem(int M, int K) {
    using namespace bitcos_p;
    if (M < 1 || M > kMaxRows) return 0;
    bitcos_p::Params p;
    const int nw = pick_nw(K / kGS);
    const int configs[4][2] = {{3, 4}, {2, 4}, {3, 3}, {2, 3}};  // (stages, log2 table copies)
    for (const auto &c : configs) {
        const int t = layout(p, M, K, nw, c[0], c[1]);
        if (t <= 227 * 1024) return (size_t)t;
    }
    return 0;
}

cudaError_t bitcos_gemv_p_launch(const GemvArgs &a, int sms) {
    using namespace bitcos_p;
    Params p;
    const int nw = pick_nw(a.K / kGS);
    const int configs[4][2] = {{3, 4}, {2, 4}, {3, 3}, {2, 3}};
    bool fit = false;
    for (const auto &c : configs) {
        if (layout(p, a.M, a.K, nw, c[0], c[1]) <= 227 * 1024) {
            fit = true;
            break;
        }
    }
    if (!fit || a.M > kMaxRows) return cudaErrorInvalidValue;
    p.A = (const uint16_t *)a.A;
    p.B = a.B;
    p.S = (const uint16_t *)a.S;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.had_L = a.had_hb ? 31 - __builtin_clz((unsigned)a.had_hb) : 0;
    p.had_signs = a.had_signs;
    p.had_scale = a.had_hb ? (float)(1.0 / std::sqrt((double)a.had_hb)) : 1.0f;
    split_groups(p.G, p.nw, p.wg);
    p.box_b = box_rows(p.KW);
    p.box_s = box_rows(p.G);
    CUtensorMap tmB, tmS;
    cudaError_t e = tc::make_map_plain(&tmB, a.B, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, p.KW, a.N, p.box_b, 32);
    if (e != cudaSuccess) return e;
    e = tc::make_map_plain(&tmS, a.S, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.G, a.N, p.box_s, 32);
    if (e != cudaSuccess) return e;
    const int nstrips = (a.N + 31) / 32;
    const int grid = nstrips < sms ? nstrips : sms;
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) {
        using DT = typename decltype(dt)::type;
        return bitcos_p::launch_t<DT, decltype(po)::value, decltype(of)::value>(a, p, tmB, tmS, grid);
    });
}

cudaError_t read_device_error_gemv_bitcos_p(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl

