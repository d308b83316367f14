// int2 upconvert decode GEMV on the 5th-generation tensor cores (tcgen05 + TMEM),
// replaces int2_fp16_upcvt_gemm (int2_fp16_upcvt.cl:193-290):
//
//   C[m,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[m,k] * code(B[k,n]) ))
//
// The MMA is transposed ("swap AB"): the 128 weight columns of a CTA are the M=128
// rows of a tcgen05.mma kind::f16 whose A operand lives in tensor memory, and the
// (up to 16) activation rows are its N=16 columns, read from shared memory.
//
//  * Thread t of the CTA owns output column n0+t = TMEM lane t.  Per 128-row scale
//    group it streams its column's 8 packed words (rows kp = 8g..8g+7) and the
//    group's scales through a cp.async ring (a warp reads 128 contiguous bytes per
//    word row); the first ring stages are issued before griddepcontrol.wait.
//  * A word is decoded in registers (one LOP3 + one HSUB2 per pair of weights,
//    pair p = rows p and p+8) and written to its TMEM lane with tcgen05.st: TMEM
//    column 8j+p of a buffer holds pair p of the j-th word, i.e. logical K 2p, 2p+1
//    of MMA j.  The activation rows are staged once per CTA in shared memory in the
//    same permuted K order (core-matrix layout, no swizzle).
//  * Half a group (4 words = 4 MMAs of K=16) is decoded into one of two TMEM A
//    buffers while the tensor core consumes the other; one elected thread issues
//    the MMAs into one of two TMEM accumulators D (128 x 16 fp32) and commits them
//    to mbarriers.  When a group's D is complete, each thread loads its lane
//    (tcgen05.ld) and adds D * S[g, n] to its fp32 accumulators -- the host gold's
//    `acc += partial * S` (int2_fp16_upcvt/main.cpp:94).
//  * K is split over SK CTAs (grid.y).  With SK <= 16 they form a thread-block
//    cluster and reduce through distributed shared memory in split order; beyond
//    that through a global workspace (last-arriving CTA sums in split order).
//    Either way the summation order is fixed: results are bitwise reproducible.
//  * Every mbarrier wait is bounded (tc::mbar_wait); a timeout sets the device
//    error word instead of hanging.
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv_common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {

namespace {

// CTA = 4 decode warps (128 threads: thread t owns output column n0+t = TMEM lane t)
//     + 1 control warp (TMEM allocation, weight bulk copies, MMA issue).
constexpr int kDecodeThreads = 128;
constexpr int kThreads = kDecodeThreads + 32;
constexpr int kCtrl = kDecodeThreads;  // control thread
constexpr int kCols = 128;             // output columns per CTA
constexpr int kStages = 6;             // weight ring depth (groups)
constexpr int kStageBytes = 8 * kCols * 4 + kCols * 2;  // 8 word rows + scale row
constexpr int kABufs = 3;              // TMEM A ring: 3 x 32 columns (4 K=16 slices each)
constexpr int kTmemCols = 128;         // A [0,96)  D0 [96,112)  D1 [112,128)
constexpr int kD0 = 96;

struct TcParams {
    const uint16_t *A;
    const uint32_t *B;
    const uint16_t *S;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K, SK, cluster, postop, out_f32;
    float *ws_part;
    unsigned *ws_cnt;
};

// shared memory: [0,256) TMEM slot + mbarriers | weight ring | activation slices
constexpr int kOffRing = 256;
constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kOffAct = (kOffRing + kRingBytes + 127) / 128 * 128;
// One K=16 activation slice in the no-swizzle K-major core-matrix layout: rows
// 0..7 x (K 0..7 | K 8..15); with <= 8 activation rows the MMA's rows 8..15 alias
// rows 0..7 (SBO = 0) and their accumulator columns are ignored.
__host__ __device__ constexpr int slice_bytes(int mrows) { return mrows > 8 ? 512 : 256; }
__host__ __device__ inline size_t tc_smem_bytes(int mrows, int max_ng) {
    return (size_t)kOffAct + (size_t)max_ng * 8 * slice_bytes(mrows);
}

template <class DT, int JP>
__device__ __forceinline__ uint32_t dec_pair(uint32_t x) {
    constexpr uint32_t both = (3u << (2 * JP)) * 0x00010001u;
    constexpr uint32_t magic = DT::kBF16 ? ((uint32_t)(134 - 2 * JP) << 7) : ((uint32_t)(25 - 2 * JP) << 10);
    constexpr uint32_t k1 = (magic | (1u << (2 * JP))) * 0x00010001u;
    uint32_t r, v;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;\n" : "=r"(r) : "r"(x), "n"(both), "r"(k1));
    if constexpr (DT::kBF16) asm("sub.rn.bf16x2 %0, %1, %2;\n" : "=r"(v) : "r"(k1), "r"(r));
    else asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(v) : "r"(k1), "r"(r));
    return v;
}

// all 8 pairs of a word into out[0..7] (pair p = rows p, p+8)
template <class DT>
__device__ __forceinline__ void dec_word(uint32_t x, uint32_t *out) {
    if constexpr (DT::kBF16) {
        const uint32_t y1 = x >> 6, y2 = x >> 12;
        out[0] = dec_pair<DT, 0>(x); out[1] = dec_pair<DT, 1>(x); out[2] = dec_pair<DT, 2>(x);
        out[3] = dec_pair<DT, 0>(y1); out[4] = dec_pair<DT, 1>(y1); out[5] = dec_pair<DT, 2>(y1);
        out[6] = dec_pair<DT, 0>(y2); out[7] = dec_pair<DT, 1>(y2);
    } else {
        const uint32_t y = x >> 10;
        out[0] = dec_pair<DT, 0>(x); out[1] = dec_pair<DT, 1>(x); out[2] = dec_pair<DT, 2>(x);
        out[3] = dec_pair<DT, 3>(x); out[4] = dec_pair<DT, 4>(x);
        out[5] = dec_pair<DT, 0>(y); out[6] = dec_pair<DT, 1>(y); out[7] = dec_pair<DT, 2>(y);
    }
}

template <class DT>
__device__ __forceinline__ void store_out(const TcParams &p, int m, int n, float v) {
    const size_t i = (size_t)m * p.N + n;
    switch (p.postop) {
    case 1: v = v * sigmoid_x(v) * DT::tof(p.Other[i]); break;
    case 2: v = v + DT::tof(p.Other[i]); break;
    case 3:
        v = v + (p.out_f32 ? reinterpret_cast<const float *>(p.Bias)[n]
                           : DT::tof(reinterpret_cast<const uint16_t *>(p.Bias)[n]));
        break;
    case 4: v = sigmoid_x(v); break;
    default: break;
    }
    if (p.out_f32) reinterpret_cast<float *>(p.C)[i] = v;
    else reinterpret_cast<uint16_t *>(p.C)[i] = DT::fromf(v);
}

struct Bars {
    uint64_t wFull[kStages], wEmpty[kStages];  // weight ring: bytes landed / stage released
    uint64_t aFull[kABufs], aFree[kABufs];     // TMEM A ring: decoded / consumed by the MMAs
    uint64_t dFull[2], dFree[2];               // accumulators: complete / read by the decode warps
};
static_assert(sizeof(Bars) + 8 <= kOffRing, "barrier area");

template <class DT, int MROWS>
__global__ void __launch_bounds__(kThreads) int2_gemv_tc_kernel(const TcParams p) {
    extern __shared__ __align__(1024) char smem[];
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem);
    Bars &bar = *reinterpret_cast<Bars *>(smem + 8);
    char *ring = smem + kOffRing;
    char *act = smem + kOffAct;
    constexpr int kSlice = slice_bytes(MROWS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kCols;
    const int ncols = min(kCols, p.N - n0);
    const int mb = blockIdx.z * MROWS;
    const int G = p.K / kGS;
    const int sk = blockIdx.y;
    const int cg0 = (int)((long long)G * sk / p.SK), cg1 = (int)((long long)G * (sk + 1) / p.SK);
    const int ng = cg1 - cg0;
    const int rows = min(MROWS, p.M - mb);
    const uint32_t stage_tx = (uint32_t)ncols * (8 * 4 + 2);

    // control thread: weight rows of group r -> ring stage r % kStages (bulk copies)
    auto load_group = [&](int r) {
        const int grp = cg0 + r, st = r % kStages;
        char *dst = ring + st * kStageBytes;
        tc::mbar_expect_tx(&bar.wFull[st], stage_tx);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            tc::bulk_g2s(dst + i * kCols * 4, p.B + (size_t)(grp * 8 + i) * p.N + n0, (uint32_t)ncols * 4,
                         &bar.wFull[st]);
        tc::bulk_g2s(dst + 8 * kCols * 4, p.S + (size_t)grp * p.N + n0, (uint32_t)ncols * 2, &bar.wFull[st]);
    };

    if (tid == kCtrl) {
#pragma unroll
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&bar.wFull[i], 1);
            tc::mbar_init(&bar.wEmpty[i], kDecodeThreads / 32);
        }
#pragma unroll
        for (int i = 0; i < kABufs; ++i) {
            tc::mbar_init(&bar.aFull[i], kDecodeThreads / 32);
            tc::mbar_init(&bar.aFree[i], 1);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&bar.dFull[i], 1);
            tc::mbar_init(&bar.dFree[i], kDecodeThreads / 32);
        }
        tc::fence_mbar_init();
        // the weights do not depend on the previous kernel: start streaming them now
        for (int r = 0; r < kStages && r < ng; ++r) load_group(r);
    }
    pdl_wait();

    // ---- setup: TMEM (control warp), activation slices (everyone) ---------------------
    if (warp == kCtrl / 32) tc::tmem_alloc(tslot, kTmemCols);
    {
        // slice w (word kp = 8cg0 + w), row m: chunk 0 = pairs 0..3, chunk 1 = pairs 4..7
        const int nw = ng * 8;
        for (int it = tid; it < rows * nw; it += kThreads) {
            const int m = it / nw, w = it - m * nw;
            const uint16_t *src = p.A + (size_t)(mb + m) * p.K + (size_t)(cg0 * 8 + w) * 16;
            const uint4 lo = __ldg(reinterpret_cast<const uint4 *>(src));
            const uint4 hi = __ldg(reinterpret_cast<const uint4 *>(src + 8));
            uint4 c0, c1;
            c0.x = __byte_perm(lo.x, hi.x, 0x5410);
            c0.y = __byte_perm(lo.x, hi.x, 0x7632);
            c0.z = __byte_perm(lo.y, hi.y, 0x5410);
            c0.w = __byte_perm(lo.y, hi.y, 0x7632);
            c1.x = __byte_perm(lo.z, hi.z, 0x5410);
            c1.y = __byte_perm(lo.z, hi.z, 0x7632);
            c1.z = __byte_perm(lo.w, hi.w, 0x5410);
            c1.w = __byte_perm(lo.w, hi.w, 0x7632);
            char *s = act + (size_t)w * kSlice + (m >> 3) * 256 + (m & 7) * 16;
            *reinterpret_cast<uint4 *>(s) = c0;
            *reinterpret_cast<uint4 *>(s + 128) = c1;
        }
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tslot;

    float acc[MROWS];
#pragma unroll
    for (int m = 0; m < MROWS; ++m) acc[m] = 0.0f;

    if (tid == kCtrl) {
        // ---- control: MMA issue ------------------------------------------------------
        constexpr uint32_t idesc = tc::idesc_f16(DT::kBF16, 128, 16);
        const uint32_t act_s = tc::smem_addr(act);
        for (int r = 0; r < ng; ++r) {
            const int d = r & 1;
            if (r >= 2) tc::mbar_wait(&bar.dFree[d], (uint32_t)(((r - 2) >> 1) & 1));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 2 * r + h, a = i % kABufs, u = i / kABufs;
                tc::mbar_wait(&bar.aFull[a], (uint32_t)(u & 1));
                tc::fence_after_sync();
                if (h == 0 && r + kStages < ng) {
                    // stage r % kStages was released when the decode warps read group r
                    tc::mbar_wait(&bar.wEmpty[r % kStages], (uint32_t)((r / kStages) & 1));
                    load_group(r + kStages);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t slice = (uint32_t)(r * 8 + 4 * h + j);
                    const uint64_t bdesc =
                        tc::sdesc_kmajor_noswz(act_s + slice * kSlice, 128, MROWS > 8 ? 256 : 0);
                    tc::mma_ts_f16(tmem + kD0 + 16 * d, tmem + 32 * a + 8 * j, bdesc, idesc,
                                   (h | j) != 0 ? 1u : 0u);
                }
                tc::mma_commit(&bar.aFree[a]);
            }
            tc::mma_commit(&bar.dFull[d]);
        }
    } else if (tid < kDecodeThreads) {
        // ---- decode warps ----------------------------------------------------------------
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float sc_prev = 0.0f;
        auto consume_d = [&](int q, float sc) {  // acc += D(group q) * S
            tc::mbar_wait(&bar.dFull[q & 1], (uint32_t)((q >> 1) & 1));
            tc::fence_after_sync();
            float dv[MROWS];
            tc::tmem_ld<MROWS>(tmem + lane_base + kD0 + 16 * (q & 1), dv);
            tc::tmem_wait_ld();
#pragma unroll
            for (int m = 0; m < MROWS; ++m) acc[m] += dv[m] * sc;
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bar.dFree[q & 1]);
        };
        for (int r = 0; r < ng; ++r) {
            const int st = r % kStages;
            tc::mbar_wait(&bar.wFull[st], (uint32_t)((r / kStages) & 1));
            const uint32_t *wrow = reinterpret_cast<const uint32_t *>(ring + st * kStageBytes);
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = wrow[i * kCols + tid];
            const float sc = DT::tof(reinterpret_cast<const uint16_t *>(wrow + 8 * kCols)[tid]);
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bar.wEmpty[st]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 2 * r + h, a = i % kABufs, u = i / kABufs;
                if (u >= 1) tc::mbar_wait(&bar.aFree[a], (uint32_t)((u - 1) & 1));
                uint32_t regs[32];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) dec_word<DT>(w[4 * h + wi], &regs[8 * wi]);
                tc::tmem_st32(tmem + lane_base + 32 * a, regs);
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&bar.aFull[a]);
            }
            if (r >= 1) consume_d(r - 1, sc_prev);
            sc_prev = sc;
        }
        consume_d(ng - 1, sc_prev);
    }
    pdl_launch_dependents();

    // ---- split-K reduction + epilogue (decode threads own the columns) -----------------
    const int col = n0 + tid;
    const bool owner = tid < kDecodeThreads && tid < ncols;
    float *red = reinterpret_cast<float *>(ring);  // ring is idle now
    __syncthreads();
    if (p.SK == 1) {
        if (owner)
            for (int m = 0; m < rows; ++m) store_out<DT>(p, mb + m, col, acc[m]);
    } else if (p.cluster) {
        if (tid < kDecodeThreads) {
#pragma unroll
            for (int m = 0; m < MROWS; ++m) red[m * kDecodeThreads + tid] = acc[m];
        }
        gemv::cluster_sync_all();
        if (gemv::cluster_ctarank() == 0 && tid < kDecodeThreads) {
            for (int s = 1; s < p.SK; ++s) {
#pragma unroll
                for (int m = 0; m < MROWS; ++m) {
                    uint32_t remote;
                    float x;
                    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n"
                                 : "=r"(remote)
                                 : "r"(tc::smem_addr(&red[m * kDecodeThreads + tid])), "r"(s));
                    asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(x) : "r"(remote));
                    acc[m] += x;
                }
            }
            if (owner)
                for (int m = 0; m < rows; ++m) store_out<DT>(p, mb + m, col, acc[m]);
        }
        gemv::cluster_sync_all();
    } else {
        if (owner)
            for (int m = 0; m < rows; ++m) __stcg(p.ws_part + ((size_t)sk * p.M + mb + m) * p.N + col, acc[m]);
        __threadfence();
        __syncthreads();
        __shared__ unsigned s_last;
        const unsigned tile = blockIdx.z * gridDim.x + blockIdx.x;
        if (tid == 0) s_last = (atomicAdd(&p.ws_cnt[tile], 1u) == (unsigned)(p.SK - 1)) ? 1u : 0u;
        __syncthreads();
        if (s_last) {
            __threadfence();
            if (owner) {
                for (int m = 0; m < rows; ++m) {
                    float t = 0.0f;
                    for (int s = 0; s < p.SK; ++s) t += __ldcg(p.ws_part + ((size_t)s * p.M + mb + m) * p.N + col);
                    store_out<DT>(p, mb + m, col, t);
                }
            }
            if (tid == 0) p.ws_cnt[tile] = 0u;
        }
    }

    // ---- teardown: every MMA has completed (the last accumulator was waited on) --------
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kCtrl / 32) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

template <class DT, int MROWS>
cudaError_t launch_tc(const GemvArgs &a) {
    TcParams p{(const uint16_t *)a.A, a.B, (const uint16_t *)a.S, a.C, (const uint16_t *)a.Other, a.Bias,
               a.M, a.N, a.K, a.SK, a.cluster, a.postop, a.out_f32, a.ws_part, a.ws_cnt};
    const int G = a.K / kGS;
    const int max_ng = (G + a.SK - 1) / a.SK;
    const size_t smem = tc_smem_bytes(MROWS, max_ng);
    auto kern = int2_gemv_tc_kernel<DT, MROWS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(smem < 46 * 1024 ? 46 * 1024 : smem));
    if (e != cudaSuccess) return e;
    if (a.cluster && a.SK > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    dim3 grid((a.N + kCols - 1) / kCols, a.SK, (a.M + MROWS - 1) / MROWS);
    // at most 4 CTAs per SM (4 x 128 TMEM columns): never wait in tcgen05.alloc
    const size_t smem_min = 46 * 1024;
    const size_t smem_launch = smem < smem_min ? smem_min : smem;
    return launch_kernel_cluster(kern, grid, dim3(kThreads), smem_launch, a.stream, dim3(1, a.cluster ? a.SK : 1, 1), p);
}

template <class DT>
cudaError_t launch_rows(const GemvArgs &a) {
    switch (tc_gemv_rows(a.M)) {
    case 1: return launch_tc<DT, 1>(a);
    case 2: return launch_tc<DT, 2>(a);
    case 4: return launch_tc<DT, 4>(a);
    case 8: return launch_tc<DT, 8>(a);
    default: return launch_tc<DT, 16>(a);
    }
}

}  // namespace

int tc_gemv_rows(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16; }

size_t int2_gemv_tc_smem(int M, int K, int SK) {
    const int G = K / kGS;
    return tc_smem_bytes(tc_gemv_rows(M), (G + SK - 1) / SK);
}

cudaError_t int2_gemv_tc_launch(const GemvArgs &a) {
    if (a.dtype == TERNOCL_BF16) return launch_rows<BF16>(a);
    return launch_rows<F16>(a);
}

cudaError_t read_device_error_gemv_tc(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
