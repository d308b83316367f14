// Persistent int2 decode GEMV for M = 1, an opt-in implementation (TERNOCL_OPT_GEMV_IMPL = 3)
// of int2_fp16_upcvt_gemm (int2_fp16_upcvt.cl:193-290):
//
//   C[0,n] = DT(epi( sum_g S[g,n] * sum_{k in g} A[0,k] * code(B[k,n]) ))
//
// The arithmetic is the integer-MMA scheme of gemv_i2d.cu: int8 weights (one LOP3 per
// four rows, 64 * code_to_value), exact fixed-point activations split into three unsigned
// digit planes plus a plane of ones, mma.sync m16n8k32 s8 x u8 -> s32, exact int32 dots
// per 128-row group recovered as floats through a 1.5 * 2^23 accumulator bias.  Here the
// fixed-point exponent is per 128-row group (E_g of max |A| over the group), folded into
// the group's scales, so every element within 2^11 of its group's maximum is exact.
//
// Work and data movement.  The matrix is cut into tiles of 128 columns and stages of 4
// groups (32 word rows); a (tile, stage) pair is a unit, and the units, tile-major, are
// split into equal contiguous ranges over a persistent grid of 3 CTAs per SM (stream-K).
// Per CTA: warp 4, lane 0 streams its units through a 4-deep ring with TMA -- per stage
// four 2-D boxes of 32 columns x 32 word rows in the 128-byte swizzle layout (one per
// consumer warp) and one box of the 4 x 128 scales -- on mbarriers; warps 0-3 each own
// 32 columns.  While working on unit i, warp w turns group w of unit i+1's activations
// into digit planes (lanes 0-7: one 16-row word row each; three rotating plane buffers,
// one named barrier per unit for the four consumer warps), then decodes and multiplies
// its 32 columns of unit i's four groups as independent accumulator chains.  A CTA whose range covers a tile entirely stores its columns with the
// fused epilogue; a tile split between CTAs gets its fp32 partials summed, in CTA order,
// by the CTA that completes it last (per-tile arrival counter in the workspace).  Without
// a workspace the ranges are whole tiles.  Every mbarrier wait is bounded.
//
// Measured on B200 it is slower than the per-launch kernel of gemv_i2d.cu (Llama-3-8B
// 4096 x 28672: 14.3 us without the split, 21 us with it, against 12.6 us): four consumer
// warps per CTA leave too few warps per scheduler to hide the MMA and shared-memory
// latencies, and a tile split over many CTAs ends in a serial fix-up.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "digit_common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {

namespace {

constexpr int kTileCols = 128;
constexpr int kConsumers = 4;                        // consumer warps, 32 columns each
constexpr int kThreads = (kConsumers + 1) * 32;      // + the producer warp
constexpr int kGroupsPerStage = 4;                   // one per consumer warp (activation conversion)
constexpr int kRowsPerStage = kGroupsPerStage * 8;   // 32 word rows
constexpr int kSliceBytes = kRowsPerStage * 32 * 4;  // a warp's 32 columns: 4 KB, 128-byte swizzle
constexpr int kScaleBytes = kGroupsPerStage * kTileCols * 2;
constexpr int kStageBytes = kConsumers * kSliceBytes + kScaleBytes;  // 17 KB
constexpr int kStages = 4;
constexpr int kPlaneBytes = kGroupsPerStage * 8 * 16;  // one digit plane of a stage

// shared memory map (from a 1024-byte aligned base)
constexpr int kPlaneBufs = 3;                              // digits of stages i, i+1 (and i-1 in flight)
constexpr int kOffPlanes = kStages * kStageBytes;          // [kPlaneBufs][3][kPlaneBytes]
constexpr int kOffFac = kOffPlanes + kPlaneBufs * 3 * kPlaneBytes;  // [kPlaneBufs][kGroupsPerStage] floats
constexpr int kOffFlag = kOffFac + kPlaneBufs * kGroupsPerStage * 4;
constexpr int kOffBars = kOffFlag + 16;
constexpr int kSmemTotal = kOffBars + 2 * kStages * 8 + 1024;  // + alignment slack
constexpr int kCtasPerSm = 3;
static_assert(kStageBytes % 1024 == 0, "swizzled slices on 1024-byte boundaries");

struct PParams {
    const uint16_t *A;
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int N, G, tiles, spt, P, U, split;
    float *ws_part;      // [P][2][kTileCols]
    unsigned *ws_cnt;    // [tiles]
};

using digit::cls;
using digit::imma;
using digit::kMagic;
using digit::kMagicBits;

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(kConsumers * 32) : "memory"); }

// first unit of CTA c
__device__ __forceinline__ int range_lo(const PParams &p, int c) {
    return p.split ? (int)((long long)p.U * c / p.P) : p.spt * (int)((long long)p.tiles * c / p.P);
}
// CTA owning unit u (stream-K ranges)
__device__ __forceinline__ int owner(const PParams &p, int u) {
    return (int)(((long long)u * p.P + p.P - 1) / p.U);
}

template <class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_i2p_kernel(const PParams p, const __grid_constant__ CUtensorMap tmB,
                                                               const __grid_constant__ CUtensorMap tmS) {
    extern __shared__ __align__(1024) char smem_raw[];
    char *smem = smem_raw + ((1024u - (tc::smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int lo = range_lo(p, blockIdx.x), hi = range_lo(p, blockIdx.x + 1);
    const int n = hi - lo;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kOffBars);
    uint64_t *empty = full + kStages;
    float *fac = reinterpret_cast<float *>(smem + kOffFac);
    int *flag = reinterpret_cast<int *>(smem + kOffFlag);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], kConsumers);
        }
        tc::fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---------------- producer: TMA weight and scale stream ----------------
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < n; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !tc::mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) break;
                const int u = lo + i, tile = u / p.spt, stg = u - tile * p.spt;
                char *st = smem + s * kStageBytes;
                tc::mbar_expect_tx(&full[s], kStageBytes);
#pragma unroll
                for (int w = 0; w < kConsumers; ++w)
                    tc::tma_load_2d(st + w * kSliceBytes, &tmB, tile * kTileCols + 32 * w, stg * kRowsPerStage, &full[s]);
                tc::tma_load_2d(st + kConsumers * kSliceBytes, &tmS, tile * kTileCols, stg * kGroupsPerStage, &full[s]);
                ++issued;
            }
            for (int i = issued - kStages < 0 ? 0 : issued - kStages; i < issued; ++i)
                tc::mbar_wait(&full[i % kStages], (i / kStages) & 1);
        }
        return;
    }

    // ---------------- consumers: warp w owns columns 32w .. 32w+31 of the tile ----------------
    const int w = warp;
    pdl_wait();  // A, the workspace and C may come from the previous kernel
    float acc[2][4];
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[b][c] = 0.0f;
    const int first_tile = lo / p.spt;

    // Stores (whole tile) or publishes (split tile) this warp's 32 columns.  Lanes t = 0
    // hold (n = 0: ones, n = 1: digit 0), lanes t = 1 (n = 2, 3: digits 1, 2) of the same
    // columns; the planes recombine to the dot in true units.
    auto flush = [&](int tile) {
        float val[2][2];
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float y2 = __shfl_down_sync(0xffffffffu, acc[b][2 * h], 1);
                const float y3 = __shfl_down_sync(0xffffffffu, acc[b][2 * h + 1], 1);
                val[b][h] = (acc[b][2 * h + 1] + 256.0f * y2) + (65536.0f * y3 - 4194304.0f * acc[b][2 * h]);
            }
        const int col0 = tile * kTileCols + 32 * w + 2 * g;
        int nc = 1, c_first = blockIdx.x;
        if (p.split) {
            c_first = owner(p, tile * p.spt);
            nc = owner(p, (tile + 1) * p.spt - 1) - c_first + 1;
        }
        if (nc == 1) {
            if (t == 0) {
#pragma unroll
                for (int b = 0; b < 2; ++b)
                    if (col0 + 16 * b < p.N)
                        epi_store2<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, 0, col0 + 16 * b, val[b][0],
                                                        val[b][1]);
            }
            return;
        }
        const int which = tile == first_tile ? 0 : 1;
        float *mine = p.ws_part + ((size_t)blockIdx.x * 2 + which) * kTileCols + 32 * w + 2 * g;
        if (t == 0) {
#pragma unroll
            for (int b = 0; b < 2; ++b) __stcg(reinterpret_cast<float2 *>(mine + 16 * b), make_float2(val[b][0], val[b][1]));
            __threadfence();
        }
        consumers_sync();
        if (tid == 0) *flag = atomicAdd(&p.ws_cnt[tile], 1u) == (unsigned)(nc - 1) ? 1 : 0;
        consumers_sync();
        if (!*flag) return;
        __threadfence();
        if (t == 0) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                float s0 = 0.0f, s1 = 0.0f;
                for (int c = c_first; c < c_first + nc; ++c) {
                    const int wc = tile == range_lo(p, c) / p.spt ? 0 : 1;
                    const float2 x = __ldcg(reinterpret_cast<const float2 *>(
                        p.ws_part + ((size_t)c * 2 + wc) * kTileCols + 32 * w + 16 * b + 2 * g));
                    s0 += x.x;
                    s1 += x.y;
                }
                if (col0 + 16 * b < p.N) epi_store2<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, 0, col0 + 16 * b, s0, s1);
            }
        }
        if (tid == 0) p.ws_cnt[tile] = 0u;  // ready for the next call
    };

    // activations of unit lo + i for this warp's group (lanes 0-7: one 16-row word row
    // each), loaded one unit ahead of their conversion so that the L2 latency overlaps
    // the multiplication of the current unit
    auto load_act = [&](int i, uint4 (&r)[2]) {
        r[0] = make_uint4(0u, 0u, 0u, 0u);
        r[1] = r[0];
        if (i >= n || lane >= 8) return;
        const int u = lo + i, stg = u - (u / p.spt) * p.spt;
        const int gi = stg * kGroupsPerStage + w;
        if (gi >= p.G) return;
        const uint4 *src = reinterpret_cast<const uint4 *>(p.A + (size_t)gi * kGS + 16 * lane);
        r[0] = __ldg(src);
        r[1] = __ldg(src + 1);
    };
    // digits of unit lo + i (group stg*4 + w) from its loaded activations into plane
    // buffer i % kPlaneBufs
    auto convert = [&](int i, const uint4 (&r)[2]) {
        const int u = lo + i, stg = u - (u / p.spt) * p.spt, pb = i % kPlaneBufs;
        char *pl = smem + kOffPlanes + pb * 3 * kPlaneBytes;
        const int gi = stg * kGroupsPerStage + w;
        const bool valid = gi < p.G;
        const uint32_t h2[8] = {r[0].x, r[0].y, r[0].z, r[0].w, r[1].x, r[1].y, r[1].z, r[1].w};
        uint32_t mx = digit::absmax_bits(h2);
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const int e = digit::exponent_for<DT>(mx);
        if (lane < 8) {
            uint32_t d0[4], d1[4], d2[4];
            digit::word_digits<DT>(h2, e, d0, d1, d2);
            char *dst = pl + (w * 8 + lane) * 16;
            *reinterpret_cast<uint4 *>(dst) = make_uint4(d0[0], d0[1], d0[2], d0[3]);
            *reinterpret_cast<uint4 *>(dst + kPlaneBytes) = make_uint4(d1[0], d1[1], d1[2], d1[3]);
            *reinterpret_cast<uint4 *>(dst + 2 * kPlaneBytes) = make_uint4(d2[0], d2[1], d2[2], d2[3]);
        }
        // 2^-e / 64 (weights are 64 x code), 0 past K, NaN for a non-finite group
        if (lane == 0) fac[pb * kGroupsPerStage + w] = valid ? digit::inverse_scale<DT>(mx, e) : 0.0f;
    };

    int cur = -1;
    uint4 ra[2], rb[2];  // activations of units i+1 (being converted) and i+2 (in flight)
    load_act(0, ra);
    load_act(1, rb);
    if (n > 0) convert(0, ra);
    for (int i = 0; i < n; ++i) {
        const int u = lo + i, tile = u / p.spt;
        if (tile != cur) {
            if (cur >= 0) flush(cur);
            cur = tile;
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[b][c] = 0.0f;
        }
        // the next unit's digits (plane buffers rotate over three: a warp still
        // multiplying unit i-1 reads a third buffer), then the barrier that publishes
        // unit i's digits of all four groups
        ra[0] = rb[0];
        ra[1] = rb[1];
        load_act(i + 2, rb);
        if (i + 1 < n) convert(i + 1, ra);
        consumers_sync();

        const int s = i % kStages, pb = i % kPlaneBufs;
        const char *pl = smem + kOffPlanes + pb * 3 * kPlaneBytes;
        if (!tc::mbar_wait(&full[s], (i / kStages) & 1)) break;
        const char *slice = smem + s * kStageBytes + w * kSliceBytes;
        const char *scl = smem + s * kStageBytes + kConsumers * kSliceBytes;
        // four groups in flight: independent accumulator chains
        int32_t d[kGroupsPerStage][2][4];
#pragma unroll
        for (int gq = 0; gq < kGroupsPerStage; ++gq) {
            const int rA = 8 * gq + 2 * t, rB = rA + 1;  // word rows of k-blocks t and 4+t
            uint2 wa[2], wb[2];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const int c = 4 * b + (g >> 1);  // 16-byte chunk of columns 16b + 2g, +1
                wa[b] = *reinterpret_cast<const uint2 *>(slice + rA * 128 + ((c ^ (rA & 7)) << 4) + 8 * (g & 1));
                wb[b] = *reinterpret_cast<const uint2 *>(slice + rB * 128 + ((c ^ (rB & 7)) << 4) + 8 * (g & 1));
            }
            // B operand: n = g: 0 ones, 1..3 digit planes 0..2, beyond zero
            uint4 ba, bb;
            if (g >= 1 && g <= 3) {
                const char *src = pl + (g - 1) * kPlaneBytes + (gq * 8 + 2 * t) * 16;
                ba = *reinterpret_cast<const uint4 *>(src);
                bb = *reinterpret_cast<const uint4 *>(src + 16);
            } else {
                const uint32_t k = g == 0 ? 0x01010101u : 0u;
                ba = make_uint4(k, k, k, k);
                bb = ba;
            }
            const uint32_t bA[4] = {ba.x, ba.y, ba.z, ba.w}, bB[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
                for (int c = 0; c < 4; ++c) d[gq][b][c] = (int32_t)kMagicBits;
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int b = 0; b < 2; ++b)
                    imma(d[gq][b], cls(wa[b].x, j), cls(wa[b].y, j), cls(wb[b].x, j), cls(wb[b].y, j), bA[j], bB[j]);
        }
#pragma unroll
        for (int gq = 0; gq < kGroupsPerStage; ++gq) {
            const float f = fac[pb * kGroupsPerStage + gq];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const uint32_t s2 = *reinterpret_cast<const uint32_t *>(scl + (gq * kTileCols + 32 * w + 16 * b + 2 * g) * 2);
                const float s_lo = DT::tof((uint16_t)(s2 & 0xFFFFu)) * f, s_hi = DT::tof((uint16_t)(s2 >> 16)) * f;
                acc[b][0] = fmaf(__int_as_float(d[gq][b][0]) - kMagic, s_lo, acc[b][0]);
                acc[b][1] = fmaf(__int_as_float(d[gq][b][1]) - kMagic, s_lo, acc[b][1]);
                acc[b][2] = fmaf(__int_as_float(d[gq][b][2]) - kMagic, s_hi, acc[b][2]);
                acc[b][3] = fmaf(__int_as_float(d[gq][b][3]) - kMagic, s_hi, acc[b][3]);
            }
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    pdl_launch_dependents();
    if (cur >= 0) flush(cur);
}

// plain (no swizzle) 2-D tensor map of a row-major [rows, cols] matrix, boxes of
// box_rows x box_cols elements
cudaError_t make_map_plain(CUtensorMap *map, const void *base, CUtensorMapDataType type, int elem_bytes, int rows,
                           int cols, int box_rows, int box_cols) {
    tc::EncodeTiledFn fn = tc::encode_tiled_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * (cuuint64_t)elem_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int sm_count_dev() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

// workspace of the stream-K split: [P][2][128] fp32 partials + one counter per tile
size_t int2_gemv_p_workspace(int N) {
    const int tiles = (N + kTileCols - 1) / kTileCols;
    const size_t cnt = ((size_t)tiles * 4 + 255) / 256 * 256;
    return cnt + (size_t)kCtasPerSm * sm_count_dev() * 2 * kTileCols * sizeof(float);
}

cudaError_t int2_gemv_p_launch(const GemvArgs &a) {
    if (a.M != 1 || a.world > 0) return cudaErrorInvalidValue;
    PParams p;
    p.A = (const uint16_t *)a.A;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.N = a.N;
    p.G = a.K / kGS;
    p.tiles = (a.N + kTileCols - 1) / kTileCols;
    p.spt = (p.G + kGroupsPerStage - 1) / kGroupsPerStage;
    p.U = p.tiles * p.spt;
    const int slots = kCtasPerSm * sm_count_dev();
    p.split = a.ws_part != nullptr ? 1 : 0;
    p.P = p.split ? (p.U < slots ? p.U : slots) : (p.tiles < slots ? p.tiles : slots);
    p.ws_part = a.ws_part;
    p.ws_cnt = a.ws_cnt;
    CUtensorMap mB, mS;
    cudaError_t e = tc::make_map_sw128(&mB, a.B, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, a.K / 16, a.N, kRowsPerStage);
    if (e != cudaSuccess) return e;
    e = make_map_plain(&mS, a.S, a.dtype == TERNOCL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       2, p.G, a.N, kGroupsPerStage, kTileCols);
    if (e != cudaSuccess) return e;
    return dispatch_epilogue<GemvArgs>(a, [&](auto dt, auto po, auto of) -> cudaError_t {
        using DT = typename decltype(dt)::type;
        auto kern = gemv_i2p_kernel<DT, decltype(po)::value, decltype(of)::value>;
        cudaError_t err = ensure_smem(kern, kSmemTotal);
        if (err != cudaSuccess) return err;
        return launch_kernel(kern, dim3(p.P), dim3(kThreads), (size_t)kSmemTotal, a.stream, p, mB, mS);
    });
}

cudaError_t read_device_error_gemv_p(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
