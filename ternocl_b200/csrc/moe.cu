// int2 MoE prefill, the kernels around the grouped GEMM (int2_moe/int2_moe_prefill.cl):
//
//   route    (int2_moe_route, :29-61)   rows per expert, meta = [E+1 row offsets |
//            E+1 row-tile offsets], perm (sorted row -> routed row g) and inv (g -> row)
//   gather   (int2_moe_gather, :63-70)  Xs[p] = X[perm[p] / topk]
//   combine  (int2_moe_combine, :143-156) O[t, n] = DT(sum_j RW[g] * Y[inv[g], n]),
//            g = t*topk + j, j in increasing order, fp32 sum
//   gather_q (int2_moe_gather_q, int2_moe_prefill_int8.cl:73-84) the int8 variant: int8
//            rows and their per-group activation scales into expert order
//
// The grouped GEMMs themselves are the tcgen05 GEMMs in grouped mode (gemm_tc.cu for
// fp16/bf16 activations, gemm_i8.cu for int8 ones).
//
// Routing: the order of the rows inside an expert is ascending in g (the reference's
// follows its local atomics), so it is deterministic.  Up to 1024 rows one CTA (like
// the reference's single work-group): counts with shared-memory atomics, then a row's
// position is its expert's offset + the count of the same expert in lower warps (a
// 32-step scan per expert) + its rank among the lanes of its warp with the same expert
// (__match_any_sync); beyond that one CTA per 1024 rows (moe_route_mc_kernel).  Expert
// ids outside [0, E) are skipped and flagged in the device error word (bit 1).
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace ternocl {
namespace {

constexpr int kRouteThreads = 1024;

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const int *__restrict__ ids, int *meta,
                                                                 int *perm, int *inv, int G, int E, int rpt) {
    extern __shared__ int sm[];
    int *cnt = sm;          // [E] rows per expert, then the running offset
    int *tot = sm + E;      // [E] this round's rows per expert
    int *wc = sm + 2 * E;   // [32][E] per-warp counts -> exclusive prefix over warps
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    for (int e = tid; e < E; e += kRouteThreads) cnt[e] = 0;
    for (int i = tid; i < 32 * E; i += kRouteThreads) wc[i] = 0;
    __syncthreads();
    bool bad = false;
    for (int g = tid; g < G; g += kRouteThreads) {
        const int e = ids[g];
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
        else bad = true;
    }
    if (bad) atomicOr(&tc::g_device_error, 2u);
    __syncthreads();
    if (tid == 0) {
        int r = 0, t = 0;
        for (int e = 0; e < E; ++e) {
            const int c = cnt[e];
            meta[e] = r;
            meta[E + 1 + e] = t;
            cnt[e] = r;  // running offset of expert e
            r += c;
            t += (c + rpt - 1) / rpt;
        }
        meta[E] = r;
        meta[2 * E + 1] = t;
    }
    __syncthreads();
    for (int base = 0; base < G; base += kRouteThreads) {
        const int g = base + tid;
        int e = g < G ? ids[g] : -1;
        if (e >= E) e = -1;
        // lanes of this warp with the same expert
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (e >= 0 && rank == 0) wc[warp * E + e] = __popc(peers);
        __syncthreads();
        for (int x = tid; x < E; x += kRouteThreads) {
            int acc = 0;
            for (int w = 0; w < 32; ++w) {
                const int c = wc[w * E + x];
                wc[w * E + x] = acc;
                acc += c;
            }
            tot[x] = acc;
        }
        __syncthreads();
        if (e >= 0) {
            const int p = cnt[e] + wc[warp * E + e] + rank;
            perm[p] = g;
            inv[g] = p;
        }
        __syncthreads();
        for (int x = tid; x < E; x += kRouteThreads) cnt[x] += tot[x];
        for (int i = tid; i < 32 * E; i += kRouteThreads) wc[i] = 0;
        __syncthreads();
    }
    pdl_launch_dependents();
}

// Multi-CTA form of the same routing (same outputs): CTA c places rows
// [1024c, 1024c + 1024).  Every CTA histograms all ids (the experts' totals -> their row
// offsets) and the ids before its chunk (its starting offset inside each expert), so no
// scratch memory is needed; CTA 0 writes meta.  Inside the chunk the placement is the
// single-CTA kernel's round.
__global__ void __launch_bounds__(kRouteThreads) moe_route_mc_kernel(const int *__restrict__ ids, int *meta,
                                                                    int *perm, int *inv, int G, int E, int rpt) {
    extern __shared__ int sm[];
    int *tot = sm;          // [E] rows per expert (all G)
    int *base = sm + E;     // [E] first row of this chunk's rows of expert e
    int *wc = sm + 2 * E;   // [32][E]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c0 = blockIdx.x * kRouteThreads;
    pdl_wait();
    for (int e = tid; e < E; e += kRouteThreads) {
        tot[e] = 0;
        base[e] = 0;
    }
    for (int i = tid; i < 32 * E; i += kRouteThreads) wc[i] = 0;
    __syncthreads();
    bool bad = false;
    for (int g = tid; g < G; g += kRouteThreads) {
        const int e = ids[g];
        if (e >= 0 && e < E) {
            atomicAdd(&tot[e], 1);
            if (g < c0) atomicAdd(&base[e], 1);
        } else {
            bad = true;
        }
    }
    if (bad && blockIdx.x == 0) atomicOr(&tc::g_device_error, 2u);
    __syncthreads();
    if (tid == 0) {
        int r = 0, t = 0;
        for (int e = 0; e < E; ++e) {
            const int c = tot[e];
            if (blockIdx.x == 0) {
                meta[e] = r;
                meta[E + 1 + e] = t;
            }
            base[e] += r;
            r += c;
            t += (c + rpt - 1) / rpt;
        }
        if (blockIdx.x == 0) {
            meta[E] = r;
            meta[2 * E + 1] = t;
        }
    }
    __syncthreads();
    const int g = c0 + tid;
    int e = g < G ? ids[g] : -1;
    if (e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wc[warp * E + e] = __popc(peers);
    __syncthreads();
    for (int x = tid; x < E; x += kRouteThreads) {
        int acc = 0;
        for (int w = 0; w < 32; ++w) {
            const int cnt = wc[w * E + x];
            wc[w * E + x] = acc;
            acc += cnt;
        }
    }
    __syncthreads();
    if (e >= 0) {
        const int pos = base[e] + wc[warp * E + e] + rank;
        perm[pos] = g;
        inv[g] = pos;
    }
    pdl_launch_dependents();
}

// one CTA row: Xs[p] = X[perm[p] / topk], 16-byte copies
__global__ void __launch_bounds__(256) moe_gather_kernel(const uint4 *__restrict__ X, const int *__restrict__ perm,
                                                        uint4 *__restrict__ Xs, int G, int K8, int topk) {
    pdl_wait();
    for (int p = blockIdx.x; p < G; p += gridDim.x) {
        const uint4 *src = X + (size_t)(perm[p] / topk) * K8;
        uint4 *dst = Xs + (size_t)p * K8;
        for (int k = threadIdx.x; k < K8; k += blockDim.x) dst[k] = src[k];
    }
    pdl_launch_dependents();
}

// int8 rows and their activation scales into expert order (int2_moe_gather_q,
// int2_moe/int2_moe_prefill_int8.cl:73-84): Xsq[p] = Xq[t], SA[g, p] = SAt[g, t] with
// t = perm[p] / topk and the scale pitches LDSA(T), LDSA(G)
__global__ void __launch_bounds__(256) moe_gather_q_kernel(const uint4 *__restrict__ Xq,
                                                          const uint16_t *__restrict__ SAt,
                                                          const int *__restrict__ perm, uint4 *__restrict__ Xsq,
                                                          uint16_t *__restrict__ SA, int T, int G, int K, int topk) {
    pdl_wait();
    const int K16 = K / 16, ngroups = K / kGS;
    const size_t ldt = (size_t)((T + 31) & ~31), ldg = (size_t)((G + 31) & ~31);
    for (int p = blockIdx.x; p < G; p += gridDim.x) {
        const int t = perm[p] / topk;
        const uint4 *src = Xq + (size_t)t * K16;
        uint4 *dst = Xsq + (size_t)p * K16;
        for (int k = threadIdx.x; k < K16; k += blockDim.x) dst[k] = src[k];
        for (int g = threadIdx.x; g < ngroups; g += blockDim.x) SA[g * ldg + p] = SAt[g * ldt + t];
    }
    pdl_launch_dependents();
}

// thread per (token t, 4 columns)
template <class DT>
__global__ void __launch_bounds__(256) moe_combine_kernel(const float *__restrict__ Y, const int *__restrict__ inv,
                                                         const uint16_t *__restrict__ RW, uint16_t *__restrict__ O,
                                                         int T, int N, int topk) {
    pdl_wait();
    const int n4 = N / 4;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < (long long)T * n4) {
        const int t = (int)(idx / n4), c = (int)(idx % n4) * 4;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int j = 0; j < topk; ++j) {
            const int g = t * topk + j;
            const float w = DT::tof(RW[g]);
            const float4 y = *reinterpret_cast<const float4 *>(Y + (size_t)inv[g] * N + c);
            s0 += w * y.x;
            s1 += w * y.y;
            s2 += w * y.z;
            s3 += w * y.w;
        }
        uint2 o;
        o.x = (uint32_t)DT::fromf(s0) | ((uint32_t)DT::fromf(s1) << 16);
        o.y = (uint32_t)DT::fromf(s2) | ((uint32_t)DT::fromf(s3) << 16);
        *reinterpret_cast<uint2 *>(O + (size_t)t * N + c) = o;
    }
    pdl_launch_dependents();
}

}  // namespace

size_t moe_route_smem(int E) { return (size_t)(2 * E + 32 * E) * sizeof(int); }

cudaError_t moe_route_launch(const int *ids, int *meta, int *perm, int *inv, int G, int E, int rpt,
                             cudaStream_t st) {
    const size_t smem = moe_route_smem(E);
    auto kern = G > kRouteThreads ? moe_route_mc_kernel : moe_route_kernel;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem(kern, smem);
        if (e != cudaSuccess) return e;
    }
    const int ctas = G > kRouteThreads ? (G + kRouteThreads - 1) / kRouteThreads : 1;
    return launch_kernel(kern, dim3(ctas), dim3(kRouteThreads), smem, st, ids, meta, perm, inv, G, E, rpt);
}

cudaError_t moe_gather_launch(const void *X, const int *perm, void *Xs, int G, int K, int topk, cudaStream_t st) {
    const int blocks = G < 148 * 16 ? G : 148 * 16;
    return launch_kernel(moe_gather_kernel, dim3(blocks), dim3(256), 0, st, (const uint4 *)X, perm, (uint4 *)Xs, G,
                         K / 8, topk);
}

cudaError_t moe_gather_q_launch(const int8_t *Xq, const void *SAt, const int *perm, int8_t *Xsq, void *SA, int T,
                                int G, int K, int topk, cudaStream_t st) {
    const int blocks = G < 148 * 16 ? G : 148 * 16;
    return launch_kernel(moe_gather_q_kernel, dim3(blocks), dim3(256), 0, st, (const uint4 *)Xq,
                         (const uint16_t *)SAt, perm, (uint4 *)Xsq, (uint16_t *)SA, T, G, K, topk);
}

cudaError_t moe_combine_launch(const float *Y, const int *inv, const void *RW, void *O, int T, int N, int topk,
                               int dtype, cudaStream_t st) {
    const long long n = (long long)T * (N / 4);
    const dim3 grid((unsigned)((n + 255) / 256));
    if (dtype == TERNOCL_BF16)
        return launch_kernel(moe_combine_kernel<BF16>, grid, dim3(256), 0, st, Y, inv, (const uint16_t *)RW,
                             (uint16_t *)O, T, N, topk);
    return launch_kernel(moe_combine_kernel<F16>, grid, dim3(256), 0, st, Y, inv, (const uint16_t *)RW,
                         (uint16_t *)O, T, N, topk);
}

cudaError_t read_device_error_moe(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

}  // namespace ternocl
