// Skeleton shared by the decode GEMVs (int2 / s8xs2 / int1 / BITCOS): CTA work
// split, cp.async weight ring, activation staging, deterministic split-K reduction
// and the fused epilogue store.  A Policy supplies the weight layout specifics.
//
// Work decomposition.  A CTA (4 warps) owns a strip of 32 output columns, 8
// activation rows (grid.z) and a contiguous range of 128-row scale groups
// (grid.y = SK cross-CTA K split); its 4 warps split that range again.  Thread
// (g = lane/4, q = lane%4) owns the MMA fragment rows g and g+8 of the strip's two
// 16-column blocks (4 output columns) and activation row g of the 8.
//
// Memory pipeline.  Each thread streams ITS OWN weight bytes of every group (the
// policy says which) through a kStages-deep cp.async ring in shared memory, so the
// bytes in flight cost no registers; the copies for the first stages are issued
// before griddepcontrol.wait (programmatic dependent launch), i.e. they overlap the
// previous kernel in the stream.  Activations are staged once per CTA, already
// permuted into the MMA fragment order, after that wait.
//
// Determinism.  The 4 warps are reduced in warp order through shared memory.  With
// 1 < SK <= 8 the SK CTAs of a strip form a thread-block cluster: each leaves its
// fp32 partial in its shared memory and cluster rank 0 sums them over distributed
// shared memory in split order.  With SK > 8 each CTA writes its partial tile to a
// global workspace, and the last CTA to arrive for the tile (atomic counter, no
// waiting) sums the SK partials in split order and resets the counter.  Either way
// the summation order is fixed, so results are bitwise reproducible.
#pragma once
#include <cmath>
#include <cuda_runtime.h>

#include "common.cuh"

namespace ternocl {
namespace gemv {

// CTA size: W warps (4, 8 or 16) split the CTA's K range; kWarps/kThreads are the
// default (and the BITCOS kernel's) size
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxWarps = 16;
constexpr int kMaxPeers = 8;  // ranks of a column-sharded GEMV (one NVLink domain)
#ifndef TERNOCL_GEMV_STAGES
#define TERNOCL_GEMV_STAGES 4
#endif
constexpr int kStages = TERNOCL_GEMV_STAGES;  // cp.async ring depth (groups per warp)

struct Params {
    const uint16_t *A;
    const uint32_t *B;
    const uint16_t *S;
    const uint32_t *SR;  // BITCOS slice ranks [ls-1][N] (unused by the other layouts)
    int ls;
    int had_L;               // BITCOS: log2 of the fused FWHT block (0: no transform)
    const int8_t *had_signs;  // its sign vector [K] (null: no sign flip)
    float had_scale;          // 1/sqrt(2^had_L), as the standalone transform
    void *C;
    const uint16_t *Other;
    const void *Bias;
    int M, N, K, SK;
    int cluster;  // 1: the SK CTAs of a strip form one thread-block cluster (SK <= 8)
    float *ws_part;
    unsigned *ws_cnt;
    // s8 x s2: int8 activations (qmode 0) and activation scales SA [K/128, ldsa]
    const int8_t *Aq;
    const uint16_t *SA;
    int ldsa, qmode;
    // column-sharded mode (world > 0): this grid computes columns [n_off, n_off + N) of a
    // C with N_out columns and stores them into its own rank's copy C_peer[rank], which
    // peer_complete then copies into every other rank's copy C_peer[r]; Other and
    // Bias are the full-width arrays.  flag_peer[r] = rank r's flags (one per rank).
    int world, rank, n_off, N_out;
    unsigned epoch;               // 0: kept on the device in flag_peer[rank][world]
    unsigned long long peer_timeout_ns;
    unsigned *done_cnt;
    unsigned *err;  // device error word of the launching library (bit 2: a peer wait timed out)
    void *C_peer[kMaxPeers];
    unsigned *flag_peer[kMaxPeers];
};

// Thread-block cluster helpers (distributed shared memory).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local_addr), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote));
    return v;
}

}  // namespace gemv
}  // namespace ternocl

#include "launch.h"

namespace ternocl {
namespace gemv {

inline Params gemv_params_impl(const GemvArgs &a) {
    Params p{};
    p.A = (const uint16_t *)a.A;
    p.B = a.B;
    p.S = (const uint16_t *)a.S;
    p.SR = a.SR;
    p.ls = a.ls;
    p.had_L = a.had_hb ? 31 - __builtin_clz((unsigned)a.had_hb) : 0;
    p.had_signs = a.had_signs;
    p.had_scale = a.had_hb ? (float)(1.0 / std::sqrt((double)a.had_hb)) : 1.0f;
    p.C = a.C;
    p.Other = (const uint16_t *)a.Other;
    p.Bias = a.Bias;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.SK = a.SK;
    p.cluster = a.cluster;
    p.ws_part = a.ws_part;
    p.ws_cnt = a.ws_cnt;
    p.Aq = a.Aq;
    p.SA = (const uint16_t *)a.SA;
    p.ldsa = (a.M + 31) & ~31;
    p.qmode = a.qmode;
    p.world = a.world;
    p.rank = a.rank;
    p.n_off = a.n_off;
    p.N_out = a.N_out;
    p.epoch = a.epoch;
    p.peer_timeout_ns = (unsigned long long)options().peer_timeout_ms * 1000000ull;
    p.done_cnt = a.done_cnt;
    p.err = a.err;
    for (int r = 0; r < kMaxPeers; ++r) {
        p.C_peer[r] = r < a.world ? a.C_peer[r] : nullptr;
        p.flag_peer[r] = r < a.world ? a.flag_peer[r] : nullptr;
    }
    return p;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Per-thread ring slot of one stage: Policy::kWords16 16-byte weight chunks + one
// 8-byte scale chunk, laid out [chunk][thread] so a warp's accesses are contiguous.
// Policy::read_words hands compute() its kWordRegs 16-byte registers from a stage:
// its own chunks, or (kSharedSlots) chunks copied by other lanes of its warp.
template <class Policy, int W>
struct Ring {
    static constexpr int kThreads = W * 32;
    static constexpr int kStageBytes = (Policy::kWords16 * 16 + 8) * kThreads;
    static constexpr int kBytes = kStages * kStageBytes;
    __device__ static uint4 *words(char *base, int stage, int c, int tid) {
        return reinterpret_cast<uint4 *>(base + stage * kStageBytes + (c * kThreads + tid) * 16);
    }
    __device__ static uint2 *scale(char *base, int stage, int tid) {
        return reinterpret_cast<uint2 *>(base + stage * kStageBytes + Policy::kWords16 * 16 * kThreads + tid * 8);
    }
};

// Bytes per staged activation row: Policy::kActBytesPerK per K element plus a pad
// that staggers the rows across shared-memory banks.
template <class Policy>
__host__ __device__ inline int act_row_bytes(int krange) {
    return krange * Policy::kActBytesPerK + Policy::kActPadBytes;
}

// Bytes of dynamic shared memory for a CTA of W warps that stages `krange` K
// elements of `rows` (<= 8) activation rows.
template <class Policy, int W>
__host__ __device__ inline size_t smem_bytes(int rows, int krange) {
    const size_t act = (size_t)rows * act_row_bytes<Policy>(krange);
    const size_t red = (size_t)W * 32 * 8 * sizeof(float);  // warp partials + CTA partial
    const size_t ring = Ring<Policy, W>::kBytes;
    return (ring > red ? ring : red) + act + Policy::extra_smem(rows, krange);
}

// smem_bytes for a runtime warp count
template <class Policy>
inline size_t smem_bytes_w(int warps, int rows, int krange) {
    return warps >= 16 ? smem_bytes<Policy, 16>(rows, krange)
                       : warps >= 8 ? smem_bytes<Policy, 8>(rows, krange) : smem_bytes<Policy, 4>(rows, krange);
}

// Reduction over the CTA's K-split warps (in warp order, through `smem`, >= 8 KB),
// then over the SK CTAs of the strip (cluster DSMEM or workspace, in split order),
// and the epilogue store.  v[h*4 + i] = this thread's partial for activation row
// mb+2q+h and column n0 + ColMap::thread_col(g, i).  Callers synchronise the CTA
// before reusing `smem`.
template <class ColMap, int W, class DT, int POSTOP, bool OUT_F32>
__device__ __forceinline__ void finish(const Params &p, char *smem, float v[8], bool colok) {
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q = lane & 3;
    const int n0 = blockIdx.x * 32;
    const int mb = blockIdx.z * 8;
    const int sk = blockIdx.y;
    float(*red)[32][8] = reinterpret_cast<float(*)[32][8]>(smem);  // [W][lane][8]
    if (warp > 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) red[warp - 1][lane][i] = v[i];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int w = 0; w < W - 1; ++w)
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] += red[w][lane][i];
    }

    int cols[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) cols[i] = n0 + ColMap::thread_col(g, i);

    auto store = [&]() {
        if (p.world > 0) {  // column-sharded: this rank's columns into its own copy of C
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = mb + 2 * q + h;
                if (m < p.M) {
                    void *Cl = p.C_peer[p.rank];
                    epi_store2<DT, POSTOP, OUT_F32>(Cl, p.Other, p.Bias, p.N_out, m, p.n_off + cols[0], v[4 * h],
                                                    v[4 * h + 1]);
                    epi_store2<DT, POSTOP, OUT_F32>(Cl, p.Other, p.Bias, p.N_out, m, p.n_off + cols[2], v[4 * h + 2],
                                                    v[4 * h + 3]);
                }
            }
            return;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = mb + 2 * q + h;
            if (m < p.M) {
                if (ColMap::kContiguousCols) {
                    epi_store2<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, m, cols[0], v[4 * h], v[4 * h + 1]);
                    epi_store2<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, m, cols[2], v[4 * h + 2], v[4 * h + 3]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        epi_store<DT, POSTOP, OUT_F32>(p.C, p.Other, p.Bias, p.N, m, cols[i], v[4 * h + i]);
                }
            }
        }
    };

    if (p.SK == 1) {
        if (warp == 0 && colok) store();
        return;
    }
    if (p.cluster) {
        // split-K across the CTAs of a cluster: partials through distributed shared
        // memory, summed by cluster rank 0 in rank (= K split) order
        float *mine = &red[W - 1][lane][0];
        if (warp == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) mine[i] = v[i];
        }
        cluster_sync_all();
        if (cluster_ctarank() == 0 && warp == 0) {
            const uint32_t la = smem_u32(mine);
            for (int r = 1; r < p.SK; ++r) {
                const float4 x0 = ld_dsmem_f4(la, (uint32_t)r);
                const float4 x1 = ld_dsmem_f4(la + 16, (uint32_t)r);
                v[0] += x0.x; v[1] += x0.y; v[2] += x0.z; v[3] += x0.w;
                v[4] += x1.x; v[5] += x1.y; v[6] += x1.z; v[7] += x1.w;
            }
            if (colok) store();
        }
        cluster_sync_all();  // keep every CTA's partial alive until rank 0 has read it
        return;
    }
    if (warp != 0) return;
    if (colok) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = mb + 2 * q + h;
            if (m < p.M) {
#pragma unroll
                for (int i = 0; i < 4; ++i) __stcg(p.ws_part + ((size_t)sk * p.M + m) * p.N + cols[i], v[4 * h + i]);
            }
        }
    }
    __threadfence();
    __syncwarp();
    const unsigned tile = blockIdx.z * gridDim.x + blockIdx.x;
    unsigned last = 0;
    if (lane == 0) last = (atomicAdd(&p.ws_cnt[tile], 1u) == (unsigned)(p.SK - 1)) ? 1u : 0u;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    if (colok) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = mb + 2 * q + h;
            if (m < p.M) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float t = 0.0f;
                    for (int s = 0; s < p.SK; ++s) t += __ldcg(p.ws_part + ((size_t)s * p.M + m) * p.N + cols[i]);
                    v[4 * h + i] = t;
                }
            }
        }
        store();
    }
    if (lane == 0) p.ws_cnt[tile] = 0u;  // ready for the next call
}

// acquire-release fences (lighter than the sequentially consistent __threadfence*)
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;\n" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;\n" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys(unsigned *ptr, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;\n" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned *ptr) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t gtimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// Column-sharded completion.  Every CTA has stored its columns into this rank's own copy
// of C; after a CTA barrier one thread makes them visible on the GPU (fence) and counts
// the CTA in.  The last CTA of the grid copies the rank's whole column slice (M rows x N
// columns, esz bytes each, in 16-byte pieces) into every other rank's copy over peer
// stores; after a CTA barrier one thread makes those stores visible to the system (one
// acquire-release fence at system scope, cumulative over the CTA's stores, as a grid
// barrier does at GPU scope), writes the call's epoch into its slot of every rank's flags (relaxed system-
// scope stores), polls until every rank has written that epoch into this rank's flags
// (relaxed system-scope loads) and then fences again (acquire), so the launch completes
// only when the whole of C has arrived.  With p.epoch == 0 the epoch is the rank's own
// call count, kept in flag_peer[rank][world] and bumped here (the same sequence on every
// rank, and no host value in the launch: a graph replays it).  The wait gives up after
// p.peer_timeout_ns (error word bit 2) and the kernel returns.
template <class P>
__device__ __forceinline__ void peer_complete(const P &p, unsigned *err, int esz) {
    __shared__ unsigned s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_acq_rel_gpu();  // release: the CTA's stores of this rank's slice
        const unsigned total = gridDim.x * gridDim.y * gridDim.z;
        s_last = atomicAdd(p.done_cnt, 1u) == total - 1 ? 1u : 0u;
        if (s_last) fence_acq_rel_gpu();  // acquire: every CTA's stores
    }
    __syncthreads();
    if (!s_last) return;
    const size_t row_bytes = (size_t)p.N * esz, pitch = (size_t)p.N_out * esz, off = (size_t)p.n_off * esz;
    const int pieces = (int)(row_bytes / 16), total_pieces = pieces * p.M;
    const char *src = reinterpret_cast<const char *>(p.C_peer[p.rank]);
    for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        char *dst = reinterpret_cast<char *>(p.C_peer[r]);
        for (int i = threadIdx.x; i < total_pieces; i += blockDim.x) {
            const int m = i / pieces, c = i - m * pieces;
            const size_t o = (size_t)m * pitch + off + (size_t)c * 16;
            *reinterpret_cast<uint4 *>(dst + o) = __ldcg(reinterpret_cast<const uint4 *>(src + o));
        }
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    fence_acq_rel_sys();  // release: the CTA's peer stores, visible to the system before the flags
    *p.done_cnt = 0u;        // ready for the next launch
    unsigned epoch = p.epoch;
    if (epoch == 0u) {
        unsigned *count = p.flag_peer[p.rank] + p.world;
        epoch = *count + 1u;
        *count = epoch;
    }
    for (int r = 0; r < p.world; ++r) st_relaxed_sys(p.flag_peer[r] + p.rank, epoch);
    const unsigned *mine = p.flag_peer[p.rank];
    const uint64_t t0 = gtimer_ns();
    for (int r = 0; r < p.world; ++r) {
        uint32_t i = 0;
        while ((int)(ld_relaxed_sys(mine + r) - epoch) < 0) {
            if ((++i & 255u) == 0 && gtimer_ns() - t0 > p.peer_timeout_ns) {
                atomicOr(err, 4u);
                return;
            }
        }
    }
    fence_acq_rel_sys();  // acquire: the peers' slices before the launch completes
}

template <class Policy, int W, class DT, int POSTOP, bool OUT_F32>
__global__ void __launch_bounds__(W * 32) gemv_kernel(const Params p) {
    using R = Ring<Policy, W>;
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q = lane & 3;
    const int n0 = blockIdx.x * 32;
    const int mb = blockIdx.z * 8;
    const int G = p.K / kGS;
    const int sk = blockIdx.y;
    const int cg0 = (int)((long long)G * sk / p.SK), cg1 = (int)((long long)G * (sk + 1) / p.SK);
    const int ng = cg1 - cg0;
    const int wg0 = cg0 + ng * warp / W, wg1 = cg0 + ng * (warp + 1) / W;
    const int rows = min(8, p.M - mb);
    const int krange = ng * kGS;
    const bool colok = n0 + Policy::thread_col0(g) < p.N;  // N % 16 == 0

    char *ring = smem;
    char *act = smem + (R::kBytes > W * 32 * 8 * 4 ? R::kBytes : W * 32 * 8 * 4);
    const int act_stride = act_row_bytes<Policy>(krange);
    char *extra = act + (size_t)rows * act_stride;

    // weight stream of this warp's groups [wg0, wg1): pointers advance by one group per issue
    const int nwg = wg1 - wg0;
    const uint32_t *wsrc = Policy::word_ptr(p, wg0, g, q, n0);
    const uint16_t *ssrc = p.S + (size_t)wg0 * p.N + n0 + Policy::thread_col0(g);
    const size_t wstride = Policy::group_stride(p), cstride = Policy::chunk_stride(p);
    int issued = 0;
    const bool copyok = Policy::copy_ok(p.N, n0, g);  // this lane's weight chunks exist
    auto issue = [&]() {
        if (issued < nwg) {
            const int stage = issued & (kStages - 1);
            if (copyok) {
#pragma unroll
                for (int c = 0; c < Policy::kWords16; ++c)
                    cp_async16(R::words(ring, stage, c, tid), wsrc + c * cstride);
            }
            if (colok) cp_async8(R::scale(ring, stage, tid), ssrc);
        }
        cp_async_commit();
        wsrc += wstride;
        ssrc += p.N;
        ++issued;
    };
    static_assert((kStages & (kStages - 1)) == 0, "ring depth must be a power of two");

#pragma unroll
    for (int i = 0; i < kStages - 1; ++i) issue();
    pdl_wait();
    Policy::template stage<DT>(p, act, act_stride, extra, mb, rows, cg0, ng);
    __syncthreads();

    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    const bool rowok = g < rows;
    const char *arow = act + (size_t)(rowok ? g : 0) * act_stride + (size_t)(wg0 - cg0) * Policy::kActGroupBytes;
    const char *xg = extra + (size_t)(wg0 - cg0) * Policy::kExtraGroupBytes;
    for (int i = 0; i < nwg; ++i) {
        cp_async_wait<kStages - 2>();
        // a policy that reads other lanes' ring slots needs their copies visible, and
        // keeps every lane's reads of the previous stage before this iteration's issue
        if (Policy::kSharedSlots) __syncwarp();
        const int stage = i & (kStages - 1);
        uint4 w[Policy::kWordRegs];
        Policy::read_words(ring + stage * R::kStageBytes, tid, W * 32, w);
        const uint2 sc = *R::scale(ring, stage, tid);
        Policy::template compute<DT>(w, sc, arow, rowok, q, xg, acc, g);
        arow += Policy::kActGroupBytes;
        xg += Policy::kExtraGroupBytes;
        issue();
    }
    cp_async_wait<0>();
    pdl_launch_dependents();

    float v[8];
    Policy::thread_values(acc, v);  // v[h*4 + i]: activation row mb+2q+h, column col(i)
    __syncthreads();  // the ring is reused for the reduction
    finish<Policy, W, DT, POSTOP, OUT_F32>(p, smem, v, colok);
    if (p.world > 0) peer_complete(p, p.err, OUT_F32 ? 4 : 2);
}

}  // namespace gemv
}  // namespace ternocl
