// Allocation-free variant of the int2 decode GEMV (ternocl_int2_upcvt_noalloc).
//
// Some callers cannot allocate device memory at the point where they run a GEMV:
// code that executes inside another framework's memory pool, real-time or embedded
// runtimes that forbid allocation after start-up, plugins whose host application owns
// every allocation.  For them this entry point takes the GEMV's split-K scratch
// (fp32 partial sums + arrival counters) from a fixed array in device memory that the
// library declares at file scope, instead of a caller-provided workspace.
//
// Properties:
//  * the array is kNoAllocScratchBytes large and is held by every GPU that loads the
//    library until the process exits;
//  * the first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it, so that first
//    call should come before any stream capture;
//  * every call shares the array and it keeps the last call's contents: the arrival
//    counters are cleared on the stream (cudaMemsetAsync) before each launch, and
//    calls that overlap on the GPU (e.g. on two streams) race on it;
//  * no cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "ternocl.h"

namespace ternocl {
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on first use).
cudaError_t scratch_ptr(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace ternocl

using namespace ternocl;

extern "C" int ternocl_int2_upcvt_noalloc(const void *A, const uint32_t *B, const void *S, void *C,
                                          const void *Other, const void *Bias, int M, int N, int K,
                                          int dtype, int postop, int out_f32, void *stream) {
    // same argument rules as ternocl_int2_upcvt
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (postop < 0 || postop > 4 || (out_f32 != 0 && out_f32 != 1)) return TERNOCL_ERR_ARG;
    if (M < 0 || N <= 0 || K <= 0 || N % 16 || K % kGS) return TERNOCL_ERR_SHAPE;
    if (!A || !B || !S || !C) return TERNOCL_ERR_ARG;
    if ((postop == 1 || postop == 2) && !Other) return TERNOCL_ERR_ARG;
    if (postop == 3 && !Bias) return TERNOCL_ERR_ARG;
    auto al = [](const void *p, size_t a) { return ((uintptr_t)p % a) == 0; };
    if (!al(A, 16) || !al(B, 16) || !al(S, 16) || !al(C, out_f32 ? 16 : 8)) return TERNOCL_ERR_ARG;
    if ((Other && !al(Other, 8)) || (Bias && !al(Bias, out_f32 ? 8 : 4))) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;

    // split-K through the scratch array: as many splits as the GEMV's own plan
    // wants (>= 2 when K has two scale groups), as long as the partials fit
    const int G = K / kGS;
    const size_t tiles = (size_t)((N + 31) / 32) * (size_t)((M + 7) / 8);
    const size_t cnt_bytes = (tiles * sizeof(unsigned) + 255) / 256 * 256;
    int sk = gemv_split_k(M, N, K);
    if (sk < 2) sk = 2;
    if (sk > G) sk = G;
    auto need = [&](int s) { return cnt_bytes + (size_t)s * M * N * sizeof(float); };
    while (sk > 2 && need(sk) > kNoAllocScratchBytes) --sk;
    if (sk >= 2 && need(sk) > kNoAllocScratchBytes) return TERNOCL_ERR_WORKSPACE;  // M*N too large
    if (int2_gemv_smem(M, K, sk) > 227 * 1024) return TERNOCL_ERR_WORKSPACE;

    GemvArgs a;
    a.A = A; a.B = B; a.S = S; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.stream = (cudaStream_t)stream;
    a.SK = sk < 1 ? 1 : sk;
    a.cluster = 0;
    if (a.SK > 1) {
        void *scratch = nullptr;
        cudaError_t e = scratch_ptr(&scratch);
        if (e != cudaSuccess) return report_cuda(e);
        a.ws_cnt = (unsigned *)scratch;
        a.ws_part = (float *)((char *)scratch + cnt_bytes);
        e = cudaMemsetAsync(scratch, 0, cnt_bytes, a.stream);  // counters start at zero
        if (e != cudaSuccess) return report_cuda(e);
    }
    return report_cuda(int2_gemv_launch(a));
}
