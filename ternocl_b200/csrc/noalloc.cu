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
//    call should come before any stream capture; the cached address belongs to the
//    device's context of that moment, so resetting the device (cudaDeviceReset) while
//    the library stays loaded is not supported;
//  * the GEMV is the one ternocl_int2_upcvt plans for a workspace of the array's size
//    (with the same kernel, warps and split); shapes whose plan would need more scratch
//    run in the forms that need none, and only shapes no form can run are refused;
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
    // same argument rules as ternocl_int2_upcvt (checked again by the planner below)
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (postop < 0 || postop > 4 || (out_f32 != 0 && out_f32 != 1)) return TERNOCL_ERR_ARG;
    if (M < 0 || N <= 0 || K <= 0 || N % 16 || K % kGS) return TERNOCL_ERR_SHAPE;
    if (!A || !B || !S || !C) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;

    // The GEMV runs exactly as ternocl_int2_upcvt plans it for a workspace of the
    // array's size: the same per-strip kernel, warps and split the plan picks (none
    // where it picks none).  A plan whose scratch would not fit the
    // array falls back to the forms that need none; a shape no form can run is refused.
    void *scratch = nullptr;
    cudaError_t e = scratch_ptr(&scratch);
    if (e != cudaSuccess) return report_cuda(e);
    // The arrival counters at the start of the array must be zero when a call begins.
    // Every completed call leaves them zero, but a call cut short (a failed launch, a
    // killed process sharing nothing else) could not; clear them on the stream.
    const size_t cnt = int2_gemv_counter_bytes(M, N);
    if (cnt > kNoAllocScratchBytes) return TERNOCL_ERR_WORKSPACE;
    e = cudaMemsetAsync(scratch, 0, cnt, (cudaStream_t)stream);
    if (e != cudaSuccess) return report_cuda(e);
    return plan_and_launch_int2_gemv(A, B, S, C, Other, Bias, M, N, K, dtype, postop, out_f32, scratch,
                                     kNoAllocScratchBytes, stream, nullptr);
}
