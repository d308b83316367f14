// Column-sharded int2 GEMV with the all-gather fused into its epilogue.
//
// Across ranks the columns of a weight matrix are independent, so rank r owns columns
// [n0, n0 + nl) (its B and S shards) and computes them; instead of a GEMV followed by an
// NCCL all-gather of the outputs, the GEMV's epilogue stores its columns straight into
// every rank's full C through peer pointers (NVLink P2P stores), and the launch
// completes only after every rank's columns have arrived (a flag handshake with
// release/acquire at system scope, done by the grid's last CTA, bounded in time).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "tc_common.cuh"
#include "ternocl.h"

namespace ternocl {

namespace {
// this translation unit's device error word, by device
unsigned *error_word() {
    static std::mutex mu;
    static unsigned *addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, tc::g_device_error) != cudaSuccess) return nullptr;
        addr[dev] = (unsigned *)p;
    }
    return addr[dev];
}
}  // namespace

cudaError_t read_device_error_allgather(unsigned *out, int reset) { return tc::read_tu_error(out, reset); }

namespace {
typedef CUresult (*AddressRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);
AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (AddressRangeFn)f;
    });
    return fn;
}
}  // namespace

}  // namespace ternocl

using namespace ternocl;

extern "C" {

int ternocl_ipc_handle(const void *ptr, void *handle, size_t *offset) {
    if (!ptr || !handle || !offset) return TERNOCL_ERR_ARG;
    AddressRangeFn fn = address_range_fn();
    if (!fn) return report_cuda(cudaErrorNotSupported);
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return report_cuda(cudaErrorInvalidValue);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, (void *)base);
    if (e != cudaSuccess) return report_cuda(e);
    std::memcpy(handle, &h, sizeof(h));
    *offset = (size_t)((CUdeviceptr)ptr - base);
    return TERNOCL_OK;
}

int ternocl_ipc_open(const void *handle, size_t offset, void **ptr) {
    if (!handle || !ptr) return TERNOCL_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return report_cuda(e);
    *ptr = (char *)base + offset;
    return TERNOCL_OK;
}

int ternocl_ipc_close(void *ptr, size_t offset) {
    if (!ptr) return TERNOCL_ERR_ARG;
    return report_cuda(cudaIpcCloseMemHandle((char *)ptr - offset));
}

size_t ternocl_gemv_allgather_workspace_size(int M, int nl, int K) {
    if (M <= 0 || nl <= 0 || K <= 0 || nl % 16 || K % kGS) return 0;
    return 256 + ternocl_gemv_workspace_size(M, nl, K);
}

int ternocl_int2_upcvt_allgather(const void *A, const uint32_t *B, const void *S, void *const *C_ranks,
                                 const void *Other, const void *Bias, int M, int N, int n0, int nl, int K,
                                 int dtype, int postop, int out_f32, int rank, int world,
                                 unsigned *const *flags_ranks, unsigned epoch, void *ws, size_t ws_bytes,
                                 void *stream) {
    if (world < 1 || world > 8 || rank < 0 || rank >= world || !C_ranks || !flags_ranks) return TERNOCL_ERR_ARG;
    if (M < 0 || N <= 0 || K <= 0 || N % 16 || K % kGS || nl <= 0 || nl % 16 || n0 < 0 || n0 % 16 ||
        n0 + nl > N)
        return TERNOCL_ERR_SHAPE;
    for (int r = 0; r < world; ++r)
        if (!C_ranks[r] || !flags_ranks[r] || ((uintptr_t)C_ranks[r] % 16)) return TERNOCL_ERR_ARG;  // 16-byte slice copy
    if (!ws || ((uintptr_t)ws % 256) || ws_bytes < ternocl_gemv_allgather_workspace_size(M, nl, K))
        return TERNOCL_ERR_WORKSPACE;
    if (M == 0) return TERNOCL_OK;
    unsigned *err = error_word();
    if (!err) return report_cuda(cudaErrorInvalidDevice);
    GemvArgs a;
    a.world = world;
    a.rank = rank;
    a.n_off = n0;
    a.N_out = N;
    a.epoch = epoch;
    a.done_cnt = (unsigned *)ws;
    a.err = err;
    for (int r = 0; r < world; ++r) {
        a.C_peer[r] = C_ranks[r];
        a.flag_peer[r] = flags_ranks[r];
    }
    // the plan and the launch of the local shard (columns [n0, n0+nl) of a width-nl GEMV)
    return plan_and_launch_int2_gemv(A, B, S, nullptr, Other, Bias, M, nl, K, dtype, postop, out_f32,
                                     (char *)ws + 256, ws_bytes - 256, stream, &a);
}

}  // extern "C"
