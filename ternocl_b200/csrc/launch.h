// Host-side launch plumbing shared by the kernel files: argument structs, the
// compile-time epilogue dispatch and the kernel launcher (with optional
// programmatic dependent launch).
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <type_traits>

#include "ternocl.h"

namespace ternocl {

struct F16;
struct BF16;

// Process-wide options (ternocl_set_option), read by every call: atomic, so that a
// thread setting one while others launch is no data race (a call sees the old or the
// new value, never a torn one).
struct Options {
    std::atomic<int> pdl{0};          // launch with programmatic stream serialization
    std::atomic<int> gemm_tile_m{0};  // prefill GEMM CTA rows: 0 = per shape, 128 or 256
    std::atomic<int> gemv_split{0};   // decode GEMV K split: 0 = planned per shape
    std::atomic<int> gemv_warps{0};   // decode GEMV warps per CTA: 0 = planned per shape
    std::atomic<int> gemm_persistent{3};  // persistent tcgen05 GEMM: 0 never, 1 MoE grouped GEMMs, 2 every
                                          // prefill GEMM, 3 MoE grouped GEMMs with K <= 1024
    std::atomic<int> gemv_impl{0};        // int2 decode GEMV: 0 per M, 1 fp16 MMA decode, 2 integer MMA per
                                          // strip (M <= 4)
    std::atomic<int> peer_timeout_ms{2000};  // limit of the column-sharded GEMV's wait for its peers
    std::atomic<int> bitcos_gemv{0};         // BITCOS decode GEMV: 0 persistent strip kernel where it applies,
                                             // 1 K-sliced
};
Options &options();

// Arguments of one GEMM/GEMV call after validation.
struct GemvArgs {
    const void *A = nullptr;
    const uint32_t *B = nullptr;
    const void *S = nullptr;
    void *C = nullptr;
    const void *Other = nullptr;
    const void *Bias = nullptr;
    int M = 0, N = 0, K = 0;
    int dtype = 0, postop = 0, out_f32 = 0;
    int SK = 1;                  // cross-CTA K split
    int warps = 4;               // warps per CTA splitting the CTA's K range (4, 8, 16)
    int cluster = 0;             // SK CTAs per thread-block cluster (DSMEM reduction)
    float *ws_part = nullptr;    // [SK][M][N] fp32 partials
    unsigned *ws_cnt = nullptr;  // per-tile arrival counters
    cudaStream_t stream = nullptr;
    // s8 x s2 path
    const int8_t *Aq = nullptr;
    const void *SA = nullptr;
    int qmode = 0;
    // BITCOS: slice ranks [ls-1][N] of the reference's ls K slices
    const uint32_t *SR = nullptr;
    int ls = 1;
    // BITCOS GEMV with the sign flip + FWHT of the activations fused into their staging
    // (had_hb = 0: off); signs int8 [K] or null
    int had_hb = 0;
    const int8_t *had_signs = nullptr;
    // column-sharded GEMV (world > 0): see gemv::Params
    int world = 0, rank = 0, n_off = 0, N_out = 0;
    unsigned epoch = 0;
    unsigned *done_cnt = nullptr;
    unsigned *err = nullptr;
    void *C_peer[8] = {};
    unsigned *flag_peer[8] = {};
};

template <class T>
struct type_tag {
    using type = T;
};

// Calls f(type_tag<DT>, integral_constant<POSTOP>, integral_constant<OUT_F32>) for
// the runtime (dtype, postop, out_f32) of `a`.
template <class Args, class F>
cudaError_t dispatch_epilogue(const Args &a, F &&f) {
    auto with_dt = [&](auto dt) -> cudaError_t {
        auto with_po = [&](auto po) -> cudaError_t {
            if (a.out_f32) return f(dt, po, std::integral_constant<bool, true>{});
            return f(dt, po, std::integral_constant<bool, false>{});
        };
        switch (a.postop) {
        case 0: return with_po(std::integral_constant<int, 0>{});
        case 1: return with_po(std::integral_constant<int, 1>{});
        case 2: return with_po(std::integral_constant<int, 2>{});
        case 3: return with_po(std::integral_constant<int, 3>{});
        default: return with_po(std::integral_constant<int, 4>{});
        }
    };
    if (a.dtype == TERNOCL_BF16) return with_dt(type_tag<BF16>{});
    return with_dt(type_tag<F16>{});
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel, device and size: the
// attribute outlives the call, and setting it on every launch costs host time in the
// decode loop (capi.cu keeps the record).
bool smem_attr_known(const void *fn, int bytes);
void smem_attr_record(const void *fn, int bytes);
template <class F>
cudaError_t ensure_smem(F *kern, size_t bytes) {
    if (bytes <= 48 * 1024 || smem_attr_known((const void *)kern, (int)bytes)) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) smem_attr_record((const void *)kern, (int)bytes);
    return e;
}

template <class... KArgs, class... Args>
cudaError_t launch_kernel_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t stream, dim3 cluster, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (options().pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster.x;
        attr[n].val.clusterDim.y = cluster.y;
        attr[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <class... KArgs, class... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args &&...args) {
    return launch_kernel_cluster(kernel, grid, block, smem, stream, dim3(1, 1, 1),
                                 std::forward<Args>(args)...);
}

// Kernel-family entry points (one per .cu file).
cudaError_t quant_a_launch(const void *A, void *SA, int8_t *Aq, int M, int K, int dtype, cudaStream_t s);
// Aq = sat_int8(rint(A * SA)) with the caller's SA (no scale computed)
cudaError_t quant_apply_launch(const void *A, const void *SA, int8_t *Aq, int M, int K, int dtype, cudaStream_t s);
cudaError_t group_dots_launch(const int8_t *Aq, const uint32_t *B, int32_t *D, int M, int N, int K,
                              cudaStream_t s);
cudaError_t int8_gemv_launch(const GemvArgs &a);
cudaError_t int1_gemv_launch(const GemvArgs &a);
cudaError_t bitcos_gemv_launch(const GemvArgs &a);
// persistent strip-pipelined BITCOS GEMV (gemv_bitcos_p.cu): M <= 8; smem 0 = not applicable
size_t bitcos_gemv_p_smem(int M, int K);
cudaError_t bitcos_gemv_p_launch(const GemvArgs &a, int sms);
cudaError_t read_device_error_gemv_bitcos_p(unsigned *out, int reset);
cudaError_t hadamard_launch(const void *x, const int8_t *signs, void *y, int rows, int K, int hb, int use_signs,
                            int dtype, cudaStream_t st);
size_t bitcos_gemv_smem(int M, int K, int SK, int had_hb = 0);
size_t int1_gemv_smem(int M, int K, int SK);
size_t int8_gemv_smem(int M, int K, int SK);
cudaError_t int2_gemv_launch(const GemvArgs &a);
size_t int2_gemv_smem(int M, int K, int SK, int warps = 4);
// int2 GEMV on integer MMAs (gemv_i2d.cu): 32 columns x <= 4 rows per CTA
constexpr int kGemvDigitMaxM = 4;
cudaError_t int2_gemv_d_launch(const GemvArgs &a);
size_t int2_gemv_d_smem(int M, int K, int SK, int warps);
// tcgen05 / TMEM decode GEMV (gemv_tc.cu): 128 columns and tc_gemv_rows(M) rows per CTA
int tc_gemv_rows(int M);
size_t int2_gemv_tc_smem(int M, int K, int SK);
cudaError_t int2_gemv_tc_launch(const GemvArgs &a);
cudaError_t read_device_error_gemv_tc(unsigned *out, int reset);
// tcgen05 prefill GEMM (gemm_tc.cu): 128 x 256 tiles, weights upconverted in shared memory
cudaError_t int2_gemm_tc_launch(const GemvArgs &a);
cudaError_t int1_gemm_tc_launch(const GemvArgs &a);
cudaError_t read_device_error_gemm_tc(unsigned *out, int reset);
// 256-row (two 128-row MMAs sharing the decoded B) rather than 128-row GEMM tiles
bool gemm_use_256_rows(int M, int N);
// BITCOS prefill GEMM (gemm_bitcos.cu): a.B = the whole BITCOS buffer, no K split
cudaError_t bitcos_gemm_tc_launch(const GemvArgs &a);
cudaError_t read_device_error_gemm_bitcos(unsigned *out, int reset);
// s8 x s2 prefill GEMM (gemm_i8.cu): a.Aq int8 [M, K], a.SA [K/128, ldsa], a.S = SB
cudaError_t int8_gemm_tc_launch(const GemvArgs &a, const int *meta = nullptr, int E = 0);
cudaError_t read_device_error_gemm_i8(unsigned *out, int reset);
// grouped (MoE) int2 GEMM over the rows of meta's experts; a.M = G rows
cudaError_t moe_gemm_tc_launch(const GemvArgs &a, const int *meta, int E);
// MoE routing / gather / combine (moe.cu)
size_t moe_route_smem(int E);
cudaError_t moe_route_launch(const int *ids, int *meta, int *perm, int *inv, int G, int E, int rpt,
                             cudaStream_t st);
cudaError_t moe_gather_launch(const void *X, const int *perm, void *Xs, int G, int K, int topk, cudaStream_t st);
cudaError_t moe_gather_q_launch(const int8_t *Xq, const void *SAt, const int *perm, int8_t *Xsq, void *SA, int T,
                                int G, int K, int topk, cudaStream_t st);
cudaError_t moe_combine_launch(const float *Y, const int *inv, const void *RW, void *O, int T, int N, int topk,
                               int dtype, cudaStream_t st);
cudaError_t read_device_error_moe(unsigned *out, int reset);
// MoE decode GEMVs (moe_decode.cu)
size_t moe_decode_smem(int G, int topk, int mode);
cudaError_t moe_decode_gate_up_launch(const int *ids, const void *X, const uint32_t *Bg, const void *Sg,
                                      const uint32_t *Bu, const void *Su, void *H, int G, int N, int K, int topk,
                                      int E, int dtype, cudaStream_t st);
cudaError_t moe_decode_down_launch(const int *ids, const void *H, const void *RW, const uint32_t *B, const void *S,
                                   float *Y, int G, int N, int K, int E, int dtype, cudaStream_t st);
cudaError_t moe_decode_down_sum_launch(const int *ids, const void *H, const void *RW, const uint32_t *B,
                                       const void *S, void *O, int T, int N, int K, int topk, int E, int dtype,
                                       cudaStream_t st);
cudaError_t moe_decode_reduce_launch(const float *Y, void *O, int T, int N, int topk, int dtype, cudaStream_t st);
cudaError_t read_device_error_moe_decode(unsigned *out, int reset);
// M from which TERNOCL_ALGO_AUTO picks the GEMM (int2_fp16_upcvt/main.cpp:160)
constexpr int kGemmMinM = 64;
// split-K factor the register-decode GEMV's planner picks when a workspace exists
int gemv_split_k(int M, int N, int K);
// CUDA error -> ternocl status (records ternocl_last_error)
int report_cuda(cudaError_t e);
// plan + launch of the register-decode int2 GEMV; `peer` (or null) carries the
// column-sharded fields of ternocl_int2_upcvt_allgather
// bytes at the start of a workspace that hold arrival counters for any int2 GEMV plan of
// an M x N output (the rest holds partial sums, which need no clearing)
size_t int2_gemv_counter_bytes(int M, int N);
int plan_and_launch_int2_gemv(const void *A, const uint32_t *B, const void *S, void *C, const void *Other,
                              const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32, void *ws,
                              size_t ws_bytes, void *stream, const GemvArgs *peer);
cudaError_t read_device_error_allgather(unsigned *out, int reset);

}  // namespace ternocl
