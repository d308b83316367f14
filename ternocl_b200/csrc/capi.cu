// extern "C" entry points of libternocl: argument validation (the reference's
// host-side checks, e.g. int2_fp16_upcvt/main.cpp:159), workspace planning and
// dispatch to the kernel families.  No entry point allocates device memory except
// ternocl_int2_int8 with qmode 1 on the tensor-core GEMM, which takes its M x K int8
// codes from a stream-ordered pool (scratch_alloc below).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "ternocl.h"

namespace ternocl {

Options &options() {
    static Options o;
    return o;
}

static thread_local char g_last_error[256] = "";

static int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return TERNOCL_OK;
    std::snprintf(g_last_error, sizeof g_last_error, "%s: %s", cudaGetErrorName(e),
                  cudaGetErrorString(e));
    return TERNOCL_ERR_CUDA;
}

static int sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (counts[dev] == 0) {
        int c = 0;
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0)
            c = 148;
        counts[dev] = c;
    }
    return counts[dev];
}

static bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// ---------------------------------------------------------------------------------
// GEMV split-K plan: enough CTAs (4 per SM) to keep every SM streaming.
struct GemvPlan {
    int SK = 1;
    int warps = 4;         // warps per CTA (register-decode GEMVs)
    bool cluster = false;  // 1 < SK <= 8: reduce through distributed shared memory
    size_t cnt_bytes = 0, part_bytes = 0;
    size_t total() const { return (SK > 1 && !cluster) ? cnt_bytes + part_bytes : 0; }
};

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// shared memory a GEMV CTA may use (activation staging + weight ring)
constexpr size_t kGemvSmemBudget = 100 * 1024;
constexpr int kMaxClusterSK = 8;  // portable thread-block cluster size

// Split-K plan of a decode GEMV whose CTAs cover `cols` columns x `rows` activation
// rows: enough CTAs to give every SM `per_sm` of them, each CTA keeping >= 1 group
// and its staged activations within the shared-memory budget.  Splits up to
// `max_cluster` reduce through distributed shared memory; beyond that (only when a
// workspace is available) through the workspace.
template <class SmemFn>
static GemvPlan gemv_plan_t(int M, int N, int K, int cols, int rows, int per_sm, int max_cluster,
                            bool allow_ws, size_t smem_budget, SmemFn smem_of_sk) {
    GemvPlan p;
    const int strips = (N + cols - 1) / cols, zb = (M + rows - 1) / rows, G = K / kGS;
    const long long tiles = (long long)strips * zb;
    const long long target = (long long)per_sm * sm_count();
    int sk = (int)((target + tiles - 1) / tiles);
    if (const int forced = options().gemv_split) sk = forced;
    if (sk > G) sk = G;
    if (sk > 64) sk = 64;
    while (sk < G && smem_of_sk(sk) > smem_budget) ++sk;
    if (sk > max_cluster && !allow_ws) sk = max_cluster;
    if (sk < 1) sk = 1;
    p.SK = sk;
    p.cluster = sk > 1 && sk <= max_cluster;
    p.cnt_bytes = round_up((size_t)tiles * sizeof(unsigned), 256);
    p.part_bytes = (size_t)sk * M * N * sizeof(float);
    return p;
}

// warp-level mma.sync GEMV (gemv_int2.cu): 32 columns x 8 rows per CTA of 4, 8 or 16
// warps
//
// Launch shape, searched on B200 over the back-to-back Llama-3-8B decode sequence with
// PDL (M=1): splitting K across CTAs pays only while there are fewer column strips than
// SMs (the cross-CTA reduction costs more than the parallelism otherwise); inside a CTA
// 16 warps split K while the CTA streams <= 32 groups, 8 beyond that, and 4 once the
// grid already holds >= 4 CTAs per SM (occupancy then matters more).  For M > 4 (this
// kernel's default range since the integer-MMA GEMV took M <= 4), re-measured from CUDA
// graph replays at M = 8: a two-way K split and 8 warps (4 at >= 4 CTAs per SM) --
// 4096x6144 26.8 -> 8.9 us, 4096x4096 18.3 -> 6.9, 4096x28672 39.3 -> 34.1,
// 14336x4096 19.7 -> 19.6 (16 warps were the slow part).
static GemvPlan gemv_plan(int M, int N, int K, bool allow_ws) {
    const int G = K / kGS, sms = sm_count();
    const long long tiles = (long long)((N + 31) / 32) * ((M + 7) / 8);
    const bool wide = M > kGemvDigitMaxM;
    const int forced = options().gemv_split;
    int sk = forced ? forced : (wide ? 2 : (tiles < sms ? 2 : 1));
    if (sk > G) sk = G;
    int warps = options().gemv_warps;
    if (!warps) {
        const int per_cta = (G + sk - 1) / sk;
        warps = tiles >= 4LL * sms ? 4 : (wide || per_cta > 32) ? 8 : 16;
    }
    GemvPlan p;
    p.SK = sk;
    while (p.SK < G && int2_gemv_smem(M, K, p.SK, warps) > kGemvSmemBudget) ++p.SK;
    if (p.SK > kMaxClusterSK && !allow_ws) p.SK = kMaxClusterSK;
    p.cluster = p.SK > 1 && p.SK <= kMaxClusterSK;
    p.cnt_bytes = round_up((size_t)tiles * sizeof(unsigned), 256);
    p.part_bytes = (size_t)p.SK * M * N * sizeof(float);
    p.warps = warps;
    return p;
}

// integer-MMA GEMV (gemv_i2d.cu, M <= 4): measured on B200 over the Llama-3-8B decode
// shapes with the launches replayed from a CUDA graph, a K split pays only when the
// column strips fill less than half of the SMs (the cluster reduction costs more than
// the extra CTAs give), and 8 warps per CTA beat 16 on K = 4096 (4 once the grid holds
// >= 4 CTAs per SM): 4096x4096 6.7 -> 4.6 us, 4096x6144 6.6 -> 5.8 us, 14336x4096 9.6
// -> 9.4 us.
//
// Re-measured over the shapes of the reference's published table (int2_fp16_upcvt/README.md,
// CUDA graphs of one shape, M = 1): with 1-2 strips per SM a long K (>= 64 groups) pays
// for a two-way split (17408x5120 14.5 -> 12.3 us).  With fewer strips than SMs, 16 warps
// per CTA measured faster per shape (4096x4096 4.55 -> 3.98 us, 14336x4096 10.58 -> 9.14)
// but slowed the bench's four-shape sequence (32.3 -> 33.8 us per step: the larger CTAs
// overlap less with the neighbouring GEMVs), so 8 stay.
static GemvPlan gemv_digit_plan(int M, int N, int K, bool allow_ws) {
    const int G = K / kGS, sms = sm_count();
    const long long tiles = (long long)((N + 31) / 32) * ((M + 3) / 4);
    int sk = 1;
    const int dwarps = tiles >= 4LL * sms ? 4 : 8;
    if (2 * tiles < sms) sk = 2;
    else if (tiles >= sms && tiles < 2LL * sms && G >= 64) sk = 2;
    if (const int forced = options().gemv_split) sk = forced;
    if (sk > G) sk = G;
    const int forced_warps = options().gemv_warps;
    const int warps = forced_warps ? forced_warps : dwarps;
    GemvPlan p;
    p.SK = sk;
    while (p.SK < G && int2_gemv_d_smem(M, K, p.SK, warps) > kGemvSmemBudget) ++p.SK;
    if (p.SK > kMaxClusterSK && !allow_ws) p.SK = kMaxClusterSK;
    p.cluster = p.SK > 1 && p.SK <= kMaxClusterSK;
    p.cnt_bytes = round_up((size_t)tiles * sizeof(unsigned), 256);
    p.part_bytes = (size_t)p.SK * M * N * sizeof(float);
    p.warps = warps;
    return p;
}

// int1 and BITCOS GEMVs: measured from CUDA graph replays on the Llama-3-8B shapes and
// the BITCOS 5376 x 21504 shape, a target of 3 CTAs per SM (the split of 6 per SM
// over-split the narrow matrices: int1 M=1 4096x4096 6.5 -> 5.6 us, BITCOS 13.8 -> 11.2
// us; int1 keeps 6 for M > 4) and at least a two-way K split (int1 at M > 4: M=8
// 4096x28672 39.5 -> 28.3 us; BITCOS at every M: 5376x21504 stays on two splits).
static int gemv_target_per_sm(int M) { return M <= kGemvDigitMaxM ? 3 : 6; }
static void gemv_min_split(GemvPlan &p, int K) {
    if (options().gemv_split || p.SK >= 2 || K / kGS < 2) return;
    const size_t per_split = p.part_bytes / (p.SK > 0 ? p.SK : 1);
    p.SK = 2;
    p.cluster = true;  // 2 <= the cluster limit: reduced through distributed shared memory
    p.part_bytes = 2 * per_split;
}

// int1 GEMV (gemv_int1.cu): same CTA shape
static GemvPlan gemv_i1_plan(int M, int N, int K, bool allow_ws) {
    GemvPlan p = gemv_plan_t(M, N, K, 32, 8, gemv_target_per_sm(M), kMaxClusterSK, allow_ws, kGemvSmemBudget,
                             [&](int sk) { return int1_gemv_smem(M, K, sk); });
    if (M > kGemvDigitMaxM) gemv_min_split(p, K);
    return p;
}

// BITCOS GEMV (gemv_bitcos.cu): same CTA shape, whole K range staged per CTA
// (with the fused transform, K splits on HB boundaries: SK <= K / HB)
static GemvPlan gemv_bitcos_plan(int M, int N, int K, bool allow_ws, int had_hb = 0) {
    GemvPlan p = gemv_plan_t(M, N, K, 32, 8, 3, kMaxClusterSK, allow_ws, kGemvSmemBudget,
                             [&](int sk) { return bitcos_gemv_smem(M, K, sk, had_hb); });
    gemv_min_split(p, K);
    if (had_hb && p.SK > K / had_hb) {
        p.SK = K / had_hb;
        p.cluster = p.SK > 1 && p.SK <= kMaxClusterSK;
    }
    return p;
}

// s8 x s2 GEMV (gemv_int8.cu): same CTA shape, int8 activation staging
// (graph replays, 27B-like shapes: 3 CTAs per SM and a two-way split at M > 4 --
// M=1 5376x21504 17.5 -> 15.5 us, M=8 5376x5376 11.6 -> 9.0 us)
static GemvPlan gemv_i8_plan(int M, int N, int K, bool allow_ws) {
    GemvPlan p = gemv_plan_t(M, N, K, 32, 8, 3, kMaxClusterSK, allow_ws, kGemvSmemBudget,
                             [&](int sk) { return int8_gemv_smem(M, K, sk); });
    if (M > kGemvDigitMaxM) gemv_min_split(p, K);
    return p;
}

// tcgen05 GEMV (gemv_tc.cu): 128 columns x tc_gemv_rows(M) rows per CTA, 4 CTAs/SM
// (each holds 128 of the SM's 512 TMEM columns; <= 52 KB of shared memory keeps 4
// of them resident)
static GemvPlan gemv_tc_plan(int M, int N, int K, bool allow_ws) {
    return gemv_plan_t(M, N, K, 128, tc_gemv_rows(M), 4, 16, allow_ws, 52 * 1024,
                       [&](int sk) { return int2_gemv_tc_smem(M, K, sk); });
}

static int check_gemm_common(const void *A, const void *B, const void *S, const void *C,
                             const void *Other, const void *Bias, int M, int N, int K, int dtype,
                             int postop, int out_f32) {
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (postop < 0 || postop > 4 || (out_f32 != 0 && out_f32 != 1)) return TERNOCL_ERR_ARG;
    if (M < 0 || N <= 0 || K <= 0) return TERNOCL_ERR_SHAPE;
    if (N % 16 || K % kGS) return TERNOCL_ERR_SHAPE;  // int2_fp16_upcvt/main.cpp:159
    if (!A || !B || !S || !C) return TERNOCL_ERR_ARG;
    if ((postop == 1 || postop == 2) && !Other) return TERNOCL_ERR_ARG;
    if (postop == 3 && !Bias) return TERNOCL_ERR_ARG;
    if (!aligned(A, 16) || !aligned(B, 16) || !aligned(S, 16) || !aligned(C, out_f32 ? 16 : 8))
        return TERNOCL_ERR_ARG;
    if (Other && !aligned(Other, 8)) return TERNOCL_ERR_ARG;
    if (Bias && !aligned(Bias, out_f32 ? 8 : 4)) return TERNOCL_ERR_ARG;
    return TERNOCL_OK;
}

int gemv_split_k(int M, int N, int K) { return gemv_plan(M, N, K, true).SK; }

// The register-decode int2 GEMV of a width-N matrix (or a width-N shard when `peer` carries
// the column-sharded fields), planned and launched.
int plan_and_launch_int2_gemv(const void *A, const uint32_t *B, const void *S, void *C, const void *Other,
                              const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32, void *ws,
                              size_t ws_bytes, void *stream, const GemvArgs *peer) {
    // in the sharded mode C is unused (the peers' C are), Other/Bias are full width
    int st = check_gemm_common(A, B, S, peer ? (const void *)A : C, peer ? nullptr : Other,
                               peer ? nullptr : Bias, M, N, K, dtype, peer ? 0 : postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (postop < 0 || postop > 4) return TERNOCL_ERR_ARG;
    if ((postop == 1 || postop == 2) && !Other) return TERNOCL_ERR_ARG;
    if (postop == 3 && !Bias) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    GemvArgs a = peer ? *peer : GemvArgs();
    a.A = A; a.B = B; a.S = S; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.stream = (cudaStream_t)stream;
    const int impl = options().gemv_impl;
    const bool digit = M <= kGemvDigitMaxM && impl != 1;
    auto plan = [&](bool allow_ws) { return digit ? gemv_digit_plan(M, N, K, allow_ws) : gemv_plan(M, N, K, allow_ws); };
    GemvPlan p = plan(ws != nullptr);
    if (p.total() > ws_bytes) p = plan(false);
    const size_t smem = digit ? int2_gemv_d_smem(M, K, p.SK, p.warps) : int2_gemv_smem(M, K, p.SK, p.warps);
    if (smem > 227 * 1024) return TERNOCL_ERR_WORKSPACE;
    a.SK = p.SK;
    a.warps = p.warps;
    a.cluster = p.cluster ? 1 : 0;
    if (p.total() > 0) {
        if (!aligned(ws, 256)) return TERNOCL_ERR_ARG;
        a.ws_cnt = (unsigned *)ws;
        a.ws_part = (float *)((char *)ws + p.cnt_bytes);
    }
    return cuda_status(digit ? int2_gemv_d_launch(a) : int2_gemv_launch(a));
}
int report_cuda(cudaError_t e) { return cuda_status(e); }

size_t int2_gemv_counter_bytes(int M, int N) {
    // one counter per (32-column strip, row block of >= 4 rows)
    const size_t tiles = (size_t)((N + 31) / 32) * (size_t)((M + 3) / 4);
    return round_up(tiles * sizeof(unsigned), 256);
}

// (kernel, device) -> dynamic shared memory attribute already set
namespace {
struct SmemAttrEntry {
    const void *fn;
    int dev, bytes;
};
std::mutex g_smem_mu;
SmemAttrEntry g_smem_attr[1024];
int g_smem_n = 0;
}  // namespace

bool smem_attr_known(const void *fn, int bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(g_smem_mu);
    for (int i = 0; i < g_smem_n; ++i)
        if (g_smem_attr[i].fn == fn && g_smem_attr[i].dev == dev) return g_smem_attr[i].bytes >= bytes;
    return false;
}

void smem_attr_record(const void *fn, int bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    std::lock_guard<std::mutex> lock(g_smem_mu);
    for (int i = 0; i < g_smem_n; ++i)
        if (g_smem_attr[i].fn == fn && g_smem_attr[i].dev == dev) {
            if (bytes > g_smem_attr[i].bytes) g_smem_attr[i].bytes = bytes;
            return;
        }
    if (g_smem_n < 1024) g_smem_attr[g_smem_n++] = {fn, dev, bytes};
}

}  // namespace ternocl

using namespace ternocl;

extern "C" {

const char *ternocl_version(void) { return "ternocl-b200 0.1.0 (sm_100a)"; }

const char *ternocl_status_string(int s) {
    switch (s) {
    case TERNOCL_OK: return "ok";
    case TERNOCL_ERR_SHAPE: return "unsupported shape (need N % 16 == 0 and K % 128 == 0)";
    case TERNOCL_ERR_ARG: return "invalid argument";
    case TERNOCL_ERR_CUDA: return "CUDA error";
    case TERNOCL_ERR_TIMEOUT: return "timed out";
    case TERNOCL_ERR_COMM: return "communication error";
    case TERNOCL_ERR_UNSUPPORTED: return "unsupported";
    case TERNOCL_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
    }
}

const char *ternocl_last_error(void) { return g_last_error; }

int ternocl_set_option(int option, int value) {
    if (option == TERNOCL_OPT_PDL) {
        return options().pdl.exchange(value ? 1 : 0);
    }
    if (option == TERNOCL_OPT_GEMM_PERSISTENT) {
        if (value < 0 || value > 3) return -1;
        return options().gemm_persistent.exchange(value);
    }
    if (option == TERNOCL_OPT_GEMV_WARPS) {
        if (value != 0 && value != 4 && value != 8 && value != 16) return -1;
        return options().gemv_warps.exchange(value);
    }
    if (option == TERNOCL_OPT_GEMV_SPLIT) {
        if (value < 0 || value > 64) return -1;
        return options().gemv_split.exchange(value);
    }
    if (option == TERNOCL_OPT_GEMV_IMPL) {
        if (value < 0 || value > 2) return -1;
        return options().gemv_impl.exchange(value);
    }
    if (option == TERNOCL_OPT_BITCOS_GEMV) {
        if (value < 0 || value > 1) return -1;
        return options().bitcos_gemv.exchange(value);
    }
    if (option == TERNOCL_OPT_PEER_TIMEOUT_MS) {
        if (value < 1 || value > 60000) return -1;
        return options().peer_timeout_ms.exchange(value);
    }
    if (option == TERNOCL_OPT_GEMM_TILE_M) {
        if (value != 0 && value != 128 && value != 256) return -1;
        return options().gemm_tile_m.exchange(value);
    }
    return -1;
}

size_t ternocl_gemv_workspace_size(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0 || N % 16 || K % kGS) return 0;
    // the largest need of the GEMVs that take a workspace (int2 on either path, int1)
    size_t need = gemv_plan(M, N, K, true).total();
    if (M <= kGemvDigitMaxM && gemv_digit_plan(M, N, K, true).total() > need) need = gemv_digit_plan(M, N, K, true).total();
    const size_t b = gemv_tc_plan(M, N, K, true).total(), c = gemv_i1_plan(M, N, K, true).total();
    if (b > need) need = b;
    if (c > need) need = c;
    return need;
}

int ternocl_device_error(int reset) {
    unsigned v = 0, t = 0;
    if (read_device_error_gemv_tc(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_gemm_tc(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_moe(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_gemm_i8(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_allgather(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_gemm_bitcos(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_moe_decode(&t, reset) != cudaSuccess) return -1;
    v |= t;
    if (read_device_error_gemv_bitcos_p(&t, reset) != cudaSuccess) return -1;
    v |= t;
    return (int)v;
}

int ternocl_int2_upcvt(const void *A, const uint32_t *B, const void *S, void *C, const void *Other,
                       const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32,
                       int algo, void *ws, size_t ws_bytes, void *stream) {
    int st = check_gemm_common(A, B, S, C, Other, Bias, M, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (algo < TERNOCL_ALGO_AUTO || algo > TERNOCL_ALGO_GEMV_TMEM) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    GemvArgs a;
    a.A = A; a.B = B; a.S = S; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.stream = (cudaStream_t)stream;
    if (algo == TERNOCL_ALGO_GEMM || (algo == TERNOCL_ALGO_AUTO && M >= kGemmMinM))
        return cuda_status(int2_gemm_tc_launch(a));
    if (algo != TERNOCL_ALGO_GEMV_TMEM)
        return plan_and_launch_int2_gemv(A, B, S, C, Other, Bias, M, N, K, dtype, postop, out_f32, ws, ws_bytes,
                                         stream, nullptr);
    GemvPlan p = gemv_tc_plan(M, N, K, ws != nullptr);
    if (p.total() > ws_bytes) p = gemv_tc_plan(M, N, K, false);
    if (int2_gemv_tc_smem(M, K, p.SK) > 227 * 1024) return TERNOCL_ERR_WORKSPACE;
    a.SK = p.SK;
    a.cluster = p.cluster ? 1 : 0;
    if (p.total() > 0) {
        if (!aligned(ws, 256)) return TERNOCL_ERR_ARG;
        a.ws_cnt = (unsigned *)ws;
        a.ws_part = (float *)((char *)ws + p.cnt_bytes);
    }
    return cuda_status(int2_gemv_tc_launch(a));
}

int ternocl_int1_upcvt(const void *A, const uint32_t *B, const void *S, void *C, const void *Other,
                       const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32,
                       int algo, void *ws, size_t ws_bytes, void *stream) {
    int st = check_gemm_common(A, B, S, C, Other, Bias, M, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (algo < TERNOCL_ALGO_AUTO || algo > TERNOCL_ALGO_GEMM) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    GemvArgs a;
    a.A = A; a.B = B; a.S = S; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.stream = (cudaStream_t)stream;
    if (algo == TERNOCL_ALGO_GEMM || (algo == TERNOCL_ALGO_AUTO && M >= kGemmMinM))
        return cuda_status(int1_gemm_tc_launch(a));
    GemvPlan p = gemv_i1_plan(M, N, K, ws != nullptr);
    if (p.total() > ws_bytes) p = gemv_i1_plan(M, N, K, false);
    if (int1_gemv_smem(M, K, p.SK) > 227 * 1024) return TERNOCL_ERR_WORKSPACE;
    a.SK = p.SK;
    a.cluster = p.cluster ? 1 : 0;
    if (p.total() > 0) {
        if (!aligned(ws, 256)) return TERNOCL_ERR_ARG;
        a.ws_cnt = (unsigned *)ws;
        a.ws_part = (float *)((char *)ws + p.cnt_bytes);
    }
    return cuda_status(int1_gemv_launch(a));
}

int ternocl_bitcos_upcvt(const void *A, const uint32_t *B, const void *S, const uint32_t *SR, int ls,
                         void *C, const void *Other, const void *Bias, int M, int N, int K, int dtype,
                         int postop, int out_f32, int algo, void *stream) {
    int st = check_gemm_common(A, B, S, C, Other, Bias, M, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (ls < 1) return TERNOCL_ERR_ARG;
    if (K % (64 * ls)) return TERNOCL_ERR_SHAPE;  // bitcos_fp16_upcvt/main.cpp:129
    if (ls > 1 && !SR) return TERNOCL_ERR_ARG;
    if (algo < TERNOCL_ALGO_AUTO || algo > TERNOCL_ALGO_GEMM) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    GemvArgs a;
    a.A = A; a.B = B; a.S = S; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.SR = SR; a.ls = ls;
    a.stream = (cudaStream_t)stream;
    // the M-tiled kernel walks all of K per tile: LS and SR do not apply
    // (bitcos_fp16_upcvt.cl:279-368; the reference selects it with --mt-m, our dispatch at
    // M >= kGemmMinM)
    if (algo == TERNOCL_ALGO_GEMM || (algo == TERNOCL_ALGO_AUTO && M >= kGemmMinM))
        return cuda_status(bitcos_gemm_tc_launch(a));
    // M <= 8: one CTA per SM over whole-K strips (no split, so LS and SR are not read)
    if (options().bitcos_gemv == 0 && bitcos_gemv_p_smem(M, K) > 0)
        return cuda_status(bitcos_gemv_p_launch(a, sm_count()));
    // no workspace in this signature: split-K stays within one thread-block cluster
    const GemvPlan p = gemv_bitcos_plan(M, N, K, false);
    if (bitcos_gemv_smem(M, K, p.SK) > 227 * 1024) return TERNOCL_ERR_WORKSPACE;
    a.SK = p.SK;
    a.cluster = p.cluster ? 1 : 0;
    return cuda_status(bitcos_gemv_launch(a));
}

int ternocl_bitcos_upcvt_hadamard(const void *A, const int8_t *signs, int use_signs, int hb, const uint32_t *B,
                                  const void *S, const uint32_t *SR, int ls, void *C, const void *Other,
                                  const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32,
                                  void *stream) {
    int st = check_gemm_common(A, B, S, C, Other, Bias, M, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (ls < 1) return TERNOCL_ERR_ARG;
    if (K % (64 * ls)) return TERNOCL_ERR_SHAPE;  // bitcos_fp16_upcvt/main.cpp:129
    if (ls > 1 && !SR) return TERNOCL_ERR_ARG;
    if (hb != 256 && hb != 512 && hb != 1024) return TERNOCL_ERR_SHAPE;  // one warp per block
    if (K % hb) return TERNOCL_ERR_SHAPE;  // hadamard_fwht.cl:68-69
    if (use_signs && (!signs || !aligned(signs, 16))) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    GemvArgs a;
    a.A = A; a.B = B; a.S = S; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.SR = SR; a.ls = ls;
    a.had_hb = hb;
    a.had_signs = use_signs ? signs : nullptr;
    a.stream = (cudaStream_t)stream;
    // M <= 8: the strip kernel, each CTA transforming its staged rows once
    if (options().bitcos_gemv == 0 && bitcos_gemv_p_smem(M, K) > 0)
        return cuda_status(bitcos_gemv_p_launch(a, sm_count()));
    const GemvPlan p = gemv_bitcos_plan(M, N, K, false, hb);
    if (bitcos_gemv_smem(M, K, p.SK, hb) > 227 * 1024) return TERNOCL_ERR_WORKSPACE;
    a.SK = p.SK;
    a.cluster = p.cluster ? 1 : 0;
    return cuda_status(bitcos_gemv_launch(a));
}

int ternocl_hadamard_fwht(const void *x, const int8_t *signs, void *y, int rows, int K, int hb, int use_signs,
                          int dtype, void *stream) {
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (hb < 256 || hb > 4096 || (hb & (hb - 1))) return TERNOCL_ERR_SHAPE;  // hadamard_fwht.cl:17-31
    if (rows < 0 || K <= 0 || K % hb) return TERNOCL_ERR_SHAPE;                // bpr = K / HB (:68)
    if (!x || !y || (use_signs && !signs)) return TERNOCL_ERR_ARG;
    if (!aligned(x, 16) || !aligned(y, 16) || (use_signs && !aligned(signs, 16))) return TERNOCL_ERR_ARG;
    if (rows == 0) return TERNOCL_OK;
    return cuda_status(hadamard_launch(x, signs, y, rows, K, hb, use_signs ? 1 : 0, dtype, (cudaStream_t)stream));
}

int ternocl_int8_ldsa(int M) { return (M + 31) & ~31; }

int ternocl_int8_quant_a(const void *A, void *SA, int8_t *Aq, int M, int K, int dtype, void *stream) {
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (M < 0 || K <= 0 || K % kGS) return TERNOCL_ERR_SHAPE;
    if (!A || !SA) return TERNOCL_ERR_ARG;
    if (!aligned(A, 8) || !aligned(SA, 2) || (Aq && !aligned(Aq, 4))) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    return cuda_status(quant_a_launch(A, SA, Aq, M, K, dtype, (cudaStream_t)stream));
}

// Stream-ordered scratch of the library, one pool per device that keeps what it has
// mapped (release threshold = max), so a steady caller maps no pages per call; under
// stream capture the allocation becomes a graph memory node.  The memory is back in the
// pool once the stream passes the matching cudaFreeAsync.
static cudaError_t scratch_alloc(void **ptr, size_t bytes, cudaStream_t s) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!pools[dev]) {
            cudaMemPoolProps props;
            std::memset(&props, 0, sizeof props);
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            cudaMemPool_t pool;
            if ((e = cudaMemPoolCreate(&pool, &props)) != cudaSuccess) return e;
            uint64_t keep = ~0ull;
            if ((e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep)) != cudaSuccess) {
                cudaMemPoolDestroy(pool);
                return e;
            }
            pools[dev] = pool;
        }
    }
    return cudaMallocFromPoolAsync(ptr, bytes, pools[dev], s);
}

int ternocl_int2_int8(const void *A, const int8_t *Aq, const void *SA, const uint32_t *B,
                      const void *SB, void *C, const void *Other, const void *Bias, int M, int N,
                      int K, int dtype, int postop, int out_f32, int qmode, int algo, void *stream) {
    if (qmode != 0 && qmode != 1) return TERNOCL_ERR_ARG;
    const void *act = qmode == 0 ? (const void *)Aq : A;  // the operand the kernel reads
    int st = check_gemm_common(act, B, SB, C, Other, Bias, M, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (!SA || !aligned(SA, 2)) return TERNOCL_ERR_ARG;
    if (algo != TERNOCL_ALGO_AUTO && algo != TERNOCL_ALGO_GEMV && algo != TERNOCL_ALGO_GEMM) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    GemvArgs a;
    a.A = A; a.B = B; a.S = SB; a.C = C; a.Other = Other; a.Bias = Bias;
    a.M = M; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.Aq = Aq; a.SA = SA; a.qmode = qmode;
    a.stream = (cudaStream_t)stream;
    // the tensor-core GEMM reads int8 codes and copies the scale rows in 16-byte units.
    // qmode 0: the caller's Aq.  qmode 1 (the reference's default scheme: quantise with the
    // caller's SA inside the GEMM, int2_int8_dpas.cl:283-290): one pass quantises A into
    // stream-ordered scratch, so each row block is quantised once rather than once per
    // 128-column tile (168 times at N = 21504); the codes are the in-kernel ones bit for
    // bit.  The GEMV kernel quantises in its own loads and serves any M in 8-row blocks.
    const bool sa16 = aligned(SA, 16);
    if (algo == TERNOCL_ALGO_GEMM && !sa16) return TERNOCL_ERR_ARG;
    if (sa16 && (algo == TERNOCL_ALGO_GEMM || (algo == TERNOCL_ALGO_AUTO && M >= kGemmMinM))) {
        if (qmode == 0) return cuda_status(int8_gemm_tc_launch(a));
        if (!aligned(A, 8)) return TERNOCL_ERR_ARG;
        void *q = nullptr;
        cudaError_t e = scratch_alloc(&q, (size_t)M * K, a.stream);
        if (e != cudaSuccess) return cuda_status(e);
        e = quant_apply_launch(A, SA, (int8_t *)q, M, K, dtype, a.stream);
        if (e == cudaSuccess) {
            a.Aq = (const int8_t *)q;
            e = int8_gemm_tc_launch(a);
        }
        const cudaError_t fe = cudaFreeAsync(q, a.stream);
        return cuda_status(e != cudaSuccess ? e : fe);
    }
    // no workspace in this signature: split-K stays within one thread-block cluster
    const GemvPlan p = gemv_i8_plan(M, N, K, false);
    if (int8_gemv_smem(M, K, p.SK) > 227 * 1024) return TERNOCL_ERR_WORKSPACE;
    a.SK = p.SK;
    a.cluster = p.cluster ? 1 : 0;
    return cuda_status(int8_gemv_launch(a));
}

int ternocl_int2_int8_group_dots(const int8_t *Aq, const uint32_t *B, int32_t *Dots, int M, int N,
                                 int K, void *stream) {
    if (M < 0 || N <= 0 || K <= 0 || N % 16 || K % kGS) return TERNOCL_ERR_SHAPE;
    if (!Aq || !B || !Dots) return TERNOCL_ERR_ARG;
    if (M == 0) return TERNOCL_OK;
    return cuda_status(group_dots_launch(Aq, B, Dots, M, N, K, (cudaStream_t)stream));
}

int ternocl_moe_rows_per_tile(void) { return 128; }

int ternocl_moe_route(const int32_t *ids, int32_t *meta, int32_t *perm, int32_t *inv, int G, int E, int rows_per_tile,
                      void *stream) {
    if (G < 0 || E < 1 || E > 1024) return TERNOCL_ERR_SHAPE;
    if (rows_per_tile != ternocl_moe_rows_per_tile()) return TERNOCL_ERR_ARG;
    if (!meta || (G > 0 && (!ids || !perm || !inv))) return TERNOCL_ERR_ARG;
    return cuda_status(moe_route_launch(ids, meta, perm, inv, G, E, rows_per_tile, (cudaStream_t)stream));
}

int ternocl_moe_gather(const void *X, const int32_t *perm, void *Xs, int G, int K, int topk, void *stream) {
    if (G < 0 || K <= 0 || K % 8 || topk < 1) return TERNOCL_ERR_SHAPE;
    if (G == 0) return TERNOCL_OK;
    if (!X || !perm || !Xs || !aligned(X, 16) || !aligned(Xs, 16)) return TERNOCL_ERR_ARG;
    return cuda_status(moe_gather_launch(X, perm, Xs, G, K, topk, (cudaStream_t)stream));
}

int ternocl_moe_gemm(const int32_t *meta, const void *A_all, const uint32_t *B_all, const void *S_all, void *C_all,
                     const void *Other_all, int G, int N, int K, int E, int dtype, int postop, int out_f32,
                     void *stream) {
    int st = check_gemm_common(A_all, B_all, S_all, C_all, Other_all, nullptr, G, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (postop == 3) return TERNOCL_ERR_ARG;  // no bias in the MoE GEMM (int2_moe_prefill.cl:95)
    if (!meta || E < 1 || E > 1024) return TERNOCL_ERR_ARG;
    if (G == 0) return TERNOCL_OK;
    GemvArgs a;
    a.A = A_all; a.B = B_all; a.S = S_all; a.C = C_all; a.Other = Other_all; a.Bias = nullptr;
    a.M = G; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.stream = (cudaStream_t)stream;
    return cuda_status(moe_gemm_tc_launch(a, meta, E));
}

int ternocl_moe_gather_q(const int8_t *Xq, const void *SAt, const int32_t *perm, int8_t *Xsq, void *SA, int T, int G,
                         int K, int topk, void *stream) {
    if (T < 0 || G < 0 || K <= 0 || K % kGS || topk < 1 || (long long)T * topk != G) return TERNOCL_ERR_SHAPE;
    if (G == 0) return TERNOCL_OK;
    if (!Xq || !SAt || !perm || !Xsq || !SA || !aligned(Xq, 16) || !aligned(Xsq, 16) || !aligned(SAt, 2) ||
        !aligned(SA, 2))
        return TERNOCL_ERR_ARG;
    return cuda_status(moe_gather_q_launch(Xq, SAt, perm, Xsq, SA, T, G, K, topk, (cudaStream_t)stream));
}

int ternocl_moe_gemm_i8(const int32_t *meta, const void *A_all, const int8_t *Aq_all, const void *SA,
                        const uint32_t *B_all, const void *SB_all, void *C_all, const void *Other_all, int G, int N,
                        int K, int num_experts, int dtype, int postop, int out_f32, int qmode, void *stream) {
    (void)A_all;  // qmode 0 reads the int8 rows only
    if (qmode != 0) return TERNOCL_ERR_ARG;
    int st = check_gemm_common(Aq_all, B_all, SB_all, C_all, Other_all, nullptr, G, N, K, dtype, postop, out_f32);
    if (st != TERNOCL_OK) return st;
    if (postop == 3) return TERNOCL_ERR_ARG;  // no bias in the MoE GEMM (int2_moe_prefill_int8.cl:93)
    if (!meta || num_experts < 1 || num_experts > 1024) return TERNOCL_ERR_ARG;
    if (!SA || !aligned(SA, 16)) return TERNOCL_ERR_ARG;  // the scale rows are copied in 16-byte units
    if (G == 0) return TERNOCL_OK;
    GemvArgs a;
    a.B = B_all; a.S = SB_all; a.C = C_all; a.Other = Other_all; a.Bias = nullptr;
    a.M = G; a.N = N; a.K = K; a.dtype = dtype; a.postop = postop; a.out_f32 = out_f32;
    a.Aq = Aq_all; a.SA = SA; a.qmode = 0;
    a.stream = (cudaStream_t)stream;
    return cuda_status(int8_gemm_tc_launch(a, meta, num_experts));
}

int ternocl_moe_combine(const float *Y, const int32_t *inv, const void *RW, void *O, int T, int N, int topk,
                        int dtype, void *stream) {
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (T < 0 || N <= 0 || N % 4 || topk < 1) return TERNOCL_ERR_SHAPE;
    if (T == 0) return TERNOCL_OK;
    if (!Y || !inv || !RW || !O || !aligned(Y, 16) || !aligned(O, 8)) return TERNOCL_ERR_ARG;
    return cuda_status(moe_combine_launch(Y, inv, RW, O, T, N, topk, dtype, (cudaStream_t)stream));
}

// ---- MoE decode (int2_moe/int2_moe.cl:63-174) ----
static int check_moe_decode(int dtype, int rows, int N, int K, int topk, int E) {
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (rows < 0 || N <= 0 || K <= 0 || N % 16 || K % kGS || topk < 1 || E < 1) return TERNOCL_ERR_SHAPE;
    return TERNOCL_OK;
}

int ternocl_moe_decode_gate_up(const int32_t *ids, const void *X, const uint32_t *Bg, const void *Sg,
                               const uint32_t *Bu, const void *Su, void *H, int G, int N, int K, int topk,
                               int num_experts, int dtype, void *stream) {
    int st = check_moe_decode(dtype, G, N, K, topk, num_experts);
    if (st != TERNOCL_OK) return st;
    if (G % topk) return TERNOCL_ERR_SHAPE;
    if (G == 0) return TERNOCL_OK;
    if (!ids || !X || !Bg || !Sg || !Bu || !Su || !H) return TERNOCL_ERR_ARG;
    if (!aligned(X, 16) || !aligned(Bg, 16) || !aligned(Bu, 16) || !aligned(Sg, 16) || !aligned(Su, 16))
        return TERNOCL_ERR_ARG;
    if (moe_decode_smem(K / kGS, topk, 0) > 227 * 1024) return TERNOCL_ERR_SHAPE;
    return cuda_status(moe_decode_gate_up_launch(ids, X, Bg, Sg, Bu, Su, H, G, N, K, topk, num_experts, dtype,
                                                 (cudaStream_t)stream));
}

int ternocl_moe_decode_down(const int32_t *ids, const void *H, const void *RW, const uint32_t *B, const void *S,
                            float *Y, int G, int N, int K, int num_experts, int dtype, void *stream) {
    int st = check_moe_decode(dtype, G, N, K, 1, num_experts);
    if (st != TERNOCL_OK) return st;
    if (G == 0) return TERNOCL_OK;
    if (!ids || !H || !RW || !B || !S || !Y) return TERNOCL_ERR_ARG;
    if (!aligned(H, 16) || !aligned(B, 16) || !aligned(S, 16)) return TERNOCL_ERR_ARG;
    if (moe_decode_smem(K / kGS, 1, 1) > 227 * 1024) return TERNOCL_ERR_SHAPE;
    return cuda_status(moe_decode_down_launch(ids, H, RW, B, S, Y, G, N, K, num_experts, dtype,
                                              (cudaStream_t)stream));
}

int ternocl_moe_decode_reduce(const float *Y, void *O, int T, int N, int topk, int dtype, void *stream) {
    if (dtype != TERNOCL_FP16 && dtype != TERNOCL_BF16) return TERNOCL_ERR_ARG;
    if (T < 0 || N <= 0 || N % 4 || topk < 1) return TERNOCL_ERR_SHAPE;
    if (T == 0) return TERNOCL_OK;
    if (!Y || !O || !aligned(Y, 16) || !aligned(O, 8)) return TERNOCL_ERR_ARG;
    return cuda_status(moe_decode_reduce_launch(Y, O, T, N, topk, dtype, (cudaStream_t)stream));
}

int ternocl_moe_decode_down_sum(const int32_t *ids, const void *H, const void *RW, const uint32_t *B,
                                const void *S, void *O, int T, int N, int K, int topk, int num_experts, int dtype,
                                void *stream) {
    int st = check_moe_decode(dtype, T, N, K, topk, num_experts);
    if (st != TERNOCL_OK) return st;
    if (T == 0) return TERNOCL_OK;
    if (!ids || !H || !RW || !B || !S || !O) return TERNOCL_ERR_ARG;
    if (!aligned(H, 16) || !aligned(B, 16) || !aligned(S, 16)) return TERNOCL_ERR_ARG;
    if (moe_decode_smem(K / kGS, topk, 2) > 227 * 1024) return TERNOCL_ERR_SHAPE;
    return cuda_status(moe_decode_down_sum_launch(ids, H, RW, B, S, O, T, N, K, topk, num_experts, dtype,
                                                  (cudaStream_t)stream));
}

}  // extern "C"
