/* ternocl -- B200 (sm_100a) ternary-weight GEMM/GEMV library, C ABI.
 *
 * Drop-in for the TernOCL OpenCL kernels: the same packed weight layouts (int2,
 * int1 "sel", BITCOS), the same per-128-group scales, the same fused epilogues, the
 * same N % 16 / K % 128 constraints and ragged-M semantics.  Each entry point takes
 * the reference kernel's positional arguments in the same order (paths below are
 * relative to the reference tree); the reference's compile-time -D options (BF16,
 * POSTOP, OUT_F32, QMODE, HB, TOPK, NUM_EXPERTS) become runtime arguments.
 *
 * Conventions
 *  - All tensor pointers are caller-owned DEVICE pointers; nothing here allocates
 *    device memory, except ternocl_int2_int8 with qmode 1 on its tensor-core GEMM
 *    (stream-ordered scratch, see there).  16-bit tensors (A, S, SA, SB, C, Other, Bias, RW) are raw
 *    fp16 or bf16 bits (`dtype`); with out_f32 the output C and Bias are fp32.
 *  - Other/Bias may be NULL when the epilogue does not read them.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *    stream-ordered and asynchronous; the caller synchronises.
 *  - Every call returns a ternocl_status; none exits, traps or blocks.
 *  - Results are deterministic: identical inputs give bit-identical outputs.
 */
#ifndef TERNOCL_H
#define TERNOCL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    TERNOCL_OK = 0,
    TERNOCL_ERR_SHAPE = 1,      /* N % 16, K % 128, K % HB, ... violated */
    TERNOCL_ERR_ARG = 2,        /* bad enum / NULL pointer / misaligned pointer */
    TERNOCL_ERR_CUDA = 3,       /* a CUDA runtime call failed (launch, attribute) */
    TERNOCL_ERR_TIMEOUT = 4,    /* a bounded device/host wait gave up */
    TERNOCL_ERR_COMM = 5,       /* multi-GPU communicator error */
    TERNOCL_ERR_UNSUPPORTED = 6,/* not available on this device / build */
    TERNOCL_ERR_WORKSPACE = 7   /* workspace too small */
} ternocl_status;

typedef enum { TERNOCL_FP16 = 0, TERNOCL_BF16 = 1 } ternocl_dtype;

/* Fused epilogue, applied to the fp32 accumulator before the output cast
 * (common/epilogue.clh:1-37). */
typedef enum {
    TERNOCL_POSTOP_NONE = 0,     /* acc */
    TERNOCL_POSTOP_SILU_MUL = 1, /* acc * sigmoid(acc) * Other[m,n]  (SwiGLU gate) */
    TERNOCL_POSTOP_ADD = 2,      /* acc + Other[m,n]                (residual)    */
    TERNOCL_POSTOP_BIAS = 3,     /* acc + Bias[n]                                  */
    TERNOCL_POSTOP_SIGMOID = 4   /* sigmoid(acc), 0 for acc <= -10                  */
} ternocl_postop;

/* Kernel choice for the GEMM/GEMV families.  AUTO picks the decode GEMV for small
 * M and the tensor-core GEMM otherwise (the reference drivers switch at M >= 64,
 * int2_fp16_upcvt/main.cpp:160).  GEMV is the register-decode GEMV on warp-level
 * MMAs; GEMV_TMEM the same contraction with the decoded weights in tensor memory and
 * tcgen05.mma (a second, independent implementation, also used for cross-checks). */
typedef enum {
    TERNOCL_ALGO_AUTO = 0,
    TERNOCL_ALGO_GEMV = 1,
    TERNOCL_ALGO_GEMM = 2,
    TERNOCL_ALGO_GEMV_TMEM = 3
} ternocl_algo;

const char *ternocl_version(void);
const char *ternocl_status_string(int status);
/* Last CUDA error string seen by this thread's ternocl calls ("" if none). */
const char *ternocl_last_error(void);
/* Device-side error word of the current device (synchronous read): bit 0 = a bounded
 * wait inside a kernel gave up (the kernel returned without hanging; its outputs are
 * invalid); bit 1 = ternocl_moe_route met an expert id outside [0, E) (that row was
 * left out).  reset != 0 clears it.  Returns -1 if it cannot be read. */
int ternocl_device_error(int reset);

/* Process-wide options.
 *  TERNOCL_OPT_PDL (default 0): launch kernels with programmatic dependent launch,
 *    so a kernel's weight prefetch overlaps the tail of the previous kernel in the
 *    stream.  Activations and workspaces are only touched after the previous
 *    kernel has completed; weights (B, S, SR) are read EARLY, so with this option
 *    on they must not be written by the immediately preceding kernel of the stream.
 *  TERNOCL_OPT_GEMM_TILE_M (default 0 = chosen per shape): rows of a prefill GEMM
 *    CTA tile, 128 or 256 (no counterpart in the reference, whose tiles are -D
 *    options of its kernels).
 *  TERNOCL_OPT_GEMV_SPLIT (default 0 = planned per shape): number of CTAs that split
 *    K in the decode GEMVs, 1..64 (clamped to K/128; above 8 it needs a workspace),
 *    the counterpart of the reference's LS tile option.
 *  TERNOCL_OPT_GEMV_WARPS (default 0 = planned per shape): warps per CTA of the int2
 *    decode GEMV (4, 8 or 16), which split the CTA's K range (the reference's SGM/LS
 *    tile options have the same role).
 *  TERNOCL_OPT_GEMM_PERSISTENT (default 3): the persistent tcgen05 GEMM (one CTA per
 *    SM over all tiles, epilogue overlapped with the next tile) for 0 = no GEMM,
 *    1 = the MoE grouped GEMMs, 2 = every prefill GEMM, 3 = the MoE grouped GEMMs with
 *    K <= 1024 (a short main loop per tile: the MoE down projection; one CTA per tile
 *    measured faster for the longer ones).
 *  TERNOCL_OPT_GEMV_IMPL (default 0 = chosen per M): the int2 decode GEMV used by
 *    ternocl_int2_upcvt at small M: 1 = fp16/bf16 MMA on decoded weights, 2 = integer
 *    MMA on int8 weights and exact fixed-point activations, one CTA per 32-column strip
 *    (M <= 4; the default there).  (Values 3 and 4, two measured-slower variants, were
 *    removed: setting them returns -1.)
 *  TERNOCL_OPT_GEMV_STAGES: reserved (it tuned one of the removed variants); setting it
 *    returns -1.
 *  TERNOCL_OPT_PEER_TIMEOUT_MS (default 2000, 1..60000): how long the column-sharded GEMV
 *    (ternocl_int2_upcvt_allgather) waits for its peers before it gives up, sets bit 2 of
 *    ternocl_device_error and returns.
 *  TERNOCL_OPT_BITCOS_GEMV (default 0): the BITCOS decode GEMV of ternocl_bitcos_upcvt:
 *    0 = at M <= 8 the persistent kernel (one CTA per SM over whole-K strips of 32
 *    columns; LS and SR are not read), else the K-sliced kernel; 1 = always the K-sliced
 *    kernel (the reference's LS split with slice ranks).
 * Options are process-wide and every call reads them when it plans its launch; setting
 * one from any thread while others call the library is safe (each is an atomic value, so
 * a call sees the old or the new setting).
 * Returns the previous value, or -1 for an unknown option or value. */
typedef enum {
    TERNOCL_OPT_PDL = 1,
    TERNOCL_OPT_GEMM_TILE_M = 2,
    TERNOCL_OPT_GEMV_SPLIT = 3,
    TERNOCL_OPT_GEMV_WARPS = 4,
    TERNOCL_OPT_GEMM_PERSISTENT = 5,
    TERNOCL_OPT_GEMV_IMPL = 6,
    TERNOCL_OPT_GEMV_STAGES = 7,
    TERNOCL_OPT_PEER_TIMEOUT_MS = 8,
    TERNOCL_OPT_BITCOS_GEMV = 9
} ternocl_option;
int ternocl_set_option(int option, int value);

/* Workspace (device scratch) a call may use for its cross-CTA split-K partial sums
 * and arrival counters.  Calls taking `ws` run without it (ws == NULL) at a lower
 * degree of parallelism.  The workspace must be zero-filled once before its first
 * use (cudaMemset) and may then be reused by any later call on the same stream;
 * the counters return to zero by themselves.  Calls that overlap on the GPU need
 * separate workspaces. */
size_t ternocl_gemv_workspace_size(int M, int N, int K);

/* ---------------------------------------------------------------------------------
 * int2 upconvert GEMM/GEMV.  Replaces int2_fp16_upcvt_gemm (int2_fp16_upcvt.cl:196-198)
 * and int2_fp16_upcvt_gemm_mt (int2_fp16_upcvt.cl:341-343):
 *   C[m,n] = DT(epi( sum_k A[m,k] * code(B[k,n]) * S[k/128, n] ))
 *   A : DT [M, K] row-major           B : uint32 [K/16, N], code of row 16kp+j at bits 2j..2j+1,
 *   S : DT [K/128, N]                     codes {0,1,3} = {0,+1,-1}
 *   C : DT (or fp32) [M, N]           Other : DT [M, N]     Bias : DT (or fp32) [N]
 * Requires N % 16 == 0, K % 128 == 0, M >= 1 (any M: ragged tiles are masked).
 */
int ternocl_int2_upcvt(const void *A, const uint32_t *B, const void *S, void *C, const void *Other,
                       const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32,
                       int algo, void *ws, size_t ws_bytes, void *stream);

/* Allocation-free int2 decode GEMV (no counterpart in the reference: its OpenCL
 * drivers always allocate their buffers).  For callers that cannot allocate device
 * memory where they run -- inside another framework's memory pool, in runtimes that
 * forbid allocation after start-up, in plugins whose host owns all allocations --
 * this computes the same C as ternocl_int2_upcvt (same arguments and rules, no
 * workspace argument) and takes its split-K scratch from a 16 MiB array the library
 * declares in device memory, which every GPU that loads the library holds until exit.
 *  - It runs the plan ternocl_int2_upcvt makes for a 16 MiB workspace (same kernel,
 *    warps and K split, bit-identical output).  A shape whose plan would need more
 *    scratch runs in the forms that need none; a shape that no form can run is
 *    rejected with TERNOCL_ERR_WORKSPACE.
 *  - The first call on a device looks up the array's address (cudaGetSymbolAddress,
 *    that device current) and keeps it; make that first call before any stream
 *    capture.  Resetting the device (cudaDeviceReset) while the library stays loaded
 *    is not supported.
 *  - All calls share the array: the arrival counters are cleared on `stream` before
 *    each launch; calls that overlap on the GPU race on it.
 *  - Calls no cudaMalloc, cudaFree or allocating library routine. */
int ternocl_int2_upcvt_noalloc(const void *A, const uint32_t *B, const void *S, void *C,
                               const void *Other, const void *Bias, int M, int N, int K, int dtype,
                               int postop, int out_f32, void *stream);

/* Column-sharded int2 GEMV with the all-gather fused into the epilogue (no counterpart in
 * the reference, which runs on one device; it replaces a GEMV per rank followed by an
 * NCCL all-gather of the outputs).  Rank `rank` of `world` (<= 8) holds the columns
 * [n0, n0 + nl) of the weights (B [K/16, nl], S [K/128, nl], contiguous shards) and
 * stores C[:, n0:n0+nl] into every rank's full C_ranks[r] ([M, N], 16-byte aligned device
 * pointers valid in this process, e.g. CUDA IPC mappings of the peers' buffers; Other
 * [M, N] and Bias [N] are full width): the CTAs store into this rank's own C, and the
 * grid's last CTA copies the slice into the other ranks' C over peer stores.  The launch
 * completes only after all ranks' columns have arrived: that CTA then writes `epoch`
 * into flags_ranks[r][rank] of every rank and
 * waits until flags_ranks[rank][r] >= epoch for all r (bounded; a timeout sets bit 2 of
 * ternocl_device_error).  flags start at 0 and a nonzero `epoch` must increase by one per
 * call, in the same order on every rank.  A rank must not read a C buffer after it has
 * launched the next call that writes it (double-buffer C if the output is consumed across
 * calls).  epoch == 0: the library counts the calls itself, on the device, in
 * flags_ranks[rank][world] (each rank's flag array then has world + 1 entries, all zero
 * at the start); no host value changes from call to call, so the call can be captured in
 * a CUDA graph and replayed, on every rank in the same order.  The wait for the peers is
 * bounded by TERNOCL_OPT_PEER_TIMEOUT_MS.  ws: >= ternocl_gemv_allgather_workspace_size(M,
 * nl, K) bytes, zeroed once, 256-byte aligned. */
size_t ternocl_gemv_allgather_workspace_size(int M, int nl, int K);
/* CUDA IPC helpers to map the peers' C and flag buffers (set-up time, not the hot path;
 * plain peer mappings, no multicast objects): the 64-byte handle and byte offset of a
 * device pointer inside its allocation, the mapping of a peer's handle + offset on the
 * current device (peer access enabled lazily), and its release. */
int ternocl_ipc_handle(const void *ptr, void *handle64, size_t *offset);
int ternocl_ipc_open(const void *handle64, size_t offset, void **ptr);
int ternocl_ipc_close(void *ptr, size_t offset);
int ternocl_int2_upcvt_allgather(const void *A, const uint32_t *B, const void *S, void *const *C_ranks,
                                 const void *Other, const void *Bias, int M, int N, int n0, int nl, int K,
                                 int dtype, int postop, int out_f32, int rank, int world,
                                 unsigned *const *flags_ranks, unsigned epoch, void *ws, size_t ws_bytes,
                                 void *stream);

/* ---------------------------------------------------------------------------------
 * int1 (binary) upconvert GEMM/GEMV.  Replaces int1_fp16_upcvt_gemm / _gemm_mt
 * (int1_fp16_upcvt.cl:166-170, 302-306).  B is the device "sel" layout, uint32
 * [K/32, N]: within K32 row kp and 16-column block n0, word (kp, n0+p) bit j =
 * sign of (row 32kp + 2p + (j&1), column n0 + j/2), bit 1 = -1
 * (int1_fp16_upcvt/main.cpp:78-92).  Other arguments as ternocl_int2_upcvt. */
int ternocl_int1_upcvt(const void *A, const uint32_t *B, const void *S, void *C, const void *Other,
                       const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32,
                       int algo, void *ws, size_t ws_bytes, void *stream);

/* ---------------------------------------------------------------------------------
 * s8 x s2 path (int2_via_int2_x_int8_dpas).
 *
 * Activation quantisation pre-kernel, replaces quant_a (int2_int8_dpas.cl:105-106):
 *   SA[g, m] = DT(127 / max(FLT_EPSILON, max_{k in group g} |A[m,k]|))  (correctly rounded)
 *   Aq[m, k] = sat_int8(rint(A[m,k] * SA[g,m]))   (round to nearest even; only if Aq != NULL)
 * SA : DT [K/128, LDSA], LDSA = (M + 31) & ~31 (int2_int8_dpas.cl:58).  Columns m >= M of
 * SA are not written. */
int ternocl_int8_ldsa(int M);
int ternocl_int8_quant_a(const void *A, void *SA, int8_t *Aq, int M, int K, int dtype,
                         void *stream);

/* s8 x s2 GEMM/GEMV, replaces int2_int8_gemv / int2_int8_gemm_mt
 * (int2_int8_dpas.cl:213-215, 316-318):
 *   C[m,n] = DT(epi( sum_g float(sum_{k in g} q[m,k] * code(B[k,n])) * (SB[g,n] * (1/SA[g,m])) ))
 * with int32 dot products per 128-group.  qmode 0: reads the int8 Aq written by
 * ternocl_int8_quant_a; qmode 1: quantises A from SA, q = sat_int8(rint(A * SA)) (Aq
 * unused; may be a dummy buffer, as the reference driver passes in qmode 1).  The
 * tensor-core GEMM (algo GEMM, or AUTO from M >= 64; SA 16-byte aligned) runs qmode 1 as
 * one quantisation pass into M x K bytes of stream-ordered scratch from a pool of the
 * library that keeps its pages (cudaMallocFromPoolAsync / cudaFreeAsync on `stream`;
 * capturable), then the int8 GEMM: the codes, and so C, equal qmode 0's.
 * B as ternocl_int2_upcvt (codes read as 2-bit two's complement). */
int ternocl_int2_int8(const void *A, const int8_t *Aq, const void *SA, const uint32_t *B,
                      const void *SB, void *C, const void *Other, const void *Bias, int M, int N,
                      int K, int dtype, int postop, int out_f32, int qmode, int algo, void *stream);

/* Debug view of the s8 x s2 contraction: Dots[m, g, n] = sum_{k in g} Aq[m,k] * code(B[k,n])
 * (int32).  Used to check the integer path bit for bit. */
int ternocl_int2_int8_group_dots(const int8_t *Aq, const uint32_t *B, int32_t *Dots, int M, int N,
                                 int K, void *stream);

/* ---------------------------------------------------------------------------------
 * BITCOS upconvert GEMM/GEMV, replaces bitcos_fp16_upcvt_gemv / _gemm_mt
 * (bitcos_fp16_upcvt.cl:179-181, 303-305).  B is one uint32 buffer: bitmap [K/32][N]
 * (bit c of word (kp,n) = weight(32kp+c, n) != 0) | offsets [N] (first sign word of
 * column n) | signs (one bit per non-zero, column-major in k, 1 -> -1) | pad
 * (common/bitcos.hpp:1-8).  SR = slice_ranks [(ls-1), N] for ls K-slices (may be NULL
 * when ls == 1).  Requires N % 16 == 0, K % 128 == 0, K % (64 * ls) == 0.  algo: GEMV,
 * GEMM (the M-tiled tcgen05 kernel; walks all of K per tile, so ls and SR are not read),
 * or AUTO (GEMM from M >= 64). */
int ternocl_bitcos_upcvt(const void *A, const uint32_t *B, const void *S, const uint32_t *SR,
                         int ls, void *C, const void *Other, const void *Bias, int M, int N, int K,
                         int dtype, int postop, int out_f32, int algo, void *stream);

/* ---------------------------------------------------------------------------------
 * Sign flip + blockwise normalised Walsh-Hadamard transform, replaces hadamard_fwht
 * (hadamard/hadamard_fwht.cl:63-64):  y = H_HB(s .* x) / sqrt(HB) per HB-wide block of
 * each row of x [rows, K]; signs int8 +-1 [K] (ignored when use_signs == 0).
 * HB in {256, 512, 1024, 2048, 4096}, K % HB == 0.  y may alias x. */
int ternocl_hadamard_fwht(const void *x, const int8_t *signs, void *y, int rows, int K, int hb,
                          int use_signs, int dtype, void *stream);

/* Hadamard-transformed BITCOS GEMV: ternocl_hadamard_fwht of A (signs, use_signs, hb)
 * followed by ternocl_bitcos_upcvt on the result, in one launch with the transform done
 * while the GEMV stages its activation slice (no intermediate in global memory).  The
 * transformed activations are bit-identical to ternocl_hadamard_fwht's.  At M <= 8 (and
 * TERNOCL_OPT_BITCOS_GEMV 0) the persistent strip kernel runs it, each CTA transforming
 * its rows once while its first strips load: the output equals the two-kernel pipeline's
 * bit for bit.  Otherwise the K-sliced GEMV kernel (8-row blocks) splits K on hb
 * boundaries and transforms each slice.  hb in {256, 512, 1024}, K % hb == 0, signs
 * 16-byte aligned. */
int ternocl_bitcos_upcvt_hadamard(const void *A, const int8_t *signs, int use_signs, int hb, const uint32_t *B,
                                  const void *S, const uint32_t *SR, int ls, void *C, const void *Other,
                                  const void *Bias, int M, int N, int K, int dtype, int postop, int out_f32,
                                  void *stream);

/* ---------------------------------------------------------------------------------
 * int2 MoE prefill (int2_moe/int2_moe_prefill.cl).  G = T * topk routed rows.
 *
 * Route, replaces int2_moe_route (int2_moe_prefill.cl:30-31): from ids[G] (expert of
 * row g = t*topk + j) build meta[2E+2] = [E+1 row offsets | E+1 row-tile offsets],
 * perm[G] (sorted row p -> g, ascending g inside an expert) and inv[G] (g -> p).
 * rows_per_tile must equal ternocl_moe_rows_per_tile() for ternocl_moe_gemm. */
int ternocl_moe_rows_per_tile(void);
int ternocl_moe_route(const int32_t *ids, int32_t *meta, int32_t *perm, int32_t *inv, int G,
                      int num_experts, int rows_per_tile, void *stream);
/* Gather, replaces int2_moe_gather (int2_moe_prefill.cl:64): Xs[p] = X[perm[p] / topk]. */
int ternocl_moe_gather(const void *X, const int32_t *perm, void *Xs, int G, int K, int topk,
                       void *stream);
/* Grouped GEMM, replaces int2_moe_gemm_mt (int2_moe_prefill.cl:75-77): for the rows p
 * of every expert e, C[p, n] = epi(A[p] . B_e[:, n]); B_all [E, K/16, N],
 * S_all [E, K/128, N]; Other_all [G, N] (POSTOP 1/2).  max_rows = G. */
int ternocl_moe_gemm(const int32_t *meta, const void *A_all, const uint32_t *B_all,
                     const void *S_all, void *C_all, const void *Other_all, int G, int N, int K,
                     int num_experts, int dtype, int postop, int out_f32, void *stream);
/* int8 variant (int2_moe/int2_moe_prefill_int8.cl), qmode 0: ternocl_int8_quant_a on the T
 * token rows gives Xq [T, K] and SAt [K/128, LDSA(T)]; gather_q, replaces int2_moe_gather_q
 * (int2_moe_prefill_int8.cl:74-75), moves them into expert order:
 *   Xsq[p] = Xq[t], SA[g, p] = SAt[g, t], t = perm[p] / topk;  SA [K/128, LDSA(G)], G = T*topk. */
int ternocl_moe_gather_q(const int8_t *Xq, const void *SAt, const int32_t *perm, int8_t *Xsq, void *SA, int T,
                         int G, int K, int topk, void *stream);
/* Grouped s8 x s2 GEMM, replaces int2_moe_gemm_mt_i8 (int2_moe_prefill_int8.cl:88-91): for
 * the rows p of every expert e,
 *   C[p, n] = epi( sum_g float(dot_g(Aq[p], B_e[:, n])) * (SB_e[g, n] * (1 / SA[g, p])) )
 * (the ternocl_int2_int8 formula per expert).  Aq_all int8 [G, K], SA [K/128, LDSA(G)]
 * (16-byte aligned), B_all [E, K/16, N], SB_all [E, K/128, N], Other_all [G, N] (POSTOP
 * 1/2), no bias.  qmode must be 0 (A_all unused): the codes of the reference's in-GEMM
 * quantisation (qmode 1) equal ternocl_int8_quant_a's, since a * SA is exact in fp32. */
int ternocl_moe_gemm_i8(const int32_t *meta, const void *A_all, const int8_t *Aq_all, const void *SA,
                        const uint32_t *B_all, const void *SB_all, void *C_all, const void *Other_all, int G,
                        int N, int K, int num_experts, int dtype, int postop, int out_f32, int qmode,
                        void *stream);
/* Combine, replaces int2_moe_combine (int2_moe_prefill.cl:144-145):
 * O[t, n] = DT(sum_j RW[t*topk+j] * Y[inv[t*topk+j], n]),  Y fp32 [G, N]. */
int ternocl_moe_combine(const float *Y, const int32_t *inv, const void *RW, void *O, int T, int N,
                        int topk, int dtype, void *stream);

/* ---------------------------------------------------------------------------------
 * int2 MoE decode (int2_moe/int2_moe.cl:63-174), every routed (token, expert) pair in one
 * launch.  ids[G] = expert of row g = t*topk + j; B* [E, K/16, N], S* [E, K/128, N] per
 * projection (E = num_experts); fp32 accumulation per 128-row group as the int2 GEMV.
 * An expert id outside [0, E) contributes zero and sets bit 1 of ternocl_device_error.
 *
 * gate_up, replaces int2_moe_gate_up (:65-67), X [T, K] with T = G / topk:
 *   H[g, n] = DT(silu(X[g/topk] . gate_e[:, n]) * (X[g/topk] . up_e[:, n]))   H [G, N] */
int ternocl_moe_decode_gate_up(const int32_t *ids, const void *X, const uint32_t *Bg, const void *Sg,
                               const uint32_t *Bu, const void *Su, void *H, int G, int N, int K, int topk,
                               int num_experts, int dtype, void *stream);
/* down, replaces int2_moe_down (:103-104): Y[g, n] = RW[g] * (H[g] . down_e[:, n]), Y fp32 [G, N] */
int ternocl_moe_decode_down(const int32_t *ids, const void *H, const void *RW, const uint32_t *B, const void *S,
                            float *Y, int G, int N, int K, int num_experts, int dtype, void *stream);
/* reduce, replaces int2_moe_reduce (:131): O[t, n] = DT(sum_j Y[t*topk + j, n]), j ascending */
int ternocl_moe_decode_reduce(const float *Y, void *O, int T, int N, int topk, int dtype, void *stream);
/* down_sum, replaces int2_moe_down_sum (:148-149), down + reduce in one launch:
 *   O[t, n] = DT(sum_j RW[g] * (H[g] . down_e[:, n])),  g = t*topk + j */
int ternocl_moe_decode_down_sum(const int32_t *ids, const void *H, const void *RW, const uint32_t *B,
                                const void *S, void *O, int T, int N, int K, int topk, int num_experts, int dtype,
                                void *stream);

/* ---------------------------------------------------------------------------------
 * Host-side weight packers (no device work).  Same layouts as the reference's
 * common/bitcos.hpp and int1 driver.
 *
 * BITCOS random ternary weights at zero density z, bit-identical to
 * bitcos_random() (common/bitcos.hpp:31-78) for the same seed and OpenMP thread
 * count.  Returns the buffer length in words; writes it when cap >= length. */
size_t ternocl_bitcos_random(int K, int N, double z, uint64_t seed, uint32_t *out, size_t cap);
/* Pack codes [K, N] (row-major, values -1/0/+1) into a BITCOS buffer. */
size_t ternocl_bitcos_pack(const int8_t *codes, int K, int N, uint32_t *out, size_t cap);
/* slice_ranks [(ls-1), N] (common/bitcos.hpp:81-94). */
int ternocl_bitcos_slice_ranks(const uint32_t *buf, int K, int N, int ls, uint32_t *out);
/* int1 per-column bit order [K/32, N] -> device sel layout (int1_fp16_upcvt/main.cpp:80-92). */
int ternocl_int1_to_sel(const uint32_t *B, uint32_t *out, int K, int N);

#ifdef __cplusplus
}
#endif
#endif /* TERNOCL_H */
