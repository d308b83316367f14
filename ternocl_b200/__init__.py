"""ternocl_b200: B200-native ternary-weight GEMM/GEMV (host-side Python mirror).

Every function here is a thin wrapper over one C-ABI entry point of libternocl.so
(include/ternocl.h), taking CUDA torch tensors for device memory: PyTorch is only the
allocator/stream plumbing, the arithmetic is the library's sm_100a kernels.  The
argument order mirrors the reference kernels' (A, B, S, C, Other, Bias, M, N, K);
the reference's compile-time options (dtype, POSTOP, OUT_F32, QMODE, HB, TOPK) are
keyword arguments.  Errors raise TernoclError; there is no CPU fallback.
"""
from ._lib import LIB_PATH, TernoclError, call, header_functions, lib  # noqa: F401

FP16, BF16 = 0, 1
POSTOP_NONE, POSTOP_SILU_MUL, POSTOP_ADD, POSTOP_BIAS, POSTOP_SIGMOID = range(5)
ALGO_AUTO, ALGO_GEMV, ALGO_GEMM, ALGO_GEMV_TMEM = 0, 1, 2, 3
OPT_PDL = 1
OPT_GEMM_TILE_M = 2
OPT_GEMV_SPLIT = 3
OPT_GEMV_WARPS = 4
OPT_GEMM_PERSISTENT = 5
OPT_GEMV_IMPL = 6
OPT_GEMV_STAGES = 7  # reserved: setting it returns -1
OPT_PEER_TIMEOUT_MS = 8
OPT_BITCOS_GEMV = 9


def _torch():
    import torch
    return torch


def dtype_code(t):
    torch = _torch()
    if t.dtype == torch.float16:
        return FP16
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError("activations must be float16 or bfloat16, got %s" % t.dtype)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream):
    torch = _torch()
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream


def _check_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("tensors must be contiguous CUDA tensors")


def set_option(option, value):
    return lib().ternocl_set_option(option, int(value))


def device_error(reset=True):
    """Device error word (bit 0: a bounded in-kernel wait timed out)."""
    return lib().ternocl_device_error(int(bool(reset)))


class Workspace:
    """Zero-initialised device scratch for split-K partials and arrival counters.

    Grows on demand (a growth allocates through torch, outside the kernel call)."""

    def __init__(self, device=None, nbytes=0):
        self.device = device
        self.buf = None
        self.reserve(nbytes)

    def reserve(self, nbytes):
        torch = _torch()
        if nbytes and (self.buf is None or self.buf.numel() < nbytes):
            self.buf = torch.zeros(int(nbytes), dtype=torch.uint8, device=self.device or "cuda")
        return self

    def ptr(self):
        return None if self.buf is None else self.buf.data_ptr()

    def nbytes(self):
        return 0 if self.buf is None else self.buf.numel()


def gemv_workspace_size(M, N, K):
    return lib().ternocl_gemv_workspace_size(M, N, K)


def _out(M, N, like, out_f32, out):
    torch = _torch()
    if out is not None:
        return out
    return torch.empty(M, N, dtype=torch.float32 if out_f32 else like.dtype, device=like.device)


def _upcvt(entry, A, B, S, postop, out_f32, other, bias, out, algo, workspace, stream):
    _check_cuda(A, B, S, other, bias, out)
    M, K = A.shape
    N = B.shape[1]
    C = _out(M, N, A, out_f32, out)
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        workspace.reserve(gemv_workspace_size(M, N, K))
        ws_ptr, ws_bytes = workspace.ptr(), workspace.nbytes()
    call(entry, _ptr(A), _ptr(B), _ptr(S), _ptr(C), _ptr(other), _ptr(bias), M, N, K,
         dtype_code(A), int(postop), int(bool(out_f32)), int(algo), ws_ptr, ws_bytes,
         _stream(stream))
    return C


def int2_upcvt(A, B, S, postop=0, out_f32=False, other=None, bias=None, out=None, algo=0,
               workspace=None, stream=None):
    """C = epi(A @ dequant_int2(B, S)); A [M,K] fp16/bf16, B int32 [K/16,N], S [K/128,N]."""
    return _upcvt("ternocl_int2_upcvt", A, B, S, postop, out_f32, other, bias, out, algo,
                  workspace, stream)


def int1_upcvt(A, B, S, postop=0, out_f32=False, other=None, bias=None, out=None, algo=0,
               workspace=None, stream=None):
    """C = epi(A @ dequant_int1(B, S)); B int32 [K/32,N] in the device sel layout."""
    return _upcvt("ternocl_int1_upcvt", A, B, S, postop, out_f32, other, bias, out, algo,
                  workspace, stream)


def int8_ldsa(M):
    """Row pitch of SA (elements): (M + 31) & ~31, as LDSA() of the reference kernel."""
    return lib().ternocl_int8_ldsa(M)


def int8_quant_a(A, write_q=True, stream=None):
    """Per-(row, 128-group) activation scales SA [K/128, ldsa(M)] (dtype of A) and, with
    write_q, the int8 codes Aq [M, K].  Returns (SA, Aq or None)."""
    torch = _torch()
    _check_cuda(A)
    M, K = A.shape
    SA = torch.zeros(K // 128, int8_ldsa(M), dtype=A.dtype, device=A.device)
    Aq = torch.empty(M, K, dtype=torch.int8, device=A.device) if write_q else None
    call("ternocl_int8_quant_a", _ptr(A), _ptr(SA), _ptr(Aq), M, K, dtype_code(A), _stream(stream))
    return SA, Aq


def int2_int8(A, B, SB, SA, Aq=None, qmode=None, postop=0, out_f32=False, other=None, bias=None,
              out=None, algo=0, stream=None):
    """s8 x s2: C = epi(sum_g float(int32 dot_g) * (SB * 1/SA)).  qmode 0 reads Aq
    (from int8_quant_a), qmode 1 quantises A in the kernel; default: 0 if Aq is given."""
    _check_cuda(A, B, SB, SA, Aq, other, bias, out)
    if qmode is None:
        qmode = 0 if Aq is not None else 1
    M, K = A.shape
    N = B.shape[1]
    C = _out(M, N, A, out_f32, out)
    call("ternocl_int2_int8", _ptr(A), _ptr(Aq), _ptr(SA), _ptr(B), _ptr(SB), _ptr(C), _ptr(other),
         _ptr(bias), M, N, K, dtype_code(A), int(postop), int(bool(out_f32)), int(qmode), int(algo),
         _stream(stream))
    return C


def int2_int8_group_dots(Aq, B, stream=None):
    """int32 Dots [M, K/128, N] = per-group sum of Aq[m, k] * code(B[k, n])."""
    torch = _torch()
    _check_cuda(Aq, B)
    M, K = Aq.shape
    N = B.shape[1]
    D = torch.empty(M, K // 128, N, dtype=torch.int32, device=Aq.device)
    call("ternocl_int2_int8_group_dots", _ptr(Aq), _ptr(B), _ptr(D), M, N, K, _stream(stream))
    return D


def bitcos_upcvt(A, B, S, SR=None, ls=1, postop=0, out_f32=False, other=None, bias=None, out=None,
                 algo=0, stream=None):
    """C = epi(A @ decode_bitcos(B) * S); B: one int32 buffer bitmap | offsets | signs | pad,
    SR: slice_ranks [ls-1, N] (None when ls == 1)."""
    _check_cuda(A, B, S, SR, other, bias, out)
    M, K = A.shape
    N = S.shape[1]
    C = _out(M, N, A, out_f32, out)
    call("ternocl_bitcos_upcvt", _ptr(A), _ptr(B), _ptr(S), _ptr(SR), int(ls), _ptr(C), _ptr(other),
         _ptr(bias), M, N, K, dtype_code(A), int(postop), int(bool(out_f32)), int(algo), _stream(stream))
    return C


def bitcos_upcvt_hadamard(A, B, S, hb, signs=None, SR=None, ls=1, postop=0, out_f32=False, other=None, bias=None,
                          out=None, stream=None):
    """C = epi(H_hb(signs * A) / sqrt(hb) @ decode_bitcos(B) * S) in one launch: the transform of
    hadamard_fwht done while the BITCOS GEMV stages its activations."""
    _check_cuda(A, B, S, SR, signs, other, bias, out)
    M, K = A.shape
    N = S.shape[1]
    C = _out(M, N, A, out_f32, out)
    call("ternocl_bitcos_upcvt_hadamard", _ptr(A), _ptr(signs), int(signs is not None), int(hb), _ptr(B), _ptr(S),
         _ptr(SR), int(ls), _ptr(C), _ptr(other), _ptr(bias), M, N, K, dtype_code(A), int(postop),
         int(bool(out_f32)), _stream(stream))
    return C


def bitcos_random(K, N, z, seed):
    """Host BITCOS buffer (numpy uint32) of random ternary weights at zero density z."""
    import numpy as np
    L = lib()
    n = L.ternocl_bitcos_random(K, N, float(z), int(seed), None, 0)
    out = np.empty(n, np.uint32)
    L.ternocl_bitcos_random(K, N, float(z), int(seed), out.ctypes.data, n)
    return out


def bitcos_pack(codes):
    """codes [K, N] int8 in {-1, 0, +1} -> host BITCOS buffer (numpy uint32)."""
    import numpy as np
    codes = np.ascontiguousarray(codes, np.int8)
    K, N = codes.shape
    L = lib()
    n = L.ternocl_bitcos_pack(codes.ctypes.data, K, N, None, 0)
    out = np.empty(n, np.uint32)
    L.ternocl_bitcos_pack(codes.ctypes.data, K, N, out.ctypes.data, n)
    return out


def bitcos_slice_ranks(buf, K, N, ls):
    """slice_ranks [ls-1, N] (numpy uint32) of a host BITCOS buffer."""
    import numpy as np
    buf = np.ascontiguousarray(buf, np.uint32)
    out = np.zeros((max(ls - 1, 0), N), np.uint32)
    if ls > 1:
        call("ternocl_bitcos_slice_ranks", buf.ctypes.data, K, N, ls, out.ctypes.data)
    return out


def hadamard_fwht(x, hb, signs=None, out=None, stream=None):
    """y = H_hb(signs * x) / sqrt(hb) per hb-wide block of each row of x [rows, K]
    (fp16/bf16); signs: int8 +-1 [K] or None.  out may be x (in place)."""
    torch = _torch()
    _check_cuda(x, signs, out)
    rows, K = x.shape
    y = torch.empty_like(x) if out is None else out
    call("ternocl_hadamard_fwht", _ptr(x), _ptr(signs), _ptr(y), rows, K, int(hb), int(signs is not None),
         dtype_code(x), _stream(stream))
    return y


def moe_rows_per_tile():
    return lib().ternocl_moe_rows_per_tile()


def moe_route(ids, num_experts, stream=None):
    """ids int32 [G] (expert of routed row g = t*topk + j) -> (meta [2E+2], perm [G], inv [G])."""
    torch = _torch()
    _check_cuda(ids)
    G = ids.numel()
    meta = torch.empty(2 * num_experts + 2, dtype=torch.int32, device=ids.device)
    perm = torch.empty(G, dtype=torch.int32, device=ids.device)
    inv = torch.empty(G, dtype=torch.int32, device=ids.device)
    call("ternocl_moe_route", _ptr(ids), _ptr(meta), _ptr(perm), _ptr(inv), G, int(num_experts),
         moe_rows_per_tile(), _stream(stream))
    return meta, perm, inv


def moe_gather(X, perm, topk, out=None, stream=None):
    """Xs[p] = X[perm[p] / topk]."""
    torch = _torch()
    _check_cuda(X, perm, out)
    G = perm.numel()
    K = X.shape[1]
    Xs = torch.empty(G, K, dtype=X.dtype, device=X.device) if out is None else out
    call("ternocl_moe_gather", _ptr(X), _ptr(perm), _ptr(Xs), G, K, int(topk), _stream(stream))
    return Xs


def moe_gemm(meta, A, B_all, S_all, num_experts, postop=0, out_f32=False, other=None, out=None, stream=None):
    """Per-expert C[p] = epi(A[p] @ dequant(B_all[e], S_all[e])) for the sorted rows p of expert e.
    A [G, K]; B_all int32 [E, K/16, N]; S_all [E, K/128, N]; other [G, N] for POSTOP 1/2."""
    _check_cuda(meta, A, B_all, S_all, other, out)
    G, K = A.shape
    N = B_all.shape[-1]
    C = _out(G, N, A, out_f32, out)
    call("ternocl_moe_gemm", _ptr(meta), _ptr(A), _ptr(B_all), _ptr(S_all), _ptr(C), _ptr(other), G, N, K,
         int(num_experts), dtype_code(A), int(postop), int(bool(out_f32)), _stream(stream))
    return C


def moe_gather_q(Xq, SAt, perm, topk, stream=None):
    """int8 rows Xq [T, K] and scales SAt [K/128, LDSA(T)] -> expert order: (Xsq [G, K], SA [K/128, LDSA(G)])."""
    torch = _torch()
    _check_cuda(Xq, SAt, perm)
    T, K = Xq.shape
    G = perm.numel()
    Xsq = torch.empty(G, K, dtype=torch.int8, device=Xq.device)
    SA = torch.empty(K // 128, int8_ldsa(G), dtype=SAt.dtype, device=Xq.device)
    call("ternocl_moe_gather_q", _ptr(Xq), _ptr(SAt), _ptr(perm), _ptr(Xsq), _ptr(SA), T, G, K, int(topk),
         _stream(stream))
    return Xsq, SA


def moe_gemm_i8(meta, Aq, SA, B_all, SB_all, num_experts, postop=0, out_f32=False, other=None, out=None,
                stream=None):
    """Grouped s8 x s2 GEMM over the expert-sorted int8 rows Aq [G, K] with scales SA [K/128, LDSA(G)];
    B_all int32 [E, K/16, N], SB_all [E, K/128, N] (fp16/bf16, the output type)."""
    _check_cuda(meta, Aq, SA, B_all, SB_all, other, out)
    G, K = Aq.shape
    N = B_all.shape[-1]
    C = _out(G, N, SB_all, out_f32, out)
    call("ternocl_moe_gemm_i8", _ptr(meta), None, _ptr(Aq), _ptr(SA), _ptr(B_all), _ptr(SB_all), _ptr(C),
         _ptr(other), G, N, K, int(num_experts), dtype_code(SB_all), int(postop), int(bool(out_f32)), 0,
         _stream(stream))
    return C


def moe_combine(Y, inv, RW, T, topk, out=None, stream=None):
    """O[t] = sum_j RW[t*topk+j] * Y[inv[t*topk+j]]; Y fp32 [G, N], RW [G] fp16/bf16."""
    torch = _torch()
    _check_cuda(Y, inv, RW, out)
    N = Y.shape[1]
    O = torch.empty(T, N, dtype=RW.dtype, device=Y.device) if out is None else out
    call("ternocl_moe_combine", _ptr(Y), _ptr(inv), _ptr(RW), _ptr(O), int(T), N, int(topk), dtype_code(RW),
         _stream(stream))
    return O


def moe_decode_gate_up(ids, X, Bg, Sg, Bu, Su, num_experts, topk, out=None, stream=None):
    """H[g] = silu(X[g/topk] . gate_e) * (X[g/topk] . up_e), e = ids[g]; Bg/Bu [E, K/16, N]."""
    torch = _torch()
    _check_cuda(ids, X, Bg, Sg, Bu, Su, out)
    G = ids.numel()
    K = X.shape[1]
    N = Sg.shape[-1]
    H = torch.empty(G, N, dtype=X.dtype, device=X.device) if out is None else out
    call("ternocl_moe_decode_gate_up", _ptr(ids), _ptr(X), _ptr(Bg), _ptr(Sg), _ptr(Bu), _ptr(Su), _ptr(H), G, N, K,
         int(topk), int(num_experts), dtype_code(X), _stream(stream))
    return H


def moe_decode_down(ids, H, RW, B, S, num_experts, out=None, stream=None):
    """Y[g] = RW[g] * (H[g] . down_e), e = ids[g]; fp32 [G, N]."""
    torch = _torch()
    _check_cuda(ids, H, RW, B, S, out)
    G, K = H.shape
    N = S.shape[-1]
    Y = torch.empty(G, N, dtype=torch.float32, device=H.device) if out is None else out
    call("ternocl_moe_decode_down", _ptr(ids), _ptr(H), _ptr(RW), _ptr(B), _ptr(S), _ptr(Y), G, N, K,
         int(num_experts), dtype_code(H), _stream(stream))
    return Y


def moe_decode_reduce(Y, T, topk, dtype, out=None, stream=None):
    """O[t] = sum_j Y[t*topk + j] (j ascending), in fp16/bf16 (dtype: a torch dtype)."""
    torch = _torch()
    _check_cuda(Y, out)
    N = Y.shape[1]
    O = torch.empty(T, N, dtype=dtype, device=Y.device) if out is None else out
    call("ternocl_moe_decode_reduce", _ptr(Y), _ptr(O), int(T), N, int(topk), dtype_code(O), _stream(stream))
    return O


def moe_decode_down_sum(ids, H, RW, B, S, num_experts, topk, out=None, stream=None):
    """O[t] = sum_j RW[g] * (H[g] . down_e), g = t*topk + j, e = ids[g]."""
    torch = _torch()
    _check_cuda(ids, H, RW, B, S, out)
    G, K = H.shape
    T = G // int(topk)
    N = S.shape[-1]
    O = torch.empty(T, N, dtype=H.dtype, device=H.device) if out is None else out
    call("ternocl_moe_decode_down_sum", _ptr(ids), _ptr(H), _ptr(RW), _ptr(B), _ptr(S), _ptr(O), T, N, K, int(topk),
         int(num_experts), dtype_code(H), _stream(stream))
    return O
