"""PyTorch custom operators over the C ABI, for a framework caller (vLLM-style linear and
MoE layers) that dispatches through torch.ops and captures CUDA graphs or traces with
torch.compile: `torch.ops.ternocl.<name>`.

Each operator runs the library's sm_100a kernels on the current CUDA stream (there is no
CPU kernel), allocates its output with the caching allocator, and has a fake (meta)
implementation giving the output's shape and dtype, so graph capture and tracing see the
operator without running it.  The activation may carry leading batch dimensions
([..., K]); they are flattened into M rows.

  int2_linear / int1_linear   ternocl_int2_upcvt / ternocl_int1_upcvt
  bitcos_linear               ternocl_bitcos_upcvt
  bitcos_hadamard_linear      ternocl_bitcos_upcvt_hadamard
  int8_linear                 ternocl_int8_quant_a + ternocl_int2_int8 (qmode 0)
  hadamard                    ternocl_hadamard_fwht
  moe_prefill                 route, gather (or quant + gather_q), up, gate (SiLU x up),
                              down, combine: the int2_moe/prefill.cpp layer
  moe_decode                  gate_up + down_sum: the int2_moe/main.cpp layer (--fused)
"""
from typing import Optional

import torch

import ternocl_b200 as tl

_NS = "ternocl"


def _rows(A):
    return A.reshape(-1, A.shape[-1]).contiguous()


def _fake_linear(A, N, out_f32):
    return A.new_empty((*A.shape[:-1], N), dtype=torch.float32 if out_f32 else A.dtype)


@torch.library.custom_op(_NS + "::int2_linear", mutates_args=())
def int2_linear(A: torch.Tensor, B: torch.Tensor, S: torch.Tensor, postop: int = 0, out_f32: bool = False,
                other: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = epi(A @ dequant_int2(B, S)); B int32 [K/16, N], S [K/128, N]."""
    C = tl.int2_upcvt(_rows(A), B, S, postop=postop, out_f32=out_f32,
                      other=None if other is None else _rows(other), bias=bias)
    return C.reshape(*A.shape[:-1], B.shape[1])


@int2_linear.register_fake
def _(A, B, S, postop=0, out_f32=False, other=None, bias=None):
    return _fake_linear(A, B.shape[1], out_f32)


@torch.library.custom_op(_NS + "::int1_linear", mutates_args=())
def int1_linear(A: torch.Tensor, B: torch.Tensor, S: torch.Tensor, postop: int = 0, out_f32: bool = False,
                other: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = epi(A @ dequant_int1(B, S)); B int32 [K/32, N] in the device sel layout."""
    C = tl.int1_upcvt(_rows(A), B, S, postop=postop, out_f32=out_f32,
                      other=None if other is None else _rows(other), bias=bias)
    return C.reshape(*A.shape[:-1], B.shape[1])


@int1_linear.register_fake
def _(A, B, S, postop=0, out_f32=False, other=None, bias=None):
    return _fake_linear(A, B.shape[1], out_f32)


@torch.library.custom_op(_NS + "::bitcos_linear", mutates_args=())
def bitcos_linear(A: torch.Tensor, B: torch.Tensor, S: torch.Tensor, SR: Optional[torch.Tensor] = None,
                  ls: int = 1, postop: int = 0, out_f32: bool = False, other: Optional[torch.Tensor] = None,
                  bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = epi(A @ decode_bitcos(B) * S); B the BITCOS buffer, S [K/128, N], SR the slice ranks."""
    C = tl.bitcos_upcvt(_rows(A), B, S, SR=SR, ls=ls, postop=postop, out_f32=out_f32,
                        other=None if other is None else _rows(other), bias=bias)
    return C.reshape(*A.shape[:-1], S.shape[1])


@bitcos_linear.register_fake
def _(A, B, S, SR=None, ls=1, postop=0, out_f32=False, other=None, bias=None):
    return _fake_linear(A, S.shape[1], out_f32)


@torch.library.custom_op(_NS + "::bitcos_hadamard_linear", mutates_args=())
def bitcos_hadamard_linear(A: torch.Tensor, B: torch.Tensor, S: torch.Tensor, hb: int,
                           signs: Optional[torch.Tensor] = None, SR: Optional[torch.Tensor] = None, ls: int = 1,
                           postop: int = 0, out_f32: bool = False, other: Optional[torch.Tensor] = None,
                           bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bitcos_linear of the sign-flipped, blockwise Hadamard-transformed A, in one launch."""
    C = tl.bitcos_upcvt_hadamard(_rows(A), B, S, hb, signs=signs, SR=SR, ls=ls, postop=postop, out_f32=out_f32,
                                 other=None if other is None else _rows(other), bias=bias)
    return C.reshape(*A.shape[:-1], S.shape[1])


@bitcos_hadamard_linear.register_fake
def _(A, B, S, hb, signs=None, SR=None, ls=1, postop=0, out_f32=False, other=None, bias=None):
    return _fake_linear(A, S.shape[1], out_f32)


@torch.library.custom_op(_NS + "::int8_linear", mutates_args=())
def int8_linear(A: torch.Tensor, B: torch.Tensor, SB: torch.Tensor, postop: int = 0, out_f32: bool = False,
                other: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """s8 x s2: A quantised per row and 128-group (quant_a), then the int8 GEMM/GEMV."""
    A2 = _rows(A)
    SA, Aq = tl.int8_quant_a(A2)
    C = tl.int2_int8(A2, B, SB, SA, Aq=Aq, qmode=0, postop=postop, out_f32=out_f32,
                     other=None if other is None else _rows(other), bias=bias)
    return C.reshape(*A.shape[:-1], B.shape[1])


@int8_linear.register_fake
def _(A, B, SB, postop=0, out_f32=False, other=None, bias=None):
    return _fake_linear(A, B.shape[1], out_f32)


@torch.library.custom_op(_NS + "::hadamard", mutates_args=())
def hadamard(x: torch.Tensor, hb: int, signs: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = H_hb(signs * x) / sqrt(hb) per hb-wide block of the last dimension."""
    return tl.hadamard_fwht(_rows(x), hb, signs=signs).reshape(x.shape)


@hadamard.register_fake
def _(x, hb, signs=None):
    return torch.empty_like(x)


@torch.library.custom_op(_NS + "::moe_prefill", mutates_args=())
def moe_prefill(X: torch.Tensor, ids: torch.Tensor, RW: torch.Tensor, Bg: torch.Tensor, Sg: torch.Tensor,
                Bu: torch.Tensor, Su: torch.Tensor, Bd: torch.Tensor, Sd: torch.Tensor, num_experts: int,
                topk: int, int8: bool = False) -> torch.Tensor:
    """The MoE prefill layer: X [T, H]; ids, RW [T, topk] (expert ids int32, gate weights);
    B*/S* the experts' int2 weights [E, K/16, N] and scales [E, K/128, N]; returns [T, H]."""
    X2 = _rows(X)
    T = X2.shape[0]
    ids1 = ids.reshape(-1).contiguous()
    meta, perm, inv = tl.moe_route(ids1, num_experts)
    if int8:
        SAt, Xq = tl.int8_quant_a(X2)
        Xsq, SA1 = tl.moe_gather_q(Xq, SAt, perm, topk)
        up = tl.moe_gemm_i8(meta, Xsq, SA1, Bu, Su, num_experts)
        H = tl.moe_gemm_i8(meta, Xsq, SA1, Bg, Sg, num_experts, postop=1, other=up)
        SA2, Hq = tl.int8_quant_a(H)
        Y = tl.moe_gemm_i8(meta, Hq, SA2, Bd, Sd, num_experts, out_f32=True)
    else:
        Xs = tl.moe_gather(X2, perm, topk)
        up = tl.moe_gemm(meta, Xs, Bu, Su, num_experts)
        H = tl.moe_gemm(meta, Xs, Bg, Sg, num_experts, postop=1, other=up)
        Y = tl.moe_gemm(meta, H, Bd, Sd, num_experts, out_f32=True)
    return tl.moe_combine(Y, inv, RW.reshape(-1).contiguous(), T, topk).reshape(X.shape)


@moe_prefill.register_fake
def _(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, num_experts, topk, int8=False):
    return torch.empty_like(X)


@torch.library.custom_op(_NS + "::moe_decode", mutates_args=())
def moe_decode(X: torch.Tensor, ids: torch.Tensor, RW: torch.Tensor, Bg: torch.Tensor, Sg: torch.Tensor,
               Bu: torch.Tensor, Su: torch.Tensor, Bd: torch.Tensor, Sd: torch.Tensor, num_experts: int,
               topk: int) -> torch.Tensor:
    """The MoE decode layer (few tokens): gate_up with the fused SwiGLU, then down_sum."""
    X2 = _rows(X)
    ids1 = ids.reshape(-1).contiguous()
    H = tl.moe_decode_gate_up(ids1, X2, Bg, Sg, Bu, Su, num_experts, topk)
    return tl.moe_decode_down_sum(ids1, H, RW.reshape(-1).contiguous(), Bd, Sd, num_experts, topk).reshape(X.shape)


@moe_decode.register_fake
def _(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, num_experts, topk):
    return torch.empty_like(X)
