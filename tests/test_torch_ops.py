"""The PyTorch custom operators (ternocl_b200/torch_ops.py): registration and fake (meta)
shapes without a GPU; on the GPU, each operator against the direct C-ABI calls it wraps
(the same kernels: bit for bit), torch.library.opcheck of the schema and fake kernel, and a
CUDA-graph capture and replay."""
import numpy as np
import pytest
import torch

import ternocl_b200.torch_ops  # noqa: F401  (registers torch.ops.ternocl)

OPS = ["int2_linear", "int1_linear", "bitcos_linear", "bitcos_hadamard_linear", "int8_linear", "hadamard",
       "moe_prefill", "moe_decode"]


def test_registered():
    for name in OPS:
        assert hasattr(torch.ops.ternocl, name), name


@pytest.mark.parametrize("out_f32", [False, True])
def test_fake_shapes(out_f32):
    A = torch.empty(3, 5, 4096, dtype=torch.bfloat16, device="meta")
    B = torch.empty(256, 6144, dtype=torch.int32, device="meta")
    S = torch.empty(32, 6144, dtype=torch.bfloat16, device="meta")
    for op in (torch.ops.ternocl.int2_linear, torch.ops.ternocl.int8_linear):
        C = op(A, B, S, 0, out_f32)
        assert C.shape == (3, 5, 6144)
        assert C.dtype == (torch.float32 if out_f32 else torch.bfloat16)
    C = torch.ops.ternocl.bitcos_linear(A, torch.empty(100, dtype=torch.int32, device="meta"), S, None, 1, 0, out_f32)
    assert C.shape == (3, 5, 6144)
    assert torch.ops.ternocl.hadamard(A, 1024).shape == A.shape
    X = torch.empty(9, 2048, dtype=torch.float16, device="meta")
    ids = torch.empty(9, 8, dtype=torch.int32, device="meta")
    RW = torch.empty(9, 8, dtype=torch.float16, device="meta")
    Bw = torch.empty(16, 128, 768, dtype=torch.int32, device="meta")
    Sw = torch.empty(16, 16, 768, dtype=torch.float16, device="meta")
    Bd = torch.empty(16, 48, 2048, dtype=torch.int32, device="meta")
    Sd = torch.empty(16, 6, 2048, dtype=torch.float16, device="meta")
    for op in (torch.ops.ternocl.moe_prefill, torch.ops.ternocl.moe_decode):
        assert op(X, ids, RW, Bw, Sw, Bw, Sw, Bd, Sd, 16, 8).shape == X.shape


# ---------------------------------------------------------------------------------- GPU
def _int2(rng, K, N, bf16):
    from ternocl_b200 import synth
    B = torch.from_numpy(synth.pack_int2(synth.ternary(rng, K, N)).view(np.int32)).cuda()
    S = torch.from_numpy(synth.scales(rng, K, N, bf16).view(np.int16)).cuda()
    return B, S.view(torch.bfloat16 if bf16 else torch.float16)


@pytest.mark.gpu
@pytest.mark.parametrize("bf16", [0, 1])
def test_linear_ops_match_direct_calls(cuda, tl, bf16):
    rng = np.random.default_rng(3)
    dt = torch.bfloat16 if bf16 else torch.float16
    K, N = 1024, 512
    B, S = _int2(rng, K, N, bf16)
    for lead in [(1,), (2, 3), (96,)]:
        A = torch.randn(*lead, K, device="cuda").to(dt)
        got = torch.ops.ternocl.int2_linear(A, B, S)
        want = tl.int2_upcvt(A.reshape(-1, K).contiguous(), B, S)
        assert got.shape == (*lead, N)
        assert torch.equal(got.reshape(-1, N), want)
        got8 = torch.ops.ternocl.int8_linear(A, B, S, 0, True)
        SA, Aq = tl.int8_quant_a(A.reshape(-1, K).contiguous())
        want8 = tl.int2_int8(A.reshape(-1, K).contiguous(), B, S, SA, Aq=Aq, qmode=0, out_f32=True)
        assert torch.equal(got8.reshape(-1, N), want8)
    x = torch.randn(4, 2048, device="cuda").to(dt)
    assert torch.equal(torch.ops.ternocl.hadamard(x, 1024), tl.hadamard_fwht(x, 1024))


@pytest.mark.gpu
def test_opcheck(cuda, tl):
    rng = np.random.default_rng(4)
    B, S = _int2(rng, 512, 256, 0)
    A = torch.randn(8, 512, device="cuda").half()
    torch.library.opcheck(torch.ops.ternocl.int2_linear.default, (A, B, S),
                          test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(torch.ops.ternocl.hadamard.default, (A, 256), test_utils=("test_schema", "test_faketensor"))


@pytest.mark.gpu
def test_cuda_graph_capture(cuda, tl):
    rng = np.random.default_rng(5)
    B, S = _int2(rng, 4096, 1024, 0)
    A = torch.randn(1, 4096, device="cuda").half()
    torch.ops.ternocl.int2_linear(A, B, S)  # first call outside the capture (library load, attributes)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        C = torch.ops.ternocl.int2_linear(A, B, S)
    A.copy_(torch.randn(1, 4096, device="cuda").half())
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(C, tl.int2_upcvt(A, B, S))


@pytest.mark.gpu
@pytest.mark.parametrize("int8", [False, True])
def test_moe_ops_match_direct_calls(cuda, tl, int8):
    rng = np.random.default_rng(6)
    T, topk, E, H, I = 40, 4, 8, 256, 384
    ids = torch.from_numpy(np.stack([rng.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)).cuda()
    RW = torch.rand(T, topk, device="cuda").half()
    X = torch.randn(T, H, device="cuda").half()
    ws = [_int2(rng, H, I, 0) for _ in range(E)], [_int2(rng, H, I, 0) for _ in range(E)], \
        [_int2(rng, I, H, 0) for _ in range(E)]
    (Bg, Sg), (Bu, Su), (Bd, Sd) = [(torch.stack([b for b, _ in w]), torch.stack([s for _, s in w])) for w in ws]
    got = torch.ops.ternocl.moe_prefill(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, E, topk, int8)
    ids1, RW1 = ids.reshape(-1), RW.reshape(-1)
    meta, perm, inv = tl.moe_route(ids1, E)
    if int8:
        SAt, Xq = tl.int8_quant_a(X)
        Xsq, SA1 = tl.moe_gather_q(Xq, SAt, perm, topk)
        up = tl.moe_gemm_i8(meta, Xsq, SA1, Bu, Su, E)
        Hh = tl.moe_gemm_i8(meta, Xsq, SA1, Bg, Sg, E, postop=1, other=up)
        SA2, Hq = tl.int8_quant_a(Hh)
        Y = tl.moe_gemm_i8(meta, Hq, SA2, Bd, Sd, E, out_f32=True)
    else:
        Xs = tl.moe_gather(X, perm, topk)
        up = tl.moe_gemm(meta, Xs, Bu, Su, E)
        Hh = tl.moe_gemm(meta, Xs, Bg, Sg, E, postop=1, other=up)
        Y = tl.moe_gemm(meta, Hh, Bd, Sd, E, out_f32=True)
    assert torch.equal(got, tl.moe_combine(Y, inv, RW1, T, topk))
    if not int8:
        got_d = torch.ops.ternocl.moe_decode(X[:2], ids[:2], RW[:2], Bg, Sg, Bu, Su, Bd, Sd, E, topk)
        Hd = tl.moe_decode_gate_up(ids[:2].reshape(-1), X[:2], Bg, Sg, Bu, Su, E, topk)
        want_d = tl.moe_decode_down_sum(ids[:2].reshape(-1), Hd, RW[:2].reshape(-1), Bd, Sd, E, topk)
        assert torch.equal(got_d, want_d)
    assert tl.device_error() == 0
