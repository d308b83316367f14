"""s8 x s2 path on the GPU vs the oracle, through the C ABI:
quant_a (int2_int8_dpas.cl:103-123; host gold compute_scale_a, main.cpp:82-92),
the int32 group dots and the GEMV (compute_gold, main.cpp:94-121, + the epilogue).

SA, Aq and the int32 dots are integer/bit work: compared bit for bit.  The GEMV's
fp32 accumulation runs in a different order than the gold's, so its outputs use the
DT / fp32 tolerances of helpers.py."""
import os

import numpy as np
import pytest

from helpers import F32_FLOOR, F32_REL_TOL, check_output, dev_any, dev_dt, dev_u32, host_dt, rel_err
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_int8.npz")

GEMV_SHAPES = [(1, 4096, 4096), (1, 4096, 6144), (3, 256, 48), (8, 1024, 512), (1, 128, 16),
               (2, 512, 272), (5, 2048, 1024), (13, 512, 256), (1, 14336, 512), (33, 1024, 128)]


def case(seed, M, K, N, bf16, postop=0, out_f32=False, all_codes=True, offgrid=None):
    rng = np.random.default_rng(seed)
    if all_codes:  # every 2-bit code, -2 included (code_to_value, main.cpp:77)
        B = rng.integers(0, 1 << 32, size=(K // 16, N), dtype=np.uint64).astype(np.uint32)
    else:
        B = synth.pack_int2(synth.ternary(rng, K, N))
    SB = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    if offgrid is not None:  # main.cpp:261-275: A placed `offgrid` LSB off the int8 grid
        A, SA = orc.int8_fake_quant(A, M, K, offgrid, bf16)
    else:
        SA = orc.int8_scale_a(A, M, K, bf16)
    other, bias = synth.epilogue_operands(rng, postop, out_f32, M, N, bf16)
    return dict(A=A, B=B, SB=SB, SA=SA, other=other, bias=bias)


def gold_out(c, M, K, N, bf16, postop, out_f32):
    acc = orc.int8_gold(c["A"], c["B"], c["SA"], c["SB"], M, K, N, bf16)
    return orc.epilogue(postop, out_f32, acc, c["other"], c["bias"], M, N, bf16)


def run_gemv(tl, c, bf16, postop, out_f32, qmode):
    import torch
    A = dev_dt(c["A"], bf16)
    B, SB = dev_u32(c["B"]), dev_dt(c["SB"], bf16)
    SA, Aq = tl.int8_quant_a(A, write_q=(qmode == 0))
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = None
    if c["bias"] is not None:
        bias = torch.from_numpy(c["bias"]).cuda() if out_f32 else dev_dt(c["bias"], bf16)
    out = tl.int2_int8(A, B, SB, SA, Aq=Aq, qmode=qmode, postop=postop, out_f32=out_f32,
                       other=other, bias=bias)
    return host_dt(out)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K", [(1, 128), (3, 256), (8, 4096), (33, 1024), (64, 512)])
def test_quant_a_bit_exact(cuda, tl, M, K, bf16):
    rng = np.random.default_rng(M * 7 + K + bf16)
    A = synth.activations(rng, M, K, bf16)
    if bf16:
        # an all-zero group: SA = bf16(127 / FLT_EPSILON).  (In fp16 that quotient
        # overflows to inf and the gold's lrintf(0 * inf) is undefined behaviour, so
        # the fp16 cases keep every group non-zero.)
        A[0, :128] = 0
    SA, Aq = tl.int8_quant_a(dev_dt(A, bf16))
    SA_h, Aq_h = host_dt(SA), Aq.cpu().numpy()
    SA_o = orc.int8_scale_a(A, M, K, bf16)
    assert np.array_equal(SA_h[:, :M], SA_o[:, :M])
    assert np.array_equal(Aq_h, orc.int8_quant(A, SA_o, M, K, bf16))


def test_quant_a_golden(cuda, tl):
    # SA from the reference's own compute_scale_a (tests/golden/make_golden.py)
    d = np.load(GOLDEN)
    for dt, bf16 in (("fp16", 0), ("bf16", 1)):
        A = d["int8_%s_A" % dt]
        M, K = A.shape
        SA, _ = tl.int8_quant_a(dev_dt(A, bf16), write_q=False)
        assert np.array_equal(host_dt(SA)[:, :M], d["int8_%s_SA" % dt][:, :M]), dt


@pytest.mark.parametrize("M,K,N", [(1, 1024, 64), (5, 512, 48), (9, 256, 128)])
def test_group_dots_bit_exact(cuda, tl, M, K, N):
    c = case(11 + M, M, K, N, 0)
    Q = orc.int8_quant(c["A"], c["SA"], M, K, 0)
    D = tl.int2_int8_group_dots(dev_any(Q), dev_u32(c["B"])).cpu().numpy()
    assert np.array_equal(D, orc.int8_group_dots(Q, c["B"], M, K, N))


@pytest.mark.parametrize("qmode", [0, 1])
@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", GEMV_SHAPES)
def test_gemv_parity(cuda, tl, M, K, N, bf16, qmode):
    c = case(300 + M + K + N, M, K, N, bf16)
    gold = gold_out(c, M, K, N, bf16, 0, False)
    out = run_gemv(tl, c, bf16, 0, False, qmode)
    check_output(out, gold, bf16, False, "s8xs2 qmode=%d M=%d K=%d N=%d bf16=%d" % (qmode, M, K, N, bf16))


@pytest.mark.parametrize("qmode", [0, 1])
@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemv_epilogues(cuda, tl, bf16, postop, out_f32, qmode):
    M, K, N = 3, 2048, 512
    c = case(50 + postop, M, K, N, bf16, postop, out_f32)
    gold = gold_out(c, M, K, N, bf16, postop, out_f32)
    out = run_gemv(tl, c, bf16, postop, out_f32, qmode)
    check_output(out, gold, bf16, out_f32, "postop=%d out_f32=%d" % (postop, out_f32))


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("offgrid", [0.0, 0.6])
def test_gemv_fake_quant(cuda, tl, bf16, offgrid):
    # the reference driver's validation input (main.cpp:261-275, --offgrid)
    M, K, N = 4, 4096, 1024
    c = case(77, M, K, N, bf16, all_codes=False, offgrid=offgrid)
    gold = gold_out(c, M, K, N, bf16, 0, False)
    for qmode in (0, 1):
        check_output(run_gemv(tl, c, bf16, 0, False, qmode), gold, bf16, False, "qmode=%d" % qmode)


def test_gemv_golden(cuda, tl):
    d = np.load(GOLDEN)
    for dt, bf16 in (("fp16", 0), ("bf16", 1)):
        k = "int8_" + dt
        A = d[k + "_A"]
        M, K = A.shape
        N = d[k + "_B"].shape[1]
        c = dict(A=A, B=d[k + "_B"], SB=d[k + "_SB"], SA=d[k + "_SA"], other=None, bias=None)
        gold = orc.epilogue(0, False, d[k + "_acc"], None, None, M, N, bf16)
        for qmode in (0, 1):
            check_output(run_gemv(tl, c, bf16, 0, False, qmode), gold, bf16, False, dt)


def test_gemv_deterministic_and_qmodes_agree(cuda, tl):
    # qmode 0 and 1 quantise identically, so both give the same bits; reruns too
    M, K, N = 4, 4096, 2048
    c = case(5, M, K, N, 0)
    outs = [run_gemv(tl, c, 0, 0, False, q) for q in (0, 1, 0, 1)]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_argument_errors(cuda, tl):
    import torch
    L = tl.lib()
    A = torch.zeros(1, 256, dtype=torch.float16, device="cuda")
    B = torch.zeros(16, 48, dtype=torch.int32, device="cuda")
    SB = torch.zeros(2, 48, dtype=torch.float16, device="cuda")
    SA = torch.zeros(2, 32, dtype=torch.float16, device="cuda")
    C = torch.zeros(1, 48, dtype=torch.float16, device="cuda")
    p = lambda t: t.data_ptr()
    # qmode must be 0 or 1; qmode 0 needs Aq
    assert L.ternocl_int2_int8(p(A), None, p(SA), p(B), p(SB), p(C), None, None, 1, 48, 256, 0, 0, 0, 2, 0,
                               None) == 2
    assert L.ternocl_int2_int8(p(A), None, p(SA), p(B), p(SB), p(C), None, None, 1, 48, 256, 0, 0, 0, 0, 0,
                               None) == 2
    # N % 16 and K % 128 (main.cpp shape checks)
    assert L.ternocl_int2_int8(p(A), None, p(SA), p(B), p(SB), p(C), None, None, 1, 40, 256, 0, 0, 0, 1, 0,
                               None) == 1
    assert L.ternocl_int8_quant_a(p(A), p(SA), None, 1, 200, 0, None) == 1


# ---- the tcgen05 kind::i8 prefill GEMM (qmode 0: quant_a first, as the reference's
# upfront-quantisation mode; int2_int8_dpas.cl:283-385)
GEMM_SHAPES = [(64, 128, 128), (100, 256, 272), (128, 1024, 512), (256, 512, 1024), (77, 4096, 256),
               (300, 1024, 400), (130, 128, 48)]


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", GEMM_SHAPES)
def test_gemm_parity(cuda, tl, M, K, N, bf16):
    c = case(900 + M + K + N, M, K, N, bf16)
    gold = gold_out(c, M, K, N, bf16, 0, False)
    A = dev_dt(c["A"], bf16)
    SA, Aq = tl.int8_quant_a(A)
    out = host_dt(tl.int2_int8(A, dev_u32(c["B"]), dev_dt(c["SB"], bf16), SA, Aq=Aq, qmode=0, algo=tl.ALGO_GEMM))
    check_output(out, gold, bf16, False, "s8xs2 gemm M=%d K=%d N=%d bf16=%d" % (M, K, N, bf16))
    assert tl.device_error() == 0


@pytest.mark.parametrize("postop,out_f32", [(0, True), (1, False), (2, False), (3, True), (4, False)])
def test_gemm_epilogues(cuda, tl, postop, out_f32):
    M, K, N = 192, 512, 512
    c = case(40 + postop, M, K, N, 0, postop, out_f32)
    gold = gold_out(c, M, K, N, 0, postop, out_f32)
    out = run_gemv(tl, c, 0, postop, out_f32, 0)  # AUTO at M >= 64 with qmode 0 -> the GEMM
    check_output(out, gold, 0, out_f32, "postop=%d out_f32=%d" % (postop, out_f32))


def test_gemm_matches_gemv_kernel(cuda, tl):
    # the same int32 group dots on both paths: outputs agree within fp32 rounding
    M, K, N = 96, 2048, 384
    c = case(8, M, K, N, 1)
    A = dev_dt(c["A"], 1)
    SA, Aq = tl.int8_quant_a(A)
    args = (A, dev_u32(c["B"]), dev_dt(c["SB"], 1), SA)
    g = host_dt(tl.int2_int8(*args, Aq=Aq, qmode=0, algo=tl.ALGO_GEMM, out_f32=True))
    v = host_dt(tl.int2_int8(*args, Aq=Aq, qmode=0, algo=tl.ALGO_GEMV, out_f32=True))
    # the int32 dots are equal; only the fp32 order of the group sums differs
    assert rel_err(g, v, F32_FLOOR) <= F32_REL_TOL


# ---- qmode 1 on the tensor-core GEMM (the reference driver's default scheme: scale
# pre-kernel, quantise in the GEMM; int2_via_int2_x_int8_dpas/main.cpp:58, 316): one pass
# quantises A with the caller's SA into pooled scratch, then the same int8 GEMM, so the
# output is qmode 0's bit for bit
@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", [(64, 128, 128), (100, 256, 272), (300, 1024, 400)])
def test_gemm_qmode1_equals_qmode0(cuda, tl, M, K, N, bf16):
    import torch
    c = case(1300 + M + K + N, M, K, N, bf16)
    A = dev_dt(c["A"], bf16)
    B, SB = dev_u32(c["B"]), dev_dt(c["SB"], bf16)
    SA, Aq = tl.int8_quant_a(A)
    SA1, none = tl.int8_quant_a(A, write_q=False)  # the scale pre-kernel alone
    assert none is None and torch.equal(SA1, SA)
    g0 = host_dt(tl.int2_int8(A, B, SB, SA, Aq=Aq, qmode=0, algo=tl.ALGO_GEMM))
    dummy = torch.zeros(64, dtype=torch.int8, device="cuda")  # the 64-byte Aq of qmode 1
    for algo in (tl.ALGO_GEMM, tl.ALGO_AUTO):
        g1 = host_dt(tl.int2_int8(A, B, SB, SA1, Aq=dummy, qmode=1, algo=algo))
        assert np.array_equal(g1.view(np.uint16), g0.view(np.uint16)), "qmode 1 algo %d" % algo
    assert torch.count_nonzero(dummy).item() == 0
    gold = gold_out(c, M, K, N, bf16, 0, False)
    check_output(g0, gold, bf16, False, "s8xs2 gemm qmode=1 M=%d K=%d N=%d" % (M, K, N))
    assert tl.device_error() == 0


def test_gemm_qmode1_in_graph(cuda, tl):
    # the scratch allocation is stream-ordered, so the call captures into a CUDA graph
    import torch
    M, K, N = 128, 512, 256
    c = case(77, M, K, N, 0)
    A = dev_dt(c["A"], 0)
    B, SB = dev_u32(c["B"]), dev_dt(c["SB"], 0)
    SA, _ = tl.int8_quant_a(A, write_q=False)
    ref = host_dt(tl.int2_int8(A, B, SB, SA, qmode=1, algo=tl.ALGO_GEMM))
    out = torch.empty(M, N, dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            tl.int2_int8(A, B, SB, SA, qmode=1, algo=tl.ALGO_GEMM, out=out)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(host_dt(out).view(np.uint16), ref.view(np.uint16))
    del g
