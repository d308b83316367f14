"""int1 ({+1,-1}) upconvert GEMV on the GPU vs the oracle (the reference's host gold,
int1_fp16_upcvt/main.cpp:95-114 + the epilogue), through the C ABI.  The device
weights are the select layout (to_sel_layout, main.cpp:80-92) of the per-column words
the gold reads."""
import os

import numpy as np
import pytest

from helpers import check_output, dev_dt, dev_u32, host_dt
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_int1.npz")

GEMV_SHAPES = [(1, 4096, 4096), (1, 4096, 6144), (3, 256, 48), (8, 1024, 512), (1, 128, 16),
               (2, 512, 272), (5, 2048, 1024), (13, 512, 256), (1, 14336, 512), (1, 128, 80)]


def case(seed, M, K, N, bf16, postop=0, out_f32=False):
    rng = np.random.default_rng(seed)
    Bpc = rng.integers(0, 1 << 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
    S = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    other, bias = synth.epilogue_operands(rng, postop, out_f32, M, N, bf16)
    return dict(A=A, Bpc=Bpc, sel=orc.int1_to_sel(Bpc, K, N), S=S, other=other, bias=bias)


def gold_out(c, M, K, N, bf16, postop, out_f32):
    acc = orc.int1_gold(c["A"], c["Bpc"], c["S"], M, K, N, bf16)
    return orc.epilogue(postop, out_f32, acc, c["other"], c["bias"], M, N, bf16)


def run(tl, c, bf16, postop, out_f32, ws=None):
    import torch
    A, B, S = dev_dt(c["A"], bf16), dev_u32(c["sel"]), dev_dt(c["S"], bf16)
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = None
    if c["bias"] is not None:
        bias = torch.from_numpy(c["bias"]).cuda() if out_f32 else dev_dt(c["bias"], bf16)
    out = tl.int1_upcvt(A, B, S, postop=postop, out_f32=out_f32, other=other, bias=bias, workspace=ws)
    return host_dt(out)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", GEMV_SHAPES)
def test_gemv_parity(cuda, tl, M, K, N, bf16):
    c = case(400 + M + K + N, M, K, N, bf16)
    gold = gold_out(c, M, K, N, bf16, 0, False)
    for ws in (None, tl.Workspace()):
        check_output(run(tl, c, bf16, 0, False, ws), gold, bf16, False,
                     "int1 M=%d K=%d N=%d bf16=%d" % (M, K, N, bf16))


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemv_epilogues(cuda, tl, bf16, postop, out_f32):
    M, K, N = 3, 2048, 512
    c = case(60 + postop, M, K, N, bf16, postop, out_f32)
    gold = gold_out(c, M, K, N, bf16, postop, out_f32)
    check_output(run(tl, c, bf16, postop, out_f32), gold, bf16, out_f32,
                 "postop=%d out_f32=%d" % (postop, out_f32))


def test_gemv_golden(cuda, tl):
    d = np.load(GOLDEN)
    for dt, bf16 in (("fp16", 0), ("bf16", 1)):
        k = "int1_" + dt
        A = d[k + "_A"]
        M, K = A.shape
        N = d[k + "_sel"].shape[1]
        c = dict(A=A, sel=d[k + "_sel"], S=d[k + "_S"], other=None, bias=None)
        gold = orc.epilogue(0, False, d[k + "_acc"], None, None, M, N, bf16)
        check_output(run(tl, c, bf16, 0, False), gold, bf16, False, dt)


def test_gemv_deterministic(cuda, tl):
    M, K, N = 4, 4096, 2048
    c = case(9, M, K, N, 1)
    ws = tl.Workspace()
    outs = [run(tl, c, 1, 0, False, w) for w in (None, ws, None, ws)]
    assert np.array_equal(outs[0], outs[2]) and np.array_equal(outs[1], outs[3])


def test_decode_bit_exact(cuda, tl):
    # A = identity: C[k, n] = sgn(k, n) * S exactly, i.e. the decoded weights of the
    # sel layout, compared with the per-column bit order the gold reads (main.cpp:76)
    K, N = 512, 96
    rng = np.random.default_rng(8)
    Bpc = rng.integers(0, 1 << 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
    c = dict(A=synth.to_dt(np.eye(K), 0), sel=orc.int1_to_sel(Bpc, K, N), S=synth.to_dt(np.ones((K // 128, N)), 0),
             other=None, bias=None)
    out = synth.from_dt(run(tl, c, 0, 0, False), 0)
    k = np.arange(K)
    pos = np.array([synth.int1_bit_pos(x) for x in k], np.uint32)[:, None]
    neg = (Bpc[k // 32][:, :] >> pos) & 1
    assert np.array_equal(out, np.where(neg == 1, -1.0, 1.0).astype(np.float32))
