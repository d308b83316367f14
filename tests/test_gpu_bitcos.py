"""BITCOS GEMV and M-tiled GEMM on the GPU vs the oracle (the reference's host gold,
bitcos_fp16_upcvt/main.cpp:64-86 with bitcos_decode_col, common/bitcos.hpp:97-106,
+ the epilogue), through the C ABI.  Buffers come from the library's host packer,
which reproduces bitcos_random (common/bitcos.hpp:31-78) bit for bit."""
import os

import numpy as np
import pytest

from helpers import check_output, dev_dt, host_dt
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_bitcos.npz")


def dev_words(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, np.uint32).view(np.int32)).cuda()


def case(tl, seed, M, K, N, z, bf16, postop=0, out_f32=False):
    rng = np.random.default_rng(seed)
    buf = tl.bitcos_random(K, N, z, seed)
    S = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    other, bias = synth.epilogue_operands(rng, postop, out_f32, M, N, bf16)
    return dict(A=A, buf=buf, S=S, other=other, bias=bias)


def gold_out(c, M, K, N, bf16, postop, out_f32):
    acc = orc.bitcos_gold(c["A"], c["buf"], c["S"], M, K, N, bf16)
    return orc.epilogue(postop, out_f32, acc, c["other"], c["bias"], M, N, bf16)


@pytest.fixture(params=[0, 1], ids=["strip", "ksliced"])
def gemv_impl(request, tl):
    """Both decode GEMVs: the persistent whole-K strip kernel (default at M <= 8) and
    the K-sliced kernel of the reference's LS split (TERNOCL_OPT_BITCOS_GEMV = 1)."""
    old = tl.set_option(tl.OPT_BITCOS_GEMV, request.param)
    yield request.param
    tl.set_option(tl.OPT_BITCOS_GEMV, old)


def run(tl, c, K, N, bf16, ls, postop=0, out_f32=False, algo=0):
    import torch
    A, B, S = dev_dt(c["A"], bf16), dev_words(c["buf"]), dev_dt(c["S"], bf16)
    SR = dev_words(tl.bitcos_slice_ranks(c["buf"], K, N, ls)) if ls > 1 else None
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = None
    if c["bias"] is not None:
        bias = torch.from_numpy(c["bias"]).cuda() if out_f32 else dev_dt(c["bias"], bf16)
    out = tl.bitcos_upcvt(A, B, S, SR=SR, ls=ls, postop=postop, out_f32=out_f32, other=other, bias=bias, algo=algo)
    return host_dt(out)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("z", [0.2, 0.35, 0.5])
@pytest.mark.parametrize("M,K,N,ls", [(1, 5376, 512, 4), (1, 5376, 512, 1), (8, 1024, 256, 2), (3, 256, 48, 4),
                                      (1, 4096, 4096, 4), (13, 512, 128, 1), (2, 5376, 272, 7)])
def test_gemv_parity(cuda, tl, gemv_impl, M, K, N, ls, z, bf16):
    c = case(tl, 500 + M + K + N + int(100 * z), M, K, N, z, bf16)
    gold = gold_out(c, M, K, N, bf16, 0, False)
    check_output(run(tl, c, K, N, bf16, ls), gold, bf16, False,
                 "bitcos M=%d K=%d N=%d ls=%d z=%.2f bf16=%d" % (M, K, N, ls, z, bf16))


@pytest.mark.parametrize("z", [0.0, 0.95, 1.0])
def test_gemv_density_extremes(cuda, tl, gemv_impl, z):
    # all non-zero, almost all zero, and an empty sign plane
    M, K, N = 2, 2048, 384
    c = case(tl, 41, M, K, N, z, 0)
    gold = gold_out(c, M, K, N, 0, 0, False)
    if z == 1.0:
        assert not np.any(gold)
    for ls in (1, 4):
        check_output(run(tl, c, K, N, 0, ls), gold, 0, False, "z=%.2f ls=%d" % (z, ls))


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemv_epilogues(cuda, tl, gemv_impl, bf16, postop, out_f32):
    M, K, N = 3, 2048, 512
    c = case(tl, 70 + postop, M, K, N, 0.35, bf16, postop, out_f32)
    gold = gold_out(c, M, K, N, bf16, postop, out_f32)
    check_output(run(tl, c, K, N, bf16, 2, postop, out_f32), gold, bf16, out_f32,
                 "postop=%d out_f32=%d" % (postop, out_f32))


def test_decode_bit_exact(cuda, tl, gemv_impl):
    # A = identity: C[k, n] = code(k, n) * S[k/128, n] exactly (one non-zero term),
    # so the output is the decoded weight matrix, compared with bitcos_decode_col
    K, N = 512, 96
    buf = tl.bitcos_random(K, N, 0.35, 3)
    S = synth.to_dt(np.ones((K // 128, N)), 0)
    eye = synth.to_dt(np.eye(K), 0)
    c = dict(A=eye, buf=buf, S=S, other=None, bias=None)
    for ls in (1, 2, 4):
        out = synth.from_dt(run(tl, c, K, N, 0, ls), 0)
        assert np.array_equal(out, orc.bitcos_decode(buf, K, N).T.astype(np.float32)), ls


def test_gemv_golden(cuda, tl, gemv_impl):
    d = np.load(GOLDEN)
    for zk in ("z35", "z05", "z95"):
        buf = d["bitcos_%s_buf" % zk]
        for dt, bf16 in (("fp16", 0), ("bf16", 1)):
            A, S = d["bitcos_%s_%s_A" % (zk, dt)], d["bitcos_%s_%s_S" % (zk, dt)]
            M, K = A.shape
            N = S.shape[1]
            gold = orc.epilogue(0, False, d["bitcos_%s_%s_acc" % (zk, dt)], None, None, M, N, bf16)
            c = dict(A=A, buf=buf, S=S, other=None, bias=None)
            for ls in (1, 2, 4):
                check_output(run(tl, c, K, N, bf16, ls), gold, bf16, False, "%s %s ls=%d" % (zk, dt, ls))


@pytest.mark.parametrize("M,N", [(1, 21504), (8, 5136)])
def test_gemv_strip_kernel_many_strips(cuda, tl, M, N):
    # more strips than SMs (each CTA walks several, through its staged ring), a last
    # strip of 16 columns (N % 32 == 16), and the last column's run (no offset follows
    # it); deterministic over reruns
    K = 5376
    c = case(tl, 900 + M, M, K, N, 0.35, 0)
    gold = gold_out(c, M, K, N, 0, 0, False)
    first = run(tl, c, K, N, 0, 4)
    check_output(first, gold, 0, False, "strip kernel M=%d N=%d" % (M, N))
    assert np.array_equal(run(tl, c, K, N, 0, 4).view(np.uint16), first.view(np.uint16))
    assert tl.device_error() == 0


def test_shape_errors(cuda, tl):
    import torch
    L = tl.lib()
    A = torch.zeros(1, 320, dtype=torch.float16, device="cuda")
    B = torch.zeros(4096, dtype=torch.int32, device="cuda")
    S = torch.zeros(2, 48, dtype=torch.float16, device="cuda")
    C = torch.zeros(1, 48, dtype=torch.float16, device="cuda")
    p = lambda t: t.data_ptr()
    # K % (64 ls) (bitcos_fp16_upcvt/main.cpp:129): 256 with ls = 3
    assert L.ternocl_bitcos_upcvt(p(A), p(B), p(S), p(B), 3, p(C), None, None, 1, 48, 256, 0, 0, 0, 0, None) == 1
    # ls > 1 needs slice ranks
    assert L.ternocl_bitcos_upcvt(p(A), p(B), p(S), None, 2, p(C), None, None, 1, 48, 256, 0, 0, 0, 0, None) == 2


# ---- M-tiled tcgen05 GEMM (bitcos_fp16_upcvt_gemm_mt, bitcos_fp16_upcvt.cl:279-368) ----
GEMM = 2


@pytest.fixture(params=[128, 256], ids=["tile128", "tile256"])
def tile_m(request, tl):
    old = tl.set_option(tl.OPT_GEMM_TILE_M, request.param)
    yield request.param
    tl.set_option(tl.OPT_GEMM_TILE_M, old)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("z", [0.2, 0.5])
@pytest.mark.parametrize("M,K,N", [(512, 5376, 512), (64, 1024, 256), (200, 2048, 272), (1, 256, 48),
                                   (300, 5376, 784), (129, 128, 16)])
def test_gemm_parity(cuda, tl, tile_m, M, K, N, z, bf16):
    c = case(tl, 900 + M + K + N + int(100 * z), M, K, N, z, bf16)
    gold = gold_out(c, M, K, N, bf16, 0, False)
    check_output(run(tl, c, K, N, bf16, 1, algo=GEMM), gold, bf16, False,
                 "bitcos gemm M=%d K=%d N=%d z=%.2f bf16=%d" % (M, K, N, z, bf16))


@pytest.mark.parametrize("z", [0.0, 0.95, 1.0])
def test_gemm_density_extremes(cuda, tl, z):
    M, K, N = 96, 2048, 384
    c = case(tl, 43, M, K, N, z, 0)
    gold = gold_out(c, M, K, N, 0, 0, False)
    check_output(run(tl, c, K, N, 0, 1, algo=GEMM), gold, 0, False, "gemm z=%.2f" % z)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemm_epilogues(cuda, tl, bf16, postop, out_f32):
    M, K, N = 160, 1024, 528
    c = case(tl, 80 + postop, M, K, N, 0.35, bf16, postop, out_f32)
    gold = gold_out(c, M, K, N, bf16, postop, out_f32)
    check_output(run(tl, c, K, N, bf16, 1, postop, out_f32, algo=GEMM), gold, bf16, out_f32,
                 "gemm postop=%d out_f32=%d" % (postop, out_f32))


def test_gemm_decode_bit_exact(cuda, tl, tile_m):
    # A = identity (M = K = 512, so AUTO picks the GEMM): C = the decoded weights
    K, N = 512, 96
    buf = tl.bitcos_random(K, N, 0.35, 5)
    S = synth.to_dt(np.ones((K // 128, N)), 0)
    eye = synth.to_dt(np.eye(K), 0)
    c = dict(A=eye, buf=buf, S=S, other=None, bias=None)
    out = synth.from_dt(run(tl, c, K, N, 0, 1), 0)
    assert np.array_equal(out, orc.bitcos_decode(buf, K, N).T.astype(np.float32))
    assert tl.device_error() == 0


def test_gemm_golden(cuda, tl):
    d = np.load(GOLDEN)
    for zk in ("z35", "z05", "z95"):
        buf = d["bitcos_%s_buf" % zk]
        for dt, bf16 in (("fp16", 0), ("bf16", 1)):
            A, S = d["bitcos_%s_%s_A" % (zk, dt)], d["bitcos_%s_%s_S" % (zk, dt)]
            M, K = A.shape
            N = S.shape[1]
            gold = orc.epilogue(0, False, d["bitcos_%s_%s_acc" % (zk, dt)], None, None, M, N, bf16)
            c = dict(A=A, buf=buf, S=S, other=None, bias=None)
            check_output(run(tl, c, K, N, bf16, 1, algo=GEMM), gold, bf16, False, "gemm %s %s" % (zk, dt))


def test_gemm_matches_gemv(cuda, tl):
    # same inputs through both kernels: identical up to fp32 summation order
    M, K, N = 8, 5376, 1024
    c = case(tl, 77, M, K, N, 0.35, 1)
    a = synth.from_dt(run(tl, c, K, N, 1, 1, algo=GEMM), 1)
    b = synth.from_dt(run(tl, c, K, N, 1, 4, algo=1), 1)
    gold = synth.from_dt(gold_out(c, M, K, N, 1, 0, False), 1)
    assert np.max(np.abs(a - b)) <= np.max(np.abs(gold)) * 2e-2
