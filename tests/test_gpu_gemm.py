"""Prefill GEMM (tcgen05, TERNOCL_ALGO_GEMM and AUTO at M >= 64) vs the oracle:
int2 (int2_fp16_upcvt/main.cpp:79-98) and int1 (int1_fp16_upcvt/main.cpp:95-114) host
gold + the epilogue, through the C ABI.  Ragged M and partial N tiles included."""
import numpy as np
import pytest

from helpers import check_output, dev_dt, dev_u32, host_dt, int2_case, int2_gold_out
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu

SHAPES = [(64, 128, 256), (100, 256, 272), (128, 1024, 512), (256, 512, 1024), (77, 4096, 256),
          (512, 1024, 768), (130, 128, 48), (1, 256, 512)]


def run_int2(tl, c, bf16, postop, out_f32, algo):
    import torch
    A, B, S = dev_dt(c["A"], bf16), dev_u32(c["B"]), dev_dt(c["S"], bf16)
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = None
    if c["bias"] is not None:
        bias = torch.from_numpy(c["bias"]).cuda() if out_f32 else dev_dt(c["bias"], bf16)
    return host_dt(tl.int2_upcvt(A, B, S, postop=postop, out_f32=out_f32, other=other, bias=bias, algo=algo))


@pytest.fixture(params=[0, 128, 256, "persistent"], ids=["tile_auto", "tile128", "tile256", "persistent"])
def tile_m(request, tl):
    """Every prefill test runs with the per-shape tile choice, with each tile forced, and
    with the persistent kernel (one CTA per SM over all tiles)."""
    if request.param == "persistent":
        old = tl.set_option(tl.OPT_GEMM_PERSISTENT, 2)
        yield request.param
        tl.set_option(tl.OPT_GEMM_PERSISTENT, old)
        return
    old = tl.set_option(tl.OPT_GEMM_TILE_M, request.param)
    yield request.param
    tl.set_option(tl.OPT_GEMM_TILE_M, old)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_int2_gemm_parity(cuda, tl, tile_m, M, K, N, bf16):
    c = int2_case(600 + M + K + N, M, K, N, bf16)
    gold = int2_gold_out(c, M, K, N, bf16, 0, False)
    check_output(run_int2(tl, c, bf16, 0, False, tl.ALGO_GEMM), gold, bf16, False,
                 "int2 gemm M=%d K=%d N=%d bf16=%d" % (M, K, N, bf16))
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("out_f32", [False, True])
def test_int2_gemm_epilogues(cuda, tl, tile_m, bf16, postop, out_f32):
    M, K, N = 192, 512, 512
    c = int2_case(80 + postop, M, K, N, bf16, postop, out_f32)
    gold = int2_gold_out(c, M, K, N, bf16, postop, out_f32)
    check_output(run_int2(tl, c, bf16, postop, out_f32, tl.ALGO_AUTO), gold, bf16, out_f32,
                 "postop=%d out_f32=%d" % (postop, out_f32))


def test_int2_gemm_decode_bit_exact(cuda, tl, tile_m):
    # A = identity: C = the upconverted weights code * S exactly, every 2-bit code
    K, N = 256, 512
    rng = np.random.default_rng(4)
    B = rng.integers(0, 1 << 32, size=(K // 16, N), dtype=np.uint64).astype(np.uint32)
    S = synth.scales(rng, K, N, 0)
    c = dict(A=synth.to_dt(np.eye(K), 0), B=B, S=S, other=None, bias=None)
    out = synth.from_dt(run_int2(tl, c, 0, 0, False, tl.ALGO_GEMM), 0)
    k = np.arange(K)[:, None]
    codes = (B[k // 16, np.arange(N)[None, :]] >> (2 * (k % 16)).astype(np.uint32)) & 3
    want = np.array([0, 1, -2, -1], np.float32)[codes] * synth.from_dt(S, 0)[k // 128, np.arange(N)[None, :]]
    assert np.array_equal(out, want)


def test_int2_gemm_deterministic(cuda, tl, tile_m):
    M, K, N = 256, 1024, 768
    c = int2_case(11, M, K, N, 1)
    outs = [run_int2(tl, c, 1, 0, False, tl.ALGO_GEMM) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


def int1_case(seed, M, K, N, bf16, postop=0, out_f32=False):
    rng = np.random.default_rng(seed)
    Bpc = rng.integers(0, 1 << 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
    S = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    other, bias = synth.epilogue_operands(rng, postop, out_f32, M, N, bf16)
    return dict(A=A, Bpc=Bpc, sel=orc.int1_to_sel(Bpc, K, N), S=S, other=other, bias=bias)


def run_int1(tl, c, bf16, postop, out_f32, algo):
    import torch
    A, B, S = dev_dt(c["A"], bf16), dev_u32(c["sel"]), dev_dt(c["S"], bf16)
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = None
    if c["bias"] is not None:
        bias = torch.from_numpy(c["bias"]).cuda() if out_f32 else dev_dt(c["bias"], bf16)
    return host_dt(tl.int1_upcvt(A, B, S, postop=postop, out_f32=out_f32, other=other, bias=bias, algo=algo))


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_int1_gemm_parity(cuda, tl, tile_m, M, K, N, bf16):
    c = int1_case(700 + M + K + N, M, K, N, bf16)
    acc = orc.int1_gold(c["A"], c["Bpc"], c["S"], M, K, N, bf16)
    gold = orc.epilogue(0, False, acc, None, None, M, N, bf16)
    check_output(run_int1(tl, c, bf16, 0, False, tl.ALGO_GEMM), gold, bf16, False,
                 "int1 gemm M=%d K=%d N=%d bf16=%d" % (M, K, N, bf16))


@pytest.mark.parametrize("postop,out_f32", [(1, False), (3, True), (4, False)])
def test_int1_gemm_epilogues(cuda, tl, tile_m, postop, out_f32):
    M, K, N = 128, 512, 256
    c = int1_case(90 + postop, M, K, N, 0, postop, out_f32)
    acc = orc.int1_gold(c["A"], c["Bpc"], c["S"], M, K, N, 0)
    gold = orc.epilogue(postop, out_f32, acc, c["other"], c["bias"], M, N, 0)
    check_output(run_int1(tl, c, 0, postop, out_f32, tl.ALGO_AUTO), gold, 0, out_f32, "postop=%d" % postop)


def test_int1_gemm_decode_bit_exact(cuda, tl, tile_m):
    K, N = 256, 512
    rng = np.random.default_rng(5)
    Bpc = rng.integers(0, 1 << 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
    S = synth.scales(rng, K, N, 0)
    c = dict(A=synth.to_dt(np.eye(K), 0), sel=orc.int1_to_sel(Bpc, K, N), S=S, other=None, bias=None)
    out = synth.from_dt(run_int1(tl, c, 0, 0, False, tl.ALGO_GEMM), 0)
    k = np.arange(K)
    pos = np.array([synth.int1_bit_pos(x) for x in k], np.uint32)[:, None]
    neg = (Bpc[k // 32] >> pos) & 1
    want = np.where(neg == 1, -1.0, 1.0).astype(np.float32) * synth.from_dt(S, 0)[k // 128]
    assert np.array_equal(out, want)
