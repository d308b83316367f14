"""Parity at the benchmark's own configurations, at full size, against the oracle (the
reference's host gold, compiled from its sources or restated and pinned to it).

* C2, the Llama-3-8B decode sweep: int2 and int1 upconvert GEMVs on all four shapes at
  M = 1, 4, 8, fp16 and bf16 (int2_fp16_upcvt/main.cpp:79-98, int1 main.cpp:95-114), and
  every epilogue on the largest shape (common/epilogue.hpp:50-67).
* C3, the s8 x s2 prefill at 27B-like shapes, M = 1, 512, 2048 (bf16): quant_a's SA and
  the int8 codes bit for bit, the outputs on 16 sampled rows (each output row depends on
  its own activation row only, int2_via_int2_x_int8_dpas/main.cpp:94-121), the int32
  group dots bit for bit on a column slice, and qmode 1 (quantise from SA in the GEMM,
  the driver's default) equal to qmode 0 bit for bit.
* C4, BITCOS with the Hadamard pre-transform, K = 5376, N = 21504, z = 0.2/0.35/0.5,
  M = 1, 8, 512 (HB = 256: 1024 does not divide 5376): the transform bit for bit and the
  outputs against bitcos_fp16_upcvt/main.cpp:64-86 (sampled rows at M = 512).
* C5, the MoE prefill layer at T = 4096, E = 128, top-8, H = 2048, I = 768 against the
  double-precision token reference of int2_moe/prefill.cpp:291-310 on 12 tokens, by the
  driver's own layer rule (max error over max |ref|, prefill.cpp:311-318).
"""
import numpy as np
import pytest

from helpers import MOE_TOL, check_output, dev_any, dev_dt, dev_u32, host_dt, moe_layer_err
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu

C2_SHAPES = [(4096, 6144), (4096, 4096), (4096, 28672), (14336, 4096)]
C3_SHAPES = [(5376, 21504), (21504, 5376), (5376, 5376)]

_cache = {}


def packed_int2(K, N):
    """Uniform ternary int2 words [K/16, N] (codes {0, 1, 3}), seeded by the shape."""
    key = ("int2", K, N)
    if key not in _cache:
        rng = np.random.default_rng(K * 31 + N)
        c = rng.integers(0, 3, size=(K // 16, 16, N), dtype=np.uint8)
        c[c == 2] = 3
        w = np.zeros((K // 16, N), np.uint32)
        for j in range(16):
            w |= c[:, j, :].astype(np.uint32) << np.uint32(2 * j)
        _cache[key] = w
    return _cache[key]


def packed_int1(K, N):
    """Uniform +-1 int1 weights: (per-column order [K/32, N], device sel layout)."""
    key = ("int1", K, N)
    if key not in _cache:
        rng = np.random.default_rng(K * 37 + N)
        col = rng.integers(0, 1 << 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
        _cache[key] = (col, orc.int1_to_sel(col, K, N))
    return _cache[key]


def sample_rows(M, n=16):
    if M <= n:
        return np.arange(M)
    rng = np.random.default_rng(M)
    return np.unique(np.concatenate([[0, M - 1], rng.choice(M, n - 2, replace=False)]))


@pytest.mark.parametrize("fmt", ["int2", "int1"])
@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M", [1, 4, 8])
@pytest.mark.parametrize("K,N", C2_SHAPES)
def test_c2_decode_sweep(cuda, tl, K, N, M, bf16, fmt):
    rng = np.random.default_rng(M * 7 + bf16 + K + N)
    S = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    dA, dS = dev_dt(A, bf16), dev_dt(S, bf16)
    ws = tl.Workspace()
    if fmt == "int2":
        B = packed_int2(K, N)
        out = host_dt(tl.int2_upcvt(dA, dev_u32(B), dS, workspace=ws))
        acc = orc.int2_gold(A, B, S, M, K, N, bf16)
    else:
        col, sel = packed_int1(K, N)
        out = host_dt(tl.int1_upcvt(dA, dev_u32(sel), dS, workspace=ws))
        acc = orc.int1_gold(A, col, S, M, K, N, bf16)
    gold = orc.epilogue(0, False, acc, None, None, M, N, bf16)
    check_output(out, gold, bf16, False, "C2 %s M=%d K=%d N=%d bf16=%d" % (fmt, M, K, N, bf16))
    assert tl.device_error() == 0


@pytest.mark.parametrize("postop,out_f32", [(p, f) for p in range(5) for f in (False, True)])
def test_c2_epilogues_full_width(cuda, tl, postop, out_f32):
    import torch
    K, N, M, bf16 = 4096, 28672, 1, 0
    rng = np.random.default_rng(40 + postop)
    B, S, A = packed_int2(K, N), synth.scales(rng, K, N, bf16), synth.activations(rng, M, K, bf16)
    other, bias = synth.epilogue_operands(rng, postop, out_f32, M, N, bf16)
    o = dev_dt(other, bf16) if other is not None else None
    b = None
    if bias is not None:
        b = torch.from_numpy(bias).cuda() if out_f32 else dev_dt(bias, bf16)
    out = host_dt(tl.int2_upcvt(dev_dt(A, bf16), dev_u32(B), dev_dt(S, bf16), postop=postop, out_f32=out_f32,
                                other=o, bias=b, workspace=tl.Workspace()))
    gold = orc.epilogue(postop, out_f32, orc.int2_gold(A, B, S, M, K, N, bf16), other, bias, M, N, bf16)
    check_output(out, gold, bf16, out_f32, "C2 postop=%d out_f32=%d" % (postop, out_f32))


@pytest.mark.parametrize("M", [1, 512, 2048])
@pytest.mark.parametrize("K,N", C3_SHAPES)
def test_c3_int8_prefill(cuda, tl, K, N, M):
    bf16 = 1
    rng = np.random.default_rng(K + N + M)
    B = packed_int2(K, N)
    SB = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    dA, dB = dev_dt(A, bf16), dev_u32(B)
    SA, Aq = tl.int8_quant_a(dA)
    out = host_dt(tl.int2_int8(dA, dB, dev_dt(SB, bf16), SA, Aq=Aq))
    rows = sample_rows(M)
    r = len(rows)
    As = np.ascontiguousarray(A[rows])
    SA_gold = orc.int8_scale_a(As, r, K, bf16)
    assert np.array_equal(host_dt(SA)[:, rows], SA_gold[:, :r]), "quant_a scales"
    Q_gold = orc.int8_quant(As, SA_gold, r, K, bf16)
    Aq_rows = Aq.cpu().numpy()[rows]
    assert np.array_equal(Aq_rows, Q_gold), "quant_a codes"
    gold = orc.epilogue(0, False, orc.int8_gold(As, B, SA_gold, SB, r, K, N, bf16), None, None, r, N, bf16)
    check_output(out[rows], gold, bf16, False, "C3 M=%d K=%d N=%d" % (M, K, N))
    # the exact int32 group dots on a column slice
    n0, ns = (N // 2) // 16 * 16, 256
    Bs = np.ascontiguousarray(B[:, n0:n0 + ns])
    D = tl.int2_int8_group_dots(dev_any(Aq_rows), dev_u32(Bs)).cpu().numpy()
    assert np.array_equal(D, orc.int8_group_dots(Q_gold, Bs, r, K, ns)), "group dots"
    # qmode 1 (the reference driver's default: scales only, quantise in the GEMM) gives
    # the same bits as qmode 0 on every path
    out1 = host_dt(tl.int2_int8(dA, dB, dev_dt(SB, bf16), SA, qmode=1))
    assert np.array_equal(out1.view(np.uint16), out.view(np.uint16)), "qmode 1 vs qmode 0"
    assert tl.device_error() == 0


@pytest.mark.parametrize("M", [1, 8, 512])
@pytest.mark.parametrize("z", [0.2, 0.35, 0.5])
def test_c4_bitcos_hadamard(cuda, tl, z, M):
    K, N, hb, bf16 = 5376, 21504, 256, 0
    key = ("bitcos", z)
    if key not in _cache:
        _cache[key] = tl.bitcos_random(K, N, z, int(z * 100))
    buf = _cache[key]
    rng = np.random.default_rng(M + int(z * 100))
    S = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    s = np.where(rng.random(K) < 0.5, -1, 1).astype(np.int8)
    y = tl.hadamard_fwht(dev_dt(A, bf16), hb, signs=dev_any(s))
    out = host_dt(tl.bitcos_upcvt(y, dev_u32(buf), dev_dt(S, bf16)))
    rows = sample_rows(M)
    r = len(rows)
    y_gold = orc.hadamard(np.ascontiguousarray(A[rows]), s, r, K, hb, 1, bf16)
    assert np.array_equal(host_dt(y)[rows], y_gold), "Hadamard transform"
    gold = orc.epilogue(0, False, orc.bitcos_gold(y_gold, buf, S, r, K, N, bf16), None, None, r, N, bf16)
    check_output(out[rows], gold, bf16, False, "C4 z=%.2f M=%d" % (z, M))
    assert tl.device_error() == 0


def test_c5_moe_layer_full_size(cuda, tl):
    T, topk, E, H, I, bf16 = 4096, 8, 128, 2048, 768, 0
    rng = np.random.default_rng(55)
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(T)]).reshape(-1).astype(np.int32)
    gates = rng.standard_normal((T, topk))
    RW = synth.to_dt((np.exp(gates) / np.exp(gates).sum(1, keepdims=True)).reshape(-1), bf16)

    def experts(K, N):
        c = rng.integers(0, 3, size=(E, K // 16, 16, N), dtype=np.uint8)
        c[c == 2] = 3
        w = np.zeros((E, K // 16, N), np.uint32)
        for j in range(16):
            w |= c[:, :, j, :].astype(np.uint32) << np.uint32(2 * j)
        s = synth.to_dt(rng.uniform(0.01, 0.05, size=(E, K // 128, N)), bf16)
        return w, s

    Bg, Sg = experts(H, I)
    Bu, Su = experts(H, I)
    Bd, Sd = experts(I, H)
    X = synth.activations(rng, T, H, bf16)
    meta, perm, inv = tl.moe_route(dev_any(ids), E)
    Xs = tl.moe_gather(dev_dt(X, bf16), perm, topk)
    up = tl.moe_gemm(meta, Xs, dev_u32(Bu), dev_dt(Su, bf16), E)
    Hh = tl.moe_gemm(meta, Xs, dev_u32(Bg), dev_dt(Sg, bf16), E, postop=1, other=up)
    Y = tl.moe_gemm(meta, Hh, dev_u32(Bd), dev_dt(Sd, bf16), E, out_f32=True)
    O = synth.from_dt(host_dt(tl.moe_combine(Y, inv, dev_dt(RW, bf16), T, topk)), bf16)
    toks = np.unique(np.concatenate([[0, 1, T // 2, T - 1], rng.choice(T, 8, replace=False)]))
    refs = [orc.moe_token_ref(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, int(t), topk, H, I, bf16) for t in toks]
    e = moe_layer_err(O[toks], refs)
    assert e <= MOE_TOL[bf16], "layer rel err %.3g over %d tokens" % (e, len(toks))
    assert tl.device_error() == 0
