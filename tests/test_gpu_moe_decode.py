"""int2 MoE decode GEMVs on the GPU (int2_moe/int2_moe.cl:63-174) vs the oracle, through the
C ABI: gate_up (both projections, SwiGLU) and down against the int2 host gold per routed
row, reduce exactly, down_sum against down + reduce, and a whole decode layer against the
double-precision token reference of the decode driver (int2_moe/main.cpp:267-291)."""
import numpy as np
import pytest

from helpers import F32_FLOOR, F32_REL_TOL, REL_TOL, check_output, dev_any, dev_dt, dev_u32, host_dt, rel_err
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu


def routing(rng, T, topk, E):
    return np.stack([rng.permutation(E)[:topk] for _ in range(T)]).reshape(-1).astype(np.int32)


def experts(rng, E, K, N, bf16):
    B = np.stack([synth.pack_int2(synth.ternary(rng, K, N)) for _ in range(E)])
    S = np.stack([synth.scales(rng, K, N, bf16) for _ in range(E)])
    return B, S


def sigmoid_ref(x):
    # common/epilogue.hpp:34 (sigmoid with the reference's clamp at -10)
    x = np.asarray(x, np.float32)
    return np.where(x <= -10.0, np.float32(0.0), np.float32(1.0) / (np.exp(-x) + np.float32(1.0))).astype(np.float32)


def layer_case(seed, T, topk, E, H, I, bf16):
    rng = np.random.default_rng(seed)
    ids = routing(rng, T, topk, E)
    X = synth.activations(rng, T, H, bf16)
    Bg, Sg = experts(rng, E, H, I, bf16)
    Bu, Su = experts(rng, E, H, I, bf16)
    Bd, Sd = experts(rng, E, I, H, bf16)
    w = rng.random((T, topk)) + 0.05
    RW = synth.to_dt((w / w.sum(1, keepdims=True)).reshape(-1), bf16)
    return dict(ids=ids, X=X, Bg=Bg, Sg=Sg, Bu=Bu, Su=Su, Bd=Bd, Sd=Sd, RW=RW)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("T,topk,E,H,I", [(1, 8, 16, 2048, 768), (3, 4, 8, 512, 256), (8, 2, 6, 1024, 384)])
def test_gate_up(cuda, tl, bf16, T, topk, E, H, I):
    c = layer_case(T + E + H, T, topk, E, H, I, bf16)
    Hd = host_dt(tl.moe_decode_gate_up(dev_any(c["ids"]), dev_dt(c["X"], bf16), dev_u32(c["Bg"]), dev_dt(c["Sg"], bf16),
                                       dev_u32(c["Bu"]), dev_dt(c["Su"], bf16), E, topk))
    for g in range(T * topk):
        t, e = g // topk, c["ids"][g]
        x = c["X"][t:t + 1]
        ag = orc.int2_gold(x, c["Bg"][e], c["Sg"][e], 1, H, I, bf16)[0]
        au = orc.int2_gold(x, c["Bu"][e], c["Su"][e], 1, H, I, bf16)[0]
        gold = synth.to_dt(ag * sigmoid_ref(ag) * au, bf16)
        check_output(Hd[g], gold, bf16, False, "gate_up row %d" % g)
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("T,topk,E,I,H", [(1, 8, 16, 768, 2048), (4, 4, 8, 256, 512)])
def test_down_reduce_and_down_sum(cuda, tl, bf16, T, topk, E, I, H):
    import torch
    rng = np.random.default_rng(3 + T + bf16)
    G = T * topk
    ids = routing(rng, T, topk, E)
    Hin = synth.activations(rng, G, I, bf16)
    Bd, Sd = experts(rng, E, I, H, bf16)
    w = rng.random((T, topk)) + 0.05
    RW = synth.to_dt((w / w.sum(1, keepdims=True)).reshape(-1), bf16)
    dids, dH, dRW, dB, dS = dev_any(ids), dev_dt(Hin, bf16), dev_dt(RW, bf16), dev_u32(Bd), dev_dt(Sd, bf16)
    Y = tl.moe_decode_down(dids, dH, dRW, dB, dS, E)
    Yh = Y.cpu().numpy()
    rw = synth.from_dt(RW, bf16)
    for g in range(G):
        gold = orc.int2_gold(Hin[g:g + 1], Bd[ids[g]], Sd[ids[g]], 1, I, H, bf16)[0] * rw[g]
        assert rel_err(Yh[g], gold, F32_FLOOR) <= F32_REL_TOL, g
    # reduce: fp32 sums in j order, one rounding to DT -> bit exact
    dt = torch.bfloat16 if bf16 else torch.float16
    O = host_dt(tl.moe_decode_reduce(Y, T, topk, dt))
    want = np.zeros((T, H), np.float32)
    for j in range(topk):
        want = (want + Yh[np.arange(T) * topk + j]).astype(np.float32)
    assert np.array_equal(O, synth.to_dt(want, bf16))
    # down_sum: the same within fp32 summation order
    O2 = host_dt(tl.moe_decode_down_sum(dids, dH, dRW, dB, dS, E, topk))
    check_output(O2, O, bf16, False, "down_sum vs down + reduce")
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("fused", [False, True])
def test_layer_vs_token_reference(cuda, tl, bf16, fused):
    import torch
    T, topk, E, H, I = 2, 8, 16, 1024, 384
    c = layer_case(11 + bf16, T, topk, E, H, I, bf16)
    dids = dev_any(c["ids"])
    Hd = tl.moe_decode_gate_up(dids, dev_dt(c["X"], bf16), dev_u32(c["Bg"]), dev_dt(c["Sg"], bf16), dev_u32(c["Bu"]),
                               dev_dt(c["Su"], bf16), E, topk)
    dRW, dB, dS = dev_dt(c["RW"], bf16), dev_u32(c["Bd"]), dev_dt(c["Sd"], bf16)
    if fused:
        O = tl.moe_decode_down_sum(dids, Hd, dRW, dB, dS, E, topk)
    else:
        O = tl.moe_decode_reduce(tl.moe_decode_down(dids, Hd, dRW, dB, dS, E), T, topk,
                                 torch.bfloat16 if bf16 else torch.float16)
    O = synth.from_dt(host_dt(O), bf16)
    for t in range(T):
        ref = orc.moe_decode_token_ref(c["X"], c["ids"], c["RW"], c["Bg"], c["Sg"], c["Bu"], c["Su"], c["Bd"],
                                       c["Sd"], t, topk, H, I, bf16)
        # the decode driver's own check (int2_moe/main.cpp:286-291): max |err| / max |ref| < 1e-2
        assert np.max(np.abs(O[t] - ref)) / np.max(np.abs(ref)) < 1e-2, t
        # and per element: one DT rounding inside (H) plus the DT output, as the prefill layer
        assert rel_err(O[t], ref) <= 4 * REL_TOL[bf16], t


def test_bad_expert_id(cuda, tl):
    T, topk, E, H, I = 1, 4, 4, 256, 128
    c = layer_case(5, T, topk, E, H, I, 0)
    ids = c["ids"].copy()
    ids[2] = 9  # >= E
    tl.device_error(reset=True)
    Hd = tl.moe_decode_gate_up(dev_any(ids), dev_dt(c["X"], 0), dev_u32(c["Bg"]), dev_dt(c["Sg"], 0), dev_u32(c["Bu"]),
                               dev_dt(c["Su"], 0), E, topk)
    import torch
    torch.cuda.synchronize()
    assert tl.device_error() & 2
    h = synth.from_dt(host_dt(Hd), 0)
    assert np.all(np.isfinite(h)) and not np.any(h[2])  # the bad row contributes zero
    tl.device_error(reset=True)
