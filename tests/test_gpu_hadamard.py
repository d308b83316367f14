"""Sign flip + blockwise FWHT on the GPU vs the oracle, bit for bit.  The oracle is
pinned to the reference kernel itself (hadamard/hadamard_fwht.cl run on the CPU,
oracle/ref_hadamard.cpp) through tests/golden/golden_hadamard.npz."""
import os

import numpy as np
import pytest

from helpers import dev_any, dev_dt, host_dt
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_hadamard.npz")
HBS = [256, 512, 1024, 2048, 4096]


def case(seed, rows, K, bf16):
    rng = np.random.default_rng(seed)
    x = synth.activations(rng, rows, K, bf16)
    s = np.where(rng.random(K) < 0.5, -1, 1).astype(np.int8)
    return x, s


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("hb", HBS)
@pytest.mark.parametrize("rows", [1, 3, 8, 33])
def test_fwht_bit_exact(cuda, tl, rows, hb, bf16):
    K = hb * (3 if hb <= 1024 else 2)
    x, s = case(rows * 13 + hb, rows, K, bf16)
    X, Sg = dev_dt(x, bf16), dev_any(s)
    for use_signs in (1, 0):
        y = host_dt(tl.hadamard_fwht(X, hb, signs=Sg if use_signs else None))
        assert np.array_equal(y, orc.hadamard(x, s, rows, K, hb, use_signs, bf16)), (use_signs, hb)


@pytest.mark.parametrize("bf16", [0, 1])
def test_fwht_baseline_shape(cuda, tl, bf16):
    # C4: K = 5376 (5376 % 1024 != 0, so HB = 256, the largest power-of-two divisor)
    rows, K, hb = 8, 5376, 256
    x, s = case(7, rows, K, bf16)
    y = host_dt(tl.hadamard_fwht(dev_dt(x, bf16), hb, signs=dev_any(s)))
    assert np.array_equal(y, orc.hadamard(x, s, rows, K, hb, 1, bf16))


def test_fwht_golden(cuda, tl):
    d = np.load(GOLDEN)
    for dt, bf16 in (("fp16", 0), ("bf16", 1)):
        for hb in HBS:
            k = "had_%s_%d" % (dt, hb)
            x, s = d[k + "_x"], d[k + "_s"]
            X = dev_dt(x, bf16)
            assert np.array_equal(host_dt(tl.hadamard_fwht(X, hb, signs=dev_any(s))), d[k + "_y"]), k
            assert np.array_equal(host_dt(tl.hadamard_fwht(X, hb)), d[k + "_y0"]), k


def test_fwht_in_place(cuda, tl):
    rows, K, hb = 4, 4096, 1024
    x, s = case(3, rows, K, 0)
    X = dev_dt(x, 0)
    tl.hadamard_fwht(X, hb, signs=dev_any(s), out=X)
    assert np.array_equal(host_dt(X), orc.hadamard(x, s, rows, K, hb, 1, 0))


def test_fwht_shape_errors(cuda, tl):
    import torch
    L = tl.lib()
    x = torch.zeros(2, 5376, dtype=torch.float16, device="cuda")
    p = x.data_ptr()
    assert L.ternocl_hadamard_fwht(p, None, p, 2, 5376, 1024, 0, 0, None) == 1  # K % HB
    assert L.ternocl_hadamard_fwht(p, None, p, 2, 5376, 128, 0, 0, None) == 1   # HB range
    assert L.ternocl_hadamard_fwht(p, None, p, 2, 5376, 768, 0, 0, None) == 1   # power of two
    assert L.ternocl_hadamard_fwht(p, None, p, 2, 5376, 256, 1, 0, None) == 2   # signs missing
