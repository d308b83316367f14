"""int2 upconvert GEMV/GEMM on the GPU vs the oracle (the reference's host gold,
int2_fp16_upcvt/main.cpp:79-98 + common/epilogue.hpp:50-67), through the C ABI."""
import numpy as np
import pytest

from helpers import check_output, dev_dt, dev_u32, host_dt, int2_case, int2_gold_out

pytestmark = pytest.mark.gpu

# shapes from the reference validation matrix (int2_fp16_upcvt/validate.sh:8-10) and
# the Llama-3-8B decode sweep, at sizes the oracle finishes in seconds
GEMV_SHAPES = [(1, 4096, 4096), (1, 4096, 6144), (4, 6144, 5120), (3, 256, 48), (8, 1024, 512),
               (1, 128, 16), (2, 512, 272), (5, 2048, 1024), (13, 512, 256), (1, 14336, 512),
               (1, 384, 272), (1, 5376, 2576)]


def run(tl, c, M, K, N, bf16, postop, out_f32, algo, ws=None):
    A, B, S = dev_dt(c["A"], bf16), dev_u32(c["B"]), dev_dt(c["S"], bf16)
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = None
    if c["bias"] is not None:
        import torch
        bias = torch.from_numpy(c["bias"]).cuda() if out_f32 else dev_dt(c["bias"], bf16)
    out = tl.int2_upcvt(A, B, S, postop=postop, out_f32=out_f32, other=other, bias=bias,
                        algo=algo, workspace=ws)
    return host_dt(out)


# GEMV implementations: fp16/bf16 mma.sync on decoded weights, integer mma.sync on int8
# weights and fixed-point activation digits (M <= 4) per 32-column strip, tcgen05/TMEM
ALGOS = ["f16", "digit", "tmem"]


@pytest.fixture
def gemv_algo(request, tl):
    """Maps an ALGOS name to (algo argument, implementation option) for the test body."""
    def select(name):
        impl = {"f16": 1, "digit": 2, "tmem": 0}[name]
        old = tl.set_option(tl.OPT_GEMV_IMPL, impl)
        request.addfinalizer(lambda: tl.set_option(tl.OPT_GEMV_IMPL, old))
        return tl.ALGO_GEMV_TMEM if name == "tmem" else tl.ALGO_GEMV
    return select


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N", GEMV_SHAPES)
def test_gemv_parity(cuda, tl, gemv_algo, M, K, N, bf16, algo):
    algo = gemv_algo(algo)
    c = int2_case(100 + M + K + N, M, K, N, bf16)
    gold = int2_gold_out(c, M, K, N, bf16, 0, False)
    ws = tl.Workspace()
    for w in (None, ws):
        out = run(tl, c, M, K, N, bf16, 0, False, algo, w)
        check_output(out, gold, bf16, False, "int2 gemv algo=%d M=%d K=%d N=%d bf16=%d" % (algo, M, K, N, bf16))
    assert tl.device_error() == 0


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("out_f32", [False, True])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 512), (3, 2048, 1024)])
def test_gemv_epilogues(cuda, tl, gemv_algo, M, K, N, bf16, postop, out_f32, algo):
    algo = gemv_algo(algo)
    # validate_epilogues.sh:19-39: every POSTOP x {DT, fp32 out} x dtype
    c = int2_case(7 * postop + M, M, K, N, bf16, postop, out_f32)
    gold = int2_gold_out(c, M, K, N, bf16, postop, out_f32)
    out = run(tl, c, M, K, N, bf16, postop, out_f32, algo, tl.Workspace())
    check_output(out, gold, bf16, out_f32, "postop=%d out_f32=%d" % (postop, out_f32))


@pytest.mark.parametrize("algo", ALGOS)
def test_gemv_deterministic(cuda, tl, gemv_algo, algo):
    algo = gemv_algo(algo)
    # main.cpp:351-353: every set reproduces set 0 bit for bit
    M, K, N = 4, 4096, 2048
    c = int2_case(5, M, K, N, 0)
    ws = tl.Workspace()
    outs = [run(tl, c, M, K, N, 0, 0, False, algo, ws) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


@pytest.mark.parametrize("M", [1, 2, 5, 8, 13, 16, 17, 40])
def test_tc_gemv_row_blocks(cuda, tl, M):
    # every activation-row block size of the TMEM GEMV (1, 2, 4, 8, 16 rows per CTA)
    K, N = 1024, 384
    c = int2_case(300 + M, M, K, N, 1)
    gold = int2_gold_out(c, M, K, N, 1, 0, False)
    out = run(tl, c, M, K, N, 1, 0, False, tl.ALGO_GEMV_TMEM, tl.Workspace())
    check_output(out, gold, 1, False, "tc gemv M=%d" % M)
    assert tl.device_error() == 0


def test_gemv_ragged_rows_untouched(cuda, tl):
    # rows >= M and columns >= N are never written
    import torch
    M, K, N = 3, 512, 48
    c = int2_case(9, M, K, N, 0)
    A, B, S = dev_dt(c["A"], 0), dev_u32(c["B"]), dev_dt(c["S"], 0)
    big = torch.full((M + 2, N), 7.0, dtype=torch.float16, device="cuda")
    tl.int2_upcvt(A, B, S, out=big[:M], algo=tl.ALGO_GEMV)
    assert torch.all(big[M:] == 7.0)


@pytest.mark.parametrize("algo", ALGOS)
def test_decode_bit_exact(cuda, tl, gemv_algo, algo):
    algo = gemv_algo(algo)
    # A = identity: C[k, n] = value(code(k, n)) * S exactly (one non-zero term), i.e.
    # the decoded weights; every 2-bit code, as code_to_value reads it (main.cpp:76)
    from ternocl_b200 import synth
    K, N = 512, 96
    rng = np.random.default_rng(8)
    B = rng.integers(0, 1 << 32, size=(K // 16, N), dtype=np.uint64).astype(np.uint32)
    S = synth.to_dt(np.ones((K // 128, N)), 0)
    c = dict(A=synth.to_dt(np.eye(K), 0), B=B, S=S, other=None, bias=None)
    out = synth.from_dt(run(tl, c, K, K, N, 0, 0, False, algo, tl.Workspace()), 0)
    k = np.arange(K)[:, None]
    codes = (B[k // 16, np.arange(N)[None, :]] >> (2 * (k % 16)).astype(np.uint32)) & 3
    assert np.array_equal(out, np.array([0, 1, -2, -1], np.float32)[codes])


@pytest.mark.parametrize("impl", ["digit"])
def test_digit_onehot_bit_exact(cuda, tl, gemv_algo, impl):
    # the integer-MMA GEMVs at M = 4 with one-hot activation rows: C[i, n] is the decoded
    # weight of row k_i exactly (every code and every position of a 16-row word)
    from ternocl_b200 import synth
    algo = gemv_algo(impl)
    K, N = 256, 64
    rng = np.random.default_rng(18)
    B = rng.integers(0, 1 << 32, size=(K // 16, N), dtype=np.uint64).astype(np.uint32)
    S = synth.to_dt(np.ones((K // 128, N)), 0)
    k = np.arange(K)[:, None]
    codes = (B[k // 16, np.arange(N)[None, :]] >> (2 * (k % 16)).astype(np.uint32)) & 3
    want = np.array([0, 1, -2, -1], np.float32)[codes]
    for k0 in range(0, 256, 4):
        eye = np.zeros((4, K))
        eye[np.arange(4), k0 + np.arange(4)] = 1.0
        c = dict(A=synth.to_dt(eye, 0), B=B, S=S, other=None, bias=None)
        out = synth.from_dt(run(tl, c, 4, K, N, 0, 0, False, algo, tl.Workspace()), 0)
        assert np.array_equal(out, want[k0:k0 + 4]), k0


@pytest.mark.parametrize("impl", ["digit"])
@pytest.mark.parametrize("bf16", [0, 1])
def test_digit_outliers_and_zero_rows(cuda, tl, gemv_algo, bf16, impl):
    # rows with a large outlier (the fixed-point step follows the row maximum), a row of
    # tiny values and an all-zero row
    from ternocl_b200 import synth
    algo = gemv_algo(impl)
    M, K, N = 4, 4096, 1024
    c = int2_case(77, M, K, N, bf16)
    A = synth.from_dt(c["A"], bf16).astype(np.float64)
    A[0, 100] = 3000.0 if not bf16 else 3.0e4
    A[1] *= 1e-4
    A[2, 5] = -800.0
    A[3] = 0.0
    c["A"] = synth.to_dt(A, bf16)
    gold = int2_gold_out(c, M, K, N, bf16, 0, False)
    out = run(tl, c, M, K, N, bf16, 0, False, algo, tl.Workspace())
    check_output(out, gold, bf16, False, "digit outliers bf16=%d" % bf16)
    assert not np.any(synth.from_dt(out, bf16)[3])
    # fp32 outputs: the reference's fp32 rule
    out = run(tl, c, M, K, N, bf16, 0, True, algo, tl.Workspace())
    check_output(out, int2_gold_out(c, M, K, N, bf16, 0, True), bf16, True, "digit outliers fp32")


@pytest.mark.parametrize("impl", ["digit"])
def test_digit_row_max_positions(cuda, tl, gemv_algo, impl):
    # the fixed-point exponent follows each row's largest |A|: put it in every position of
    # a 16-byte load (low and high halves of each 32-bit pair) with larger values elsewhere
    # in the other half-words, so a lost maximum would overflow the digits
    from ternocl_b200 import synth
    algo = gemv_algo(impl)
    M, K, N = 4, 1024, 256
    c = int2_case(91, M, K, N, 0)
    for pos in range(8):
        A = np.full((M, K), 0.5)
        A[:, 1::2] = 3.0          # high halves of the first load
        A[:, 8:] = -2.0
        A[:, pos] = 7.5           # the row maximum
        A[1] *= -1.0
        c["A"] = synth.to_dt(A, 0)
        gold = int2_gold_out(c, M, K, N, 0, 0, False)
        check_output(run(tl, c, M, K, N, 0, 0, False, algo, tl.Workspace()), gold, 0, False, "max at %d" % pos)
