"""The command-line drivers (ternocl_b200/bin): the reference drivers' flags and stdout
lines (int2_fp16_upcvt/main.cpp:378-431, int1_fp16_upcvt/main.cpp:385-437,
int2_via_int2_x_int8_dpas/main.cpp:440-488, bitcos_fp16_upcvt/main.cpp:337-387,
int2_moe/prefill.cpp:81-111), which the reference's bench and validate scripts grep.
Without a GPU: usage and flag errors.  On the GPU: small runs whose own validation
against their host gold must pass."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "ternocl_b200", "bin")
DRIVERS = ["int2_fp16_upcvt", "int1_fp16_upcvt", "int2_int8", "bitcos_fp16_upcvt", "int2_moe_prefill", "int2_moe"]

AVG_DEV = re.compile(r"^Avg dev   time: [0-9.]+ ms \([0-9.]+ GFLOPS, [0-9.]+ GiB/s", re.M)
VALID = re.compile(r"^Validation summary: (\d+)/(\d+) sets PASSED$", re.M)
REL = re.compile(r"^validation \[set 0/\d+\]: max rel err \S+ \(tolerance \S+: within\)$", re.M)
COMPARE = re.compile(r"^validation \[set 0/\d+\]: max abs diff \S+ (\(idx \d+\), max ULP diff \d+ \(idx \d+\)|, max rel diff \S+), "
                     r"pass rate 100%$", re.M)


def drv(name, *args, timeout=600):
    path = os.path.join(BIN, name)
    if not os.path.exists(path):
        pytest.skip("drivers not built (make -C ternocl_b200/drivers)")
    return subprocess.run([path] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("name", DRIVERS)
def test_usage(name):
    moe = name.startswith("int2_moe")
    r = drv(name, "--help") if not moe else drv(name, "--bogus")
    text = r.stdout + r.stderr
    assert "--m" in text or "--t" in text
    assert r.returncode == (0 if not moe else 1)


@pytest.mark.parametrize("name", DRIVERS[:4])
def test_flag_errors(name):
    assert drv(name, "--dtype", "fp8").returncode == 1
    assert drv(name, "--postop", "7").returncode == 1
    assert drv(name, "--no-such-flag").returncode == 1


@pytest.mark.gpu
@pytest.mark.parametrize("name", DRIVERS[:4])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("m", [1, 96])
def test_validates(name, dtype, m):
    r = drv(name, "--m", m, "--n", 512, "--k", 1024, "--dtype", dtype, "--sets", 2, "--iters", 3, "--seed", 1)
    assert r.returncode == 0, r.stderr
    out = r.stdout
    assert AVG_DEV.search(out), out
    assert COMPARE.search(out), out
    # beside the reference's rule: the relative error the tests hold the library to
    assert REL.search(out), out
    assert VALID.search(out).groups() == ("2", "2"), out
    if name == "int2_int8":
        assert re.search(r"^scale_a: 0/\d+ differ from host$", out, re.M), out
        assert re.search(r"^Avg dev   pre : [0-9.]+ ms$", out, re.M), out


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["int2_fp16_upcvt", "int2_int8"])
@pytest.mark.parametrize("postop,out_f32", [(1, False), (3, True), (4, False)])
def test_validates_epilogues(name, postop, out_f32):
    args = ["--m", 8, "--n", 256, "--k", 512, "--sets", 2, "--iters", 2, "--postop", postop, "--seed", 2]
    r = drv(name, *(args + (["--out-f32"] if out_f32 else [])))
    assert VALID.search(r.stdout).groups() == ("2", "2"), r.stdout


@pytest.mark.gpu
def test_distinct_sets_and_tile_flags():
    r = drv("int2_fp16_upcvt", "--m", 4, "--n", 256, "--k", 512, "--sets", 3, "--iters", 2, "--distinct-sets",
            "--sgm", 4, "--ls", 2, "--grf128")
    assert VALID.search(r.stdout).groups() == ("3", "3"), r.stdout
    assert "Ignored" in r.stdout and "--sgm 4" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("int8", [None, 0, 1])
def test_moe_prefill_check(int8):
    args = ["--t", 256, "--e", 16, "--topk", 4, "--h", 512, "--i", 256, "--sets", 2, "--iters", 2, "--check", 2]
    r = drv("int2_moe_prefill", *(args + (["--int8", int8] if int8 is not None else [])))
    assert r.returncode == 0, r.stderr
    assert re.search(r"^check \(2 tokens\): max_abs_err \S+ \(max \|ref\| \S+, rel \S+\) PASS$", r.stdout, re.M), r.stdout
    assert re.search(r"\| layer [0-9.]+ us, [0-9.]+ TFLOPS, x48 = [0-9.]+ ms$", r.stdout, re.M), r.stdout
    if int8 is not None:
        assert "int8 activations, qmode %d" % int8 in r.stdout
        assert re.search(r"quant_x [0-9.]+ us .*quant_h [0-9.]+ us", r.stdout), r.stdout


def test_moe_prefill_int8_flag_errors():
    assert drv("int2_moe_prefill", "--int8", "2").returncode == 1


@pytest.mark.gpu
@pytest.mark.parametrize("fused", [False, True])
def test_moe_decode_check(fused):
    args = ["--t", 2, "--e", 16, "--topk", 4, "--h", 512, "--i", 256, "--sets", 2, "--iters", 2]
    r = drv("int2_moe", *(args + (["--fused"] if fused else [])))
    assert r.returncode == 0, r.stderr
    assert re.search(r"^check: max_abs_err \S+ \(max \|ref\| \S+, rel \S+\) PASS$", r.stdout, re.M), r.stdout
    assert re.search(r"\| layer [0-9.]+ us, [0-9.]+ GiB/s, x48 layers = [0-9.]+ ms$", r.stdout, re.M), r.stdout
