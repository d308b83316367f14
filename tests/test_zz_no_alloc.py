"""The allocation-free GEMV entry point, ternocl_int2_upcvt_noalloc.

It serves callers that cannot allocate device memory where they run a GEMV (code
inside another framework's memory pool, runtimes that forbid allocation after
start-up, plugins whose host owns every allocation): its split-K scratch lives in a
fixed 16 MiB device array declared by the library.  These tests call it through the C
ABI, twice in a row on the same inputs (the shared array keeps the previous call's
contents, so the second call checks that it starts from a clean state), and compare
each result with the oracle (the reference's host gold) and bit for bit with the
regular entry point, ternocl_int2_upcvt, given a workspace of the array's size: the
allocation-free call runs the same plan.  The file is named to be collected last, and
each test works whether it runs alone in a fresh process or after the whole suite.
"""
import ctypes

import numpy as np
import pytest

from helpers import check_output, dev_dt, dev_u32, host_dt, int2_case, int2_gold_out

pytestmark = pytest.mark.gpu

SCRATCH = 16 << 20

CASES = [
    (1, 4096, 4096, 0, 0),    # integer-MMA GEMV, one CTA per 32-column strip (no split)
    (3, 2048, 1024, 1, 0),    # the same at M = 3
    (8, 1024, 512, 0, 3),     # fp16-MMA GEMV (M > 4) with a K split
    (1, 14336, 512, 1, 1),
    (1, 128, 16, 0, 0),       # one scale group: no split, no scratch
    (63, 256, 32768, 0, 2),   # the plan's partial sums (16.5 MiB) exceed the array: runs
                              # without scratch (split inside thread-block clusters)
]


@pytest.mark.parametrize("M,K,N,bf16,postop", CASES)
def test_noalloc_matches_oracle_and_regular_entry_twice(cuda, tl, M, K, N, bf16, postop):
    torch = cuda
    c = int2_case(900 + M + N, M, K, N, bf16, postop, False)
    gold = int2_gold_out(c, M, K, N, bf16, postop, False)
    A, B, S = dev_dt(c["A"], bf16), dev_u32(c["B"]), dev_dt(c["S"], bf16)
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = dev_dt(c["bias"], bf16) if c["bias"] is not None else None
    L = tl.lib()
    stream = torch.cuda.current_stream().cuda_stream
    # the regular entry point with a zeroed workspace of exactly the array's size
    ws = torch.zeros(SCRATCH, dtype=torch.uint8, device="cuda")
    ref_out = torch.empty((M, N), dtype=A.dtype, device="cuda")
    st = L.ternocl_int2_upcvt(A.data_ptr(), B.data_ptr(), S.data_ptr(), ref_out.data_ptr(),
                              other.data_ptr() if other is not None else None,
                              bias.data_ptr() if bias is not None else None,
                              M, N, K, bf16, postop, 0, tl.ALGO_GEMV, ws.data_ptr(), SCRATCH, stream)
    assert st == 0, L.ternocl_status_string(st)
    ref = host_dt(ref_out)
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=A.dtype, device="cuda")
        st = L.ternocl_int2_upcvt_noalloc(A.data_ptr(), B.data_ptr(), S.data_ptr(), out.data_ptr(),
                                          other.data_ptr() if other is not None else None,
                                          bias.data_ptr() if bias is not None else None,
                                          M, N, K, bf16, postop, 0, stream)
        assert st == 0, L.ternocl_status_string(st)
        torch.cuda.synchronize()
        got = host_dt(out)
        check_output(got, gold, bf16, False, "noalloc call %d M=%d K=%d N=%d" % (call, M, K, N))
        assert np.array_equal(got, ref), "call %d differs from ternocl_int2_upcvt" % call
    assert tl.device_error() == 0


def test_noalloc_rejects_shapes_no_form_can_run(cuda, tl):
    # M=63, N=65536, K=2^20: the split-K partials need far more than the 16 MiB array, and
    # without them a CTA would stage 2 MB of activations; the call is refused before any
    # device work on the operands (the pointers are never touched)
    L = tl.lib()
    p = ctypes.c_void_p(1 << 20)
    st = L.ternocl_int2_upcvt_noalloc(p, p, p, p, None, None, 63, 65536, 1 << 20, 0, 0, 0, None)
    assert st == 7  # TERNOCL_ERR_WORKSPACE
    assert b"workspace" in L.ternocl_status_string(st)
