"""The allocation-free GEMV entry point, ternocl_int2_upcvt_noalloc.

It serves callers that cannot allocate device memory where they run a GEMV (code
inside another framework's memory pool, runtimes that forbid allocation after
start-up, plugins whose host owns every allocation): its split-K scratch lives in a
fixed device array declared by the library.  These tests call it through the C ABI
and compare it with the regular entry point, ternocl_int2_upcvt, on the same inputs,
twice in a row (the shared scratch keeps the previous call's contents, so the second
call checks that it is reset properly).  The file is named to be collected last, and
each test works whether it runs alone in a fresh process or after the whole suite.
"""
import ctypes

import numpy as np
import pytest

from helpers import REL_TOL, dev_dt, dev_u32, host_dt, int2_case, rel_err
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu

CASES = [(1, 4096, 4096, 0, 0), (3, 2048, 1024, 1, 0), (8, 1024, 512, 0, 3), (1, 14336, 512, 1, 1)]


@pytest.mark.parametrize("M,K,N,bf16,postop", CASES)
def test_noalloc_matches_regular_entry_point_twice(cuda, tl, M, K, N, bf16, postop):
    torch = cuda
    c = int2_case(900 + M + N, M, K, N, bf16, postop, False)
    A, B, S = dev_dt(c["A"], bf16), dev_u32(c["B"]), dev_dt(c["S"], bf16)
    other = dev_dt(c["other"], bf16) if c["other"] is not None else None
    bias = dev_dt(c["bias"], bf16) if c["bias"] is not None else None
    ref = host_dt(tl.int2_upcvt(A, B, S, postop=postop, other=other, bias=bias, workspace=tl.Workspace()))
    L = tl.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=A.dtype, device="cuda")
        st = L.ternocl_int2_upcvt_noalloc(A.data_ptr(), B.data_ptr(), S.data_ptr(), out.data_ptr(),
                                          other.data_ptr() if other is not None else None,
                                          bias.data_ptr() if bias is not None else None,
                                          M, N, K, bf16, postop, 0, stream)
        assert st == 0, L.ternocl_status_string(st)
        torch.cuda.synchronize()
        got = host_dt(out)
        e = rel_err(synth.from_dt(got, bf16), synth.from_dt(ref, bf16))
        assert e <= REL_TOL[bf16], "call %d: rel err %.3g vs ternocl_int2_upcvt" % (call, e)
    assert tl.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda, tl):
    # 2 x M x N fp32 partial sums of M=64, N=65536 need 32 MiB > the 16 MiB array; the
    # call is refused before any device work (the pointers are never touched)
    L = tl.lib()
    p = ctypes.c_void_p(1 << 20)
    st = L.ternocl_int2_upcvt_noalloc(p, p, p, p, None, None, 64, 65536, 1024, 0, 0, 0, None)
    assert st == 7  # TERNOCL_ERR_WORKSPACE
    assert b"workspace" in L.ternocl_status_string(st)
