"""Multi-GPU paths on >= 2 GPUs (skipped with fewer): the column-sharded GEMV with the
all-gather fused into its epilogue (peer stores + flag handshake) and the expert-parallel
MoE over NCCL all-to-all, each against the single-GPU result of the same problem."""
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def ngpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def spawn(fn, world, tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["PYTHONPATH"] = os.pathsep.join([HERE, os.path.dirname(HERE), os.environ.get("PYTHONPATH", "")])
    mp.spawn(fn, args=(world, port, str(tmp_path)), nprocs=world, join=True)


@pytest.fixture(scope="module")
def workers():
    sys.path.insert(0, HERE)
    import multi_gpu_workers
    return multi_gpu_workers


@pytest.mark.skipif(ngpus() < 2, reason="needs 2 GPUs")
def test_fused_allgather_gemv(workers, tmp_path):
    world = 2
    spawn(workers.fused_gemv_worker, world, tmp_path)
    for (M, K, N) in [(1, 4096, 4096), (3, 1024, 272), (8, 2048, 6144)]:
        ds = [torch.load(tmp_path / ("fused_%d_%d_%d_%d.pt" % (M, K, N, r))) for r in range(world)]
        for d in ds:
            assert d["err"] == 0
            for o in d["outs"]:
                # every rank holds every rank's columns, bit-identical to that rank's own
                # single-GPU GEMV of its shard
                for src in ds:
                    assert torch.equal(o[:, src["n0"]:src["n0"] + src["nl"]], src["shard"]), (M, K, N)


@pytest.mark.skipif(ngpus() < 2, reason="needs 2 GPUs")
def test_expert_parallel_moe(workers, tmp_path):
    world = 2
    spawn(workers.ep_moe_worker, world, tmp_path)
    for r in range(world):
        d = torch.load(tmp_path / ("ep_%d.pt" % r))
        assert torch.allclose(d["O"].float(), d["ref"].float(), rtol=2e-3, atol=2e-3)


def test_peer_wait_times_out_and_gpu_stays_usable(tl):
    """Failure detection without a GPU fault: one GPU plays rank 0 of a two-rank
    column-sharded GEMV whose rank 1 never arrives (its flag is never written).  The
    kernel's wait for the peer gives up after the limit set here (50 ms), sets bit 2 of
    the device error word and returns; its own columns are already stored everywhere,
    and the context keeps working (a plain GEMV afterwards matches the oracle).  The
    reference has no such path: its drivers exit on any error (int2_fp16_upcvt/main.cpp:40-48)."""
    import ctypes
    import time

    import numpy as np

    from helpers import check_output, dev_dt, dev_u32, host_dt, int2_case, int2_gold_out
    assert torch.cuda.is_available()
    M, K, N, world = 1, 1024, 512, 2
    c = int2_case(3, M, K, N, 0)
    A, B, S = dev_dt(c["A"], 0), dev_u32(c["B"]), dev_dt(c["S"], 0)
    nl = N // world  # rank 0 holds columns [0, nl)
    Bs, Ss = B[:, :nl].contiguous(), S[:, :nl].contiguous()
    Cs = [torch.zeros(M, N, dtype=torch.float16, device="cuda") for _ in range(world)]
    flags = [torch.zeros(world + 1, dtype=torch.int32, device="cuda") for _ in range(world)]
    L = tl.lib()
    ws = torch.zeros(L.ternocl_gemv_allgather_workspace_size(M, nl, K), dtype=torch.uint8, device="cuda")
    cptr = (ctypes.c_void_p * world)(*[x.data_ptr() for x in Cs])
    fptr = (ctypes.c_void_p * world)(*[x.data_ptr() for x in flags])
    torch.cuda.synchronize()
    tl.device_error(reset=True)
    old = tl.set_option(tl.OPT_PEER_TIMEOUT_MS, 50)
    try:
        t0 = time.perf_counter()
        st = L.ternocl_int2_upcvt_allgather(A.data_ptr(), Bs.data_ptr(), Ss.data_ptr(), cptr, None, None, M, N, 0,
                                            nl, K, 0, 0, 0, 0, world, fptr, 0, ws.data_ptr(), ws.numel(),
                                            torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
    finally:
        tl.set_option(tl.OPT_PEER_TIMEOUT_MS, old)
    assert tl.device_error() & 4, "the peer wait did not report its timeout"
    assert 0.04 <= waited < 5.0, waited
    tl.device_error(reset=True)
    assert tl.device_error() == 0
    # rank 0 announced itself to both ranks (call count 1) and stored its columns in both Cs
    assert flags[1].cpu().tolist()[0] == 1 and flags[0].cpu().tolist()[0] == 1
    assert flags[0].cpu().tolist()[world] == 1
    gold = int2_gold_out(c, M, K, N, 0, 0, False)
    for Cr in Cs:
        check_output(host_dt(Cr)[:, :nl], gold[:, :nl], 0, False, "rank 0 columns after the timeout")
    # the context is intact: a regular GEMV runs and matches the oracle
    out = host_dt(tl.int2_upcvt(A, B, S, workspace=tl.Workspace()))
    check_output(out, gold, 0, False, "GEMV after the timeout")
    assert tl.device_error() == 0
