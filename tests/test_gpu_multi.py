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
