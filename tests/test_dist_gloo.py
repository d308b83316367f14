"""Multi-GPU host logic (ternocl_b200.dist) as 2 gloo ranks on CPU, with CPU stand-ins for
the kernels: the column-sharded GEMV's all-gather assembly and the expert-parallel MoE's
rank routing, count exchange and two all-to-alls must reproduce the single-process
result."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn(fn, world, tmp_path):
    os.environ["PYTHONPATH"] = os.pathsep.join([HERE, os.path.dirname(HERE), os.environ.get("PYTHONPATH", "")])
    mp.spawn(fn, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)


@pytest.fixture(scope="module")
def workers():
    sys.path.insert(0, HERE)
    import dist_workers
    return dist_workers


def test_sharded_gemv_matches_single_rank(workers, tmp_path):
    spawn(workers.gemv_worker, 2, tmp_path)
    C0, C1 = torch.load(tmp_path / "gemv_0.pt"), torch.load(tmp_path / "gemv_1.pt")
    assert torch.equal(C0, C1)  # every rank holds the gathered output
    rng = np.random.default_rng(11)
    from ternocl_b200 import synth
    M, K, N = 3, 512, 272
    A = torch.from_numpy(synth.activations(rng, M, K, 0).view(np.float16))
    B = torch.from_numpy(synth.pack_int2(synth.ternary(rng, K, N)).view(np.int32))
    S = torch.from_numpy(synth.scales(rng, K, N, 0).view(np.float16))
    assert torch.equal(C0, workers.cpu_upcvt(A, B, S))


def test_expert_parallel_moe_matches_single_rank(workers, tmp_path):
    spawn(workers.moe_worker, 2, tmp_path)
    O = torch.cat([torch.load(tmp_path / "moe_0.pt"), torch.load(tmp_path / "moe_1.pt")])
    p = workers.moe_problem()
    from ternocl_b200 import dist as tdist
    ref = tdist.ExpertParallelMoE(p["E"], p["topk"], p["Bg"], p["Sg"], p["Bu"], p["Su"], p["Bd"], p["Sd"],
                                  kernels=workers.CpuKernels())(p["X"], p["ids"], p["RW"])
    assert O.shape == ref.shape
    assert torch.allclose(O.float(), ref.float(), rtol=2e-3, atol=1e-3)


def test_absent_rank_ends_the_collective_with_an_error(workers, tmp_path):
    # failure detection on the host: a rank that never arrives makes the other rank's next
    # collective fail within the process group's timeout (3 s), no hang
    spawn(workers.absent_rank_worker, 2, tmp_path)
    d = torch.load(tmp_path / "absent_0.pt")
    assert d["outcome"].startswith("error"), d
    assert d["seconds"] < 30.0, d


def test_shard_pays_policy():
    # a layer is split over the ranks only where the weight-streaming time it saves per
    # rank exceeds the sharded launch's completion cost; more ranks save more
    from ternocl_b200 import dist as tdist
    assert not tdist.shard_pays(4096, 28672, 1)
    assert not tdist.shard_pays(4096, 28672, 2)  # 31 MB: ~6 us saved per rank, < 10 us
    assert tdist.shard_pays(4096, 28672, 2, completion_us=5.0)
    assert not tdist.shard_pays(4096, 4096, 8)  # 4.5 MB: under 2 us saved
    assert tdist.shard_pays(5120, 248320, 2)  # a 27B lm_head (326 MB): ~65 us saved
    for K, N in [(4096, 6144), (5120, 34816), (17408, 5120)]:
        pays = [tdist.shard_pays(K, N, w) for w in (2, 4, 8)]
        assert pays == sorted(pays)  # once it pays at some world size, it pays at larger ones
