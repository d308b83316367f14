"""Worker bodies for the multi-process (gloo, CPU) tests of ternocl_b200.dist: CPU
stand-ins for the CUDA kernels (numpy, the oracle's routing) so that the sharding and
all-to-all bookkeeping runs without a GPU."""
import os

import numpy as np
import torch
import torch.distributed as dist

from oracle import api as orc
from ternocl_b200 import dist as tdist
from ternocl_b200 import synth


def init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def dequant(B, S, K):
    """int2 words [K/16, N] + fp16 scales -> float64 weights [K, N]."""
    N = B.shape[-1]
    k = np.arange(K)[:, None]
    codes = (B.astype(np.uint32)[k // 16, np.arange(N)[None, :]] >> (2 * (k % 16)).astype(np.uint32)) & 3
    vals = np.array([0.0, 1.0, -2.0, -1.0])[codes]
    return vals * synth.from_dt(S, 0).astype(np.float64)[k // 128, np.arange(N)[None, :]]


def cpu_upcvt(A, B, S, postop=0, other=None, out_f32=False):
    K = A.shape[1]
    c = A.double().numpy() @ dequant(B.numpy().view(np.uint32), S.numpy().view(np.uint16), K)
    if postop == 1:
        c = c / (1.0 + np.exp(-c)) * other.double().numpy()
    return torch.from_numpy(c.astype(np.float32)) if out_f32 else torch.from_numpy(c).half()


class CpuKernels(tdist.Kernels):
    def __init__(self):
        self.route = self._route
        self.gather = lambda X, perm, topk: X[perm.long() // topk].contiguous()
        self.gemm = self._gemm
        self.combine = self._combine

    @staticmethod
    def _route(ids, E):
        meta, perm, inv = orc.moe_route(ids.numpy(), E, 128)
        return torch.from_numpy(meta), torch.from_numpy(perm), torch.from_numpy(inv)

    @staticmethod
    def _gemm(meta, A, B, S, E, postop=0, other=None, out_f32=False):
        m = meta.numpy()
        N = B.shape[-1]
        out = torch.zeros(A.shape[0], N, dtype=torch.float32 if out_f32 else torch.float16)
        for e in range(E):
            r0, r1 = int(m[e]), int(m[e + 1])
            if r1 > r0:
                out[r0:r1] = cpu_upcvt(A[r0:r1], B[e], S[e], postop, other[r0:r1] if other is not None else None,
                                       out_f32)
        return out

    @staticmethod
    def _combine(Y, inv, RW, T, topk):
        w = RW.double().view(T, topk)
        rows = Y.double()[inv.long()].view(T, topk, -1)
        return (rows * w[:, :, None]).sum(1).half()


def moe_problem(seed=3, T=48, topk=4, E=8, H=256, I=128):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(T)]).reshape(-1).astype(np.int32)
    X = torch.from_numpy(synth.activations(rng, T, H, 0).view(np.float16))
    RW = torch.from_numpy(synth.to_dt(rng.random(T * topk), 0).view(np.float16))

    def w(K, N):
        B = np.stack([synth.pack_int2(synth.ternary(rng, K, N)) for _ in range(E)])
        S = np.stack([synth.scales(rng, K, N, 0) for _ in range(E)])
        return torch.from_numpy(B.view(np.int32)), torch.from_numpy(S.view(np.float16))

    Bg, Sg = w(H, I)
    Bu, Su = w(H, I)
    Bd, Sd = w(I, H)
    return dict(ids=torch.from_numpy(ids), X=X, RW=RW, Bg=Bg, Sg=Sg, Bu=Bu, Su=Su, Bd=Bd, Sd=Sd, E=E, topk=topk, T=T)


def moe_worker(rank, world, port, outdir):
    init(rank, world, port)
    p = moe_problem()
    EP, Tl = p["E"] // world, p["T"] // world
    ex = slice(rank * EP, (rank + 1) * EP)
    tok = slice(rank * Tl, (rank + 1) * Tl)
    rows = slice(rank * Tl * p["topk"], (rank + 1) * Tl * p["topk"])
    layer = tdist.ExpertParallelMoE(p["E"], p["topk"], p["Bg"][ex], p["Sg"][ex], p["Bu"][ex], p["Su"][ex],
                                    p["Bd"][ex], p["Sd"][ex], kernels=CpuKernels())
    O = layer(p["X"][tok].contiguous(), p["ids"][rows].contiguous(), p["RW"][rows].contiguous())
    torch.save(O, os.path.join(outdir, "moe_%d.pt" % rank))
    dist.barrier()
    dist.destroy_process_group()


def gemv_worker(rank, world, port, outdir):
    init(rank, world, port)
    rng = np.random.default_rng(11)
    M, K, N = 3, 512, 272  # N / world not a multiple of 16: the last rank takes the rest
    A = torch.from_numpy(synth.activations(rng, M, K, 0).view(np.float16))
    B = torch.from_numpy(synth.pack_int2(synth.ternary(rng, K, N)).view(np.int32))
    S = torch.from_numpy(synth.scales(rng, K, N, 0).view(np.float16))
    n0, nl = tdist.column_shard(N, world, rank)
    C = tdist.sharded_upcvt(A, B[:, n0:n0 + nl].contiguous(), S[:, n0:n0 + nl].contiguous(), N, upcvt=cpu_upcvt)
    torch.save(C, os.path.join(outdir, "gemv_%d.pt" % rank))
    dist.barrier()
    dist.destroy_process_group()


def absent_rank_worker(rank, world, port, tmp):
    """Rank 1 joins the group and then leaves without taking part in the step (it never
    arrives at the all-gather of the sharded GEMV); rank 0's collective must end with an
    error within the group's short timeout instead of waiting for ever."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    dist.barrier()
    if rank != 0:
        return  # leaves between steps: nothing of it is in flight
    rng = np.random.default_rng(11)
    M, K, N = 3, 512, 272
    A = torch.from_numpy(synth.activations(rng, M, K, 0).view(np.float16))
    B = torch.from_numpy(synth.pack_int2(synth.ternary(rng, K, N)).view(np.int32))
    S = torch.from_numpy(synth.scales(rng, K, N, 0).view(np.float16))
    n0, nl = tdist.column_shard(N, world, rank)
    t0 = time.perf_counter()
    outcome = "completed"
    try:
        tdist.sharded_upcvt(A, B[:, n0:n0 + nl].contiguous(), S[:, n0:n0 + nl].contiguous(), N, upcvt=cpu_upcvt)
    except Exception as e:  # gloo: timeout, or the peer's connection closed
        outcome = "error: " + type(e).__name__
    torch.save({"outcome": outcome, "seconds": time.perf_counter() - t0}, os.path.join(tmp, "absent_0.pt"))
