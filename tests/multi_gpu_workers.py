"""Bodies of the >= 2-GPU tests (NCCL, one process per GPU): the fused all-gather GEMV
and the expert-parallel MoE with the CUDA kernels, checked against a single-GPU run of the
same problem.  NVLS is off (NCCL_NVLS_ENABLE=0) and the peer mappings are plain CUDA IPC."""
import os

import numpy as np
import torch
import torch.distributed as dist

import ternocl_b200 as tl
from ternocl_b200 import dist as tdist
from ternocl_b200 import synth


def init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))


def fused_gemv_worker(rank, world, port, outdir):
    init(rank, world, port)
    try:
        for (M, K, N, postop) in [(1, 4096, 4096, 0), (3, 1024, 272, 1), (8, 2048, 6144, 3)]:
            rng = np.random.default_rng(M + K + N)
            A = synth.activations(rng, M, K, 0)
            B = synth.pack_int2(synth.ternary(rng, K, N))
            S = synth.scales(rng, K, N, 0)
            other, bias = synth.epilogue_operands(rng, postop, False, M, N, 0)
            dev = torch.device("cuda", rank)
            dA = torch.from_numpy(A.view(np.float16)).to(dev)
            n0, nl = tdist.column_shard(N, world, rank)
            dB = torch.from_numpy(np.ascontiguousarray(B[:, n0:n0 + nl]).view(np.int32)).to(dev)
            dS = torch.from_numpy(np.ascontiguousarray(S[:, n0:n0 + nl]).view(np.float16)).to(dev)
            dO = torch.from_numpy(other.view(np.float16)).to(dev) if other is not None else None
            dBi = torch.from_numpy(bias.view(np.float16)).to(dev) if bias is not None else None
            g = tdist.FusedAllGatherGemv(M, N, K, torch.float16, dev)
            outs = []
            for it in range(3):  # both buffers, and a third call reusing the first
                outs.append(g(dA, dB, dS, postop=postop, other=dO, bias=dBi).clone())
            torch.cuda.synchronize()
            # this rank's columns by the single-GPU entry point on the same shard (same plan)
            shard = tl.int2_upcvt(dA, dB, dS, postop=postop,
                                  other=dO[:, n0:n0 + nl].contiguous() if dO is not None else None,
                                  bias=dBi[n0:n0 + nl].contiguous() if dBi is not None else None)
            err = tl.device_error()
            torch.save(dict(outs=[o.cpu() for o in outs], shard=shard.cpu(), n0=n0, nl=nl, err=err),
                       os.path.join(outdir, "fused_%d_%d_%d_%d.pt" % (M, K, N, rank)))
            g.close()
            dist.barrier()
    finally:
        dist.destroy_process_group()


def ep_moe_worker(rank, world, port, outdir):
    init(rank, world, port)
    try:
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(3)
        T, topk, E, H, I = 256, 4, 8, 256, 384
        ids = np.stack([rng.permutation(E)[:topk] for _ in range(T)]).reshape(-1).astype(np.int32)
        X = synth.activations(rng, T, H, 0)
        RW = synth.to_dt(rng.random(T * topk), 0)

        def w(K, N):
            B = np.stack([synth.pack_int2(synth.ternary(rng, K, N)) for _ in range(E)])
            S = np.stack([synth.scales(rng, K, N, 0) for _ in range(E)])
            return torch.from_numpy(B.view(np.int32)).to(dev), torch.from_numpy(S.view(np.float16)).to(dev)

        Bg, Sg = w(H, I)
        Bu, Su = w(H, I)
        Bd, Sd = w(I, H)
        dX = torch.from_numpy(X.view(np.float16)).to(dev)
        dids = torch.from_numpy(ids).to(dev)
        dRW = torch.from_numpy(RW.view(np.float16)).to(dev)
        EP, Tl = E // world, T // world
        ex, tok, rows = slice(rank * EP, (rank + 1) * EP), slice(rank * Tl, (rank + 1) * Tl), \
            slice(rank * Tl * topk, (rank + 1) * Tl * topk)
        layer = tdist.ExpertParallelMoE(E, topk, Bg[ex].contiguous(), Sg[ex].contiguous(), Bu[ex].contiguous(),
                                        Su[ex].contiguous(), Bd[ex].contiguous(), Sd[ex].contiguous())
        O = layer(dX[tok].contiguous(), dids[rows].contiguous(), dRW[rows].contiguous())
        # the single-GPU layer on the full problem
        meta, perm, inv = tl.moe_route(dids, E)
        Xs = tl.moe_gather(dX, perm, topk)
        up = tl.moe_gemm(meta, Xs, Bu, Su, E)
        Hh = tl.moe_gemm(meta, Xs, Bg, Sg, E, postop=1, other=up)
        Y = tl.moe_gemm(meta, Hh, Bd, Sd, E, out_f32=True)
        ref = tl.moe_combine(Y, inv, dRW, T, topk)
        torch.cuda.synchronize()
        torch.save(dict(O=O.cpu(), ref=ref[tok].cpu()), os.path.join(outdir, "ep_%d.pt" % rank))
        dist.barrier()
    finally:
        dist.destroy_process_group()
