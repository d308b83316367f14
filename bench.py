#!/usr/bin/env python3
"""Benchmark of the ternocl_b200 hot path (one JSON line on rank 0).

Workload (the benchmark's headline configuration): M=1 int2 upconvert GEMV, fp16,
on the four Llama-3-8B decode shapes (K, N) = (4096, 6144), (4096, 4096),
(4096, 28672), (14336, 4096); ternary weights uniform over {-1,0,+1}, group-128
scales uniform [0.01, 0.05], activations N(0, 1); distinct weight sets rotated so
that more than 2 GiB of weights stream (every call reads its weights from HBM, none
from the 126 MB L2).  One step = one GEMV per shape, each on the next weight set.

  value      weight-stream GB/s (B + S bytes / time, all ranks), inputs resident in HBM;
             (one GPU: the K timed steps replayed as one CUDA graph, PDL edges kept;
             --no-graph: host calls with programmatic dependent launch)
  e2e        same metric through the C ABI with host buffers: activations copied
             host->device and outputs device->host inside the timed region
  roofline   the GEMV kernel's weight bytes per launch / its mean launch time vs the
             measured HBM copy bandwidth (MEASURED_PEAKS.json)
  cpu_baseline  the reference's own host gold (compute_gold, compiled from the
             reference sources into oracle/_ref) on the host cores, bounded sample

Secondary figure on the same line (`secondary.prefill`, 1 GPU): the M=2048 int2 fp16
prefill GEMM (tcgen05) on the same four shapes, TFLOP/s (2*M*N*K per GEMM) against the
measured sustained bf16 GEMM peak.  `--workload prefill` makes it the headline instead.
`--workload moe` times the MoE prefill layer, `--workload hadamard` the sign flip + FWHT of
the BITCOS config (rows 1, 8 and 512; HBM GB/s).

With N GPUs (torchrun) the weight columns of every layer are split across the ranks
and the outputs are all-gathered over NCCL inside the timed region (strong scaling).
`--impl reference` times the reference's CPU implementation of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 6144), (4096, 4096), (4096, 28672), (14336, 4096)]  # (K, N), Llama-3-8B
M = 1
WEIGHTS_GIB = 2.0
METRIC = "M=1 int2 GEMV weight-stream HBM GB/s"
WORKLOAD = "llama3-8b decode GEMV sweep, int2_fp16_upcvt, M=1, fp16 (configs[1])"


def weight_bytes(K, N):
    return K * N // 4 + (K // 128) * N * 2


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def peaks_tensor(region_s):
    """Dense bf16 GEMM peak for a timed region of `region_s` seconds: the burst figure
    under a second (the clocks have not settled under the power cap yet), the sustained
    figure for longer regions."""
    burst = region_s < 1.0
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if burst:
            return d["bf16_tflops"], "measured burst"
        return d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured sustained"
    return (1590.0, "fallback burst") if burst else (1400.0, "fallback sustained")


def peaks_int8(region_s):
    """Dense int8 tensor peak: twice the bf16 figure (the nominal dense rates are 4.5 POPS
    int8 against 2.25 PFLOP/s bf16 on B200); no int8 GEMM is measured by the pool."""
    v, kind = peaks_tensor(region_s)
    return 2.0 * v, "2 x %s bf16 GEMM (int8:bf16 nominal dense ratio)" % kind


def time_events(stream, fn, reps):
    """ms per call of fn() (launches on `stream`), CUDA events around `reps` calls."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def device_int2_words(K, N, gen, dev):
    """Uniform ternary int2 words [K/16, N] (codes {0, 1, 3}) generated on the device."""
    import torch
    out = torch.empty(K // 16, N, dtype=torch.int32, device=dev)
    shifts = (2 * torch.arange(16, device=dev, dtype=torch.int64)).view(1, 16, 1)
    rows = max(1, (1 << 24) // (16 * N))
    for r0 in range(0, K // 16, rows):
        r1 = min(K // 16, r0 + rows)
        c = torch.randint(0, 3, (r1 - r0, 16, N), generator=gen, device=dev, dtype=torch.int64)
        c = torch.where(c == 2, torch.full_like(c, 3), c)
        w = (c << shifts).sum(dim=1)
        out[r0:r1] = torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)
    return out


def check(tl, name, st):
    if st != 0:
        raise tl.TernoclError(name, st)


def cpu_loop(fn, budget_s):
    """Runs fn() (one bounded unit of CPU work) until budget_s has passed; returns
    (units done, seconds)."""
    fn()  # warm-up (page-in, thread pool)
    n, el = 0, 0.0
    while el < budget_s:
        t0 = time.perf_counter()
        fn()
        el += time.perf_counter() - t0
        n += 1
    return n, el


def profile_traffic():
    """Per-launch DRAM traffic of the GEMV from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "int2_gemv_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons, active = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU reference arm
class CpuReference:
    """The reference's compute_gold (oracle/_ref: int2_fp16_upcvt/main.cpp:79-98 compiled
    from the reference sources) on this host's cores, on the same workload; falls back
    to the oracle's restatement ("port") where oracle/_ref is absent."""

    def __init__(self):
        from oracle import api as orc
        from ternocl_b200 import synth
        self.threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
        rng = np.random.default_rng(0)
        self.cases = []
        for K, N in SHAPES:
            self.cases.append((synth.activations(rng, M, K, 0), synth.pack_int2(synth.ternary(rng, K, N)),
                               synth.scales(rng, K, N, 0), K, N))
        self.kind = "reference" if orc.ref_available() else "port"
        self.gold = orc.Ref.int2_gold if self.kind == "reference" else orc.int2_gold

    def one_pass(self):
        """One step: one GEMV per shape. Returns seconds."""
        t0 = time.perf_counter()
        for A, B, S, K, N in self.cases:
            self.gold(A, B, S, M, K, N, 0)
        return time.perf_counter() - t0

    def sample(self, budget_s=8.0):
        """(weight GB/s, threads, kind, description) over a bounded number of passes."""
        self.one_pass()
        el, n = 0.0, 0
        while el < budget_s:
            el += self.one_pass()
            n += 1
        gb = n * sum(weight_bytes(K, N) for K, N in SHAPES) / 1e9
        return gb / el, self.threads, self.kind, "%d passes over the 4 shapes, %.1f s, M=1 fp16, seed 0" % (n, el)


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref = CpuReference()
    for _ in range(args.warmup):
        ref.one_pass()
    # bounded: at most ~60 s of timed passes whatever --steps asks
    t_pass = ref.one_pass()
    n = max(1, min(args.steps, int(60.0 / max(t_pass, 1e-6))))
    el = sum(ref.one_pass() for _ in range(n))
    value = n * sum(weight_bytes(K, N) for K, N in SHAPES) / el / 1e9
    desc = "%d of %d requested steps (one GEMV per shape each), %.1f s" % (n, args.steps, el)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
            "n_gpus": args.gpus, "steps": n, "warmup": args.warmup, "ms_per_step": el / n * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic", "config": {"workload": WORKLOAD, "M": M, "shapes_KxN": SHAPES},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": ref.threads, "kind": ref.kind,
                             "sample": desc},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- prefill
PREFILL_M = 2048


def prefill_setup(tl, synth, dev):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    layers = []
    for K, N in SHAPES:
        rng = np.random.default_rng(K * 3 + N)
        B = torch.from_numpy(synth.pack_int2(synth.ternary(rng, K, N)).view(np.int32)).to(dev)
        S = (torch.rand(K // 128, N, generator=g, device=dev) * 0.04 + 0.01).half()
        A = torch.randn(PREFILL_M, K, generator=g, device=dev).half()
        C = torch.empty(PREFILL_M, N, dtype=torch.float16, device=dev)
        layers.append(dict(K=K, N=N, A=A, B=B, S=S, C=C))
    return layers


def prefill_step(tl, L, layers, sp):
    for ly in layers:
        st = L.ternocl_int2_upcvt(ly["A"].data_ptr(), ly["B"].data_ptr(), ly["S"].data_ptr(), ly["C"].data_ptr(),
                                  None, None, PREFILL_M, ly["N"], ly["K"], 0, 0, 0, tl.ALGO_GEMM, None, 0, sp)
        if st != 0:
            raise tl.TernoclError("ternocl_int2_upcvt", st)


def prefill_measure(tl, synth, dev, steps, warmup, profile_range=False):
    """M=2048 int2 prefill GEMMs over the four shapes: (TFLOP/s, ms per step, launches)."""
    import torch
    L = tl.lib()
    layers = prefill_setup(tl, synth, dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    for _ in range(warmup):
        prefill_step(tl, L, layers, sp)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if profile_range:
        torch.cuda.cudart().cudaProfilerStart()
    ev0.record(stream)
    for _ in range(steps):
        prefill_step(tl, L, layers, sp)
    ev1.record(stream)
    torch.cuda.synchronize()
    if profile_range:
        torch.cuda.cudart().cudaProfilerStop()
    ms = ev0.elapsed_time(ev1) / steps
    flops = sum(2.0 * PREFILL_M * N * K for K, N in SHAPES)
    return flops / (ms * 1e-3) / 1e12, ms, steps * len(layers)


# ----------------------------------------------------------------------------- MoE prefill
MOE = dict(T=4096, H=2048, I=768, E=128, topk=8)


def moe_setup(tl, synth, dev, seed=5):
    """C5: 4096 tokens, 128 experts, top-8 distinct uniform, gates softmax(N(0,1)),
    ternary int2 gate/up [E, H/16, I] and down [E, I/16, H], scales U(0.01, 0.05)."""
    import torch
    T, H, I, E, topk = MOE["T"], MOE["H"], MOE["I"], MOE["E"], MOE["topk"]
    rng = np.random.default_rng(seed)
    ids = np.argsort(rng.random((T, E)), axis=1)[:, :topk].astype(np.int32).reshape(-1)
    g = rng.standard_normal((T, topk))
    rw = (np.exp(g) / np.exp(g).sum(1, keepdims=True)).reshape(-1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)

    shifts = (2 * torch.arange(16, device=dev, dtype=torch.int64)).view(1, 16, 1)

    def weights(K, N):
        B = torch.empty(E, K // 16, N, dtype=torch.int32, device=dev)
        for e in range(E):  # uniform {0, +1, -1} -> codes {0, 1, 3}, 16 per word
            codes = torch.randint(0, 3, (K // 16, 16, N), generator=gen, device=dev, dtype=torch.int64)
            codes = torch.where(codes == 2, torch.full_like(codes, 3), codes)
            w = (codes << shifts).sum(dim=1)
            B[e] = torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)
        S = (torch.rand(E, K // 128, N, generator=gen, device=dev) * 0.04 + 0.01).half()
        return B, S

    Bg, Sg = weights(H, I)
    Bu, Su = weights(H, I)
    Bd, Sd = weights(I, H)
    G = T * topk
    return dict(ids=torch.from_numpy(ids).to(dev), RW=torch.from_numpy(rw).half().to(dev),
                X=torch.randn(T, H, generator=gen, device=dev).half(), Bg=Bg, Sg=Sg, Bu=Bu, Su=Su, Bd=Bd, Sd=Sd,
                Xs=torch.empty(G, H, dtype=torch.float16, device=dev),
                up=torch.empty(G, I, dtype=torch.float16, device=dev),
                Hh=torch.empty(G, I, dtype=torch.float16, device=dev),
                Y=torch.empty(G, H, dtype=torch.float32, device=dev),
                O=torch.empty(T, H, dtype=torch.float16, device=dev))


def moe_layer(tl, m, stream=None):
    """route -> gather -> up, gate (SiLU-mul with up), down (fp32) -> combine: 6 launches."""
    E, topk = MOE["E"], MOE["topk"]
    meta, perm, inv = tl.moe_route(m["ids"], E, stream=stream)
    tl.moe_gather(m["X"], perm, topk, out=m["Xs"], stream=stream)
    tl.moe_gemm(meta, m["Xs"], m["Bu"], m["Su"], E, out=m["up"], stream=stream)
    tl.moe_gemm(meta, m["Xs"], m["Bg"], m["Sg"], E, postop=1, other=m["up"], out=m["Hh"], stream=stream)
    tl.moe_gemm(meta, m["Hh"], m["Bd"], m["Sd"], E, out_f32=True, out=m["Y"], stream=stream)
    tl.moe_combine(m["Y"], inv, m["RW"], MOE["T"], topk, out=m["O"], stream=stream)


def moe_measure(tl, synth, dev, steps, warmup, cpu=True):
    """(tokens/s, TFLOP/s, ms per layer, e2e dict, cpu_baseline dict) of the C5 MoE prefill
    layer; e2e: the tokens copied in from pinned host memory and the layer output copied
    back every step."""
    import torch
    m = moe_setup(tl, synth, dev)
    for _ in range(warmup):
        moe_layer(tl, m)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        moe_layer(tl, m)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    G = MOE["T"] * MOE["topk"]
    flops = 2.0 * G * (2 * MOE["H"] * MOE["I"] + MOE["I"] * MOE["H"])
    hX = m["X"].cpu().pin_memory()
    hO = torch.empty(m["O"].shape, dtype=m["O"].dtype).pin_memory()
    t0 = time.perf_counter()
    for _ in range(steps):
        m["X"].copy_(hX, non_blocking=True)
        moe_layer(tl, m)
        hO.copy_(m["O"], non_blocking=True)
        stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / steps
    e2e = {"value": MOE["T"] / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": hX.numel() * 2,
           "d2h_bytes_per_step": hO.numel() * 2}
    return MOE["T"] / (ms * 1e-3), flops / (ms * 1e-3) / 1e12, ms, e2e, (moe_cpu_baseline(m) if cpu else None)


def run_moe(args, tl, synth, dev, world, rank, local):
    """--workload moe: the C5 layer; on N GPUs expert-parallel (E/N experts and T/N
    tokens per rank, NCCL all-to-all of the routed rows; strong scaling)."""
    import torch
    import torch.distributed as dist
    from ternocl_b200 import dist as tdist
    m = moe_setup(tl, synth, dev)  # every rank builds the same problem, keeps its share
    E, topk, T = MOE["E"], MOE["topk"], MOE["T"]
    if world > 1:
        EP, Tl = E // world, T // world
        ex, tok = slice(rank * EP, (rank + 1) * EP), slice(rank * Tl, (rank + 1) * Tl)
        rows = slice(rank * Tl * topk, (rank + 1) * Tl * topk)
        layer = tdist.ExpertParallelMoE(E, topk, m["Bg"][ex].contiguous(), m["Sg"][ex].contiguous(),
                                        m["Bu"][ex].contiguous(), m["Su"][ex].contiguous(), m["Bd"][ex].contiguous(),
                                        m["Sd"][ex].contiguous())
        X, ids, RW = m["X"][tok].contiguous(), m["ids"][rows].contiguous(), m["RW"][rows].contiguous()
        run = lambda: layer(X, ids, RW)
    else:
        X = m["X"]
        run = lambda: moe_layer(tl, m)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        run()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        if args.profile_range:
            torch.cuda.cudart().cudaProfilerStart()
        ev0.record(stream)
        for _ in range(args.steps):
            run()
        ev1.record(stream)
        barrier()
        if args.profile_range:
            torch.cuda.cudart().cudaProfilerStop()
    ms = ev0.elapsed_time(ev1) / args.steps
    # end to end: tokens in from pinned host memory, layer output back every step
    hX = X.cpu().pin_memory()
    hO = torch.empty(X.shape, dtype=X.dtype).pin_memory()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        X.copy_(hX, non_blocking=True)
        O = run()
        hO.copy_(O if O is not None else m["O"], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    barrier()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    G = T * topk
    flops = 2.0 * G * (2 * MOE["H"] * MOE["I"] + MOE["I"] * MOE["H"])
    pk = peaks_tensor(ms * args.steps * 1e-3)
    if rank == 0:
        # one GPU: route, gather, 3 grouped GEMMs, combine; expert-parallel: route and
        # gather twice (by owning rank, then by local expert)
        launches = 6 if world == 1 else 8
        line = {"metric": "MoE prefill tokens/s", "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
                "config": {"workload": "int2 MoE prefill layer (configs[4])", **MOE,
                           "l2": "inputs larger than L2: ~650 MB of weights, routed rows and intermediates",
                           "parallelism": "expert-parallel x%d, NCCL all-to-all" % world if world > 1 else "single GPU"},
                "roofline": {"bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12 / world, "peak": pk[0],
                             "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / world / pk[0],
                             "peak_kind": pk[1], "kernel": "gemm_kernel<Int2Gemm, HALVES> (grouped)",
                             "traffic": None},
                "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": hX.numel() * 2 * world,
                        "d2h_bytes_per_step": hO.numel() * 2 * world},
                "gpu_launches": launches * args.steps, "clocks": clk.summary(),
                "cpu_baseline": moe_cpu_baseline(m) if world == 1 and not args.no_cpu_baseline else None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_prefill(args, tl, synth, dev, world, rank, local):
    """--workload prefill: the M=2048 GEMMs as the headline (replicas on N GPUs: weak scaling)."""
    import torch
    import torch.distributed as dist
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier(device_ids=[local])
        tf, ms, launches = prefill_measure(tl, synth, dev, args.steps, args.warmup, args.profile_range)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = sum(2.0 * PREFILL_M * N * K for K, N in SHAPES)
    value = world * flops / (ms * 1e-3) / 1e12
    pk = peaks_tensor(ms * args.steps * 1e-3)
    if rank == 0:
        line = {"metric": "M=2048 int2 fp16 prefill TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
                "config": {"workload": "int2_fp16_upcvt prefill GEMM (M-tiled), M=2048, llama3-8b shapes",
                           "M": PREFILL_M, "shapes_KxN": SHAPES,
                           "l2": "inputs larger than L2: one step touches ~340 MB (A, B, S, C of 4 shapes)",
                           "parallelism": "replicas x%d" % world if world > 1 else "single GPU"},
                "roofline": {"bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12, "peak": pk[0],
                             "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / pk[0], "peak_kind": pk[1],
                             "kernel": "gemm_kernel<Int2Gemm>", "traffic": None},
                "gpu_launches": launches, "clocks": clk.summary(), "cpu_baseline": None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- Hadamard
# The BITCOS config's pre-transform: K = 5376 with HB = 256, the largest power-of-two
# block dividing K (the config's HB = 1024 does not divide 5376), fp16, sign flip on.
HAD = dict(K=5376, HB=256, rows=(1, 8, 512))
HAD_SET_BYTES = 256 << 20  # distinct input rows streamed per row count (2x the L2)


def run_hadamard(args, tl, synth, dev, world, rank, local):
    """--workload hadamard: ternocl_hadamard_fwht at rows 1, 8 and 512.  One step = one
    call per row count, each on the next of enough distinct input sets to stream
    HAD_SET_BYTES, so no set is read from L2 again.  Bytes per call (algorithmic):
    rows*K*2 read + rows*K*2 written + K sign bytes.  One GPU: each row count's K timed
    calls are one CUDA-graph replay (the first replay, which uploads the graph, untimed).
    N GPUs: independent replicas (weak scaling), time = max over ranks."""
    import torch
    import torch.distributed as dist
    K, HB = HAD["K"], HAD["HB"]
    rng = np.random.default_rng(11)
    signs = torch.from_numpy(np.where(rng.random(K) < 0.5, -1, 1).astype(np.int8)).to(dev)
    stream = torch.cuda.current_stream(dev)
    per = []  # (rows, bytes per call, ms per call)
    with ClockSampler(local) as clk:
        for rows in HAD["rows"]:
            nsets = max(1, -(-HAD_SET_BYTES // (rows * K * 2)))
            X = torch.randn(nsets * rows, K, device=dev, dtype=torch.float16)
            Y = torch.empty_like(X)

            def call(i, cs=None):
                s = (i % nsets) * rows
                tl.hadamard_fwht(X[s:s + rows], HB, signs, out=Y[s:s + rows], stream=cs)

            for i in range(args.warmup):
                call(nsets - 1 - i % nsets)
            torch.cuda.synchronize()
            graph = None
            if world == 1 and args.graph:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    cs = torch.cuda.current_stream(dev).cuda_stream
                    for i in range(args.steps):
                        call(i, cs)
                graph.replay()  # upload
                torch.cuda.synchronize()
            if world > 1:
                dist.barrier(device_ids=[local])
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if args.profile_range:
                torch.cuda.cudart().cudaProfilerStart()
            ev0.record(stream)
            if graph is not None:
                graph.replay()
            else:
                for i in range(args.steps):
                    call(i)
            ev1.record(stream)
            torch.cuda.synchronize()
            if args.profile_range:
                torch.cuda.cudart().cudaProfilerStop()
            ms = ev0.elapsed_time(ev1) / args.steps
            if world > 1:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            per.append((rows, 2 * rows * K * 2 + K, ms))
            del graph, X, Y
            torch.cuda.empty_cache()
    step_bytes = sum(b for _, b, _ in per)
    step_ms = sum(ms for _, _, ms in per)
    peak, peak_kind = peaks()
    rows_d, bytes_d, ms_d = max(per, key=lambda p: p[2])  # the dominant launch
    traffic = None  # DRAM bytes per 512-row launch from the committed ncu summary
    tp = os.path.join(ROOT, "profiles", "hadamard_traffic.json")
    if rows_d == 512 and os.path.exists(tp):
        with open(tp) as f:
            tb = json.load(f)["dram_bytes_per_launch"]
        traffic = sum(tb) / len(tb)
    if rank == 0:
        line = {"metric": "Hadamard sign flip + FWHT HBM GB/s", "value": world * step_bytes / (step_ms * 1e-3) / 1e9,
                "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
                "data": "synthetic",
                "config": {"workload": "hadamard_fwht of the BITCOS config (configs[3]): K=5376, HB=256, signs",
                           "rows": list(HAD["rows"]),
                           "l2": "inputs larger than L2: %d MiB of distinct rows per row count" % (HAD_SET_BYTES >> 20),
                           "parallelism": "replicas x%d" % world if world > 1 else "single GPU",
                           "per_rows": [{"rows": r, "us_per_call": ms * 1e3, "GBps": b / (ms * 1e-3) / 1e9}
                                        for r, b, ms in per]},
                "roofline": {"bound": "hbm", "achieved": bytes_d / (ms_d * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": bytes_d / (ms_d * 1e-3) / 1e9 / peak, "peak_kind": peak_kind,
                             "kernel": "hadamard_fwht (rows=%d)" % rows_d, "traffic": traffic},
                "gpu_launches": args.steps * len(per), "clocks": clk.summary(), "cpu_baseline": None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- C3: s8 x s2 prefill
# bf16 activations quantised per row and 128-group (ternocl_int8_quant_a), then
# the s8 x s2 GEMM with int32 accumulation; the quantisation pre-kernel is inside the timed
# region, as the reference driver times `pre` + `gemm` (int2_via_int2_x_int8_dpas/main.cpp:368-387).
INT8 = dict(shapes=[(5376, 21504), (21504, 5376), (5376, 5376)], M=2048)
INT8_METRIC = "M=2048 s8xs2 prefill TFLOP/s (quant_a + GEMM, 27B-like shapes)"


def int8_measure(tl, dev, steps, warmup, cpu=True, e2e=True):
    import torch
    L = tl.lib()
    M = INT8["M"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(31)
    ka = [K * M for K, _ in INT8["shapes"]]
    kc = [N * M for _, N in INT8["shapes"]]
    dA = torch.randn(sum(ka), generator=gen, device=dev).bfloat16()
    dC = torch.empty(sum(kc), dtype=torch.bfloat16, device=dev)
    oa, oc = np.cumsum([0] + ka), np.cumsum([0] + kc)
    ly = []
    for j, (K, N) in enumerate(INT8["shapes"]):
        ly.append(dict(K=K, N=N, B=device_int2_words(K, N, gen, dev),
                       SB=(torch.rand(K // 128, N, generator=gen, device=dev) * 0.04 + 0.01).bfloat16(),
                       A=dA[oa[j]:oa[j + 1]].view(M, K), C=dC[oc[j]:oc[j + 1]].view(M, N),
                       SA=torch.zeros(K // 128, (M + 31) & ~31, dtype=torch.bfloat16, device=dev),
                       Aq=torch.empty(M, K, dtype=torch.int8, device=dev)))
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def pre(x):
        check(tl, "ternocl_int8_quant_a", L.ternocl_int8_quant_a(x["A"].data_ptr(), x["SA"].data_ptr(),
                                                                x["Aq"].data_ptr(), M, x["K"], 1, sp))

    def gemm(x):
        check(tl, "ternocl_int2_int8", L.ternocl_int2_int8(x["A"].data_ptr(), x["Aq"].data_ptr(), x["SA"].data_ptr(),
                                                           x["B"].data_ptr(), x["SB"].data_ptr(), x["C"].data_ptr(),
                                                           None, None, M, x["N"], x["K"], 1, 0, 0, 0, 0, sp))

    def step():
        for x in ly:
            pre(x)
            gemm(x)

    # qmode 1, the reference driver's default scheme (main.cpp:58): the pre-kernel writes
    # the scales only and the GEMM call quantises A from them (one pass into pooled scratch)
    def step_q1():
        for x in ly:
            check(tl, "ternocl_int8_quant_a", L.ternocl_int8_quant_a(x["A"].data_ptr(), x["SA"].data_ptr(), None,
                                                                    M, x["K"], 1, sp))
            check(tl, "ternocl_int2_int8", L.ternocl_int2_int8(x["A"].data_ptr(), None, x["SA"].data_ptr(),
                                                               x["B"].data_ptr(), x["SB"].data_ptr(),
                                                               x["C"].data_ptr(), None, None, M, x["N"], x["K"], 1,
                                                               0, 0, 1, 0, sp))

    for _ in range(warmup):
        step()
        step_q1()
    t_step = time_events(stream, step, steps)
    t_step_q1 = time_events(stream, step_q1, steps)
    t_pre = time_events(stream, lambda: [pre(x) for x in ly], steps)
    t_gemm = time_events(stream, lambda: [gemm(x) for x in ly], steps)
    flops = sum(2.0 * M * N * K for K, N in INT8["shapes"])
    tf, tf_gemm = flops / (t_step * 1e-3) / 1e12, flops / (t_gemm * 1e-3) / 1e12
    peak, kind = peaks_int8(t_gemm * steps * 1e-3)
    out = {"metric": INT8_METRIC, "value": tf, "unit": "TFLOP/s", "ms_per_step": t_step, "dtype": "bf16",
           "config": {"workload": "int2_via_int2_x_int8_dpas prefill (configs[2]): quant_a + s8xs2 GEMM, bf16",
                      "M": M, "shapes_KxN": INT8["shapes"], "qmode": 0,
                      "l2": "inputs larger than L2: one step touches ~400 MB (A, Aq, B, C of 3 shapes)"},
           "pre_ms": t_pre, "gemm_ms": t_gemm,
           "qmode1": {"ms_per_step": t_step_q1, "value": flops / (t_step_q1 * 1e-3) / 1e12,
                      "note": "scales pre-kernel + GEMM quantising from SA (quant pass + int8 GEMM per shape)"},
           "roofline": {"bound": "tensor", "achieved": tf_gemm, "peak": peak, "unit": "TFLOP/s",
                        "frac": tf_gemm / peak, "peak_kind": kind, "kernel": "gemm_i8 (tcgen05 kind::i8), GEMM alone",
                        "traffic": None},
           "gpu_launches": 2 * len(ly) * steps, "cpu_baseline": None, "e2e": None}
    if e2e:
        hA = dA.cpu().pin_memory()
        hC = torch.empty(dC.shape, dtype=dC.dtype).pin_memory()
        n = max(3, min(steps, 10))
        for _ in range(2):
            dA.copy_(hA, non_blocking=True)
            step()
            hC.copy_(dC, non_blocking=True)
            stream.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            dA.copy_(hA, non_blocking=True)
            step()
            hC.copy_(dC, non_blocking=True)
            stream.synchronize()
        es = (time.perf_counter() - t0) / n
        out["e2e"] = {"value": flops / es / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": hA.numel() * 2,
                      "d2h_bytes_per_step": hC.numel() * 2}
    if cpu:
        from oracle import api as orc
        R = orc.Ref if orc.ref_available() else None
        rows = 2
        host = []
        for x in ly:
            A = x["A"][:rows].cpu().view(torch.int16).numpy().view(np.uint16)
            host.append((A, x["B"].cpu().numpy().view(np.uint32), x["SB"].cpu().view(torch.int16).numpy().view(np.uint16),
                         x["K"], x["N"]))

        def one():
            for A, B, SB, K, N in host:
                if R is not None:
                    SA = R.int8_scale_a(A, rows, K, 1)
                    R.int8_gold(A, B, SA, SB, rows, K, N, 1)
                else:
                    SA = orc.int8_scale_a(A, rows, K, 1)
                    orc.int8_gold(A, B, SA, SB, rows, K, N, 1)

        nrun, el = cpu_loop(one, 8.0)
        cflops = nrun * sum(2.0 * rows * N * K for K, N in INT8["shapes"])
        out["cpu_baseline"] = {"value": cflops / el / 1e12, "unit": "TFLOP/s",
                               "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
                               "kind": "reference" if R is not None else "port",
                               "sample": "%d passes of compute_scale_a + compute_gold on %d rows of each of the 3 "
                                         "shapes (M=2048 workload), %.1f s" % (nrun, rows, el)}
    return out


# ----------------------------------------------------------------------------- C4: BITCOS + Hadamard
# K=5376, N=21504, zero fraction z in {0.2, 0.35, 0.5}, M in {1, 8, 512}, fp16; the
# activations go through the sign flip + FWHT (HB=256: the config's 1024 does not divide 5376)
# and then the BITCOS GEMV (M <= 8; at M <= 4 in one launch, ternocl_bitcos_upcvt_hadamard,
# both timings recorded) or the M-tiled GEMM (M = 512: hadamard_fwht, then the GEMM).  Bytes as the reference's
# model (bitcos_fp16_upcvt/main.cpp:286-300): the BITCOS buffer + scales (+ A and C).
BITCOS = dict(K=5376, N=21504, z=(0.2, 0.35, 0.5), M=(1, 8, 512), HB=256, sets=3)
BITCOS_METRIC = "M=1 BITCOS GEMV weight-stream HBM GB/s (Hadamard pre-transform included, K=5376 N=21504)"


def bitcos_measure(tl, dev, steps, warmup, cpu=True, e2e=True):
    import torch
    L = tl.lib()
    K, N, HB = BITCOS["K"], BITCOS["N"], BITCOS["HB"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(41)
    rng = np.random.default_rng(41)
    host_bufs, bufs, srs, S = {}, {}, {}, {}
    LS = 4
    while LS > 1 and K % (64 * LS):
        LS //= 2
    for zi, z in enumerate(BITCOS["z"]):
        host_bufs[z] = [tl.bitcos_random(K, N, z, 100 * zi + k) for k in range(BITCOS["sets"])]
        bufs[z] = [torch.from_numpy(b.view(np.int32)).to(dev) for b in host_bufs[z]]
        # slice ranks at the reference driver's default LS = 4 (bitcos_fp16_upcvt/main.cpp:122-123,194)
        srs[z] = [torch.from_numpy(tl.bitcos_slice_ranks(b, K, N, LS).view(np.int32)).to(dev) for b in host_bufs[z]]
        S[z] = (torch.rand(K // 128, N, generator=gen, device=dev) * 0.04 + 0.01).half()
    signs_h = np.where(rng.random(K) < 0.5, -1, 1).astype(np.int8)
    signs = torch.from_numpy(signs_h).to(dev)
    A = {M: torch.randn(M, K, generator=gen, device=dev).half() for M in BITCOS["M"]}
    Y = {M: torch.empty(M, K, dtype=torch.float16, device=dev) for M in BITCOS["M"]}
    C = {M: torch.empty(M, N, dtype=torch.float16, device=dev) for M in BITCOS["M"]}
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def had(M):
        check(tl, "ternocl_hadamard_fwht", L.ternocl_hadamard_fwht(A[M].data_ptr(), signs.data_ptr(), Y[M].data_ptr(),
                                                                   M, K, HB, 1, 0, sp))

    def gemv(M, z, i):
        check(tl, "ternocl_bitcos_upcvt", L.ternocl_bitcos_upcvt(Y[M].data_ptr(), bufs[z][i].data_ptr(),
                                                                 S[z].data_ptr(), srs[z][i].data_ptr(), LS,
                                                                 C[M].data_ptr(), None, None, M, N, K, 0, 0, 0, 0, sp))

    def fused(M, z, i):
        # the transform and the GEMV in one launch (the strip kernel at M <= 8)
        check(tl, "ternocl_bitcos_upcvt_hadamard",
              L.ternocl_bitcos_upcvt_hadamard(A[M].data_ptr(), signs.data_ptr(), 1, HB, bufs[z][i].data_ptr(),
                                              S[z].data_ptr(), srs[z][i].data_ptr(), LS, C[M].data_ptr(), None, None,
                                              M, N, K, 0, 0, 0, sp))

    per = []
    for M in BITCOS["M"]:
        for z in BITCOS["z"]:
            ctr = [0]

            def two_kernels(M=M, z=z):
                had(M)
                gemv(M, z, ctr[0] % BITCOS["sets"])
                ctr[0] += 1

            def one_launch(M=M, z=z):
                fused(M, z, ctr[0] % BITCOS["sets"])
                ctr[0] += 1

            # one launch where it measured faster (M = 1: 32.9 against 36.7 us); at M = 8 each
            # CTA's transform of 8 rows costs more than the standalone kernel (41.0 against 39.8)
            pipeline = one_launch if M <= 4 else two_kernels

            def alone(M=M, z=z):
                gemv(M, z, ctr[0] % BITCOS["sets"])
                ctr[0] += 1

            reps = steps if M < 512 else max(3, steps // 10)
            for _ in range(warmup):
                pipeline()
            t_pipe = time_events(stream, pipeline, reps)
            t_two = time_events(stream, two_kernels, reps) if pipeline is one_launch else t_pipe
            t_one = time_events(stream, one_launch, reps) if M <= 8 and pipeline is not one_launch else t_pipe
            t_gemv = time_events(stream, alone, reps)
            wbytes = host_bufs[z][0].size * 4 + (K // 128) * N * 2
            per.append(dict(M=M, z=z, us_per_call=t_pipe * 1e3, two_kernel_us=t_two * 1e3,
                            one_launch_us=t_one * 1e3 if M <= 8 else None, gemv_us=t_gemv * 1e3,
                            launch="fused transform + GEMV" if M <= 4 else
                            "hadamard_fwht, then GEMV" if M <= 8 else "hadamard_fwht, then GEMM",
                            weight_bytes=wbytes,
                            GBps=wbytes / (t_pipe * 1e-3) / 1e9 if M <= 8 else None,
                            TFLOPs=2.0 * M * N * K / (t_pipe * 1e-3) / 1e12))
    m1 = [q for q in per if q["M"] == 1]
    value = sum(q["weight_bytes"] for q in m1) / (sum(q["us_per_call"] for q in m1) * 1e-6) / 1e9
    mid = [q for q in m1 if q["z"] == 0.35][0]
    ach = mid["weight_bytes"] / (mid["gemv_us"] * 1e-6) / 1e9
    peak, peak_kind = peaks()
    out = {"metric": BITCOS_METRIC, "value": value, "unit": "GB/s", "ms_per_step": sum(q["us_per_call"] for q in m1) / 1e3,
           "dtype": "fp16",
           "config": {"workload": "bitcos_fp16_upcvt + hadamard_fwht (configs[3])", "K": K, "N": N, "HB": HB, "LS": LS,
                      "z": list(BITCOS["z"]), "M": list(BITCOS["M"]),
                      "l2": "inputs larger than L2: %d BITCOS buffers (~%d MB) rotated per call" % (
                          len(BITCOS["z"]) * BITCOS["sets"], sum(b.size * 4 for z in BITCOS["z"] for b in host_bufs[z]) >> 20),
                      "per_call": per},
           "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                        "peak_kind": peak_kind, "kernel": "bitcos GEMV, M=1, z=0.35 (alone)", "traffic": None},
           "gpu_launches": steps * len(m1), "cpu_baseline": None, "e2e": None}
    if e2e:
        hA = A[1].cpu().pin_memory()
        hC = torch.empty(1, N, dtype=torch.float16).pin_memory()
        n, tot, t0 = 0, 0.0, time.perf_counter()
        for it in range(steps):
            for z in BITCOS["z"]:
                A[1].copy_(hA, non_blocking=True)
                fused(1, z, it % BITCOS["sets"])
                hC.copy_(C[1], non_blocking=True)
                stream.synchronize()
                tot += host_bufs[z][0].size * 4 + (K // 128) * N * 2
        es = time.perf_counter() - t0
        out["e2e"] = {"value": tot / es / 1e9, "unit": "GB/s", "h2d_bytes_per_step": hA.numel() * 2 * len(BITCOS["z"]),
                      "d2h_bytes_per_step": hC.numel() * 2 * len(BITCOS["z"])}
    if cpu:
        from oracle import api as orc
        R = orc.Ref if orc.ref_available() else None
        Ah = A[1].cpu().view(torch.int16).numpy().view(np.uint16)
        Sh = {z: S[z].cpu().view(torch.int16).numpy().view(np.uint16) for z in BITCOS["z"]}

        def one():
            for z in BITCOS["z"]:
                if R is not None:
                    y = R.hadamard(Ah, signs_h, 1, K, HB, 1, 0)
                    R.bitcos_gold(y, host_bufs[z][0], Sh[z], 1, K, N, 0)
                else:
                    y = orc.hadamard(Ah, signs_h, 1, K, HB, 1, 0)
                    orc.bitcos_gold(y, host_bufs[z][0], Sh[z], 1, K, N, 0)

        nrun, el = cpu_loop(one, 8.0)
        cb = nrun * sum(host_bufs[z][0].size * 4 + (K // 128) * N * 2 for z in BITCOS["z"])
        out["cpu_baseline"] = {"value": cb / el / 1e9, "unit": "GB/s",
                               "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
                               "kind": "reference" if R is not None else "port",
                               "sample": "%d passes of the hadamard_fwht kernel source run on the CPU + the BITCOS "
                                         "compute_gold at M=1 over the three z, %.1f s" % (nrun, el)}
    return out


# M=1 decode GEMV shapes of the reference's published table (int2_fp16_upcvt/README.md,
# "Decode GEMV, M = 1"): name, K, N, the reference's published OpenCL time on Arc Pro B70 (us)
README_GEMV_SHAPES = [("8B qkv", 4096, 6144, 14.39), ("8B o_proj", 4096, 4096, 10.35),
                      ("8B gate_up", 4096, 24576, 47.23), ("8B down", 12288, 4096, 25.19),
                      ("8B lm_head", 4096, 151680, 278.9), ("27B gate_up", 5120, 34816, 86.81),
                      ("27B down", 17408, 5120, 42.76), ("27B in_proj_qkvz", 5120, 16384, 40.05),
                      ("27B out_proj", 6144, 5120, 17.16), ("27B qkv", 5120, 14336, 35.54),
                      ("27B lm_head", 5120, 248320, 572.5)]


def gemv_shapes_measure(tl, dev, reps=20, cpu=True):
    """M=1 fp16 int2 GEMV per shape of the reference's published table: back-to-back
    launches of one shape in a CUDA graph over weight sets rotated past L2 (>= 400 MB),
    us per call, weight GB/s and its fraction of the measured HBM peak; the o_proj shape
    is configs[0] (M=1, K=N=4096, the host-reference config), timed also with the
    reference's own host gold (oracle/_ref) on this host's cores."""
    import torch
    L = tl.lib()
    peak, peak_kind = peaks()
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    out = []
    c1 = None
    for name, K, N, b70 in README_GEMV_SHAPES:
        wb = weight_bytes(K, N)
        nsets = max(2, int(np.ceil(400e6 / wb)))
        B0 = device_int2_words(K, N, gen, dev)
        Bs = [B0] + [B0.view(-1)[torch.randperm(B0.numel(), generator=gen, device=dev)].view_as(B0).contiguous()
                     for _ in range(nsets - 1)]
        Ss = [(torch.rand(K // 128, N, generator=gen, device=dev) * 0.04 + 0.01).half() for _ in range(nsets)]
        A = torch.randn(1, K, generator=gen, device=dev).half()
        C = torch.empty(1, N, dtype=torch.float16, device=dev)
        ws = tl.Workspace(dev, tl.gemv_workspace_size(1, N, K))

        def call(i, cs):
            check(tl, "ternocl_int2_upcvt", L.ternocl_int2_upcvt(A.data_ptr(), Bs[i % nsets].data_ptr(),
                                                                 Ss[i % nsets].data_ptr(), C.data_ptr(), None, None,
                                                                 1, N, K, 0, 0, 0, tl.ALGO_GEMV, ws.ptr(), ws.nbytes(),
                                                                 cs))
        torch.cuda.synchronize()
        for i in range(nsets):
            call(i, torch.cuda.current_stream(dev).cuda_stream)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for i in range(reps):
                call(i, torch.cuda.current_stream(dev).cuda_stream)
        gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        gbs = wb / (us * 1e-6) / 1e9
        out.append({"shape": name, "K": K, "N": N, "us": us, "GBps": gbs, "frac": gbs / peak,
                    "reference_b70_us": b70, "speedup_vs_reference_b70": b70 / us})
        del gr, Bs, Ss, B0
        torch.cuda.empty_cache()
        if (K, N) == (4096, 4096):
            c1 = {"metric": "M=1 int2 GEMV weight-stream HBM GB/s (configs[0]: K=N=4096, fp16)", "value": gbs,
                  "unit": "GB/s", "us_per_call": us,
                  "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                               "peak_kind": peak_kind}, "cpu_baseline": None}
    if cpu and c1 is not None:
        from oracle import api as orc
        from ternocl_b200 import synth
        rng = np.random.default_rng(0)
        A0, B0, S0 = (synth.activations(rng, 1, 4096, 0), synth.pack_int2(synth.ternary(rng, 4096, 4096)),
                      synth.scales(rng, 4096, 4096, 0))
        kind = "reference" if orc.ref_available() else "port"
        gold = orc.Ref.int2_gold if kind == "reference" else orc.int2_gold
        n, el = cpu_loop(lambda: gold(A0, B0, S0, 1, 4096, 4096, 0), 3.0)
        c1["cpu_baseline"] = {"value": n * weight_bytes(4096, 4096) / el / 1e9, "unit": "GB/s",
                              "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)), "kind": kind,
                              "sample": "%d calls of compute_gold at M=1, K=N=4096, seed 0, %.1f s" % (n, el)}
    return out, c1


def moe_cpu_baseline(m, budget_s=8.0):
    """The MoE layer's token reference (int2_moe/prefill.cpp:291-310, double precision; the
    restatement, pinned through its parts) on the host cores: tokens/s over a bounded
    number of tokens of the same workload."""
    import torch
    from oracle import api as orc

    def h16(t):
        return t.cpu().view(torch.int16).numpy().view(np.uint16)

    def h32(t):
        return t.cpu().numpy().view(np.uint32)

    X, RW, ids = h16(m["X"]), h16(m["RW"]), m["ids"].cpu().numpy()
    W = [h32(m["Bg"]), h16(m["Sg"]), h32(m["Bu"]), h16(m["Su"]), h32(m["Bd"]), h16(m["Sd"])]
    tok = [0]

    def one():
        orc.moe_token_ref(X, ids, RW, *W, tok[0] % MOE["T"], MOE["topk"], MOE["H"], MOE["I"], 0)
        tok[0] += 1

    n, el = cpu_loop(one, budget_s)
    return {"value": n / el, "unit": "tokens/s", "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
            "kind": "port", "sample": "%d tokens of the double-precision token reference, %.1f s" % (n, el)}


def emit(args, line, clocks, world=1):
    """Prints a secondary measurement as its own JSON line (--workload int8 / bitcos)."""
    full = {"metric": line["metric"], "value": line["value"], "unit": line["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": line["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": line["dtype"], "data": "synthetic",
            "config": dict(line["config"], parallelism="replicas x%d" % world if world > 1 else "single GPU"),
            "roofline": line["roofline"], "e2e": line["e2e"], "gpu_launches": line["gpu_launches"],
            "clocks": clocks, "cpu_baseline": line["cpu_baseline"]}
    for k in ("pre_ms", "gemm_ms", "qmode1"):
        if k in line:
            full[k] = line[k]
    print(json.dumps(full), flush=True)


def run_replicated(args, tl, dev, world, rank, local):
    """--workload int8 / bitcos: configs[2] / configs[3] as the line; N GPUs run replicas
    (weak scaling), the time per step is the max over ranks."""
    import torch
    import torch.distributed as dist
    fn = int8_measure if args.workload == "int8" else bitcos_measure
    cpu = world == 1 and not args.no_cpu_baseline
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier(device_ids=[local])
        line = fn(tl, dev, args.steps, args.warmup, cpu=cpu, e2e=True)
    if world > 1:
        t = torch.tensor([line["ms_per_step"]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        scale = line["ms_per_step"] / float(t.item())
        line["value"] *= world * scale
        line["ms_per_step"] = float(t.item())
    if rank == 0:
        emit(args, line, clk.summary(), world)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed region with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "int8", "bitcos", "moe", "hadamard"],
                    help="decode: the headline M=1 GEMV sweep (+ the other configs as secondary figures); "
                         "prefill: the int2 fp16 M=2048 GEMMs on the 8B shapes; int8: the s8xs2 prefill of configs[2] "
                         "(quant_a + GEMM); bitcos: configs[3], Hadamard + BITCOS GEMV/GEMM; moe: the MoE prefill "
                         "layer (expert-parallel on N GPUs); hadamard: the sign flip + FWHT of the BITCOS config")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--shard-all", action="store_true",
                    help="N>1: split every layer's columns over the ranks (default: only where it pays)")
    ap.add_argument("--nccl-gather", action="store_true",
                    help="N>1: GEMV + NCCL all-gather instead of the GEMV with the all-gather fused in its epilogue")
    ap.add_argument("--graph", dest="graph", action="store_true", default=True,
                    help="one GPU: capture the K timed steps into one CUDA graph (the default; a decode loop "
                         "replays its launches, and the replay does not depend on the host's launch rate)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="time host calls with PDL instead of the graph replay")
    ap.add_argument("--sets", type=int, default=0,
                    help="weight sets to rotate (default: enough for %.0f GiB)" % WEIGHTS_GIB)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    import torch.distributed as dist

    import ternocl_b200 as tl
    from ternocl_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime
    one_rank_group = False
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    elif args.shard_all and args.workload == "decode":
        # one GPU in the sharded mode: the fused all-gather GEMV with a single rank (its
        # completion protocol without peers), for measuring that protocol's own cost
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev, timeout=datetime.timedelta(seconds=120))
        one_rank_group = True
    tl.set_option(tl.OPT_PDL, 0 if args.no_pdl else 1)
    if args.workload == "prefill":
        return run_prefill(args, tl, synth, dev, world, rank, local)
    if args.workload == "moe":
        return run_moe(args, tl, synth, dev, world, rank, local)
    if args.workload == "hadamard":
        return run_hadamard(args, tl, synth, dev, world, rank, local)
    if args.workload in ("int8", "bitcos"):
        return run_replicated(args, tl, dev, world, rank, local)

    # With N GPUs: splitting a layer's columns over the ranks (the all-gather fused into
    # the GEMV) pays only where it saves more weight-streaming time per rank than the
    # sharded launch's completion costs (dist.shard_pays, measured ~10 us at two ranks),
    # which none of these layers does.  So by default the N ranks run N independent
    # decode streams (replicas: each rank the whole step on its own weights, no
    # collective; weak scaling, the value counts every rank's weights).  --shard-all (the
    # fused all-gather) or --nccl-gather split every layer instead (strong scaling, each
    # layer's weights counted once).
    from ternocl_b200 import dist as tdist
    sharded = (world > 1 and args.nccl_gather) or args.shard_all
    shard = {(K, N): sharded for K, N in SHAPES}

    # per-rank column slices (multiples of 16)
    def cols(K, N):
        if not shard[(K, N)]:
            return 0, N
        per = (N // world) // 16 * 16
        n0 = rank * per
        return n0, (per if rank < world - 1 else N - n0)

    set_bytes = sum(weight_bytes(K, cols(K, N)[1]) for K, N in SHAPES)
    full_set_bytes = sum(weight_bytes(K, N) for K, N in SHAPES)
    nsets = args.sets or max(1, int(np.ceil(WEIGHTS_GIB * (1 << 30) / full_set_bytes)))
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    layers = []  # per shape: dict
    for K, N in SHAPES:
        n0, nl = cols(K, N)
        rng = np.random.default_rng(K * 7 + N)
        A = torch.randn(M, K, generator=g, device=dev).half()
        # one packed set generated on the host (uniform ternary), further sets are
        # device-side permutations of its words -> distinct data, same distribution
        B0 = torch.from_numpy(synth.pack_int2(synth.ternary(rng, K, nl)).view(np.int32)).to(dev)
        Bs, Ss = [], []
        for s in range(nsets):
            perm = torch.randperm(B0.numel(), generator=g, device=dev)
            Bs.append(B0.view(-1)[perm].view_as(B0).contiguous())
            Ss.append((torch.rand(K // 128, nl, generator=g, device=dev) * 0.04 + 0.01).half())
        C = torch.empty(M, nl, dtype=torch.float16, device=dev)
        Cfull = torch.empty(world, M, nl, dtype=torch.float16, device=dev) if shard[(K, N)] else None
        ws = tl.Workspace(dev, tl.gemv_workspace_size(M, nl, K))
        layers.append(dict(K=K, N=N, n0=n0, nl=nl, A=A, B=Bs, S=Ss, C=C, Cfull=Cfull, ws=ws, shard=shard[(K, N)]))
    del B0
    torch.cuda.synchronize()

    L = tl.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def gemv(ly, s, sp=sp):
        st = L.ternocl_int2_upcvt(ly["A"].data_ptr(), ly["B"][s].data_ptr(), ly["S"][s].data_ptr(),
                                  ly["C"].data_ptr(), None, None, M, ly["nl"], ly["K"], 0, 0, 0,
                                  tl.ALGO_GEMV, ly["ws"].ptr(), ly["ws"].nbytes(), sp)
        if st != 0:
            raise tl.TernoclError("ternocl_int2_upcvt", st)

    fused = None
    if (world > 1 and not args.nccl_gather) or one_rank_group:
        fused = [tdist.FusedAllGatherGemv(M, ly["N"], ly["K"], torch.float16, dev) if ly["shard"] else None
                 for ly in layers]

    def step(i):
        s = i % nsets
        if fused is not None:  # each launch leaves the full C on every rank
            for ly, fg in zip(layers, fused):
                if fg is not None:
                    fg(ly["A"], ly["B"][s], ly["S"][s])
                else:
                    gemv(ly, s)
            return
        for ly in layers:
            gemv(ly, s)
        for ly in layers:
            if ly["shard"]:
                dist.all_gather_into_tensor(ly["Cfull"], ly["C"])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    # one untimed pass over every set (the reference's warm-up rule) + W warm-up steps
    for i in range(max(nsets, args.warmup)):
        step(i)
    barrier()

    # A decode loop replays captured launches: on one GPU the K timed steps (4 GEMV
    # launches each, weight set i % nsets) are captured once into a CUDA graph and the
    # timed region is one replay of it (the C ABI allocates nothing, so its calls capture).
    # With N GPUs the fused column-sharded GEMV keeps its handshake epoch on the device, so
    # its steps are captured the same way on every rank and the ranks replay together.
    timed_graph = None
    if args.graph and (world == 1 or fused is not None):
        torch.cuda.synchronize()
        timed_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(timed_graph):
            cs = torch.cuda.current_stream(dev).cuda_stream
            for i in range(args.steps):
                for j, ly in enumerate(layers):
                    if fused is not None and fused[j] is not None:
                        fused[j](ly["A"], ly["B"][i % nsets], ly["S"][i % nsets], stream=cs)
                    else:
                        gemv(ly, i % nsets, cs)
        if world > 1:
            dist.barrier(device_ids=[local])
        timed_graph.replay()  # the first replay uploads the graph: keep it out of the timed region
        torch.cuda.synchronize()

    def timed_steps():
        if timed_graph is not None:
            timed_graph.replay()
        else:
            for i in range(args.steps):
                step(i)


    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        if args.profile_range:
            torch.cuda.cudart().cudaProfilerStart()
        ev0.record(stream)
        timed_steps()
        ev1.record(stream)
        barrier()
        if args.profile_range:
            torch.cuda.cudart().cudaProfilerStop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    # the whole job's weights per step: each layer once when sharded, every rank's own
    # copy when the ranks are independent replicas
    job_bytes = full_set_bytes * (world if (world > 1 and not sharded) else 1)
    value = job_bytes / (ms_per_step * 1e-3) / 1e9

    # kernel-only timing (no collectives) for the roofline: GEMV launches back to back
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev2.record(stream)
    if timed_graph is not None:
        timed_graph.replay()
    else:
        for i in range(args.steps):
            for ly in layers:
                gemv(ly, i % nsets)
    ev3.record(stream)
    barrier()
    kern_ms = ev2.elapsed_time(ev3)
    launches = args.steps * len(layers)
    achieved = set_bytes * args.steps / (kern_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()

    # end to end through the C ABI with host buffers (pinned), rank-local: per step one
    # copy of the four activation vectors in (one pinned buffer), the four GEMVs, one copy
    # of the four outputs out, and a synchronisation (the decode loop reads its result)
    hA = [torch.randn(M, ly["K"]).half().pin_memory() for ly in layers]
    hC = [torch.empty(M, ly["nl"], dtype=torch.float16).pin_memory() for ly in layers]
    h2d = sum(x.numel() * 2 for x in hA)
    d2h = sum(x.numel() * 2 for x in hC)
    packed = not sharded  # one GPU, or independent replicas: each rank the whole step
    if packed:
        ka = [ly["K"] * M for ly in layers]
        kc = [ly["nl"] * M for ly in layers]
        hAall = torch.cat([x.reshape(-1) for x in hA]).pin_memory()
        hCall = torch.empty(sum(kc), dtype=torch.float16).pin_memory()
        dAall = torch.empty(sum(ka), dtype=torch.float16, device=dev)
        dCall = torch.empty(sum(kc), dtype=torch.float16, device=dev)
        oa = np.cumsum([0] + ka)
        oc = np.cumsum([0] + kc)
        e2e_layers = [dict(ly, A=dAall[oa[j]:oa[j + 1]].view(M, ly["K"]), C=dCall[oc[j]:oc[j + 1]].view(M, ly["nl"]))
                      for j, ly in enumerate(layers)]

    def e2e_step(i):
        s = i % nsets
        if packed:
            dAall.copy_(hAall, non_blocking=True)
            for ly in e2e_layers:
                gemv(ly, s)
            hCall.copy_(dCall, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            return
        for j, ly in enumerate(layers):
            ly["A"].copy_(hA[j], non_blocking=True)
            if fused is not None and fused[j] is not None:
                out = fused[j](ly["A"], ly["B"][s], ly["S"][s])
                hC[j].copy_(out[:, ly["n0"]:ly["n0"] + ly["nl"]], non_blocking=True)
                continue
            gemv(ly, s)
            if ly["shard"]:
                dist.all_gather_into_tensor(ly["Cfull"], ly["C"])
            hC[j].copy_(ly["C"], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for i in range(args.warmup):
        e2e_step(i)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    barrier()
    e2e_s = (time.perf_counter() - t0) / args.steps
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = job_bytes / e2e_s / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, kind, desc = CpuReference().sample()
        cpu = {"value": v, "unit": "GB/s", "cores": cores, "kind": kind, "sample": desc}

    secondary = None
    if world == 1 and not args.no_secondary:
        tf, pms, _ = prefill_measure(tl, synth, dev, steps=min(args.steps, 20), warmup=3)
        pk = peaks_tensor(pms * min(args.steps, 20) * 1e-3)
        mt, mtf, mms, me2e, mcpu = moe_measure(tl, synth, dev, steps=min(args.steps, 10), warmup=2,
                                               cpu=not args.no_cpu_baseline)
        pk_moe = peaks_tensor(mms * min(args.steps, 10) * 1e-3)
        secondary_moe = {"metric": "MoE prefill tokens/s (T=4096, H=2048, I=768, E=128, top-8, fp16)", "value": mt,
                         "unit": "tokens/s", "ms_per_layer": mms, "tflops": mtf,
                         "roofline": {"bound": "tensor", "achieved": mtf, "peak": pk_moe[0], "unit": "TFLOP/s",
                                      "frac": mtf / pk_moe[0], "peak_kind": pk_moe[1]},
                         "e2e": me2e, "cpu_baseline": mcpu}
        sec_int8 = int8_measure(tl, dev, steps=min(args.steps, 20), warmup=3, cpu=not args.no_cpu_baseline)
        sec_bitcos = bitcos_measure(tl, dev, steps=min(args.steps, 50), warmup=3, cpu=not args.no_cpu_baseline)
        gshapes, c1 = gemv_shapes_measure(tl, dev, cpu=not args.no_cpu_baseline)
        secondary = {"int8_prefill": sec_int8, "bitcos": sec_bitcos, "moe": secondary_moe, "c1_host_config": c1,
                     "gemv_shapes_m1": {"metric": "M=1 int2 fp16 GEMV per shape of the reference's published table "
                                                  "(int2_fp16_upcvt/README.md), CUDA graph of back-to-back launches",
                                        "unit": "GB/s", "shapes": gshapes},
                     "prefill": {"metric": "M=2048 int2 fp16 prefill TFLOP/s (tcgen05 GEMM)", "value": tf,
                                 "unit": "TFLOP/s", "ms_per_step": pms, "M": PREFILL_M, "shapes_KxN": SHAPES,
                                 "roofline": {"bound": "tensor", "achieved": tf, "peak": pk[0], "unit": "TFLOP/s",
                                              "frac": tf / pk[0], "peak_kind": pk[1]}}}

    if rank == 0:
        tr = profile_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak" if (world > 1 and not sharded) else "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M, "shapes_KxN": SHAPES, "weight_sets": nsets,
                       "weights_gib": round(nsets * full_set_bytes / 2 ** 30, 3),
                       "l2": "inputs larger than L2: %d rotating weight sets" % nsets,
                       "parallelism": ("N-sharded columns x%d + %s" % (
                           world, "NCCL all-gather" if args.nccl_gather else
                           "all-gather fused into the GEMV epilogue (NVLink peer stores)")) if sharded else
                       ("%d independent decode streams (replicas, no collective): column sharding saves less "
                        "than a sharded launch's completion (~10 us at 2 ranks) on every layer" % world)
                       if world > 1 else "single GPU",
                       "pdl": not args.no_pdl,
                       "launch": "one CUDA graph of the K timed steps" if timed_graph is not None else "host calls, PDL"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "kernel": "gemv_i2d_kernel (integer-MMA int2 GEMV)", "launches": launches,
                         "bytes_per_step": set_bytes,
                         "traffic": tr.get("bytes_per_step") if tr else None},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        if secondary:
            line["secondary"] = secondary
        print(json.dumps(line), flush=True)
    timed_graph = None
    if fused is not None:
        torch.cuda.synchronize()
        for fg in fused:
            if fg is not None:
                fg.close()
    if world > 1 or one_rank_group:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
