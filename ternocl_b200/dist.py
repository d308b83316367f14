"""Multi-GPU paths: one process per GPU, torch.distributed (NCCL over NVLink) for the
collectives, this library's kernels for the compute.

* Column-sharded decode GEMV (``column_shard``, ``sharded_upcvt``): the columns of a
  weight matrix are independent (B, S, Bias and Other are column-indexed), so rank r
  keeps columns [n0, n0 + nl) (multiples of 16), computes its slice of C and the slices
  are all-gathered.
* Expert-parallel MoE prefill (``ExpertParallelMoE``): rank r owns experts
  [r E/P, (r+1) E/P) and T/P tokens.  Routed rows are sorted by owning rank (the route
  kernel with the ranks as "experts"), counts are exchanged, the rows travel with one
  all-to-all, the owner runs route/gather/grouped GEMMs (up, gate with SiLU-mul, down)
  on them, the fp32 results travel back with a second all-to-all and the source rank
  combines them with its gate weights.

The kernel entry points are parameters (default: the CUDA ones of ``ternocl_b200``), so
the host-side bookkeeping can be exercised with CPU stand-ins under the gloo backend.
"""
import torch
import torch.distributed as dist


def column_shard(N, world, rank, align=16):
    """(n0, nl): rank's contiguous column slice; all but the last are equal multiples of align."""
    per = (N // world) // align * align
    n0 = rank * per
    return n0, (per if rank < world - 1 else N - n0)


# Completion cost of one column-sharded GEMV launch (its last CTA copies the rank's slice
# to the peers, fences at system scope and waits for the peers' flags), measured on B200:
# ~4.5 us per call with one rank (no NVLink) and ~8-12 us with two; and the rate at
# which a decode GEMV streams its weights (~2.5 TB/s on the Llama-3-8B shapes).
SHARD_COMPLETION_US = 10.0
SHARD_STREAM_GBS = 2500.0


def shard_pays(K, N, world, completion_us=SHARD_COMPLETION_US, stream_gbs=SHARD_STREAM_GBS):
    """Whether splitting the columns of a K x N int2 GEMV over `world` ranks saves more
    weight-streaming time per rank than the sharded launch's completion costs.  Layers
    for which it does not are better replicated (every rank runs the whole GEMV and has
    the whole output, with no collective)."""
    if world <= 1:
        return False
    weights = K * N // 4 + (K // 128) * N * 2
    saved_us = weights * (1.0 - 1.0 / world) / (stream_gbs * 1e3)
    return saved_us > completion_us


def sharded_upcvt(A, B_shard, S_shard, N, upcvt=None, group=None, **kw):
    """C [M, N] = epi(A @ dequant(B, S)) with this rank holding columns column_shard(N, ...)."""
    if upcvt is None:
        from . import int2_upcvt as upcvt
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    C = upcvt(A, B_shard, S_shard, **kw)
    if world == 1:
        return C
    M = C.shape[0]
    widths = [column_shard(N, world, r)[1] for r in range(world)]
    wmax = max(widths)
    buf = C if C.shape[1] == wmax else torch.nn.functional.pad(C, (0, wmax - C.shape[1]))
    parts = [torch.empty(M, wmax, dtype=C.dtype, device=C.device) for _ in range(world)]
    dist.all_gather(parts, buf.contiguous(), group=group)
    return torch.cat([p[:, :w] for p, w in zip(parts, widths)], dim=1)


def ipc_peers(t, group=None):
    """Every rank's tensor `t` (same shape and dtype on every rank) as device pointers valid
    in this process: its own, and the peers' mapped by CUDA IPC (plain peer mappings).
    Returns (pointers, mapped) where mapped lists (pointer, offset) to release later."""
    import ctypes
    from ._lib import call
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    h = (ctypes.c_uint8 * 64)()
    off = ctypes.c_size_t(0)
    call("ternocl_ipc_handle", t.data_ptr(), ctypes.addressof(h), ctypes.byref(off))
    mine = torch.tensor(list(bytes(h)) + list(int(off.value).to_bytes(8, "little")), dtype=torch.uint8,
                        device=t.device)
    everyone = torch.empty(world, mine.numel(), dtype=torch.uint8, device=t.device)
    dist.all_gather_into_tensor(everyone, mine, group=group)
    rows = everyone.cpu().numpy()
    ptrs, mapped = [], []
    for r in range(world):
        if r == rank:
            ptrs.append(t.data_ptr())
            continue
        hh = (ctypes.c_uint8 * 64).from_buffer_copy(rows[r][:64].tobytes())
        o = int.from_bytes(rows[r][64:72].tobytes(), "little")
        p = ctypes.c_void_p(0)
        call("ternocl_ipc_open", ctypes.addressof(hh), o, ctypes.byref(p))
        ptrs.append(p.value)
        mapped.append((p.value, o))
    return ptrs, mapped


class FusedAllGatherGemv:
    """Column-sharded int2 GEMV whose epilogue writes this rank's columns into every
    rank's C (ternocl_int2_upcvt_allgather): C [M, N] is complete on every rank when the
    launch finishes, with no separate collective.  Two C buffers alternate between calls
    so a rank may read the previous output while the next call is being written.  The
    call count that orders the ranks' handshakes is kept on the device (epoch 0), so a
    sequence of calls can be captured in a CUDA graph and replayed on every rank."""

    def __init__(self, M, N, K, dtype, device, group=None):
        import ctypes
        from . import dtype_code, lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.M, self.N, self.K = M, N, K
        self.n0, self.nl = column_shard(N, self.world, self.rank)
        self.dt = dtype_code(torch.empty(0, dtype=dtype))
        self.C = [torch.empty(M, N, dtype=dtype, device=device) for _ in range(2)]
        # one flag per rank + this rank's call count (the device-kept epoch)
        self.flags = torch.zeros(self.world + 1, dtype=torch.int32, device=device)
        self.ws = torch.zeros(lib().ternocl_gemv_allgather_workspace_size(M, self.nl, K), dtype=torch.uint8,
                              device=device)
        self._mapped = []
        self.c_ptrs = []
        for c in self.C:
            ptrs, mapped = ipc_peers(c, group)
            self.c_ptrs.append((ctypes.c_void_p * self.world)(*ptrs))
            self._mapped += mapped
        fptrs, mapped = ipc_peers(self.flags, group)
        self.f_ptrs = (ctypes.c_void_p * self.world)(*fptrs)
        self._mapped += mapped
        self.calls = 0
        dist.barrier(group=group)

    def __call__(self, A, B_shard, S_shard, postop=0, other=None, bias=None, stream=None):
        """A [M, K]; B_shard [K/16, nl], S_shard [K/128, nl] = this rank's columns.  Returns C."""
        from . import _ptr, _stream, call
        self.calls += 1
        buf = self.calls & 1
        call("ternocl_int2_upcvt_allgather", _ptr(A), _ptr(B_shard), _ptr(S_shard), self.c_ptrs[buf], _ptr(other),
             _ptr(bias), self.M, self.N, self.n0, self.nl, self.K, self.dt, int(postop), 0, self.rank, self.world,
             self.f_ptrs, 0, self.ws.data_ptr(), self.ws.numel(), _stream(stream))
        return self.C[buf]

    def close(self):
        from ._lib import lib
        for p, o in self._mapped:
            lib().ternocl_ipc_close(p, o)
        self._mapped = []


class Kernels:
    """The four MoE kernel entry points (CUDA by default)."""

    def __init__(self, route=None, gather=None, gemm=None, combine=None):
        from . import moe_combine, moe_gather, moe_gemm, moe_route
        self.route = route or moe_route
        self.gather = gather or moe_gather
        self.gemm = gemm or moe_gemm
        self.combine = combine or moe_combine


class ExpertParallelMoE:
    """One MoE prefill layer over P ranks.  Weights are this rank's experts:
    Bg/Bu int32 [E/P, H/16, I], Bd [E/P, I/16, H], scales [E/P, K/128, N]."""

    def __init__(self, num_experts, topk, Bg, Sg, Bu, Su, Bd, Sd, group=None, kernels=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world:
            raise ValueError("experts must split evenly over the ranks")
        self.E, self.EP, self.topk = num_experts, num_experts // self.world, topk
        self.Bg, self.Sg, self.Bu, self.Su, self.Bd, self.Sd = Bg, Sg, Bu, Su, Bd, Sd
        self.k = kernels or Kernels()

    def _a2a(self, x, out_rows, in_rows):
        out = torch.empty((sum(out_rows),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(out, x.contiguous(), output_split_sizes=out_rows, input_split_sizes=in_rows,
                               group=self.group)
        return out

    def __call__(self, X, ids, RW):
        """X [T_local, H] (fp16/bf16), ids int32 [T_local*topk] (global expert ids, row g =
        t*topk + j), RW [T_local*topk] gate weights -> O [T_local, H]."""
        k, topk = self.k, self.topk
        T = X.shape[0]
        # 1. routed rows sorted by owning rank
        dest = torch.div(ids, self.EP, rounding_mode="floor").to(torch.int32)
        meta_d, perm_d, inv_d = k.route(dest, self.world)
        meta_h = meta_d[: self.world + 1].tolist()
        send = [meta_h[r + 1] - meta_h[r] for r in range(self.world)]
        Xsend = k.gather(X, perm_d, topk)
        local_ids = (ids.long()[perm_d.long()] - dest.long()[perm_d.long()] * self.EP).to(torch.int32)
        # 2. counts, then rows and their local expert ids
        if self.world > 1:
            sc = torch.tensor(send, dtype=torch.int64, device=X.device)
            rc = torch.empty_like(sc)
            dist.all_to_all_single(rc, sc, group=self.group)
            recv = rc.tolist()
            Xrecv = self._a2a(Xsend, recv, send)
            ids_recv = self._a2a(local_ids, recv, send)
        else:
            recv, Xrecv, ids_recv = send, Xsend, local_ids
        # 3. this rank's experts on the received rows
        meta_e, perm_e, inv_e = k.route(ids_recv, self.EP)
        Xs = k.gather(Xrecv, perm_e, 1)
        up = k.gemm(meta_e, Xs, self.Bu, self.Su, self.EP)
        Hh = k.gemm(meta_e, Xs, self.Bg, self.Sg, self.EP, postop=1, other=up)
        Y = k.gemm(meta_e, Hh, self.Bd, self.Sd, self.EP, out_f32=True)
        Yrecv = Y.index_select(0, inv_e.long())  # back to the received order
        # 4. results to their source rank (destination-sorted order), weighted combine
        Yback = self._a2a(Yrecv, send, recv) if self.world > 1 else Yrecv
        return k.combine(Yback, inv_d, RW, T, topk)
