"""Tensor-parallel sharding of packed stores over the GPUs of one node.

The packed rows of a store are independent, so a decoder's linears split the
Megatron way (one process per GPU, NCCL over NVLink for the exchange):

* column-parallel (q/k/v, gate/up): rank r keeps rows [N r / P, N (r+1) / P)
  of the indices and scales; the codebook (2 KiB) is replicated.  The output
  is the rank's slice of the features -- no communication.
* row-parallel (o, down): rank r keeps the k range [K r / P, K (r+1) / P),
  cut at group boundaries (K / P a multiple of the group), which is exactly
  the feature slice the preceding column-parallel linear produced locally
  (o reads q, down reads up).  The outputs are partial sums over k; one
  all-reduce (SUM) per row-parallel linear completes them.

So a layer costs two all-reduces of [m, hidden], after o and after down.
``shard_store`` cuts an existing store (row layout, any device) and returns a
store of the same kind; ``TPLinearStack`` runs the packed linears of a decode
step on the shards: the linears through libepq.so, fp32 partial sums, the
all-reduce through ``torch.distributed`` (NCCL on GPUs), the whole step
recorded in one CUDA graph.
"""
import torch

from .runtime import PackedWeight, _pack4

COLUMN = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")
ROW = ("o_proj", "down_proj")


def split_range(total, rank, world, align=1):
    """[lo, hi) of rank's equal share of `total`; shares must be multiples of `align`."""
    if total % world or (total // world) % align:
        raise ValueError(f"cannot split {total} into {world} equal parts aligned to {align}")
    share = total // world
    return rank * share, (rank + 1) * share


def _rows_values(store):
    """Per-position indices [rows, in_features / vec] (u8) and scales [rows, groups]."""
    idx = store.index_rows()
    sc = store.scale.detach()
    return idx, sc


def _make(store, shape, idx_rows, scale, device):
    idx = idx_rows.contiguous().reshape(-1)
    if store.vec == 1 and store.levels <= 16:
        idx = torch.from_numpy(_pack4(idx.cpu().numpy(), store.levels))
    st = PackedWeight(shape, idx.cpu(), scale.contiguous().cpu(), store.cb.detach().cpu().clone(),
                      store.group, store.levels, vec=store.vec, gpu_layout=store.GPU_LAYOUT)
    return st.to(device) if device is not None else st


def shard_store(store, rank, world, dim, device=None):
    """Rank's shard of `store`: dim "rows" (column-parallel) or "cols" (row-parallel)."""
    n, k = store.out_features, store.in_features
    idx, sc = _rows_values(store)
    if dim == "rows":
        lo, hi = split_range(n, rank, world)
        return _make(store, (hi - lo, k), idx[lo:hi], sc[lo:hi], device)
    if dim == "cols":
        lo, hi = split_range(k, rank, world, align=store.group)
        if store.vec == 4:
            part = idx[:, lo // 4:hi // 4]
        else:
            part = idx[:, lo:hi]
        g0, g1 = lo // store.group, hi // store.group
        return _make(store, (n, hi - lo), part, sc[:, g0:g1], device)
    raise ValueError("dim must be 'rows' or 'cols'")


def shard_blocks(blocks, rank, world, device=None):
    """Shard every layer of a LinearStack-style block list (dicts of name -> store)."""
    out = []
    for b in blocks:
        out.append({name: shard_store(st, rank, world, "rows" if name in COLUMN else "cols", device)
                    for name, st in b.items()})
    return out


class TPLinearStack:
    """The packed linears of one decode step on this rank's shards.

    Per layer: q/k/v (column-parallel, one fused launch) -> o (row-parallel,
    fp32 partial sums) -> all-reduce -> gate/up (column-parallel, one launch)
    -> down (row-parallel) -> all-reduce; the reduced down output, cast to the
    activation dtype, feeds the next layer.  ``linear_fn(x, stores, outs,
    out_dtype)`` defaults to libepq.so's ``linear_multi``; the all-reduce is
    ``torch.distributed.all_reduce`` on ``group``.  Partial sums are fp32 for
    16-bit activations (otherwise the activation dtype).
    """

    def __init__(self, blocks, m=1, dtype=torch.bfloat16, device=None, group=None,
                 linear_fn=None):
        import torch.distributed as dist
        self.blocks = blocks
        self.m = m
        self.dtype = dtype
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        b0 = blocks[0]
        self.device = torch.device(device) if device is not None else b0["q_proj"].packed.device
        if linear_fn is None:
            from . import _native

            def linear_fn(x, stores, outs, out_dtype):
                return _native.linear_multi(x, stores, out_dtype=out_dtype, outs=outs)
        self.linear_fn = linear_fn
        mk = lambda n, dt=dtype: torch.zeros((m, n), dtype=dt, device=self.device)  # noqa: E731
        hidden = b0["o_proj"].out_features
        self.x = mk(b0["q_proj"].in_features)
        self.q, self.k, self.v = (mk(b0[n].out_features) for n in ("q_proj", "k_proj", "v_proj"))
        self.part_dtype = torch.float32 if dtype in (torch.bfloat16, torch.float16) else dtype
        self.part = mk(hidden, self.part_dtype)         # row-parallel partial sums
        self.h = mk(hidden)
        self.g, self.u = mk(b0["gate_proj"].out_features), mk(b0["up_proj"].out_features)
        self.out = mk(b0["down_proj"].out_features)
        self.graph = None
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.launches_per_step = 4 * len(blocks)
        self.allreduces_per_step = 2 * len(blocks)

    def _reduce(self, t):
        import torch.distributed as dist
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def step_eager(self):
        h = self.x
        for b in self.blocks:
            self.linear_fn(h, [b["q_proj"], b["k_proj"], b["v_proj"]], [self.q, self.k, self.v],
                           self.q.dtype)
            self.linear_fn(self.q, [b["o_proj"]], [self.part], self.part_dtype)
            self.h.copy_(self._reduce(self.part))
            self.linear_fn(self.h, [b["gate_proj"], b["up_proj"]], [self.g, self.u], self.g.dtype)
            self.linear_fn(self.u, [b["down_proj"]], [self.part], self.part_dtype)
            self.out.copy_(self._reduce(self.part))
            h = self.out
        return self.out

    def capture(self):
        """Warm up (kernels, workspaces, NCCL) and record one step in a CUDA graph."""
        from . import _native
        with torch.cuda.stream(self.stream):
            for grp in ([self.blocks[0][n] for n in ("q_proj", "k_proj", "v_proj")],
                        [self.blocks[0]["o_proj"]],
                        [self.blocks[0]["gate_proj"], self.blocks[0]["up_proj"]],
                        [self.blocks[0]["down_proj"]]):
                _native.reserve_workspace(grp, self.m, self.device)
            self.step_eager()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.step_eager()
        self.graph = g
        return self

    def replay(self):
        self.graph.replay()
        return self.out

    def release(self):
        """Drop the CUDA graph (it holds NCCL work; release before destroying the group)."""
        self.graph = None

    def __call__(self, x_host, out_host=None):
        if self.graph is None:
            self.capture()
        self.x.copy_(x_host, non_blocking=True)
        self.graph.replay()
        if out_host is None:
            out_host = torch.empty(self.out.shape, dtype=self.out.dtype, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        return out_host


def full_step_reference(blocks, x, linear_fn, out_dtype=None):
    """The same step on unsharded stores (for checking the sharded result).

    ``linear_fn(x, stores, outs, out_dtype)`` returns the list of outputs.
    """
    h = x
    for b in blocks:
        q = linear_fn(h, [b["q_proj"]], None, out_dtype)[0]
        o = linear_fn(q, [b["o_proj"]], None, out_dtype)[0]
        u = linear_fn(o, [b["up_proj"]], None, out_dtype)[0]
        h = linear_fn(u, [b["down_proj"]], None, out_dtype)[0]
    return h


def exchange_peer_pointers(t, group=None):
    """Map every rank's allocation holding tensor `t` into this process (CUDA IPC).

    Returns, per rank, the address of that rank's `t` as seen here (this
    rank's own pointer unchanged) and the mapped bases to release with
    ``close_peer_pointers``.  One process per GPU; the GPUs must reach each
    other over NVLink (peer access)."""
    import torch.distributed as dist
    from cuda.bindings import driver as cu
    from cuda.bindings import runtime as rt
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    ptr = t.data_ptr()
    err, base, _size = cu.cuMemGetAddressRange(ptr)
    if err != cu.CUresult.CUDA_SUCCESS:
        raise RuntimeError(f"epure: cuMemGetAddressRange failed ({err})")
    base = int(base)
    err, handle = rt.cudaIpcGetMemHandle(base)
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"epure: cudaIpcGetMemHandle failed ({err})")
    mine = (bytes(handle.reserved), ptr - base)
    allv = [None] * world
    dist.all_gather_object(allv, mine, group=group)
    ptrs, opened = [], []
    for r, (hbytes, off) in enumerate(allv):
        if r == rank:
            ptrs.append(ptr)
            continue
        h = rt.cudaIpcMemHandle_t()
        h.reserved = hbytes
        err, pbase = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"epure: cudaIpcOpenMemHandle of rank {r} failed ({err})")
        opened.append(int(pbase))
        ptrs.append(int(pbase) + off)
    return ptrs, opened


def close_peer_pointers(opened):
    from cuda.bindings import runtime as rt
    for b in opened:
        rt.cudaIpcCloseMemHandle(b)


class TPChainedLinearStack:
    """The decode chain of a tensor-parallel shard stack as ONE persistent launch per rank.

    Each rank prepares the chain kernel's workspace over its shards
    (``LinearStack(..., tp=(rank, world), gpu_layout="tiled")``), maps every
    rank's workspace (CUDA IPC) and marks the steps whose input is summed over
    ranks: the q/k/v step of every layer after the first (down is
    row-parallel), every gate/up step (o is row-parallel), and the final
    output.  Inside the kernel each rank publishes its sum of every input slice
    it stages and adds the peers' over NVLink -- the all-reduce after o and
    down happens in the decode kernel itself, with no collective launch.
    """

    def __init__(self, stack, group=None, dtype=torch.bfloat16, device=None):
        import torch.distributed as dist
        from . import _native
        self.stack = stack
        self.device = torch.device(device or stack.device)
        steps = stack.chain_steps()
        self.ws = _native.chain_prepare(steps)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        ptrs, self._opened = exchange_peer_pointers(self.ws, group)
        # per layer: qkv (input = previous down, row-parallel, except the very first), o, gate/up, down
        remote = []
        for li in range(len(stack.blocks)):
            remote += [li > 0, False, True, False]
        remote.append(True)        # final output = down (row-parallel)
        _native.chain_set_tp(self.ws, self.rank, self.world, ptrs, remote)
        dist.barrier(group)        # every rank's workspace is ready before any run
        k0 = steps[0][0][0].in_features
        last, feed = steps[-1]
        self.x = torch.zeros((1, k0), dtype=dtype, device=self.device)
        self.out = torch.zeros((1, last[feed].out_features), dtype=dtype, device=self.device)
        self.graph = None
        self.stream = torch.cuda.Stream(device=self.device)
        self.launches_per_step = 1

    def step_eager(self):
        from . import _native
        _native.chain_run(self.ws, self.x, self.out)
        return self.out

    def capture(self):
        with torch.cuda.stream(self.stream):
            self.step_eager()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.step_eager()
        self.graph = g
        return self

    def replay(self):
        self.graph.replay()
        return self.out

    def release(self):
        self.graph = None
        torch.cuda.synchronize(self.device)
        close_peer_pointers(self._opened)
        self._opened = []

    def __call__(self, x_host, out_host=None):
        if self.graph is None:
            self.capture()
        self.x.copy_(x_host, non_blocking=True)
        self.graph.replay()
        if out_host is None:
            out_host = torch.empty(self.out.shape, dtype=self.out.dtype, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        return out_host


__all__ = ["shard_store", "shard_blocks", "split_range", "TPLinearStack", "TPChainedLinearStack",
           "full_step_reference", "exchange_peer_pointers", "close_peer_pointers", "COLUMN", "ROW"]
