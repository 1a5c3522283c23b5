"""Tensor-parallel sharding (epure.tp) on the CPU: shard math and gloo ranks.

* A column shard (rows) and a row shard (group-aligned k range) of a store
  materialise to exactly the matching slice of the full weight, for vector and
  scalar (4-bit and 8-bit) codebooks; splits that break a group are refused.
* 2 and 4 gloo ranks run TPLinearStack's decode step (column-parallel q/k/v and
  gate/up, row-parallel o and down with an all-reduce after each) with the
  oracle's float64 linear, and every rank ends with the unsharded step's
  result (<= 1e-12 relative).
"""
import os
from datetime import timedelta

import numpy as np
import pytest
import torch

from epure import synthetic, tp
from epure.synthetic import DecoderShapes

TINY = DecoderShapes("tiny", 2, 512, 1024, 8, 2, 64, 1000)


def _scalar_store(n, k, levels, seed):
    from epure import PackedWeight
    from epure.runtime import _pack4
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, levels, size=n * k, dtype=np.uint8)
    scale = (np.abs(rng.standard_normal((n, -(-k // 128)))) * 0.02).astype(np.float16)
    cb = rng.standard_normal(levels).astype(np.float32)
    return PackedWeight((n, k), _pack4(idx, levels), scale, cb, 128, levels)


@pytest.mark.parametrize("kind", ["vec4", "scalar16", "scalar256"])
def test_shards_are_slices(kind):
    n, k, world = 96, 512, 4
    if kind == "vec4":
        st = synthetic.make_store(n, k, device="cpu", seed=1)
    else:
        st = _scalar_store(n, k, 16 if kind == "scalar16" else 256, seed=2)
    full = st.materialize(torch.float32)
    for r in range(world):
        rows = tp.shard_store(st, r, world, "rows")
        lo, hi = r * n // world, (r + 1) * n // world
        assert rows.out_features == hi - lo and rows.in_features == k
        assert torch.equal(rows.materialize(torch.float32), full[lo:hi])
        cols = tp.shard_store(st, r, world, "cols")
        lo, hi = r * k // world, (r + 1) * k // world
        assert cols.out_features == n and cols.in_features == hi - lo
        assert torch.equal(cols.materialize(torch.float32), full[:, lo:hi])


def test_split_must_keep_groups():
    st = synthetic.make_store(64, 384, device="cpu", seed=3)
    with pytest.raises(ValueError):
        tp.shard_store(st, 0, 2, "cols")          # 192 is not a multiple of 128
    with pytest.raises(ValueError):
        tp.shard_store(st, 0, 5, "rows")          # 64 rows into 5 parts
    with pytest.raises(ValueError):
        synthetic.LinearStack(TINY, device="cpu", tp=(0, 8))   # o: 512 / 8 = 64 < group


def _oracle_linear():
    from oracle import oracle as O

    def fn(x, stores, outs=None, out_dtype=None):
        res = []
        for i, st in enumerate(stores):
            y = O.linear_exact(x.double().numpy(), st.index_rows().numpy(), st.scale.float().numpy(),
                               st.cb.float().numpy(), st.out_features, st.in_features, st.vec,
                               st.group, st.levels)
            t = torch.from_numpy(np.ascontiguousarray(y))
            if outs is not None:
                outs[i].copy_(t)
                res.append(outs[i])
            else:
                res.append(t)
        return res
    return fn


def _worker(rank, world, port, result_q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        stack = synthetic.LinearStack(TINY, device="cpu", seed=11)     # same full model everywhere
        shards = tp.shard_blocks(stack.blocks, rank, world)
        runner = tp.TPLinearStack(shards, m=3, dtype=torch.float64, device="cpu",
                                  linear_fn=_oracle_linear())
        g = torch.Generator().manual_seed(5)
        runner.x.copy_(torch.randn(3, TINY.hidden, generator=g, dtype=torch.float64))
        out = runner.step_eager().clone()
        want = tp.full_step_reference(stack.blocks, runner.x.clone(), _oracle_linear())
        err = float((out - want).abs().max() / want.abs().max())
        result_q.put((rank, err, runner.allreduces_per_step))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_match_unsharded(world):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(r for r, _, _ in results) == list(range(world))
    for _, err, n_ar in results:
        assert err <= 1e-12
        assert n_ar == 2 * TINY.layers
