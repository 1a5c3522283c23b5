"""Tensor-parallel decode on 2 GPUs (NCCL): sharded step == single-GPU step.

Each rank builds the same 2-layer Llama-3-8B-shaped stack (same seed), keeps
its shards (column-parallel q/k/v, gate/up; row-parallel o, down), and runs
TPLinearStack's CUDA graph (libepq.so kernels + NCCL all-reduce after o and
down).  The result equals the unsharded chain of single-GPU launches within
1e-2 (bf16 activations between linears; the row-parallel sums are fp32 and
only their split differs).  Needs at least 2 GPUs; skipped otherwise.
"""
import os
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, m, q):
    import torch.distributed as dist
    from epure import synthetic, tp, _native
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    runner = None
    try:
        stack = synthetic.LinearStack(synthetic.LLAMA3_8B, layers=2, device=dev, seed=21,
                                      gpu_layout="mma16")
        shards = tp.shard_blocks(stack.blocks, rank, world, device=dev)
        runner = tp.TPLinearStack(shards, m=m, dtype=torch.bfloat16, device=dev).capture()
        g = torch.Generator(device=dev).manual_seed(9)
        x = torch.randn(m, 4096, generator=g, device=dev).to(torch.bfloat16)
        runner.x.copy_(x)
        out = runner.replay().float().clone()
        torch.cuda.synchronize(dev)

        def lin(h, stores, outs, out_dtype):
            return _native.linear_multi(h, stores, out_dtype=out_dtype, outs=outs)
        want = tp.full_step_reference(stack.blocks, x, lin).float()
        err = float((out - want).abs().max() / want.abs().max())
        q.put((rank, err, _native.device_error()))
    finally:
        if runner is not None:
            runner.release()
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [1, 4])
def test_tp2_matches_single_gpu(m):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, derr in res:
        assert derr == 0
        assert err <= 1e-2, (rank, err)


def _chain_worker(rank, world, port, q):
    import torch.distributed as dist
    from epure import synthetic, tp, _native
    from epure.decode import ChainedLinearStack
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    runner = None
    try:
        full = synthetic.LinearStack(synthetic.LLAMA3_8B, layers=2, device=dev, seed=31,
                                     gpu_layout="tiled")
        shards = synthetic.LinearStack.from_blocks(
            synthetic.LLAMA3_8B, tp.shard_blocks(full.blocks, rank, world, device=dev), dev)
        runner = tp.TPChainedLinearStack(shards, dtype=torch.float32).capture()
        g = torch.Generator(device=dev).manual_seed(9)
        x = torch.randn(1, 4096, generator=g, device=dev)
        outs = []
        for r in range(3):                       # consecutive runs on the same workspaces
            runner.x.copy_(x * (1 + r))
            outs.append(runner.replay().clone())
        torch.cuda.synchronize(dev)
        single = ChainedLinearStack(full, dtype=torch.float32)
        errs = []
        for r in range(3):
            single.x.copy_(x * (1 + r))
            want = single.step_eager().clone()
            errs.append(float((outs[r] - want).abs().max() / want.abs().max()))
        torch.cuda.synchronize(dev)
        q.put((rank, errs, outs[0].cpu(), _native.device_error()))
    finally:
        if runner is not None:
            runner.release()
        dist.destroy_process_group()


def test_tp2_chain_matches_single_gpu():
    """TP inside the persistent chain: ranks exchange slice sums over NVLink in the kernel."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_chain_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, errs, _, derr in res:
        assert derr == 0
        assert max(errs) <= 1e-4, (rank, errs)
    assert torch.equal(res[0][2], res[1][2])     # every rank ends with the same output
