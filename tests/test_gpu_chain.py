"""The persistent chain kernel (epq_chain_prepare / epq_chain_run) on the GPU.

A chain keeps intermediate activations as fp32 partial sums (never rounded to
the activation dtype), so it is compared with the exact float64 chain of the
oracle's dense expansion (<= 1e-4 relative) and with sequential fp32
single-linear calls through the C ABI (<= 1e-4 relative).  Runs are bitwise
repeatable and the workspace serves any number of consecutive runs.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from epure import _native
    _native.load_library()
    yield
    assert _native.device_error() == 0


def _store(n, k, seed):
    from epure import synthetic
    return synthetic.make_store(n, k, device=DEV, seed=seed, gpu_layout="tiled")


def _exact(st, x64, oracle_mod):
    idx = st.index_rows().cpu().numpy()
    w = oracle_mod.dequantize_f64(idx, st.scale.float().cpu().numpy(), st.cb.float().cpu().numpy(),
                                  st.out_features, st.in_features, 4, 128, 256)
    return x64 @ w.T


def test_small_chain_vs_exact(oracle_mod):
    from epure import _native
    a, b = _store(96, 512, 1), _store(37, 512, 2)
    c = _store(200, 96, 3)
    d1, d2 = _store(64, 200, 4), _store(40, 200, 5)
    steps = [([a, b], 0), ([c], 0), ([d1, d2], 1)]
    ws = _native.chain_prepare(steps)
    x = torch.randn(1, 512, device=DEV).to(torch.bfloat16)
    out = torch.empty(1, 40, device=DEV)
    _native.chain_run(ws, x, out)
    x64 = x.double().cpu().numpy()
    want = _exact(d2, _exact(c, _exact(a, x64, oracle_mod), oracle_mod), oracle_mod)
    got = out.double().cpu().numpy()
    assert oracle_mod.rel_err(got, want) <= 1e-4


def _sequential(steps, x):
    """fp32 single-linear calls (general kernel), chained through each step's feed."""
    from epure import _native
    h = x.float()
    for stores, feed in steps:
        h = _native.linear(h, stores[feed], out_dtype=torch.float32)
    return h


def test_8b_layers_vs_sequential():
    from epure import _native, synthetic
    stack = synthetic.LinearStack(synthetic.LLAMA3_8B, layers=2, device=DEV, seed=77,
                                  gpu_layout="tiled")
    steps = stack.chain_steps()
    ws = _native.chain_prepare(steps)
    outs = []
    for r in range(3):                       # consecutive runs on one workspace
        x = (torch.randn(1, 4096, device=DEV) * (1 + r)).to(torch.bfloat16)
        out = torch.empty(1, 4096, device=DEV)
        _native.chain_run(ws, x, out)
        want = _sequential(steps, x)
        err = float((out - want).abs().max() / want.abs().max())
        assert err <= 1e-4, (r, err)
        outs.append((x, out.clone()))
    # bitwise repeatable
    x, first = outs[0]
    again = torch.empty_like(first)
    _native.chain_run(ws, x, again)
    assert torch.equal(again, first)


def test_chained_stack_runner_and_graph():
    from epure import synthetic
    from epure.decode import ChainedLinearStack
    stack = synthetic.LinearStack(synthetic.QWEN3_1_7B, layers=3, device=DEV, seed=5,
                                  gpu_layout="tiled")
    runner = ChainedLinearStack(stack).capture()
    xh = torch.randn(1, 2048).to(torch.bfloat16).pin_memory()
    oh = runner(xh)
    torch.cuda.synchronize()
    want = _sequential(stack.chain_steps(), xh.to(DEV)).cpu()
    assert float((oh.float() - want).abs().max() / want.abs().max()) <= 1e-2   # bf16 output


def test_chain_rejects_bad_wiring():
    from epure import _native
    a = _store(96, 512, 1)
    b = _store(64, 100, 2)                   # k=100 != 96
    with pytest.raises(RuntimeError, match="input width"):
        _native.chain_prepare([([a], 0), ([b], 0)])
    m = __import__("epure").synthetic.make_store(64, 512, device=DEV, seed=3, gpu_layout="mma16")
    with pytest.raises(RuntimeError, match="EPQ_LAYOUT_TILED"):
        _native.chain_prepare([([m], 0)])


@pytest.mark.parametrize("n_steps", [1, 2, 3, 4, 5, 6])
def test_many_consecutive_runs_any_length(n_steps, oracle_mod):
    """Tagged partials in a ring of three buffers: whatever the chain length, each
    of many consecutive runs (different inputs) reads only the current step's
    partials -- a stale word from an earlier step or run would show up here."""
    from epure import _native
    widths = [256, 384, 128, 512, 256, 384, 256]
    stores = [_store(widths[i + 1], widths[i], 40 + i) for i in range(n_steps)]
    steps = [([st], 0) for st in stores]
    ws = _native.chain_prepare(steps)
    for r in range(17):
        x = (torch.randn(1, widths[0], device=DEV) * (1 + 0.1 * r)).to(torch.bfloat16)
        out = torch.empty(1, widths[n_steps], device=DEV)
        _native.chain_run(ws, x, out)
        h = x.double().cpu().numpy()
        for st in stores:
            h = _exact(st, h, oracle_mod)
        assert oracle_mod.rel_err(out.double().cpu().numpy(), h) <= 1e-4, (n_steps, r)
