"""The tensor-core backward on the GPU: dX = dY W and dscale, dcb from dY^T X tiles.

With 16-bit activations and m >= 64, epq_linear_bwd computes dscale and dcb on
the tensor cores: dW = dY^T X in fp32 (exact products of the 16-bit inputs,
fp32 accumulation) reduced in the epilogue, dW never written.  Compared with
the float64 gradients of the same 16-bit inputs (the autograd of
materialize + F.linear, oracle.grads_reference): <= 2e-4 relative per tensor;
and with the general (SIMT) kernel on fp32 copies of the same inputs.  dX
(W decoded along its rows into tensor memory, exactly the reference's bf16
weight) in fp32 equals the float64 product dY W_bf16 to fp32 accumulation noise.
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


@pytest.fixture(params=["mma16", "tiled"])
def gpu_layout(request):
    from epure import PackedWeight
    old = PackedWeight.GPU_LAYOUT
    PackedWeight.GPU_LAYOUT = request.param
    yield request.param
    PackedWeight.GPU_LAYOUT = old


def _inputs(m, n, k, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(m, k, generator=g, device=DEV).to(dtype)
    dy = (torch.randn(m, n, generator=g, device=DEV) * 0.1).to(dtype)
    return x, dy


def _want(O, st, x, dy):
    idx = st.index_rows().cpu().numpy()
    sc = st.scale.detach().float().cpu().numpy()
    cb = st.cb.detach().float().cpu().numpy()
    return O.grads_reference(x.double().cpu().numpy(), dy.double().cpu().numpy(), idx, sc, cb,
                             st.out_features, st.in_features, 4, 128, 256)


def _rel(a, b):
    a = a.detach().double().cpu().numpy().reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("n,k,m", [(128, 128, 64), (200, 256, 100), (1024, 4096, 256),
                                   (6144, 2048, 512), (96, 1024, 1000)])
def test_dscale_dcb_vs_float64(n, k, m, oracle_mod, gpu_layout):
    from epure import _native, synthetic
    st = synthetic.make_store(n, k, device=DEV, seed=n + k)
    assert st.layout == gpu_layout
    x, dy = _inputs(m, n, k, seed=m)
    _, dscale, dcb = _native.linear_bwd(x, dy, st, need_dx=False)
    _, want_ds, want_dcb = _want(oracle_mod, st, x, dy)
    assert _rel(dscale, want_ds) <= 2e-4
    assert _rel(dcb, want_dcb) <= 2e-4


def test_matches_general_kernel_and_dx_path(oracle_mod):
    """The tensor-core reduction agrees with the SIMT kernel on fp32 copies; dX is unchanged."""
    from epure import _native, synthetic
    st = synthetic.make_store(512, 1024, device=DEV, seed=3)
    x, dy = _inputs(192, 512, 1024, seed=4)
    dx16, ds16, dcb16 = _native.linear_bwd(x, dy, st)
    dx32, ds32, dcb32 = _native.linear_bwd(x.float(), dy.float(), st)
    assert _rel(ds16, ds32.double().cpu().numpy()) <= 2e-4
    assert _rel(dcb16, dcb32.double().cpu().numpy()) <= 2e-4
    want_dx, _, _ = _want(oracle_mod, st, x, dy)
    assert _rel(dx16.float(), want_dx) <= 1e-2          # bf16 output
    assert _rel(dx32, want_dx) <= 1e-5


def test_fp16_and_trainable_fp32_scales(oracle_mod):
    from epure import _native, synthetic
    st = synthetic.make_store(256, 512, device=DEV, seed=8, scale_dtype=torch.float32)
    x, dy = _inputs(128, 256, 512, seed=9, dtype=torch.float16)
    _, dscale, dcb = _native.linear_bwd(x, dy, st, need_dx=False)
    _, want_ds, want_dcb = _want(oracle_mod, st, x, dy)
    assert _rel(dscale, want_ds) <= 2e-4
    assert _rel(dcb, want_dcb) <= 2e-4


def test_autograd_fine_tune_step(oracle_mod):
    """make_trainable + a bf16 forward/backward through PackedLinear reaches the fused kernels."""
    import torch.nn as nn
    from epure import PackedLinear, make_trainable, snapshot_indices, synthetic, verify_frozen
    st = synthetic.make_store(384, 1024, device=DEV, seed=12)
    model = nn.Module()
    model.proj = PackedLinear(st)
    snap = snapshot_indices(model)
    make_trainable(model, mode="both", verbose=False)
    x, gy = _inputs(256, 384, 1024, seed=13)
    (model.proj(x).float() * gy.float()).sum().backward()
    s = model.proj.store
    _, want_ds, want_dcb = _want(oracle_mod, s, x, gy)
    assert _rel(s.scale.grad, want_ds) <= 2e-4
    assert _rel(s.cb.grad.reshape(-1), want_dcb) <= 2e-4
    verify_frozen(model, snap)


def _w16_f64(O, st, dtype="bfloat16"):
    idx = st.index_rows().cpu().numpy()
    return O.materialize(idx, st.scale.detach().float().cpu().numpy(), st.cb.detach().float().cpu().numpy(),
                         st.out_features, st.in_features, 4, 128, 256, dtype).astype(np.float64)


@pytest.mark.parametrize("n,k,m", [(128, 128, 64), (192, 256, 100), (1024, 4096, 256),
                                   (6144, 2048, 512), (64, 1024, 17), (2048, 512, 300)])
def test_dx_tensor_cores(n, k, m, oracle_mod, gpu_layout):
    from epure import _native, synthetic
    O = oracle_mod
    st = synthetic.make_store(n, k, device=DEV, seed=2 * n + k)
    x, dy = _inputs(m, n, k, seed=m + 1)
    dx32, _, _ = _native.linear_bwd(x, dy, st, need_dscale=False, need_dcb=False,
                                    dx_dtype=torch.float32)
    want = dy.double().cpu().numpy() @ _w16_f64(O, st)
    assert _rel(dx32, want) <= (1e-5 if n <= 4096 else 3e-5)
    dx16, _, _ = _native.linear_bwd(x, dy, st, need_dscale=False, need_dcb=False)
    want_dx, _, _ = _want(O, st, x, dy)
    assert _rel(dx16.float(), want_dx) <= 1e-2


def test_dx_fp16_and_fp32_scales(oracle_mod):
    from epure import _native, synthetic
    O = oracle_mod
    st = synthetic.make_store(256, 512, device=DEV, seed=21, scale_dtype=torch.float32)
    x, dy = _inputs(96, 256, 512, seed=22, dtype=torch.float16)
    dx32, _, _ = _native.linear_bwd(x, dy, st, need_dscale=False, need_dcb=False,
                                    dx_dtype=torch.float32)
    want = dy.double().cpu().numpy() @ _w16_f64(O, st, "float16")
    assert _rel(dx32, want) <= 1e-5
