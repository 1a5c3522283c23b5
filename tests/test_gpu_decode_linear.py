"""The batch-1..16 tensor-core GEMV and its fused decode launches (epq_decode_linear).

* The GEMV contracts the reference's own bf16 / fp16 weight: with an fp32
  output it equals the float64 product of x and ``materialize(dtype)``
  (runtime.py:78-89, bit-exact on the GPU) to fp32 summation error, 1e-5
  relative (5e-5 at k = 14336).
* The fused prologue / epilogues reproduce the block's torch formulation
  (RMSNorm in fp32 rounded to bf16, the residual add of two bf16 tensors,
  ``(silu(g.float()) * u.float()).to(bf16)``) to bf16 rounding: max error
  within 1e-2 of the largest value, on full Llama-3-8B projection shapes.
Every call goes through the C ABI (include/epq_decode.h, include/epq.h).
"""
import pytest
import torch
import torch.nn.functional as F

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


def _store(n, k, seed, scale_dtype=torch.float16):
    from epure import synthetic
    return synthetic.make_store(n, k, device=DEV, seed=seed, gpu_layout="mma16", scale_dtype=scale_dtype)


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _rms(x, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


@pytest.mark.parametrize("n,k", [(64, 2048), (37, 256), (6144, 4096), (4096, 14336), (200, 640)])
@pytest.mark.parametrize("m", [1, 3, 8, 16])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemv_contracts_reference_weight(n, k, m, dtype):
    from epure import _native
    st = _store(n, k, seed=n + k + m)
    x = torch.randn(m, k, device=DEV).to(dtype)
    w = st.materialize(dtype)                                       # the reference's weight
    want = x.double() @ w.double().T
    (got32,) = _native.linear_multi(x, [st], out_dtype=torch.float32)
    assert _rel(got32, want) <= (5e-5 if k > 4096 else 1e-5)
    (got,) = _native.linear_multi(x, [st])
    assert _rel(got, F.linear(x, w)) <= 1e-2


def test_gemv_fp32_trainable_scales():
    """fp32 scales (after make_trainable) are rounded to the activation type first."""
    from epure import _native
    st = _store(512, 2048, seed=3, scale_dtype=torch.float32)
    x = torch.randn(2, 2048, device=DEV).to(torch.bfloat16)
    (got32,) = _native.linear_multi(x, [st], out_dtype=torch.float32)
    assert _rel(got32, x.double() @ st.materialize(torch.bfloat16).double().T) <= 1e-5


@pytest.mark.parametrize("m", [1, 2])
def test_rmsnorm_prologue_and_residual(m):
    from epure import _native
    eps = 1e-5
    qkv = [_store(4096, 4096, 1), _store(1024, 4096, 2), _store(1024, 4096, 3)]
    o = _store(4096, 4096, 4)
    h = torch.randn(m, 4096, device=DEV).to(torch.bfloat16)
    outs = _native.decode_linear(h, qkv, prologue=_native.PRO_RMSNORM, eps=eps)
    y = _rms(h, eps)
    for got, st in zip(outs, qkv):
        assert _rel(got, F.linear(y, st.materialize(torch.bfloat16))) <= 1e-2
    att = torch.randn(m, 4096, device=DEV).to(torch.bfloat16)
    want = h + F.linear(att, o.materialize(torch.bfloat16))
    h2 = h.clone()
    _native.decode_linear(att, [o], epilogue=_native.EPI_RESIDUAL, outs=[h2])
    assert _rel(h2, want) <= 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_silu_pair_epilogue(dtype):
    from epure import _native
    eps = 1e-6
    gate, up = _store(14336, 4096, 5), _store(14336, 4096, 6)
    h = torch.randn(1, 4096, device=DEV).to(dtype)
    (a,) = _native.decode_linear(h, [gate, up], prologue=_native.PRO_RMSNORM,
                                 epilogue=_native.EPI_SILU_MUL, eps=eps)
    y = _rms(h, eps)
    g = F.linear(y, gate.materialize(dtype))
    u = F.linear(y, up.materialize(dtype))
    want = (F.silu(g.float()) * u.float()).to(dtype)
    assert a.shape == (1, 14336)
    assert _rel(a, want) <= 1e-2


def test_fused_chain_is_deterministic():
    """Two runs of the same fused layer give bitwise equal results."""
    from epure import _native
    gate, up, down = _store(6144, 2048, 7), _store(6144, 2048, 8), _store(2048, 6144, 9)
    h0 = torch.randn(1, 2048, device=DEV).to(torch.bfloat16)
    res = []
    for _ in range(2):
        h = h0.clone()
        (a,) = _native.decode_linear(h, [gate, up], prologue=_native.PRO_RMSNORM,
                                     epilogue=_native.EPI_SILU_MUL)
        _native.decode_linear(a, [down], epilogue=_native.EPI_RESIDUAL, outs=[h])
        res.append(h)
    assert torch.equal(res[0], res[1])


def test_decode_linear_rejects_bad_combinations():
    from epure import _native
    a, b = _store(64, 1024, 10), _store(32, 1024, 11)
    x = torch.randn(1, 1024, device=DEV).to(torch.bfloat16)
    with pytest.raises(RuntimeError):
        _native.decode_linear(x, [a, b], epilogue=_native.EPI_SILU_MUL)        # unequal rows
    h = torch.zeros(1, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        _native.decode_linear(x, [a, a], epilogue=_native.EPI_RESIDUAL, outs=[h, h])
    big = _store(64, 40960, 12)
    xb = torch.randn(1, 40960, device=DEV).to(torch.bfloat16)
    with pytest.raises(RuntimeError):
        _native.decode_linear(xb, [big], prologue=_native.PRO_RMSNORM)       # x too large to stage
