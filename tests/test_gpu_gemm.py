"""The tensor-core dequant-GEMM (tcgen05, batches of more than 16 rows) on the GPU.

The kernel dequantises each weight exactly as the reference's bf16 path does
(``cb.to(bf16)[idx] * scale.to(bf16)``, rounded to bf16; runtime.py:78-89) and
accumulates ``x @ W^T`` in fp32 on the tensor cores.  So:
* fp32 outputs equal the float64 product of the bf16-rounded operands to fp32
  accumulation noise (<= 1e-5 relative): this pins the decoded weights to the
  reference's materialize(bf16) bit for bit;
* bf16 outputs are within 1e-2 of the reference's F.linear(x, materialize(bf16))
  and within 8e-3 of the exact float64 product;
* the result matches torch's own bf16 GEMM on the materialised weight.
Every call goes through the C ABI (epq_linear / epq_linear_multi).
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


def _store(n, k, seed, **kw):
    from epure import synthetic
    return synthetic.make_store(n, k, device=DEV, seed=seed, **kw)


def _x(m, k, dtype=torch.bfloat16, seed=3):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(m, k, generator=g, device=DEV).to(dtype)


def _oracle_in(st):
    return (st.index_rows().cpu().numpy(), st.scale.float().cpu().numpy(),
            st.cb.float().cpu().numpy())


def _bf16_operands_f64(O, st, x, dtype="bfloat16"):
    """float64 product of the dtype-rounded activations and materialize(dtype)."""
    idx, sc, cb = _oracle_in(st)
    n, k = st.out_features, st.in_features
    w = O.materialize(idx, sc, cb, n, k, 4, 128, 256, dtype).astype(np.float64)
    return x.float().cpu().numpy().astype(np.float64) @ w.T


@pytest.mark.parametrize("m", [17, 64, 100, 256, 300])
def test_config0_fp32_out_pins_bf16_weights(m, oracle_mod, gpu_layout):
    """K=2048, N=6144: fp32 outputs = exact product of bf16 operands (fp32 accumulation)."""
    from epure import _native
    O = oracle_mod
    st = _store(6144, 2048, seed=0)
    assert st.layout == gpu_layout
    x = _x(m, 2048)
    with torch.no_grad():
        out = _native.linear(x, st, out_dtype=torch.float32).cpu().numpy()
    want = _bf16_operands_f64(O, st, x)
    assert O.rel_err(out, want) <= 1e-5


@pytest.mark.parametrize("m", [17, 128, 2048])
def test_config0_bf16_vs_reference(m, oracle_mod, gpu_layout):
    """bf16 outputs vs the reference's bf16 path and vs the exact product."""
    from epure.kernels import cuda
    O = oracle_mod
    st = _store(6144, 2048, seed=1)
    x = _x(m, 2048, seed=4)
    with torch.no_grad():
        out = cuda.linear(x, st).float().cpu().numpy()
    idx, sc, cb = _oracle_in(st)
    xs = x.float().cpu().numpy()
    ref = O.round_bf16(_bf16_operands_f64(O, st, x).astype(np.float32))
    assert O.rel_err(out, ref) <= 1e-2
    exact = O.linear_exact(xs, idx, sc, cb, 6144, 2048, 4, 128, 256)
    assert O.rel_err(out, exact) <= 8e-3


def test_matches_torch_bf16_gemm(gpu_layout):
    """Same result as the reference's fallback F.linear(x, materialize(bf16)) run by torch."""
    from epure.kernels import cuda
    st = _store(4096, 4096, seed=2)
    x = _x(512, 4096, seed=5)
    with torch.no_grad():
        out = cuda.linear(x, st).float()
        ref = torch.nn.functional.linear(x, st.materialize(torch.bfloat16)).float()
    assert float((out - ref).abs().max() / ref.abs().max()) <= 1e-2
    # identical weights and fp32 accumulation: almost every element is the same bf16 value
    assert float((out != ref).float().mean()) < 0.05


@pytest.mark.parametrize("n,k,m", [(1, 128, 17), (17, 128, 40), (200, 256, 33), (4096, 14336, 64),
                                   (28672, 4096, 24), (1024, 8192, 257), (37, 200, 20)])
def test_shapes_vs_oracle(n, k, m, oracle_mod, gpu_layout):
    """8B/70B shapes, partial row tiles and token tiles (k = 200 runs the general kernel)."""
    from epure import _native
    O = oracle_mod
    st = _store(n, k, seed=n + k)
    x = _x(m, k, seed=7)
    with torch.no_grad():
        out = _native.linear(x, st, out_dtype=torch.float32).cpu().numpy()
    if k % 128 == 0:
        want = _bf16_operands_f64(O, st, x)
        # fp32 accumulation noise grows with k (1.9e-5 measured at k = 14336); the
        # bf16-weight pin itself is the k <= 4096 cases at 1e-5
        assert O.rel_err(out, want) <= (1e-5 if k <= 4096 else 5e-5)
    else:
        idx, sc, cb = _oracle_in(st)
        exact = O.linear_exact(x.float().cpu().numpy(), idx, sc, cb, n, k, 4, 128, 256)
        assert O.rel_err(out, exact) <= 1e-5


def test_fp16_activations_and_fp32_scales(oracle_mod, gpu_layout):
    """fp16 activations decode in fp16; fp32 (trainable) scales round to the activation type."""
    from epure import _native
    O = oracle_mod
    st = _store(640, 1024, seed=11)
    x = _x(96, 1024, dtype=torch.float16, seed=8)
    with torch.no_grad():
        out = _native.linear(x, st, out_dtype=torch.float32).cpu().numpy()
    assert O.rel_err(out, _bf16_operands_f64(O, st, x, "float16")) <= 1e-5
    st32 = _store(640, 1024, seed=12, scale_dtype=torch.float32)
    xb = _x(48, 1024, seed=9)
    with torch.no_grad():
        out = _native.linear(xb, st32, out_dtype=torch.float32).cpu().numpy()
    assert O.rel_err(out, _bf16_operands_f64(O, st32, xb)) <= 1e-5


def test_fused_equals_separate_and_repeatable(gpu_layout):
    """q/k/v fused launch equals single-store launches bit for bit; reruns are identical."""
    from epure.kernels import cuda
    sts = [_store(n, 4096, seed=20 + i) for i, n in enumerate((4096, 1024, 1024))]
    x = _x(200, 4096, seed=10)
    with torch.no_grad():
        fused = cuda.linear_multi(x, sts)
        single = [cuda.linear(x, s) for s in sts]
        again = cuda.linear_multi(x, sts)
    for a, b, c in zip(fused, single, again):
        assert torch.equal(a, b)
        assert torch.equal(a, c)


def test_strided_activations(oracle_mod):
    """A row stride larger than k (a column slice of a wider buffer)."""
    from epure import _native
    O = oracle_mod
    st = _store(256, 512, seed=13)
    big = _x(40, 640, seed=11)
    x = big[:, :512]
    with torch.no_grad():
        out = _native.linear(x, st, out_dtype=torch.float32).cpu().numpy()
    assert O.rel_err(out, _bf16_operands_f64(O, st, x)) <= 1e-5


def test_full_size_prefill_linearity():
    """Prefill of 2048 rows through the 8B gate projection: f(2 x) = 2 f(x) exactly (fp32 out)."""
    from epure import _native
    st = _store(14336, 4096, seed=14)
    x = _x(2048, 4096, seed=12)
    with torch.no_grad():
        a = _native.linear(x, st, out_dtype=torch.float32)
        b = _native.linear((x.float() * 2).to(torch.bfloat16), st, out_dtype=torch.float32)
    assert torch.equal(b, 2 * a)
