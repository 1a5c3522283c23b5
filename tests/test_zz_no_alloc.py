"""epq_linear_noalloc: the batch-1 linear for callers that cannot allocate.

Some callers cannot call cudaMalloc where they run the op -- a plugin inside a
serving engine whose memory manager owns the whole device, or a loop where an
allocation could block or fail.  epq_linear_noalloc serves them with a
library-owned static device scratch instead of a caller workspace.  This test
calls it through the C ABI twice in a row and checks each result against the
regular entry point (epq_linear_multi with a workspace) on the same inputs.
It lives in its own file, collected last, and passes both alone in a fresh
process and after the other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from epure import _native
    return _native.load_library()


def _tiled_stores(shapes, seed):
    from epure import PackedWeight, synthetic
    old = PackedWeight.GPU_LAYOUT
    PackedWeight.GPU_LAYOUT = "tiled"
    try:
        sts = [synthetic.make_store(n, k, device=DEV, seed=seed + i) for i, (n, k) in enumerate(shapes)]
    finally:
        PackedWeight.GPU_LAYOUT = old
    assert all(s.layout == "tiled" for s in sts)
    return sts


def _noalloc(lib, stores, x):
    from epure import _native
    count = len(stores)
    descs = (_native.EpqStore * count)(*[_native.describe_store(s) for s in stores])
    outs = [torch.empty(1, s.out_features, dtype=x.dtype, device=DEV) for s in stores]
    ptrs = (ctypes.c_void_p * count)(*[o.data_ptr() for o in outs])
    rc = lib.epq_linear_noalloc(descs, count, x.data_ptr(), _native.dtype_code(x.dtype), ptrs,
                                _native.dtype_code(x.dtype),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.epq_last_error()
    return outs


@pytest.mark.parametrize("shapes,dtype", [
    ([(6144, 2048)], torch.bfloat16),
    ([(4096, 4096), (1024, 4096), (1024, 4096)], torch.bfloat16),
    ([(37, 200)], torch.float32),
])
def test_noalloc_matches_workspace_entry_point(lib, shapes, dtype):
    from epure import _native
    stores = _tiled_stores(shapes, seed=900)
    for call in range(2):
        x = torch.randn(1, shapes[0][1], device=DEV).to(dtype)
        got = _noalloc(lib, stores, x)
        want = _native.linear_multi(x, stores)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            err = float((g.float() - w.float()).abs().max() / w.float().abs().max())
            assert err <= 1e-5, (call, err)
    assert _native.device_error() == 0


def test_noalloc_rejects_oversized_and_unsupported(lib):
    from epure import _native
    assert lib.epq_linear_noalloc_max_scratch() == 4 << 20
    # 8192 x 28672 needs 224 groups x 512 row blocks x 16 x 4 B of partial sums (> 4 MiB).
    big = _tiled_stores([(8192, 28672)], seed=5)
    x = torch.randn(1, 28672, device=DEV).to(torch.bfloat16)
    d = (_native.EpqStore * 1)(_native.describe_store(big[0]))
    out = torch.empty(1, 8192, dtype=torch.bfloat16, device=DEV)
    ptrs = (ctypes.c_void_p * 1)(out.data_ptr())
    rc = lib.epq_linear_noalloc(d, 1, x.data_ptr(), 2, ptrs, 2, None)
    assert rc == -6 and b"static scratch" in lib.epq_last_error()
    # A row-layout store is not served by this entry point.
    from epure import synthetic
    rows = synthetic.make_store(64, 256, vec=1, device="cpu", seed=1).to(DEV)
    d = (_native.EpqStore * 1)(_native.describe_store(rows))
    xs = torch.randn(1, 256, device=DEV)
    o = torch.empty(1, 64, device=DEV)
    rc = lib.epq_linear_noalloc(d, 1, xs.data_ptr(), 0, (ctypes.c_void_p * 1)(o.data_ptr()), 0, None)
    assert rc == -8


def test_noalloc_rejects_too_many_row_blocks(lib):
    """More 16-row blocks than the static scratch has completion counters (16384):
    refused before launch, although the partial sums themselves would fit."""
    from epure import _native
    stores = _tiled_stores([(70000, 128)] * 4, seed=40)          # 4 x 4375 row blocks
    x = torch.randn(1, 128, device=DEV).to(torch.bfloat16)
    d = (_native.EpqStore * 4)(*[_native.describe_store(s) for s in stores])
    outs = [torch.empty(1, 70000, dtype=torch.bfloat16, device=DEV) for _ in stores]
    ptrs = (ctypes.c_void_p * 4)(*[o.data_ptr() for o in outs])
    rc = lib.epq_linear_noalloc(d, 4, x.data_ptr(), 2, ptrs, 2, None)
    assert rc == -8 and b"row blocks" in lib.epq_last_error()


def test_noalloc_large_then_small_then_large(lib):
    """Calls of different sizes in a row reuse the one static scratch: the counters a
    large call used must not leak into the next, smaller one (or back)."""
    from epure import _native
    big = _tiled_stores([(6144, 2048), (1024, 2048)], seed=60)
    small = _tiled_stores([(37, 200)], seed=70)
    for stores in (big, small, big, small):
        x = torch.randn(1, stores[0].in_features, device=DEV).to(torch.bfloat16)
        got = _noalloc(lib, stores, x)
        want = _native.linear_multi(x, stores)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            assert float((g.float() - w.float()).abs().max() / w.float().abs().max()) <= 1e-5
    assert _native.device_error() == 0
