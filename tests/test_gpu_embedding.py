"""Packed embedding rows on the GPU (epq_embedding behind PackedEmbedding.forward).

PackedEmbedding (runtime.py:129-160) returns the rows of the dequantised table
for a batch of ids with materialize's rounding.  On a CUDA tensor it now decodes
only those rows in one kernel; the result must equal the same rows of the
materialised table bit for bit, for every store format and output dtype.
"""
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


FORMATS = [
    dict(vec=1, levels=16, group=64),       # the reference's 4-bit scalar codebook
    dict(vec=1, levels=256, group=128),     # 8-bit scalar codebook
    dict(vec=4, levels=256, group=128, gpu_layout="mma16"),
    dict(vec=4, levels=256, group=128, gpu_layout="tiled"),
]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_embedding_rows_equal_materialized_rows(fmt, dtype):
    from epure import synthetic
    from epure.runtime import PackedEmbedding
    st = synthetic.make_store(300, 512, device=DEV, seed=7, **fmt)
    g = torch.Generator(device=DEV).manual_seed(1)
    ids = torch.randint(0, 300, (3, 5), generator=g, device=DEV)
    ids[0, 0] = ids[2, 4] = 299                 # repeated id and the last row
    got = PackedEmbedding(st, dtype=dtype)(ids)
    want = st.materialize(dtype)[ids]
    assert got.shape == (3, 5, 512) and got.dtype == dtype
    assert torch.equal(got, want)


def test_embedding_empty_batch():
    from epure import synthetic
    from epure.runtime import PackedEmbedding
    st = synthetic.make_store(64, 256, device=DEV, seed=2)
    out = PackedEmbedding(st, dtype=torch.bfloat16)(torch.zeros(0, dtype=torch.long, device=DEV))
    assert out.shape == (0, 256)


def test_negative_ids_count_from_the_end():
    """As torch indexing does: id -1 is the last row."""
    from epure import synthetic
    from epure.runtime import PackedEmbedding
    st = synthetic.make_store(100, 256, device=DEV, seed=4)
    ids = torch.tensor([[-1, 0, -100, 5]], device=DEV)
    got = PackedEmbedding(st, dtype=torch.bfloat16)(ids)
    w = st.materialize(torch.bfloat16)
    assert torch.equal(got[0], w[torch.tensor([99, 0, 0, 5], device=DEV)])


def test_ids_on_the_host_are_moved_to_the_store(monkeypatch):
    from epure import _native, synthetic
    from epure.runtime import PackedEmbedding
    st = synthetic.make_store(64, 256, device=DEV, seed=5)
    ids = torch.tensor([3, 63, 0])
    got = _native.embedding(st, ids, torch.bfloat16)
    assert got.device == st.packed.device
    assert torch.equal(got, st.materialize(torch.bfloat16)[ids.to(DEV)])
    monkeypatch.setattr(_native, "CHECK_IDS", True)
    with pytest.raises(IndexError):
        PackedEmbedding(st, dtype=torch.bfloat16)(torch.tensor([64], device=DEV))
