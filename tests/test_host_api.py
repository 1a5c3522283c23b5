"""The drop-in host API (epure.runtime / epure.finetune) on the CPU, against the
reference's recorded outputs.  No GPU is needed: on the CPU a PackedLinear runs
the fused CPU kernel for f32 activations and materializes for 16-bit ones (and
whenever gradients are needed), as the reference does with its Rust extension."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import golden_cases, load_golden


def _store(z):
    from epure import PackedWeight
    cb = z["cb"]
    return PackedWeight((z["n"], z["k"]), z["idx_rows"].ravel().copy(), z["scale"].copy(),
                        cb.copy(), z["group"], z["levels"], vec=z["vec"])


@pytest.mark.parametrize("case", golden_cases())
def test_materialize_matches_reference(case):
    z = load_golden(case)
    st = _store(z)
    assert torch.equal(st.materialize(torch.float32), torch.from_numpy(z["w32"]))
    assert torch.equal(st.materialize(torch.bfloat16).float(), torch.from_numpy(z["wbf"]))


@pytest.mark.parametrize("case", golden_cases())
def test_packed_linear_cpu_matches_reference(case):
    from epure import PackedLinear
    z = load_golden(case)
    lin = PackedLinear(_store(z))
    x = torch.from_numpy(z["x"])
    out = lin(x.to(torch.bfloat16))
    assert torch.equal(out.float(), torch.from_numpy(z["outbf"]))
    out32 = lin(x)
    assert torch.allclose(out32, torch.from_numpy(z["out32"]), rtol=0, atol=1e-5)


class _Holder(nn.Module):
    def __init__(self, st):
        super().__init__()
        self.proj = __import__("epure").PackedLinear(st)

    def forward(self, t):
        return self.proj(t)


@pytest.mark.parametrize("case", golden_cases())
def test_finetune_gradients_cpu(case):
    from epure import make_trainable, snapshot_indices, verify_frozen
    z = load_golden(case)
    model = _Holder(_store(z))
    snap = snapshot_indices(model)
    params = make_trainable(model, mode="both", verbose=False)
    assert len(params) == 2 and all(p.dtype == torch.float32 for p in params)
    x = torch.from_numpy(z["x"]).clone().requires_grad_(True)
    (model(x) * torch.from_numpy(z["gy"])).sum().backward()
    st = model.proj.store
    assert torch.allclose(st.scale.grad, torch.from_numpy(z["dscale"]), rtol=1e-5, atol=1e-7)
    assert torch.allclose(st.cb.grad.reshape(-1), torch.from_numpy(z["dcb"]).reshape(-1),
                          rtol=1e-5, atol=1e-6)
    assert torch.allclose(x.grad, torch.from_numpy(z["dx"]), rtol=1e-5, atol=1e-6)
    assert verify_frozen(model, snap) is True


@pytest.mark.parametrize("case", [c for c in golden_cases() if c.startswith("vec1")])
def test_snapshot_digest_matches_reference(case):
    from epure import snapshot_indices
    z = load_golden(case)
    snap = snapshot_indices(_Holder(_store(z)))
    assert list(snap.values()) == [str(z["snapshot"])]


def test_verify_frozen_detects_moved_index():
    from epure import snapshot_indices, verify_frozen
    z = load_golden("vec1_l16")
    model = _Holder(_store(z))
    snap = snapshot_indices(model)
    model.proj.store.packed[3] ^= 1
    with pytest.raises(RuntimeError, match="proj"):
        verify_frozen(model, snap)


def test_make_trainable_modes_and_tied_store():
    from epure import PackedEmbedding, PackedLinear, make_trainable
    z = load_golden("vec4_l256")
    st = _store(z)
    m = nn.Module()
    m.emb = PackedEmbedding(st, torch.float32)
    m.head = PackedLinear(st)
    with pytest.raises(ValueError):
        make_trainable(m, mode="cb")
    p = make_trainable(m, mode="scale", verbose=False)
    assert len(p) == 1 and p[0] is st.scale
    p2 = make_trainable(m, mode="both", verbose=False)   # idempotent on promoted stores
    assert len(p2) == 2 and p2[0] is st.scale and p2[1] is st.cb


def test_packed_embedding_rows():
    from epure import PackedEmbedding
    z = load_golden("vec4_l256_ragged")
    emb = PackedEmbedding(_store(z), torch.float32)
    ids = torch.tensor([[0, 5, 36], [36, 1, 2]])
    got = emb(ids)
    want = torch.from_numpy(z["w32"])[ids]
    assert torch.equal(got, want)


@pytest.mark.parametrize("layout", ["tiled", "mma16"])
def test_tiled_view_inverts_tiling(layout):
    """index_rows undoes the kernel-native byte orders (numpy model of the relayout kernels)."""
    from epure import PackedWeight
    rng = np.random.default_rng(1)
    n, k, vec, group = 37, 200, 4, 128
    rows = rng.integers(0, 256, (n, k // vec), dtype=np.uint8)
    p, ng = group // vec, -(-k // group)
    if layout == "tiled":
        rb = -(-n // 16)
        buf = np.zeros((ng, rb, p, 16), np.uint8)
        for r in range(n):
            for j in range(k // vec):
                buf[j // p, r // 16, j % p, r % 16] = rows[r, j]
    else:
        rb = -(-n // 16)
        buf = np.zeros((rb, ng, 32, 16), np.uint8)
        for r in range(n):
            for j in range(k // vec):
                jj = j % 32
                buf[r // 16, j // 32, 4 * (r % 8) + jj % 4, 8 * ((r % 16) // 8) + jj // 4] = rows[r, j]
    st = PackedWeight((n, k), rows.ravel(), np.zeros((n, ng), np.float16),
                      np.zeros((256, 4), np.float16), group, 256, vec=4)
    st._buffers["packed"] = torch.from_numpy(buf.ravel())
    st.layout = layout
    assert np.array_equal(st.index_rows().numpy(), rows)
    sel = torch.tensor([0, 17, 36])
    assert np.array_equal(st.index_rows(sel).numpy(), rows[[0, 17, 36]])


def test_cuda_backend_declines_cpu_tensor():
    from epure.kernels import cpu, cuda
    z = load_golden("vec4_l256")
    st = _store(z)
    assert cuda.linear(torch.zeros(1, z["k"]), st) is None
    # the CPU backend serves f32 activations and declines 16-bit ones (as the reference's does)
    out = cpu.linear(torch.zeros(1, z["k"]), st)
    assert out is not None and torch.equal(out, torch.zeros(1, z["n"]))
    assert cpu.linear(torch.zeros(1, z["k"], dtype=torch.bfloat16), st) is None


def test_synthetic_shapes():
    from epure import synthetic
    s = synthetic.LLAMA3_8B
    assert s.packed_weights() == 32 * (4096 * 4096 * 2 + 1024 * 4096 * 2 + 14336 * 4096 * 3)
    assert abs(synthetic.QWEN3_1_7B.packed_weights() - 1.409e9) / 1.409e9 < 0.01
