"""The container reader and the loader (epure.container, epure.runtime.apply_to /
read_stores / resolve / _runtime_dtype) on small synthetic ``.ebin`` files.

The containers are written by tests/ebin_synth.py with raw (uncoded) index
streams and read with ``rans_decode`` swapped for an identity decoder -- the
rANS coder ``constriction`` is not installed here.  ``apply_to`` is compared
with what the reference's own ``apply_to`` did with the same files
(tests/golden/loader_l*.json, made by tests/golden/make_loader_golden.py):
which module each tensor lands in (embedding, linear with its bias, dense
convolution and router, packed expert slab, tied lm_head), and the values.
"""
import json
import os
import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import ebin_synth as S
from conftest import GOLDEN, golden_cases, load_golden


@pytest.fixture
def identity_codec(monkeypatch):
    from epure import container
    monkeypatch.setattr(container, "rans_decode", S.identity_decode)


def _close(a, b, rel):
    return abs(a - b) <= rel * max(abs(b), 1e-12)


@pytest.mark.parametrize("levels", [16, 256])
def test_apply_to_matches_reference(levels, tmp_path, identity_codec):
    from epure import apply_to
    with open(os.path.join(GOLDEN, f"loader_l{levels}.json")) as f:
        want = json.load(f)
    path = str(tmp_path / "toy.ebin")
    S.make_container(path, levels=levels, group=16)
    model = S.toy_model()
    apply_to(model, path, device="cpu", cfg=model.config, verbose=False, dtype=torch.float32)
    assert S.describe_model(model) == want["structure"]
    assert model.config.tie_word_embeddings is want["tie_flag"] is False
    assert (model.lm_head.store is model.model.embed_tokens.store) is want["lm_head_is_embedding_store"]
    got = {n: float(p.double().sum()) for n, p in model.named_parameters()}
    assert got.keys() == want["dense_sums"].keys()
    for n, v in want["dense_sums"].items():
        assert _close(got[n], v, 1e-6), n
    x = torch.linspace(-1, 1, 32)
    layer = model.model.layers[0]
    assert _close(float(layer.self_attn.q_proj(x[None]).double().sum()), want["q_proj_out_sum"], 1e-5)
    assert _close(float(model.model.embed_tokens(torch.tensor([[1, 5, 63]])).double().sum()),
                  want["embed_rows_sum"], 1e-5)
    assert _close(float(model.lm_head(x[None]).double().sum()), want["lm_head_out_sum"], 1e-5)


def test_packed_values_and_expert_slab(tmp_path, identity_codec):
    from epure import apply_to, container
    path = str(tmp_path / "toy.ebin")
    vals = S.make_container(path, levels=16, group=16)
    model = S.toy_model()
    apply_to(model, path, cfg=model.config, verbose=False, dtype=torch.float32)
    layer = model.model.layers[0]
    idx, sc, cb = vals["model.layers.0.self_attn.q_proj.weight"]
    w = torch.from_numpy(container.dequantize(idx, sc, cb, (48, 32), 16))
    x = torch.randn(3, 32)
    assert torch.allclose(layer.self_attn.q_proj(x), F.linear(x, w, layer.self_attn.q_proj.bias), atol=1e-5)
    # the expert slab is dense only while its owner runs
    assert layer.mlp.experts.gate_up is None
    layer.mlp.experts(torch.randn(32))
    idx, sc, cb = vals["model.layers.0.mlp.experts.gate_up"]
    slab = container.dequantize(idx, sc, cb, (4, 16, 32), 16)
    assert torch.equal(layer.mlp.experts.seen, torch.from_numpy(slab))
    assert layer.mlp.experts.gate_up is None
    assert len(model._epure_holders) == 1


def test_vector_codebook_container(tmp_path, identity_codec):
    from epure import container
    from epure.runtime import read_stores
    spec = [("layers.0.mlp.up_proj.weight", (40, 256), True), ("layers.0.mlp.down_proj.weight", (24, 256), True)]
    path = str(tmp_path / "vec.ebin")
    vals = S.make_container(path, levels=256, group=128, vec=4, spec=spec)
    stores = read_stores(path)
    for name, (idx, sc, cb) in vals.items():
        st = stores[name]
        assert st.vec == 4 and cb.shape == (256, 4)
        want = container.dequantize(idx, sc, cb, st.shape, 128)
        assert np.array_equal(st.materialize(torch.float32).numpy(), want)


@pytest.mark.parametrize("world", [2, 4])
def test_read_stores_cuts_tensor_parallel_shards(tmp_path, identity_codec, world):
    from epure.runtime import read_stores
    spec = [("l.0.self_attn.q_proj.weight", (64, 512), True), ("l.0.self_attn.o_proj.weight", (32, 512), True),
            ("l.0.mlp.gate_proj.weight", (48, 512), True), ("l.0.mlp.down_proj.weight", (32, 512), True),
            ("embed_tokens.weight", (16, 512), True)]
    path = str(tmp_path / "tp.ebin")
    S.make_container(path, levels=256, group=128, vec=4, spec=spec)
    full = read_stores(path)
    for rank in range(world):
        part = read_stores(path, tp=(rank, world))
        for name, st in full.items():
            w, ws = st.materialize(torch.float32), part[name].materialize(torch.float32)
            if "q_proj" in name or "gate_proj" in name:
                n = st.out_features // world
                assert torch.equal(ws, w[rank * n:(rank + 1) * n])
            elif "o_proj" in name or "down_proj" in name:
                k = st.in_features // world
                assert torch.equal(ws, w[:, rank * k:(rank + 1) * k])
            else:
                assert torch.equal(ws, w)


@pytest.mark.parametrize("case", golden_cases())
def test_dequantize_matches_reference(case):
    """container.dequantize against the reference's (bit-exact float32)."""
    from epure import container
    z = load_golden(case)
    n, k, vec, levels = z["n"], z["k"], z["vec"], z["levels"]
    if vec == 4:
        idx, cb = z["idx_rows"], z["cb"].reshape(levels, 4)
    else:
        raw = z["idx_rows"]
        if levels <= 16:       # the reference's nibble-packed bytes, even position low
            raw = np.stack([raw & 0x0F, raw >> 4], axis=-1).reshape(-1)[:n * k]
        idx, cb = raw.reshape(n, k), z["cb"]
    got = container.dequantize(idx, z["scale"], cb, (n, k), z["group"])
    assert got.dtype == np.float32
    assert np.array_equal(got, z["dequant"])


def test_container_errors_and_summary(tmp_path, identity_codec):
    from epure import container
    path = str(tmp_path / "toy.ebin")
    S.make_container(path, levels=16, group=16)
    d = container.describe(path)
    assert d["compressed_tensors"] == 5 and d["raw_tensors"] == 2 and d["levels"] == 16
    assert container.extras(path) == {"config.json": b'{"model_type": "toy"}'}
    bad = tmp_path / "bad.ebin"
    bad.write_bytes(b"NOTEBIN!" + b"\0" * 16)
    with pytest.raises(ValueError):
        container.read_header(str(bad))
    short = tmp_path / "short.ebin"
    short.write_bytes(S.MAGIC + b"\1\2")
    with pytest.raises(ValueError):
        container.read_header(str(short))
    assert np.allclose(container.symbol_probabilities([0, 1, 2]), [0.25, 0.25, 0.5])


def test_resolve_and_runtime_dtype(tmp_path):
    from epure.runtime import _runtime_dtype, resolve
    f = tmp_path / "m.ebin"
    f.write_bytes(b"")
    assert resolve(str(f)) == str(f)
    with pytest.raises(FileNotFoundError):
        resolve("no-such-file.ebin")
    with pytest.raises(FileNotFoundError):
        resolve(str(tmp_path / "missing" / "m.ebin"))
    ns = types.SimpleNamespace
    assert _runtime_dtype(ns(torch_dtype="bfloat16"), "cpu") is torch.float32
    assert _runtime_dtype(ns(torch_dtype=None, dtype="float16"), "cuda") is torch.float16
    want = torch.bfloat16 if torch.cuda.is_available() and torch.cuda.is_bf16_supported() else torch.float32
    assert _runtime_dtype(ns(torch_dtype="bfloat16", dtype="float16"), "cuda") is want


def test_parameters_on_meta_keeps_buffers():
    from epure.runtime import _parameters_on_meta

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(4, 4)
            self.register_buffer("inv_freq", torch.arange(3.0))

    with _parameters_on_meta():
        m = M()
    assert m.lin.weight.device.type == "meta"
    assert torch.equal(m.inv_freq, torch.arange(3.0))
    assert torch.nn.Module.register_parameter.__name__ == "register_parameter"
