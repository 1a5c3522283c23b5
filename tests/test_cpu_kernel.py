"""The CPU fused kernel behind epure.kernels.cpu.linear (libepq_cpu.so, include/epq_cpu.h)
and the fine-tuning loop on the CPU.

* Bit-equal to the C restatement of the reference's Rust kernel
  (oracle/epq_oracle.c, kernel/src/lib.rs:36-151) on every golden store: both
  follow lib.rs's f32 order (per group, unfused multiply then add, group sums
  added in order), so any difference is a bug.
* ``PackedLinear`` on a CPU f32 activation takes that kernel and matches the
  reference's F.linear(x, materialize(f32)) golden to 1e-5; it declines for bf16
  activations and whenever autograd needs gradients (the materialize path then
  runs, as in the reference).
* ``ScaleTuner`` trains a tiny packed language model on the CPU: the loss goes
  down, scales and codebooks move, indices do not (verify_frozen).
"""
import types

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from conftest import golden_cases, load_golden


def _store(z):
    from epure import PackedWeight
    return PackedWeight((z["n"], z["k"]), z["idx_rows"].ravel().copy(), z["scale"].copy(),
                        z["cb"].copy(), z["group"], z["levels"], vec=z["vec"])


@pytest.fixture(scope="module", autouse=True)
def _built():
    from epure.kernels import cpu
    if not cpu.available():
        pytest.fail("libepq_cpu.so is not built (run __graft_entry__.build())")


@pytest.mark.parametrize("case", golden_cases())
@pytest.mark.parametrize("threads", [1, 0])
def test_bit_equal_to_lib_rs_restatement(case, threads, oracle_mod):
    from epure.kernels import cpu
    z = load_golden(case)
    st = _store(z)
    n, k = z["n"], z["k"]
    want = oracle_mod.c_dequant_matmul(z["x"], z["idx_rows"], z["scale"].astype(np.float32), z["cb"], n, k,
                                       z["vec"], z["group"], z["levels"])
    lib = cpu._load()
    x = np.ascontiguousarray(z["x"], np.float32)
    packed = np.ascontiguousarray(st.packed_2d().numpy())
    sc = np.ascontiguousarray(z["scale"].astype(np.float32))
    cb = np.ascontiguousarray(z["cb"], np.float32).reshape(-1)
    out = np.empty((z["m"], n), np.float32)
    bits = 4 if (z["vec"] == 1 and z["levels"] <= 16) else 8
    rc = lib.epq_cpu_linear(x.ctypes.data, z["m"], k, packed.ctypes.data, packed.shape[1], bits, z["vec"],
                            z["levels"], cb.ctypes.data, sc.ctypes.data, sc.shape[1], z["group"], n,
                            out.ctypes.data, n, threads)
    assert rc == 0
    assert np.array_equal(out, want)


@pytest.mark.parametrize("case", golden_cases())
def test_packed_linear_cpu_path(case, monkeypatch):
    from epure import PackedLinear
    from epure.kernels import cpu
    z = load_golden(case)
    lin = PackedLinear(_store(z))
    calls = []
    real = cpu.linear
    monkeypatch.setattr(cpu, "linear", lambda *a, **kw: calls.append(1) or real(*a, **kw))
    x = torch.from_numpy(z["x"])
    with torch.no_grad():
        out = lin(x)
        outbf = lin(x.to(torch.bfloat16))
    assert calls and real(x, lin.store) is not None
    assert np.abs(out.numpy() - z["out32"]).max() <= 1e-5 * np.abs(z["out32"]).max()
    assert real(x.to(torch.bfloat16), lin.store) is None          # declines: materialize runs
    assert torch.equal(outbf.float(), torch.from_numpy(z["outbf"]))


def test_declines_when_gradients_are_needed():
    from epure import make_trainable
    from epure.kernels import cpu
    from epure import PackedLinear
    z = load_golden("vec1_l16")
    m = nn.Module()
    m.proj = PackedLinear(_store(z))
    x = torch.from_numpy(z["x"])
    assert cpu.linear(x, m.proj.store) is not None
    make_trainable(m, "scale", verbose=False)
    assert cpu.linear(x, m.proj.store) is None
    with torch.no_grad():
        assert cpu.linear(x, m.proj.store) is not None


def test_rejects_bad_arguments():
    from epure.kernels import cpu
    lib = cpu._load()
    buf = np.zeros(64, np.float32)
    idx = np.zeros(64, np.uint8)
    assert lib.epq_cpu_linear(buf.ctypes.data, 1, 8, idx.ctypes.data, 8, 8, 3, 16, buf.ctypes.data,
                              buf.ctypes.data, 1, 8, 1, buf.ctypes.data, 1, 1) < 0      # vec 3
    assert lib.epq_cpu_linear(buf.ctypes.data, 1, 8, idx.ctypes.data, 1, 8, 1, 16, buf.ctypes.data,
                              buf.ctypes.data, 1, 8, 1, buf.ctypes.data, 1, 1) < 0      # row too short
    assert b"row_bytes" in lib.epq_cpu_last_error()


class TinyLM(nn.Module):
    """Embedding -> packed linear -> SiLU -> packed lm_head, next-token cross-entropy."""

    def __init__(self, vocab=64, hidden=128, seed=0):
        super().__init__()
        from epure import PackedEmbedding, PackedLinear
        from epure.synthetic import make_store
        self.embed = PackedEmbedding(make_store(vocab, hidden, device="cpu", seed=seed, levels=16, vec=1,
                                                group=64), torch.float32)
        self.mid = PackedLinear(make_store(hidden, hidden, device="cpu", seed=seed + 1))
        self.head = PackedLinear(make_store(vocab, hidden, device="cpu", seed=seed + 2))

    def forward(self, input_ids, labels=None):
        h = self.embed(input_ids)
        logits = self.head(F.silu(self.mid(h)) * 4.0)
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1))
        return types.SimpleNamespace(loss=loss, logits=logits)


def test_scale_tuner_trains_codebooks_and_scales():
    from epure import ScaleTuner, snapshot_indices
    torch.manual_seed(0)
    model = TinyLM()
    before = {n: (s.scale.detach().clone(), s.cb.detach().clone())
              for n, s in [("mid", model.mid.store), ("head", model.head.store)]}
    digests = snapshot_indices(model)
    tuner = ScaleTuner(model, mode="both", lr=3e-2)
    batch = torch.randint(0, 64, (4, 16), generator=torch.Generator().manual_seed(1))
    losses = [tuner.step(batch) for _ in range(25)]
    assert losses[-1] < 0.9 * losses[0], losses
    assert tuner.finish() is model
    assert snapshot_indices(model) == digests
    for name, st in [("mid", model.mid.store), ("head", model.head.store)]:
        assert not torch.equal(st.scale.detach(), before[name][0].float())
        assert not torch.equal(st.cb.detach(), before[name][1].float())
        assert not st.scale.requires_grad and not st.cb.requires_grad


def test_scale_tuner_catches_a_moved_index():
    from epure import ScaleTuner
    model = TinyLM(seed=5)
    tuner = ScaleTuner(model, mode="scale", lr=1e-3)
    tuner.step(torch.randint(0, 64, (2, 8)))
    model.head.store.packed[0] ^= 1
    with pytest.raises(RuntimeError, match="head"):
        tuner.finish()
