"""Tiny synthetic ``.ebin`` containers and a toy module tree to load them into.

Shared by tests/test_loader.py and tests/golden/make_loader_golden.py (which
runs the reference's own ``apply_to`` on the same container).  The index
streams are stored uncompressed: tests swap ``container.rans_decode`` for
``identity_decode``, because the rANS coder (``constriction``) is not
installed here.  Everything else is the container format exactly: MAGIC,
blobs, JSON header, u64 little-endian header offset.
"""
import json
import struct
import types

import numpy as np
import torch
import torch.nn as nn

MAGIC = b"EBIN0001"


def identity_decode(blob, chunks, counts):
    """Stand-in for rans_decode on streams stored as raw u8 symbols."""
    n = sum(int(c[1]) for c in chunks)
    return np.frombuffer(blob, dtype=np.uint8)[:n].copy()


class _Writer:
    def __init__(self):
        self.blobs = bytearray(MAGIC)

    def add(self, data):
        rec = [len(self.blobs), len(data)]
        self.blobs += data
        return rec

    def finish(self, header):
        off = len(self.blobs)
        return bytes(self.blobs) + json.dumps(header).encode() + struct.pack("<Q", off)


# (name, shape, compressed) of the toy model's tensors.
TENSORS = [
    ("model.embed_tokens.weight", (64, 32), True),
    ("model.layers.0.self_attn.q_proj.weight", (48, 32), True),
    ("model.layers.0.self_attn.q_proj.bias", (48,), False),
    ("model.layers.0.mlp.experts.gate_up", (4, 16, 32), True),
    ("model.layers.0.mlp.router.weight", (4, 32), True),
    ("model.layers.0.conv.weight", (8, 8, 3), True),
    ("model.layers.0.norm.weight", (32,), False),
]


def make_container(path, levels=16, group=16, vec=1, seed=0, chunk=500, spec=None):
    """Writes a container of ``spec`` (default: the toy model's TENSORS); returns
    {name: (idx [rows, k/vec] u8, scale f16, cb f32 [levels] or [levels, vec])}."""
    rng = np.random.default_rng(seed)
    w = _Writer()
    tensors, values = [], {}
    for name, shape, packed in (spec or TENSORS):
        if not packed:
            data = rng.standard_normal(shape).astype(np.float16)
            tensors.append({"name": name, "kind": "raw", "shape": list(shape), "data": w.add(data.tobytes())})
            continue
        k = shape[-1]
        per = vec if k % vec == 0 else 1
        rows = int(np.prod(shape[:-1]))
        idx = rng.integers(0, levels, (rows, k // per), dtype=np.uint8)
        ng = -(-k // group)
        scale = np.abs(rng.normal(0, 0.05, (rows, ng))).astype(np.float16)
        cb = rng.standard_normal(levels * per).astype(np.float32)
        stream = idx.reshape(-1)
        chunks = [[len(stream[i:i + chunk]), len(stream[i:i + chunk])] for i in range(0, len(stream), chunk)]
        counts = np.bincount(stream, minlength=levels).tolist()
        tensors.append({"name": name, "kind": "epure", "shape": list(shape),
                        "cb": w.add(cb.tobytes()), "scale": w.add(scale.tobytes()),
                        "scale_shape": [rows, ng], "idx": w.add(stream.tobytes()),
                        "chunks": chunks, "counts": counts})
        values[name] = (idx, scale, cb.reshape(levels, per) if per > 1 else cb)
    header = {"format": "ebin-test", "levels": levels, "group": group, "tensors": tensors,
              "extras": {"config.json": w.add(b'{"model_type": "toy"}')}}
    if vec != 1:
        header["vec"] = vec
    with open(path, "wb") as f:
        f.write(w.finish(header))
    return values


class _Experts(nn.Module):
    def __init__(self):
        super().__init__()
        self.gate_up = nn.Parameter(torch.zeros(4, 16, 32))
        self.seen = None

    def forward(self, x):
        self.seen = None if self.gate_up is None else self.gate_up.detach().clone()
        return torch.einsum("ek,enk->en", x.expand(4, -1), self.gate_up)


class _Router(nn.Module):
    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(4, 32))

    def forward(self, x):
        return x @ self.weight.T, None


def toy_model():
    """The module tree the container's names address (HF-style paths)."""
    m = nn.Module()
    m.config = types.SimpleNamespace(tie_word_embeddings=True)
    m.model = nn.Module()
    m.model.embed_tokens = nn.Embedding(64, 32)
    layer = nn.Module()
    layer.self_attn = nn.Module()
    layer.self_attn.q_proj = nn.Linear(32, 48, bias=True)
    layer.mlp = nn.Module()
    layer.mlp.experts = _Experts()
    layer.mlp.router = _Router()
    layer.conv = nn.Conv1d(8, 8, 3, bias=False)
    layer.norm = nn.Module()
    layer.norm.weight = nn.Parameter(torch.zeros(32))
    m.model.layers = nn.ModuleList([layer])
    m.lm_head = nn.Linear(32, 64, bias=False)
    return m


def describe_model(model):
    """{path: class name} of the modules and frozen dense parameters that apply_to sets."""
    out = {}
    for name, mod in model.named_modules():
        if name:
            out[name] = type(mod).__name__
    for name, p in model.named_parameters():
        out[name] = "Parameter:" + str(tuple(p.shape))
    return out
