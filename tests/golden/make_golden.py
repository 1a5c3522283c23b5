"""Generate the golden fixtures in this directory from the REFERENCE implementation.

Run (in a container that has the reference checkout; the GPU box does not):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/epure-runtime

It imports the reference package ``epure`` from that checkout and records, for a
handful of small seeded stores, what the reference's own code computes:

* ``PackedWeight.materialize(float32 | bfloat16)``  (epure/runtime.py:78-89)
* ``container.dequantize``                          (epure/container.py:70-88)
* ``F.linear(x, materialize(dtype))`` -- the path ``PackedLinear.forward`` takes
  for bf16 activations on a GPU and for every activation without the Rust
  extension (epure/runtime.py:123-124)
* gradients w.r.t. x, scale and codebook after ``make_trainable(mode="both")``
  (epure/finetune.py:49-102), through the reference's autograd path
* ``snapshot_indices`` digests (epure/finetune.py:105-117)

Vector-codebook stores (one index per 4 weights, a 256x4 codebook) have no
counterpart in the reference.  They are pinned through the reference's own
``materialize`` by expanding every vector index ``e`` at sub-position ``p`` into
the scalar index ``4*e + p`` of the flattened 1024-entry codebook and handing
``PackedWeight`` that int32 index array with ``levels=1024`` (levels > 16 keeps
``_unpack4`` a pass-through, and ``F.embedding`` accepts int32 indices).

Outputs: one ``<case>.npz`` per case.  Inputs are stored alongside outputs, so the
tests never need the reference.
"""
import os
import sys

import numpy as np

CASES = [
    # name, n, k, m, vec, levels, group, seed
    ("vec1_l16", 48, 320, 3, 1, 16, 128, 11),
    ("vec1_l256", 40, 384, 2, 1, 256, 128, 12),
    ("vec1_l16_g64", 33, 256, 4, 1, 16, 64, 13),
    ("vec4_l256", 64, 512, 1, 4, 256, 128, 14),
    ("vec4_l256_m8", 96, 1024, 8, 4, 256, 128, 15),
    ("vec4_l256_ragged", 37, 200, 5, 4, 256, 128, 16),
]


def make_inputs(n, k, m, vec, levels, group, seed):
    """Seeded inputs with the benchmark's value distributions.

    idx ~ U{0..levels-1}; vector codebooks are fp16 N(0,1) (stored here as the
    fp16 values in float32); scalar codebooks are float32 N(0,1) as in the
    reference (runtime.py:243); scales are fp16 |N(0, 0.02)|; activations are
    bf16-representable N(0,1).
    """
    rng = np.random.default_rng(seed)
    ng = -(-k // group)
    if vec == 4:
        idx = rng.integers(0, levels, size=(n, k // 4), dtype=np.uint8)
        cb = rng.standard_normal((levels, 4)).astype(np.float16).astype(np.float32)
    else:
        idx = rng.integers(0, levels, size=(n, k), dtype=np.uint8)
        cb = rng.standard_normal(levels).astype(np.float32)
    scale = np.abs(rng.normal(0.0, 0.02, size=(n, ng))).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float32)
    # round x to bf16 so the same activations are exact in every dtype path
    u = x.view(np.uint32).astype(np.uint64)
    x = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)
    gy = rng.standard_normal((m, n)).astype(np.float32)
    return idx, cb, scale, x, gy


def main(ref_root):
    sys.path.insert(0, ref_root)
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from epure import container, finetune, runtime

    out_dir = os.path.dirname(os.path.abspath(__file__))
    for name, n, k, m, vec, levels, group, seed in CASES:
        idx, cb, scale, x, gy = make_inputs(n, k, m, vec, levels, group, seed)
        if vec == 4:
            lin = (idx.astype(np.int32)[:, :, None] * 4 +
                   np.arange(4, dtype=np.int32)[None, None, :]).reshape(n, k)
            packed_ref = np.ascontiguousarray(lin.ravel())
            cb_ref = np.ascontiguousarray(cb.ravel())
            levels_ref = levels * 4
            idx_rows = idx                       # our row layout: [n, k/4] u8
        else:
            packed_ref = runtime._pack4(idx, levels)
            cb_ref = cb
            levels_ref = levels
            idx_rows = packed_ref                # the reference's own bytes
        store = runtime.PackedWeight((n, k), packed_ref.copy(), scale.copy(),
                                     cb_ref.copy(), group, levels_ref)
        w32 = store.materialize(torch.float32)
        wbf = store.materialize(torch.bfloat16)
        deq = container.dequantize(
            (lin if vec == 4 else idx).reshape(n, k), scale, cb_ref, (n, k), group)
        xt = torch.from_numpy(x)
        out32 = F.linear(xt, w32)
        outbf = F.linear(xt.to(torch.bfloat16), wbf)

        # autograd through the reference's fine-tune path
        class Holder(nn.Module):
            def __init__(self, st):
                super().__init__()
                self.proj = runtime.PackedLinear(st)

            def forward(self, t):
                return self.proj(t)

        gstore = runtime.PackedWeight((n, k), packed_ref.copy(), scale.copy(),
                                      cb_ref.copy(), group, levels_ref)
        model = Holder(gstore)
        snap = finetune.snapshot_indices(model)
        params = finetune.make_trainable(model, mode="both", verbose=False)
        xg = xt.clone().requires_grad_(True)
        y = model(xg)
        (y * torch.from_numpy(gy)).sum().backward()
        finetune.verify_frozen(model, snap)
        dscale = gstore.scale.grad.numpy().copy()
        dcb = gstore.cb.grad.numpy().copy()
        dx = xg.grad.numpy().copy()
        assert len(params) == 2

        np.savez_compressed(
            os.path.join(out_dir, f"{name}.npz"),
            n=n, k=k, m=m, vec=vec, levels=levels, group=group, seed=seed,
            idx_rows=np.ascontiguousarray(idx_rows), cb=cb, scale=scale, x=x, gy=gy,
            w32=w32.numpy(), wbf=wbf.float().numpy(), dequant=deq,
            out32=out32.numpy(), outbf=outbf.float().numpy(),
            dx=dx, dscale=dscale, dcb=dcb,
            snapshot=np.array(list(snap.values())[0]),
        )
        print(f"{name}: n={n} k={k} m={m} vec={vec} levels={levels} group={group}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the epure-runtime checkout>")
    main(sys.argv[1])
