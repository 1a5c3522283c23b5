"""Compressed-state fine-tuning: train codebooks and scales, never indices.

A packed weight is ``cb[idx] * scale``.  With ``idx`` frozen that expression
is smooth in ``cb`` and ``scale``, so ordinary backprop trains them and the
result is still the same container with new codebooks and scales.  Public
surface of the reference's epure/finetune.py:

    MODES = ("scale", "codebook", "both")
    packed_weights(model)                  -> (name, store) pairs   finetune.py:42-46
    make_trainable(model, mode, verbose)   -> list of parameters    finetune.py:49-102
    snapshot_indices(model)                -> {name: digest}        finetune.py:105-117
    verify_frozen(model, snapshot)         -> True or RuntimeError  finetune.py:120-132
    trainable_forward(model, enable)       -> model                 finetune.py:135-143
    ScaleTuner(model, mode, lr, device)    .step() / .finish()      finetune.py:146-176

Gradients on a GPU come from libepq.so's fused backward (dX, dscale and dcb
from the activations and the output gradient, the dense dW never formed), so
no forward switch is needed; ``trainable_forward`` only records the flag the
reference's runtime reads.  Digests are blake2b-128 of the row-layout index
bytes: identical to the reference's for its scalar-codebook stores, and the
same on every device for vector stores (a GPU store hashes its row layout, not
its kernel tiling).
"""
import hashlib

import torch
import torch.nn as nn

from .runtime import PackedEmbedding, PackedLinear, PackedWeight  # noqa: F401

MODES = ("scale", "codebook", "both")
_TRAINED = {"scale": ("scale",), "codebook": ("cb",), "both": ("scale", "cb")}


def packed_weights(model):
    """(module path, store) for every PackedLinear / PackedEmbedding in ``model``
    (a store shared by two modules -- a tied lm_head -- appears under both)."""
    return ((name, mod.store) for name, mod in model.named_modules()
            if isinstance(mod, (PackedLinear, PackedEmbedding)))


def _unique_stores(model):
    stores = {}
    for _, store in packed_weights(model):
        stores.setdefault(id(store), store)
    return list(stores.values())


def _trainable(store, attr):
    """``store.<attr>`` as an fp32 Parameter that requires grad.

    A buffer is replaced by a Parameter once; a store reached again (tied
    modules) keeps its Parameter.  Cached kernel descriptors point at the old
    buffer and are dropped.  A GPU store's scales stay group-major (the layout
    the kernels read)."""
    cur = getattr(store, attr)
    if isinstance(cur, nn.Parameter):
        return cur.requires_grad_(True)
    value = cur.detach().float()
    if attr == "scale" and store.layout != "rows":
        value = PackedWeight._group_major(value)
    else:
        value = value.clone()
    for key in ("_hot_cache", "_epq_desc"):
        store.__dict__.pop(key, None)
    del store._buffers[attr]
    param = nn.Parameter(value, requires_grad=True)
    setattr(store, attr, param)
    return param


def make_trainable(model, mode="both", verbose=True):
    """Freeze everything, then make the scales and/or codebooks of every packed
    store trainable fp32 parameters.  Indices stay frozen buffers.  Returns the
    parameters for an optimizer (each store once, scale before codebook)."""
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}")
    for p in model.parameters():
        p.requires_grad_(False)
    stores = _unique_stores(model)
    params = [_trainable(st, attr) for st in stores for attr in _TRAINED[mode]]
    if verbose:
        n_train = sum(p.numel() for p in params)
        n_values = n_train + sum(st.out_features * st.in_features for st in stores)
        print(f"  mode {mode}: {len(stores)} packed tensors, {n_train / 1e6:.2f}M trainable "
              f"({100 * n_train / max(n_values, 1):.2f}% of weight values)")
    return params


def _index_digest(store):
    rows = store.packed if store.layout == "rows" else store.packed_2d()
    data = rows.detach().contiguous().cpu().numpy().tobytes()
    return hashlib.blake2b(data, digest_size=16).hexdigest()


def snapshot_indices(model):
    """{module path: blake2b-128 hex digest of its store's index bytes}.

    A hash, not a checksum: swapping two indices changes it."""
    return {name: _index_digest(store) for name, store in packed_weights(model)}


def verify_frozen(model, snapshot):
    """True when every index buffer in ``snapshot`` is unchanged; otherwise
    RuntimeError naming how many moved and the first of them."""
    now = snapshot_indices(model)
    moved = [name for name, digest in snapshot.items() if now.get(name) != digest]
    if moved:
        raise RuntimeError(f"{len(moved)} index buffers changed during training "
                           f"(first: {moved[0]}). Indices must stay frozen.")
    return True


def trainable_forward(model, enable=True):
    """Records ``enable`` on every store (``store._force_materialize``), the switch
    the reference's runtime uses to route training through ``materialize``.
    Here the packed path is differentiable on its own, so nothing else changes."""
    for store in _unique_stores(model):
        store._force_materialize = enable
    return model


class ScaleTuner:
    """A small AdamW loop over the codebooks / scales of a model whose forward
    takes ``(input_ids, labels=...)`` and returns an object with ``.loss``
    (a Hugging Face causal LM).  ``finish()`` proves the indices never moved."""

    def __init__(self, model, mode="both", lr=1e-4, device=None):
        self.model = model
        if device is None:
            device = next((p.device for p in model.parameters()), torch.device("cpu"))
        self.device = device
        self.params = make_trainable(model, mode)
        self.snapshot = snapshot_indices(model)
        self.opt = torch.optim.AdamW(self.params, lr=lr)
        trainable_forward(model, True)

    def step(self, input_ids, labels=None):
        """One optimizer step on a batch; returns the loss before the update."""
        if labels is None:
            labels = input_ids
        loss = self.model(input_ids.to(self.device), labels=labels.to(self.device)).loss
        loss.backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return float(loss.detach())

    def finish(self):
        """Check the indices, freeze the trained tensors, return the model."""
        verify_frozen(self.model, self.snapshot)
        trainable_forward(self.model, False)
        for p in self.params:
            p.requires_grad_(False)
        return self.model
