"""Fine-tune a compressed model without decompressing it (epure/finetune.py drop-in).

A packed weight is ``cb[index] * scale``; with the indices frozen the expression
is smooth in ``cb`` and ``scale``.  Same API as the reference:

    packed_weights(model)                 finetune.py:42-46
    make_trainable(model, mode, verbose)  finetune.py:49-102  -> list of params
    snapshot_indices(model)               finetune.py:105-117 -> {name: digest}
    verify_frozen(model, snapshot)        finetune.py:120-132 -> True or raises
    trainable_forward(model, enable)      finetune.py:135-143
    ScaleTuner(model, mode, lr, device)   finetune.py:146-176

On a GPU the gradients come from the fused backward kernel (dX, dscale, dcb
from the activation and output gradients; the dense dW is never formed), so
the reference's forced-materialize switch is unnecessary; ``trainable_forward``
is kept for API compatibility and only records the flag.

``snapshot_indices`` hashes the stored index bytes.  For scalar-codebook
stores they are the reference's own bytes, so digests agree with the
reference's; a vector-codebook store on a GPU hashes its tiled bytes.
"""
import torch
import torch.nn as nn

from .runtime import PackedEmbedding, PackedLinear, PackedWeight  # noqa: F401

MODES = ("scale", "codebook", "both")


def packed_weights(model):
    """Every PackedWeight in the model, with the path that owns it."""
    for name, mod in model.named_modules():
        if isinstance(mod, (PackedLinear, PackedEmbedding)):
            yield name, mod.store


def make_trainable(model, mode="both", verbose=True):
    """Promote codebook and/or scale buffers to trainable fp32 parameters.

    Everything else -- including every index -- is left frozen.  Returns the
    list of parameters to hand an optimizer.
    """
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}")

    for p in model.parameters():
        p.requires_grad_(False)

    def _promote(store, attr):
        """Buffer -> Parameter, once; idempotent for stores reached twice (tied heads)."""
        cur = getattr(store, attr)
        if isinstance(cur, nn.Parameter):
            cur.requires_grad_(True)
            return cur
        store.__dict__.pop("_hot_cache", None)
        store.__dict__.pop("_epq_desc", None)
        store._buffers.pop(attr, None)
        # clone keeps the strides, so a group-major scale stays group-major
        setattr(store, attr, nn.Parameter(cur.detach().float().clone(), requires_grad=True))
        return getattr(store, attr)

    params, seen = [], set()
    for _, store in packed_weights(model):
        if id(store) in seen:
            continue
        seen.add(id(store))
        if mode in ("scale", "both"):
            params.append(_promote(store, "scale"))
        if mode in ("codebook", "both"):
            params.append(_promote(store, "cb"))
    n_tensors = len(seen)

    n_train = sum(p.numel() for p in params)
    _uniq = {id(s): s for _, s in packed_weights(model)}.values()
    n_total = n_train + sum(s.out_features * s.in_features for s in _uniq)
    if verbose:
        print(f"  mode {mode}: {n_tensors} packed tensors, "
              f"{n_train/1e6:.2f}M trainable "
              f"({100*n_train/max(n_total,1):.2f}% of weight values)")
    return params


def snapshot_indices(model):
    """Fingerprint every index buffer (blake2b-128 of its bytes), so drift can be proven absent."""
    import hashlib

    return {name: hashlib.blake2b(store.packed.detach().cpu().numpy().tobytes(),
                                  digest_size=16).hexdigest()
            for name, store in packed_weights(model)}


def verify_frozen(model, snapshot):
    """Confirm training changed no index. Raises RuntimeError naming the first that did."""
    now = snapshot_indices(model)
    moved = [k for k, v in snapshot.items() if now.get(k) != v]
    if moved:
        raise RuntimeError(
            f"{len(moved)} index buffers changed during training "
            f"(first: {moved[0]}). Indices must stay frozen.")
    return True


def trainable_forward(model, enable=True):
    """Kept for API compatibility: the packed GPU path is already differentiable."""
    for _, store in packed_weights(model):
        store._force_materialize = enable
    return model


class ScaleTuner:
    """Minimal training loop for codebook/scale adaptation (finetune.py:146-176)."""

    def __init__(self, model, mode="both", lr=1e-4, device=None):
        self.model = model
        self.device = device or next(
            (p.device for p in model.parameters()), torch.device("cpu"))
        self.params = make_trainable(model, mode)
        self.snapshot = snapshot_indices(model)
        self.opt = torch.optim.AdamW(self.params, lr=lr)
        trainable_forward(model, True)

    def step(self, input_ids, labels=None):
        labels = input_ids if labels is None else labels
        out = self.model(input_ids.to(self.device), labels=labels.to(self.device))
        out.loss.backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return float(out.loss.detach())

    def finish(self):
        """Stop training and prove the indices never moved."""
        verify_frozen(self.model, self.snapshot)
        trainable_forward(self.model, False)
        for p in self.params:
            p.requires_grad_(False)
        return self.model
