"""epure (B200) -- run codebook-compressed models with the weights left packed.

Drop-in for the public API of epure-runtime v0.2.4 (epure/__init__.py:11-37):

    from epure import load, make_trainable, snapshot_indices, verify_frozen

On a GPU every packed linear runs libepq.so, hand-written sm_100a kernels
behind a C ABI (include/epq.h); indices are decoded inside the matmul and the
dense weight is never written.
"""
from .container import describe, extras, read_header
from .finetune import (
    ScaleTuner,
    make_trainable,
    packed_weights,
    snapshot_indices,
    trainable_forward,
    verify_frozen,
)
from .runtime import (
    PackedEmbedding,
    PackedLinear,
    PackedWeight,
    apply_to,
    load,
    resolve,
)

__version__ = "0.2.4"

__all__ = [
    "load", "apply_to", "resolve", "describe", "extras", "read_header",
    "PackedWeight", "PackedLinear", "PackedEmbedding",
    "make_trainable", "packed_weights", "snapshot_indices", "verify_frozen",
    "trainable_forward", "ScaleTuner",
    "__version__",
]
