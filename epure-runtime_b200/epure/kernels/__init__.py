"""Fused dequantize-and-matmul backends (epure/kernels/__init__.py in the reference).

Both backends keep the reference's contract ``linear(x, store, ...) -> Tensor |
None`` (kernels/__init__.py:1-12), with one change on the GPU: the CUDA backend
never declines.  A CUDA activation always runs libepq.so's kernels and any
failure raises ``RuntimeError``; there is no silent materialize fallback there.
The CPU backend declines (returns ``None``) exactly where the reference's does
when its Rust extension is absent, and the caller then materializes.
"""
from . import cpu, cuda

__all__ = ["cpu", "cuda"]
