"""CUDA backend: libepq.so's sm_100a kernels behind the reference's contract.

Replaces epure/kernels/cuda.py of the reference (which dispatched to Triton,
declined every non-fp16 activation and fell back to materialize).  Here:

* ``linear(x, store)`` (cuda.py:88 in the reference) serves any float dtype and
  any number of rows, and never returns ``None`` for a CUDA tensor; bad inputs
  and launch failures raise ``RuntimeError`` with the library's message.
* The call is an autograd function: with ``scale``/``cb`` promoted to
  parameters (``make_trainable``) or ``x.requires_grad``, the backward runs the
  fused compressed-state kernel (dX, dscale, dcb; indices never written).
* ``linear_multi(x, stores)`` runs several stores that share one activation
  (q/k/v, gate/up) in a single launch.
* ``available()`` is True when the library loads and a GPU is present.
"""
import torch

from .. import _native

IMPORT_ERROR = None
try:
    _native.load_library()
    HAVE_LIB = True
except Exception as _exc:            # reported loudly by every GPU call
    HAVE_LIB = False
    IMPORT_ERROR = _exc


def available():
    return HAVE_LIB and torch.cuda.is_available()


def _require():
    if not HAVE_LIB:
        raise RuntimeError(f"epure: CUDA kernels unavailable ({IMPORT_ERROR}); "
                           "there is no fallback on the GPU path") from IMPORT_ERROR


class _PackedLinearFn(torch.autograd.Function):
    """out = x @ (cb[idx] * scale)^T with gradients for x, scale and cb."""

    @staticmethod
    def forward(ctx, x, scale, cb, store):
        ctx.store = store
        ctx.save_for_backward(x)
        return _native.linear(x, store)

    @staticmethod
    def backward(ctx, gout):
        (x,) = ctx.saved_tensors
        store = ctx.store
        need_dx, need_ds, need_dcb = ctx.needs_input_grad[:3]
        dx, dscale, dcb = _native.linear_bwd(x, gout, store, need_dx, need_ds, need_dcb)
        if dscale is not None:
            dscale = dscale.to(store.scale.dtype)
        if dcb is not None:
            dcb = dcb.view(store.cb.shape).to(store.cb.dtype)
        return dx, dscale, dcb, None


def _wants_grad(x, store):
    return torch.is_grad_enabled() and (
        x.requires_grad or store.scale.requires_grad or store.cb.requires_grad)


def linear(x, store):
    """``x @ dequant(store).T`` on CUDA.  Returns ``None`` only for a CPU tensor."""
    if not x.is_cuda:
        return None
    _require()
    if len(store.shape) != 2:
        raise RuntimeError("epure: packed linear needs a 2-D store")
    if _wants_grad(x, store):
        return _PackedLinearFn.apply(x, store.scale, store.cb, store)
    return _native.linear(x, store)


def linear_multi(x, stores):
    """One launch for several stores sharing ``x``; returns one output per store."""
    _require()
    if any(_wants_grad(x, s) for s in stores):
        return [linear(x, s) for s in stores]
    return _native.linear_multi(x, stores)
