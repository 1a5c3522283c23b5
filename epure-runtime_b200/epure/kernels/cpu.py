"""CPU backend: the fused dequant-matmul of libepq_cpu.so (include/epq_cpu.h).

The reference binds its Rust kernel here (epure/kernels/cpu.py:37-70,
kernel/src/lib.rs:96-151).  This module binds a C++/OpenMP kernel with the
same arithmetic (bit-equal results) and the same contract: ``linear(x, store,
cache)`` returns ``x @ W^T`` or ``None`` to decline, and the caller then
materialises the weight.  It declines for non-f32 activations (as the
reference does: converting them would cost more than the kernel saves), for
rank > 2 stores, when autograd needs gradients (the kernel has no backward;
``PackedWeight.materialize`` on the CPU is differentiable), and when the
library is not built.  Unlike the reference it also serves 8-bit scalar and
4-weight vector codebooks.  Per-store numpy views are cached in ``cache``
(keyed by the store and its buffers) so a batch-1 call does no conversion.
"""
import ctypes
import os
import threading

import numpy as np
import torch

_HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("EPURE_LIBEPQ_CPU") or os.path.join(_HERE, "libepq_cpu.so")

_lib = None
_lock = threading.Lock()


def _load():
    global _lib
    with _lock:
        if _lib is None and os.path.exists(LIB_PATH):
            lib = ctypes.CDLL(LIB_PATH)
            P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
            lib.epq_cpu_linear.argtypes = [P, I64, I64, P, I64, I32, I32, I32, P, P, I64, I64, I64, P, I64, I32]
            lib.epq_cpu_threads.restype = ctypes.c_int
            lib.epq_cpu_last_error.restype = ctypes.c_char_p
            _lib = lib
        return _lib


HAVE_RUST = False      # the reference's flag name: its Rust extension is never present here


def available():
    return _load() is not None


def threads():
    lib = _load()
    return lib.epq_cpu_threads() if lib is not None else 0


def _views(store, cache):
    key = (id(store), store.packed.data_ptr(), store.scale.data_ptr(), store.cb.data_ptr(),
           store.scale.dtype, store.cb.dtype)
    hit = cache.get(id(store)) if cache is not None else None
    if hit is not None and hit[0] == key:
        return hit[1]
    packed = np.ascontiguousarray(store.packed_2d().numpy())
    scale = np.ascontiguousarray(store.scale.detach().to(torch.float32).numpy())
    cb = np.ascontiguousarray(store.cb.detach().to(torch.float32).numpy()).reshape(-1)
    views = (packed, scale, cb)
    if cache is not None:
        cache[id(store)] = (key, views)
    return views


def linear(x, store, cache=None):
    """``x @ dequant(store).T`` for a CPU f32 activation, or ``None`` to decline."""
    lib = _load()
    if lib is None or x.is_cuda or store.packed.is_cuda or len(store.shape) != 2:
        return None
    if x.dtype != torch.float32:
        return None
    if torch.is_grad_enabled() and (x.requires_grad or store.scale.requires_grad or store.cb.requires_grad):
        return None
    shape = x.shape
    x2 = np.ascontiguousarray(x.detach().reshape(-1, shape[-1]).numpy())
    packed, scale, cb = _views(store, cache)
    m, k, n = x2.shape[0], store.in_features, store.out_features
    bits = 4 if (store.vec == 1 and store.levels <= 16) else 8
    out = np.empty((m, n), dtype=np.float32)
    rc = lib.epq_cpu_linear(x2.ctypes.data, m, k, packed.ctypes.data, packed.shape[1], bits, store.vec,
                            store.levels, cb.ctypes.data, scale.ctypes.data, scale.shape[1], store.group,
                            n, out.ctypes.data, n, 0)
    if rc != 0:
        raise RuntimeError(f"epure: epq_cpu_linear failed (status {rc}): "
                           f"{lib.epq_cpu_last_error().decode(errors='replace')}")
    return torch.from_numpy(out).reshape(*shape[:-1], n)
