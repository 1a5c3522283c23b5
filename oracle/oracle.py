"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the fused codebook dequant-matmul.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module.  The product package never does: its GPU path has no
CPU fallback.

Two restatements of the reference live here:

* numpy (this file): the reference's dense expansion and its two users.
    - ``materialize``  restates ``PackedWeight.materialize`` (epure/runtime.py:78-89)
      and ``container.dequantize`` (epure/container.py:70-88): ``w[n,k] =
      cb[idx[n,k]] * scale[n, k // group]``, with the casts that
      ``materialize(dtype)`` applies (``cb.to(dtype)``, ``scale.to(dtype)``, the
      product rounded to ``dtype``).
    - ``linear_reference`` restates ``PackedLinear.forward``'s GPU path for bf16
      (epure/runtime.py:123-124): ``F.linear(x, materialize(x.dtype))`` -- a
      bf16 GEMM with fp32 accumulation, emulated here in float64 over the bf16
      operands and rounded to bf16 once.
    - ``grads_reference`` restates the autograd of that path used for
      fine-tuning (epure/finetune.py:26-28, fine-tuning/README.md:64-68):
      ``dW = dY^T X``, ``dscale[n,g] = sum_{k in g} dW[n,k] * cb[idx[n,k]]``,
      ``dcb[l] = sum_{idx == l} dW * scale``, ``dX = dY W``.
* C (``epq_oracle.c``, loaded by ``c_dequant_matmul``): the Rust fused CPU
  kernel kernel/src/lib.rs:36-151, restated with the same summation order.

A vector codebook (``vec=4``: one index per 4 weights, ``cb[levels, 4]``) is the
layout the benchmark configuration uses; the reference has no such format.  It
is restated here as the same expression with ``w[n, 4j+p] = cb[idx[n,j], p] *
scale[n, (4j+p) // group]``.  tests/golden/make_golden.py pins it to the
reference's own ``materialize`` by expanding each vector index into the scalar
index ``4*idx + p`` of a flattened 1024-entry codebook.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libepq_oracle.so")


# --------------------------------------------------------------------------
# bf16 / fp16 rounding helpers (round to nearest even, as torch's casts do)
# --------------------------------------------------------------------------
def round_bf16(a):
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def round_f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def round_to(a, dtype):
    if dtype == "float32":
        return np.asarray(a, np.float32)
    if dtype == "bfloat16":
        return round_bf16(a)
    if dtype == "float16":
        return round_f16(a)
    raise ValueError(dtype)


# --------------------------------------------------------------------------
# index (un)packing -- epure/runtime.py:34-54
# --------------------------------------------------------------------------
def pack4(idx, levels):
    """runtime.py:34-45 ``_pack4``: two indices per byte (even k low) when levels<=16."""
    idx = np.ascontiguousarray(idx, dtype=np.uint8).ravel()
    if levels > 16:
        return idx
    if idx.size % 2:
        idx = np.append(idx, np.uint8(0))
    return (idx[0::2] | (idx[1::2] << 4)).astype(np.uint8)


def unpack4(packed, n, levels):
    """runtime.py:48-54 ``_unpack4``."""
    packed = np.asarray(packed)
    if levels > 16:
        return packed[:n]
    out = np.empty(packed.size * 2, np.uint8)
    out[0::2] = packed & 0x0F
    out[1::2] = packed >> 4
    return out[:n]


def scalar_indices(idx_rows, n, k, vec, levels):
    """Per-weight index array [n, k] (int64) from the row-major index layout."""
    if vec == 4:
        iv = np.asarray(idx_rows, np.uint8).reshape(n, k // 4).astype(np.int64)
        return iv
    return unpack4(np.asarray(idx_rows).ravel(), n * k, levels).reshape(n, k).astype(np.int64)


# --------------------------------------------------------------------------
# dense expansion -- runtime.py:78-89, container.py:70-88
# --------------------------------------------------------------------------
def materialize(idx_rows, scale, cb, n, k, vec, group, levels, dtype="float32"):
    """Dense W[n, k] as ``PackedWeight.materialize(dtype)`` computes it.

    ``cb.to(dtype)`` and ``scale.to(dtype)`` are applied before the product and
    the product is rounded to ``dtype`` (runtime.py:85-88).  Returns float32
    values that are exactly representable in ``dtype``.
    """
    cb = np.asarray(cb, np.float32).reshape(levels, vec) if vec == 4 else \
        np.asarray(cb, np.float32).reshape(-1)
    cbd = round_to(cb, dtype)
    scd = round_to(np.asarray(scale, np.float32), dtype)
    iv = scalar_indices(idx_rows, n, k, vec, levels)
    if vec == 4:
        w = cbd[iv].reshape(n, k)          # [n, k/4, 4] -> [n, k]
    else:
        w = cbd[iv]
    sc = np.repeat(scd, group, axis=1)[:, :k]
    return round_to(w * sc, dtype)


def dequantize_f64(idx_rows, scale, cb, n, k, vec, group, levels):
    """Exact (float64) dense weight from the stored values, no rounding."""
    cb = np.asarray(cb, np.float64)
    iv = scalar_indices(idx_rows, n, k, vec, levels)
    w = cb.reshape(levels, vec)[iv].reshape(n, k) if vec == 4 else cb.reshape(-1)[iv]
    sc = np.repeat(np.asarray(scale, np.float64), group, axis=1)[:, :k]
    return w * sc


def linear_reference(x, idx_rows, scale, cb, n, k, vec, group, levels, dtype="bfloat16"):
    """``F.linear(x, materialize(dtype))`` (runtime.py:123-124), fp32-accumulate GEMM.

    The GEMM is done in float64 over the ``dtype``-rounded operands, then rounded
    to ``dtype`` once; a cuBLAS fp32-accumulate result differs from this by
    summation-order noise only.
    """
    w = materialize(idx_rows, scale, cb, n, k, vec, group, levels, dtype).astype(np.float64)
    xd = round_to(np.asarray(x, np.float32), dtype).astype(np.float64)
    return round_to((xd @ w.T).astype(np.float32), dtype)


def linear_exact(x, idx_rows, scale, cb, n, k, vec, group, levels):
    """x @ W^T in float64 from the stored (un-rounded) codebook and scales."""
    w = dequantize_f64(idx_rows, scale, cb, n, k, vec, group, levels)
    return np.asarray(x, np.float64) @ w.T


def grads_reference(x, dy, idx_rows, scale, cb, n, k, vec, group, levels):
    """Gradients of ``sum(dy * (x @ W^T))`` w.r.t. x, scale and cb, in float64.

    This is the autograd of ``materialize`` + ``F.linear`` that fine-tuning
    relies on (finetune.py:26-28): ``dX = dY W``, ``dW = dY^T X``,
    ``dscale[n,g] = sum_{k in g} dW[n,k] cb[idx[n,k]]`` and
    ``dcb[l] = sum_{idx==l} dW * scale`` (fine-tuning/README.md:64-68).
    Returns (dx [m,k], dscale [n, ng], dcb [levels*vec]).
    """
    x = np.asarray(x, np.float64)
    dy = np.asarray(dy, np.float64)
    w = dequantize_f64(idx_rows, scale, cb, n, k, vec, group, levels)
    dx = dy @ w
    dw = dy.T @ x                                   # [n, k]
    ng = np.asarray(scale).shape[1]
    iv = scalar_indices(idx_rows, n, k, vec, levels)
    cbv = np.asarray(cb, np.float64).reshape(levels, vec) if vec == 4 else \
        np.asarray(cb, np.float64).reshape(-1)
    cw = cbv[iv].reshape(n, k) if vec == 4 else cbv[iv]
    prod = dw * cw
    kpad = ng * group
    prod_p = np.zeros((n, kpad)); prod_p[:, :k] = prod
    dscale = prod_p.reshape(n, ng, group).sum(-1)
    sc = np.repeat(np.asarray(scale, np.float64), group, axis=1)[:, :k]
    contrib = dw * sc
    if vec == 4:
        lin = (iv[:, :, None] * 4 + np.arange(4)[None, None, :]).reshape(n, k)
    else:
        lin = iv
    dcb = np.bincount(lin.ravel(), weights=contrib.ravel(), minlength=levels * vec)
    return dx, dscale, dcb


# --------------------------------------------------------------------------
# the C restatement of kernel/src/lib.rs
# --------------------------------------------------------------------------
_lib = None


def build_c_oracle(force=False):
    """Compile epq_oracle.c into oracle/_build/ (gcc, OpenMP, no FP contraction)."""
    os.makedirs(os.path.dirname(LIB_PATH), exist_ok=True)
    src = os.path.join(HERE, "epq_oracle.c")
    if not force and os.path.exists(LIB_PATH) and \
            os.path.getmtime(LIB_PATH) >= os.path.getmtime(src):
        return LIB_PATH
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-std=c11", src, "-o", LIB_PATH]
    subprocess.check_call(cmd)
    return LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build_c_oracle()
        lib = ctypes.CDLL(LIB_PATH)
        f = lib.epq_oracle_dequant_matmul
        f.restype = ctypes.c_int
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        f.argtypes = [P, I64, I64, P, I64, I64, P, I64, P, I, I, I64, I, P, I]
        lib.epq_oracle_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def c_threads():
    return _load().epq_oracle_threads()


def c_dequant_matmul(x, idx_rows, scale, cb, n, k, vec, group, levels, threads=0):
    """lib.rs ``dequant_matmul`` restated in C: f32 in, f32 out [m, n]."""
    lib = _load()
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    m = x.shape[0]
    packed = np.ascontiguousarray(idx_rows, np.uint8).reshape(n, -1)
    sc = np.ascontiguousarray(scale, np.float32).reshape(n, -1)
    cbf = np.ascontiguousarray(cb, np.float32).ravel()
    four_bit = 1 if (vec == 1 and levels <= 16) else 0
    out = np.empty((m, n), np.float32)
    rc = lib.epq_oracle_dequant_matmul(
        x.ctypes.data, m, k, packed.ctypes.data, n, packed.shape[1], sc.ctypes.data,
        sc.shape[1], cbf.ctypes.data, levels, vec, group, four_bit, out.ctypes.data,
        threads)
    if rc != 0:
        raise ValueError("epq_oracle_dequant_matmul rejected its arguments")
    return out


# --------------------------------------------------------------------------
# relative-error measure used by every parity test
# --------------------------------------------------------------------------
def rel_err(got, want):
    """max |got - want| / max |want|  (the per-layer relative error)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.abs(want).max()
    return float(np.abs(got - want).max() / (den if den > 0 else 1.0))
