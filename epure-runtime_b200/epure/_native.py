"""ctypes binding of libepq.so, the C-ABI CUDA library (include/epq.h).

This is the only module that touches the native library.  It turns torch
tensors into the plain pointers and sizes of the C ABI, owns the per-stream
workspaces the batch-1 kernel needs, and raises ``RuntimeError`` with the
library's own message whenever a call returns a non-zero status.  There is no
fallback: if the library is missing, every GPU call raises.
"""
import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# The library next to this file, unless EPURE_LIBEPQ names another build.
LIB_PATH = os.environ.get("EPURE_LIBEPQ") or os.path.join(_HERE, "libepq.so")

EPQ_F32, EPQ_F16, EPQ_BF16 = 0, 1, 2
LAYOUT_ROWS, LAYOUT_TILED, LAYOUT_MMA16 = 0, 1, 2
LAYOUT_CODES = {"rows": LAYOUT_ROWS, "tiled": LAYOUT_TILED, "mma16": LAYOUT_MMA16}

_DT = {torch.float32: EPQ_F32, torch.float16: EPQ_F16, torch.bfloat16: EPQ_BF16}

# EPURE_CHECK_IDS=1: range-check embedding ids on the host before the kernel
# (one device-to-host read per call; out-of-range ids then raise IndexError as
# torch indexing does, instead of giving zero rows and a device error flag).
CHECK_IDS = os.environ.get("EPURE_CHECK_IDS", "0") not in ("", "0")


class EpqStore(ctypes.Structure):
    _fields_ = [
        ("idx", ctypes.c_void_p),
        ("layout", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("vec", ctypes.c_int32),
        ("levels", ctypes.c_int32),
        ("group", ctypes.c_int32),
        ("cb_dtype", ctypes.c_int32),
        ("cb", ctypes.c_void_p),
        ("scale_dtype", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("scale", ctypes.c_void_p),
        ("scale_stride_n", ctypes.c_int64),
        ("scale_stride_g", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
    ]


class EpqChainStep(ctypes.Structure):
    _fields_ = [("stores", EpqStore * 4), ("count", ctypes.c_int32), ("feed", ctypes.c_int32)]


EXPORTS = (
    "epq_abi_version", "epq_last_error", "epq_device_error", "epq_layout_bytes",
    "epq_relayout", "epq_linear_workspace_bytes", "epq_linear_multi", "epq_linear",
    "epq_linear_bwd", "epq_materialize", "epq_linear_noalloc", "epq_linear_noalloc_max_scratch",
    "epq_chain_workspace_bytes", "epq_chain_prepare", "epq_chain_run", "epq_chain_set_tp",
    "epq_add_rmsnorm", "epq_rope_kv", "epq_attn_decode", "epq_attn_decode_workspace_bytes",
    "epq_silu_mul", "epq_argmax", "epq_argmax_workspace_bytes", "epq_attn_rope_decode",
    "epq_embedding", "epq_decode_linear", "epq_program_create", "epq_program_add_linear",
    "epq_program_add_attention", "epq_program_workspace_bytes", "epq_program_finalize", "epq_program_run",
    "epq_program_destroy",
)

_lib = None
_lock = threading.Lock()


def load_library(path=None):
    """Load libepq.so (once) and declare its signatures.  Raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = path or LIB_PATH
        if not os.path.exists(path):
            raise RuntimeError(
                f"epure: the CUDA library {path} is not built; run "
                "`python epure-runtime_b200/build_native.py` (or __graft_entry__.build()).")
        lib = ctypes.CDLL(path)
        P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        SP = ctypes.POINTER(EpqStore)
        lib.epq_abi_version.restype = ctypes.c_int
        lib.epq_last_error.restype = ctypes.c_char_p
        lib.epq_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
        lib.epq_layout_bytes.restype = I64
        lib.epq_layout_bytes.argtypes = [I32, I64, I64, I32, I32]
        lib.epq_relayout.argtypes = [P, I32, I64, I64, I32, I32, P, P]
        lib.epq_linear_workspace_bytes.argtypes = [SP, I32, I64, ctypes.POINTER(I64)]
        lib.epq_linear_multi.argtypes = [SP, I32, P, I32, I64, I64, P, P, I32, P, I64, P]
        lib.epq_linear.argtypes = [SP, P, I32, I64, I64, P, I64, I32, P, I64, P]
        lib.epq_linear_bwd.argtypes = [SP, P, I64, P, I64, I32, I64, P, I64, I32, P, P, P]
        lib.epq_materialize.argtypes = [SP, P, I64, I32, P]
        lib.epq_linear_noalloc.argtypes = [SP, I32, P, I32, P, I32, P]
        lib.epq_linear_noalloc_max_scratch.restype = I64
        CP = ctypes.POINTER(EpqChainStep)
        lib.epq_chain_workspace_bytes.argtypes = [CP, I32, ctypes.POINTER(I64)]
        lib.epq_chain_prepare.argtypes = [CP, I32, P, I64, P]
        lib.epq_chain_run.argtypes = [P, P, I32, P, I32, P]
        lib.epq_chain_set_tp.argtypes = [P, I32, I32, ctypes.POINTER(P), ctypes.POINTER(ctypes.c_uint8),
                                         I32, P]
        lib.epq_embedding.argtypes = [SP, P, I64, P, I64, I32, P]
        F32 = ctypes.c_float
        lib.epq_add_rmsnorm.argtypes = [P, P, P, P, I64, I64, F32, I32, P]
        lib.epq_rope_kv.argtypes = [P, P, P, P, I64, I32, I32, I32, P, P, P, P, I64, I32, F32, I32, P]
        lib.epq_attn_decode.argtypes = [P, P, P, P, I64, I32, I32, I32, F32, P, I32, P, I64, P]
        lib.epq_attn_decode_workspace_bytes.restype = I64
        lib.epq_attn_decode_workspace_bytes.argtypes = [I32, I32, I32]
        lib.epq_argmax.argtypes = [P, I64, P, P, I64, P]
        lib.epq_attn_rope_decode.argtypes = [P, P, P, P, I32, I32, I32, P, P, P, P, I64, I32, F32, F32, P, I32,
                                             P, I64, P]
        lib.epq_argmax_workspace_bytes.restype = I64
        lib.epq_argmax_workspace_bytes.argtypes = []
        lib.epq_silu_mul.argtypes = [P, P, P, I64, I32, P]
        lib.epq_decode_linear.argtypes = [SP, I32, P, I32, I64, I64, I32, F32, P, P, I32, P]
        lib.epq_program_create.argtypes = [ctypes.POINTER(P)]
        lib.epq_program_add_linear.argtypes = [P, SP, I32, P, I64, I32, F32, P, P, I32]
        lib.epq_program_add_attention.argtypes = [P, P, P, P, P, I32, I32, I32, P, P, P, P, I64, I32, F32, F32, P]
        lib.epq_program_workspace_bytes.restype = I64
        lib.epq_program_workspace_bytes.argtypes = [P]
        lib.epq_program_finalize.argtypes = [P, P, I64, P]
        lib.epq_program_run.argtypes = [P, P]
        lib.epq_program_destroy.restype = None
        lib.epq_program_destroy.argtypes = [P]
        for name in EXPORTS:
            getattr(lib, name)          # every declared entry point must be exported
        if lib.epq_abi_version() != 1:
            raise RuntimeError(f"epure: {path} has ABI {lib.epq_abi_version()}, expected 1")
        _lib = lib
        return lib


def _check(rc, what):
    if rc != 0:
        msg = _lib.epq_last_error().decode(errors="replace")
        raise RuntimeError(f"epure: {what} failed (status {rc}): {msg}")


def dtype_code(dt):
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"epure: dtype {dt} is not supported by the CUDA kernels") from None


def _stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------
# store description
# ---------------------------------------------------------------------------
def describe_store(store):
    """The C ``epq_store`` for a PackedWeight (cached until a buffer changes)."""
    packed, scale, cb = store.packed, store.scale, store.cb
    key = (id(packed), packed.data_ptr(), id(scale), scale.data_ptr(), scale.dtype,
           id(cb), cb.data_ptr(), cb.dtype, store.layout)
    hit = store.__dict__.get("_epq_desc")
    if hit is not None and hit[0] == key:
        return hit[1]
    if scale.dim() != 2:
        raise RuntimeError("epure: scale must be 2-D [rows, groups]")
    d = EpqStore()
    d.idx = packed.data_ptr()
    d.layout = LAYOUT_CODES[store.layout]
    d.bits = 4 if (store.vec == 1 and store.levels <= 16) else 8
    d.vec = store.vec
    d.levels = store.levels
    d.group = store.group
    d.cb_dtype = dtype_code(cb.dtype)
    d.cb = cb.data_ptr()
    d.scale_dtype = dtype_code(scale.dtype)
    d.scale = scale.data_ptr()
    d.scale_stride_n = scale.stride(0)
    d.scale_stride_g = scale.stride(1)
    d.n = store.out_features
    d.k = store.in_features
    if not cb.is_contiguous():
        raise RuntimeError("epure: codebook must be contiguous")
    store.__dict__["_epq_desc"] = (key, d, (packed, scale, cb))
    return d


# ---------------------------------------------------------------------------
# workspaces: one zero-filled buffer per (device, stream), grown on demand
# ---------------------------------------------------------------------------
_workspaces = {}


def workspace(device, stream_ptr, nbytes):
    if nbytes <= 0:
        return None, 0
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        buf = torch.zeros(size, dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf, buf.numel()


def reserve_workspace(stores, m=1, device=None):
    """Allocate the workspace a later call will need (before CUDA graph capture)."""
    lib = load_library()
    descs = (EpqStore * len(stores))(*[describe_store(s) for s in stores])
    need = ctypes.c_int64(0)
    _check(lib.epq_linear_workspace_bytes(descs, len(stores), m, ctypes.byref(need)),
           "epq_linear_workspace_bytes")
    device = device or stores[0].packed.device
    workspace(device, _stream_ptr(device), need.value)
    return need.value


# ---------------------------------------------------------------------------
# calls
# ---------------------------------------------------------------------------
def linear_multi(x, stores, out_dtype=None, outs=None):
    """``[x @ W_i^T for each store]`` in one launch; all stores share x (same k)."""
    lib = load_library()
    if not x.is_cuda:
        raise RuntimeError("epure: linear_multi needs a CUDA activation")
    k = stores[0].in_features
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if x2.shape[-1] != k:
        raise RuntimeError(f"epure: activation has {x2.shape[-1]} features, store expects {k}")
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    out_dtype = out_dtype or x.dtype
    count = len(stores)
    descs = (EpqStore * count)(*[describe_store(s) for s in stores])
    if outs is None:
        outs = [torch.empty((m, s.out_features), dtype=out_dtype, device=x.device) for s in stores]
    out_ptrs = (ctypes.c_void_p * count)(*[o.data_ptr() for o in outs])
    ldo = (ctypes.c_int64 * count)(*[o.stride(0) if o.dim() == 2 else s.out_features
                                     for o, s in zip(outs, stores)])
    stream = _stream_ptr(x.device)
    need = ctypes.c_int64(0)
    _check(lib.epq_linear_workspace_bytes(descs, count, m, ctypes.byref(need)),
           "epq_linear_workspace_bytes")
    ws, ws_bytes = workspace(x.device, stream, need.value)
    rc = lib.epq_linear_multi(descs, count, x2.data_ptr(), dtype_code(x2.dtype), m,
                              x2.stride(0), out_ptrs, ldo, dtype_code(out_dtype),
                              ws.data_ptr() if ws is not None else None, ws_bytes, stream)
    _check(rc, "epq_linear_multi")
    return [o.reshape(*shape[:-1], s.out_features) for o, s in zip(outs, stores)]


def linear(x, store, out_dtype=None):
    return linear_multi(x, [store], out_dtype)[0]


def linear_bwd(x, dy, store, need_dx=True, need_dscale=True, need_dcb=True, dx_dtype=None):
    """(dx, dscale [n, ng] f32, dcb [levels*vec] f32) of ``sum(dy * (x @ W^T))``.

    ``dx`` has ``dx_dtype`` (default: x's dtype)."""
    lib = load_library()
    k, n = store.in_features, store.out_features
    x2 = x.reshape(-1, k).contiguous()
    dy2 = dy.reshape(-1, n).to(x2.dtype).contiguous()
    m = x2.shape[0]
    dev = x.device
    d = describe_store(store)
    dx_dtype = dx_dtype or x.dtype
    dx = torch.empty((m, k), dtype=dx_dtype, device=dev) if need_dx else None
    ng = -(-k // store.group)
    dscale = torch.empty((n, ng), dtype=torch.float32, device=dev) if need_dscale else None
    dcb = torch.empty(store.levels * store.vec, dtype=torch.float32, device=dev) \
        if need_dcb else None
    rc = lib.epq_linear_bwd(
        ctypes.byref(d), x2.data_ptr(), x2.stride(0), dy2.data_ptr(), dy2.stride(0),
        dtype_code(x2.dtype), m, dx.data_ptr() if dx is not None else None, k,
        dtype_code(dx_dtype), dscale.data_ptr() if dscale is not None else None,
        dcb.data_ptr() if dcb is not None else None, _stream_ptr(dev))
    _check(rc, "epq_linear_bwd")
    return (dx.reshape(*x.shape[:-1], k) if dx is not None else None), dscale, dcb


def materialize(store, dtype):
    lib = load_library()
    d = describe_store(store)
    w = torch.empty((store.out_features, store.in_features), dtype=dtype,
                    device=store.packed.device)
    _check(lib.epq_materialize(ctypes.byref(d), w.data_ptr(), w.stride(0), dtype_code(dtype),
                               _stream_ptr(w.device)), "epq_materialize")
    return w


def embedding(store, ids, dtype):
    """Rows ``ids`` (any shape, int64 on the store's device) of the dequantised table,
    materialize's rounding in ``dtype``: a tensor ``[*ids.shape, in_features]``."""
    lib = load_library()
    d = describe_store(store)
    dev = store.packed.device
    flat = ids.reshape(-1).to(dev, torch.int64).contiguous()      # ids from another device are copied over
    if CHECK_IDS and flat.numel():
        n = store.out_features
        if bool(((flat < -n) | (flat >= n)).any()):
            raise IndexError(f"epure: embedding id out of range for {n} rows")
    out = torch.empty((flat.numel(), store.in_features), dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        _check(lib.epq_embedding(ctypes.byref(d), flat.data_ptr(), flat.numel(), out.data_ptr(), out.stride(0),
                                 dtype_code(dtype), _stream_ptr(dev)), "epq_embedding")
    return out.view(*ids.shape, store.in_features)


def layout_bytes(layout, n, k, vec, group):
    return int(load_library().epq_layout_bytes(LAYOUT_CODES[layout], n, k, vec, group))


def relayout(idx_rows, layout, n, k, vec, group):
    """Row-layout u8 indices on the GPU -> a new buffer in ``layout`` ("tiled" / "mma16")."""
    lib = load_library()
    src = idx_rows.contiguous()
    nbytes = layout_bytes(layout, n, k, vec, group)
    if nbytes < 0:
        raise RuntimeError(f"epure: layout {layout} does not support n={n} k={k} vec={vec} "
                           f"group={group}")
    dst = torch.empty(nbytes, dtype=torch.uint8, device=src.device)
    _check(lib.epq_relayout(src.data_ptr(), LAYOUT_CODES[layout], n, k, vec, group,
                            dst.data_ptr(), _stream_ptr(src.device)), "epq_relayout")
    return dst


# ---------------------------------------------------------------------------
# chains: a sequence of batch-1 linears in one persistent launch
# ---------------------------------------------------------------------------
def chain_prepare(steps):
    """``steps``: list of (stores, feed).  Returns the prepared workspace (uint8 tensor)."""
    lib = load_library()
    arr = (EpqChainStep * len(steps))()
    keep = []
    for j, (stores, feed) in enumerate(steps):
        arr[j].count = len(stores)
        arr[j].feed = feed
        for i, st in enumerate(stores):
            arr[j].stores[i] = describe_store(st)
            keep.append(st)
    need = ctypes.c_int64(0)
    _check(lib.epq_chain_workspace_bytes(arr, len(steps), ctypes.byref(need)),
           "epq_chain_workspace_bytes")
    dev = steps[0][0][0].packed.device
    ws = torch.zeros(need.value, dtype=torch.uint8, device=dev)
    _check(lib.epq_chain_prepare(arr, len(steps), ws.data_ptr(), ws.numel(), _stream_ptr(dev)),
           "epq_chain_prepare")
    return ws


def chain_set_tp(ws, rank, world, peer_ptrs, remote_input):
    """Tensor-parallel chain: peer_ptrs[r] = rank r's workspace as mapped here (ints)."""
    lib = load_library()
    peers = (ctypes.c_void_p * world)(*peer_ptrs)
    flags = (ctypes.c_uint8 * len(remote_input))(*[1 if f else 0 for f in remote_input])
    _check(lib.epq_chain_set_tp(ws.data_ptr(), rank, world, peers, flags, len(remote_input),
                                _stream_ptr(ws.device)), "epq_chain_set_tp")


def chain_run(ws, x, out):
    lib = load_library()
    _check(lib.epq_chain_run(ws.data_ptr(), x.data_ptr(), dtype_code(x.dtype), out.data_ptr(),
                             dtype_code(out.dtype), _stream_ptr(x.device)), "epq_chain_run")
    return out


def device_error():
    lib = load_library()
    flag = ctypes.c_int(0)
    _check(lib.epq_device_error(ctypes.byref(flag)), "epq_device_error")
    return flag.value


# -- decode-step glue (include/epq_decode.h) ------------------------------------------

def _ptr(t):
    return t.data_ptr() if t is not None else None


def add_rmsnorm(x, add=None, h_out=None, eps=1e-6):
    """(h, y): h = x + add (or x), y = RMSNorm(h) with weight 1, row-wise over the last dim."""
    lib = load_library()
    n = x.shape[-1]
    m = x.numel() // n
    y = torch.empty_like(x)
    _check(lib.epq_add_rmsnorm(x.data_ptr(), _ptr(add), _ptr(h_out), y.data_ptr(), m, n, eps,
                               dtype_code(x.dtype), _stream_ptr(x.device)), "epq_add_rmsnorm")
    return y


def rope_kv(q, k, v, pos, cos, sin, k_cache, v_cache, qk_norm, eps=1e-6):
    """Rotates q [m, H, hd] in place and writes rotated k and v at ``pos`` into the caches."""
    lib = load_library()
    m, H, hd = q.shape
    _check(lib.epq_rope_kv(q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), m, H,
                           k.shape[1], hd, cos.data_ptr(), sin.data_ptr(), k_cache.data_ptr(),
                           v_cache.data_ptr(), k_cache.shape[0], int(qk_norm), eps, dtype_code(q.dtype),
                           _stream_ptr(q.device)), "epq_rope_kv")


def attn_decode_workspace(heads, kv_heads, head_dim, device):
    """A zeroed workspace for attn_decode (reusable by consecutive calls on one stream)."""
    n = load_library().epq_attn_decode_workspace_bytes(heads, kv_heads, head_dim)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def attn_decode(q, k_cache, v_cache, pos, scale, ws=None):
    """One query token against cache positions 0..pos[0]; q [H, hd] -> [H, hd]."""
    lib = load_library()
    H, hd = q.shape[-2], q.shape[-1]
    out = torch.empty((H, hd), dtype=q.dtype, device=q.device)
    _check(lib.epq_attn_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), pos.data_ptr(),
                               k_cache.shape[0], H, k_cache.shape[-2], hd, scale, out.data_ptr(), dtype_code(q.dtype),
                               _ptr(ws), ws.numel() if ws is not None else 0,
                               _stream_ptr(q.device)), "epq_attn_decode")
    return out


def attn_rope_decode(q, k, v, pos, cos, sin, k_cache, v_cache, qk_norm, eps, scale, ws):
    """RoPE (and q/k norm) + KV write + attention for one token; q [H, hd], k, v [KV, hd]."""
    lib = load_library()
    H, hd = q.shape[-2], q.shape[-1]
    out = torch.empty((H, hd), dtype=q.dtype, device=q.device)
    _check(lib.epq_attn_rope_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), H,
                                    k.shape[-2], hd, cos.data_ptr(), sin.data_ptr(), k_cache.data_ptr(),
                                    v_cache.data_ptr(), k_cache.shape[0], int(qk_norm), eps, scale, out.data_ptr(),
                                    dtype_code(q.dtype), ws.data_ptr(), ws.numel(), _stream_ptr(q.device)),
           "epq_attn_rope_decode")
    return out


def argmax_workspace(device):
    return torch.zeros(load_library().epq_argmax_workspace_bytes(), dtype=torch.uint8, device=device)


def argmax(x, out, ws):
    """out[0] (int64, device) = the first index of the maximum of the float32 vector x."""
    lib = load_library()
    _check(lib.epq_argmax(x.data_ptr(), x.numel(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                          _stream_ptr(x.device)), "epq_argmax")
    return out


def silu_mul(g, u):
    lib = load_library()
    out = torch.empty_like(g)
    _check(lib.epq_silu_mul(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), dtype_code(g.dtype),
                            _stream_ptr(g.device)), "epq_silu_mul")
    return out


PRO_NONE, PRO_RMSNORM = 0, 1
EPI_STORE, EPI_RESIDUAL, EPI_SILU_MUL = 0, 1, 2


def decode_linear(x, stores, prologue=PRO_NONE, epilogue=EPI_STORE, outs=None, eps=1e-6):
    """A decode-step packed linear with the block glue fused in (epq_decode_linear).

    ``x`` [m, k] bf16/f16 (m <= 16).  ``prologue=PRO_RMSNORM`` normalises x first;
    ``epilogue=EPI_RESIDUAL`` adds the result into ``outs[0]`` (a residual stream,
    updated in place); ``EPI_SILU_MUL`` (stores = [gate, up]) returns
    silu(gate(x)) * up(x).  Returns the list of written outputs."""
    lib = load_library()
    if not x.is_cuda:
        raise RuntimeError("epure: decode_linear needs a CUDA activation")
    k = stores[0].in_features
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[-1] != k:
        raise RuntimeError(f"epure: activation has {x2.shape[-1]} features, store expects {k}")
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    count = len(stores)
    if outs is None:
        if epilogue == EPI_RESIDUAL:
            raise RuntimeError("epure: the residual epilogue needs the residual stream as outs[0]")
        n_out = 1 if epilogue == EPI_SILU_MUL else count
        outs = [torch.empty((m, s.out_features), dtype=x.dtype, device=x.device) for s in stores[:n_out]]
    for o in outs:
        if o.dtype != x.dtype or o.device != x.device or o.stride(-1) != 1:
            raise RuntimeError("epure: decode_linear outputs must be contiguous rows of x's dtype and device")
    wr = outs if len(outs) == count else outs + [outs[0]] * (count - len(outs))
    descs = (EpqStore * count)(*[describe_store(s) for s in stores])
    out_ptrs = (ctypes.c_void_p * count)(*[o.data_ptr() for o in wr])
    ldo = (ctypes.c_int64 * count)(*[o.stride(0) if o.dim() == 2 else s.out_features
                                     for o, s in zip(wr, stores)])
    _check(lib.epq_decode_linear(descs, count, x2.data_ptr(), dtype_code(x2.dtype), m, x2.stride(0),
                                 int(prologue), float(eps), out_ptrs, ldo, int(epilogue),
                                 _stream_ptr(x.device)), "epq_decode_linear")
    return outs


class DecodeProgram:
    """A whole decode token as one persistent kernel (epq_program_*).

    Record the token's steps in order with ``linear`` (as ``decode_linear``, m = 1)
    and ``attention`` (as ``attn_rope_decode``), then ``finalize()`` once and
    ``run()`` per token.  The program keeps the data pointers of every tensor it
    was given: they (and the stores) must stay alive and in place; the object
    holds references to them."""

    def __init__(self, device):
        self.lib = load_library()
        self.device = torch.device(device)
        self._keep = []
        h = ctypes.c_void_p()
        _check(self.lib.epq_program_create(ctypes.byref(h)), "epq_program_create")
        self._h = h
        self.ws = None
        self.steps = 0

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.lib.epq_program_destroy(h)
            self._h = None

    def linear(self, x, stores, outs, prologue=PRO_NONE, epilogue=EPI_STORE, eps=1e-6):
        k = stores[0].in_features
        if x.dtype != torch.bfloat16 or x.device != self.device or x.numel() != k or not x.is_contiguous():
            raise RuntimeError("epure: a program linear takes one contiguous bf16 row of k values on its device")
        count = len(stores)
        for o in outs:
            if o.dtype != x.dtype or o.device != x.device or not o.is_contiguous():
                raise RuntimeError("epure: program outputs must be contiguous bf16 rows on the program's device")
        wr = outs if len(outs) == count else outs + [outs[0]] * (count - len(outs))
        descs = (EpqStore * count)(*[describe_store(s) for s in stores])
        out_ptrs = (ctypes.c_void_p * count)(*[o.data_ptr() for o in wr])
        ldo = (ctypes.c_int64 * count)(*[s.out_features for s in stores])
        _check(self.lib.epq_program_add_linear(self._h, descs, count, x.data_ptr(), k, int(prologue), float(eps),
                                               out_ptrs, ldo, int(epilogue)), "epq_program_add_linear")
        self._keep += [x, *outs, *stores]
        self.steps += 1

    def attention(self, q, k, v, pos, cos, sin, k_cache, v_cache, qk_norm, eps, scale, out):
        H, hd = q.shape[-2], q.shape[-1]
        _check(self.lib.epq_program_add_attention(
            self._h, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), H, k.shape[-2], hd,
            cos.data_ptr(), sin.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
            int(qk_norm), float(eps), float(scale), out.data_ptr()), "epq_program_add_attention")
        self._keep += [q, k, v, pos, cos, sin, k_cache, v_cache, out]
        self.steps += 1

    def finalize(self):
        with torch.cuda.device(self.device):
            n = int(self.lib.epq_program_workspace_bytes(self._h))
            if n < 0:
                _check(n, "epq_program_workspace_bytes")
            self.ws = torch.empty(n, dtype=torch.uint8, device=self.device)
            _check(self.lib.epq_program_finalize(self._h, self.ws.data_ptr(), n, _stream_ptr(self.device)),
                   "epq_program_finalize")
        return self

    def run(self):
        with torch.cuda.device(self.device):
            _check(self.lib.epq_program_run(self._h, _stream_ptr(self.device)), "epq_program_run")
