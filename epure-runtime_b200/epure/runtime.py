"""Packed stores and the modules that run them -- a drop-in for epure/runtime.py.

Same public names, signatures and return types as the reference
(epure-runtime v0.2.4, epure/runtime.py):

    PackedWeight(shape, packed, scale, cb, group, levels)        runtime.py:57-89
    PackedLinear(store, bias=None)                               runtime.py:92-126
    PackedEmbedding(store, dtype=torch.float16)                  runtime.py:129-160
    apply_to(model, path, device, cfg, verbose, dtype)           runtime.py:214-305
    resolve(path, filename)                                      runtime.py:308-320
    load(path, device=None) -> (model, tokenizer)                runtime.py:373-415

Differences, all on the GPU path:

* ``PackedLinear.forward`` on a CUDA activation always runs the sm_100a kernels
  of libepq.so (any dtype, any batch).  It never falls back to
  ``materialize`` + cuBLAS, and a failure raises instead of degrading.  The
  call is an autograd function, so fine-tuning gradients reach ``scale`` and
  ``cb`` through the fused backward (the reference's ``trainable_forward``
  switch is not needed; finetune.py:135-143).
* A store may hold a 4-weight vector codebook (``vec=4``: one u8 index per 4
  weights along k, ``cb`` of shape [levels, 4]).  Moved to a GPU, such a store
  (group 128) is re-laid out once into the kernel-native tiled index layout
  and its scales are kept group-major (``scale`` is still indexed
  ``[row, group]``).  Moving it back to the CPU restores the row layout.
* ``materialize`` on a GPU runs a kernel that reproduces the reference's
  rounding bit for bit (cb and scale cast to ``dtype`` first, product rounded
  to ``dtype``).
"""
import os

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import container
from .kernels import cpu as cpu_kernel
from .kernels import cuda as cuda_kernel

_BUFFER_CACHE = {}

# The reference switches CUDA calls with at least this many rows to
# materialize + cuBLAS (runtime.py:26-31).  Here the packed kernels serve every
# batch size, so the value is kept only for compatibility of the environment
# variable; it does not change the GPU path.
_DENSE_ABOVE = int(os.environ.get("EPURE_DENSE_ABOVE", "8"))


def _pack4(idx, levels):
    """Two 4-bit indices per byte (even position low) when levels <= 16 (runtime.py:34-45)."""
    idx = np.ascontiguousarray(idx, dtype=np.uint8).ravel()
    if levels > 16:
        return idx
    if idx.size % 2:
        idx = np.append(idx, np.uint8(0))
    return (idx[0::2] | (idx[1::2] << 4)).astype(np.uint8)


def _unpack4(packed, n, levels):
    """Inverse of ``_pack4`` on a torch tensor (runtime.py:48-54)."""
    if levels > 16:
        return packed[:n]
    lo, hi = packed & 0x0F, packed >> 4
    out = torch.empty(packed.numel() * 2, dtype=torch.uint8, device=packed.device)
    out[0::2], out[1::2] = lo, hi
    return out[:n]


def _as_tensor(a):
    return a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))


class PackedWeight(nn.Module):
    """Indices, per-group scales and a codebook -- the resident representation.

    ``vec`` (default 1, the reference's scalar codebook) is the number of
    consecutive weights one index covers; with ``vec=4`` ``packed`` is the
    row-major [rows, in_features / 4] u8 array and ``cb`` is [levels, 4].
    """

    TILE_GROUP = 128   # the group size the tiled GPU layouts serve
    # GPU index layout of vector stores: "mma16" (the tensor-core GEMV, any batch
    # up to 16) or "tiled" (the batch-1 LUT kernel).
    GPU_LAYOUT = os.environ.get("EPURE_GPU_LAYOUT", "mma16")

    def __init__(self, shape, packed, scale, cb, group, levels, vec=1, gpu_layout=None):
        super().__init__()
        if vec not in (1, 4):
            raise ValueError("vec must be 1 or 4")
        if gpu_layout is not None:
            if gpu_layout not in ("mma16", "tiled"):
                raise ValueError("gpu_layout must be 'mma16' or 'tiled'")
            self.GPU_LAYOUT = gpu_layout
        self.levels, self.group, self.vec = levels, group, vec
        self.shape = tuple(shape)
        self.in_features = self.shape[-1]
        rows = 1
        for d in self.shape[:-1]:
            rows *= d
        self.out_features = rows          # experts fold into rows for rank>2
        if vec == 4 and self.in_features % 4:
            raise ValueError("a vector codebook needs in_features divisible by 4")
        self.layout = "rows"
        self.register_buffer("packed", _as_tensor(packed), persistent=False)
        self.register_buffer("scale", _as_tensor(scale), persistent=False)
        self.register_buffer("cb", _as_tensor(cb), persistent=False)
        self._sync_layout()

    # -- layout management --------------------------------------------------
    def _tiling_wanted(self):
        return (self.packed.is_cuda and self.vec == 4 and self.levels <= 256
                and self.group == self.TILE_GROUP and len(self.shape) == 2)

    def _sync_layout(self):
        """Keep the index layout matched to the device (tiled on a GPU, rows on CPU)."""
        from . import _native
        want = self.GPU_LAYOUT if self._tiling_wanted() else "rows"
        if want == self.layout:
            return
        n, k = self.out_features, self.in_features
        if want != "rows":
            if self.layout != "rows":
                self._buffers["packed"] = self._rows_from_tiled().reshape(-1).contiguous()
            rows = self.packed.reshape(n, k // self.vec)
            self._buffers["packed"] = _native.relayout(rows, want, n, k, self.vec, self.group)
            sc = self.scale
            gm = self._group_major(sc.data if isinstance(sc, nn.Parameter) else sc)
            if isinstance(sc, nn.Parameter):
                sc.data = gm
            else:
                self._buffers["scale"] = gm
        else:
            self._buffers["packed"] = self._rows_from_tiled().reshape(-1).contiguous()
        self.layout = want
        self.__dict__.pop("_epq_desc", None)
        self.__dict__.pop("_hot_cache", None)

    @staticmethod
    def _group_major(sc):
        """[rows, groups] scales stored group-major, rows padded to 16 (a strided view).

        The kernels read the 16 scales of a 16-row block at one group as one
        contiguous run; padded rows hold 0.
        """
        n, ng = sc.shape
        npad = -(-n // 16) * 16
        store = torch.zeros((ng, npad), dtype=sc.dtype, device=sc.device)
        store[:, :n] = sc.t()
        return store[:, :n].t()

    def _apply(self, fn, recurse=True):
        if self.layout != "rows":
            # Device moves go through the row layout so the bytes stay meaningful.
            rows = self._rows_from_tiled().reshape(-1).contiguous()
            self._buffers["packed"] = rows
            self.layout = "rows"
        out = super()._apply(fn, recurse)
        self.__dict__.pop("_epq_desc", None)
        self._sync_layout()
        return out

    def _tiled_view(self):
        """The tiled bytes as a strided [row block, row in block, ...] view (no copy).

        "tiled": byte ((g*RB + rb)*P + l)*16 + rr  ->  [rb, rr, g, l]
        "mma16": byte ((rb*NG + g)*32 + 4*rr + q)*16 + 8*h + s  ->  [rb, h, rr, g, s, q]
        (row = 16*rb + rr or 16*rb + 8*h + rr; position j = g*P + l or g*32 + 4*s + q).
        """
        n, k, vec, g = self.out_features, self.in_features, self.vec, self.group
        p, ng = g // vec, -(-k // g)
        if self.layout == "tiled":
            return self.packed.view(ng, -(-n // 16), p, 16).permute(1, 3, 0, 2), 16
        t = self.packed.view(-(-n // 16), ng, 8, 4, 2, 8).permute(0, 4, 2, 1, 5, 3)
        return t.reshape(-(-n // 16), 16, ng, 8, 4), 16

    def _rows_from_tiled(self, rows=None):
        n, kpos = self.out_features, self.in_features // self.vec
        t, blk = self._tiled_view()
        if rows is None:
            full = t.reshape(t.shape[0] * blk, -1)
            return full[:n, :kpos].contiguous()
        sel = t[rows // blk, rows % blk]
        return sel.reshape(rows.numel(), -1)[:, :kpos]

    def index_rows(self, rows=None):
        """Per-position indices as [rows, in_features / vec] (u8, row layout)."""
        if self.layout != "rows":
            return self._rows_from_tiled(rows)
        kpos = self.in_features // self.vec
        if self.vec == 4 or self.levels > 16:
            full = self.packed[:self.out_features * kpos].view(self.out_features, kpos)
        else:
            full = _unpack4(self.packed, self.out_features * self.in_features, self.levels
                            ).view(self.out_features, self.in_features)
        return full if rows is None else full[rows]

    def packed_2d(self):
        """[rows, bytes-per-row] view of the row layout (a copy for tiled stores)."""
        if self.layout != "rows":
            return self._rows_from_tiled()
        cols = (self.in_features // 4 if self.vec == 4 else
                self.in_features if self.levels > 16 else (self.in_features + 1) // 2)
        return self.packed.view(self.out_features, cols)

    # -- dense expansion ----------------------------------------------------
    def materialize(self, dtype=torch.float16):
        """Expand to a dense tensor. Fallback only -- the kernels avoid this.

        Same values as the reference (runtime.py:78-89): cb and scale are cast
        to ``dtype`` and the product is rounded to ``dtype``.  Differentiable
        in ``scale`` and ``cb`` on the CPU path.
        """
        needs_grad = torch.is_grad_enabled() and (self.scale.requires_grad or self.cb.requires_grad)
        if self.packed.is_cuda and not needs_grad:
            from . import _native
            w = _native.materialize(self, dtype)
            return w.reshape(self.shape) if len(self.shape) > 2 else w
        idx = self.index_rows()
        n, k = self.out_features, self.in_features
        cbd = self.cb.to(dtype)
        if self.vec == 4:
            w = F.embedding(idx.int(), cbd.reshape(self.levels, 4)).reshape(n, k)
        else:
            w = F.embedding(idx.int(), cbd.view(-1, 1).contiguous()).squeeze(-1)
        sc = self.scale.to(dtype).repeat_interleave(self.group, dim=1)
        w = w * sc[:, :k]
        return w.reshape(self.shape) if len(self.shape) > 2 else w


class PackedLinear(nn.Module):
    def __init__(self, store, bias=None):
        super().__init__()
        self.store = store
        self.bias = bias

    def forward(self, x):
        s = self.store
        if len(s.shape) == 2:
            out = None
            if x.is_cuda:
                # Every batch size runs the packed kernels; errors raise.
                out = cuda_kernel.linear(x, s)
            elif s.levels <= 16:
                out = cpu_kernel.linear(x, s, _BUFFER_CACHE)
            if out is not None:
                return out + self.bias if self.bias is not None else out

        w = s.materialize(x.dtype)
        out = F.linear(x, w, self.bias)
        del w
        return out


class PackedEmbedding(nn.Module):
    """Expands only the rows a batch actually asks for (runtime.py:129-160)."""

    def __init__(self, store, dtype=torch.float16):
        super().__init__()
        self.store = store
        self.dtype = dtype
        self.num_embeddings = store.out_features
        self.embedding_dim = store.in_features

    def forward(self, ids):
        s = self.store
        if ids.is_cuda and s.packed.is_cuda and len(s.shape) == 2:
            # libepq.so decodes only the requested rows (epq_embedding), same rounding
            from . import _native
            return _native.embedding(s, ids, self.dtype)
        flat = ids.reshape(-1)
        n_in = s.in_features
        idx = s.index_rows(flat).to(torch.long)
        if s.vec == 4:
            w = s.cb.reshape(s.levels, 4)[idx].reshape(flat.numel(), n_in).to(self.dtype)
        else:
            w = s.cb[idx].to(self.dtype)
        sc = s.scale[flat].to(self.dtype)
        for gi, start in enumerate(range(0, n_in, s.group)):
            end = min(start + s.group, n_in)
            w[:, start:end] *= sc[:, gi:gi + 1]
        return w.view(*ids.shape, n_in)

    @property
    def weight(self):
        return self.store.materialize(self.dtype)


class _ExpertHolder:
    """Keeps a stacked expert slab packed except while its module runs (runtime.py:163-186)."""

    def __init__(self, mod, attr, store, dtype=torch.float16):
        self.mod, self.attr, self.store = mod, attr, store
        self.dtype = dtype
        if attr in mod._parameters:
            del mod._parameters[attr]
        mod.register_forward_pre_hook(self._attach)
        mod.register_forward_hook(self._release)
        setattr(mod, attr, None)

    def _attach(self, mod, _a):
        setattr(mod, self.attr, self.store.materialize(self.dtype))

    def _release(self, mod, _a, _o):
        setattr(mod, self.attr, None)


def _get(root, dotted):
    cur = root
    for p in dotted.split("."):
        if not hasattr(cur, p):
            return None
        cur = getattr(cur, p)
    return cur


def _set(root, dotted, mod):
    parts = dotted.split(".")
    parent = root
    for p in parts[:-1]:
        parent = getattr(parent, p)
    setattr(parent, parts[-1], mod)


def _assign(root, dotted, tensor):
    parts = dotted.split(".")
    parent = root
    for p in parts[:-1]:
        parent = getattr(parent, p)
    setattr(parent, parts[-1], nn.Parameter(tensor, requires_grad=False))


def attach_store(model, name, store, dtype, holders, embed_holder):
    """Swap the module that owns tensor ``name`` for its packed form.

    The module-type rules of the reference's ``apply_to`` (runtime.py:251-287):
    embeddings -> PackedEmbedding, linears -> PackedLinear, convolutions and
    unrecognised owners -> dense, rank-3 expert slabs -> _ExpertHolder.
    Returns "packed" or "dense".
    """
    mod_name = name[:-7] if name.endswith(".weight") else name
    target = _get(model, mod_name)
    if type(target) is nn.Embedding or "embed_tokens" in name:
        embed_holder.append(store)
        _set(model, mod_name, PackedEmbedding(store, dtype))
        return "packed"
    if isinstance(target, nn.Linear):
        _set(model, mod_name, PackedLinear(store, getattr(target, "bias", None)))
        return "packed"
    if isinstance(target, (nn.Conv1d, nn.Conv2d, nn.Conv3d)):
        _assign(model, name, store.materialize(dtype))
        return "dense"
    if len(store.shape) == 3:
        owner_path, _, attr = mod_name.rpartition(".")
        owner = _get(model, owner_path) if owner_path else model
        if owner is not None and (attr in getattr(owner, "_parameters", {})
                                  or hasattr(owner, attr)):
            holders.append(_ExpertHolder(owner, attr, store, dtype))
            return "packed"
    _assign(model, name, store.materialize(dtype))
    return "dense"


def tie_lm_head(model, cfg, embed_store, verbose=True):
    """Tied lm_head -> PackedLinear over the embedding store (runtime.py:289-300)."""
    if cfg is not None and getattr(cfg, "tie_word_embeddings", False) and embed_store:
        _set(model, "lm_head", PackedLinear(embed_store))
        cfg.tie_word_embeddings = False
        if hasattr(model, "config"):
            model.config.tie_word_embeddings = False
        if verbose:
            print("  tied lm_head -> embedding store")


def apply_to(model, path, device="cpu", cfg=None, verbose=True, dtype=None):
    """Replace a module tree's weights with packed stores, in place (runtime.py:214-305).

    Reads the ``.ebin`` container; each compressed tensor becomes a
    PackedWeight on ``device`` (vector-codebook stores are laid out for the
    GPU kernels as they land there).
    """
    if dtype is None:
        dtype = next((p.dtype for p in model.parameters()
                      if p.is_floating_point()), torch.float16)
    header = container.read_header(path)
    group, levels = header["group"], header["levels"]
    vec = int(header.get("vec", 1))
    n_packed = n_dense = 0
    embed = []
    holders = []

    with open(path, "rb") as f:
        for t in header["tensors"]:
            name = t["name"]
            if t["kind"] == "raw":
                arr = np.frombuffer(container.read_blob(f, t["data"]),
                                    np.float16).reshape(t["shape"])
                _assign(model, name,
                        torch.from_numpy(arr.copy()).to(device=device, dtype=dtype))
                n_dense += 1
                continue
            cb = np.frombuffer(container.read_blob(f, t["cb"]), np.float32).copy()
            if vec == 4:
                cb = cb.reshape(-1, 4)
            scale = np.frombuffer(container.read_blob(f, t["scale"]), np.float16
                                  ).reshape(t["scale_shape"]).copy()
            idx = container.rans_decode(container.read_blob(f, t["idx"]),
                                        t["chunks"], t["counts"])
            packed = idx if vec == 4 else _pack4(idx, levels)
            store = PackedWeight(t["shape"], packed, scale, cb, group, levels,
                                 vec=vec).to(device)
            kind = attach_store(model, name, store, dtype, holders, embed)
            if kind == "packed":
                n_packed += 1
            else:
                n_dense += 1

    tie_lm_head(model, cfg, embed[0] if embed else None, verbose)
    if holders:
        model._epure_holders = holders
    if verbose:
        print(f"  {n_packed} packed + {n_dense} dense tensors from {path}")
    return model


def resolve(path, filename="model.ebin"):
    """Accept either a local ``.ebin`` or a Hugging Face repo id (runtime.py:308-320)."""
    if os.path.exists(path):
        return path
    if "/" not in path or os.path.isabs(path):
        raise FileNotFoundError(path)
    from huggingface_hub import hf_hub_download
    return hf_hub_download(repo_id=path, filename=filename)


def _runtime_dtype(cfg, device):
    """Run in the checkpoint's training precision, never narrowing bf16 to fp16 (runtime.py:323-370)."""
    if device == "cpu":
        return torch.float32
    want = getattr(cfg, "torch_dtype", None)
    if want is None:
        want = getattr(cfg, "dtype", None)
    if isinstance(want, str):
        want = getattr(torch, want, None)
    if want is torch.bfloat16:
        if torch.cuda.is_available() and torch.cuda.is_bf16_supported():
            chosen = torch.bfloat16
        else:
            chosen = torch.float32
    else:
        chosen = torch.float16
    print(f"  epure: config declares {want}, running in {chosen}", flush=True)
    return chosen


def load(path, device=None):
    """Load a ``.ebin`` as a model, from a local path or a HF repo id (runtime.py:373-415).

    Returns (model, tokenizer).
    """
    import transformers
    from transformers import AutoConfig, AutoModelForCausalLM, AutoTokenizer

    path = resolve(path)
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    tmp = path + ".meta"
    os.makedirs(tmp, exist_ok=True)
    for name, data in container.extras(path).items():
        with open(os.path.join(tmp, name), "wb") as f:
            f.write(data)

    cfg = AutoConfig.from_pretrained(tmp)
    cfg.use_cache = True
    tok = AutoTokenizer.from_pretrained(tmp)
    arch = (getattr(cfg, "architectures", None) or [None])[0]
    factory = getattr(transformers, arch, None) if arch else None
    if factory is None:
        factory = AutoModelForCausalLM
    with torch.device("meta"):
        model = (factory.from_config(cfg) if factory is AutoModelForCausalLM
                 else factory(cfg))
    chosen_dtype = _runtime_dtype(cfg, device)
    model = model.to_empty(device=device).to(dtype=chosen_dtype)
    apply_to(model, path, device=device, cfg=cfg, dtype=chosen_dtype)
    return model.eval(), tok
