"""Packed stores and the modules that run them -- a drop-in for epure/runtime.py.

Same public names, signatures and return types as the reference
(epure-runtime v0.2.4, epure/runtime.py):

    PackedWeight(shape, packed, scale, cb, group, levels)        runtime.py:57-89
    PackedLinear(store, bias=None)                               runtime.py:92-126
    PackedEmbedding(store, dtype=torch.float16)                  runtime.py:129-160
    apply_to(model, path, device, cfg, verbose, dtype)           runtime.py:214-305
    resolve(path, filename)                                      runtime.py:308-320
    load(path, device=None) -> (model, tokenizer)                runtime.py:373-415

plus ``read_stores(path, device, tp)`` (the container's stores by name,
optionally cut into this rank's tensor-parallel shards at load).

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
import contextlib
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
            else:
                # f32 CPU activations run the fused C++ kernel (it declines
                # otherwise, and when autograd needs this call's gradients)
                out = cpu_kernel.linear(x, s, _BUFFER_CACHE)
            if out is not None:
                return out + self.bias if self.bias is not None else out
        elif x.is_cuda:
            # A stacked (rank > 2) store is not one linear: the reference's
            # fallback would hand F.linear a 3-D weight.  Say so instead.
            raise RuntimeError(f"epure: PackedLinear needs a 2-D store, got shape {tuple(s.shape)}; "
                               "stacked expert slabs are served by PackedParameter")

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


# ---------------------------------------------------------------------------
# loading a container into a module tree
# ---------------------------------------------------------------------------
_MISSING = object()


def _walk(root, dotted):
    """The object at attribute path ``dotted`` below ``root`` (None if a step is missing)."""
    obj = root
    for step in dotted.split("."):
        obj = getattr(obj, step, _MISSING)
        if obj is _MISSING:
            return None
    return obj


def _owner(root, dotted):
    """(module holding the last step of ``dotted``, that step's name)."""
    head, _, leaf = dotted.rpartition(".")
    return (root.get_submodule(head) if head else root), leaf


def _replace_module(root, dotted, module):
    parent, leaf = _owner(root, dotted)
    setattr(parent, leaf, module)


def _install_dense(root, dotted, tensor):
    """A frozen dense parameter at ``dotted`` (replacing what was there)."""
    parent, leaf = _owner(root, dotted)
    setattr(parent, leaf, nn.Parameter(tensor, requires_grad=False))


class PackedParameter:
    """A stacked expert slab (rank-3 parameter of a module that does its own
    batched matmul) kept packed: the owner gets the dense tensor from a forward
    pre-hook and drops it in a forward hook, so only the module currently
    running holds a dense copy (the reference's _ExpertHolder,
    runtime.py:163-186)."""

    def __init__(self, owner, attr, store, dtype=torch.float16):
        self.owner, self.attr, self.store, self.dtype = owner, attr, store, dtype
        owner._parameters.pop(attr, None)
        setattr(owner, attr, None)
        self.handles = (owner.register_forward_pre_hook(self._expand),
                        owner.register_forward_hook(self._drop))

    def _expand(self, module, args):
        setattr(module, self.attr, self.store.materialize(self.dtype))

    def _drop(self, module, args, output):
        setattr(module, self.attr, None)


def placement(model, name, rank):
    """Where a compressed tensor ``name`` of the given rank goes in ``model``.

    Returns (kind, path): "embedding" / "linear" (path = the module to swap for
    PackedEmbedding / PackedLinear), "experts" (path = the parameter kept
    packed by a PackedParameter) or "dense" (path = the parameter to overwrite
    with the decoded tensor).  The rules are the reference's
    (runtime.py:251-287):

    * an ``nn.Embedding`` (exactly that type; subclasses have their own forward
      signatures) or any tensor named ``*embed_tokens*``  -> embedding;
    * an ``nn.Linear`` (or subclass)                      -> linear, bias kept;
    * a convolution (rank 3/4 weight, not an expert slab)  -> dense;
    * another rank-3 tensor whose owner has that attribute -> experts;
    * anything else (routers, odd modules)                 -> dense.
    """
    module_path = name[:-len(".weight")] if name.endswith(".weight") else name
    target = _walk(model, module_path)
    if type(target) is nn.Embedding or "embed_tokens" in name:
        return "embedding", module_path
    if isinstance(target, nn.Linear):
        return "linear", module_path
    if isinstance(target, (nn.Conv1d, nn.Conv2d, nn.Conv3d)):
        return "dense", name
    if rank == 3:
        holder_path, _, attr = module_path.rpartition(".")
        holder = _walk(model, holder_path) if holder_path else model
        if holder is not None and (attr in getattr(holder, "_parameters", {}) or hasattr(holder, attr)):
            return "experts", module_path
    return "dense", name


def _read_store(ebin, rec, levels, group, vec):
    """The PackedWeight (CPU, row layout) of one compressed header entry."""
    cb = np.frombuffer(ebin.blob(rec["cb"]), np.float32).copy()
    if vec > 1:
        cb = cb.reshape(-1, vec)
    scale = np.frombuffer(ebin.blob(rec["scale"]), np.float16).reshape(rec["scale_shape"]).copy()
    codes = container.rans_decode(ebin.blob(rec["idx"]), rec["chunks"], rec["counts"])
    packed = codes if vec > 1 else _pack4(codes, levels)
    return PackedWeight(rec["shape"], packed, scale, cb, group, levels, vec=vec)


def _raw_tensor(ebin, rec):
    return torch.from_numpy(np.frombuffer(ebin.blob(rec["data"]), np.float16).reshape(rec["shape"]).copy())


def apply_to(model, path, device="cpu", cfg=None, verbose=True, dtype=None):
    """Put the weights of container ``path`` into ``model``, in place (runtime.py:214-305).

    Raw tensors become frozen dense parameters in ``dtype`` (default: the
    model's current floating dtype, since ``load`` chose it).  Compressed ones
    become PackedWeight stores on ``device`` -- vector-codebook stores are laid
    out for the GPU kernels as they land there -- placed by ``placement``.  A
    config with ``tie_word_embeddings`` gets an lm_head over the embedding's
    store, and the flag is cleared so a later ``tie_weights()`` does not look
    for a dense embedding parameter.  Returns ``model``.
    """
    if dtype is None:
        dtype = next((p.dtype for p in model.parameters() if p.is_floating_point()), torch.float16)
    counts = {"packed": 0, "dense": 0}
    embed_store = None
    holders = []
    with container.Ebin(path) as ebin:
        levels, group, vec = ebin.header["levels"], ebin.header["group"], ebin.vec
        for rec in ebin.tensors():
            name = rec["name"]
            if rec["kind"] == "raw":
                _install_dense(model, name, _raw_tensor(ebin, rec).to(device=device, dtype=dtype))
                counts["dense"] += 1
                continue
            store = _read_store(ebin, rec, levels, group, vec).to(device)
            kind, where = placement(model, name, len(rec["shape"]))
            if kind == "embedding":
                embed_store = store
                _replace_module(model, where, PackedEmbedding(store, dtype))
            elif kind == "linear":
                _replace_module(model, where, PackedLinear(store, getattr(_walk(model, where), "bias", None)))
            elif kind == "experts":
                holders.append(PackedParameter(*_owner(model, where), store, dtype))
            else:
                _install_dense(model, where, store.materialize(dtype).to(device))
            counts["dense" if kind == "dense" else "packed"] += 1

    if cfg is not None and getattr(cfg, "tie_word_embeddings", False) and embed_store is not None:
        _replace_module(model, "lm_head", PackedLinear(embed_store))
        cfg.tie_word_embeddings = False
        if hasattr(model, "config"):
            model.config.tie_word_embeddings = False
        if verbose:
            print("  tied lm_head -> embedding store")
    if holders:
        model._epure_holders = holders
    if verbose:
        print(f"  {counts['packed']} packed + {counts['dense']} dense tensors from {path}")
    return model


def read_stores(path, device="cpu", tp=None):
    """Every compressed tensor of container ``path`` as a PackedWeight, by name.

    For callers that run their own decoder on the stores (epure.model,
    epure.tp) instead of a module tree.  ``tp=(rank, world)`` keeps only this
    rank's tensor-parallel shard of each decoder projection, cut on the host
    before the shard is moved to ``device``: rows of ``*q_proj`` / ``k_proj`` /
    ``v_proj`` / ``gate_proj`` / ``up_proj`` (column-parallel) and group-aligned
    columns of ``*o_proj`` / ``down_proj`` (row-parallel); other tensors are
    returned whole."""
    from . import tp as tp_mod
    out = {}
    with container.Ebin(path) as ebin:
        levels, group, vec = ebin.header["levels"], ebin.header["group"], ebin.vec
        for rec in ebin.tensors():
            if rec["kind"] == "raw":
                continue
            store = _read_store(ebin, rec, levels, group, vec)
            stem = rec["name"][:-len(".weight")] if rec["name"].endswith(".weight") else rec["name"]
            leaf = stem.rpartition(".")[2]
            if tp is not None and tp[1] > 1 and leaf in tp_mod.COLUMN + tp_mod.ROW:
                dim = "rows" if leaf in tp_mod.COLUMN else "cols"
                store = tp_mod.shard_store(store, tp[0], tp[1], dim)
            out[rec["name"]] = store.to(device)
    return out


def resolve(path, filename="model.ebin"):
    """A local ``.ebin`` path as given, or a Hugging Face repo id ("org/name")
    fetched into the hub cache (runtime.py:308-320)."""
    if os.path.exists(path):
        return path
    if os.path.isabs(path) or "/" not in path:
        raise FileNotFoundError(path)
    from huggingface_hub import hf_hub_download
    return hf_hub_download(repo_id=path, filename=filename)


def _declared_dtype(cfg):
    """The training dtype a transformers config declares (``torch_dtype`` before
    ``dtype``: transformers fills ``dtype`` with a default of its own)."""
    for key in ("torch_dtype", "dtype"):
        value = getattr(cfg, key, None)
        if value is not None:
            return getattr(torch, value, None) if isinstance(value, str) else value
    return None


def _runtime_dtype(cfg, device):
    """The dtype a model runs in (runtime.py:323-370): float32 on the CPU; on a GPU
    bfloat16 when the checkpoint was trained in it (float32 where bf16 is not
    supported -- never float16, whose range overflows bf16-trained
    activations), float16 otherwise.  The choice is printed."""
    if str(device) == "cpu":
        return torch.float32
    want = _declared_dtype(cfg)
    if want is torch.bfloat16:
        bf16_ok = torch.cuda.is_available() and torch.cuda.is_bf16_supported()
        chosen = torch.bfloat16 if bf16_ok else torch.float32
    else:
        chosen = torch.float16
    print(f"  epure: config declares {want}, running in {chosen}", flush=True)
    return chosen


@contextlib.contextmanager
def _parameters_on_meta():
    """Build modules with their parameters on the meta device and their buffers
    real: every parameter is overwritten from the container, while buffers
    computed at construction (rotary tables) are not stored in it."""
    register = nn.Module.register_parameter

    def to_meta(module, name, param):
        if param is not None and param.device.type != "meta":
            param = nn.Parameter(param.detach().to("meta"), requires_grad=param.requires_grad)
        register(module, name, param)

    nn.Module.register_parameter = to_meta
    try:
        yield
    finally:
        nn.Module.register_parameter = register


def load(path, device=None):
    """(model, tokenizer) from a ``.ebin`` path or Hugging Face repo id (runtime.py:373-415).

    The config and tokenizer files bundled in the container are written next
    to it (``<path>.meta/``); the model class is the config's declared
    architecture (AutoModelForCausalLM when transformers has no such class),
    built with parameters on the meta device and filled by ``apply_to``."""
    import transformers

    path = resolve(path)
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    meta_dir = path + ".meta"
    os.makedirs(meta_dir, exist_ok=True)
    for fname, data in container.extras(path).items():
        with open(os.path.join(meta_dir, fname), "wb") as f:
            f.write(data)
    cfg = transformers.AutoConfig.from_pretrained(meta_dir)
    cfg.use_cache = True
    tok = transformers.AutoTokenizer.from_pretrained(meta_dir)
    arch = (getattr(cfg, "architectures", None) or [None])[0]
    cls = getattr(transformers, arch, None) if arch else None
    with _parameters_on_meta():
        model = cls(cfg) if cls is not None else transformers.AutoModelForCausalLM.from_config(cfg)
    dtype = _runtime_dtype(cfg, device)
    model = model.to(dtype=dtype)
    apply_to(model, path, device=device, cfg=cfg, dtype=dtype)
    return model.eval(), tok
