"""Reader for ``.ebin`` containers (the public surface of the reference's
epure/container.py: MAGIC, rans_decode, read_header, read_blob, dequantize,
extras, describe).

File layout (the format itself is fixed by the reference, container.py:7-13):

    bytes [0, 8)            MAGIC = b"EBIN0001"
    bytes [8, H)            payload blobs, back to back
    bytes [H, end - 8)      UTF-8 JSON header
    bytes [end - 8, end)    H as an unsigned 64-bit little-endian integer

A blob is addressed by an ``[offset, length]`` record in the header.  Every
header tensor entry is either ``{"kind": "raw", "data": rec, "shape": ...}``
(fp16 values) or a compressed one with ``"cb"`` (fp32 codebook), ``"scale"``
(fp16, ``"scale_shape"``), ``"idx"`` (entropy-coded index stream cut into
``"chunks"`` of ``[nbytes, nsymbols]``) and ``"counts"`` (the integer symbol
frequencies the coder was built from).  Containers of vector codebooks carry
``"vec": 4`` in the header (one index per 4 weights, cb of levels x 4 values);
the reference's own files have no such key and mean ``vec = 1``.

Index streams are rANS-coded by the third-party ``constriction`` package
(>= 0.3, the reference's pyproject.toml:29): each chunk is an ANS stack of
32-bit words decoded with a categorical model whose probabilities are the
stored counts, each floored at 1, normalised.  That decoder is not in this
repository's environment; ``rans_decode`` imports it on first use and raises
ImportError without it.
"""
import json
import os
import struct

import numpy as np

MAGIC = b"EBIN0001"
_TRAILER = struct.Struct("<Q")


# ---------------------------------------------------------------------------
# the container as an object
# ---------------------------------------------------------------------------
class Ebin:
    """An open ``.ebin``: its parsed header and random access to its blobs.

    ``with Ebin(path) as c: c.header, c.blob(rec)``.  The module functions
    below are the reference's entry points, written on top of this.
    """

    def __init__(self, path):
        self.path = path
        self._f = open(path, "rb")
        try:
            self.header = self._parse()
        except Exception:
            self._f.close()
            raise

    def _parse(self):
        f = self._f
        if f.read(len(MAGIC)) != MAGIC:
            raise ValueError(f"{self.path} is not an .ebin file")
        size = f.seek(0, os.SEEK_END)
        if size < len(MAGIC) + _TRAILER.size:
            raise ValueError(f"{self.path}: truncated .ebin")
        f.seek(size - _TRAILER.size)
        (start,) = _TRAILER.unpack(f.read(_TRAILER.size))
        stop = size - _TRAILER.size
        if not len(MAGIC) <= start <= stop:
            raise ValueError(f"{self.path}: header offset {start} outside the file")
        f.seek(start)
        return json.loads(f.read(stop - start))

    def blob(self, rec):
        """Bytes of the blob whose header record is ``[offset, length]``."""
        offset, length = int(rec[0]), int(rec[1])
        self._f.seek(offset)
        data = self._f.read(length)
        if len(data) != length:
            raise ValueError(f"{self.path}: blob [{offset}, {length}] runs past the end")
        return data

    @property
    def vec(self):
        return int(self.header.get("vec", 1))

    def tensors(self):
        return self.header["tensors"]

    def close(self):
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---------------------------------------------------------------------------
# index stream decoding
# ---------------------------------------------------------------------------
def symbol_probabilities(counts):
    """The coder's categorical distribution: counts floored at 1, normalised (float64).

    Both sides of the coder must build this identically for decoding to be
    exact, which is why the header stores integer counts."""
    p = np.maximum(np.asarray(counts, dtype=np.float64), 1.0)
    return p / p.sum()


def _chunk_spans(chunks):
    """(byte offset, byte length, symbol count) of each coded chunk."""
    offset = 0
    for nbytes, nsym in chunks:
        yield offset, int(nbytes), int(nsym)
        offset += int(nbytes)


def rans_decode(blob, chunks, counts):
    """The u8 index stream of one tensor, decoded chunk by chunk and concatenated."""
    import constriction

    model = constriction.stream.model.Categorical(symbol_probabilities(counts), perfect=False)
    view = memoryview(blob)
    out = []
    for offset, nbytes, nsym in _chunk_spans(chunks):
        words = np.frombuffer(view[offset:offset + nbytes], dtype=np.uint32)
        out.append(np.asarray(constriction.stream.stack.AnsCoder(words).decode(model, nsym), dtype=np.uint8))
    return np.concatenate(out) if out else np.empty(0, dtype=np.uint8)


# ---------------------------------------------------------------------------
# the reference's module-level entry points
# ---------------------------------------------------------------------------
def read_header(path):
    """The parsed JSON header of ``path`` (ValueError if it is not an .ebin)."""
    with Ebin(path) as c:
        return c.header


def read_blob(f, rec):
    """Bytes of blob ``rec`` = ``[offset, length]`` from an open binary file."""
    f.seek(int(rec[0]))
    return f.read(int(rec[1]))


def dequantize(idx, scale, cb, shape, group):
    """Float32 weights ``cb[idx] * scale`` of the given shape.

    Leading dimensions fold into rows (a stacked expert slab is one tall
    matrix over the last axis).  ``scale`` is [rows, ceil(k / group)];
    ``cb`` is 1-D (one index per weight) or [levels, vec] (one index per
    ``vec`` weights).  Each weight is one float32 product, as in the
    reference (container.py:70-88)."""
    shape = tuple(int(d) for d in shape)
    k = shape[-1]
    rows = int(np.prod(shape[:-1], dtype=np.int64)) if len(shape) > 1 else 1
    cb = np.asarray(cb, dtype=np.float32)
    per_index = 1 if cb.ndim == 1 else cb.shape[1]
    codes = np.asarray(idx).reshape(rows, -1)[:, : -(-k // per_index)]
    values = cb[codes].reshape(rows, -1)[:, :k]
    scales = np.asarray(scale, dtype=np.float32).reshape(rows, -1)
    return (values * np.repeat(scales, group, axis=1)[:, :k]).reshape(shape)


def extras(path):
    """The non-tensor files bundled in the container (config, tokenizer), by name."""
    with Ebin(path) as c:
        return {name: c.blob(rec) for name, rec in c.header.get("extras", {}).items()}


def describe(path):
    """A summary of the container (``epure info``)."""
    with Ebin(path) as c:
        h = c.header
    kinds = [t["kind"] for t in h["tensors"]]
    packed = sum(1 for kind in kinds if kind == "epure")
    return {
        "path": path,
        "format": h["format"],
        "levels": h["levels"],
        "group": h["group"],
        "compressed_tensors": packed,
        "raw_tensors": len(kinds) - packed,
        "size_bytes": os.path.getsize(path),
        "bundled": sorted(h.get("extras", {})),
    }
