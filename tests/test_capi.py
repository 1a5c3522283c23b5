"""The C-ABI library loads, exports every entry point include/*.h declares, and
validates its arguments on the host (no kernel is launched here)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


CPU_HEADER = "epq_cpu.h"      # declared by libepq_cpu.so (the CPU kernel), not libepq.so


def _declared(cpu=False):
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h") and (h == CPU_HEADER) == cpu:
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(epq_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from epure import _native
    return _native.load_library()


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert "epq_linear" in names and "epq_linear_bwd" in names
    for name in names:
        assert hasattr(lib, name), name


def test_python_binding_covers_header():
    from epure import _native
    assert set(_declared()) <= set(_native.EXPORTS)


def test_cpu_library_exports_its_header():
    from epure.kernels import cpu
    lib = cpu._load()
    assert lib is not None
    names = _declared(cpu=True)
    assert "epq_cpu_linear" in names
    for name in names:
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.epq_abi_version() == 1


def test_layout_bytes(lib):
    assert lib.epq_layout_bytes(1, 6144, 2048, 4, 128) == 16 * 384 * 32 * 16
    assert lib.epq_layout_bytes(1, 37, 200, 4, 128) == 2 * 3 * 32 * 16
    assert lib.epq_layout_bytes(2, 6144, 2048, 4, 128) == 16 * 384 * 512
    assert lib.epq_layout_bytes(2, 37, 200, 4, 128) == 2 * 3 * 512
    assert lib.epq_layout_bytes(2, 64, 256, 4, 64) == -1      # mma16 needs 32 positions per group
    assert lib.epq_layout_bytes(1, -1, 8, 4, 128) == -1
    assert lib.epq_layout_bytes(1, 8, 8, 3, 128) == -1
    assert lib.epq_layout_bytes(0, 8, 8, 4, 128) == -1


def _store(**kw):
    from epure._native import EpqStore
    s = EpqStore()
    s.idx, s.cb, s.scale = 16, 16, 16          # never dereferenced: validation fails first
    s.layout, s.bits, s.vec, s.levels, s.group = 1, 8, 4, 256, 128
    s.cb_dtype, s.scale_dtype = 1, 1
    s.scale_stride_n, s.scale_stride_g, s.n, s.k = 1, 64, 64, 256
    for k, v in kw.items():
        setattr(s, k, v)
    return s


@pytest.mark.parametrize("field,value,code", [
    ("vec", 3, -8), ("bits", 5, -8), ("levels", 300, -1), ("levels", 0, -1),
    ("group", 0, -1), ("k", 258, -2), ("cb_dtype", 7, -3), ("layout", 9, -1),
    ("n", -1, -1),
])
def test_bad_store_rejected(lib, field, value, code):
    s = _store(**{field: value})
    out = ctypes.c_void_p(16)
    rc = lib.epq_linear(ctypes.byref(s), ctypes.c_void_p(16), 2, 1, 256, out, 64, 2, None, 0, None)
    assert rc == code
    assert lib.epq_last_error()


def test_four_bit_tiled_rejected(lib):
    s = _store(bits=4, vec=1, levels=16)
    rc = lib.epq_linear(ctypes.byref(s), ctypes.c_void_p(16), 2, 1, 256, ctypes.c_void_p(16), 64, 2,
                        None, 0, None)
    assert rc == -5


def test_multi_count_and_k_mismatch(lib):
    from epure._native import EpqStore
    arr = (EpqStore * 2)(_store(), _store(k=512))
    outs = (ctypes.c_void_p * 2)(16, 16)
    rc = lib.epq_linear_multi(arr, 2, ctypes.c_void_p(16), 2, 1, 512, outs, None, 2, None, 0, None)
    assert rc == -2
    rc = lib.epq_linear_multi(arr, 0, ctypes.c_void_p(16), 2, 1, 512, outs, None, 2, None, 0, None)
    assert rc == -1


def test_workspace_query(lib):
    from epure._native import EpqStore
    arr = (EpqStore * 1)(_store(n=64, k=256))
    b = ctypes.c_int64(-1)
    assert lib.epq_linear_workspace_bytes(arr, 1, 1, ctypes.byref(b)) == 0
    # the fixed 64 KiB counter region + 2 groups x 64 rows of fp32 partials
    assert b.value == 65536 + 512
    assert lib.epq_linear_workspace_bytes(arr, 1, 2, ctypes.byref(b)) == 0
    assert b.value == 0          # batch > 1 runs kernels without scratch
