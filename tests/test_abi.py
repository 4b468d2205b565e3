"""CPU tests of the C ABI library: it loads, exports every symbol declared in
include/moe_b200.h, and rejects invalid arguments before touching a GPU."""
import ctypes
import os
import re

import pytest

import doantotnghiepmoe_b200 as M
from doantotnghiepmoe_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    L = M.lib()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert names <= set(_lib.SIGNATURES), names - set(_lib.SIGNATURES)


def test_invalid_dims_rejected_without_gpu():
    out = ctypes.c_void_p()
    bad = _lib.MoeDims(0, 8, 4, 2, 0, 1, 1)
    assert M.lib().moe_create(0, ctypes.byref(bad), ctypes.byref(out)) == _lib.MOE_ERR_INVALID
    bad = _lib.MoeDims(16, 8, 4, 5, 0, 1, 1)  # top_k > experts
    assert M.lib().moe_create(0, ctypes.byref(bad), ctypes.byref(out)) == _lib.MOE_ERR_INVALID
    assert M.lib().moe_expert_kernels_init(0, 0, 8, 2, ctypes.byref(out)) == _lib.MOE_ERR_INVALID
    assert M.lib().moe_create(0, None, ctypes.byref(out)) == _lib.MOE_ERR_INVALID


def test_product_never_loads_the_oracle():
    """The checker stays test infrastructure: nothing in the package imports,
    links or dlopens the oracle."""
    pkg = os.path.join(ROOT, "doantotnghiepmoe_b200")
    pat = re.compile(r"(import\s+oracle|from\s+oracle|libmoe_oracle|moe_oracle\.h)")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(dirpath, f)).read()
                assert not pat.search(text), f


def test_noalloc_rejects_before_touching_a_gpu():
    """moe_layer_forward_noalloc checks its arguments and the fixed scratch
    size on the host, before any CUDA call: T = 85 at the OLMoE shape needs
    more than the 8 MiB array, and H above 65536 is out of range."""
    fake = ctypes.c_void_p(256)  # never dereferenced: the call returns first
    err = ctypes.create_string_buffer(256)
    dims = _lib.MoeDims(2048, 1024, 64, 8, 0, 85, 1)
    st = M.lib().moe_layer_forward_noalloc(ctypes.byref(dims), fake, fake, fake,
                                           _lib.MOE_ROUTER_F32, fake, None, fake, 85, None,
                                           err, len(err))
    assert st == _lib.MOE_ERR_INVALID and b"scratch" in err.value
    dims = _lib.MoeDims(65537, 16, 4, 2, 0, 1, 1)
    st = M.lib().moe_layer_forward_noalloc(ctypes.byref(dims), fake, fake, fake,
                                           _lib.MOE_ROUTER_F32, fake, None, fake, 1, None,
                                           err, len(err))
    assert st == _lib.MOE_ERR_INVALID
