"""CPU: the C-ABI library loads and exports every symbol include/heliox_b200.h declares."""
import ctypes as C
import os
import re

import pytest

from heliox_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", fn)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(hx_[a-z0-9_]+)\s*\(", src))
    return names


def test_header_declares_entries():
    names = _declared()
    for must in ("hx_create", "hx_load_group", "hx_forward_capture", "hx_backward", "hx_reduce_grads_f32"):
        assert must in names


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    missing = [n for n in sorted(_declared()) if not hasattr(L, n)]
    assert not missing, missing


def test_bindings_cover_header():
    assert _declared() <= set(_lib.SIGNATURES)


def test_abi_version():
    assert _lib.load().hx_abi_version() == 6


def test_create_without_gpu_fails_loudly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.load()
    ctx = C.c_void_p()
    assert L.hx_create(C.byref(ctx), 0) != 0
    from heliox_b200.runtime import HxError, Sim

    with pytest.raises(HxError):
        Sim(0)
