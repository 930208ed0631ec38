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
    assert _lib.load().hx_abi_version() == 8


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


def _header_enum(prefix):
    src = open(os.path.join(ROOT, "include", "heliox_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"\b(" + prefix + r"[A-Z0-9_]+)\s*=\s*(\d+)", src)}


def test_library_type_and_kind_tables_agree():
    """The library mechanism types and parameter kinds are listed in four
    places: the header's enums, the Python kind table, the model's type order
    and the loader's type names.  They must agree index for index."""
    from heliox_b200.model import LIB_FIELDS, LIB_NAMES, LIB_NTRAIN

    types = _header_enum("HX_LIB_")
    kinds = _header_enum("HX_P_")
    assert types["HX_LIB_NTYPE"] == _lib.HX_LIB_NTYPE == len(LIB_NAMES)
    assert kinds["HX_P_COUNT"] == _lib.HX_P_COUNT
    alias = {"CaDynamics_E2": "CADYN"}
    for t, nm in enumerate(LIB_NAMES):
        key = "HX_LIB_" + alias.get(nm, nm.upper())
        assert types.get(key) == t, (nm, key, types.get(key))
        for j, f in enumerate(LIB_FIELDS[nm][: LIB_NTRAIN[nm]]):
            k = kinds["HX_P_CADYN_GAMMA"] + (j if nm == "CaDynamics_E2" else t)
            assert _lib.HX_P[f"{nm}.{f}"] == k, (nm, f)
    lib_kinds = sorted(v for k, v in _lib.HX_P.items() if v >= kinds["HX_P_CADYN_GAMMA"])
    assert lib_kinds == list(range(kinds["HX_P_CADYN_GAMMA"], kinds["HX_P_COUNT"]))
    src = open(os.path.join(ROOT, "heliox_b200", "csrc", "hx_runtime_lib.cu")).read()
    body = re.search(r"kTypeName\[HX_LIB_NTYPE\]\s*=\s*\{(.*?)\};", src, flags=re.S).group(1)
    assert re.findall(r'"([^"]+)"', body) == list(LIB_NAMES)


def test_oracle_library_types_follow_the_model_order():
    """The CPU oracle's library type enum (the checker's tables are passed to it
    by index) lists the types in the model's order."""
    from heliox_b200.model import LIB_NAMES

    src = open(os.path.join(ROOT, "oracle", "hx_oracle.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    body = re.search(r"\b(HXO_NA_ION\b.*?)\bHXO_LIB_NTYPE\b", src, flags=re.S).group(1)
    names = re.findall(r"\bHXO_([A-Z0-9_]+)", body)
    alias = {"CaDynamics_E2": "CADYN"}
    assert names == [alias.get(nm, nm.upper()) for nm in LIB_NAMES]
