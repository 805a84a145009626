"""The C ABI library loads without a GPU and exports exactly what include/b2g.h
declares; the product path has no CPU fallback."""
import os
import re

import pytest

import b2g
from b2g import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fn in os.listdir(inc):
        if fn.endswith(".h"):
            text = open(os.path.join(inc, fn)).read()
            names |= set(re.findall(r"B2G_API\s+[\w\s\*]+?\b(b2g_\w+)\s*\(", text))
    return names


def exported_symbols():
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_library_loads():
    lib = _lib.load()
    assert lib.b2g_abi_version() == 1


def test_every_declared_symbol_is_exported():
    decl = declared_symbols()
    assert len(decl) >= 15
    exp = exported_symbols()
    missing = decl - exp
    assert not missing, f"declared but not exported: {sorted(missing)}"
    extra = {s for s in exp if s.startswith("b2g_")} - decl
    assert not extra, f"exported but not declared: {sorted(extra)}"


def test_python_binding_covers_the_header():
    assert declared_symbols() == set(_lib.EXPORTED)


def test_status_strings():
    lib = _lib.load()
    for s in range(7):
        assert lib.b2g_status_string(s)


def test_no_cpu_fallback_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(b2g.B2GError) as e:
        b2g.Engine(0)
    assert e.value.status == 5  # B2G_ERR_NO_DEVICE
