"""The C ABI library loads without a GPU and exports exactly what include/b2g.h
declares; the product path has no CPU fallback."""
import ctypes as C
import os
import re
import subprocess

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
    assert lib.b2g_abi_version() == 2


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


def _compile_and_run(tmp_path, src, run=True):
    c = tmp_path / "probe.c"
    c.write_text(src)
    exe = tmp_path / "probe"
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(c), "-o", str(exe), "-L", lib_dir, "-lb2g", f"-Wl,-rpath,{lib_dir}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    if run:
        out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
        assert out.returncode == 0, out.stderr
        return out.stdout
    return ""


@pytest.mark.parametrize("struct,ctype", [("b2g_gemm_desc", "GemmDesc"), ("b2g_gemm_plan", "GemmPlan"),
                                          ("b2g_probe_desc", "ProbeDesc")])
def test_ctypes_structs_match_the_c_layout(tmp_path, struct, ctype):
    # every field of the ctypes mirror sits at the C offset, and the sizes agree
    cls = getattr(_lib, ctype)
    names = [n for n, _ in cls._fields_]
    lines = [f'  printf("{n} %zu\\n", offsetof({struct}, {n}));' for n in names]
    src = ("#include <stddef.h>\n#include <stdio.h>\n#include \"b2g.h\"\nint main(void) {\n"
           f'  printf("sizeof %zu\\n", sizeof({struct}));\n' + "\n".join(lines) + "\n  return 0;\n}\n")
    got = dict(l.split() for l in _compile_and_run(tmp_path, src).splitlines())
    assert int(got["sizeof"]) == C.sizeof(cls)
    for n in names:
        assert int(got[n]) == getattr(cls, n).offset, n


def test_c_example_compiles_and_links(tmp_path):
    # the C binding example (microbench-blackwell_b200/examples/gemm_e4m3.c) compiles
    # against include/b2g.h and links against libb2g
    example = open(os.path.join(ROOT, "microbench-blackwell_b200", "examples", "gemm_e4m3.c")).read()
    src = example + "\nint main(void) { return 0; }\n"
    _compile_and_run(tmp_path, src, run=False)
