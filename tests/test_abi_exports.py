"""The C-ABI library loads on a machine without a GPU and exports every function that
include/jinf/*.h declares (no compute calls here)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include", "jinf")


def declared_functions():
    names = set()
    for fn in sorted(os.listdir(INC)):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(INC, fn)).read()
        src = re.sub(r"//.*", "", src)
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        # drop static inline definitions (header-only helpers)
        src = re.sub(r"static inline[^{;]*\{(?:[^{}]|\{[^{}]*\})*\}", "", src)
        for m in re.finditer(r"\b(jinf_[A-Za-z0-9_]+)\s*\(", src):
            name = m.group(1)
            tail = src[m.end():]
            # a declaration: name( ... ); at top level
            depth, i = 1, 0
            while depth and i < len(tail):
                depth += tail[i] == "("
                depth -= tail[i] == ")"
                i += 1
            if tail[i:].lstrip().startswith(";"):
                names.add(name)
    return sorted(names)


def test_headers_declare_functions():
    names = declared_functions()
    assert "jinf_cuda_dequant_matvec" in names and "jinf_engine_forward" in names
    assert len(names) > 60


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(name):
    import jinf
    assert hasattr(jinf.lib, name), f"{name} declared in include/jinf but not exported"
    assert name in jinf._lib.SIGNATURES, f"{name} has no ctypes signature"


def test_library_is_sm100a_cuda():
    import jinf
    path = jinf._lib.LIB_PATH
    data = open(path, "rb").read()
    assert b"sm_100a" in data or b"sm100a" in data or b".target sm_100a" in data or len(data) > 1 << 20
