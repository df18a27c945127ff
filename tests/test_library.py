"""CPU checks of the C-ABI library: it loads without a GPU and exports every entry point that
include/b200_paged.h declares (no compute calls)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", fn)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", src, flags=re.M):
            name = m.group(1)
            if name not in ("if", "while", "for", "return", "sizeof", "defined"):
                names.add(name)
    return names


def test_library_exports_every_declared_symbol(pkg):
    from llm_serving_b200 import _native
    lib = ctypes.CDLL(_native.LIB_PATH)
    declared = _declared()
    assert "paged_attention" in declared and "b200_paged_decode" in declared
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes binding covers the same set
    assert declared == set(_native.exported_symbols())
    _native.lib()  # binds every signature


def test_status_strings(pkg):
    from llm_serving_b200 import _native
    L = _native.lib()
    assert L.b200_status_string(0) == b"ok"
    assert L.b200_status_string(2) == b"out of memory"
