"""Invariants of the package sources, checked by reading them:

* no deliberate device trap: every failure is a status bit the host reads;
* the product (the package) never imports the parity oracle."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "low-latency-distributed-llm-serving-infrastructure-custom-k8s-control-plane_b200")
SOURCE_EXT = (".cu", ".cuh", ".h", ".hpp", ".c", ".cc", ".cpp", ".py")


def _sources(top=PKG):
    for d, dirs, files in os.walk(top):
        dirs[:] = [x for x in dirs if not x.startswith(("_", "."))]
        for f in files:
            if f.endswith(SOURCE_EXT) or f == "Makefile":
                yield os.path.join(d, f)


def _grep(pattern, files):
    rx = re.compile(pattern)
    hits = []
    for p in files:
        with open(p, errors="replace") as fh:
            for i, line in enumerate(fh, 1):
                if rx.search(line):
                    hits.append(f"{os.path.relpath(p, ROOT)}:{i}")
    return hits


def test_no_device_traps():
    # the __trap() intrinsic, or a trap instruction inside an inline-asm string
    assert _grep(r"__" + r"trap\s*\(|\"\s*" + r"trap\s*;", list(_sources())) == []


def test_product_does_not_import_the_oracle():
    py = [p for p in _sources() if p.endswith(".py")]
    assert _grep(r"^\s*(from|import)\s+oracle\b", py) == []
