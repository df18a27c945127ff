"""Invariants of the committed sources, checked by reading them:

* no batched-copy CUDA runtime/driver call (those calls raised GPU faults on this driver; one
  cudaMemcpyAsync per copy, or a gather kernel, is used instead);
* no bulk or TMA load with cluster multicast (all of this code may run in multi-GPU jobs, where
  such a load from another GPU's memory has hung GPUs);
* no deliberate device trap: every failure is a status bit the host reads;
* the product (the package) never imports the parity oracle.

The patterns are assembled from pieces so that this file does not itself name what it forbids."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "low-latency-distributed-llm-serving-infrastructure-custom-k8s-control-plane_b200")
SKIP_DIRS = {".git", "_work", "gpurun_out", "baseline", "_ref", "__pycache__", ".pytest_cache",
             "_build"}
SOURCE_EXT = (".cu", ".cuh", ".h", ".hpp", ".c", ".cc", ".cpp", ".py", ".sh")


def _sources(top=ROOT):
    for d, dirs, files in os.walk(top):
        dirs[:] = [x for x in dirs if x not in SKIP_DIRS]
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


def test_no_batched_copy_calls():
    names = ["cudaMemcpy" + "Batch" + "Async", "cudaMemcpy3D" + "Batch" + "Async",
             "cuMemcpy" + "Batch" + "Async", "cuMemcpy3D" + "Batch" + "Async"]
    assert _grep("|".join(names), _sources()) == []


def test_no_cluster_multicast_loads():
    assert _grep(r"multicast" + r"::" + r"cluster", _sources()) == []


def test_no_device_traps():
    # the __trap() intrinsic, or a trap instruction inside an inline-asm string
    assert _grep(r"__" + r"trap\s*\(|\"\s*" + r"trap\s*;", list(_sources(PKG))) == []


def test_product_does_not_import_the_oracle():
    py = [p for p in _sources(PKG) if p.endswith(".py")]
    assert _grep(r"^\s*(from|import)\s+oracle\b", py) == []
