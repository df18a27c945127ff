"""Helpers for reading the ragged entries of tests/golden/golden.npz."""
import json


def ragged(golden, prefix):
    flat = golden[prefix + "tables_flat"]
    offs = golden[prefix + "tables_offs"]
    return [flat[offs[i]:offs[i + 1]].tolist() for i in range(len(offs) - 1)]


def jload(golden, key):
    return json.loads(str(golden[key]))
