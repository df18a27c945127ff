"""The drop-in PageAllocator / SequenceBlockTable (host C++ in libb200paged.so) against the
reference's own binding compiled from its sources (oracle/_ref, built by `make -C oracle ref`):
random operation streams -- allocation, sharing, freeing, swapping out and in, releasing swapped
blocks, token appends and releases, with valid and invalid ids alike -- must give the same return
values, the same exception types and messages, and the same counters after every operation.
Blocks a SequenceBlockTable still holds are not freed or swapped out behind its back: the
reference then frees them again from the table's destructor, which throws there and ends the
process.  Skipped where the reference build is absent."""
import glob
import importlib.util
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_REF = glob.glob(os.path.join(ROOT, "oracle", "_ref", "llm_allocator_cpp*.so"))

pytestmark = pytest.mark.skipif(not _REF, reason="compiled reference binding absent")


def _reference_module():
    spec = importlib.util.spec_from_file_location("llm_allocator_cpp", _REF[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _call(fn, *args):
    try:
        return ("ok", fn(*args))
    except Exception as e:  # compared by type and message
        return (type(e).__name__, str(e))


def _counters(a):
    return (a.get_num_free_blocks(), a.get_num_free_cpu_blocks(), a.get_total_blocks(),
            round(a.get_utilization_percentage(), 9))


@pytest.mark.parametrize("seed", range(12))
def test_random_operations_match_the_reference(pkg, seed):
    from llm_serving_b200 import llm_allocator_cpp as ours
    ref = _reference_module()
    rng = np.random.default_rng(seed)
    nb = int(rng.integers(1, 24))
    bs = int(rng.choice([1, 4, 16]))
    ncpu = int(rng.integers(0, 8))
    a, r = ours.PageAllocator(nb, bs, 8, ncpu), ref.PageAllocator(nb, bs, 8, ncpu)
    tables = []  # (ours, reference) SequenceBlockTable pairs
    for step in range(600):
        op = int(rng.integers(0, 10))
        bid = int(rng.integers(-2, nb + 2))
        cid = int(rng.integers(-2, ncpu + 2))
        owned = {b for ta, _ in tables for b in ta.get_physical_blocks()}
        if op in (3, 4) and bid in owned:
            continue
        if op == 0:
            got, exp = _call(a.allocate_block), _call(r.allocate_block)
        elif op == 1:
            n = int(rng.integers(0, 5))
            got, exp = _call(a.allocate_blocks, n), _call(r.allocate_blocks, n)
        elif op == 2:
            got, exp = _call(a.share_block, bid), _call(r.share_block, bid)
        elif op == 3:
            got, exp = _call(a.free_block, bid), _call(r.free_block, bid)
        elif op == 4:
            got, exp = _call(a.swap_out, bid), _call(r.swap_out, bid)
        elif op == 5:
            got, exp = _call(a.swap_in, cid), _call(r.swap_in, cid)
        elif op == 6:
            got, exp = _call(a.get_cpu_block_id, bid), _call(r.get_cpu_block_id, bid)
        elif op == 7:
            got, exp = _call(a.release_swapped_block, cid), _call(r.release_swapped_block, cid)
        elif op == 8:
            if not tables or rng.random() < 0.3:
                tables.append((ours.SequenceBlockTable(a), ref.SequenceBlockTable(r)))
            ta, tr = tables[int(rng.integers(len(tables)))]
            n = int(rng.integers(1, 2 * bs + 2))
            got = [_call(ta.append_token) for _ in range(n)]
            exp = [_call(tr.append_token) for _ in range(n)]
            assert ta.get_physical_blocks() == list(tr.get_physical_blocks())
            assert ta.get_tokens_count() == tr.get_tokens_count()
        else:
            if not tables:
                continue
            ta, tr = tables.pop(int(rng.integers(len(tables))))
            got, exp = _call(ta.release), _call(tr.release)
        assert got == exp, (step, op, bid, cid, got, exp)
        assert _counters(a) == _counters(r), (step, op)
