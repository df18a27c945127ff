"""The drop-in llm_allocator_cpp module (host C++ allocator in libb200paged.so) against the
behaviour the reference's own binding tests pin (tests/unit/test_allocator_bindings.py) and the
golden traces recorded from the reference allocator.  Host code only: runs without a GPU."""
import gc

import numpy as np
import pytest

from golden_util import jload


@pytest.fixture(scope="module")
def la(pkg):
    from llm_serving_b200 import llm_allocator_cpp
    return llm_allocator_cpp


def test_invalid_geometry(la):
    with pytest.raises(ValueError, match="tokens_per_block"):
        la.PageAllocator(1, 0, 4, 1)
    with pytest.raises(ValueError, match="bytes_per_token"):
        la.PageAllocator(1, 4, 0, 1)


def test_zero_cpu_pool_disables_device_ptr(la):
    a = la.PageAllocator(2, 4, 4, 0)
    assert a.is_zero_copy() is True
    assert a.get_device_ptr(0) == 0
    assert a.get_num_free_cpu_blocks() == 0


def test_refcounts_and_errors(la):
    a = la.PageAllocator(3, 4, 4, 1)
    assert a.allocate_block() == 0 and a.allocate_block() == 1
    assert a.get_num_free_blocks() == 1
    a.share_block(0)
    a.free_block(0)
    assert a.get_num_free_blocks() == 1
    a.free_block(0)
    assert a.get_num_free_blocks() == 2
    with pytest.raises(RuntimeError, match="Double-free"):
        a.free_block(0)
    with pytest.raises(RuntimeError, match="Cannot share"):
        a.share_block(0)
    with pytest.raises(IndexError, match="Block ID out of range"):
        a.free_block(3)
    with pytest.raises(IndexError, match="Block ID out of range"):
        a.free_block(-1)


def test_swap_roundtrip_and_host_pointer(la):
    a = la.PageAllocator(2, 4, 4, 1)
    g = a.allocate_block()
    c = a.swap_out(g)
    assert c == 0 and a.get_cpu_block_id(g) == 0 and a.get_host_ptr(c) != 0
    assert a.get_num_free_blocks() == 2 and a.get_num_free_cpu_blocks() == 0
    with pytest.raises(RuntimeError, match="ref_count != 1"):
        a.swap_out(g)
    s = a.swap_in(c)
    assert s == 1 and a.get_num_free_blocks() == 1 and a.get_num_free_cpu_blocks() == 1
    with pytest.raises(RuntimeError, match="is not swapped out"):
        a.get_cpu_block_id(g)
    a.free_block(s)
    assert a.get_num_free_blocks() == 2


def test_release_swapped_block(la):
    a = la.PageAllocator(1, 4, 4, 1)
    g = a.allocate_block()
    c = a.swap_out(g)
    assert a.get_num_free_cpu_blocks() == 0
    a.release_swapped_block(c)
    assert a.get_num_free_cpu_blocks() == 1
    with pytest.raises(RuntimeError, match="is not swapped out"):
        a.get_cpu_block_id(g)


def test_sequence_table(la):
    a = la.PageAllocator(8, 4, 4, 2)
    t = la.SequenceBlockTable(a)
    for _ in range(5):
        t.append_token()
    assert t.get_physical_blocks() == [0, 1] and t.get_tokens_count() == 5
    assert a.get_num_free_blocks() == 6
    t.release()
    assert t.get_physical_blocks() == [] and t.get_tokens_count() == 0
    assert a.get_num_free_blocks() == 8
    t.release()
    assert a.get_num_free_blocks() == 8
    with pytest.raises(TypeError):
        t.release(a)


def test_sequence_table_validation_and_replace(la):
    a = la.PageAllocator(8, 4, 4, 0)
    t = la.SequenceBlockTable(a)
    with pytest.raises(IndexError, match="Block ID out of range"):
        t.append_block(-1)
    with pytest.raises(IndexError, match="Block ID out of range"):
        t.append_block(8)
    old, new = a.allocate_block(), a.allocate_block()
    t.append_block(old)
    with pytest.raises(IndexError, match="Block ID out of range"):
        t.replace_block(old, 8)
    with pytest.raises(RuntimeError, match="not found in block table"):
        t.replace_block(99, new)
    t.replace_block(old, new)
    assert t.get_physical_blocks() == [new]
    t.release()
    a.free_block(old)
    assert a.get_num_free_blocks() == 8


def test_sequence_table_keeps_allocator_alive(la):
    a = la.PageAllocator(4, 4, 4, 0)
    t = la.SequenceBlockTable(a)
    t.append_token()
    del a
    gc.collect()
    t.release()
    assert t.get_physical_blocks() == [] and t.get_tokens_count() == 0


def test_oom_messages(la):
    a = la.PageAllocator(1, 4, 4, 0)
    a.allocate_block()
    with pytest.raises(RuntimeError, match="Out of Memory"):
        a.allocate_block()
    with pytest.raises(RuntimeError, match="Out of Memory"):
        a.allocate_blocks(1)


def test_allocator_trace_matches_reference(golden, la):
    tr = jload(golden, "alloc_trace")
    a = la.PageAllocator(tr["total_blocks"], tr["block_size"], 64, 0)
    tabs = {}
    for kind, sid, n, ok, blocks, free_after, _ in tr["ops"]:
        if kind == "release":
            t = tabs.pop(sid)
            assert t.get_physical_blocks() == blocks
            t.release()
        else:
            t = tabs.setdefault(sid, la.SequenceBlockTable(a))
            got = 1
            try:
                t.append_tokens(n)
            except RuntimeError:
                got = 0
            assert got == ok and t.get_physical_blocks() == blocks
        assert a.get_num_free_blocks() == free_after


def test_random_ops_match_oracle_fifo(la, oracle):
    rng = np.random.default_rng(3)
    a = la.PageAllocator(32, 4, 4, 4)
    f = oracle.Fifo(32)
    live = []
    for _ in range(3000):
        r = rng.random()
        if r < 0.45:
            n = int(rng.integers(0, 5))
            try:
                x = a.allocate_blocks(n)
            except RuntimeError:
                with pytest.raises(RuntimeError):
                    f.allocate_blocks(n)
                continue
            assert x == f.allocate_blocks(n)
            live.extend(x)
        elif r < 0.55 and live:
            b = live[int(rng.integers(len(live)))]
            a.share_block(b)
            f.share_block(b)
            live.append(b)
        elif live:
            b = live.pop(int(rng.integers(len(live))))
            a.free_block(b)
            f.free_block(b)
        assert a.get_num_free_blocks() == f.get_num_free_blocks()


def test_block_size_counts_tokens_not_bytes(la):
    """tokens_per_block is the block size; the host swap pool is sized in bytes from it
    (the reference's test_block_size_is_tokens_not_bytes)."""
    bytes_per_token = 2 * 8 * 4 * 2            # heads x head_dim x fp32 x (K and V)
    a = la.PageAllocator(total_blocks=10, tokens_per_block=4, bytes_per_token=bytes_per_token,
                         total_cpu_blocks=32)
    assert a.get_block_size() == 4
    assert a.get_bytes_per_token() == bytes_per_token
    assert a.get_host_pool_bytes() == 32 * 4 * bytes_per_token
