"""Prefix sharing and copy-on-write in the device block pool, bit-exact against the reference
allocator's semantics (the host mirror of PageAllocator / SequenceBlockTable driven with the same
calls: share_block + append_block, allocate_block + replace_block + free_block, release): block
tables, free counts and the order of the free list; and the copy-on-write data movement on the
device (K6 fed by the pool's recorded block pairs)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

NB, BS = 24, 16


def _ref_fifo(alloc):
    """The mirror's free list in FIFO order (taking every free block, which hands them out in
    queue order)."""
    return alloc.allocate_blocks(alloc.get_num_free_blocks())


def test_share_copy_on_write_and_release_match_reference(pkg):
    from llm_serving_b200.block_manager import DeviceBlockPool
    from llm_serving_b200.llm_allocator_cpp import PageAllocator, SequenceBlockTable
    pool = DeviceBlockPool(NB, BS, max_seqs=8, max_blocks_per_seq=16)
    ref = PageAllocator(NB, BS, 64)
    A, B, C = SequenceBlockTable(ref), SequenceBlockTable(ref), SequenceBlockTable(ref)

    pool.append_tokens(0, 40)          # A: 3 blocks
    for _ in range(40):
        A.append_token()
    pool.append_tokens(1, 20)          # B: 2 blocks
    for _ in range(20):
        B.append_token()
    pool.share(2, 0, 2)                # C takes A's first 2 blocks
    for b in A.get_physical_blocks()[:2]:
        ref.share_block(b)
        C.append_block(b)
    pool.copy_on_write(2, 1)           # C gets a private copy of its second block
    old = C.get_physical_blocks()[1]
    new = ref.allocate_block()
    C.replace_block(old, new)
    ref.free_block(old)
    pool.flush()
    assert pool.table(0) == list(A.get_physical_blocks())
    assert pool.table(1) == list(B.get_physical_blocks())
    assert pool.table(2) == list(C.get_physical_blocks())
    assert pool.get_num_free_blocks() == ref.get_num_free_blocks()
    o, n = pool.cow_pairs()
    assert o.tolist() == [old] and n.tolist() == [new]

    pool.release(0)                    # A: its first block is still C's, the others come free
    A.release()
    pool.flush()
    assert pool.get_num_free_blocks() == ref.get_num_free_blocks()
    pool.append_tokens(3, 33)          # D: 3 blocks from the front of the free list
    D = SequenceBlockTable(ref)
    for _ in range(33):
        D.append_token()
    pool.release(2)                    # C: now the last owner of A's first block
    C.release()
    pool.flush()
    assert pool.table(3) == list(D.get_physical_blocks())
    assert pool.get_num_free_blocks() == ref.get_num_free_blocks()
    assert pool.free_queue() == _ref_fifo(ref)
    assert pool.status() == 0


def test_copy_on_write_copies_the_block_data(pkg):
    from llm_serving_b200.engine import Sequence
    from llm_serving_b200.kv_cache import PagedKVCacheManager
    m = PagedKVCacheManager(NB, BS, 4, 64, dtype=torch.bfloat16, num_layers=3, device="cuda",
                            max_seqs=8, max_blocks_per_seq=16)
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    m.key_cache.copy_(torch.randn(m.key_cache.shape, generator=g, device="cuda"))
    m.value_cache.copy_(torch.randn(m.value_cache.shape, generator=g, device="cuda"))
    a, c = Sequence(1, [1] * 40), Sequence(2, [1] * 32)
    m.allocate_prefix_blocks(a)
    m.pool.flush()
    m.share_prefix(a, c, 2)
    m.pool.flush()
    assert m.pool.table(c.block_table.slot) == m.pool.table(a.block_table.slot)[:2]
    assert c.block_table.get_tokens_count() == 2 * BS
    before_k, before_v = m.key_cache.clone(), m.value_cache.clone()
    m.copy_on_write(c, [0, 1])
    torch.cuda.synchronize()
    ta, tc = m.pool.table(a.block_table.slot), m.pool.table(c.block_table.slot)
    assert tc[0] not in ta and tc[1] not in ta
    for i in range(2):
        assert torch.equal(m.key_cache[:, tc[i]], before_k[:, ta[i]])
        assert torch.equal(m.value_cache[:, tc[i]], before_v[:, ta[i]])
    # A's blocks are untouched and still A's
    assert torch.equal(m.key_cache[:, ta], before_k[:, ta])
    m.free_sequence(a)
    m.free_sequence(c)
    m.pool.flush()
    assert m.pool.get_num_free_blocks() == NB
    assert m.pool.status() == 0


def test_share_argument_checks(pkg):
    from llm_serving_b200.block_manager import DeviceBlockPool
    pool = DeviceBlockPool(NB, BS, max_seqs=4, max_blocks_per_seq=8)
    pool.append_tokens(0, 20)
    pool.append_tokens(1, 5)
    with pytest.raises(ValueError):
        pool.share(1, 0, 1)            # receiving slot not empty
    with pytest.raises(ValueError):
        pool.share(2, 0, 3)            # more blocks than the source holds
    with pytest.raises(IndexError):
        pool.copy_on_write(0, 5)       # no such table entry
    pool.flush()
    assert pool.status() == 0
