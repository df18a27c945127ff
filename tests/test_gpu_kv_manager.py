"""The device PagedKVCacheManager against the behaviour the reference's own KV-cache tests pin
(tests/unit/test_kv_cache.py of the reference): prefix and single-token writes, slot mappings
that address the physical blocks in sequence order, flat ragged scatters that leave other
sequences alone, the HF-layout gather, freeing, and the ValueErrors for missing block tables,
wrong token shapes, unallocated tokens and mismatched lengths.  Same geometry as the reference's
fixture (10 blocks of 4 tokens, 2 heads, head_dim 8, one layer, fp32), on the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def kv(pkg):
    from llm_serving_b200.kv_cache import PagedKVCacheManager
    return PagedKVCacheManager(total_blocks=10, block_size=4, num_heads=2, head_dim=8,
                               dtype=torch.float32, num_layers=1, device="cuda", max_seqs=16)


def _seq(kv, seq_id, n):
    from llm_serving_b200.engine import Sequence
    s = Sequence(seq_id, list(range(n)))
    kv.allocate_prefix_blocks(s)
    return s


def test_prefix_and_single_token_writes(kv):
    from llm_serving_b200.engine import Sequence
    s = Sequence(1, [10, 20, 30, 40, 50])
    kv.allocate_prefix_blocks(s)
    assert s.block_table.get_tokens_count() == 5
    assert len(s.block_table.get_physical_blocks()) == 2
    keys, values = torch.randn(1, 5, 2, 8), torch.randn(1, 5, 2, 8)
    slots = kv.write_prefix_kv(s, keys, values)
    assert slots.numel() == 5
    flat_k = kv.key_cache[0].reshape(-1, 2, 8)
    assert torch.equal(flat_k[slots].cpu(), keys[0])

    t = _seq(kv, 2, 4)
    t.append_token(50)
    kv.allocate_slot_for_next_token(t)
    kt, vt = torch.randn(1, 2, 8), torch.randn(1, 2, 8)
    kv.write_single_token_kv(t, kt, vt)
    assert t.block_table.get_tokens_count() == 5
    blocks = t.block_table.get_physical_blocks()
    assert len(blocks) == 2
    assert torch.equal(kv.value_cache[0, blocks[1], 0].cpu(), vt[0])


def test_writes_and_mappings_need_a_block_table(kv):
    from llm_serving_b200.engine import Sequence
    s = Sequence(4, [1])
    tok = torch.zeros(1, 2, 8)
    with pytest.raises(ValueError, match="no block table"):
        kv.write_single_token_kv(s, tok, tok)
    with pytest.raises(ValueError, match="no block table"):
        kv.build_slot_mapping([s], [0], [1])


def test_free_sequence_returns_its_blocks(kv):
    pool = kv.get_allocator()
    free0 = pool.get_num_free_blocks()
    s = _seq(kv, 3, 4)
    assert pool.get_num_free_blocks() == free0 - 1
    kv.free_sequence(s)
    assert pool.get_num_free_blocks() == free0 and s.block_table is None


def test_gather_kv_cache_round_trip(kv):
    s = _seq(kv, 1, 4)
    keys, values = torch.randn(1, 4, 2, 8), torch.randn(1, 4, 2, 8)
    kv.write_prefix_kv(s, keys, values)
    got = kv.gather_kv_cache(s, read_len=4)
    assert len(got) == 1
    gk, gv = got[0]
    assert gk.shape == (1, 2, 4, 8) and gv.shape == (1, 2, 4, 8)
    assert torch.equal(gk.cpu(), keys[0].unsqueeze(0).transpose(1, 2))
    assert torch.equal(gv.cpu(), values[0].unsqueeze(0).transpose(1, 2))
    assert kv.gather_kv_cache(s, read_len=0) is None


def test_slot_mappings_address_physical_slots_in_order(kv):
    a = _seq(kv, 1, 6)
    ba = a.block_table.get_physical_blocks()
    expect = [ba[0] * 4 + i for i in range(4)] + [ba[1] * 4 + i for i in range(2)]
    assert kv.build_slot_mapping([a], [0], [6]).cpu().tolist() == expect
    assert kv.build_slot_mapping([a], [3], [1]).cpu().tolist() == [ba[0] * 4 + 3]
    b = _seq(kv, 2, 5)
    both = kv.build_slot_mapping([a, b], [0, 0], [3, 5])
    one = torch.cat([kv.build_slot_mapping([a], [0], [3]), kv.build_slot_mapping([b], [0], [5])])
    assert torch.equal(both, one)


def test_scatter_of_a_flat_ragged_batch(kv):
    a, b = _seq(kv, 1, 3), _seq(kv, 2, 2)
    slots = kv.build_slot_mapping([a, b], [0, 0], [3, 2])
    keys, values = torch.randn(5, 1, 2, 8), torch.randn(5, 1, 2, 8)
    kv.scatter_kv(keys, values, slots)
    ba, bb = a.block_table.get_physical_blocks(), b.block_table.get_physical_blocks()
    for t in range(3):
        assert torch.equal(kv.key_cache[0, ba[0], t].cpu(), keys[t, 0])
        assert torch.equal(kv.value_cache[0, ba[0], t].cpu(), values[t, 0])
    for t in range(2):
        assert torch.equal(kv.key_cache[0, bb[0], t].cpu(), keys[3 + t, 0])
        assert torch.equal(kv.value_cache[0, bb[0], t].cpu(), values[3 + t, 0])


def test_scatter_leaves_other_sequences_alone(kv):
    a, b = _seq(kv, 1, 4), _seq(kv, 2, 4)
    ka, kb = torch.randn(4, 1, 2, 8), torch.randn(4, 1, 2, 8)
    kv.scatter_kv(ka, ka.clone(), kv.build_slot_mapping([a], [0], [4]))
    kv.scatter_kv(kb, kb.clone(), kv.build_slot_mapping([b], [0], [4]))
    bb = b.block_table.get_physical_blocks()
    for t in range(4):
        assert torch.equal(kv.key_cache[0, bb[0], t].cpu(), kb[t, 0])


def test_argument_errors(kv):
    s = _seq(kv, 1, 4)
    slots = kv.build_slot_mapping([s], [0], [2])
    with pytest.raises(ValueError):
        kv.scatter_kv(torch.randn(2, 2, 8), torch.randn(2, 2, 8), slots)   # no layer axis
    with pytest.raises(ValueError):
        kv.build_slot_mapping([s], [0], [5])                                # 5 > 4 allocated
    with pytest.raises(ValueError):
        kv.build_slot_mapping([s], [0, 1], [4])                             # lengths differ
