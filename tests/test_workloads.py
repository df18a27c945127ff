"""The seeded synthetic batches stand in for the BASELINE configurations: their shapes, sizes and
distributions are the ones BASELINE.json states, and their block tables are a valid paged layout
(disjoint physical blocks covering every sequence's tokens, a shuffled pool)."""
import numpy as np


def _check_layout(b):
    flat = [x for t in b.tables for x in t]
    assert len(flat) == len(set(flat)), "a physical block serves two sequences"
    assert min(flat) >= 0 and max(flat) < b.total_blocks
    for t, n in zip(b.tables, b.context_lens):
        assert len(t) == -(-int(n) // b.block_size), "table does not cover the context exactly"
    slots = b.slot_mapping()
    assert slots.shape == (b.num_tokens,) and len(set(slots.tolist())) == b.num_tokens
    bt = b.block_tables()
    assert bt.shape == (b.num_seqs, b.max_blocks) and bt.dtype == np.int32
    cu = b.cu_seqlens()
    assert cu[0] == 0 and cu[-1] == b.num_tokens and (np.diff(cu) >= 0).all()


def test_config1(pkg):
    b = pkg.workloads.config1(seed=0)
    assert (b.num_seqs, b.num_query_heads, b.num_kv_heads, b.head_dim, b.block_size) == (8, 12, 12, 64, 16)
    assert b.total_blocks == 512 and abs(b.scale - 1 / 8) < 1e-12
    assert (b.context_lens >= 1).all() and (b.context_lens <= 512).all()
    assert (b.new_token_counts == 1).all()
    _check_layout(b)


def test_config2(pkg):
    b = pkg.workloads.config2(seed=0)
    assert (b.num_seqs, b.num_query_heads, b.num_kv_heads, b.head_dim, b.block_size) == (256, 32, 8, 128, 16)
    ctx = b.context_lens
    assert ctx.min() >= 16 and ctx.max() <= 4096
    assert 800 <= np.median(ctx) <= 1300                      # lognormal, median 1024
    sigma = np.std(np.log(ctx[(ctx > 16) & (ctx < 4096)]))
    assert 0.6 <= sigma <= 1.0                                 # sigma 0.8 (clipping narrows it)
    assert (b.new_token_counts == 1).all()
    used = sum(len(t) for t in b.tables)
    assert used <= b.total_blocks <= int(used * 1.07) + 1      # ~5 % slack
    pairs = [(t[i], t[i + 1]) for t in b.tables for i in range(len(t) - 1)]
    assert sum(y == x + 1 for x, y in pairs) < 0.05 * len(pairs)   # a shuffled free list
    _check_layout(b)


def test_config3(pkg):
    b = pkg.workloads.config3(seed=0)
    assert b.num_seqs == 256 and (b.num_query_heads, b.num_kv_heads, b.head_dim) == (32, 8, 128)
    pre, dec = slice(0, 16), slice(16, 256)
    assert ((b.new_token_counts[pre] >= 128) & (b.new_token_counts[pre] <= 2048)).all()
    assert ((b.start_positions[pre] >= 0) & (b.start_positions[pre] <= 2048)).all()
    assert (b.new_token_counts[dec] == 1).all()
    assert 16 <= b.context_lens[dec].min() and b.context_lens[dec].max() <= 4096
    _check_layout(b)
