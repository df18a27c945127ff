"""Pins the CPU oracle (the parity checker) to the reference: golden fixtures produced by the
reference's own code (tests/golden/make_golden.py), the literal values of the reference's unit
tests, and -- where the compiled reference is present -- the reference kernel itself."""
import numpy as np
import pytest

from golden_util import jload, ragged


def test_metadata_matches_reference_step_context(golden, oracle):
    for name in golden["meta_cases"]:
        p = f"meta_{name}_"
        tables = ragged(golden, p)
        md = oracle.step_metadata(tables, golden[p + "tokens"].tolist(),
                                  golden[p + "starts"].tolist(), golden[p + "counts"].tolist(),
                                  4, with_mask=True)
        for key in ("cu_seqlens", "cu_context_offsets", "context_lens", "scatter_slots",
                    "gather_slots", "position_ids"):
            np.testing.assert_array_equal(md[key], golden[p + key], err_msg=f"{name}:{key}")
        np.testing.assert_array_equal(md["attention_mask"], golden[p + "mask"])
        bt, cl = oracle.build_block_tables(tables, golden[p + "tokens"].tolist())
        np.testing.assert_array_equal(bt, golden[p + "block_tables"])
        np.testing.assert_array_equal(cl, golden[p + "bt_context_lens"])


def test_reference_unit_test_literals(oracle):
    # tests/unit/test_attention_backends.py:177-226 (cu_seqlens, positions, 6x6 mask)
    fifo = oracle.Fifo(8)
    tabs = []
    for n in (4, 2, 3):
        t = oracle.SeqTable(fifo, 4)
        t.append_tokens(n)
        tabs.append(t)
    md = oracle.step_metadata([t.blocks for t in tabs], [4, 2, 3], [0, 0, 0], [4, 2, 3], 4)
    assert md["cu_seqlens"].tolist() == [0, 4, 6, 9]
    assert md["cu_context_offsets"].tolist() == [0, 4, 6, 9]
    md2 = oracle.step_metadata([t.blocks for t in tabs[:2]], [4, 2], [0, 0], [4, 2], 4, True)
    assert md2["position_ids"].tolist() == [[0, 1, 2, 3, 0, 1]]
    expected = np.array([[1, 0, 0, 0, 0, 0], [1, 1, 0, 0, 0, 0], [1, 1, 1, 0, 0, 0],
                         [1, 1, 1, 1, 0, 0], [0, 0, 0, 0, 1, 0], [0, 0, 0, 0, 1, 1]], bool)
    np.testing.assert_array_equal(md2["attention_mask"][0, 0], expected)
    # tests/unit/test_allocator_bindings.py:25-35 and :89-107 (FIFO order, refcounts)
    f = oracle.Fifo(3)
    assert f.allocate_block() == 0 and f.allocate_block() == 1
    f.share_block(0)
    f.free_block(0)
    assert f.get_num_free_blocks() == 1
    f.free_block(0)
    assert f.get_num_free_blocks() == 2
    with pytest.raises(RuntimeError, match="Double-free"):
        f.free_block(0)
    with pytest.raises(RuntimeError, match="Cannot share"):
        f.share_block(0)
    with pytest.raises(IndexError, match="Block ID out of range"):
        f.free_block(3)
    f8 = oracle.Fifo(8)
    t = oracle.SeqTable(f8, 4)
    t.append_tokens(5)
    assert t.blocks == [0, 1] and f8.get_num_free_blocks() == 6
    t.release()
    assert f8.get_num_free_blocks() == 8
    # tests/stress/test_03_ragged_layout.py:10-42 (padded block tables, context lens)
    f20 = oracle.Fifo(20)
    tabs = []
    for n in (1, 7, 13):
        t = oracle.SeqTable(f20, 4)
        t.append_tokens(n)
        tabs.append(t)
    bt, cl = oracle.build_block_tables([t.blocks for t in tabs], [1, 7, 13])
    assert bt.shape == (3, 4) and cl.tolist() == [1, 7, 13]
    assert bt[0, 1:].tolist() == [-1, -1, -1] and bt[1, 2:].tolist() == [-1, -1]
    assert -1 not in bt[2].tolist()


def test_allocator_trace_matches_reference(golden, oracle):
    tr = jload(golden, "alloc_trace")
    fifo = oracle.Fifo(tr["total_blocks"])
    tabs = {}
    for kind, sid, n, ok, blocks, free_after, _ in tr["ops"]:
        if kind in ("new", "append"):
            t = tabs.setdefault(sid, oracle.SeqTable(fifo, tr["block_size"]))
            got_ok = 1
            try:
                t.append_tokens(n)
            except RuntimeError:
                got_ok = 0
            assert got_ok == ok
            assert t.blocks == blocks
        else:
            t = tabs.pop(sid)
            assert t.blocks == blocks
            t.release()
        assert fifo.get_num_free_blocks() == free_after


def test_scheduler_trace_matches_reference(golden, oracle):
    tr = jload(golden, "sched_trace")
    fifo = oracle.Fifo(tr["total_blocks"])
    tabs = {}
    for step in tr["steps"]:
        for kind, sid, n in step["calls"]:
            if kind == "free":
                tabs.pop(sid).release()
            else:
                tabs.setdefault(sid, oracle.SeqTable(fifo, tr["block_size"])).append_tokens(n)
        assert {int(k): v for k, v in step["tables"].items()} == \
            {k: t.blocks for k, t in tabs.items()}
        assert fifo.get_num_free_blocks() == step["free"]


def test_attention_cases_bit_exact(golden, oracle):
    for name in golden["attn_cases"]:
        p = f"attn_{name}_"
        q, kc, vc = golden[p + "q"], golden[p + "k_cache"], golden[p + "v_cache"]
        out = oracle.paged_attention(q, kc, vc, 1, golden[p + "gather_slots"], golden[p + "mask"],
                                     float(golden[p + "scale"]))
        np.testing.assert_array_equal(out, golden[p + "out"], err_msg=str(name))
        tables = ragged(golden, p)
        bt = np.zeros((len(tables), max(len(t) for t in tables)), np.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = t
        rg = oracle.paged_ragged(q[0].transpose(1, 0, 2), kc, vc, 1, bt, golden[p + "starts"],
                                 golden[p + "counts"], float(golden[p + "scale"]))
        np.testing.assert_array_equal(rg, golden[p + "out"][0], err_msg=str(name))


def test_config1_bit_exact(golden, oracle):
    import hashlib
    from config1_inputs import config1_inputs
    b, q, kc, vc, gs, mask = config1_inputs()
    h = hashlib.sha256()
    for a in (q, kc, vc, gs, mask):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(golden["config1_digest"]), "config-1 generator drifted"
    out = oracle.paged_attention(q, kc, vc, 0, gs, mask, b.scale)
    np.testing.assert_array_equal(out, golden["config1_out"])
    rg = oracle.paged_ragged(q[0].transpose(1, 0, 2), kc, vc, 0, np.maximum(b.block_tables(), 0),
                             b.start_positions, b.new_token_counts, b.scale)
    np.testing.assert_array_equal(rg, golden["config1_out"][0])


@pytest.mark.skipif(not __import__("os").path.exists(
    __import__("os").path.join(__import__("os").path.dirname(__file__), "..", "oracle", "_ref",
                               "libref_paged_kernels.so")), reason="compiled reference absent")
def test_oracle_matches_compiled_reference_random(oracle):
    ref = oracle.RefKernel()
    rng = np.random.default_rng(5)
    for trial in range(6):
        hkv = int(rng.choice([1, 2, 4]))
        hq = hkv * int(rng.choice([1, 2, 3, 4]))
        d = int(rng.choice([8, 16, 64]))
        bs = int(rng.choice([1, 4, 16]))
        S = int(rng.integers(1, 6))
        counts = rng.integers(1, 9, size=S)
        starts = rng.integers(0, 40, size=S)
        ctx = starts + counts
        nb_need = [-(-int(c) // bs) for c in ctx]
        NB = sum(nb_need) + 3
        perm = rng.permutation(NB)
        tables, off = [], 0
        for n in nb_need:
            tables.append(perm[off:off + n].tolist())
            off += n
        kc = rng.standard_normal((2, NB, bs, hkv, d), dtype=np.float32)
        vc = rng.standard_normal((2, NB, bs, hkv, d), dtype=np.float32)
        md = oracle.step_metadata(tables, ctx.tolist(), starts.tolist(), counts.tolist(), bs, True)
        q = rng.standard_normal((1, hq, int(counts.sum()), d), dtype=np.float32)
        scale = float(rng.uniform(0.05, 1.0))
        r = ref.paged_attention(q, kc, vc, trial % 2, md["gather_slots"], md["attention_mask"],
                                scale)
        o = oracle.paged_attention(q, kc, vc, trial % 2, md["gather_slots"], md["attention_mask"],
                                   scale)
        np.testing.assert_array_equal(o, r)
        bt = np.zeros((S, max(nb_need)), np.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = t
        rg = oracle.paged_ragged(q[0].transpose(1, 0, 2), kc, vc, trial % 2, bt, starts, counts,
                                 scale)
        np.testing.assert_array_equal(rg, r[0])


def test_empty_context_gives_zeros(oracle):
    q = np.ones((1, 2, 3, 8), np.float32)
    kc = np.ones((1, 2, 4, 1, 8), np.float32)
    out = oracle.paged_attention(q, kc, kc, 0, np.zeros(0, np.int32), np.zeros((1, 1, 3, 0), np.uint8),
                                 0.5)
    assert out.shape == (1, 3, 2, 8) and not out.any()


@pytest.mark.skipif(not __import__("os").path.exists(
    __import__("os").path.join(__import__("os").path.dirname(__file__), "..", "oracle", "_ref",
                               "libref_paged_kernels.so")), reason="compiled reference absent")
def test_oracle_matches_compiled_reference_random_masks(oracle):
    """Arbitrary masks (not block-diagonal causal), with a fully masked row and a fully open one:
    the oracle stays bit-exact to the reference kernel, and a fully masked row is zeros
    (paged_kernels.cpp:27-104)."""
    ref = oracle.RefKernel()
    rng = np.random.default_rng(17)
    hkv, hq, d, bs, NB = 2, 6, 16, 4, 12
    nq, nctx = 7, 30
    kc = rng.standard_normal((1, NB, bs, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((1, NB, bs, hkv, d), dtype=np.float32)
    q = rng.standard_normal((1, hq, nq, d), dtype=np.float32)
    gs = rng.permutation(NB * bs)[:nctx].astype(np.int32)
    mask = (rng.random((1, 1, nq, nctx)) < 0.4).astype(np.uint8)
    mask[0, 0, 2] = 0
    mask[0, 0, 5] = 1
    r = ref.paged_attention(q, kc, vc, 0, gs, mask, 0.3)
    o = oracle.paged_attention(q, kc, vc, 0, gs, mask, 0.3)
    np.testing.assert_array_equal(o, r)
    assert not o[0, 2].any() and np.isfinite(o).all()


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_oracle_scatter_matches_reference_index_put(oracle, dtype):
    """reshape_and_cache as the reference writes it (manager.py:150-168):
    cache[layer].view(-1, Hkv, D)[slot_mapping] = k, here with torch index_put on the same
    arrays; bit-exact.  Slots past the pool (the reference would raise) and negative padding
    slots (torch would wrap them) are skipped, and the oracle counts both."""
    import torch
    rng = np.random.default_rng(3)
    L, NB, BS, H, D = 2, 9, 4, 3, 16
    kc = rng.standard_normal((L, NB, BS, H, D)).astype(dtype)
    vc = rng.standard_normal((L, NB, BS, H, D)).astype(dtype)
    n = 20
    slots = rng.permutation(NB * BS)[:n].astype(np.int64)
    k = rng.standard_normal((n, H, D)).astype(dtype)
    v = rng.standard_normal((n, H, D)).astype(dtype)
    ref_k, ref_v = torch.from_numpy(kc.copy()), torch.from_numpy(vc.copy())
    ref_k[1].view(-1, H, D)[torch.from_numpy(slots)] = torch.from_numpy(k)
    ref_v[1].view(-1, H, D)[torch.from_numpy(slots)] = torch.from_numpy(v)
    got_k, got_v = kc.copy(), vc.copy()
    assert oracle.reshape_and_cache(k, v, got_k, got_v, slots, 1) == 0
    np.testing.assert_array_equal(got_k, ref_k.numpy())
    np.testing.assert_array_equal(got_v, ref_v.numpy())
    # padding and out-of-range entries
    bad = slots.copy()
    bad[0], bad[1] = -1, NB * BS
    got_k2, got_v2 = kc.copy(), vc.copy()
    assert oracle.reshape_and_cache(k, v, got_k2, got_v2, bad, 1) == 2   # both skipped
    keep = slice(2, None)
    ref_k2 = torch.from_numpy(kc.copy())
    ref_k2[1].view(-1, H, D)[torch.from_numpy(slots[keep])] = torch.from_numpy(k[keep])
    np.testing.assert_array_equal(got_k2, ref_k2.numpy())


def test_metadata_matches_reference_fuzz(oracle):
    """40 random steps recorded from the reference's PagedStepContext + build_block_tables
    (tests/golden/meta_fuzz.json.gz): mixed prefill / decode / chunk rows, block sizes 1-16,
    shuffled pools."""
    import gzip
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "meta_fuzz.json.gz")
    with gzip.open(path, "rt") as f:
        cases = json.load(f)
    assert len(cases) == 40
    for i, c in enumerate(cases):
        md = oracle.step_metadata(c["tables"], c["tokens"], c["starts"], c["counts"],
                                  c["block_size"])
        for key in ("cu_seqlens", "cu_context_offsets", "context_lens", "scatter_slots",
                    "gather_slots"):
            assert md[key].tolist() == c[key], (i, key)
        assert md["position_ids"][0].tolist() == c["position_ids"], i
        bt, cl = oracle.build_block_tables(c["tables"], c["tokens"])
        assert bt.tolist() == c["block_tables"] and cl.tolist() == c["bt_context_lens"], i
