"""GPU parity of reshape_and_cache (K2), the device block pool (K5) and the step metadata (K4):
bit-exact against the oracle and against fixtures recorded from the reference's own allocator,
scheduler and PagedStepContext."""
import numpy as np
import pytest
import torch

from golden_util import jload, ragged

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(pkg):
    from llm_serving_b200 import paged_ops
    return paged_ops


@pytest.fixture(scope="module")
def bm(pkg):
    from llm_serving_b200 import block_manager
    return block_manager


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_reshape_and_cache_bit_exact(ops, oracle, dtype):
    L, NB, BS, Hkv, D = 3, 40, 16, 4, 64
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    kc = torch.randn((L, NB, BS, Hkv, D), generator=g, device="cuda").to(dtype)
    vc = torch.randn((L, NB, BS, Hkv, D), generator=g, device="cuda").to(dtype)
    n = 150
    slots = torch.randperm(NB * BS, generator=torch.Generator().manual_seed(2))[:n].cuda()
    # the HF layout: (1, Hkv, Ntok, D) transposed to (Ntok, Hkv, D), a strided view
    k4 = torch.randn((1, Hkv, n, D), generator=g, device="cuda").to(dtype)
    v4 = torch.randn((1, Hkv, n, D), generator=g, device="cuda").to(dtype)
    k = k4.squeeze(0).transpose(0, 1)
    v = v4.squeeze(0).transpose(0, 1)
    if dtype != torch.bfloat16:
        kref, vref = kc.cpu().numpy().copy(), vc.cpu().numpy().copy()
    if dtype == torch.bfloat16:
        kref, vref = kc.view(torch.int16).cpu().numpy().copy(), vc.view(torch.int16).cpu().numpy().copy()
        kin, vin = k.contiguous().view(torch.int16).cpu().numpy(), v.contiguous().view(torch.int16).cpu().numpy()
    else:
        kin, vin = k.contiguous().cpu().numpy(), v.contiguous().cpu().numpy()
    bad = oracle.reshape_and_cache(kin, vin, kref, vref, slots.cpu().numpy(), 1)
    assert bad == 0
    ops.reshape_and_cache(k, v, kc, vc, slots, 1)
    got_k = (kc.view(torch.int16) if dtype == torch.bfloat16 else kc).cpu().numpy()
    got_v = (vc.view(torch.int16) if dtype == torch.bfloat16 else vc).cpu().numpy()
    assert np.array_equal(got_k, kref) and np.array_equal(got_v, vref)
    assert ops.read_status(kc.device) == 0


def test_reshape_and_cache_padding_and_bad_slots(ops):
    kc = torch.zeros((1, 4, 4, 2, 64), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    k = torch.ones((3, 2, 64), dtype=torch.bfloat16, device="cuda")
    slots = torch.tensor([-1, 5, 16], dtype=torch.int64, device="cuda")  # pad, ok, out of range
    ops.reshape_and_cache(k, k, kc, vc, slots, 0)
    flat = kc.view(-1, 2, 64)
    assert (flat[5] == 1).all() and (flat.sum() == 128)
    assert ops.read_status(kc.device) & 2  # B200_DEVICE_BAD_SLOT


def test_pool_replays_reference_allocator_trace(golden, bm, oracle):
    tr = jload(golden, "alloc_trace")
    pool = bm.DeviceBlockPool(tr["total_blocks"], tr["block_size"], 512, 64)
    slot_of = {}
    for kind, sid, n, ok, blocks, free_after, _ in tr["ops"]:
        if kind == "release":
            pool.release(slot_of.pop(sid))
        else:
            slot = slot_of.setdefault(sid, sid % 512)
            got_ok = 1
            try:
                pool.append_tokens(slot, n)
            except RuntimeError:
                got_ok = 0
            assert got_ok == ok
        assert pool.get_num_free_blocks() == free_after
        pool.flush()
        if kind != "release":
            assert pool.table(slot_of[sid]) == blocks
    # the free queue itself matches the oracle FIFO driven the same way
    fifo = oracle.Fifo(tr["total_blocks"])
    tabs = {}
    for kind, sid, n, ok, blocks, _, _ in tr["ops"]:
        if kind == "release":
            tabs.pop(sid).release()
        else:
            t = tabs.setdefault(sid, oracle.SeqTable(fifo, tr["block_size"]))
            try:
                t.append_tokens(n)
            except RuntimeError:
                pass
    assert pool.free_queue() == fifo.free_queue()
    assert pool.status() == 0


def test_pool_replays_reference_scheduler_trace_batched(golden, bm):
    """One flush per engine step (the batched device path), including recompute-preemption."""
    tr = jload(golden, "sched_trace")
    pool = bm.DeviceBlockPool(tr["total_blocks"], tr["block_size"], 64, 64)
    for step in tr["steps"]:
        for kind, sid, n in step["calls"]:
            if kind == "free":
                pool.release(sid)
            else:
                pool.append_tokens(sid, n)
        pool.flush()
        assert pool.get_num_free_blocks() == step["free"]
        tables = {int(k): v for k, v in step["tables"].items()}
        for sid, blocks in tables.items():
            assert pool.table(sid) == blocks
    assert pool.status() == 0


def test_step_metadata_matches_reference_context(golden, bm, oracle):
    for name in golden["meta_cases"]:
        p = f"meta_{name}_"
        tables = ragged(golden, p)
        tokens = golden[p + "tokens"]
        starts, counts = golden[p + "starts"], golden[p + "counts"]
        pool = bm.DeviceBlockPool(64, 4, 16, 32)
        # replay the reference's allocation order: every prompt (the cached prefix), then this
        # step's new tokens, sequence by sequence
        for s, n in enumerate(starts.tolist()):
            pool.append_tokens(s, n)
        for s, n in enumerate(counts.tolist()):
            pool.append_tokens(s, n)
        pool.flush()
        assert [pool.tokens(s) for s in range(len(tables))] == tokens.tolist()
        assert [pool.table(s) for s in range(len(tables))] == tables
        S = len(tables)
        md = pool.build_step_metadata(
            torch.arange(S, dtype=torch.int32, device="cuda"),
            torch.from_numpy(starts).cuda(), torch.from_numpy(counts).cuda(),
            int(counts.sum()), bt_stride=golden[p + "block_tables"].shape[1],
            with_gather_slots=True, num_context_tokens=int((starts + counts).sum()))
        assert np.array_equal(md["cu_seqlens"].cpu().numpy(), golden[p + "cu_seqlens"])
        assert np.array_equal(md["cu_context_offsets"].cpu().numpy(), golden[p + "cu_context_offsets"])
        assert np.array_equal(md["context_lens"].cpu().numpy(), golden[p + "context_lens"])
        assert np.array_equal(md["position_ids"].cpu().numpy(), golden[p + "position_ids"][0])
        assert np.array_equal(md["slot_mapping"].cpu().numpy(), golden[p + "scatter_slots"])
        assert np.array_equal(md["gather_slots"].cpu().numpy(), golden[p + "gather_slots"])
        assert np.array_equal(md["block_tables"].cpu().numpy(), golden[p + "block_tables"])
        assert pool.status() == 0


def test_step_metadata_config3_scale(pkg, bm, oracle):
    """Config-3 sized mixed step (16 prefill chunks + 240 decodes) on a shuffled pool."""
    b = pkg.workloads.config3(seed=0)
    nfill = 64
    nb = b.total_blocks
    per_fill = nb // nfill
    pool = bm.DeviceBlockPool(nb, 16, b.num_seqs + nfill, max(512, per_fill))
    # shuffle the free list: fillers take the whole pool, then release in a random order
    rng = np.random.default_rng(0)
    fillers = [b.num_seqs + i for i in range(nfill)]
    for f in fillers:
        pool.append_tokens(f, 16 * per_fill)
    pool.flush()
    for i in rng.permutation(nfill):
        pool.release(fillers[i])
    pool.flush()
    fifo_expect = pool.free_queue()
    starts = b.start_positions.astype(np.int32)
    counts = b.new_token_counts.astype(np.int32)
    for s in range(b.num_seqs):
        pool.append_tokens(s, int(starts[s] + counts[s]))
    pool.flush()
    tables = [pool.table(s) for s in range(b.num_seqs)]
    # the blocks handed out are the head of the shuffled queue, in sequence order
    flat = [x for t in tables for x in t]
    assert flat == fifo_expect[:len(flat)]
    md = pool.build_step_metadata(torch.arange(b.num_seqs, dtype=torch.int32, device="cuda"),
                                  torch.from_numpy(starts).cuda(), torch.from_numpy(counts).cuda(),
                                  int(counts.sum()), bt_stride=max(len(t) for t in tables))
    ref = oracle.step_metadata(tables, (starts + counts).tolist(), starts.tolist(),
                               counts.tolist(), 16)
    assert np.array_equal(md["cu_seqlens"].cpu().numpy(), ref["cu_seqlens"])
    assert np.array_equal(md["slot_mapping"].cpu().numpy(), ref["scatter_slots"])
    assert np.array_equal(md["position_ids"].cpu().numpy(), ref["position_ids"][0])
    bt, _ = oracle.build_block_tables(tables, (starts + counts).tolist())
    assert np.array_equal(md["block_tables"].cpu().numpy(), bt)


def _raw_metadata(pool, slots, starts, counts, num_tokens, room, bt_stride,
                  num_context_tokens=None, ctx_room=0):
    """b200_build_step_metadata called directly, with outputs `room` entries longer than the
    capacity the call declares and filled with a sentinel, so what lands past the capacity is
    visible (and stays inside memory this test owns)."""
    from llm_serving_b200 import _native as N
    dev = torch.device("cuda")
    S = len(slots)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
    d_slots, d_start, d_count = i32(slots), i32(starts), i32(counts)
    out = {
        "cu": torch.full((S + 1,), -7, dtype=torch.int64, device=dev),
        "cc": torch.full((S + 1,), -7, dtype=torch.int64, device=dev),
        "ctx": torch.full((S,), -7, dtype=torch.int32, device=dev),
        "pos": torch.full((num_tokens + room,), -7, dtype=torch.int64, device=dev),
        "slot": torch.full((num_tokens + room,), -7, dtype=torch.int64, device=dev),
        "bt": torch.full((S, bt_stride), -7, dtype=torch.int32, device=dev),
    }
    gather = None
    if num_context_tokens is not None:
        gather = torch.full((num_context_tokens + ctx_room,), -7, dtype=torch.int64, device=dev)
    N.check(N.lib().b200_build_step_metadata(
        pool._h, d_slots.data_ptr(), d_start.data_ptr(), d_count.data_ptr(), S, num_tokens,
        out["cu"].data_ptr(), out["cc"].data_ptr(), out["ctx"].data_ptr(), out["pos"].data_ptr(),
        out["slot"].data_ptr(), out["bt"].data_ptr(), bt_stride,
        None if gather is None else gather.data_ptr(),
        0 if gather is None else num_context_tokens, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out, gather


def test_step_metadata_stays_inside_its_outputs(bm):
    """Counts that overrun the declared output sizes, a sequence slot outside the pool and a
    negative count are flagged (B200_DEVICE_BAD_STEP) and skipped; nothing is written past the
    capacities, and the consistent sequences still get exact metadata."""
    from llm_serving_b200 import _native as N
    pool = bm.DeviceBlockPool(32, 16, max_seqs=4, max_blocks_per_seq=8)
    pool.append_tokens(0, 20)
    pool.append_tokens(1, 40)
    pool.flush()
    t0, t1 = pool.table(0), pool.table(1)
    assert pool.status() == 0

    # 1. the second sequence's 25 tokens do not fit a 30-token capacity after the first's 10
    out, _ = _raw_metadata(pool, [0, 1], [10, 15], [10, 25], num_tokens=30, room=8, bt_stride=4)
    assert pool.status() & N.DEVICE_BAD_STEP
    assert out["pos"][:10].tolist() == list(range(10, 20))
    assert out["slot"][:10].tolist() == [t0[p // 16] * 16 + p % 16 for p in range(10, 20)]
    assert (out["pos"][10:] == -7).all() and (out["slot"][10:] == -7).all()
    assert out["cu"].tolist() == [0, 10, 35] and out["ctx"].tolist() == [20, 40]
    assert out["bt"][1].tolist() == t1 + [-1]

    # 2. gather slots: a 50-entry capacity holds the first sequence's 20, not the second's 40
    out, g = _raw_metadata(pool, [0, 1], [19, 39], [1, 1], num_tokens=2, room=0, bt_stride=3,
                           num_context_tokens=50, ctx_room=16)
    assert pool.status() & N.DEVICE_BAD_STEP
    assert g[:20].tolist() == [t0[p // 16] * 16 + p % 16 for p in range(20)]
    assert (g[20:] == -7).all()

    # 3. a slot outside the pool and a negative count: flagged, treated as empty sequences
    out, _ = _raw_metadata(pool, [7, 1, 0], [0, 39, 0], [1, 1, -3], num_tokens=2, room=4,
                           bt_stride=3)
    st = pool.status()
    assert st & N.DEVICE_BAD_STEP and st & N.DEVICE_BAD_BLOCK
    assert out["bt"][0].tolist() == [-1, -1, -1] and out["slot"][0].item() == -1
    assert out["pos"][1].item() == 39 and out["slot"][1].item() == t1[2] * 16 + 39 % 16
    assert out["cu"].tolist() == [0, 1, 2, 2] and out["ctx"][2].item() == 0
    assert (out["pos"][2:] == -7).all()

    # a consistent call afterwards is clean
    _raw_metadata(pool, [0, 1], [19, 39], [1, 1], num_tokens=2, room=0, bt_stride=3)
    assert pool.status() == 0


def test_step_metadata_matches_reference_fuzz(bm):
    """The device pool and K4 on 40 random steps recorded from the reference (shuffled pools,
    block sizes 1-16, mixed prefill / decode / chunk rows): the pool replays the reference's
    allocation order (filler tables released in the recorded order, then the prompts, then the
    step's new tokens) and K4's outputs equal the reference's."""
    import gzip
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "meta_fuzz.json.gz")
    with gzip.open(path, "rt") as f:
        cases = json.load(f)
    for i, c in enumerate(cases):
        S, F, bs = len(c["prompts"]), len(c["fillers"]), c["block_size"]
        width = max([len(t) for t in c["tables"]] + [-(-n // bs) for n in c["fillers"]] + [1])
        pool = bm.DeviceBlockPool(c["total_blocks"], bs, S + F, width)
        for k, n in enumerate(c["fillers"]):
            pool.append_tokens(S + k, n)
        pool.flush()
        for k in c["release_order"]:
            pool.release(S + k)
        pool.flush()
        for s, n in enumerate(c["prompts"]):
            pool.append_tokens(s, n)
        for s in range(S):
            pool.append_tokens(s, c["tokens"][s] - c["prompts"][s])
        pool.flush()
        assert [pool.table(s) for s in range(S)] == c["tables"], i
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")
        md = pool.build_step_metadata(
            torch.arange(S, dtype=torch.int32, device="cuda"), i32(c["starts"]), i32(c["counts"]),
            sum(c["counts"]), bt_stride=len(c["block_tables"][0]), with_gather_slots=True,
            num_context_tokens=sum(c["context_lens"]))
        for key in ("cu_seqlens", "cu_context_offsets", "context_lens", "gather_slots",
                    "block_tables"):
            assert md[key].cpu().tolist() == c[key], (i, key)
        assert md["slot_mapping"].cpu().tolist() == c["scatter_slots"], i
        assert md["position_ids"].cpu().tolist() == c["position_ids"], i
        assert pool.status() == 0, i
