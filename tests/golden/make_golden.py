"""Generate the golden fixtures in tests/golden/ by running the REFERENCE implementation.

Run in a container that has the reference tree and its compiled binding:

    make -C oracle ref
    PYTHONPATH=<reference checkout>:oracle/_ref python tests/golden/make_golden.py

It imports the reference's own Python (app.memory.manager.PagedKVCacheManager,
app.model.paged_attention.PagedStepContext, app.scheduler.Scheduler, app.engine.LLMEngine with
its MockModelClient) and its C++ binding llm_allocator_cpp (PageAllocator, SequenceBlockTable,
paged_attention) compiled from the reference sources, and records what they produce on seeded
inputs.  Nothing from the reference is copied into the fixtures except those outputs and the
seeded inputs that produced them.  The GPU box never runs this script; the tests only read the
fixtures it wrote.
"""
from __future__ import annotations

import gzip
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import llm_allocator_cpp  # noqa: E402  (reference binding, from oracle/_ref)
from app.memory.manager import PagedKVCacheManager  # noqa: E402
from app.model.paged_attention import PagedStepContext  # noqa: E402
from app.scheduler.scheduler import Scheduler  # noqa: E402
from app.scheduler.sequence import Sequence  # noqa: E402
from app.engine.llm_engine import LLMEngine  # noqa: E402
from app.model.client import MockModelClient  # noqa: E402

import __graft_entry__  # noqa: E402

workloads = __graft_entry__.load_package().workloads


def _ragged(lists):
    flat = np.asarray([x for l in lists for x in l], dtype=np.int32)
    offs = np.zeros(len(lists) + 1, dtype=np.int64)
    offs[1:] = np.cumsum([len(l) for l in lists])
    return flat, offs


def metadata_cases(out):
    """PagedStepContext + build_block_tables on ragged prefill / decode / mixed steps."""
    cases = [
        ("prefill_4_2_3", [4, 2, 3], "prefill", None),
        ("prefill_7_2_5_1", [7, 2, 5, 1], "prefill", None),
        ("decode_4_2", [4, 2], "decode", None),
        ("decode_boundary", [4, 8, 3, 12, 1], "decode", None),
        ("mixed", [9, 3, 14, 6], "mixed", [0, 1]),
    ]
    for name, lens, kind, decode_idx in cases:
        store = PagedKVCacheManager(total_blocks=64, block_size=4, num_heads=2, head_dim=8,
                                    num_layers=1, device="cpu")
        seqs = []
        for i, n in enumerate(lens):
            s = Sequence(seq_id=i + 1, prompt_token_ids=list(range(n)))
            store.allocate_prefix_blocks(s)
            seqs.append(s)
        if kind == "prefill":
            starts, counts = [0] * len(seqs), list(lens)
        elif kind == "decode":
            for s in seqs:
                store.allocate_slot_for_next_token(s)
            starts = [s.block_table.get_tokens_count() - 1 for s in seqs]
            counts = [1] * len(seqs)
        else:  # decode for decode_idx, a 3-token chunk on top of the cached prefix otherwise
            starts, counts = [], []
            for i, s in enumerate(seqs):
                prev = s.block_table.get_tokens_count()
                n_new = 1 if i in decode_idx else 3
                for _ in range(n_new):
                    store.allocate_slot_for_next_token(s)
                starts.append(prev)
                counts.append(n_new)
        ctx = PagedStepContext(store, seqs, starts, counts)
        tables = [list(s.block_table.get_physical_blocks()) for s in seqs]
        flat, offs = _ragged(tables)
        bt, cl = store.build_block_tables(seqs)
        p = f"meta_{name}_"
        out[p + "tables_flat"] = flat
        out[p + "tables_offs"] = offs
        out[p + "tokens"] = np.asarray([s.block_table.get_tokens_count() for s in seqs], np.int32)
        out[p + "starts"] = np.asarray(starts, np.int32)
        out[p + "counts"] = np.asarray(counts, np.int32)
        out[p + "cu_seqlens"] = ctx.cu_seqlens.numpy()
        out[p + "cu_context_offsets"] = ctx.cu_context_offsets.numpy()
        out[p + "context_lens"] = np.asarray(ctx.context_lens, np.int64)
        out[p + "scatter_slots"] = ctx.scatter_slots.numpy()
        out[p + "gather_slots"] = ctx.gather_slots.numpy()
        out[p + "position_ids"] = ctx.position_ids(torch.device("cpu")).numpy()
        out[p + "mask"] = ctx.attention_mask(torch.device("cpu")).numpy()
        out[p + "block_tables"] = bt.numpy()
        out[p + "bt_context_lens"] = cl.numpy()
    out["meta_cases"] = np.asarray([c[0] for c in cases])


def metadata_fuzz(num_cases=40, seed=77):
    """PagedStepContext + build_block_tables on random steps (tests/golden/meta_fuzz.json.gz):
    1-12 sequences with prompts of 1-40 tokens on a pool of block size 1-16 whose free list was
    first shuffled by filler tables; each sequence is a whole-prompt prefill, a decode, or a chunk
    of new tokens on its cached prompt.  Records the inputs (including the filler allocations and
    the release order that shuffled the pool, and the prompt lengths, so the device pool can
    replay the same allocation order) and every output."""
    rng = np.random.default_rng(seed)
    cases = []
    for _ in range(num_cases):
        bs = int(rng.choice([1, 2, 4, 8, 16]))
        S = int(rng.integers(1, 13))
        prompts = [int(x) for x in rng.integers(1, 41, size=S)]
        kinds = [str(k) for k in rng.choice(["prefill", "decode", "chunk"], size=S)]
        extra = [0 if k == "prefill" else (1 if k == "decode" else int(rng.integers(2, 20)))
                 for k in kinds]
        need = sum(-(-(p + e) // bs) for p, e in zip(prompts, extra))
        total = need + int(rng.integers(0, need + 1))
        store = PagedKVCacheManager(total_blocks=total, block_size=bs, num_heads=2, head_dim=8,
                                    num_layers=1, device="cpu")
        # shuffle the free list: filler tables take blocks, then give them back in random order
        fillers = [int(x) for x in rng.integers(1, 3 * bs + 1, size=int(rng.integers(0, 4)))]
        tabs = []
        for n in fillers:
            if -(-n // bs) > store.get_allocator().get_num_free_blocks():
                break
            t = llm_allocator_cpp.SequenceBlockTable(store.get_allocator())
            for _ in range(n):
                t.append_token()
            tabs.append(t)
        fillers = fillers[:len(tabs)]
        release_order = [int(i) for i in rng.permutation(len(tabs))]
        for i in release_order:
            tabs[i].release()
        seqs = []
        for i, n in enumerate(prompts):
            q = Sequence(seq_id=i + 1, prompt_token_ids=list(range(n)))
            store.allocate_prefix_blocks(q)
            seqs.append(q)
        starts, counts = [], []
        for q, k, e in zip(seqs, kinds, extra):
            prev = q.block_table.get_tokens_count()
            for _ in range(e):
                store.allocate_slot_for_next_token(q)
            if k == "prefill":
                starts.append(0)
                counts.append(prev)
            else:
                starts.append(prev if k == "chunk" else prev + e - 1)
                counts.append(e)
        ctx = PagedStepContext(store, seqs, starts, counts)
        bt, cl = store.build_block_tables(seqs)
        cases.append({
            "block_size": bs, "total_blocks": total, "fillers": fillers,
            "release_order": release_order, "prompts": prompts,
            "tables": [list(map(int, q.block_table.get_physical_blocks())) for q in seqs],
            "tokens": [int(q.block_table.get_tokens_count()) for q in seqs],
            "starts": starts, "counts": counts,
            "cu_seqlens": ctx.cu_seqlens.tolist(),
            "cu_context_offsets": ctx.cu_context_offsets.tolist(),
            "context_lens": [int(x) for x in ctx.context_lens],
            "scatter_slots": ctx.scatter_slots.tolist(),
            "gather_slots": ctx.gather_slots.tolist(),
            "position_ids": ctx.position_ids(torch.device("cpu"))[0].tolist(),
            "block_tables": bt.tolist(), "bt_context_lens": cl.tolist()})
    path = os.path.join(HERE, "meta_fuzz.json.gz")
    with gzip.open(path, "wt") as f:
        json.dump(cases, f, separators=(",", ":"))
    print("wrote", path, os.path.getsize(path), "bytes")


def allocator_trace(out, seed=7, total_blocks=20, block_size=4, num_ops=400):
    """Seeded append/release/share/free ops on the reference PageAllocator/SequenceBlockTable.
    Records every op and the blocks each op handed out, so the FIFO order (including the order
    freed blocks re-enter the queue) is pinned."""
    rng = np.random.default_rng(seed)
    alloc = llm_allocator_cpp.PageAllocator(total_blocks, block_size, 64, 0)
    tables = {}
    ops = []  # (kind, seq, arg, result_blocks, free_after)
    next_id = 0
    for _ in range(num_ops):
        r = rng.random()
        if r < 0.35 or not tables:
            sid = next_id
            next_id += 1
            n = int(rng.integers(1, 3 * block_size + 1))
            t = llm_allocator_cpp.SequenceBlockTable(alloc)
            before = alloc.get_num_free_blocks()
            try:
                for _ in range(n):
                    t.append_token()
                ok = 1
            except RuntimeError:
                ok = 0
            tables[sid] = t
            ops.append(("new", sid, n, ok, list(t.get_physical_blocks()),
                        alloc.get_num_free_blocks(), before))
        elif r < 0.6:
            sid = int(rng.choice(list(tables)))
            t = tables[sid]
            n = int(rng.integers(1, block_size + 2))
            before = alloc.get_num_free_blocks()
            try:
                for _ in range(n):
                    t.append_token()
                ok = 1
            except RuntimeError:
                ok = 0
            ops.append(("append", sid, n, ok, list(t.get_physical_blocks()),
                        alloc.get_num_free_blocks(), before))
        else:
            sid = int(rng.choice(list(tables)))
            t = tables.pop(sid)
            blocks = list(t.get_physical_blocks())
            t.release()
            ops.append(("release", sid, 0, 1, blocks, alloc.get_num_free_blocks(), 0))
    out["alloc_trace"] = np.asarray(json.dumps({
        "seed": seed, "total_blocks": total_blocks, "block_size": block_size,
        "ops": ops}))


def record_schedule(seed, total_blocks, block_size, num_requests, max_batch_size=6,
                    max_num_batched_tokens=64, max_model_len=200, max_prompt=24, max_out=20):
    """The reference Scheduler + LLMEngine (MockModelClient) on one seeded request stream.
    Returns (steps, finished): per step, the allocator calls in order, every live sequence's
    block table afterwards, the free-block count and the preemption count; finished is False
    when requests were still waiting after 400 steps (a prompt longer than the token budget is
    never admitted, and the reference engine keeps stepping)."""
    rng = np.random.default_rng(seed)
    kv = PagedKVCacheManager(total_blocks=total_blocks, block_size=block_size, num_heads=2,
                             head_dim=8, num_layers=16, device="cpu")
    calls = []
    orig = (kv.allocate_prefix_blocks, kv.allocate_slot_for_next_token, kv.free_sequence)

    def prefix(seq):
        before = seq.block_table.get_tokens_count() if seq.block_table is not None else 0
        orig[0](seq)
        calls.append(("prefix", seq.seq_id, seq.total_len - before))

    def slot(seq):
        orig[1](seq)
        calls.append(("append", seq.seq_id, 1))

    def free(seq):
        had = seq.block_table is not None
        orig[2](seq)
        if had:
            calls.append(("free", seq.seq_id, 0))

    kv.allocate_prefix_blocks, kv.allocate_slot_for_next_token, kv.free_sequence = prefix, slot, free
    sched = Scheduler(kv_cache_manager=kv, max_batch_size=max_batch_size,
                      max_num_batched_tokens=max_num_batched_tokens, block_size=block_size,
                      max_model_len=max_model_len)
    eng = LLMEngine(kv_cache_manager=kv, scheduler=sched, model_client=MockModelClient())
    seqs = []
    for _ in range(num_requests):
        plen = int(rng.integers(1, max_prompt))
        seqs.append(eng.add_request(prompt_token_ids=list(range(plen)),
                                    max_tokens=int(rng.integers(2, max_out))))
    steps = []
    for _ in range(400):
        if not eng.has_unfinished_requests():
            break
        calls.clear()
        eng.step()
        live = {s.seq_id: list(s.block_table.get_physical_blocks())
                for s in seqs if s.block_table is not None}
        steps.append({"calls": list(calls), "tables": live,
                      "free": kv.get_allocator().get_num_free_blocks(),
                      "preemptions": sched.preemption_count})
    return steps, not eng.has_unfinished_requests()


def scheduler_trace(out, seed=11, total_blocks=40, block_size=4, num_requests=14):
    """One stream on a pool small enough to force recompute-preemption."""
    steps, _ = record_schedule(seed, total_blocks, block_size, num_requests)
    out["sched_trace"] = np.asarray(json.dumps({
        "seed": seed, "total_blocks": total_blocks, "block_size": block_size, "steps": steps}))


def scheduler_fuzz(num_streams=40, seed=2025):
    """Many streams with random pool sizes, block sizes, batch and token budgets and request
    mixes (tests/golden/sched_fuzz.json.gz): admission limits and recompute-preemption in many
    combinations.  Each entry holds the parameters and the recorded steps."""
    rng = np.random.default_rng(seed)
    streams = []
    while len(streams) < num_streams:
        p = {"seed": int(rng.integers(0, 1 << 30)),
             "block_size": int(rng.choice([1, 2, 4, 8, 16])),
             "num_requests": int(rng.integers(1, 20)),
             "max_batch_size": int(rng.integers(1, 10)),
             "max_num_batched_tokens": int(rng.choice([16, 32, 64, 256])),
             "max_prompt": int(rng.integers(2, 40)),
             "max_out": int(rng.integers(3, 30))}
        p["max_model_len"] = p["max_prompt"] + p["max_out"] + 8
        # every request must fit the pool on its own (the scheduler rejects it otherwise)
        need = -(-p["max_model_len"] // p["block_size"])
        p["total_blocks"] = int(need + rng.integers(0, 3 * need))
        try:
            steps, finished = record_schedule(p["seed"], p["total_blocks"], p["block_size"],
                                    p["num_requests"], p["max_batch_size"],
                                    p["max_num_batched_tokens"], p["max_model_len"],
                                    p["max_prompt"], p["max_out"])
        except ValueError:
            continue  # a request the reference refuses at add time (too long for the budget)
        streams.append({"params": p, "steps": steps, "finished": finished})
    path = os.path.join(HERE, "sched_fuzz.json.gz")
    with gzip.open(path, "wt") as f:
        json.dump(streams, f, separators=(",", ":"))
    print("wrote", path, os.path.getsize(path), "bytes")


def attention_cases(out):
    """The reference C++ kernel (llm_allocator_cpp.paged_attention) on the gather slots and mask
    that the reference PagedStepContext builds, as NativePagedBackend.attend issues it."""
    cases = [
        ("decode_gqa", [5, 17, 1, 33], "decode", 6, 2, 16, 0.25, 1.0),
        ("mixed_gqa", [9, 3, 14, 6], "mixed", 8, 2, 16, 0.3, 1.0),
        ("prefill_mha", [4, 2, 3], "prefill", 4, 4, 8, 0.35, 1.0),
        ("decode_large_values", [7, 2, 5, 1], "decode", 6, 2, 8, 0.35, 50.0),
    ]
    rng = np.random.default_rng(2024)
    for name, lens, kind, hq, hkv, d, scale, mag in cases:
        store = PagedKVCacheManager(total_blocks=64, block_size=4, num_heads=hkv, head_dim=d,
                                    num_layers=2, device="cpu")
        # shuffle the pool first so the block tables are not the identity
        t0 = llm_allocator_cpp.SequenceBlockTable(store.get_allocator())
        for _ in range(4 * 20):
            t0.append_token()
        keep = llm_allocator_cpp.SequenceBlockTable(store.get_allocator())
        for _ in range(4 * 5):
            keep.append_token()
        t0.release()
        seqs = []
        for i, n in enumerate(lens):
            s = Sequence(seq_id=i + 1, prompt_token_ids=list(range(n)))
            store.allocate_prefix_blocks(s)
            seqs.append(s)
        if kind == "prefill":
            starts, counts = [0] * len(seqs), list(lens)
        elif kind == "decode":
            for s in seqs:
                store.allocate_slot_for_next_token(s)
            starts = [s.block_table.get_tokens_count() - 1 for s in seqs]
            counts = [1] * len(seqs)
        else:
            starts, counts = [], []
            for i, s in enumerate(seqs):
                prev = s.block_table.get_tokens_count()
                n_new = 1 if i % 2 == 0 else 4
                for _ in range(n_new):
                    store.allocate_slot_for_next_token(s)
                starts.append(prev)
                counts.append(n_new)
        ctx = PagedStepContext(store, seqs, starts, counts)
        kc = (rng.standard_normal(store.key_cache.shape) * mag).astype(np.float32)
        vc = (rng.standard_normal(store.value_cache.shape) * mag).astype(np.float32)
        q = (rng.standard_normal((1, hq, ctx.num_query_tokens, d)) * mag).astype(np.float32)
        mask = ctx.attention_mask(torch.device("cpu")).to(torch.uint8).numpy()
        gs = ctx.gather_slots.to(torch.int32).numpy()
        o = llm_allocator_cpp.paged_attention(q, kc, vc, 1, gs, mask, scale)
        p = f"attn_{name}_"
        flat, offs = _ragged([list(s.block_table.get_physical_blocks()) for s in seqs])
        out[p + "q"] = q
        out[p + "k_cache"] = kc
        out[p + "v_cache"] = vc
        out[p + "gather_slots"] = gs
        out[p + "mask"] = mask
        out[p + "scale"] = np.float32(scale)
        out[p + "starts"] = np.asarray(starts, np.int32)
        out[p + "counts"] = np.asarray(counts, np.int32)
        out[p + "tables_flat"] = flat
        out[p + "tables_offs"] = offs
        out[p + "out"] = o
    out["attn_cases"] = np.asarray([c[0] for c in cases])


def config1_case(out):
    """Config 1 exactly as NativePagedBackend.attend issues it: one batched call with the
    reference's gather slots and dense decode mask.  Inputs are regenerated from the seeds by
    config1_inputs() (tests/golden/config1_inputs.py); only their digest and the reference
    output are stored."""
    sys.path.insert(0, HERE)
    from config1_inputs import config1_inputs
    b, q, kc, vc, gs, mask = config1_inputs()
    o = llm_allocator_cpp.paged_attention(q, kc, vc, 0, gs, mask, np.float32(b.scale))
    h = hashlib.sha256()
    for a in (q, kc, vc, gs, mask):
        h.update(np.ascontiguousarray(a).tobytes())
    out["config1_out"] = o
    out["config1_digest"] = np.asarray(h.hexdigest())


def main():
    out = {}
    metadata_cases(out)
    allocator_trace(out)
    scheduler_trace(out)
    attention_cases(out)
    config1_case(out)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if sys.argv[1:] == ["sched_fuzz"]:
        scheduler_fuzz()
    elif sys.argv[1:] == ["meta_fuzz"]:
        metadata_fuzz()
    else:
        main()
