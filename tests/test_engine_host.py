"""CPU tests of the engine's host side: the scheduler policy against the reference's recorded
Scheduler trace, and the tensor-parallel sharding of the model (2 gloo ranks vs 1)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from golden_util import jload


class HostKV:
    """Test stand-in for the KV manager on the host allocator mirror (llm_allocator_cpp
    drop-in); records the allocation calls the scheduler makes."""

    def __init__(self, la, total_blocks, block_size):
        self.allocator = la.PageAllocator(total_blocks, block_size, 64, 0)
        self.la = la
        self.block_size = block_size
        self.calls = []

    def get_allocator(self):
        return self.allocator

    def allocate_prefix_blocks(self, seq):
        if seq.block_table is None:
            seq.block_table = self.la.SequenceBlockTable(self.allocator)
        n = seq.total_len - seq.block_table.get_tokens_count()
        seq.block_table.append_tokens(n)
        self.calls.append(("prefix", seq.seq_id, n))

    def allocate_slot_for_next_token(self, seq):
        seq.block_table.append_token()
        self.calls.append(("append", seq.seq_id, 1))

    def free_sequence(self, seq):
        if seq.block_table is not None:
            seq.block_table.release()
            seq.block_table = None
            self.calls.append(("free", seq.seq_id, 0))


def test_scheduler_policy_replays_reference_trace(golden, pkg):
    """Same requests as the recorded reference run (tests/golden/make_golden.py:
    scheduler_trace): identical allocator calls, block tables and preemptions every step."""
    from llm_serving_b200 import llm_allocator_cpp as la
    from llm_serving_b200.engine import Scheduler, Sequence
    tr = jload(golden, "sched_trace")
    kv = HostKV(la, tr["total_blocks"], tr["block_size"])
    sched = Scheduler(kv, max_batch_size=6, max_num_batched_tokens=64, max_model_len=200)
    rng = np.random.default_rng(tr["seed"])
    seqs = []
    for i in range(14):
        plen = int(rng.integers(1, 24))
        s = Sequence(i + 1, list(range(plen)), max_tokens=int(rng.integers(2, 20)))
        sched.add_sequence(s)
        seqs.append(s)
    for step in tr["steps"]:
        kv.calls.clear()
        out = sched.schedule()
        # the reference engine appends one token to every scheduled sequence, prefills first,
        # then frees the finished ones (app/engine/llm_engine.py:237-258)
        for s in out.scheduled_prefills + out.scheduled_decodes:
            s.append_token(100 + s.total_len)
        for s in out.scheduled_prefills + out.scheduled_decodes:
            if s.is_finished():
                sched.free_sequence(s)
        assert [tuple(c) for c in kv.calls] == [tuple(c) for c in step["calls"]]
        live = {s.seq_id: s.block_table.get_physical_blocks() for s in seqs
                if s.block_table is not None}
        assert live == {int(k): v for k, v in step["tables"].items()}
        assert kv.allocator.get_num_free_blocks() == step["free"]
        assert sched.preemption_count == step["preemptions"]
    assert not sched.has_unfinished_sequences()


def _dense_attend_factory(pos, hq, hkv):
    """Causal attention over the tokens of ONE sequence held in memory (test stand-in for the
    paged kernels, so the model math can run on CPU)."""
    def attend(layer, q, k, v):
        G = hq // hkv
        kk = k.float().repeat_interleave(G, dim=1)
        vv = v.float().repeat_interleave(G, dim=1)
        s = torch.einsum("thd,shd->hts", q.float(), kk) / (q.shape[-1] ** 0.5)
        n = q.shape[0]
        mask = torch.triu(torch.ones(n, n, dtype=torch.bool), 1)
        s = s.masked_fill(mask, float("-inf"))
        return torch.einsum("hts,shd->thd", s.softmax(-1), vv).to(q.dtype)
    return attend


def _tp_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from llm_serving_b200.model import LlamaShape, TPLlama
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    shape = LlamaShape(2, 64, 8, 4, 16, 96, 50)
    m = TPLlama(shape, rank, world, torch.device("cpu"), torch.float32, seed=3, full_init=True)
    ids = torch.tensor([5, 17, 3, 42, 8, 1, 49])
    pos = torch.arange(len(ids))
    h = m.forward(ids, pos, _dense_attend_factory(pos, m.hq, m.hkv))
    logits = m.logits(h)
    tok = m.greedy(h)
    if rank == 0:
        q.put((logits.numpy(), tok.numpy()))
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tensor_parallel_sharding_matches_single_rank(pkg):
    ctx = mp.get_context("spawn")
    results = {}
    for world in (1, 2):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
        for p in procs:
            p.start()
        results[world] = q.get(timeout=240)
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    l1, t1 = results[1]
    l2, t2 = results[2]
    np.testing.assert_allclose(l2, l1, rtol=1e-4, atol=1e-5)
    assert (t1 == t2).all()
    assert (t1 == l1.argmax(-1)).all()


class SlottedKV(HostKV):
    """HostKV with the device pool's two fixed limits: table rows of `row` blocks and `slots`
    sequence slots."""

    def __init__(self, la, total_blocks, block_size, row, slots):
        super().__init__(la, total_blocks, block_size)
        self.max_blocks_per_seq = row
        self.slots = slots

    def num_free_sequence_slots(self):
        return self.slots

    def allocate_prefix_blocks(self, seq):
        if seq.block_table is None:
            assert self.slots > 0, "admitted without a free sequence slot"
            self.slots -= 1
        super().allocate_prefix_blocks(seq)

    def free_sequence(self, seq):
        if seq.block_table is not None:
            self.slots += 1
        super().free_sequence(seq)


def test_scheduler_respects_device_pool_limits(pkg):
    from llm_serving_b200 import llm_allocator_cpp as la
    from llm_serving_b200.engine import Scheduler, Sequence
    kv = SlottedKV(la, total_blocks=64, block_size=4, row=3, slots=2)
    sched = Scheduler(kv, max_batch_size=8, max_num_batched_tokens=1024, max_model_len=64)
    with pytest.raises(ValueError, match="block table row"):
        sched.add_sequence(Sequence(1, [1] * 9, max_tokens=4))    # 13 tokens = 4 blocks > 3
    seqs = [Sequence(i, [1] * 3, max_tokens=2) for i in range(2, 6)]
    for s in seqs:
        sched.add_sequence(s)
    out = sched.schedule()
    assert [s.seq_id for s in out.scheduled_prefills] == [2, 3]   # two slots, two admissions
    assert [s.seq_id for s in out.ignored_sequences] == [4, 5]
    for s in out.scheduled_prefills:                               # both finish: slots come back
        s.append_token(0)
        s.append_token(0)
        sched.free_sequence(s)
    out = sched.schedule()
    assert [s.seq_id for s in out.scheduled_prefills] == [4, 5]
