"""The config-5 engine leg of bench.py must exercise recompute-preemption at every tensor-parallel
size of the scaling run ("block pool at 95 % occupancy ... forcing
preemption/recompute").  Host-only: the bench's own request set (bench.engine5_workload) is
replayed through this package's Scheduler (the reference policy, app/scheduler/scheduler.py:84-151)
with a KV manager that only counts blocks, for the warm-up and timed steps the bench runs."""
import numpy as np
import pytest

import bench


class CountingKV:
    """Block accounting of a paged KV cache (no data): what the scheduler reads and calls."""

    def __init__(self, total_blocks, block_size, max_blocks_per_seq):
        self.block_size = block_size
        self.max_blocks_per_seq = max_blocks_per_seq
        self.total = total_blocks
        self.free = total_blocks

    # allocator view
    def get_allocator(self):
        return self

    def get_num_free_blocks(self):
        return self.free

    def get_total_blocks(self):
        return self.total

    def _grow(self, seq, tokens):
        t = seq.block_table
        need = -(-(t["tokens"] + tokens) // self.block_size)
        assert need - t["blocks"] <= self.free, "scheduler allocated beyond the free blocks"
        self.free -= need - t["blocks"]
        t["blocks"], t["tokens"] = need, t["tokens"] + tokens

    def allocate_prefix_blocks(self, seq):
        if seq.block_table is None:
            seq.block_table = _Table()
        self._grow(seq, seq.total_len - seq.block_table["tokens"])

    def allocate_slot_for_next_token(self, seq):
        self._grow(seq, 1)

    def free_sequence(self, seq):
        if seq.block_table is not None:
            self.free += seq.block_table["blocks"]
            seq.block_table = None


class _Table(dict):
    def __init__(self):
        super().__init__(tokens=0, blocks=0)

    def get_tokens_count(self):
        return self["tokens"]


@pytest.mark.parametrize("world,expect_seqs", [(1, 14), (2, 30), (4, 57), (8, 115)])
def test_engine5_leg_preempts_at_every_tp_size(pkg, world, expect_seqs):
    from llm_serving_b200.engine import Scheduler, Sequence, SequenceStatus
    w5 = bench.engine5_workload(world, 40.0)
    assert len(w5["ctxs"]) == expect_seqs
    kv = CountingKV(w5["blocks"], 16, -(-bench.ENGINE5_MAX_LEN // 16))
    sched = Scheduler(kv, max_batch_size=32 * world,
                      max_num_batched_tokens=bench.ENGINE5_MAX_LEN * world,
                      max_model_len=bench.ENGINE5_MAX_LEN)
    sid = 0
    for c, o in zip(w5["ctxs"], w5["out_lens"]):  # placed in the cache, as if prefilled
        sid += 1
        s = Sequence(sid, [1] * c, max_tokens=int(o))
        kv.allocate_prefix_blocks(s)
        s.output_token_ids.append(2)
        s.status = SequenceStatus.RUNNING
        sched.running.append(s)
    used = w5["blocks"] - kv.free
    assert 0.90 * w5["blocks"] < used <= 0.95 * w5["blocks"]
    for c, o in zip(w5["wait_lens"], w5["wait_outs"]):
        sid += 1
        sched.add_sequence(Sequence(sid, [1] * int(c), max_tokens=int(o)))
    warmup, steps = 3, 600  # the default run's warm-up and --engine-steps
    prefill_tokens = 0
    for step in range(warmup + steps):
        if step == warmup:
            p0 = sched.preemption_count
        out = sched.schedule()
        if step >= warmup:
            prefill_tokens += sum(s.total_len for s in out.scheduled_prefills)
        for s in out.scheduled_prefills + out.scheduled_decodes:
            s.append_token(3)
        for s in out.scheduled_prefills + out.scheduled_decodes:
            if s.is_finished():
                sched.free_sequence(s)
    assert sched.preemption_count - p0 > 0
    assert prefill_tokens > 0
    assert kv.free >= 0
