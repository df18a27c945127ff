"""The scheduler policy against 40 request streams recorded from the reference's own Scheduler +
LLMEngine (tests/golden/sched_fuzz.json.gz, made by tests/golden/make_golden.py sched_fuzz):
random pool sizes, block sizes 1-16, batch and token budgets and request mixes, with admission
limits and recompute-preemption in many combinations.  Every step must make the same allocator
calls in the same order and leave the same block tables, free-block count and preemption count,
and the stream must end as the reference's did (some never finish there either)."""
import gzip
import json
import os

import numpy as np
import pytest

from test_engine_host import HostKV

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sched_fuzz.json.gz")


def _streams():
    with gzip.open(FIXTURE, "rt") as f:
        return json.load(f)


@pytest.mark.parametrize("index", range(40))
def test_scheduler_replays_reference_stream(pkg, index):
    from llm_serving_b200 import llm_allocator_cpp as la
    from llm_serving_b200.engine import Scheduler, Sequence
    stream = _streams()[index]
    p = stream["params"]
    kv = HostKV(la, p["total_blocks"], p["block_size"])
    sched = Scheduler(kv, max_batch_size=p["max_batch_size"],
                      max_num_batched_tokens=p["max_num_batched_tokens"],
                      max_model_len=p["max_model_len"])
    rng = np.random.default_rng(p["seed"])
    seqs = []
    for i in range(p["num_requests"]):
        plen = int(rng.integers(1, p["max_prompt"]))
        s = Sequence(i + 1, list(range(plen)), max_tokens=int(rng.integers(2, p["max_out"])))
        sched.add_sequence(s)
        seqs.append(s)
    for n, step in enumerate(stream["steps"]):
        kv.calls.clear()
        out = sched.schedule()
        for s in out.scheduled_prefills + out.scheduled_decodes:
            s.append_token(100 + s.total_len)
        for s in out.scheduled_prefills + out.scheduled_decodes:
            if s.is_finished():
                sched.free_sequence(s)
        assert [tuple(c) for c in kv.calls] == [tuple(c) for c in step["calls"]], n
        live = {s.seq_id: s.block_table.get_physical_blocks() for s in seqs
                if s.block_table is not None}
        assert live == {int(k): v for k, v in step["tables"].items()}, n
        assert kv.allocator.get_num_free_blocks() == step["free"], n
        assert sched.preemption_count == step["preemptions"], n
    # some streams never finish in the reference either: a prompt longer than the token
    # budget is never admitted
    assert sched.has_unfinished_sequences() == (not stream["finished"])
