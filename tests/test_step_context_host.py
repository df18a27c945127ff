"""The host side of the device PagedStepContext -- offsets, lengths, maxima, the decode flag,
positions and the dense block-diagonal causal mask built from the metadata -- against the step
contexts recorded from the reference's own PagedStepContext (tests/golden/golden.npz).  A host
stand-in for the device KV manager serves the oracle's metadata, so this runs without a GPU; the
device metadata itself is checked bit-exact by the gpu-marked tests."""
import numpy as np
import torch

from golden_util import ragged


class OracleStore:
    """Serves step metadata computed by the oracle as host tensors, keyed by sequence index."""

    torch_device = torch.device("cpu")

    def __init__(self, oracle, tables, tokens, block_size):
        self.oracle, self.tables, self.tokens, self.bs = oracle, tables, tokens, block_size

    def step_metadata(self, seqs, starts, counts, with_gather_slots=False):
        md = self.oracle.step_metadata([self.tables[s] for s in seqs],
                                       [self.tokens[s] for s in seqs], starts, counts, self.bs)
        bt, _ = self.oracle.build_block_tables([self.tables[s] for s in seqs],
                                               [self.tokens[s] for s in seqs])
        out = {"slot_mapping": torch.from_numpy(md["scatter_slots"]),
               "position_ids": torch.from_numpy(md["position_ids"][0]),
               "block_tables": torch.from_numpy(bt),
               "context_lens": torch.tensor([s + c for s, c in zip(starts, counts)],
                                            dtype=torch.int32),
               "cu_seqlens": torch.from_numpy(md["cu_seqlens"])}
        if with_gather_slots:
            out["gather_slots"] = torch.from_numpy(md["gather_slots"])
        return out


def test_step_context_matches_reference_contexts(golden, oracle, pkg):
    from llm_serving_b200.step_context import PagedStepContext
    cpu = torch.device("cpu")
    for name in golden["meta_cases"]:
        p = f"meta_{name}_"
        tables = ragged(golden, p)
        tokens = golden[p + "tokens"].tolist()
        starts, counts = golden[p + "starts"].tolist(), golden[p + "counts"].tolist()
        store = OracleStore(oracle, tables, tokens, 4)
        ctx = PagedStepContext(store, list(range(len(tables))), starts, counts)
        assert ctx.cu_seqlens.tolist() == golden[p + "cu_seqlens"].tolist(), name
        assert ctx.cu_context_offsets.tolist() == golden[p + "cu_context_offsets"].tolist(), name
        assert ctx.context_lens == golden[p + "context_lens"].tolist(), name
        assert ctx.num_query_tokens == int(sum(counts))
        assert ctx.max_query_len == max(counts) and ctx.max_context_len == max(ctx.context_lens)
        assert ctx.is_decode == all(c == 1 for c in counts)
        assert np.array_equal(ctx.position_ids(cpu).numpy(), golden[p + "position_ids"]), name
        assert np.array_equal(ctx.attention_mask(cpu).numpy(), golden[p + "mask"]), name
        assert np.array_equal(ctx.gather_slots.numpy(), golden[p + "gather_slots"]), name
        assert np.array_equal(ctx.scatter_slots.numpy(), golden[p + "scatter_slots"]), name


def test_empty_step_context(oracle, pkg):
    from llm_serving_b200.step_context import PagedStepContext
    ctx = PagedStepContext(OracleStore(oracle, [], [], 4), [], [], [])
    assert ctx.num_query_tokens == 0 and ctx.num_context_tokens == 0 and not ctx.is_decode
    assert ctx.cu_seqlens.tolist() == [0] and ctx.gather_slots.numel() == 0
    assert ctx.attention_mask(torch.device("cpu")).shape == (1, 1, 0, 0)
