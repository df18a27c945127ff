"""The decode workspace the engine shares between its captured decode graphs must cover every
batch bucket, not only the largest: the split plan gives small batches shorter splits (so that
the SMs keep work), so a smaller bucket can need more scratch per sequence than the largest one.
A closed-loop config-4 run of 2000 requests once reached a mid-sized bucket whose scratch exceeded
the largest bucket's and the decode refused to run ("decode workspace too small").  Host-only:
the workspace size is computed from shapes alone."""
import ctypes

import torch


def test_graph_workspace_covers_every_bucket(pkg):
    from llm_serving_b200 import _native as N
    from llm_serving_b200 import paged_ops
    from llm_serving_b200.engine import _GRAPH_BUCKETS, graph_decode_workspace_bytes
    # config-4 decode geometry (bf16, 32 query / 8 KV heads, head dim 64, block size 16) at the
    # engine's context bound 8192 with up to 256 decoding sequences
    kc = torch.empty((16, 64, 16, 8, 64), dtype=torch.bfloat16)
    width, bound, max_rows = 512, 8192, 256
    per_bucket = {}
    for rows in _GRAPH_BUCKETS:
        if rows > max_rows:
            break
        q = torch.empty((rows, 32, 64), dtype=torch.bfloat16)
        bt = torch.empty((rows, width), dtype=torch.int32)
        ctx = torch.empty(rows, dtype=torch.int32)
        p = paged_ops.decode_params(q, kc, kc, 0, bt, ctx, 0.125, q, bound)
        per_bucket[rows] = int(N.lib().b200_paged_decode_workspace_bytes(ctypes.byref(p)))
    need = graph_decode_workspace_bytes(32, kc, kc, width, bound, max_rows, 0.125)
    assert need == max(per_bucket.values())
    # the smallest buckets get shorter splits: more scratch per sequence than the largest bucket
    assert per_bucket[1] / 1 > per_bucket[max_rows] / max_rows
