"""Seeded inputs of BASELINE config 1 (shared by make_golden.py and the tests).

8 decode sequences, context U[1,512], 12/12 heads, head_dim 64, block size 16, fp32 N(0,1), block
tables as consecutive chunks of a random permutation of a 512-block pool, scale 1/8.  The gather
slots and the dense decode mask are the ones PagedStepContext builds for such a step
(app/model/paged_attention.py:64-69, :92-118): each sequence's context slots in order, and a mask
that lets query s see exactly its own sequence's context.
"""
import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)


def config1_inputs(seed: int = 0, value_seed: int = 1):
    import __graft_entry__
    wl = __graft_entry__.load_package().workloads
    b = wl.config1(seed)
    rng = np.random.default_rng(value_seed)
    shape = (1, b.total_blocks, b.block_size, b.num_kv_heads, b.head_dim)
    kc = rng.standard_normal(shape, dtype=np.float32)
    vc = rng.standard_normal(shape, dtype=np.float32)
    q = rng.standard_normal((1, b.num_query_heads, b.num_seqs, b.head_dim), dtype=np.float32)
    ctx = b.context_lens
    gs = np.concatenate([np.asarray(t, np.int64)[np.arange(c) // 16] * 16 + np.arange(c) % 16
                         for t, c in zip(b.tables, ctx)]).astype(np.int32)
    owner = np.repeat(np.arange(b.num_seqs), ctx)
    mask = (owner[None, :] == np.arange(b.num_seqs)[:, None]).astype(np.uint8)[None, None]
    return b, q, kc, vc, gs, mask
