"""CPU checks of the torch front end's argument handling for the rotary-fused cache write and the
whole-block copy: what has to be refused is refused before any device work (these run without a
GPU; the kernels' own results are checked by the gpu-marked tests)."""
import pytest
import torch


def test_copy_blocks_refuses_pageable_host_caches(pkg):
    from llm_serving_b200 import paged_ops
    k = torch.zeros((1, 4, 16, 2, 64), dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    with pytest.raises(ValueError, match="page-locked"):
        paged_ops.copy_blocks(k, v, k.clone(), v.clone(), [0], [1])


def test_copy_blocks_requires_both_or_neither_value_cache(pkg):
    from llm_serving_b200 import paged_ops
    k = torch.zeros((1, 4, 16, 2, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        paged_ops.copy_blocks(k, k, k, None, [0], [1])


def test_rope_cache_write_has_no_cpu_fallback(pkg):
    from llm_serving_b200 import paged_ops
    kc = torch.zeros((1, 4, 16, 2, 64), dtype=torch.bfloat16)
    qkv = torch.zeros((3, 8 * 64), dtype=torch.bfloat16)
    pos = torch.zeros(3, dtype=torch.int64)
    inv = torch.ones(32)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        paged_ops.rope_reshape_and_cache(qkv, pos, inv, 4, kc, kc.clone(), pos.clone(), 0)


def test_graph_buckets_cover_batches(pkg):
    from llm_serving_b200 import engine
    b = engine._GRAPH_BUCKETS
    assert b == sorted(b) and b[0] == 1 and b[-1] >= 2048
    # every batch size up to 256 pads by fewer than 8 rows
    for n in range(1, 257):
        up = next(x for x in b if x >= n)
        assert up - n < 8
