"""The torch-tensor entry points of the drop-in llm_allocator_cpp module on the GPU: decode and
prefill within the bf16 tolerance of the oracle, the cache write and the step metadata equal to
the package path, each run on an explicit stream (a torch.cuda.Stream and a raw handle)."""
import numpy as np
import pytest
import torch

from gpu_util import device_batch, oracle_ragged

pytestmark = pytest.mark.gpu

BF16_ABS = 2e-2


def test_decode_and_prefill_entry_points(pkg, oracle):
    from llm_serving_b200 import llm_allocator_cpp as la
    s = torch.cuda.Stream()
    b = pkg.workloads.custom(seed=3, context_lens=[40, 1, 600, 129], new_token_counts=[1] * 4,
                             num_query_heads=32, num_kv_heads=8, head_dim=128, block_size=16)
    q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=5)
    torch.cuda.synchronize()
    out = la.paged_attention_decode(q, kc, vc, 0, bt, ctx, b.scale, stream=s)
    out_raw = la.paged_attention_decode(q, kc, vc, 0, bt, ctx, b.scale, stream=s.cuda_stream)
    s.synchronize()
    ref = oracle_ragged(oracle, b, q, kc, vc)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= BF16_ABS
    assert torch.equal(out, out_raw)

    m = pkg.workloads.custom(seed=6, context_lens=[300, 17, 1, 64, 129], new_token_counts=[120, 17, 1, 1, 33],
                             num_query_heads=32, num_kv_heads=8, head_dim=128, block_size=16)
    q, kc, vc, bt, ctx = device_batch(m, torch.bfloat16, seed=12)
    cu = torch.from_numpy(m.cu_seqlens()).cuda()
    torch.cuda.synchronize()
    out = la.paged_prefill(q, kc, vc, 0, bt, cu, ctx, m.scale, stream=s)
    s.synchronize()
    ref = oracle_ragged(oracle, m, q, kc, vc)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= BF16_ABS


def test_cache_write_and_metadata_entry_points(pkg):
    from llm_serving_b200 import llm_allocator_cpp as la
    from llm_serving_b200 import paged_ops
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    kc = torch.randn((2, 24, 16, 4, 64), generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    k = torch.randn((30, 4, 64), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn_like(k)
    slots = torch.randperm(24 * 16, device="cuda")[:30]
    kc2, vc2 = kc.clone(), vc.clone()
    torch.cuda.synchronize()
    la.reshape_and_cache(k, v, kc, vc, slots, 1, stream=s)
    s.synchronize()
    paged_ops.reshape_and_cache(k, v, kc2, vc2, slots, 1)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)

    pool = la.DeviceBlockPool(24, 16, max_seqs=4, max_blocks_per_seq=8)
    pool.append_tokens(0, 20)
    pool.append_tokens(1, 33)
    pool.flush()
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")
    args = (i32([0, 1]), i32([10, 32]), i32([10, 1]), 11)
    torch.cuda.synchronize()
    md = la.build_step_metadata(pool, *args, stream=s)
    s.synchronize()
    ref = pool.build_step_metadata(*args)
    for key in ("cu_seqlens", "context_lens", "position_ids", "slot_mapping", "block_tables"):
        assert torch.equal(md[key], ref[key]), key
    assert pool.status() == 0
