"""The allocation-free decode entry point, b200_paged_decode_static, called through the C ABI.

It exists for callers that cannot allocate device memory while they decode (a server that handed
nearly all free HBM to its KV block pool, a plain C caller without a device allocator, a loop that
must not take cudaMalloc's synchronisation); its scratch is a fixed static array in device memory
shared by every call.  This test checks it against the workspace-taking entry point
(b200_paged_decode) on two different batches in a row -- so the second call also proves that what
the first call left in the shared array does not leak into the result -- and that a batch needing
more scratch than the array holds is rejected before anything is launched.  It lives in its own
file, collected last, and must pass both on its own in a fresh process and after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import device_batch

pytestmark = pytest.mark.gpu

BF16_ABS = 2e-2


def _static_decode(native, paged_ops, q, kc, vc, bt, ctx, scale, max_ctx):
    out = torch.full(q.shape, float("nan"), dtype=kc.dtype, device=q.device)
    status = paged_ops.status_word(q.device)
    p = paged_ops.decode_params(q, kc, vc, 0, bt, ctx, scale, out, max_ctx, status=status)
    rc = native.lib().b200_paged_decode_static(ctypes.byref(p),
                                               torch.cuda.current_stream().cuda_stream)
    native.check(rc)
    return out


def test_static_decode_matches_workspace_decode_twice(pkg):
    from llm_serving_b200 import _native, paged_ops
    batches = [
        pkg.workloads.config2(seed=0),  # the bench workload (256 sequences, GQA 32/8, D 128)
        pkg.workloads.custom(seed=5, context_lens=[1, 17, 4000, 640, 33],
                             new_token_counts=[1] * 5, num_query_heads=32, num_kv_heads=8,
                             head_dim=128, block_size=16),
    ]
    for i, b in enumerate(batches):
        q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=20 + i)
        max_ctx = int(b.context_lens.max())
        ref = paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, b.scale, max_ctx)
        got = _static_decode(_native, paged_ops, q, kc, vc, bt, ctx, b.scale, max_ctx)
        torch.cuda.synchronize()
        diff = (got.float() - ref.float()).abs().max().item()
        assert np.isfinite(diff) and diff <= BF16_ABS, (i, diff)
        assert paged_ops.read_status(q.device) == 0


def test_static_decode_rejects_batches_beyond_its_scratch(pkg):
    from llm_serving_b200 import _native, paged_ops
    b = pkg.workloads.custom(seed=1, context_lens=[16] * 4, new_token_counts=[1] * 4,
                             num_query_heads=32, num_kv_heads=8, head_dim=128, block_size=16)
    q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=1)
    out = torch.empty_like(q)
    # a host bound of 2^24 tokens per sequence sizes the plan far past 64 MiB
    p = paged_ops.decode_params(q, kc, vc, 0, bt, ctx, b.scale, out, 1 << 24)
    need = _native.lib().b200_paged_decode_workspace_bytes(ctypes.byref(p))
    assert need > (64 << 20)
    with pytest.raises(ValueError, match="allocation-free decode holds"):
        _native.check(_native.lib().b200_paged_decode_static(
            ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
