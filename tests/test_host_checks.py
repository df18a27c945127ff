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


def _decode_args(D=64, dtype=torch.bfloat16, q_dtype=None, q_dim=None, rows=3):
    kc = torch.zeros((1, 4, 16, 2, D), dtype=dtype)
    q = torch.zeros((rows, 4, q_dim or D), dtype=q_dtype or dtype)
    bt = torch.zeros((3, 4), dtype=torch.int32)
    ctx = torch.ones(3, dtype=torch.int32)
    return q, kc, kc.clone(), bt, ctx


def test_decode_refuses_a_query_the_kernels_would_misread(pkg):
    """The C ABI reads the query as the cache's dtype and head dim: a mismatch must be refused
    before any pointer reaches the library."""
    from llm_serving_b200 import paged_ops
    q, kc, vc, bt, ctx = _decode_args(q_dim=32)
    with pytest.raises(ValueError, match="head dim"):
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, 0.125, 1)
    q, kc, vc, bt, ctx = _decode_args(q_dtype=torch.float32)
    with pytest.raises(ValueError, match="dtype"):
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, 0.125, 1)
    q, kc, vc, bt, ctx = _decode_args(rows=2)
    with pytest.raises(ValueError, match="rows"):
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, 0.125, 1)
    q, kc, vc, bt, ctx = _decode_args()
    with pytest.raises(ValueError, match="out"):
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, 0.125, 1, out=torch.zeros((3, 4, 32),
                                                                                dtype=kc.dtype))
    with pytest.raises(ValueError, match="value_cache"):
        paged_ops.paged_decode(q, kc, vc[:, :2].contiguous(), 0, bt, ctx, 0.125, 1)
    with pytest.raises(ValueError, match="int32"):
        paged_ops.paged_decode(q, kc, vc, 0, bt.long(), ctx, 0.125, 1)
    with pytest.raises(ValueError, match="fewer rows"):
        paged_ops.paged_decode(q, kc, vc, 0, bt[:2], ctx, 0.125, 1)
    # well-formed host tensors: refused for being on the host, never computed there
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, 0.125, 1)


def test_prefill_checks_its_ragged_metadata(pkg):
    from llm_serving_b200 import paged_ops
    q, kc, vc, bt, ctx = _decode_args()
    cu = torch.tensor([0, 1, 2, 3], dtype=torch.int64)
    with pytest.raises(ValueError, match="cu_seqlens"):
        paged_ops.paged_prefill(q, kc, vc, 0, bt, cu.int(), ctx, 0.125, 1, 1)
    with pytest.raises(ValueError, match="cu_seqlens"):
        paged_ops.paged_prefill(q, kc, vc, 0, bt, cu[:3], ctx, 0.125, 1, 1)
    with pytest.raises(ValueError, match="head dim"):
        paged_ops.paged_prefill(q[..., :32], kc, vc, 0, bt, cu, ctx, 0.125, 1, 1)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        paged_ops.paged_prefill(q, kc, vc, 0, bt, cu, ctx, 0.125, 1, 1)


def test_workspace_is_per_stream(pkg):
    from llm_serving_b200 import paged_ops
    ws = paged_ops.Workspace()
    cpu = torch.device("cpu")
    a, b = ws.get(cpu, 1000, 1), ws.get(cpu, 1000, 2)
    assert a.data_ptr() != b.data_ptr()
    assert ws.get(cpu, 500, 1).data_ptr() == a.data_ptr()      # reused while large enough
    assert ws.get(cpu, 4000, 1).numel() >= 4000                # grown when not


def test_dropin_module_has_the_tensor_entry_points(pkg):
    """The drop-in llm_allocator_cpp module carries the torch-tensor entry points of the B200
    path next to the reference's classes, and they refuse host tensors (no CPU fallback)."""
    from llm_serving_b200 import block_manager
    from llm_serving_b200 import llm_allocator_cpp as la
    for name in ("paged_attention_decode", "paged_prefill", "reshape_and_cache",
                 "build_step_metadata"):
        assert callable(getattr(la, name))
    assert la.DeviceBlockPool is block_manager.DeviceBlockPool
    q, kc, vc, bt, ctx = _decode_args()
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        la.paged_attention_decode(q, kc, vc, 0, bt, ctx, 0.125)
    with pytest.raises(ValueError, match="head dim"):
        la.paged_attention_decode(q[..., :32], kc, vc, 0, bt, ctx, 0.125)
    cu = torch.tensor([0, 1, 2, 3], dtype=torch.int64)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        la.paged_prefill(q, kc, vc, 0, bt, cu, ctx, 0.125)
    k = torch.zeros((3, 2, 64), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        la.reshape_and_cache(k, k.clone(), kc, vc, cu[:3], 0)


def test_backend_selection_names(pkg, monkeypatch):
    """The reference's backend names (attention_backends.py:126-144): 'native' and its 'hip'
    alias, 'auto'; 'torch' (the reference's own SDPA backend) and unknown names are refused."""
    from llm_serving_b200 import attention_backends as ab
    with pytest.raises(ValueError, match="reference"):
        ab.select_backend("torch")
    with pytest.raises(ValueError, match="Unsupported"):
        ab.select_backend("bogus")
    backend = ab.NativePagedBackend()
    assert backend.supports(None, 5) and not backend.supports(None, 0)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_backend_selection_without_a_device_fails_loudly(pkg, monkeypatch):
    """Without a CUDA device every name that resolves to the native backend raises; 'auto' does
    not fall back to a host path."""
    from llm_serving_b200 import attention_backends as ab
    for name in ("native", "hip", "auto"):
        with pytest.raises(RuntimeError, match="CUDA device"):
            ab.select_backend(name)
    monkeypatch.setenv(ab.BACKEND_ENV_VAR, "hip")
    with pytest.raises(RuntimeError):
        ab.select_backend()
    with pytest.raises(RuntimeError, match="no CPU path"):
        ab.NativePagedBackend().attend(torch.zeros(1, 2, 1, 8), None, 0, None, 1.0, 0.0)
