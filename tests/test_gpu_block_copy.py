"""GPU parity of the whole-block copy (K6, b200_copy_blocks): device -> device (the copy made
before writing a shared block), device -> page-locked host -> device (swap out / swap in, with
the block bookkeeping of the reference allocator's swap_out / swap_in), out-of-range ids flagged
and skipped, pageable host memory refused before any launch.  Every comparison is bit-exact."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L, NB, BS, HKV, D = 3, 40, 16, 4, 64


@pytest.fixture(scope="module")
def ops(pkg):
    from llm_serving_b200 import paged_ops
    return paged_ops


def _caches(dtype, nb=NB, seed=0, device="cuda"):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    k = torch.randn((L, nb, BS, HKV, D), generator=g, device=device).to(dtype)
    v = torch.randn((L, nb, BS, HKV, D), generator=g, device=device).to(dtype)
    return k, v


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_copy_blocks_device_to_device(ops, dtype):
    sk, sv = _caches(dtype, seed=1)
    dk, dv = _caches(dtype, nb=24, seed=2)
    src, dst = [5, 7, 30, 39, 0], [1, 2, 23, 0, 9]
    ek, ev = dk.clone(), dv.clone()
    ek[:, dst] = sk[:, src]
    ev[:, dst] = sv[:, src]
    ops.read_status(torch.device("cuda"))
    ops.copy_blocks(sk, sv, dk, dv, src, dst)
    torch.cuda.synchronize()
    assert torch.equal(dk, ek) and torch.equal(dv, ev)
    assert ops.read_status(torch.device("cuda")) == 0


def test_manager_copy_blocks_within_cache(pkg, ops):
    from llm_serving_b200.kv_cache import PagedKVCacheManager
    m = PagedKVCacheManager(NB, BS, HKV, D, dtype=torch.bfloat16, num_layers=L, device="cuda")
    k, v = _caches(torch.bfloat16, seed=3)
    m.key_cache.copy_(k)
    m.value_cache.copy_(v)
    m.copy_blocks([3, 4], [20, 21])
    torch.cuda.synchronize()
    k[:, [20, 21]] = k[:, [3, 4]]
    v[:, [20, 21]] = v[:, [3, 4]]
    assert torch.equal(m.key_cache, k) and torch.equal(m.value_cache, v)


def test_swap_out_and_in_round_trip(pkg, ops):
    """Reference bookkeeping (swap_out frees the device block and returns a host block id;
    swap_in takes a fresh device block), data moved by HostSwapSpace; the freed device blocks are
    overwritten in between, as their next owner would."""
    from llm_serving_b200.kv_cache import HostSwapSpace, PagedKVCacheManager
    from llm_serving_b200.llm_allocator_cpp import PageAllocator
    m = PagedKVCacheManager(NB, BS, HKV, D, dtype=torch.bfloat16, num_layers=L, device="cuda")
    k, v = _caches(torch.bfloat16, seed=4)
    m.key_cache.copy_(k)
    m.value_cache.copy_(v)
    alloc = PageAllocator(NB, BS, HKV * D * 2 * 2 * L, total_cpu_blocks=8)
    gpu_ids = alloc.allocate_blocks(5)
    saved_k, saved_v = k[:, gpu_ids].clone(), v[:, gpu_ids].clone()
    space = HostSwapSpace(m, 8)
    cpu_ids = [alloc.swap_out(b) for b in gpu_ids]
    space.swap_out(gpu_ids, cpu_ids)
    space.sync()
    assert torch.equal(space.key_cache[:, cpu_ids], saved_k.cpu())
    assert torch.equal(space.value_cache[:, cpu_ids], saved_v.cpu())
    m.key_cache[:, gpu_ids] = 0
    m.value_cache[:, gpu_ids] = 0
    new_ids = [alloc.swap_in(c) for c in cpu_ids]
    space.swap_in(cpu_ids, new_ids)
    space.sync()
    assert torch.equal(m.key_cache[:, new_ids], saved_k)
    assert torch.equal(m.value_cache[:, new_ids], saved_v)
    assert ops.read_status(torch.device("cuda")) == 0


def test_copy_blocks_flags_out_of_range_ids(ops):
    sk, sv = _caches(torch.bfloat16, seed=5)
    dk, dv = _caches(torch.bfloat16, nb=8, seed=6)
    ek, ev = dk.clone(), dv.clone()
    ek[:, 2] = sk[:, 1]
    ev[:, 2] = sv[:, 1]
    ops.read_status(torch.device("cuda"))
    ops.copy_blocks(sk, sv, dk, dv, [1, 3, NB], [2, 8, 0])  # dst 8 and src NB are out of range
    torch.cuda.synchronize()
    from llm_serving_b200 import _native as N
    assert ops.read_status(torch.device("cuda")) & N.DEVICE_BAD_BLOCK
    assert torch.equal(dk, ek) and torch.equal(dv, ev)


def test_copy_blocks_refuses_pageable_host_memory(ops):
    from llm_serving_b200 import _native as N
    sk, sv = _caches(torch.bfloat16, seed=7)
    pageable = torch.zeros((L, NB, BS, HKV, D), dtype=torch.bfloat16)
    assert not pageable.is_pinned()
    with pytest.raises(ValueError):
        ops.copy_blocks(sk, sv, pageable, pageable.clone(), [0], [0])
    # the C entry point itself refuses a pageable host pointer (no kernel is launched)
    geom = ops.cache_geometry(sk)
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    buf = np.zeros(sk.numel(), dtype=np.uint16)
    rc = N.lib().b200_copy_blocks(sk.data_ptr(), None, ctypes.byref(geom),
                                  buf.ctypes.data, None, ctypes.byref(geom), ids.data_ptr(),
                                  ids.data_ptr(), 1, None,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == N.ERR_INVALID_ARGUMENT
    assert not buf.any()


def test_strategy_copy_blocks_key_only(pkg):
    from llm_serving_b200.kv_cache import CudaKVCacheStrategy
    st = CudaKVCacheStrategy(torch.cuda.current_device())
    src, _ = st.allocate_cache(NB, BS, L, HKV, D, torch.float16)
    dst, _ = st.allocate_cache(NB, BS, L, HKV, D, torch.float16)
    src.normal_()
    dst.zero_()
    st.copy_blocks(src, dst, [2, 11, 37])
    exp = torch.zeros_like(dst)
    exp[:, [2, 11, 37]] = src[:, [2, 11, 37]]
    assert torch.equal(dst, exp)
