"""Drop-in for the reference's pybind module ``llm_allocator_cpp`` (csrc/src/bindings.cpp:79-117).

* ``PageAllocator``      -- the host C++ allocator in libb200paged.so (b200_host_*), with the
                            reference's FIFO / refcount / swap semantics and exception types
                            (csrc/include/page_allocator.hpp:45-374).
* ``SequenceBlockTable`` -- per-sequence block list over a PageAllocator
                            (page_allocator.hpp:376-475); keeps its allocator alive.
* ``paged_attention``    -- the reference kernel's contract (bindings.cpp:10-76) executed by the
                            B200 kernel behind the C symbol ``paged_attention``.  CUDA tensors in
                            -> CUDA tensor out, with no copies; numpy arrays or CPU tensors are
                            copied to the GPU and the result is returned as numpy, as the
                            reference returns it.  There is no CPU execution path.
* ``paged_attention_decode``, ``paged_prefill``, ``reshape_and_cache``, ``build_step_metadata``
  and ``DeviceBlockPool`` -- the torch-tensor entry points of the B200 path (device tensors,
  an optional stream), for callers that bind this module rather than the package.
"""
from __future__ import annotations

import ctypes
from typing import List

from . import _native as N


def _chk(rc: int) -> None:
    N.check(rc, host_message=True)


class PageAllocator:
    def __init__(self, total_blocks: int, tokens_per_block: int, bytes_per_token: int,
                 total_cpu_blocks: int = 32) -> None:
        for v in (total_blocks, tokens_per_block, bytes_per_token, total_cpu_blocks):
            if int(v) < 0:  # size_t arguments in the reference binding
                raise TypeError("incompatible constructor arguments (negative size)")
        h = ctypes.c_void_p()
        _chk(N.lib().b200_host_allocator_create(int(total_blocks), int(tokens_per_block),
                                                int(bytes_per_token), int(total_cpu_blocks),
                                                ctypes.byref(h)))
        self._h = h
        # bound now: at interpreter exit this module's globals may be gone before __del__ runs
        self._destroy = N.lib().b200_host_allocator_destroy

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._destroy(h)
            self._h = None

    def allocate_block(self) -> int:
        out = ctypes.c_int32()
        _chk(N.lib().b200_host_allocate_block(self._h, ctypes.byref(out)))
        return out.value

    def allocate_blocks(self, count: int) -> List[int]:
        if int(count) < 0:
            raise TypeError("count must be non-negative")
        buf = (ctypes.c_int32 * max(1, int(count)))()
        _chk(N.lib().b200_host_allocate_blocks(self._h, int(count), buf))
        return list(buf[:int(count)])

    def share_block(self, block_id: int) -> None:
        _chk(N.lib().b200_host_share_block(self._h, int(block_id)))

    def free_block(self, block_id: int) -> None:
        _chk(N.lib().b200_host_free_block(self._h, int(block_id)))

    def swap_out(self, gpu_block_id: int) -> int:
        out = ctypes.c_int32()
        _chk(N.lib().b200_host_swap_out(self._h, int(gpu_block_id), ctypes.byref(out)))
        return out.value

    def swap_in(self, cpu_block_id: int) -> int:
        out = ctypes.c_int32()
        _chk(N.lib().b200_host_swap_in(self._h, int(cpu_block_id), ctypes.byref(out)))
        return out.value

    def get_cpu_block_id(self, gpu_block_id: int) -> int:
        out = ctypes.c_int32()
        _chk(N.lib().b200_host_get_cpu_block_id(self._h, int(gpu_block_id), ctypes.byref(out)))
        return out.value

    def release_swapped_block(self, cpu_block_id: int) -> None:
        _chk(N.lib().b200_host_release_swapped_block(self._h, int(cpu_block_id)))

    def get_host_ptr(self, cpu_block_id: int) -> int:
        out = ctypes.c_uint64()
        _chk(N.lib().b200_host_get_host_ptr(self._h, int(cpu_block_id), ctypes.byref(out)))
        return out.value

    def get_device_ptr(self, gpu_block_id: int) -> int:
        out = ctypes.c_uint64()
        _chk(N.lib().b200_host_get_device_ptr(self._h, int(gpu_block_id), ctypes.byref(out)))
        return out.value

    def is_zero_copy(self) -> bool:
        # host swap pool in plain host memory, as the reference's CPU memory backend
        return True

    def get_block_size(self) -> int:
        return int(N.lib().b200_host_block_size(self._h))

    def get_bytes_per_token(self) -> int:
        return int(N.lib().b200_host_bytes_per_token(self._h))

    def get_host_pool_bytes(self) -> int:
        return int(N.lib().b200_host_pool_bytes(self._h))

    def get_num_free_blocks(self) -> int:
        return int(N.lib().b200_host_num_free_blocks(self._h))

    def get_num_free_cpu_blocks(self) -> int:
        return int(N.lib().b200_host_num_free_cpu_blocks(self._h))

    def get_total_blocks(self) -> int:
        return int(N.lib().b200_host_total_blocks(self._h))

    def get_utilization_percentage(self) -> float:
        return float(N.lib().b200_host_utilization(self._h))


class SequenceBlockTable:
    """append_token allocates a block whenever the token count is a multiple of the block size
    (page_allocator.hpp:426-434); release frees in table order (:461-469)."""

    def __init__(self, allocator: PageAllocator) -> None:
        self._allocator = allocator  # keep-alive, as py::keep_alive<1, 2> in the reference
        self._block_size = allocator.get_block_size()
        self._blocks: List[int] = []
        self._tokens = 0

    def append_token(self) -> None:
        if self._tokens % self._block_size == 0:
            self._blocks.append(self._allocator.allocate_block())
        self._tokens += 1

    def append_tokens(self, n: int) -> None:
        """n x append_token, with one allocator call for the whole run of new blocks when they
        fit (same blocks and same partial result on OOM as the token-by-token loop)."""
        n = int(n)
        bs = self._block_size
        need = (self._tokens + n + bs - 1) // bs - (self._tokens + bs - 1) // bs
        if need <= self._allocator.get_num_free_blocks():
            if need:
                self._blocks.extend(self._allocator.allocate_blocks(need))
            self._tokens += n
            return
        for _ in range(n):
            self.append_token()

    def append_block(self, block_id: int) -> None:
        if int(block_id) < 0 or int(block_id) >= self._allocator.get_total_blocks():
            raise IndexError(f"Block ID out of range: {int(block_id)}")
        self._blocks.append(int(block_id))

    def replace_block(self, old_block_id: int, new_block_id: int) -> None:
        if int(new_block_id) < 0 or int(new_block_id) >= self._allocator.get_total_blocks():
            raise IndexError(f"Block ID out of range: {int(new_block_id)}")
        try:
            i = self._blocks.index(int(old_block_id))
        except ValueError:
            raise RuntimeError(f"Block ID {int(old_block_id)} not found in block table") from None
        self._blocks[i] = int(new_block_id)

    def release(self) -> None:
        for b in self._blocks:
            self._allocator.free_block(b)
        self._blocks = []
        self._tokens = 0

    def get_physical_blocks(self) -> List[int]:
        return list(self._blocks)

    def get_tokens_count(self) -> int:
        return self._tokens


def paged_attention(query, key_cache, value_cache, layer_idx, gather_slots, attention_mask,
                    scaling):
    """The reference binding's contract (csrc/src/bindings.cpp:10-76) on the B200 kernel.

    Inputs may be numpy arrays or torch tensors, on the host or on the GPU; host inputs are
    force-cast to the binding's types (fp32, int32 slots, uint8 mask) and copied to the device.
    Device caches must already be fp32, the only cache type the reference kernel takes: the
    whole cache is never converted on the device.  Returns a numpy array (1, Nq, Hq, D) fp32,
    as the binding does, so the reference's unchanged caller
    (app/model/attention_backends.py:108-117, ``torch.from_numpy(output)``) works as is.  The
    device-tensor form that returns a CUDA tensor is ``paged_ops.paged_attention_masked``."""
    import numpy as np
    import torch

    from .paged_ops import paged_attention_masked

    if not torch.cuda.is_available():
        raise RuntimeError("paged_attention runs on the GPU; no CUDA device is available")
    types = (np.float32, np.float32, np.float32, np.int32, np.uint8)
    args = [query, key_cache, value_cache, gather_slots, attention_mask]
    dev = next((a.device for a in args if isinstance(a, torch.Tensor) and a.is_cuda),
               torch.device("cuda", torch.cuda.current_device()))
    t = []
    for a, ty in zip(args, types):
        if isinstance(a, torch.Tensor) and a.is_cuda:
            t.append(a.to(dev))
            continue
        if isinstance(a, torch.Tensor):
            a = a.detach().numpy() if a.dtype != torch.bfloat16 else a.detach().float().numpy()
        t.append(torch.from_numpy(np.ascontiguousarray(a, dtype=ty)).to(dev))
    out = paged_attention_masked(t[0], t[1], t[2], int(layer_idx), t[3], t[4], float(scaling))
    return out.cpu().numpy()


# ---- torch-tensor entry points of the B200 path ---------------------------------------------
# Device tensors in, device tensors out, enqueued on `stream` (a torch.cuda.Stream, a raw
# cudaStream_t handle, or None for the current stream).  None of them needs a host upper bound
# read from the device: the context bound is the block tables' width times the block size.

def _on_stream(stream, device):
    import contextlib

    import torch
    if stream is None:
        return contextlib.nullcontext()
    if isinstance(stream, int):
        stream = torch.cuda.ExternalStream(stream, device=device)
    return torch.cuda.stream(stream)


def _context_bound(block_tables, key_cache) -> int:
    return int(block_tables.shape[-1]) * int(key_cache.shape[2])


def paged_attention_decode(query, key_cache, value_cache, layer_idx, block_tables, context_lens,
                           scale, out=None, stream=None):
    """Decode attention through block tables: query (S, Hq, D), caches (L, NB, BS, Hkv, D),
    block_tables (S, max_blocks) int32, context_lens (S,) int32 -> out (S, Hq, D)."""
    from .paged_ops import paged_decode
    with _on_stream(stream, query.device):
        return paged_decode(query, key_cache, value_cache, int(layer_idx), block_tables,
                            context_lens, float(scale), _context_bound(block_tables, key_cache),
                            out=out)


def paged_prefill(query, key_cache, value_cache, layer_idx, block_tables, cu_seqlens,
                  context_lens, scale, out=None, stream=None):
    """Ragged causal attention (prefill chunks and mixed steps): query (Ntok, Hq, D),
    cu_seqlens (S+1,) int64, context_lens (S,) int32 -> out (Ntok, Hq, D)."""
    from .paged_ops import paged_prefill as _prefill
    with _on_stream(stream, query.device):
        return _prefill(query, key_cache, value_cache, int(layer_idx), block_tables, cu_seqlens,
                        context_lens, float(scale), int(query.shape[0]),
                        _context_bound(block_tables, key_cache), out=out)


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping, layer_idx, stream=None):
    """key/value (Ntok, Hkv, D) -> their cache slots (slot_mapping (Ntok,) int64)."""
    from .paged_ops import reshape_and_cache as _write
    with _on_stream(stream, key.device):
        _write(key, value, key_cache, value_cache, slot_mapping, int(layer_idx))


def build_step_metadata(pool, seq_slots, start_positions, new_token_counts, num_tokens,
                        bt_stride=None, stream=None):
    """Per-step metadata on the device from a DeviceBlockPool: cu_seqlens, cu_context_offsets,
    context_lens, position_ids, slot_mapping and padded block_tables, as a dict of tensors."""
    with _on_stream(stream, pool.device):
        return pool.build_step_metadata(seq_slots, start_positions, new_token_counts,
                                        int(num_tokens), bt_stride=bt_stride)


def __getattr__(name):
    # the device block pool, imported on first use (it needs torch; the allocator classes above
    # do not)
    if name == "DeviceBlockPool":
        from .block_manager import DeviceBlockPool
        return DeviceBlockPool
    raise AttributeError(name)
