"""Device-resident block pool (K5) and the per-step metadata builder (K4).

``DeviceBlockPool`` replaces the GPU-block bookkeeping of the reference's PageAllocator and
SequenceBlockTable (csrc/include/page_allocator.hpp:78-177, :426-469) on the engine's batched
path: the FIFO free list and one block-table row per sequence slot live in device memory and are
updated by one kernel per ``flush()``.  The host object keeps only counts (free blocks, tokens and
blocks per slot), which is all the scheduler consults (app/scheduler/scheduler.py:100-104,
:128-130).  Block ids reach the host only through the explicit ``table()`` / ``free_queue()``
reads used by tests and debugging.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import torch

from . import _native as N
from .paged_ops import _stream


class _DeviceArray:
    """Minimal __cuda_array_interface__ holder so torch can view library-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


class DeviceBlockPool:
    def __init__(self, total_blocks: int, block_size: int, max_seqs: int,
                 max_blocks_per_seq: int, device: Optional[torch.device] = None) -> None:
        self.device = torch.device(device or "cuda")
        if self.device.type != "cuda":
            raise RuntimeError("DeviceBlockPool lives in GPU memory (no CPU fallback)")
        self.total_blocks = int(total_blocks)
        self.block_size = int(block_size)
        self.max_seqs = int(max_seqs)
        self.max_blocks_per_seq = int(max_blocks_per_seq)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            N.check(N.lib().b200_pool_create(self.total_blocks, self.block_size, self.max_seqs,
                                             self.max_blocks_per_seq, ctypes.byref(h)))
        self._h = h
        L = N.lib()
        self._tables = torch.as_tensor(
            _DeviceArray(L.b200_pool_tables(h), (self.max_seqs, self.max_blocks_per_seq), "<i4"),
            device=self.device)
        self._status = torch.as_tensor(_DeviceArray(L.b200_pool_status(h), (1,), "<i4"),
                                       device=self.device)

    def close(self) -> None:
        """Free the pool's device memory; the ``tables`` view and the status view die with it."""
        if getattr(self, "_h", None):
            self._tables = self._status = None
            N.lib().b200_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- queued ops (host side, no device work) -------------------------------------------
    def append_tokens(self, slot: int, n: int) -> None:
        """Append n tokens to a sequence slot; raises RuntimeError (after appending the tokens
        that fit) when the pool runs dry, like the reference's per-token loop."""
        N.check(N.lib().b200_pool_append_tokens(self._h, int(slot), int(n)))

    def release(self, slot: int) -> None:
        N.check(N.lib().b200_pool_release(self._h, int(slot)))

    def share(self, dst_slot: int, src_slot: int, num_blocks: int) -> None:
        """The empty ``dst_slot`` takes the first ``num_blocks`` blocks of ``src_slot`` (each
        gains an owner; it returns to the free list with its last owner's release)."""
        N.check(N.lib().b200_pool_share(self._h, int(dst_slot), int(src_slot), int(num_blocks)))

    def copy_on_write(self, slot: int, block_index: int) -> None:
        """Queue: table entry ``block_index`` of ``slot`` gets a fresh block (the old one loses an
        owner).  After the flush, ``cow_pairs()`` gives the (old, new) ids to copy."""
        N.check(N.lib().b200_pool_copy_on_write(self._h, int(slot), int(block_index)))

    def cow_pairs(self):
        """(old, new) block ids of the last flush's copy-on-write replacements, as int32 device
        views (empty when there were none)."""
        old, new = ctypes.c_void_p(), ctypes.c_void_p()
        n = int(N.lib().b200_pool_cow_pairs(self._h, ctypes.byref(old), ctypes.byref(new)))
        if n == 0:
            e = torch.empty(0, dtype=torch.int32, device=self.device)
            return e, e
        mk = lambda ptr: torch.as_tensor(_DeviceArray(ptr.value, (n,), "<i4"), device=self.device)
        return mk(old), mk(new)

    def flush(self, stream: Optional[int] = None) -> None:
        with torch.cuda.device(self.device):
            N.check(N.lib().b200_pool_flush(self._h, _stream(self.device) if stream is None
                                            else stream))

    # ---- host counts ----------------------------------------------------------------------
    def get_num_free_blocks(self) -> int:
        return int(N.lib().b200_pool_num_free_blocks(self._h))

    def get_total_blocks(self) -> int:
        return self.total_blocks

    def get_block_size(self) -> int:
        return self.block_size

    def tokens(self, slot: int) -> int:
        return int(N.lib().b200_pool_tokens(self._h, int(slot)))

    def num_blocks(self, slot: int) -> int:
        return int(N.lib().b200_pool_num_blocks(self._h, int(slot)))

    # ---- device views ---------------------------------------------------------------------
    @property
    def tables(self) -> torch.Tensor:
        """(max_seqs, max_blocks_per_seq) int32 device view; -1 = no block."""
        return self._tables

    def table(self, slot: int) -> List[int]:
        """Physical blocks of a slot (device read; synchronises)."""
        n = self.num_blocks(slot)
        return self._tables[slot, :n].tolist()

    def free_queue(self) -> List[int]:
        out = (ctypes.c_int32 * max(1, self.total_blocks))()
        with torch.cuda.device(self.device):
            n = N.lib().b200_pool_snapshot_free(self._h, out, self.total_blocks,
                                                _stream(self.device))
        if n < 0:
            raise RuntimeError("pool snapshot failed")
        return list(out[:n])

    def status(self, reset: bool = True) -> int:
        v = int(self._status.item())
        if reset:
            self._status.zero_()
        return v

    # ---- K4 -------------------------------------------------------------------------------
    def build_step_metadata(self, seq_slots: torch.Tensor, start_positions: torch.Tensor,
                            new_token_counts: torch.Tensor, num_tokens: int,
                            bt_stride: Optional[int] = None,
                            with_gather_slots: bool = False,
                            num_context_tokens: Optional[int] = None) -> Dict[str, torch.Tensor]:
        """Device version of PagedStepContext + build_block_tables for the sequences in
        ``seq_slots`` (int32 device tensors of S entries).  ``num_tokens`` (and, for gather
        slots, ``num_context_tokens``) are host-known sizes used to allocate the outputs."""
        S = int(seq_slots.numel())
        dev = self.device
        bt_stride = int(bt_stride if bt_stride is not None else self.max_blocks_per_seq)
        out = {
            "cu_seqlens": torch.empty(S + 1, dtype=torch.int64, device=dev),
            "cu_context_offsets": torch.empty(S + 1, dtype=torch.int64, device=dev),
            "context_lens": torch.empty(S, dtype=torch.int32, device=dev),
            "position_ids": torch.empty(int(num_tokens), dtype=torch.int64, device=dev),
            "slot_mapping": torch.empty(int(num_tokens), dtype=torch.int64, device=dev),
            "block_tables": torch.empty((S, bt_stride), dtype=torch.int32, device=dev),
        }
        gather = None
        if with_gather_slots:
            gather = torch.empty(int(num_context_tokens), dtype=torch.int64, device=dev)
            out["gather_slots"] = gather
        for t in (seq_slots, start_positions, new_token_counts):
            if (t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous() or
                    t.numel() != S):
                raise ValueError("seq_slots, start_positions, new_token_counts: contiguous int32 "
                                 "CUDA tensors of one entry per sequence")
        with torch.cuda.device(dev):
            N.check(N.lib().b200_build_step_metadata(
                self._h, seq_slots.data_ptr(), start_positions.data_ptr(),
                new_token_counts.data_ptr(), S, int(num_tokens), out["cu_seqlens"].data_ptr(),
                out["cu_context_offsets"].data_ptr(), out["context_lens"].data_ptr(),
                out["position_ids"].data_ptr(), out["slot_mapping"].data_ptr(),
                out["block_tables"].data_ptr(), bt_stride,
                None if gather is None else gather.data_ptr(),
                0 if gather is None else gather.numel(), _stream(dev)))
        return out
