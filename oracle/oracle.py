"""CPU oracle for the paged-attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` import this
module, and only as the checker.  The product (the CUDA library and its host mirror) never imports
it.

Contents, each citing the reference (Pakanor/Low-Latency-Distributed-LLM-Serving-Infrastructure-
Custom-K8s-Control-Plane) code it restates:

* ``paged_attention``      -- csrc/src/bindings.cpp:10-76 around csrc/src/paged_kernels.cpp:7-105
                              (C restatement in paged_oracle.c).
* ``paged_ragged``         -- the same arithmetic per sequence with the causal window of
                              app/model/paged_attention.py:92-118, read through block tables.
* ``slot_mapping``         -- app/memory/manager.py:104-128 and :301-333.
* ``step_metadata``        -- PagedStepContext, app/model/paged_attention.py:40-135.
* ``build_block_tables``   -- app/memory/manager.py:236-271.
* ``Fifo`` / ``SeqTable``  -- PageAllocator / SequenceBlockTable GPU-block bookkeeping,
                              csrc/include/page_allocator.hpp:78-177 and :410-469.
* ``RefKernel``            -- the reference's own kernel compiled from its sources into
                              oracle/_ref (see oracle/Makefile), used to pin the restatement and
                              as the timed CPU baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_paged.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_KERNEL_PATH = os.path.join(REF_DIR, "libref_paged_kernels.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class PagedDims(ctypes.Structure):
    """Field order of PagedAttentionDims, csrc/include/paged_kernels.h:11-20."""

    _fields_ = [
        ("num_query_heads", ctypes.c_int32),
        ("num_query_tokens", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("total_blocks", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("num_context_tokens", ctypes.c_int32),
    ]


def build(force: bool = False) -> None:
    """Compile liboracle_paged.so (and oracle/_ref when the reference tree is present)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle_paged.so"], check=True)


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_paged_attention.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int32, PagedDims, _i32p,
                                             _u8p, ctypes.c_float, _f32p, _f32p]
        L.oracle_paged_attention.restype = None
        L.oracle_paged_ragged.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_int32] * 7 + [
            _i32p, ctypes.c_int32, _i32p, _i32p, ctypes.c_float, _f32p]
        L.oracle_paged_ragged.restype = None
        L.oracle_reshape_and_cache.argtypes = [ctypes.c_void_p] * 4 + [
            ctypes.c_int32, ctypes.c_int64, ctypes.c_int64, _i64p, ctypes.c_int64]
        L.oracle_reshape_and_cache.restype = ctypes.c_int64
        L.oracle_fifo_create.argtypes = [ctypes.c_int32]
        L.oracle_fifo_create.restype = ctypes.c_void_p
        L.oracle_fifo_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_fifo_allocate.argtypes = [ctypes.c_void_p, ctypes.c_int32, _i32p]
        L.oracle_fifo_allocate.restype = ctypes.c_int32
        for name in ("oracle_fifo_free", "oracle_fifo_share"):
            getattr(L, name).argtypes = [ctypes.c_void_p, ctypes.c_int32]
            getattr(L, name).restype = ctypes.c_int32
        L.oracle_fifo_num_free.argtypes = [ctypes.c_void_p]
        L.oracle_fifo_num_free.restype = ctypes.c_int32
        L.oracle_fifo_snapshot.argtypes = [ctypes.c_void_p, _i32p]
        L.oracle_fifo_snapshot.restype = ctypes.c_int32
        _LIB = L
    return _LIB


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


# --------------------------------------------------------------------------------------------
# bf16 <-> fp32 (round to nearest even), for building bf16 inputs and upcasting them
# --------------------------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------------------------
# Attention
# --------------------------------------------------------------------------------------------

def paged_attention(query: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray,
                    layer_idx: int, gather_slots: np.ndarray, attention_mask: np.ndarray,
                    scaling: float) -> np.ndarray:
    """Mirror of the reference binding (bindings.cpp:10-76): query (1,Hq,Nq,D), caches
    (L,NB,BS,Hkv,D), gather_slots (Nctx,), mask (1,1,Nq,Nctx) -> output (1,Nq,Hq,D) fp32."""
    q = np.ascontiguousarray(query, dtype=np.float32)
    kc = np.ascontiguousarray(key_cache, dtype=np.float32)
    vc = np.ascontiguousarray(value_cache, dtype=np.float32)
    gs = np.ascontiguousarray(gather_slots, dtype=np.int32)
    m = np.ascontiguousarray(attention_mask, dtype=np.uint8)
    if q.ndim != 4 or kc.ndim != 5 or gs.ndim != 1 or m.ndim != 4:
        raise RuntimeError("query 4-D, key_cache 5-D, gather_slots 1-D, mask 4-D required")
    dims = PagedDims(q.shape[1], q.shape[2], q.shape[3], kc.shape[0], kc.shape[1], kc.shape[2],
                     kc.shape[3], gs.shape[0])
    if dims.num_query_heads % dims.num_kv_heads != 0:
        raise RuntimeError("num_query_heads must be a multiple of num_kv_heads for GQA")
    if layer_idx < 0 or layer_idx >= dims.num_layers:
        raise RuntimeError("layer_idx out of range")
    out = np.empty((1, dims.num_query_tokens, dims.num_query_heads, dims.head_dim), np.float32)
    scratch = np.empty((max(1, dims.num_query_tokens * dims.num_query_heads * gs.shape[0]),),
                       np.float32)
    lib().oracle_paged_attention(_p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), layer_idx, dims,
                                 _p(gs, _i32p), _p(m, _u8p), float(scaling), _p(out, _f32p),
                                 _p(scratch, _f32p))
    return out


def paged_ragged(q: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray, layer_idx: int,
                 block_tables: np.ndarray, start_positions: Sequence[int],
                 new_token_counts: Sequence[int], scaling: float) -> np.ndarray:
    """Causal attention through block tables.  q (Ntok,Hq,D) fp32; caches (L,NB,BS,Hkv,D) fp32;
    block_tables (S, max_blocks) int32.  Returns (Ntok,Hq,D) fp32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(key_cache, dtype=np.float32)
    vc = np.ascontiguousarray(value_cache, dtype=np.float32)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    st = np.ascontiguousarray(start_positions, dtype=np.int32)
    ct = np.ascontiguousarray(new_token_counts, dtype=np.int32)
    L, NB, BS, Hkv, D = kc.shape
    Hq = q.shape[1]
    out = np.zeros_like(q)
    if bt.ndim != 2:
        bt = bt.reshape(len(st), -1)
    lib().oracle_paged_ragged(_p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), layer_idx, NB, BS, Hkv,
                              Hq, D, len(st), _p(bt, _i32p), bt.shape[1], _p(st, _i32p),
                              _p(ct, _i32p), float(scaling), _p(out, _f32p))
    return out


def reshape_and_cache(key: np.ndarray, value: np.ndarray, key_cache: np.ndarray,
                      value_cache: np.ndarray, slot_mapping: np.ndarray, layer_idx: int) -> int:
    """In-place scatter of (Ntok,Hkv,D) rows into the caches (manager.py:150-168).  Returns the
    number of slots skipped: negative padding slots and slots past the pool."""
    assert key_cache.flags.c_contiguous and value_cache.flags.c_contiguous
    k = np.ascontiguousarray(key, dtype=key_cache.dtype)
    v = np.ascontiguousarray(value, dtype=value_cache.dtype)
    sm = np.ascontiguousarray(slot_mapping, dtype=np.int64)
    L, NB, BS, Hkv, D = key_cache.shape
    row_bytes = Hkv * D * key_cache.itemsize
    return int(lib().oracle_reshape_and_cache(k.ctypes.data, v.ctypes.data, key_cache.ctypes.data,
                                              value_cache.ctypes.data, layer_idx, NB * BS,
                                              row_bytes, _p(sm, _i64p), sm.shape[0]))


# --------------------------------------------------------------------------------------------
# Step metadata (PagedStepContext) and block tables
# --------------------------------------------------------------------------------------------

def cumulative_offsets(counts: Sequence[int]) -> np.ndarray:
    """_cumulative_offsets, app/model/paged_attention.py:121-125 (int64, leading 0)."""
    out = np.zeros(len(counts) + 1, dtype=np.int64)
    if len(counts):
        out[1:] = np.cumsum(np.asarray(counts, dtype=np.int64))
    return out


def sequence_slots(physical_blocks: Sequence[int], block_size: int, tokens_count: int,
                   start_token: int, token_count: int) -> np.ndarray:
    """_sequence_slots, app/memory/manager.py:301-333 (including its ValueError checks)."""
    if start_token < 0 or token_count < 0:
        raise ValueError("start_token and token_count must be non-negative")
    if start_token + token_count > tokens_count:
        raise ValueError("tokens exceed allocated tokens")
    if token_count == 0:
        return np.zeros((0,), dtype=np.int64)
    t = np.arange(start_token, start_token + token_count, dtype=np.int64)
    blocks = np.asarray(physical_blocks, dtype=np.int64)
    return blocks[t // block_size] * block_size + t % block_size


def slot_mapping(tables: Sequence[Sequence[int]], tokens_counts: Sequence[int],
                 start_tokens: Sequence[int], token_counts: Sequence[int],
                 block_size: int) -> np.ndarray:
    """build_slot_mapping, app/memory/manager.py:104-128: per-sequence slots, concatenated."""
    if not (len(tables) == len(start_tokens) == len(token_counts)):
        raise ValueError("sequences, start_tokens and token_counts must have the same length")
    parts = [sequence_slots(tb, block_size, n, s, c)
             for tb, n, s, c in zip(tables, tokens_counts, start_tokens, token_counts)]
    parts = [p for p in parts if p.size]
    return np.concatenate(parts) if parts else np.zeros((0,), dtype=np.int64)


def step_metadata(tables: Sequence[Sequence[int]], tokens_counts: Sequence[int],
                  start_positions: Sequence[int], new_token_counts: Sequence[int],
                  block_size: int, with_mask: bool = False) -> dict:
    """PagedStepContext, app/model/paged_attention.py:40-118."""
    if not (len(tables) == len(start_positions) == len(new_token_counts)):
        raise ValueError("sequences, start_positions and new_token_counts must match")
    context_lens = [s + c for s, c in zip(start_positions, new_token_counts)]       # :57-59
    md = {
        "context_lens": np.asarray(context_lens, dtype=np.int64),
        "cu_seqlens": cumulative_offsets(new_token_counts),                        # :61
        "cu_context_offsets": cumulative_offsets(context_lens),                    # :62
        "scatter_slots": slot_mapping(tables, tokens_counts, start_positions,
                                      new_token_counts, block_size),               # :64-66
        "gather_slots": slot_mapping(tables, tokens_counts, [0] * len(tables),
                                     context_lens, block_size),                    # :67-69
    }
    pos = [np.arange(s, s + c, dtype=np.int64) for s, c in zip(start_positions, new_token_counts)]
    md["position_ids"] = (np.concatenate(pos) if pos else np.zeros((0,), np.int64))[None, :]  # :81-90
    if with_mask:                                                                  # :92-118
        qi = np.repeat(np.arange(len(tables)), new_token_counts)
        ci = np.repeat(np.arange(len(tables)), context_lens)
        qpos = md["position_ids"][0]
        cpos = np.arange(int(md["cu_context_offsets"][-1])) - md["cu_context_offsets"][ci]
        mask = (ci[None, :] == qi[:, None]) & (cpos[None, :] <= qpos[:, None])
        md["attention_mask"] = mask[None, None]
    return md


def build_block_tables(tables: Sequence[Sequence[int]], tokens_counts: Sequence[int]):
    """build_block_tables, app/memory/manager.py:236-271: (S, max_blocks) int32 padded with -1,
    and context_lens int32."""
    S = len(tables)
    if S == 0:
        return np.zeros((0, 0), np.int32), np.zeros((0,), np.int32)
    mb = max(len(t) for t in tables)
    bt = np.full((S, mb), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        if len(t):
            bt[i, :len(t)] = t
    return bt, np.asarray(tokens_counts, dtype=np.int32)


# --------------------------------------------------------------------------------------------
# FIFO allocator
# --------------------------------------------------------------------------------------------

class Fifo:
    """GPU-block bookkeeping of PageAllocator (page_allocator.hpp:78-177) over the C ring."""

    def __init__(self, total_blocks: int) -> None:
        self.total = total_blocks
        self._h = lib().oracle_fifo_create(total_blocks)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().oracle_fifo_destroy(self._h)
            self._h = None

    def allocate_blocks(self, count: int) -> List[int]:
        out = np.zeros(max(count, 1), dtype=np.int32)
        rc = lib().oracle_fifo_allocate(self._h, count, _p(out, _i32p))
        if rc != 0:
            raise RuntimeError("Out of Memory: Not enough free blocks available in KV-Cache pool!")
        return out[:count].tolist()

    def allocate_block(self) -> int:
        return self.allocate_blocks(1)[0]

    def free_block(self, block_id: int) -> None:
        rc = lib().oracle_fifo_free(self._h, block_id)
        if rc == -3:
            raise IndexError(f"Block ID out of range: {block_id}")
        if rc == -2:
            raise RuntimeError(f"Double-free or free on unallocated block detected: ID {block_id}")

    def share_block(self, block_id: int) -> None:
        rc = lib().oracle_fifo_share(self._h, block_id)
        if rc == -3:
            raise IndexError(f"Block ID out of range: {block_id}")
        if rc == -2:
            raise RuntimeError(f"Cannot share unallocated block {block_id}")

    def get_num_free_blocks(self) -> int:
        return int(lib().oracle_fifo_num_free(self._h))

    def free_queue(self) -> List[int]:
        out = np.zeros(max(self.total, 1), dtype=np.int32)
        n = lib().oracle_fifo_snapshot(self._h, _p(out, _i32p))
        return out[:n].tolist()


class SeqTable:
    """SequenceBlockTable (page_allocator.hpp:376-475): append_token allocates one block when
    tokens_count % block_size == 0 (:426-434); release frees in table order (:461-469)."""

    def __init__(self, fifo: Fifo, block_size: int) -> None:
        self.fifo = fifo
        self.block_size = block_size
        self.blocks: List[int] = []
        self.tokens = 0

    def append_token(self) -> None:
        if self.tokens % self.block_size == 0:
            self.blocks.append(self.fifo.allocate_block())
        self.tokens += 1

    def append_tokens(self, n: int) -> None:
        for _ in range(n):
            self.append_token()

    def release(self) -> None:
        for b in self.blocks:
            self.fifo.free_block(b)
        self.blocks = []
        self.tokens = 0


# --------------------------------------------------------------------------------------------
# The reference's own kernel, compiled from its sources (oracle/_ref)
# --------------------------------------------------------------------------------------------

class RefKernel:
    """ctypes handle on oracle/_ref/libref_paged_kernels.so -- the reference's paged_attention
    (csrc/src/paged_kernels.cpp:7-105) built with its own CPU flags.  Thread count follows
    OMP_NUM_THREADS (or omp_set_num_threads through ``set_threads``)."""

    def __init__(self, path: str = REF_KERNEL_PATH) -> None:
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = ctypes.CDLL(path)
        self.lib.paged_attention.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int32, PagedDims, _i32p,
                                             _u8p, ctypes.c_float, _f32p, _f32p, ctypes.c_void_p]
        self.lib.paged_attention.restype = None
        try:
            gomp = ctypes.CDLL("libgomp.so.1")
            gomp.omp_set_num_threads.argtypes = [ctypes.c_int]
            self._gomp = gomp
        except OSError:
            self._gomp = None

    @staticmethod
    def available(path: str = REF_KERNEL_PATH) -> bool:
        return os.path.exists(path)

    def set_threads(self, n: int) -> None:
        if self._gomp is not None:
            self._gomp.omp_set_num_threads(int(n))

    def paged_attention(self, query, key_cache, value_cache, layer_idx, gather_slots,
                        attention_mask, scaling, scratch: Optional[np.ndarray] = None):
        q = np.ascontiguousarray(query, dtype=np.float32)
        kc = np.ascontiguousarray(key_cache, dtype=np.float32)
        vc = np.ascontiguousarray(value_cache, dtype=np.float32)
        gs = np.ascontiguousarray(gather_slots, dtype=np.int32)
        m = np.ascontiguousarray(attention_mask, dtype=np.uint8)
        dims = PagedDims(q.shape[1], q.shape[2], q.shape[3], kc.shape[0], kc.shape[1],
                         kc.shape[2], kc.shape[3], gs.shape[0])
        out = np.empty((1, dims.num_query_tokens, dims.num_query_heads, dims.head_dim),
                       np.float32)
        need = max(1, dims.num_query_tokens * dims.num_query_heads * gs.shape[0])
        if scratch is None or scratch.size < need:
            scratch = np.empty((need,), np.float32)
        self.lib.paged_attention(_p(q, _f32p), _p(kc, _f32p), _p(vc, _f32p), int(layer_idx), dims,
                                 _p(gs, _i32p), _p(m, _u8p), float(scaling), _p(out, _f32p),
                                 _p(scratch, _f32p), None)
        return out
