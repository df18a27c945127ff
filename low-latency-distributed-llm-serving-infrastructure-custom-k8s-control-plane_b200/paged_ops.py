"""Torch-tensor front end of the C ABI: device tensors in, device tensors out.

torch is used here for device memory and streams only; every computation runs in
libb200paged.so.  Each function raises if a tensor is not on a CUDA device -- there is no CPU
fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native as N

_DTYPES = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16, torch.float16: N.DTYPE_F16}


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("libb200paged kernels need CUDA tensors (no CPU fallback)")


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def cache_geometry(key_cache: torch.Tensor) -> N.CacheGeometry:
    if key_cache.dim() != 5:
        raise ValueError("key_cache must be 5-D (layers, blocks, block_size, heads, dim)")
    if not key_cache.is_contiguous():
        raise ValueError("caches must be contiguous (L, NB, BS, Hkv, D)")
    if key_cache.dtype not in _DTYPES:
        raise ValueError(f"unsupported cache dtype {key_cache.dtype}")
    L, NB, BS, Hkv, D = key_cache.shape
    return N.CacheGeometry(L, NB, BS, Hkv, D, _DTYPES[key_cache.dtype])


class Workspace:
    """Grow-only device scratch buffer per (device, stream), 256-byte aligned.  Keyed by stream
    because the kernels of one call use the scratch until they finish: two streams sharing one
    buffer would race, and a buffer replaced by a larger one is released in the order of the
    stream that used it."""

    def __init__(self):
        self._buf = {}

    def get(self, device: torch.device, nbytes: int, stream: int) -> torch.Tensor:
        key = (device.type, device.index, stream)
        buf = self._buf.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._buf[key] = buf
        return buf


_WORKSPACE = Workspace()
_STATUS = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The device status word the kernels flag (one per GPU; ``cuda`` without an index means
    the current device, so it names the same word as ``cuda:<current>``)."""
    device = torch.device(device)
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (device.type, index)
    if key not in _STATUS:
        _STATUS[key] = torch.zeros(1, dtype=torch.int32, device=torch.device(device.type, index))
    return _STATUS[key]


def read_status(device: torch.device, reset: bool = True) -> int:
    s = status_word(device)
    v = int(s.item())
    if reset:
        s.zero_()
    return v


def _check_attention_args(query, key_cache, value_cache, out, block_tables, context_lens,
                          num_rows_needed) -> N.CacheGeometry:
    """Shape and dtype rules the C ABI cannot see (its query and output carry no dtype or head
    dim of their own: the kernels read them as the cache's).  ``num_rows_needed``: query rows the
    kernels index directly (None when a row map places them)."""
    geom = cache_geometry(key_cache)
    if value_cache.shape != key_cache.shape or value_cache.dtype != key_cache.dtype:
        raise ValueError("value_cache must have the key cache's shape and dtype")
    if not value_cache.is_contiguous():
        raise ValueError("caches must be contiguous (L, NB, BS, Hkv, D)")
    if query.dim() != 3 or query.stride(-1) != 1:
        raise ValueError("query must be (rows, Hq, D) with the head dim contiguous")
    if query.shape[2] != geom.head_dim:
        raise ValueError(f"query head dim {query.shape[2]} != cache head dim {geom.head_dim}")
    if query.dtype != key_cache.dtype:
        raise ValueError(f"query dtype {query.dtype} must match the cache dtype {key_cache.dtype}")
    if num_rows_needed is not None and query.shape[0] < num_rows_needed:
        raise ValueError(f"query has {query.shape[0]} rows, the batch needs {num_rows_needed}")
    if out is not None:
        if out.dtype != key_cache.dtype:
            raise ValueError(f"out dtype {out.dtype} must match the cache dtype {key_cache.dtype}")
        if out.shape != query.shape or out.stride(-1) != 1:
            raise ValueError("out must have the query's shape with the head dim contiguous")
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise ValueError("block_tables and context_lens must be int32")
    if block_tables.dim() not in (1, 2) or block_tables.stride(-1) != 1:
        raise ValueError("block_tables must be (S, max_blocks) with unit stride along a row")
    if context_lens.dim() != 1 or not context_lens.is_contiguous():
        raise ValueError("context_lens must be a contiguous (S,) tensor")
    if block_tables.dim() == 2 and block_tables.shape[0] < context_lens.shape[0]:
        raise ValueError("block_tables has fewer rows than context_lens has sequences")
    return geom


def decode_params(query, key_cache, value_cache, layer_idx, block_tables, context_lens, scale,
                  out, max_context_len, query_rows=None, status=None) -> N.DecodeParams:
    geom = _check_attention_args(query, key_cache, value_cache, out, block_tables, context_lens,
                                 context_lens.shape[0] if query_rows is None else None)
    if query_rows is not None and (query_rows.dtype != torch.int32 or
                                   query_rows.shape != context_lens.shape):
        raise ValueError("query_rows must be int32 with one entry per sequence")
    p = N.DecodeParams()
    p.query = query.data_ptr()
    p.q_stride_row, p.q_stride_head = query.stride(0), query.stride(1)
    p.query_rows = _ptr(query_rows)
    p.key_cache, p.value_cache = key_cache.data_ptr(), value_cache.data_ptr()
    p.geom = geom
    p.layer_idx = int(layer_idx)
    p.num_query_heads = query.shape[1]
    p.block_tables = block_tables.data_ptr()
    p.block_table_stride = block_tables.stride(0) if block_tables.dim() == 2 else 0
    p.context_lens = context_lens.data_ptr()
    p.num_seqs = context_lens.shape[0]
    p.max_context_len = int(max_context_len)
    p.scale = float(scale)
    p.out = out.data_ptr()
    p.o_stride_row, p.o_stride_head = out.stride(0), out.stride(1)
    p.status_word = _ptr(status)
    return p


def paged_decode(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 layer_idx: int, block_tables: torch.Tensor, context_lens: torch.Tensor,
                 scale: float, max_context_len: int, out: Optional[torch.Tensor] = None,
                 query_rows: Optional[torch.Tensor] = None,
                 workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention (one new token per sequence) read through block tables (K1).
    query (rows, Hq, D); caches (L, NB, BS, Hkv, D); block_tables (S, max_blocks) int32;
    context_lens (S,) int32.  Returns out (rows, Hq, D) in the cache dtype."""
    if out is None:
        out = torch.empty_like(query, dtype=key_cache.dtype)
    p = decode_params(query, key_cache, value_cache, layer_idx, block_tables, context_lens, scale,
                      out, max_context_len, query_rows)
    _require_cuda(query, key_cache, value_cache, block_tables, context_lens, query_rows, out)
    p.status_word = status_word(query.device).data_ptr()
    L = N.lib()
    stream = _stream(query.device)
    need = L.b200_paged_decode_workspace_bytes(ctypes.byref(p))
    ws = workspace if workspace is not None else _WORKSPACE.get(query.device, need, stream)
    N.check(L.b200_paged_decode(ctypes.byref(p), ws.data_ptr() if need else None, ws.numel(),
                                stream))
    return out


def paged_prefill(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                  layer_idx: int, block_tables: torch.Tensor, cu_seqlens: torch.Tensor,
                  context_lens: torch.Tensor, scale: float, max_query_len: int,
                  max_context_len: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Ragged causal attention through block tables (prefill chunks / mixed steps).
    query (Ntok, Hq, D); cu_seqlens (S+1,) int64; context_lens (S,) int32."""
    if out is None:
        out = torch.empty_like(query, dtype=key_cache.dtype)
    geom = _check_attention_args(query, key_cache, value_cache, out, block_tables, context_lens,
                                 None)
    if block_tables.dim() != 2:
        raise ValueError("block_tables must be (S, max_blocks)")
    if (cu_seqlens.dtype != torch.int64 or cu_seqlens.dim() != 1 or
            not cu_seqlens.is_contiguous() or cu_seqlens.numel() != context_lens.numel() + 1):
        raise ValueError("cu_seqlens must be a contiguous int64 (S+1,) tensor")
    _require_cuda(query, key_cache, value_cache, block_tables, cu_seqlens, context_lens, out)
    p = N.PrefillParams()
    p.query = query.data_ptr()
    p.q_stride_token, p.q_stride_head = query.stride(0), query.stride(1)
    p.key_cache, p.value_cache = key_cache.data_ptr(), value_cache.data_ptr()
    p.geom = geom
    p.layer_idx = int(layer_idx)
    p.num_query_heads = query.shape[1]
    p.block_tables = block_tables.data_ptr()
    p.block_table_stride = block_tables.stride(0)
    p.cu_seqlens = cu_seqlens.data_ptr()
    p.context_lens = context_lens.data_ptr()
    p.num_seqs = context_lens.shape[0]
    p.num_tokens = query.shape[0]
    p.max_query_len = int(max_query_len)
    p.max_context_len = int(max_context_len)
    p.scale = float(scale)
    p.out = out.data_ptr()
    p.o_stride_token, p.o_stride_head = out.stride(0), out.stride(1)
    p.status_word = status_word(query.device).data_ptr()
    L = N.lib()
    stream = _stream(query.device)
    need = L.b200_paged_prefill_workspace_bytes(ctypes.byref(p))
    ws = _WORKSPACE.get(query.device, need, stream) if need else None
    N.check(L.b200_paged_prefill(ctypes.byref(p), None if ws is None else ws.data_ptr(),
                                 0 if ws is None else ws.numel(), stream))
    return out


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor,
                      value_cache: torch.Tensor, slot_mapping: torch.Tensor,
                      layer_idx: int) -> None:
    """key/value (Ntok, Hkv, D) (any strides, D contiguous) -> cache slots (K2)."""
    _require_cuda(key, value, key_cache, value_cache, slot_mapping)
    geom = cache_geometry(key_cache)
    if key.dtype != key_cache.dtype or value.dtype != value_cache.dtype:
        raise ValueError("key/value dtype must match the cache dtype")
    if slot_mapping.dtype != torch.int64:
        raise ValueError("slot_mapping must be int64")
    if key.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError("head dim must be contiguous")
    N.check(N.lib().b200_reshape_and_cache(
        key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0),
        value.stride(1), key_cache.data_ptr(), value_cache.data_ptr(), ctypes.byref(geom),
        int(layer_idx), slot_mapping.data_ptr(), slot_mapping.numel(),
        status_word(key.device).data_ptr(), _stream(key.device)))


def rope_reshape_and_cache(qkv: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
                           num_query_heads: int, key_cache: torch.Tensor,
                           value_cache: torch.Tensor, slot_mapping: torch.Tensor, layer_idx: int,
                           q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotary embedding fused into the slot write (K2 with rotary).

    qkv (Ntok, (Hq + 2*Hkv) * D) = the fused QKV projection output (rows [q | k | v], unit
    stride inside a row); positions (Ntok,) int64; inv_freq (D/2,) fp32.  Rotated k and v go to
    their cache slots; returns the rotated q as (Ntok, Hq, D) (written into ``q_out`` if given).
    Bit-identical to rotate-half rotary in fp32 followed by ``reshape_and_cache``."""
    _require_cuda(qkv, positions, inv_freq, key_cache, value_cache, slot_mapping)
    geom = cache_geometry(key_cache)
    if qkv.dtype != key_cache.dtype or value_cache.dtype != key_cache.dtype:
        raise ValueError("qkv dtype must match the cache dtype")
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be (tokens, row) with unit stride inside a row")
    if positions.dtype != torch.int64 or slot_mapping.dtype != torch.int64:
        raise ValueError("positions and slot_mapping must be int64")
    if inv_freq.dtype != torch.float32 or not inv_freq.is_contiguous():
        raise ValueError("inv_freq must be contiguous float32")
    n = qkv.shape[0]
    D = geom.head_dim
    if qkv.shape[1] < (int(num_query_heads) + 2 * geom.num_kv_heads) * D:
        raise ValueError("qkv rows shorter than the q, k and v heads")
    if q_out is None:
        q_out = torch.empty((n, num_query_heads, D), dtype=qkv.dtype, device=qkv.device)
    if q_out.stride(2) != 1 or q_out.stride(1) != D:
        raise ValueError("q_out must have contiguous heads")
    N.check(N.lib().b200_rope_reshape_and_cache(
        qkv.data_ptr(), qkv.stride(0), n, int(num_query_heads), positions.data_ptr(),
        inv_freq.data_ptr(), q_out.data_ptr(), q_out.stride(0), key_cache.data_ptr(),
        value_cache.data_ptr(), ctypes.byref(geom), int(layer_idx), slot_mapping.data_ptr(),
        status_word(qkv.device).data_ptr(), _stream(qkv.device)))
    return q_out


def _block_ids(ids, device: torch.device) -> torch.Tensor:
    if isinstance(ids, torch.Tensor):
        t = ids.to(dtype=torch.int32)
        if t.is_cuda or t.is_pinned():
            return t.contiguous()
        return t.contiguous().to(device)
    return torch.tensor(list(ids), dtype=torch.int32, device=device)


def copy_blocks(src_key_cache: torch.Tensor, src_value_cache: Optional[torch.Tensor],
                dst_key_cache: torch.Tensor, dst_value_cache: Optional[torch.Tensor],
                src_blocks, dst_blocks, device: Optional[torch.device] = None) -> None:
    """Copy whole blocks (every layer) between two caches of the same per-block geometry (K6):
    block ``src_blocks[i]`` of the source K (and V) caches -> block ``dst_blocks[i]`` of the
    destination.  Caches are (L, NB, BS, Hkv, D) tensors on the GPU or in page-locked host memory
    (``pin_memory``): GPU -> host is a swap out, host -> GPU a swap in, GPU -> GPU the copy made
    before writing a shared block.  The value caches may both be None (key caches only).
    Asynchronous on the current stream of ``device`` (default: the GPU side's device)."""
    caches = [t for t in (src_key_cache, src_value_cache, dst_key_cache, dst_value_cache)
              if t is not None]
    for t in caches:
        if not (t.is_cuda or t.is_pinned()):
            raise ValueError("caches must be on the GPU or in page-locked host memory")
    if (src_value_cache is None) != (dst_value_cache is None):
        raise ValueError("value caches must be both given or both None")
    gpu = [t.device for t in caches if t.is_cuda]
    dev = torch.device(device) if device is not None else (gpu[0] if gpu else
                                                            torch.device("cuda"))
    sg, dg = cache_geometry(src_key_cache), cache_geometry(dst_key_cache)
    for a, b in ((src_value_cache, src_key_cache), (dst_value_cache, dst_key_cache)):
        if a is not None and a.shape != b.shape:
            raise ValueError("key and value caches of one side must have the same shape")
    s_ids, d_ids = _block_ids(src_blocks, dev), _block_ids(dst_blocks, dev)
    if s_ids.numel() != d_ids.numel():
        raise ValueError("src_blocks and dst_blocks must have the same length")
    with torch.cuda.device(dev):
        N.check(N.lib().b200_copy_blocks(
            src_key_cache.data_ptr(), None if src_value_cache is None else src_value_cache.data_ptr(),
            ctypes.byref(sg), dst_key_cache.data_ptr(),
            None if dst_value_cache is None else dst_value_cache.data_ptr(), ctypes.byref(dg),
            s_ids.data_ptr(), d_ids.data_ptr(), s_ids.numel(), status_word(dev).data_ptr(),
            _stream(dev)))


def paged_attention_masked(query: torch.Tensor, key_cache: torch.Tensor,
                           value_cache: torch.Tensor, layer_idx: int, gather_slots: torch.Tensor,
                           attention_mask: torch.Tensor, scaling: float) -> torch.Tensor:
    """The reference kernel's contract (csrc/src/bindings.cpp:10-76) on device tensors:
    query (1,Hq,Nq,D), fp32 caches (L,NB,BS,Hkv,D), gather_slots (Nctx,), mask (1,1,Nq,Nctx)
    -> (1,Nq,Hq,D) fp32 on the device.  Runs ``b200_paged_attention``, the status-returning form
    of the C symbol ``paged_attention`` (same kernel, same arguments).  The caches must be fp32,
    as in the reference; they are never converted here (a whole-cache copy per layer per call
    would cost far more than the attention).  The query is cast to fp32 if it is not already."""
    _require_cuda(query, key_cache, value_cache, gather_slots, attention_mask)
    if query.dim() != 4:
        raise RuntimeError("query must be 4-D (1, heads, seq, dim)")
    if key_cache.dim() != 5:
        raise RuntimeError("key_cache must be 5-D (layers, blocks, block_size, heads, dim)")
    if gather_slots.dim() != 1:
        raise RuntimeError("gather_slots must be 1-D")
    if attention_mask.dim() != 4:
        raise RuntimeError("attention_mask must be 4-D (1, 1, query, context)")
    for name, c in (("key_cache", key_cache), ("value_cache", value_cache)):
        if c.dtype != torch.float32:
            raise TypeError(f"{name} must be float32 (the reference kernel's cache type), got "
                            f"{c.dtype}; the bf16/f16 paths are paged_decode / paged_prefill")
    if value_cache.shape != key_cache.shape:
        raise RuntimeError("key_cache and value_cache must have the same shape")
    q = query.to(torch.float32).contiguous()
    kc = key_cache.contiguous()
    vc = value_cache.contiguous()
    gs = gather_slots.to(torch.int32).contiguous()
    m = attention_mask.to(torch.uint8).contiguous()
    dims = N.PagedAttentionDims(q.shape[1], q.shape[2], q.shape[3], kc.shape[0], kc.shape[1],
                                kc.shape[2], kc.shape[3], gs.shape[0])
    if dims.num_query_heads % dims.num_kv_heads != 0:
        raise RuntimeError("num_query_heads must be a multiple of num_kv_heads for GQA")
    if layer_idx < 0 or layer_idx >= dims.num_layers:
        raise RuntimeError("layer_idx out of range")
    out = torch.empty((1, dims.num_query_tokens, dims.num_query_heads, dims.head_dim),
                      dtype=torch.float32, device=q.device)
    if dims.num_query_tokens == 0:
        return out
    L = N.lib()
    rc = L.b200_paged_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), int(layer_idx), dims,
                                gs.data_ptr(), m.data_ptr(), float(scaling), out.data_ptr(),
                                status_word(q.device).data_ptr(), _stream(q.device))
    N.check(rc)
    return out
