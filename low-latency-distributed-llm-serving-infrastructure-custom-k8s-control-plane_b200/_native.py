"""ctypes binding of libb200paged.so (C ABI declared in include/b200_paged.h).

The library is the product: there is no CPU fallback.  If it is missing, or the CUDA device is
absent, the calls below raise instead of computing anything on the host.  Status codes map onto
the exception types the reference's pybind layer raises for the same conditions
(csrc/src/bindings.cpp; pinned by tests/unit/test_allocator_bindings.py): invalid argument ->
ValueError, out of range -> IndexError, out of memory / runtime -> RuntimeError.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200paged.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_OUT_OF_MEMORY = 2
ERR_OUT_OF_RANGE = 3
ERR_RUNTIME = 4
ERR_UNSUPPORTED = 5
ERR_CUDA = 6

DEVICE_BAD_BLOCK = 1
DEVICE_BAD_SLOT = 2
DEVICE_TIMEOUT = 4
DEVICE_BAD_OP = 8
DEVICE_BAD_STEP = 16

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p
c_f = ctypes.c_float
c_sz = ctypes.c_size_t


class PagedAttentionDims(ctypes.Structure):
    """csrc/include/paged_kernels.h:11-20 field order."""
    _fields_ = [(n, c_i32) for n in ("num_query_heads", "num_query_tokens", "head_dim",
                                      "num_layers", "total_blocks", "block_size", "num_kv_heads",
                                      "num_context_tokens")]


class CacheGeometry(ctypes.Structure):
    _fields_ = [(n, c_i32) for n in ("num_layers", "total_blocks", "block_size", "num_kv_heads",
                                      "head_dim", "dtype")]


class DecodeParams(ctypes.Structure):
    _fields_ = [
        ("query", c_vp), ("q_stride_row", c_i64), ("q_stride_head", c_i64), ("query_rows", c_vp),
        ("key_cache", c_vp), ("value_cache", c_vp), ("geom", CacheGeometry), ("layer_idx", c_i32),
        ("num_query_heads", c_i32), ("block_tables", c_vp), ("block_table_stride", c_i32),
        ("context_lens", c_vp), ("num_seqs", c_i32), ("max_context_len", c_i32), ("scale", c_f),
        ("out", c_vp), ("o_stride_row", c_i64), ("o_stride_head", c_i64), ("status_word", c_vp),
    ]


class PrefillParams(ctypes.Structure):
    _fields_ = [
        ("query", c_vp), ("q_stride_token", c_i64), ("q_stride_head", c_i64),
        ("key_cache", c_vp), ("value_cache", c_vp), ("geom", CacheGeometry), ("layer_idx", c_i32),
        ("num_query_heads", c_i32), ("block_tables", c_vp), ("block_table_stride", c_i32),
        ("cu_seqlens", c_vp), ("context_lens", c_vp), ("num_seqs", c_i32), ("num_tokens", c_i32),
        ("max_query_len", c_i32), ("max_context_len", c_i32), ("scale", c_f), ("out", c_vp),
        ("o_stride_token", c_i64), ("o_stride_head", c_i64), ("status_word", c_vp),
    ]


# (name, restype, argtypes) for every entry point of include/b200_paged.h
SIGNATURES = [
    ("b200_status_string", ctypes.c_char_p, [ctypes.c_int]),
    ("b200_last_error", ctypes.c_char_p, []),
    ("paged_attention", None, [c_vp, c_vp, c_vp, c_i32, PagedAttentionDims, c_vp, c_vp, c_f, c_vp,
                               c_vp, c_vp]),
    ("b200_paged_attention", ctypes.c_int, [c_vp, c_vp, c_vp, c_i32, PagedAttentionDims, c_vp,
                                            c_vp, c_f, c_vp, c_vp, c_vp]),
    ("b200_paged_decode_workspace_bytes", c_sz, [ctypes.POINTER(DecodeParams)]),
    ("b200_paged_decode", ctypes.c_int, [ctypes.POINTER(DecodeParams), c_vp, c_sz, c_vp]),
    ("b200_paged_decode_static", ctypes.c_int, [ctypes.POINTER(DecodeParams), c_vp]),
    ("b200_set_decode_split_tokens", None, [c_i32]),
    ("b200_paged_prefill_workspace_bytes", c_sz, [ctypes.POINTER(PrefillParams)]),
    ("b200_paged_prefill", ctypes.c_int, [ctypes.POINTER(PrefillParams), c_vp, c_sz, c_vp]),
    ("b200_set_prefill_cuda_cores", None, [c_i32]),
    ("b200_set_prefill_kernel", None, [c_i32]),
    ("b200_set_prefill_poly_exp", None, [c_i32]),
    ("b200_reshape_and_cache", ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp,
                                              ctypes.POINTER(CacheGeometry), c_i32, c_vp, c_i32,
                                              c_vp, c_vp]),
    ("b200_rope_reshape_and_cache", ctypes.c_int, [c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp,
                                                   c_i64, c_vp, c_vp,
                                                   ctypes.POINTER(CacheGeometry), c_i32, c_vp,
                                                   c_vp, c_vp]),
    ("b200_copy_blocks", ctypes.c_int, [c_vp, c_vp, ctypes.POINTER(CacheGeometry), c_vp, c_vp,
                                        ctypes.POINTER(CacheGeometry), c_vp, c_vp, c_i32, c_vp,
                                        c_vp]),
    ("b200_pool_create", ctypes.c_int, [c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(c_vp)]),
    ("b200_pool_destroy", ctypes.c_int, [c_vp]),
    ("b200_pool_append_tokens", ctypes.c_int, [c_vp, c_i32, c_i32]),
    ("b200_pool_release", ctypes.c_int, [c_vp, c_i32]),
    ("b200_pool_share", ctypes.c_int, [c_vp, c_i32, c_i32, c_i32]),
    ("b200_pool_copy_on_write", ctypes.c_int, [c_vp, c_i32, c_i32]),
    ("b200_pool_cow_pairs", c_i32, [c_vp, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp)]),
    ("b200_pool_flush", ctypes.c_int, [c_vp, c_vp]),
    ("b200_pool_num_free_blocks", c_i32, [c_vp]),
    ("b200_pool_tokens", c_i32, [c_vp, c_i32]),
    ("b200_pool_num_blocks", c_i32, [c_vp, c_i32]),
    ("b200_pool_tables", c_vp, [c_vp]),
    ("b200_pool_table_stride", c_i32, [c_vp]),
    ("b200_pool_ring", c_vp, [c_vp]),
    ("b200_pool_status", c_vp, [c_vp]),
    ("b200_pool_snapshot_free", c_i32, [c_vp, ctypes.POINTER(c_i32), c_i32, c_vp]),
    ("b200_build_step_metadata", ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp,
                                                c_vp, c_vp, c_vp, c_vp, c_i32, c_vp, c_i64,
                                                c_vp]),
    ("b200_host_allocator_create", ctypes.c_int, [c_i64, c_i64, c_i64, c_i64,
                                                  ctypes.POINTER(c_vp)]),
    ("b200_host_allocator_destroy", None, [c_vp]),
    ("b200_host_allocate_block", ctypes.c_int, [c_vp, ctypes.POINTER(c_i32)]),
    ("b200_host_allocate_blocks", ctypes.c_int, [c_vp, c_i64, ctypes.POINTER(c_i32)]),
    ("b200_host_share_block", ctypes.c_int, [c_vp, c_i32]),
    ("b200_host_free_block", ctypes.c_int, [c_vp, c_i32]),
    ("b200_host_swap_out", ctypes.c_int, [c_vp, c_i32, ctypes.POINTER(c_i32)]),
    ("b200_host_swap_in", ctypes.c_int, [c_vp, c_i32, ctypes.POINTER(c_i32)]),
    ("b200_host_get_cpu_block_id", ctypes.c_int, [c_vp, c_i32, ctypes.POINTER(c_i32)]),
    ("b200_host_release_swapped_block", ctypes.c_int, [c_vp, c_i32]),
    ("b200_host_get_host_ptr", ctypes.c_int, [c_vp, c_i32, ctypes.POINTER(ctypes.c_uint64)]),
    ("b200_host_get_device_ptr", ctypes.c_int, [c_vp, c_i32, ctypes.POINTER(ctypes.c_uint64)]),
    ("b200_host_num_free_blocks", c_i64, [c_vp]),
    ("b200_host_num_free_cpu_blocks", c_i64, [c_vp]),
    ("b200_host_total_blocks", c_i64, [c_vp]),
    ("b200_host_block_size", c_i64, [c_vp]),
    ("b200_host_bytes_per_token", c_i64, [c_vp]),
    ("b200_host_pool_bytes", c_i64, [c_vp]),
    ("b200_host_utilization", ctypes.c_double, [c_vp]),
    ("b200_host_last_message", ctypes.c_char_p, []),
]

_LIB = None


def lib() -> ctypes.CDLL:
    """Load libb200paged.so (built in-tree by ``make -C <package>/csrc``)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                               "(the CUDA library is required; there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def exported_symbols():
    return [s[0] for s in SIGNATURES]


_EXC = {ERR_INVALID_ARGUMENT: ValueError, ERR_UNSUPPORTED: ValueError, ERR_OUT_OF_RANGE: IndexError,
        ERR_OUT_OF_MEMORY: RuntimeError, ERR_RUNTIME: RuntimeError, ERR_CUDA: RuntimeError}


def check(rc: int, host_message: bool = False) -> None:
    if rc == OK:
        return
    L = lib()
    msg = (L.b200_host_last_message() if host_message else L.b200_last_error()) or b""
    text = msg.decode(errors="replace") or L.b200_status_string(rc).decode()
    raise _EXC.get(rc, RuntimeError)(text)
