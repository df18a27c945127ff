"""Drop-in for app/model/attention_backends.py: the backend plug-in interface with the B200
native backend behind it.

``NativePagedBackend`` keeps the reference's ``supports``/``attend`` contract
(attention_backends.py:81-117) but runs on the GPU kernels and is no longer decode-only:
decode steps go to the split-K decode kernel (K1), prefill and mixed steps to the ragged causal
kernel.  The reference's ``torch`` backend (gather + SDPA) is the reference's own code and is not
re-provided here; asking for it raises, and nothing falls back to it silently.
"""
from __future__ import annotations

import os
from abc import ABC, abstractmethod
from typing import Optional

import torch

BACKEND_ENV_VAR = "LLM_PAGED_BACKEND"
TORCH_BACKEND = "torch"
NATIVE_BACKEND = "native"


def native_kernel_available() -> bool:
    try:
        from . import _native
        _native.lib()
    except Exception:
        return False
    return torch.cuda.is_available()


class AttentionBackend(ABC):
    name: str = ""

    @abstractmethod
    def supports(self, context, num_query_tokens: int) -> bool:
        ...

    @abstractmethod
    def attend(self, query: torch.Tensor, store, layer_idx: int, context, scaling: float,
               dropout: float) -> torch.Tensor:
        ...


class NativePagedBackend(AttentionBackend):
    name = NATIVE_BACKEND

    def supports(self, context, num_query_tokens: int) -> bool:
        return num_query_tokens > 0

    def attend(self, query: torch.Tensor, store, layer_idx: int, context, scaling: float,
               dropout: float) -> torch.Tensor:
        """query (1, Hq, Nq, D) as HF hands it over (any strides, D contiguous) ->
        (1, Nq, Hq, D), the shape the reference returns."""
        if not native_kernel_available():
            raise RuntimeError("libb200paged.so is not loadable or no CUDA device is present; "
                               "the native backend has no CPU path")
        if dropout:
            raise ValueError("the paged attention kernels are inference kernels (dropout 0)")
        from . import paged_ops
        q = query[0].transpose(0, 1)  # (Nq, Hq, D) view
        if q.stride(-1) != 1:
            q = q.contiguous()
        if context.is_decode:
            out = paged_ops.paged_decode(q, store.key_cache, store.value_cache, layer_idx,
                                         context.block_tables, context.context_lens_device,
                                         scaling, context.max_context_len)
        else:
            out = paged_ops.paged_prefill(q, store.key_cache, store.value_cache, layer_idx,
                                          context.block_tables, context.cu_seqlens_device,
                                          context.context_lens_device, scaling,
                                          context.max_query_len, context.max_context_len)
        return out.unsqueeze(0)


_BACKENDS = {NATIVE_BACKEND: NativePagedBackend}


def select_backend(requested: Optional[str] = None) -> AttentionBackend:
    """Same names as the reference (attention_backends.py:126-144): 'auto', 'native', 'hip'
    (alias of native); 'torch' names the reference's SDPA backend, which this package does not
    ship."""
    name = (requested or os.getenv(BACKEND_ENV_VAR) or "auto").lower()
    if name in ("auto", "hip"):
        name = NATIVE_BACKEND
    if name == TORCH_BACKEND:
        raise ValueError("the 'torch' SDPA backend belongs to the reference package; this package "
                         "provides the native B200 backend only")
    if name not in _BACKENDS:
        raise ValueError(f"Unsupported {BACKEND_ENV_VAR} '{name}'. Use 'auto' or 'native'.")
    backend = _BACKENDS[name]()
    if not native_kernel_available():
        raise RuntimeError(f"{BACKEND_ENV_VAR}={name} requires libb200paged.so and a CUDA device")
    return backend
