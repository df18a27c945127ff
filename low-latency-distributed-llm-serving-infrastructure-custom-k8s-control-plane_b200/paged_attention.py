"""Per-layer attention hook, same calling convention as app/model/paged_attention.py:138-207.

``paged_attention_forward`` is what transformers calls through ALL_ATTENTION_FUNCTIONS["paged"]:
it writes the layer's new K/V into the paged cache (reshape_and_cache, K2) and attends through
the block tables on the GPU (NativePagedBackend).  There is no inline SDPA fallback: an
unsupported shape raises.
"""
from __future__ import annotations

from typing import Optional

import torch

from .attention_backends import NativePagedBackend

PAGED_ATTENTION_NAME = "paged"

# Pluggable backend, as the reference's hook (paged_attention.py:22-25); None = native.
_BACKEND = None
_NATIVE = None


def _backend():
    global _NATIVE
    if _BACKEND is not None:
        return _BACKEND
    if _NATIVE is None:
        _NATIVE = NativePagedBackend()
    return _NATIVE


def paged_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                            value: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                            dropout: float = 0.0, scaling: Optional[float] = None,
                            **kwargs) -> tuple:
    context = module.paged_context
    store = context.store
    layer_idx = module.layer_idx
    new_keys = key.squeeze(0).transpose(0, 1)      # (Ntok, Hkv, D) view
    new_values = value.squeeze(0).transpose(0, 1)
    store.scatter_layer_kv(layer_idx, new_keys, new_values, context.scatter_slots)
    scale = scaling if scaling is not None else module.scaling
    backend = _backend()
    if not backend.supports(context, query.shape[2]):
        raise ValueError(f"backend {backend.name!r} does not support this step "
                         f"({query.shape[2]} query tokens)")
    return backend.attend(query, store, layer_idx, context, scale, dropout), None


def _decoder(model) -> torch.nn.Module:
    for attribute in ("model", "transformer", "base_model"):
        candidate = getattr(model, attribute, None)
        if candidate is not None and hasattr(candidate, "layers"):
            return candidate
    return model


def register_paged_attention(model) -> None:
    """Route every decoder layer of ``model`` through the paged attention."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_ATTENTION_FUNCTIONS.register(PAGED_ATTENTION_NAME, paged_attention_forward)
    for layer in _decoder(model).layers:
        layer.self_attn.paged_context = None
    model.config._attn_implementation = PAGED_ATTENTION_NAME


def run_paged_forward(model, context, input_ids: torch.Tensor) -> torch.Tensor:
    """One flat forward pass whose KV lands in the paged blocks; returns the logits."""
    for layer in _decoder(model).layers:
        layer.self_attn.paged_context = context
    position_ids = context.position_ids(input_ids.device)
    outputs = model(input_ids, position_ids=position_ids, use_cache=False)
    return outputs.logits
