"""Device version of PagedStepContext (app/model/paged_attention.py:37-135).

Same constructor and attributes as the reference; the per-token metadata (slot mapping, positions,
block tables, context lengths, offsets) is built on the GPU by the metadata kernels (K4) from one
small upload of (slot, start, count) per sequence, instead of per-sequence host tensors.  The host
keeps the integer bookkeeping the engine reads back (context_lens list, cu_seqlens on the CPU,
token totals, max lengths).
"""
from __future__ import annotations

from typing import List, Optional

import torch


def _cumulative_offsets(counts: List[int]) -> torch.Tensor:
    """paged_attention.py:121-125: int64 offsets with a leading 0 (host tensor)."""
    out = torch.zeros(len(counts) + 1, dtype=torch.long)
    if counts:
        out[1:] = torch.cumsum(torch.tensor(counts, dtype=torch.long), 0)
    return out


class PagedStepContext:
    def __init__(self, store, sequences, start_positions: List[int],
                 new_token_counts: List[int]) -> None:
        if not (len(sequences) == len(start_positions) == len(new_token_counts)):
            raise ValueError(
                f"sequences ({len(sequences)}), start_positions ({len(start_positions)}) "
                f"and new_token_counts ({len(new_token_counts)}) must have the same length")
        self.store = store
        self.sequences = list(sequences)
        self.start_positions = [int(x) for x in start_positions]
        self.new_token_counts = [int(x) for x in new_token_counts]
        self.context_lens = [s + c for s, c in zip(self.start_positions, self.new_token_counts)]
        self.cu_seqlens = _cumulative_offsets(self.new_token_counts)
        self.cu_context_offsets = _cumulative_offsets(self.context_lens)
        self.max_query_len = max(self.new_token_counts, default=0)
        self.max_context_len = max(self.context_lens, default=0)
        self.is_decode = bool(self.sequences) and all(c == 1 for c in self.new_token_counts)
        self._gather: Optional[torch.Tensor] = None
        self._mask: Optional[torch.Tensor] = None
        if self.sequences:
            md = store.step_metadata(self.sequences, self.start_positions, self.new_token_counts)
            self.device_metadata = md
            self.scatter_slots = md["slot_mapping"]
            self.block_tables = md["block_tables"]
            self.context_lens_device = md["context_lens"]
            self.cu_seqlens_device = md["cu_seqlens"]
            self._position_ids = md["position_ids"]
        else:
            dev = store.torch_device
            self.device_metadata = {}
            self.scatter_slots = torch.empty((0,), dtype=torch.long, device=dev)
            self.block_tables = torch.empty((0, 1), dtype=torch.int32, device=dev)
            self.context_lens_device = torch.empty((0,), dtype=torch.int32, device=dev)
            self.cu_seqlens_device = torch.zeros((1,), dtype=torch.long, device=dev)
            self._position_ids = torch.empty((0,), dtype=torch.long, device=dev)

    @property
    def num_query_tokens(self) -> int:
        return int(self.cu_seqlens[-1])

    @property
    def num_context_tokens(self) -> int:
        return int(self.cu_context_offsets[-1])

    @property
    def gather_slots(self) -> torch.Tensor:
        """Every context token's slot, sequence by sequence (built on demand: the paged kernels
        read through the block tables and never need it)."""
        if self._gather is None:
            if not self.sequences:
                self._gather = torch.empty((0,), dtype=torch.long, device=self.store.torch_device)
            else:
                md = self.store.step_metadata(self.sequences, self.start_positions,
                                              self.new_token_counts, with_gather_slots=True)
                self._gather = md["gather_slots"]
        return self._gather

    def position_ids(self, device: torch.device) -> torch.Tensor:
        """Flat per-token positions restarting at every sequence (paged_attention.py:81-90)."""
        return self._position_ids.to(device).unsqueeze(0)

    def attention_mask(self, device: torch.device) -> torch.Tensor:
        """Dense block-diagonal causal mask (paged_attention.py:92-118), for callers of the
        reference's dense form only; the paged kernels apply the same causal rule themselves."""
        if self._mask is not None and self._mask.device == device:
            return self._mask
        counts = torch.tensor(self.new_token_counts, dtype=torch.long, device=device)
        ctx = torch.tensor(self.context_lens, dtype=torch.long, device=device)
        seq_ids = torch.arange(len(self.sequences), device=device)
        qi = torch.repeat_interleave(seq_ids, counts)
        ci = torch.repeat_interleave(seq_ids, ctx)
        qpos = self._position_ids.to(device)
        cpos = torch.arange(self.num_context_tokens, device=device) - \
            self.cu_context_offsets.to(device)[ci]
        self._mask = ((ci.unsqueeze(0) == qi.unsqueeze(1)) &
                      (cpos.unsqueeze(0) <= qpos.unsqueeze(1))).unsqueeze(0).unsqueeze(0)
        return self._mask
