"""Random-init Llama-style decoder for the engine rows (BASELINE configs 4 and 5), tensor-parallel
by KV head.

The reference serves a transformers Llama whose attention goes through its paged hook
(app/model/paged_attention.py:138-207); here the decoder is a lean torch module whose attention
is the B200 path: reshape_and_cache (K2) + paged decode (K1) / ragged causal prefill (K3) over
the device block pool's tables (K4/K5).  GEMMs, norms and RoPE are torch (cuBLAS) ops.

Tensor parallelism over `world` ranks (one process per GPU): rank r owns KV heads
[r*Hkv/world, (r+1)*Hkv/world) and their query heads (QKV column-parallel), the matching slice of
the MLP (gate/up column-parallel); o_proj and down_proj are row-parallel and followed by an NCCL
all-reduce (sum) -- the only exchange steps.  The LM head is vocab-parallel; greedy sampling
takes each rank's local (max, argmax) and all-gathers them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F


@dataclass
class LlamaShape:
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0


CONFIG4 = LlamaShape(16, 2048, 32, 8, 64, 8192, 32000)
CONFIG5 = LlamaShape(32, 4096, 32, 8, 128, 14336, 128256, rope_theta=500000.0)


class TPLlama:
    """Weights of one tensor-parallel rank, random-initialised from a seed.

    ``full_init=True`` draws every full weight from one generator and slices this rank's part,
    so different world sizes hold the same model (used by the TP parity tests); otherwise each
    shard is drawn from its own seed (fast start-up of large shapes)."""

    def __init__(self, shape: LlamaShape, rank: int = 0, world: int = 1,
                 device: Optional[torch.device] = None, dtype: torch.dtype = torch.bfloat16,
                 seed: int = 0, full_init: bool = False, group=None) -> None:
        if shape.num_kv_heads % world or shape.num_heads % world or shape.ffn % world:
            raise ValueError("heads and ffn must divide by the tensor-parallel world size")
        self.shape, self.rank, self.world, self.group = shape, rank, world, group
        self.device = torch.device(device or "cuda")
        self.dtype = dtype
        s = shape
        self.hq = s.num_heads // world
        self.hkv = s.num_kv_heads // world
        self.ffn = s.ffn // world
        self.vocab_shard = (s.vocab + world - 1) // world
        self.vocab_lo = rank * self.vocab_shard
        self.vocab_hi = min(s.vocab, self.vocab_lo + self.vocab_shard)
        D = s.head_dim
        std = 0.02
        g = torch.Generator(device=self.device)

        def draw(name_seed: int, full_shape, rows=None, cols=None):
            if full_init:
                g.manual_seed(seed * 1000003 + name_seed)
                w = torch.randn(full_shape, generator=g, device=self.device, dtype=torch.float32)
                if rows is not None:
                    w = w[rows]
                if cols is not None:
                    w = w[:, cols]
                return (w * std).to(dtype).contiguous()
            g.manual_seed(seed * 1000003 + name_seed * 131 + rank)
            shp = list(full_shape)
            if rows is not None:
                shp[0] = len(range(*rows.indices(full_shape[0]))) if isinstance(rows, slice) else len(rows)
            if cols is not None:
                shp[1] = len(range(*cols.indices(full_shape[1]))) if isinstance(cols, slice) else len(cols)
            return (torch.randn(shp, generator=g, device=self.device, dtype=torch.float32) * std).to(dtype)

        def head_rows(n_heads_total, n_local):
            lo = rank * n_local * D
            return slice(lo, lo + n_local * D)

        self.embed = draw(1, (s.vocab, s.hidden))
        self.final_norm = torch.ones(s.hidden, device=self.device, dtype=dtype)
        self.lm_head = draw(2, (s.vocab, s.hidden), rows=slice(self.vocab_lo, self.vocab_hi))
        self.layers = []
        for li in range(s.num_layers):
            base = 100 + 10 * li
            wq = draw(base + 0, (s.num_heads * D, s.hidden), rows=head_rows(s.num_heads, self.hq))
            wk = draw(base + 1, (s.num_kv_heads * D, s.hidden), rows=head_rows(s.num_kv_heads, self.hkv))
            wv = draw(base + 2, (s.num_kv_heads * D, s.hidden), rows=head_rows(s.num_kv_heads, self.hkv))
            wo = draw(base + 3, (s.hidden, s.num_heads * D), cols=head_rows(s.num_heads, self.hq))
            f0 = rank * self.ffn
            wg = draw(base + 4, (s.ffn, s.hidden), rows=slice(f0, f0 + self.ffn))
            wu = draw(base + 5, (s.ffn, s.hidden), rows=slice(f0, f0 + self.ffn))
            wd = draw(base + 6, (s.hidden, s.ffn), cols=slice(f0, f0 + self.ffn))
            self.layers.append({
                "wqkv": torch.cat([wq, wk, wv], 0).contiguous(),
                "wo": wo, "wgu": torch.cat([wg, wu], 0).contiguous(), "wd": wd,
                "n1": torch.ones(s.hidden, device=self.device, dtype=dtype),
                "n2": torch.ones(s.hidden, device=self.device, dtype=dtype),
            })
        inv = 1.0 / (s.rope_theta ** (torch.arange(0, D, 2, device=self.device,
                                                   dtype=torch.float32) / D))
        self._inv_freq = inv

    # ---- collectives ------------------------------------------------------------------------
    def _all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(x, group=self.group)
        return x

    # ---- pieces ----------------------------------------------------------------------------
    def _rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        # rotate-half RoPE on (tokens, heads, D)
        d2 = x.shape[-1] // 2
        x1, x2 = x[..., :d2].float(), x[..., d2:].float()
        c, s_ = cos[:, None, :], sin[:, None, :]
        return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_], dim=-1).to(x.dtype)

    def _norm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return F.rms_norm(x, (x.shape[-1],), w, self.shape.rms_eps)

    @property
    def inv_freq(self) -> torch.Tensor:
        """Rotary frequencies (head_dim/2,) fp32 on the device."""
        return self._inv_freq

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, attend=None,
                attend_qkv=None) -> torch.Tensor:
        """input_ids, positions: (Ntok,) on the device.  Either ``attend(layer, q, k, v)`` gets
        the rotated q/k and v, writes the layer's new K/V into the paged cache and returns the
        attention output (Ntok, hq, D); or ``attend_qkv(layer, qkv)`` gets the raw QKV
        projection rows (Ntok, (hq + 2*hkv) * D) and does rotary, cache write and attention
        itself (the fused path).  Returns the final hidden states (Ntok, hidden)."""
        s = self.shape
        D = s.head_dim
        if attend_qkv is None:
            ang = positions.float()[:, None] * self._inv_freq[None, :]
            cos, sin = torch.cos(ang), torch.sin(ang)
        h = F.embedding(input_ids, self.embed)
        nq, nkv = self.hq * D, self.hkv * D
        for li, L in enumerate(self.layers):
            x = self._norm(h, L["n1"])
            qkv = F.linear(x, L["wqkv"])
            if attend_qkv is not None:
                o = attend_qkv(li, qkv)
            else:
                q = self._rope(qkv[:, :nq].view(-1, self.hq, D), cos, sin)
                k = self._rope(qkv[:, nq:nq + nkv].view(-1, self.hkv, D), cos, sin)
                v = qkv[:, nq + nkv:].view(-1, self.hkv, D)
                o = attend(li, q, k, v)
            h = h + self._all_reduce(F.linear(o.reshape(-1, nq), L["wo"]))
            x = self._norm(h, L["n2"])
            gu = F.linear(x, L["wgu"])
            a = F.silu(gu[:, :self.ffn]) * gu[:, self.ffn:]
            h = h + self._all_reduce(F.linear(a, L["wd"]))
        return self._norm(h, self.final_norm)

    def greedy(self, hidden_last: torch.Tensor) -> torch.Tensor:
        """Greedy next token for each row of (S, hidden), on the device (vocab-parallel)."""
        logits = F.linear(hidden_last, self.lm_head).float()
        val, idx = logits.max(dim=-1)
        idx = idx + self.vocab_lo
        if self.world == 1:
            return idx
        import torch.distributed as dist
        both = torch.stack([val, idx.float()], 0).contiguous()
        gathered = [torch.empty_like(both) for _ in range(self.world)]
        dist.all_gather(gathered, both, group=self.group)
        g = torch.stack(gathered, 0)  # (world, 2, S)
        best = g[:, 0, :].argmax(dim=0)  # lowest rank wins ties, i.e. the lowest vocab id
        return g[best, 1, torch.arange(g.shape[2], device=g.device)].long()

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Full logits (for tests): gathers the vocab shards."""
        lg = F.linear(hidden, self.lm_head).float()
        if self.world == 1:
            return lg
        import torch.distributed as dist
        parts = [torch.empty_like(lg) for _ in range(self.world)]
        dist.all_gather(parts, lg.contiguous(), group=self.group)
        return torch.cat(parts, -1)[:, :self.shape.vocab]


def kv_bytes_per_token(shape: LlamaShape, world: int = 1, elem: int = 2) -> int:
    return shape.num_layers * (shape.num_kv_heads // world) * shape.head_dim * elem * 2


def param_bytes(shape: LlamaShape, world: int = 1, elem: int = 2) -> int:
    s = shape
    per_layer = (s.num_heads + 2 * s.num_kv_heads) * s.head_dim * s.hidden // world + \
        s.hidden * s.num_heads * s.head_dim // world + 3 * s.ffn * s.hidden // world
    return elem * (s.num_layers * per_layer + s.vocab * s.hidden + math.ceil(s.vocab / world) * s.hidden)
