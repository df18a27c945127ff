"""Seeded synthetic workloads for the paged-attention hot path.

The reference names no public benchmark or dataset; every input here is synthetic, drawn from a
recorded seed with numpy's PCG64 (structure: context lengths, block pools, block tables) so the
same seed gives the same batch on every machine.  Tensor values (Q/K/V) are drawn by the caller,
either with numpy (small cases, CPU) or with a seeded torch generator on the device (large cases).

Layouts follow the reference: caches (L, NB, BS, Hkv, D) (app/memory/strategies.py:82-86), block
tables (S, max_blocks) int32 padded with -1 (app/memory/manager.py:236-271), slot =
block * BS + offset (app/memory/manager.py:320-333).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List

import numpy as np


@dataclass
class PagedBatch:
    """Structure of one engine step over a paged KV pool."""

    name: str
    num_query_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    total_blocks: int
    start_positions: np.ndarray      # (S,) int32 -- tokens already cached before this step
    new_token_counts: np.ndarray     # (S,) int32 -- tokens this step adds (1 for decode)
    tables: List[List[int]]          # physical blocks per sequence, covering start+count tokens
    scale: float
    dtype: str = "bf16"
    seed: int = 0
    free_list: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))

    @property
    def num_seqs(self) -> int:
        return len(self.tables)

    @property
    def context_lens(self) -> np.ndarray:
        return (self.start_positions + self.new_token_counts).astype(np.int32)

    @property
    def num_tokens(self) -> int:
        return int(self.new_token_counts.sum())

    @property
    def max_blocks(self) -> int:
        return max((len(t) for t in self.tables), default=0)

    def block_tables(self) -> np.ndarray:
        bt = np.full((self.num_seqs, max(self.max_blocks, 1)), -1, dtype=np.int32)
        for i, t in enumerate(self.tables):
            bt[i, :len(t)] = t
        return bt

    def cu_seqlens(self) -> np.ndarray:
        out = np.zeros(self.num_seqs + 1, np.int64)
        out[1:] = np.cumsum(self.new_token_counts)
        return out

    def slot_mapping(self) -> np.ndarray:
        """Slots of the new tokens, concatenated in sequence order (manager.py:104-128)."""
        parts = []
        for t, s, c in zip(self.tables, self.start_positions, self.new_token_counts):
            pos = np.arange(s, s + c, dtype=np.int64)
            parts.append(np.asarray(t, np.int64)[pos // self.block_size] * self.block_size
                         + pos % self.block_size)
        return np.concatenate(parts) if parts else np.zeros(0, np.int64)

    def kv_bytes(self, elem_bytes: int) -> int:
        """Algorithmic K+V bytes of one attention pass: every context token of every KV head is
        read once (GQA groups share the read)."""
        return int(self.context_lens.astype(np.int64).sum()) * self.num_kv_heads * self.head_dim \
            * elem_bytes * 2


def _assign_blocks(rng: np.random.Generator, ctx: np.ndarray, block_size: int, slack: float,
                   shuffled: bool):
    need = [(-(-int(c) // block_size)) for c in ctx]
    total = int(math.ceil(sum(need) * (1.0 + slack))) + 1
    free = rng.permutation(total).astype(np.int32) if shuffled else np.arange(total, dtype=np.int32)
    tables, off = [], 0
    for n in need:
        tables.append(free[off:off + n].tolist())
        off += n
    return tables, total, free[off:]


def config1(seed: int = 0) -> PagedBatch:
    """Config 1: 8 decode sequences, context U[1,512], 12/12 heads, D 64, BS 16, fp32, block
    tables as consecutive chunks of a random permutation of a 512-block pool, scale 1/8."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 513, size=8).astype(np.int32)
    perm = rng.permutation(512).astype(np.int32)
    tables, off = [], 0
    for c in ctx:
        n = -(-int(c) // 16)
        tables.append(perm[off:off + n].tolist())
        off += n
    return PagedBatch("config1", 12, 12, 64, 16, 512, ctx - 1, np.ones(8, np.int32), tables,
                      1.0 / 8.0, "fp32", seed, perm[off:])


def lognormal_contexts(rng: np.random.Generator, n: int, median: float, sigma: float, lo: int,
                       hi: int) -> np.ndarray:
    x = np.exp(rng.normal(math.log(median), sigma, size=n))
    return np.clip(np.rint(x), lo, hi).astype(np.int32)


def config2(seed: int = 0, num_seqs: int = 256) -> PagedBatch:
    """Config 2: decode at scale.  256 sequences, context lognormal (median 1024, sigma 0.8)
    clipped to [16, 4096], 32 q heads / 8 KV heads, D 128, BS 16, bf16.  The block pool holds the
    batch plus 5% slack, handed out from a shuffled free list; each sequence's newest token is
    written by reshape_and_cache before attention reads it."""
    rng = np.random.default_rng(seed)
    ctx = lognormal_contexts(rng, num_seqs, 1024.0, 0.8, 16, 4096)
    tables, total, free = _assign_blocks(rng, ctx, 16, 0.05, shuffled=True)
    return PagedBatch("config2", 32, 8, 128, 16, total, ctx - 1, np.ones(num_seqs, np.int32),
                      tables, 1.0 / math.sqrt(128.0), "bf16", seed, free)


def config3(seed: int = 0, num_prefill: int = 16, num_decode: int = 240) -> PagedBatch:
    """Config 3: mixed ragged step.  16 prefill chunks of U[128,2048] new tokens on top of
    U[0,2048] cached tokens (causal), packed with 240 decodes (context lognormal, median 1024),
    32/8 heads, D 128, BS 16, bf16."""
    rng = np.random.default_rng(seed)
    chunk = rng.integers(128, 2049, size=num_prefill).astype(np.int32)
    prior = rng.integers(0, 2049, size=num_prefill).astype(np.int32)
    dctx = lognormal_contexts(rng, num_decode, 1024.0, 0.8, 16, 4096)
    starts = np.concatenate([prior, dctx - 1]).astype(np.int32)
    counts = np.concatenate([chunk, np.ones(num_decode, np.int32)]).astype(np.int32)
    tables, total, free = _assign_blocks(rng, starts + counts, 16, 0.05, shuffled=True)
    return PagedBatch("config3", 32, 8, 128, 16, total, starts, counts, tables,
                      1.0 / math.sqrt(128.0), "bf16", seed, free)


def custom(seed: int, context_lens, new_token_counts, num_query_heads: int, num_kv_heads: int,
           head_dim: int, block_size: int, dtype: str = "bf16", slack: float = 0.25,
           shuffled: bool = True, scale: float | None = None) -> PagedBatch:
    """Arbitrary ragged batch for parity tests (context_lens include the new tokens)."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(context_lens, np.int32)
    cnt = np.asarray(new_token_counts, np.int32)
    tables, total, free = _assign_blocks(rng, ctx, block_size, slack, shuffled)
    return PagedBatch("custom", num_query_heads, num_kv_heads, head_dim, block_size, total,
                      ctx - cnt, cnt, tables,
                      scale if scale is not None else 1.0 / math.sqrt(head_dim), dtype, seed,
                      free)


def config4_requests(num: int, rate: float = 20.0, vocab: int = 32000, seed: int = 4,
                     total: int = 2000):
    """Config 4's request stream: `total` requests with Poisson arrivals at `rate` per second
    (first at t=0), prompt lengths lognormal(median 512, sigma 0.8) clipped to [1, 4096] of
    uniform token ids, output lengths uniform in [64, 512].  Returns (arrival times (total,),
    prompts of the first `num` requests, output lengths (total,))."""
    rng = np.random.default_rng(seed)
    gaps = rng.exponential(1.0 / rate, size=total)
    arrivals = np.cumsum(gaps) - gaps[0]
    plens = np.clip(np.rint(np.exp(rng.normal(math.log(512), 0.8, size=total))), 1,
                    4096).astype(int)
    olens = rng.integers(64, 513, size=total)
    prompts = [rng.integers(0, vocab, size=int(L)).tolist() for L in plens[:num]]
    return arrivals, prompts, olens
