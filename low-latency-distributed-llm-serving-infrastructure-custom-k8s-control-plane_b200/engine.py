"""Continuous-batching engine over the B200 path (BASELINE configs 4 and 5).

Scheduling policy and engine API follow the reference:
  * ``Sequence``  -- app/scheduler/sequence.py:14-55 (tokens, status, max_tokens / EOS finish);
  * ``Scheduler`` -- app/scheduler/scheduler.py:15-165: running sequences decode first; a
    sequence that needs a new block when none is free is preempted (blocks freed, re-queued at the
    front for recompute, :100-112); waiting sequences are admitted whole, in order, while blocks
    and the batched-token budget allow (:124-145);
  * ``Engine``    -- app/engine/llm_engine.py:20-260 (add_request / step /
    has_unfinished_requests).
Differences that are the point of the rebuild: block allocation goes to the device block pool
(K5), the step's metadata is built on the device (K4), the prefill and decode groups run as one
mixed forward, and sampling is a greedy argmax on the device with one host read per step
(instead of one ``int(argmax)`` per sequence, llm_engine.py:200-204).

Pure decode steps replay a CUDA graph captured per batch-size bucket (step metadata, the whole
model forward with the fused rotary/cache-write and decode kernels, greedy sampling): the host
work per step is the scheduler, one pool flush, two small pinned copies and the token read-back.
Rows that pad a batch up to its bucket repeat the shortest real sequence; they recompute its
token and write identical K/V bytes to the same slot, and their outputs are dropped.

Tensor parallel runs: every rank runs the same engine on the same requests; scheduling is
deterministic, the sampled tokens are identical on all ranks (vocab-parallel greedy over
all-reduced hidden states), and rank 0's arrival decisions are broadcast each step, so every rank
takes the same collective steps in the same order.
"""
from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass
from enum import Enum
from typing import Dict, List, Optional

import torch

from . import _native as N
from . import paged_ops
from .kv_cache import PagedKVCacheManager


class SequenceStatus(Enum):
    WAITING = "WAITING"
    RUNNING = "RUNNING"
    FINISHED = "FINISHED"


class Sequence:
    def __init__(self, seq_id: int, prompt_token_ids: List[int], max_tokens: int = 128,
                 eos_token_id: Optional[int] = None) -> None:
        if not prompt_token_ids:
            raise ValueError(f"Sequence {seq_id}: Prompt and prompt_token_ids cannot be both empty.")
        self.seq_id = seq_id
        self.prompt_token_ids = list(prompt_token_ids)
        self.output_token_ids: List[int] = []
        self.max_tokens = max_tokens
        self.eos_token_id = eos_token_id
        self.status = SequenceStatus.WAITING
        self.block_table = None
        self.arrival = 0.0
        self.first_token_time: Optional[float] = None
        self.finish_time: Optional[float] = None

    @property
    def total_len(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    def get_token_ids(self) -> List[int]:
        return self.prompt_token_ids + self.output_token_ids

    def append_token(self, token_id: int) -> None:
        self.output_token_ids.append(token_id)
        if token_id == self.eos_token_id or len(self.output_token_ids) >= self.max_tokens:
            self.status = SequenceStatus.FINISHED

    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED


@dataclass
class SchedulerOutputs:
    scheduled_prefills: List[Sequence]
    scheduled_decodes: List[Sequence]
    ignored_sequences: List[Sequence]


class Scheduler:
    def __init__(self, kv_cache_manager: PagedKVCacheManager, max_batch_size: int = 256,
                 max_num_batched_tokens: int = 16384, max_model_len: int = 8192) -> None:
        self.kv = kv_cache_manager
        self.allocator = kv_cache_manager.get_allocator()
        self.block_size = kv_cache_manager.block_size
        self.max_batch_size = max_batch_size
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.preemption_count = 0
        self.waiting: List[Sequence] = []
        self.running: List[Sequence] = []

    def add_sequence(self, seq: Sequence) -> None:
        need = seq.total_len + seq.max_tokens
        if need > self.max_model_len:
            raise ValueError(f"Sequence {seq.seq_id} exceeds max_model_len: "
                             f"prompt+max_tokens ({need}) > {self.max_model_len}")
        blocks = (need + self.block_size - 1) // self.block_size
        if blocks > self.allocator.get_total_blocks():
            raise ValueError(f"Sequence {seq.seq_id} requires {blocks} blocks but the KV cache "
                             f"pool has only {self.allocator.get_total_blocks()} blocks")
        # the device pool's table rows have a fixed width (a host allocator has none)
        row = getattr(self.kv, "max_blocks_per_seq", None)
        if row is not None and blocks > row:
            raise ValueError(f"Sequence {seq.seq_id} requires {blocks} blocks but a block table "
                             f"row holds {row}")
        self.waiting.append(seq)

    def has_unfinished_sequences(self) -> bool:
        return bool(self.waiting or self.running)

    def schedule(self) -> SchedulerOutputs:
        decodes: List[Sequence] = []
        prefills: List[Sequence] = []
        active: List[Sequence] = []
        for seq in self.running:
            if seq.is_finished():
                self.kv.free_sequence(seq)
                continue
            if len(decodes) >= self.max_batch_size:
                active.append(seq)
                continue
            tokens = seq.block_table.get_tokens_count() if seq.block_table is not None else 0
            needs_block = tokens > 0 and tokens % self.block_size == 0
            if needs_block and self.allocator.get_num_free_blocks() < 1:
                seq.status = SequenceStatus.WAITING
                self.kv.free_sequence(seq)
                self.preemption_count += 1
                self.waiting.insert(0, seq)
                continue
            if seq.block_table is not None:
                self.kv.allocate_slot_for_next_token(seq)
            active.append(seq)
            decodes.append(seq)
        self.running = active
        budget = len(decodes)
        ignored: List[Sequence] = []
        # the device pool has a fixed number of sequence slots (table rows): a sequence waits for
        # one like it waits for blocks (a host allocator has no such limit)
        free_slots = getattr(self.kv, "num_free_sequence_slots", None)
        slots = free_slots() if free_slots is not None else None
        i = 0
        while i < len(self.waiting):
            seq = self.waiting[i]
            need = (seq.total_len + self.block_size - 1) // self.block_size
            # max_batch_size bounds the decode group only (scheduler.py:94-96); admission is
            # limited by free blocks and the batched-token budget (:128-138)
            if (need > self.allocator.get_num_free_blocks()
                    or budget + seq.total_len > self.max_num_batched_tokens
                    or slots == 0):
                ignored.append(seq)
                i += 1
                continue
            self.waiting.pop(i)
            self.kv.allocate_prefix_blocks(seq)
            if slots is not None:
                slots -= 1
            seq.status = SequenceStatus.RUNNING
            self.running.append(seq)
            prefills.append(seq)
            budget += seq.total_len
        return SchedulerOutputs(prefills, decodes, ignored)

    def free_sequence(self, seq: Sequence) -> None:
        self.kv.free_sequence(seq)
        seq.status = SequenceStatus.FINISHED
        if seq in self.running:
            self.running.remove(seq)
        if seq in self.waiting:
            self.waiting.remove(seq)


# batch-size buckets of the captured decode graphs
_GRAPH_BUCKETS = [1, 2, 4] + list(range(8, 257, 8)) + list(range(288, 2049, 32))


def graph_decode_workspace_bytes(num_query_heads: int, key_cache: torch.Tensor,
                                 value_cache: torch.Tensor, max_blocks_per_seq: int,
                                 ctx_bound: int, max_rows: int, scale: float) -> int:
    """Bytes of one decode workspace that serves every captured batch bucket up to `max_rows`
    rows at the context bound.  The decode's split plan depends on the batch size -- a smaller
    batch gets shorter splits so that every SM still has work -- so a bucket below the largest
    can need more scratch than the largest one: the maximum over all buckets is taken.  Only
    shapes and strides are read (no kernel runs), so this works on the host as well."""
    L = N.lib()
    D = key_cache.shape[-1]
    dev = key_cache.device
    q = torch.empty((max_rows, num_query_heads, D), dtype=key_cache.dtype, device=dev)
    bt = torch.empty((max_rows, max_blocks_per_seq), dtype=torch.int32, device=dev)
    ctx = torch.empty(max_rows, dtype=torch.int32, device=dev)
    need = 256
    for rows in _GRAPH_BUCKETS:
        if rows > max_rows:
            break
        p = paged_ops.decode_params(q[:rows], key_cache, value_cache, 0, bt[:rows], ctx[:rows],
                                    scale, q[:rows], ctx_bound)
        need = max(need, int(L.b200_paged_decode_workspace_bytes(ctypes.byref(p))))
    return need


class _DecodeGraph:
    """Static buffers and the captured graph of one decode bucket (``rows`` sequences)."""

    def __init__(self, rows: int, device: torch.device) -> None:
        self.rows = rows
        # rows of (sequence slot, start position, new-token count) and the input token ids
        self.h_meta = torch.zeros((3, rows), dtype=torch.int32).pin_memory()
        self.h_ids = torch.zeros(rows, dtype=torch.int64).pin_memory()
        self.h_meta_np = self.h_meta.numpy()
        self.h_ids_np = self.h_ids.numpy()
        self.d_meta = torch.zeros((3, rows), dtype=torch.int32, device=device)
        self.d_ids = torch.zeros(rows, dtype=torch.int64, device=device)
        self.graph = torch.cuda.CUDAGraph()
        self.out: Optional[torch.Tensor] = None


class Engine:
    def __init__(self, model, kv_cache_manager: PagedKVCacheManager, scheduler: Scheduler,
                 cuda_graphs: bool = True) -> None:
        self.model = model
        self.kv = kv_cache_manager
        self.scheduler = scheduler
        self.device = kv_cache_manager.torch_device
        self.seq_counter = 0
        self.scale = 1.0 / (model.shape.head_dim ** 0.5)
        self.steps = 0
        self.tokens_generated = 0
        self.prefill_tokens = 0
        self.graph_steps = 0
        self.cuda_graphs = cuda_graphs
        self._graphs: Dict[int, _DecodeGraph] = {}
        self._graph_pool = None
        self._graph_ws: Optional[torch.Tensor] = None
        # decode graphs size their split plan and workspace for this context bound
        self._ctx_bound = int(scheduler.max_model_len)
        self._max_rows = next((b for b in _GRAPH_BUCKETS if b >= scheduler.max_batch_size),
                              _GRAPH_BUCKETS[-1])

    def add_request(self, prompt_token_ids: List[int], max_tokens: int = 128,
                    eos_token_id: Optional[int] = None, arrival: float = 0.0) -> Sequence:
        self.seq_counter += 1
        seq = Sequence(self.seq_counter, prompt_token_ids, max_tokens, eos_token_id)
        seq.arrival = arrival
        self.scheduler.add_sequence(seq)
        return seq

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished_sequences()

    def release_graphs(self) -> None:
        """Drop the captured decode graphs.  Under tensor parallelism they hold NCCL calls, and
        a process group must not be destroyed while such a graph is alive (its teardown then
        waits forever): call this before ``destroy_process_group``.  Decoding afterwards simply
        captures again."""
        torch.cuda.synchronize(self.device)
        for g in self._graphs.values():
            g.graph.reset()
            g.out = None
        self._graphs.clear()
        self._graph_pool = None
        self._graph_ws = None

    def step(self) -> Dict[str, List[Sequence]]:
        """One continuous-batching step.  NVTX ranges mark its phases on a timeline profile:
        ``engine.step`` around it, ``schedule``, then ``decode_graph`` (replay of a captured
        decode step) or ``eager_step`` (prefill or mixed batch); the C library adds one range per
        kernel-launching call inside them."""
        nvtx = torch.cuda.nvtx
        nvtx.range_push("engine.step")
        try:
            return self._step(nvtx)
        finally:
            nvtx.range_pop()

    def _step(self, nvtx) -> Dict[str, List[Sequence]]:
        nvtx.range_push("schedule")
        out = self.scheduler.schedule()
        nvtx.range_pop()
        seqs = out.scheduled_prefills + out.scheduled_decodes
        if not seqs:
            return {"finished": [], "running": []}
        next_tokens = None
        if self.cuda_graphs and not out.scheduled_prefills:
            nvtx.range_push("decode_graph")
            next_tokens = self._graph_decode(out.scheduled_decodes)
            nvtx.range_pop()
        if next_tokens is None:
            nvtx.range_push("eager_step")
            next_tokens = self._eager_step(out)
            nvtx.range_pop()
        now = time.perf_counter()
        for s, t in zip(seqs, next_tokens):
            if s.first_token_time is None:
                s.first_token_time = now
            s.append_token(int(t))
        self.tokens_generated += len(seqs)
        self.steps += 1
        finished = [s for s in seqs if s.is_finished()]
        for s in finished:
            s.finish_time = now
            self.scheduler.free_sequence(s)
        return {"finished": finished, "running": [s for s in seqs if not s.is_finished()]}

    # ---- eager step (prefill or mixed batches) -------------------------------------------------
    def _eager_step(self, out: SchedulerOutputs) -> List[int]:
        seqs = out.scheduled_prefills + out.scheduled_decodes
        ids: List[int] = []
        starts: List[int] = []
        counts: List[int] = []
        for s in out.scheduled_prefills:
            toks = s.get_token_ids()  # whole prompt (and earlier outputs after a preemption)
            ids.extend(toks)
            starts.append(0)
            counts.append(len(toks))
        for s in out.scheduled_decodes:
            ids.append(s.output_token_ids[-1] if s.output_token_ids else s.prompt_token_ids[-1])
            starts.append(s.block_table.get_tokens_count() - 1)
            counts.append(1)
        self.prefill_tokens += sum(counts) - len(out.scheduled_decodes)
        dev = self.device
        input_ids = torch.tensor(ids, dtype=torch.long).pin_memory().to(dev, non_blocking=True)
        md = self.kv.step_metadata(seqs, starts, counts)
        is_decode = not out.scheduled_prefills
        max_q = max(counts)
        max_ctx = max(s + c for s, c in zip(starts, counts))
        kc, vc = self.kv.key_cache, self.kv.value_cache
        bt, ctx, cu = md["block_tables"], md["context_lens"], md["cu_seqlens"]
        slots = md["slot_mapping"]
        scale = self.scale
        positions = md["position_ids"]
        inv_freq = self.model.inv_freq
        hq = self.model.hq

        def attend_qkv(layer, qkv):
            # rotary + cache write in one kernel, then attention over the paged cache
            q = paged_ops.rope_reshape_and_cache(qkv, positions, inv_freq, hq, kc, vc, slots,
                                                 layer)
            if is_decode:
                return paged_ops.paged_decode(q, kc, vc, layer, bt, ctx, scale, max_ctx)
            return paged_ops.paged_prefill(q, kc, vc, layer, bt, cu, ctx, scale, max_q, max_ctx)

        with torch.inference_mode():
            hidden = self.model.forward(input_ids, positions, attend_qkv=attend_qkv)
            last = hidden.index_select(0, cu[1:] - 1)
            return self.model.greedy(last).cpu().tolist()

    # ---- captured decode step --------------------------------------------------------------------
    def _decode_body(self, g: _DecodeGraph) -> torch.Tensor:
        """One decode step over g's static inputs: K4 metadata, forward, greedy (capturable: no
        host synchronisation, fixed shapes and pointers)."""
        pool = self.kv.pool
        md = pool.build_step_metadata(g.d_meta[0], g.d_meta[1], g.d_meta[2], g.rows,
                                      bt_stride=pool.max_blocks_per_seq)
        positions, slots = md["position_ids"], md["slot_mapping"]
        bt, ctx = md["block_tables"], md["context_lens"]
        kc, vc = self.kv.key_cache, self.kv.value_cache
        inv_freq, hq, scale = self.model.inv_freq, self.model.hq, self.scale
        bound, ws = self._ctx_bound, self._graph_ws

        def attend_qkv(layer, qkv):
            q = paged_ops.rope_reshape_and_cache(qkv, positions, inv_freq, hq, kc, vc, slots,
                                                 layer)
            return paged_ops.paged_decode(q, kc, vc, layer, bt, ctx, scale, bound, workspace=ws)

        hidden = self.model.forward(g.d_ids, positions, attend_qkv=attend_qkv)
        return self.model.greedy(hidden)

    def _graph_workspace(self) -> torch.Tensor:
        """Decode workspace shared by every captured graph (graphs never run concurrently), sized
        once for every bucket at the context bound so no capture ever reallocates it."""
        if self._graph_ws is None:
            need = graph_decode_workspace_bytes(self.model.hq, self.kv.key_cache,
                                                self.kv.value_cache,
                                                self.kv.pool.max_blocks_per_seq, self._ctx_bound,
                                                self._max_rows, self.scale)
            self._graph_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._graph_ws

    def _graph_decode(self, decodes: List[Sequence]) -> Optional[List[int]]:
        B = len(decodes)
        rows = next((b for b in _GRAPH_BUCKETS if b >= B), None)
        if rows is None or rows > self._max_rows:
            return None
        g = self._graphs.get(rows)
        fresh = g is None
        if fresh:
            g = _DecodeGraph(rows, self.device)
        tokens = [s.block_table.get_tokens_count() for s in decodes]
        donor = min(range(B), key=lambda i: tokens[i])  # pad rows repeat the shortest sequence
        m, ids = g.h_meta_np, g.h_ids_np
        for i, s in enumerate(decodes):
            m[0, i] = s.block_table.slot
            m[1, i] = tokens[i] - 1
            ids[i] = s.output_token_ids[-1] if s.output_token_ids else s.prompt_token_ids[-1]
        m[0, B:] = m[0, donor]
        m[1, B:] = m[1, donor]
        m[2, :] = 1
        ids[B:] = ids[donor]
        self.kv.pool.flush()  # this step's slot allocations, before the metadata kernel reads them
        g.d_meta.copy_(g.h_meta, non_blocking=True)
        g.d_ids.copy_(g.h_ids, non_blocking=True)
        if fresh:
            self._capture(g)
        g.graph.replay()
        self.graph_steps += 1
        return g.out[:B].cpu().tolist()

    def _capture(self, g: _DecodeGraph) -> None:
        """Warm up on a side stream, then capture.  The warm-up runs execute this step's decode on
        its real inputs; repeating it is idempotent (same K/V bytes to the same slots) and the
        replay that follows produces the step's tokens."""
        self._graph_workspace()
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side), torch.inference_mode():
            for _ in range(2):
                self._decode_body(g)
        cur.wait_stream(side)
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        with torch.inference_mode(), torch.cuda.graph(g.graph, pool=self._graph_pool):
            g.out = self._decode_body(g)
        self._graphs[g.rows] = g


def build_engine(shape, total_blocks: int, block_size: int = 16, rank: int = 0, world: int = 1,
                 device=None, dtype=torch.bfloat16, seed: int = 0, max_batch_size: int = 256,
                 max_num_batched_tokens: int = 16384, max_model_len: int = 8192,
                 full_init: bool = False, group=None, cuda_graphs: bool = True) -> Engine:
    from .model import TPLlama
    device = torch.device(device or "cuda")
    model = TPLlama(shape, rank, world, device, dtype, seed, full_init=full_init, group=group)
    max_blocks = (max_model_len + block_size - 1) // block_size
    kv = PagedKVCacheManager(total_blocks, block_size, shape.num_kv_heads // world,
                             shape.head_dim, dtype=dtype, num_layers=shape.num_layers,
                             device=device, max_seqs=max(16 * max_batch_size, 4096),
                             max_blocks_per_seq=max_blocks)
    sched = Scheduler(kv, max_batch_size, max_num_batched_tokens, max_model_len)
    return Engine(model, kv, sched, cuda_graphs=cuda_graphs)
