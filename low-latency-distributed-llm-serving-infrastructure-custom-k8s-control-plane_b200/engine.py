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

Tensor parallel runs: every rank runs the same engine on the same requests; scheduling is
deterministic, the sampled tokens are identical on all ranks (vocab-parallel greedy over
all-reduced hidden states), and rank 0's arrival decisions are broadcast each step, so every rank
takes the same collective steps in the same order.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from enum import Enum
from typing import Dict, List, Optional

import torch

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
        i = 0
        while i < len(self.waiting):
            seq = self.waiting[i]
            need = (seq.total_len + self.block_size - 1) // self.block_size
            # max_batch_size bounds the decode group only (scheduler.py:94-96); admission is
            # limited by free blocks and the batched-token budget (:128-138)
            if (need > self.allocator.get_num_free_blocks()
                    or budget + seq.total_len > self.max_num_batched_tokens):
                ignored.append(seq)
                i += 1
                continue
            self.waiting.pop(i)
            self.kv.allocate_prefix_blocks(seq)
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


class Engine:
    def __init__(self, model, kv_cache_manager: PagedKVCacheManager, scheduler: Scheduler) -> None:
        self.model = model
        self.kv = kv_cache_manager
        self.scheduler = scheduler
        self.device = kv_cache_manager.torch_device
        self.seq_counter = 0
        self.scale = 1.0 / (model.shape.head_dim ** 0.5)
        self.steps = 0
        self.tokens_generated = 0
        self.prefill_tokens = 0

    def add_request(self, prompt_token_ids: List[int], max_tokens: int = 128,
                    eos_token_id: Optional[int] = None, arrival: float = 0.0) -> Sequence:
        self.seq_counter += 1
        seq = Sequence(self.seq_counter, prompt_token_ids, max_tokens, eos_token_id)
        seq.arrival = arrival
        self.scheduler.add_sequence(seq)
        return seq

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished_sequences()

    def step(self) -> Dict[str, List[Sequence]]:
        out = self.scheduler.schedule()
        seqs = out.scheduled_prefills + out.scheduled_decodes
        if not seqs:
            return {"finished": [], "running": []}
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

        def attend(layer, q, k, v):
            paged_ops.reshape_and_cache(k, v, kc, vc, slots, layer)
            if is_decode:
                return paged_ops.paged_decode(q, kc, vc, layer, bt, ctx, scale, max_ctx)
            return paged_ops.paged_prefill(q, kc, vc, layer, bt, cu, ctx, scale, max_q, max_ctx)

        with torch.inference_mode():
            hidden = self.model.forward(input_ids, md["position_ids"], attend)
            last = hidden.index_select(0, cu[1:] - 1)
            next_tokens = self.model.greedy(last).cpu().tolist()
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


def build_engine(shape, total_blocks: int, block_size: int = 16, rank: int = 0, world: int = 1,
                 device=None, dtype=torch.bfloat16, seed: int = 0, max_batch_size: int = 256,
                 max_num_batched_tokens: int = 16384, max_model_len: int = 8192,
                 full_init: bool = False, group=None) -> Engine:
    from .model import TPLlama
    device = torch.device(device or "cuda")
    model = TPLlama(shape, rank, world, device, dtype, seed, full_init=full_init, group=group)
    max_blocks = (max_model_len + block_size - 1) // block_size
    kv = PagedKVCacheManager(total_blocks, block_size, shape.num_kv_heads // world,
                             shape.head_dim, dtype=dtype, num_layers=shape.num_layers,
                             device=device, max_seqs=max(16 * max_batch_size, 4096),
                             max_blocks_per_seq=max_blocks)
    sched = Scheduler(kv, max_batch_size, max_num_batched_tokens, max_model_len)
    return Engine(model, kv, sched)
