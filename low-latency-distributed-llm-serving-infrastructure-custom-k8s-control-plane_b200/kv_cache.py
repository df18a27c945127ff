"""Device version of the reference's KV-cache manager (app/memory/manager.py:12-333).

Same class name, constructor, methods and errors as ``PagedKVCacheManager``, so the reference's
Scheduler and engine drive it unchanged; underneath, block allocation goes to the device block
pool (K5), slot mappings and block tables come from the metadata kernels (K4) and the KV write is
reshape_and_cache (K2).  The caches are ``(L, NB, BS, Hkv, D)`` tensors on the GPU
(app/memory/strategies.py:110-115).
"""
from __future__ import annotations

from typing import List, Optional, Tuple, Union

import torch

from . import paged_ops
from .block_manager import DeviceBlockPool


class DeviceSequenceTable:
    """Stands in for ``seq.block_table``: the sequence's row in the device block pool.  Exposes the
    two reads the reference's scheduler and engine make (get_tokens_count, get_physical_blocks)."""

    def __init__(self, pool: DeviceBlockPool, slot: int) -> None:
        self.pool = pool
        self.slot = slot

    def get_tokens_count(self) -> int:
        return self.pool.tokens(self.slot)

    def get_physical_blocks(self) -> List[int]:
        self.pool.flush()
        return self.pool.table(self.slot)

    def append_token(self) -> None:
        self.pool.append_tokens(self.slot, 1)

    def release(self) -> None:
        self.pool.release(self.slot)


class PagedKVCacheManager:
    @classmethod
    def from_model_config(cls, config, total_blocks: int, block_size: int,
                          total_cpu_blocks: int = 32, dtype: torch.dtype = torch.bfloat16,
                          device: Optional[Union[str, torch.device]] = None,
                          strategy=None, max_seqs: int = 1024,
                          max_blocks_per_seq: Optional[int] = None) -> "PagedKVCacheManager":
        num_attention_heads = config.num_attention_heads
        num_kv_heads = getattr(config, "num_key_value_heads", num_attention_heads)
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // num_attention_heads
        return cls(total_blocks=total_blocks, block_size=block_size, num_heads=num_kv_heads,
                   head_dim=head_dim, total_cpu_blocks=total_cpu_blocks, dtype=dtype,
                   num_layers=config.num_hidden_layers, device=device, max_seqs=max_seqs,
                   max_blocks_per_seq=max_blocks_per_seq)

    def __init__(self, total_blocks: int, block_size: int, num_heads: int, head_dim: int,
                 total_cpu_blocks: int = 32, dtype: torch.dtype = torch.bfloat16,
                 num_layers: int = 1, device: Optional[Union[str, torch.device]] = None,
                 strategy=None, max_seqs: int = 1024,
                 max_blocks_per_seq: Optional[int] = None) -> None:
        dev = torch.device(device or "cuda")
        if dev.type != "cuda":
            raise RuntimeError("the B200 paged KV cache lives in GPU memory (no CPU path)")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.block_size = block_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.num_layers = num_layers
        self.dtype = dtype
        self._device = dev
        self.total_cpu_blocks = total_cpu_blocks
        self.max_blocks_per_seq = int(max_blocks_per_seq or total_blocks)
        self.pool = DeviceBlockPool(total_blocks, block_size, max_seqs, self.max_blocks_per_seq,
                                    dev)
        self.allocator = self.pool
        shape = (num_layers, total_blocks, block_size, num_heads, head_dim)
        self.key_cache = torch.empty(shape, dtype=dtype, device=dev)
        self.value_cache = torch.empty(shape, dtype=dtype, device=dev)
        self._free_slots = list(range(max_seqs - 1, -1, -1))

    @property
    def device(self) -> str:
        return str(self._device)

    @property
    def torch_device(self) -> torch.device:
        return self._device

    def get_allocator(self) -> DeviceBlockPool:
        return self.pool

    def num_free_sequence_slots(self) -> int:
        """Sequence slots (rows of the device block tables) not held by a sequence."""
        return len(self._free_slots)

    # ---- allocation (app/memory/manager.py:82-102) ---------------------------------------
    def init_sequence_table(self, seq) -> None:
        if seq.block_table is None:
            if not self._free_slots:
                raise RuntimeError("no free sequence slot in the device block pool")
            seq.block_table = DeviceSequenceTable(self.pool, self._free_slots.pop())

    def allocate_prefix_blocks(self, seq) -> None:
        self.init_sequence_table(seq)
        needed = seq.total_len - seq.block_table.get_tokens_count()
        if needed > 0:
            self.pool.append_tokens(seq.block_table.slot, needed)

    def allocate_slot_for_next_token(self, seq) -> None:
        assert seq.block_table is not None
        self.pool.append_tokens(seq.block_table.slot, 1)

    def free_sequence(self, seq) -> None:
        if seq.block_table is not None:
            self.pool.release(seq.block_table.slot)
            self._free_slots.append(seq.block_table.slot)
            seq.block_table = None

    # ---- metadata (manager.py:104-128, :236-271) -----------------------------------------
    def _check_ranges(self, sequences, start_tokens, token_counts) -> None:
        if not (len(sequences) == len(start_tokens) == len(token_counts)):
            raise ValueError(
                f"sequences ({len(sequences)}), start_tokens ({len(start_tokens)}) "
                f"and token_counts ({len(token_counts)}) must have the same length")
        for seq, start, count in zip(sequences, start_tokens, token_counts):
            if seq.block_table is None:
                raise ValueError(f"Sequence {seq.seq_id} has no block table")
            if start < 0 or count < 0:
                raise ValueError(f"Sequence {seq.seq_id}: start_token ({start}) and "
                                 f"token_count ({count}) must be non-negative")
            tokens = seq.block_table.get_tokens_count()
            if start + count > tokens:
                raise ValueError(f"Sequence {seq.seq_id}: tokens [{start}, {start + count}) "
                                 f"exceed allocated tokens ({tokens})")

    def step_metadata(self, sequences, start_tokens, token_counts, with_gather_slots=False,
                      bt_stride: Optional[int] = None):
        """K4 over the given sequences (flushes queued pool ops first)."""
        self._check_ranges(sequences, start_tokens, token_counts)
        self.pool.flush()
        dev = self._device
        host = torch.tensor([[s.block_table.slot for s in sequences], list(start_tokens),
                             list(token_counts)], dtype=torch.int32)
        d = host.to(dev, non_blocking=False)
        ntok = int(sum(token_counts))
        nctx = int(sum(s + c for s, c in zip(start_tokens, token_counts)))
        if bt_stride is None:
            bt_stride = max([self.pool.num_blocks(s.block_table.slot) for s in sequences] + [1])
        return self.pool.build_step_metadata(d[0], d[1], d[2], ntok, bt_stride=bt_stride,
                                             with_gather_slots=with_gather_slots,
                                             num_context_tokens=nctx)

    def build_slot_mapping(self, sequences, start_tokens: List[int],
                           token_counts: List[int]) -> torch.Tensor:
        if not sequences:
            self._check_ranges(sequences, start_tokens, token_counts)
            return torch.empty((0,), dtype=torch.long, device=self._device)
        return self.step_metadata(sequences, start_tokens, token_counts)["slot_mapping"]

    def build_block_tables(self, sequences) -> Tuple[torch.Tensor, torch.Tensor]:
        if len(sequences) == 0:
            return (torch.empty((0, 0), dtype=torch.int32, device=self._device),
                    torch.empty((0,), dtype=torch.int32, device=self._device))
        live = [s for s in sequences if s.block_table is not None]
        if len(live) != len(sequences):
            raise ValueError("build_block_tables needs sequences with block tables")
        tokens = [s.block_table.get_tokens_count() for s in sequences]
        md = self.step_metadata(sequences, [0] * len(sequences), tokens)
        return md["block_tables"], md["context_lens"]

    # ---- KV write (manager.py:130-168) ---------------------------------------------------
    def _validate_layer_idx(self, layer_idx: int) -> None:
        if layer_idx < 0 or layer_idx >= self.num_layers:
            raise ValueError(
                f"Layer index {layer_idx} out of range (num_layers={self.num_layers})")

    def _validate_token_tensors(self, keys, values, expected_shape) -> None:
        if keys.shape != values.shape:
            raise ValueError(f"Keys shape {keys.shape} != Values shape {values.shape}")
        if tuple(keys.shape) != tuple(expected_shape):
            raise ValueError(f"Expected keys shape {tuple(expected_shape)}, got {tuple(keys.shape)}")

    def scatter_kv(self, keys: torch.Tensor, values: torch.Tensor,
                   slot_mapping: torch.Tensor) -> None:
        self._validate_token_tensors(
            keys, values, (slot_mapping.numel(), self.num_layers, self.num_heads, self.head_dim))
        for layer_idx in range(self.num_layers):
            self.scatter_layer_kv(layer_idx, keys[:, layer_idx], values[:, layer_idx],
                                  slot_mapping)

    def scatter_layer_kv(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor,
                         slot_mapping: torch.Tensor) -> None:
        self._validate_layer_idx(layer_idx)
        self._validate_token_tensors(keys, values,
                                     (slot_mapping.numel(), self.num_heads, self.head_dim))
        if slot_mapping.numel() == 0:
            return
        dev = self._device
        k = keys.to(device=dev, dtype=self.dtype)
        v = values.to(device=dev, dtype=self.dtype)
        if k.stride(-1) != 1:
            k = k.contiguous()
        if v.stride(-1) != 1:
            v = v.contiguous()
        paged_ops.reshape_and_cache(k, v, self.key_cache, self.value_cache,
                                    slot_mapping.to(device=dev, dtype=torch.int64), layer_idx)

    # ---- compatibility reads (manager.py:170-234); not on the hot path --------------------
    def gather_layer_keys(self, layer_idx: int, slot_indices: torch.Tensor) -> torch.Tensor:
        self._validate_layer_idx(layer_idx)
        return self.key_cache[layer_idx].view(-1, self.num_heads, self.head_dim).index_select(
            0, slot_indices.to(self._device))

    def gather_layer_values(self, layer_idx: int, slot_indices: torch.Tensor) -> torch.Tensor:
        self._validate_layer_idx(layer_idx)
        return self.value_cache[layer_idx].view(-1, self.num_heads, self.head_dim).index_select(
            0, slot_indices.to(self._device))

    def gather_kv_cache(self, seq, read_len: Optional[int] = None):
        """The sequence's first ``read_len`` tokens (default: all it holds) of every layer as
        ``((key, value), ...)`` in the HF past-key-value layout (1, Hkv, read_len, D), gathered
        from its blocks (manager.py:207-234); None without a block table or for read_len <= 0."""
        if seq.block_table is None:
            return None
        blocks = seq.block_table.get_physical_blocks()
        if read_len is None:
            read_len = seq.block_table.get_tokens_count()
        if read_len <= 0:
            return None
        ids = torch.tensor(blocks, dtype=torch.long, device=self._device)
        out = []
        for layer in range(self.num_layers):
            k = self.key_cache[layer].index_select(0, ids).reshape(-1, self.num_heads,
                                                                    self.head_dim)[:read_len]
            v = self.value_cache[layer].index_select(0, ids).reshape(-1, self.num_heads,
                                                                      self.head_dim)[:read_len]
            out.append((k.unsqueeze(0).transpose(1, 2), v.unsqueeze(0).transpose(1, 2)))
        return tuple(out)

    def write_prefix_kv(self, seq, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
        if keys.shape != values.shape:
            raise ValueError(f"Keys shape {keys.shape} != Values shape {values.shape}")
        seq_len = keys.shape[1]
        if seq_len == 0 or seq.block_table is None:
            return torch.empty((0,), dtype=torch.long, device=self._device)
        slot_mapping = self.build_slot_mapping([seq], [0], [seq_len])
        self.scatter_kv(keys.transpose(0, 1), values.transpose(0, 1), slot_mapping)
        return slot_mapping

    def write_single_token_kv(self, seq, key_token: torch.Tensor,
                              value_token: torch.Tensor) -> None:
        if seq.block_table is None:
            raise ValueError(f"Sequence {seq.seq_id} has no block table")
        token_index = seq.block_table.get_tokens_count() - 1
        slot_mapping = self.build_slot_mapping([seq], [token_index], [1])
        self.scatter_kv(key_token.unsqueeze(0), value_token.unsqueeze(0), slot_mapping)

    # ---- prefix sharing (page_allocator.hpp:142-149, :409-424) --------------------------------
    def share_prefix(self, src_seq, dst_seq, num_blocks: int) -> None:
        """``dst_seq`` (no blocks yet) starts with the first ``num_blocks`` blocks of ``src_seq``
        (shared, not copied): its table holds them and it counts num_blocks * block_size
        tokens.  Before either sequence writes into a shared block, call ``copy_on_write``."""
        self.init_sequence_table(dst_seq)
        self.pool.share(dst_seq.block_table.slot, src_seq.block_table.slot, num_blocks)

    def copy_on_write(self, seq, block_indices) -> None:
        """Give ``seq`` private copies of its shared blocks at the given table indices: fresh
        blocks replace them in its table (flushed now) and the K/V of every layer is copied from
        the old blocks on the device, with no host round trip for the block ids."""
        for i in block_indices:
            self.pool.copy_on_write(seq.block_table.slot, int(i))
        self.pool.flush()
        old, new = self.pool.cow_pairs()
        if old.numel():
            paged_ops.copy_blocks(self.key_cache, self.value_cache, self.key_cache,
                                  self.value_cache, old, new, device=self._device)

    # ---- block copies (strategies.py:117-122) -------------------------------------------------
    def copy_blocks(self, src_blocks, dst_blocks) -> None:
        """Copy device blocks ``src_blocks[i] -> dst_blocks[i]`` (every layer, K and V) -- the
        copy a caller makes before writing a block it shares with another sequence
        (PageAllocator::share_block / SequenceBlockTable::replace_block,
        csrc/include/page_allocator.hpp:142-149, :416-424).  Asynchronous on the current stream."""
        paged_ops.copy_blocks(self.key_cache, self.value_cache, self.key_cache, self.value_cache,
                              src_blocks, dst_blocks, device=self._device)


class HostSwapSpace:
    """Page-locked host blocks with the device cache's per-block layout: the swap space behind
    PageAllocator::swap_out / swap_in (csrc/include/page_allocator.hpp:179-241), which keep only
    the bookkeeping of which device block went to which host block.  The data moves with one
    kernel per call (K6), the device reading or writing the pinned host memory directly over the
    host link; calls are asynchronous on the current stream of the cache's device."""

    def __init__(self, manager: PagedKVCacheManager, num_blocks: int) -> None:
        L, _, BS, H, D = manager.key_cache.shape
        shape = (L, int(num_blocks), BS, H, D)
        self.manager = manager
        self.key_cache = torch.empty(shape, dtype=manager.dtype, pin_memory=True)
        self.value_cache = torch.empty(shape, dtype=manager.dtype, pin_memory=True)

    def swap_out(self, device_blocks, host_blocks) -> None:
        """Device block ``device_blocks[i]`` -> host block ``host_blocks[i]``."""
        m = self.manager
        paged_ops.copy_blocks(m.key_cache, m.value_cache, self.key_cache, self.value_cache,
                              device_blocks, host_blocks, device=m.torch_device)

    def swap_in(self, host_blocks, device_blocks) -> None:
        """Host block ``host_blocks[i]`` -> device block ``device_blocks[i]``."""
        m = self.manager
        paged_ops.copy_blocks(self.key_cache, self.value_cache, m.key_cache, m.value_cache,
                              host_blocks, device_blocks, device=m.torch_device)

    def sync(self) -> None:
        torch.cuda.current_stream(self.manager.torch_device).synchronize()


class CudaKVCacheStrategy:
    """The reference's CUDA cache strategy (app/memory/strategies.py:100-129) over this
    library: same methods; ``copy_blocks`` moves block ``bid`` of every layer for each id in
    ``physical_blocks`` with one kernel instead of one ``copy_`` per block.  Block ids index the
    block dimension (dim 1) of the (L, NB, BS, Hkv, D) layout."""

    def __init__(self, device_id: int = 0) -> None:
        self._device = torch.device(f"cuda:{device_id}")

    @property
    def device(self) -> torch.device:
        return self._device

    def allocate_cache(self, total_blocks, block_size, num_layers, num_heads, head_dim, dtype):
        shape = (num_layers, total_blocks, block_size, num_heads, head_dim)
        return (torch.empty(shape, dtype=dtype, device=self._device),
                torch.empty(shape, dtype=dtype, device=self._device))

    def copy_blocks(self, src_cache: torch.Tensor, dst_cache: torch.Tensor,
                    physical_blocks) -> None:
        paged_ops.copy_blocks(src_cache, None, dst_cache, None, physical_blocks,
                              physical_blocks, device=self._device)
        self.sync()

    def sync(self) -> None:
        torch.cuda.current_stream(self._device).synchronize()

    @property
    def requires_copy_on_swap(self) -> bool:
        return True
