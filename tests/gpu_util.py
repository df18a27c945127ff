"""Shared helpers of the GPU parity tests: device batches from the seeded workloads, and the CPU
oracle run on the same values (bf16/f16 upcast exactly to fp32)."""
import numpy as np
import torch


def device_batch(b, dtype, seed=0, device="cuda", num_layers=1, layer=0, scale_values=1.0):
    """Caches (L, NB, BS, Hkv, D), queries (Ntok, Hq, D), block tables and lengths on `device`."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    shape = (num_layers, b.total_blocks, b.block_size, b.num_kv_heads, b.head_dim)
    kc = (torch.randn(shape, generator=g, device=device) * scale_values).to(dtype)
    vc = (torch.randn(shape, generator=g, device=device) * scale_values).to(dtype)
    q = (torch.randn((b.num_tokens, b.num_query_heads, b.head_dim), generator=g, device=device)
         * scale_values).to(dtype)
    bt = torch.from_numpy(b.block_tables()).to(device)
    ctx = torch.from_numpy(b.context_lens.astype(np.int32)).to(device)
    return q, kc, vc, bt, ctx


def oracle_ragged(oracle, b, q, kc, vc, layer=0):
    """fp32 CPU oracle on the exact values of the device tensors."""
    bt = np.maximum(b.block_tables(), 0)
    return oracle.paged_ragged(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                               vc.float().cpu().numpy(), layer, bt, b.start_positions,
                               b.new_token_counts, b.scale)


def max_rel(out: np.ndarray, ref: np.ndarray) -> float:
    """max |out - ref| relative to max |ref| (the fp32 parity measure)."""
    return float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))
