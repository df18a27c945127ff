"""GPU parity of the attention kernels against the CPU oracle (which is pinned to the reference's
own kernel by tests/test_oracle.py).  Tolerances from the north-star contract: fp32 paths within
1e-5 relative (max |diff| / max |ref|), bf16/f16 paths within 2e-2 absolute of the fp32 oracle
computed on the same (exactly upcast) values."""
import numpy as np
import pytest
import torch

from gpu_util import device_batch, max_rel, oracle_ragged
from golden_util import ragged

pytestmark = pytest.mark.gpu

FP32_REL = 1e-5
BF16_ABS = 2e-2


@pytest.fixture(scope="module")
def ops(pkg):
    from llm_serving_b200 import paged_ops
    return paged_ops


def test_reference_signature_config1(golden, ops):
    """Config 1 through b200_paged_attention, the status-returning form of the reference-signature
    symbol (the void symbol itself: tests/test_gpu_reference_binding.py)."""
    from config1_inputs import config1_inputs
    b, q, kc, vc, gs, mask = config1_inputs()
    dev = torch.device("cuda")
    out = ops.paged_attention_masked(torch.from_numpy(q).to(dev), torch.from_numpy(kc).to(dev),
                                     torch.from_numpy(vc).to(dev), 0,
                                     torch.from_numpy(gs).to(dev), torch.from_numpy(mask).to(dev),
                                     b.scale)
    ref = golden["config1_out"]
    assert max_rel(out.cpu().numpy(), ref) <= FP32_REL
    assert ops.read_status(dev) == 0


def test_block_table_decode_fp32_config1(golden, ops):
    from config1_inputs import config1_inputs
    b, q, kc, vc, gs, mask = config1_inputs()
    dev = torch.device("cuda")
    qd = torch.from_numpy(q[0].transpose(1, 0, 2).copy()).to(dev)  # (S, Hq, D)
    out = ops.paged_decode(qd, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev), 0,
                           torch.from_numpy(b.block_tables()).to(dev),
                           torch.from_numpy(b.context_lens).to(dev), b.scale,
                           int(b.context_lens.max()))
    assert max_rel(out.cpu().numpy(), golden["config1_out"][0]) <= FP32_REL


def test_golden_cases_masked_and_ragged(golden, ops):
    dev = torch.device("cuda")
    for name in golden["attn_cases"]:
        p = f"attn_{name}_"
        q, kc, vc = golden[p + "q"], golden[p + "k_cache"], golden[p + "v_cache"]
        scale = float(golden[p + "scale"])
        ref = golden[p + "out"]
        out = ops.paged_attention_masked(torch.from_numpy(q).to(dev), torch.from_numpy(kc).to(dev),
                                         torch.from_numpy(vc).to(dev), 1,
                                         torch.from_numpy(golden[p + "gather_slots"]).to(dev),
                                         torch.from_numpy(golden[p + "mask"]).to(dev), scale)
        assert max_rel(out.cpu().numpy(), ref) <= FP32_REL, name
        tables = ragged(golden, p)
        bt = np.full((len(tables), max(len(t) for t in tables)), -1, np.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = t
        counts = golden[p + "counts"]
        ctx = (golden[p + "starts"] + counts).astype(np.int32)
        cu = np.zeros(len(counts) + 1, np.int64)
        cu[1:] = np.cumsum(counts)
        qt = torch.from_numpy(q[0].transpose(1, 0, 2).copy()).to(dev)
        out2 = ops.paged_prefill(qt, torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev), 1,
                                 torch.from_numpy(bt).to(dev), torch.from_numpy(cu).to(dev),
                                 torch.from_numpy(ctx).to(dev), scale, int(counts.max()),
                                 int(ctx.max()))
        assert max_rel(out2.cpu().numpy(), ref[0]) <= FP32_REL, name


def _decode_case(pkg, oracle, ops, b, dtype, seed=0, split=0, layers=1, layer=0):
    lib = pkg._native.lib()
    lib.b200_set_decode_split_tokens(split)
    try:
        q, kc, vc, bt, ctx = device_batch(b, dtype, seed, num_layers=layers)
        out = ops.paged_decode(q, kc, vc, layer, bt, ctx, b.scale, int(b.context_lens.max()))
        torch.cuda.synchronize()
        ref = oracle_ragged(oracle, b, q, kc, vc, layer)
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        err = np.abs(got - ref).max()
        assert err <= BF16_ABS, f"max abs err {err}"
        assert ops.read_status(q.device) == 0
        return err
    finally:
        lib.b200_set_decode_split_tokens(0)


def test_decode_bf16_config2(pkg, oracle, ops):
    """Config 2 (256 sequences, lognormal contexts, GQA 32/8, D 128, bf16): the new token of each
    sequence is written by reshape_and_cache, then decode reads it back through the table."""
    b = pkg.workloads.config2(seed=0)
    q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=3)
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    newk = torch.randn((b.num_seqs, b.num_kv_heads, b.head_dim), generator=g, device="cuda").to(
        torch.bfloat16)
    newv = torch.randn((b.num_seqs, b.num_kv_heads, b.head_dim), generator=g, device="cuda").to(
        torch.bfloat16)
    slots = torch.from_numpy(b.slot_mapping()).cuda()
    ops.reshape_and_cache(newk, newv, kc, vc, slots, 0)
    out = ops.paged_decode(q, kc, vc, 0, bt, ctx, b.scale, int(b.context_lens.max()))
    torch.cuda.synchronize()
    ref = oracle_ragged(oracle, b, q, kc, vc)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= BF16_ABS, err
    assert ops.read_status(q.device) == 0


@pytest.mark.parametrize("hd,bs,hq,hkv,ctx,split", [
    (128, 16, 32, 8, [1, 2, 15, 16, 17, 31, 33, 100, 511, 512, 513, 1000], 0),
    (128, 16, 32, 8, [4096, 3000, 16, 1], 64),       # many splits, last-CTA merge
    (64, 16, 32, 8, [5, 64, 700, 2049], 128),        # config-4 head dim
    (128, 32, 16, 2, [1, 31, 32, 33, 900], 0),       # block size 32, GQA 8
    (128, 8, 8, 8, [1, 7, 8, 9, 250], 0),            # block size 8, MHA
    (128, 16, 32, 2, [17, 400, 1300], 256),          # GQA 16 -> two head chunks
    (64, 64, 4, 1, [63, 64, 65, 1000], 0),           # MQA, block size 64
])
def test_decode_bf16_edge_cases(pkg, oracle, ops, hd, bs, hq, hkv, ctx, split):
    b = pkg.workloads.custom(seed=len(ctx), context_lens=ctx, new_token_counts=[1] * len(ctx),
                             num_query_heads=hq, num_kv_heads=hkv, head_dim=hd, block_size=bs)
    _decode_case(pkg, oracle, ops, b, torch.bfloat16, seed=hd + bs, split=split)


def test_decode_f16_and_layer_offset(pkg, oracle, ops):
    b = pkg.workloads.custom(seed=2, context_lens=[3, 77, 300], new_token_counts=[1, 1, 1],
                             num_query_heads=16, num_kv_heads=4, head_dim=128, block_size=16)
    _decode_case(pkg, oracle, ops, b, torch.float16, seed=5, layers=3, layer=2)


def test_decode_small_head_dims_use_cuda_core_path(pkg, oracle, ops):
    # head_dim 8 / 16 (the reference's unit-test shapes) and block size 4 fall outside the
    # tensor-core tile rules and run on the CUDA-core kernel
    for hd, bs in ((8, 4), (16, 4), (32, 1)):
        b = pkg.workloads.custom(seed=hd, context_lens=[1, 5, 9, 33], new_token_counts=[1] * 4,
                                 num_query_heads=6, num_kv_heads=2, head_dim=hd, block_size=bs)
        _decode_case(pkg, oracle, ops, b, torch.bfloat16, seed=hd)


@pytest.mark.parametrize("hd,bs,hq,hkv,ctx", [
    (64, 16, 12, 12, [1, 4080, 4096, 4097, 5000]),   # 255 / 256 / 257 blocks: one and two passes
    (128, 1, 8, 2, [1, 255, 256, 257, 700]),         # block size 1: a pass every 256 tokens
    (32, 5, 16, 4, [3, 1279, 1280, 1281, 2600]),     # odd block size, GQA 4
    (256, 16, 4, 2, [33, 4100]),                     # head dim 256 (4 warps)
])
def test_decode_fp32_row_kernel_passes(pkg, oracle, ops, hd, bs, hq, hkv, ctx):
    """fp32 caches take the CUDA-core row kernel, which stages a row's block ids 256 at a time:
    contexts just below, at and above a pass boundary, and several passes, against the oracle
    within 1e-5 relative."""
    b = pkg.workloads.custom(seed=hd + bs, context_lens=ctx, new_token_counts=[1] * len(ctx),
                             num_query_heads=hq, num_kv_heads=hkv, head_dim=hd, block_size=bs)
    q, kc, vc, bt, cl = device_batch(b, torch.float32, seed=bs)
    out = ops.paged_decode(q, kc, vc, 0, bt, cl, b.scale, int(b.context_lens.max()))
    ref = oracle_ragged(oracle, b, q, kc, vc)
    assert max_rel(out.cpu().numpy(), ref) <= FP32_REL
    assert ops.read_status(q.device) == 0


def test_prefill_fp32_row_kernel_long_context(pkg, oracle, ops):
    """Ragged fp32 prefill (the row kernel's cu_seqlens form) over prior contexts that cross the
    block-id staging passes."""
    b = pkg.workloads.custom(seed=11, context_lens=[4200, 300, 5000], new_token_counts=[40, 300, 7],
                             num_query_heads=8, num_kv_heads=2, head_dim=64, block_size=16)
    q, kc, vc, bt, cl = device_batch(b, torch.float32, seed=3)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(b.new_token_counts)]).astype(np.int64))
    out = ops.paged_prefill(q, kc, vc, 0, bt, cu.to(q.device), cl, b.scale,
                            int(b.new_token_counts.max()), int(b.context_lens.max()))
    ref = oracle_ragged(oracle, b, q, kc, vc)
    assert max_rel(out.cpu().numpy(), ref) <= FP32_REL
    assert ops.read_status(q.device) == 0


def test_decode_strided_query_and_rows(pkg, oracle, ops):
    """HF hands the query over as a transposed view; the kernels take strides, and query_rows
    places each sequence's row (mixed batches)."""
    b = pkg.workloads.custom(seed=4, context_lens=[40, 1, 600, 129], new_token_counts=[1] * 4,
                             num_query_heads=32, num_kv_heads=8, head_dim=128, block_size=16)
    q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=11)
    qbig = torch.zeros((b.num_seqs * 2, 32, 256), dtype=torch.bfloat16, device="cuda")
    rows = torch.tensor([6, 0, 3, 5], dtype=torch.int32, device="cuda")
    qbig[rows.long(), :, :128] = q
    qv = qbig[:, :, :128]
    out = torch.full((b.num_seqs * 2, 32, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    ops.paged_decode(qv, kc, vc, 0, bt, ctx, b.scale, int(b.context_lens.max()), out=out,
                     query_rows=rows)
    ref = oracle_ragged(oracle, b, q, kc, vc)
    got = out[rows.long()].float().cpu().numpy()
    assert np.abs(got - ref).max() <= BF16_ABS
    untouched = [i for i in range(8) if i not in (6, 0, 3, 5)]
    assert (out[untouched].float() == 7.0).all()


def test_decode_empty_context_writes_zeros(pkg, ops):
    b = pkg.workloads.custom(seed=1, context_lens=[5, 0, 9], new_token_counts=[1, 0, 1],
                             num_query_heads=8, num_kv_heads=2, head_dim=128, block_size=16)
    q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=1)
    q = torch.randn((3, 8, 128), device="cuda").to(torch.bfloat16)
    out = torch.full((3, 8, 128), 3.0, dtype=torch.bfloat16, device="cuda")
    ops.paged_decode(q, kc, vc, 0, bt, ctx, b.scale, 9, out=out)
    assert (out[1] == 0).all()


def test_prefill_mixed_bf16(pkg, oracle, ops):
    """A mixed ragged step (prefill chunks on cached prefixes + decodes), bf16."""
    b = pkg.workloads.custom(seed=6, context_lens=[300, 17, 1, 64, 129, 1000],
                             new_token_counts=[120, 17, 1, 1, 33, 1], num_query_heads=32,
                             num_kv_heads=8, head_dim=128, block_size=16)
    q, kc, vc, bt, ctx = device_batch(b, torch.bfloat16, seed=12)
    cu = torch.from_numpy(b.cu_seqlens()).cuda()
    out = ops.paged_prefill(q, kc, vc, 0, bt, cu, ctx, b.scale,
                            int(b.new_token_counts.max()), int(b.context_lens.max()))
    ref = oracle_ragged(oracle, b, q, kc, vc)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= BF16_ABS


def _prefill_case(pkg, oracle, ops, b, dtype, seed, cuda_cores=False, kernel=1):
    lib = pkg._native.lib()
    lib.b200_set_prefill_cuda_cores(1 if cuda_cores else 0)
    lib.b200_set_prefill_kernel(kernel)
    try:
        q, kc, vc, bt, ctx = device_batch(b, dtype, seed)
        cu = torch.from_numpy(b.cu_seqlens()).cuda()
        out = ops.paged_prefill(q, kc, vc, 0, bt, cu, ctx, b.scale, int(b.new_token_counts.max()),
                                int(b.context_lens.max()))
        torch.cuda.synchronize()
        ref = oracle_ragged(oracle, b, q, kc, vc)
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        err = np.abs(got - ref).max()
        assert err <= BF16_ABS, f"max abs err {err}"
        assert ops.read_status(q.device) == 0
        return got
    finally:
        lib.b200_set_prefill_cuda_cores(0)
        lib.b200_set_prefill_kernel(1)  # the default


@pytest.mark.parametrize("hd,bs,hq,hkv,ctx,cnt", [
    (128, 16, 32, 8, [300, 17, 1, 64, 129, 1000], [120, 17, 1, 1, 33, 1]),   # mixed, GQA 4
    (128, 16, 32, 8, [2125], [2125]),                                       # long fresh prompt
    (128, 16, 32, 8, [64, 65, 63, 127, 128, 129], [64, 1, 63, 30, 128, 2]), # tile edges
    (64, 16, 32, 8, [700, 90, 33], [200, 90, 5]),                           # head_dim 64
    (128, 32, 16, 2, [500, 31, 257], [100, 31, 257]),                       # GQA 8, block 32
    (128, 16, 8, 8, [300, 129], [150, 129]),                                # MHA (128 tokens/tile)
    (128, 16, 32, 16, [260, 40], [260, 7]),                                 # GQA 2
])
@pytest.mark.parametrize("kernel", [0, 1, 2])
def test_prefill_tcgen05_parity(pkg, oracle, ops, hd, bs, hq, hkv, ctx, cnt, kernel):
    b = pkg.workloads.custom(seed=sum(cnt), context_lens=ctx, new_token_counts=cnt,
                             num_query_heads=hq, num_kv_heads=hkv, head_dim=hd, block_size=bs)
    _prefill_case(pkg, oracle, ops, b, torch.bfloat16, seed=hd + hq, kernel=kernel)


def test_prefill_tcgen05_f16_and_agrees_with_cuda_cores(pkg, oracle, ops):
    b = pkg.workloads.custom(seed=8, context_lens=[333, 70, 12], new_token_counts=[100, 70, 1],
                             num_query_heads=32, num_kv_heads=8, head_dim=128, block_size=16)
    _prefill_case(pkg, oracle, ops, b, torch.float16, seed=2)
    tc = _prefill_case(pkg, oracle, ops, b, torch.bfloat16, seed=3)
    cc = _prefill_case(pkg, oracle, ops, b, torch.bfloat16, seed=3, cuda_cores=True)
    assert np.abs(tc - cc).max() <= BF16_ABS


@pytest.mark.parametrize("kernel", [1, 2])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_prefill_poly_exp_modes(pkg, oracle, ops, mode, kernel):
    """The two-tile and the dual-stream kernels with none, a quarter or half of their softmax
    exponentials computed by the cubic on the FMA pipe: same bf16 bound against the oracle
    (ragged chunks on prefixes, GQA 4, D 128 and D 64)."""
    lib = pkg._native.lib()
    lib.b200_set_prefill_poly_exp(mode)
    try:
        for hd, seed in ((128, 31), (64, 32)):
            b = pkg.workloads.custom(seed=seed, context_lens=[700, 129, 1, 260, 2000],
                                     new_token_counts=[300, 129, 1, 77, 513], num_query_heads=32,
                                     num_kv_heads=8, head_dim=hd, block_size=16)
            _prefill_case(pkg, oracle, ops, b, torch.bfloat16, seed=seed, kernel=kernel)
    finally:
        lib.b200_set_prefill_poly_exp(1)  # the default


@pytest.mark.parametrize("kernel", [0, 1, 2])
def test_prefill_config3_subset(pkg, oracle, ops, kernel):
    """4 of config 3's prefill chunks (on their cached prefixes) packed with 16 of its decodes."""
    full = pkg.workloads.config3(seed=0)
    idx = [0, 1, 2, 3] + list(range(16, 32))
    b = pkg.workloads.custom(seed=3, context_lens=full.context_lens[idx],
                             new_token_counts=full.new_token_counts[idx], num_query_heads=32,
                             num_kv_heads=8, head_dim=128, block_size=16)
    _prefill_case(pkg, oracle, ops, b, torch.bfloat16, seed=4, kernel=kernel)


def test_masked_kernel_random_masks(oracle, ops):
    """The reference-signature kernel on arbitrary masks (a fully masked row gives zeros), fp32,
    against the oracle within 1e-5 relative."""
    rng = np.random.default_rng(17)
    hkv, hq, d, bs, NB = 2, 6, 64, 16, 12
    nq, nctx = 9, 150
    kc = rng.standard_normal((2, NB, bs, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((2, NB, bs, hkv, d), dtype=np.float32)
    q = rng.standard_normal((1, hq, nq, d), dtype=np.float32)
    gs = rng.permutation(NB * bs)[:nctx].astype(np.int32)
    mask = (rng.random((1, 1, nq, nctx)) < 0.3).astype(np.uint8)
    mask[0, 0, 4] = 0
    mask[0, 0, 7] = 1
    ref = oracle.paged_attention(q, kc, vc, 1, gs, mask, 0.125)
    dev = torch.device("cuda")
    out = ops.paged_attention_masked(torch.from_numpy(q).to(dev), torch.from_numpy(kc).to(dev),
                                     torch.from_numpy(vc).to(dev), 1, torch.from_numpy(gs).to(dev),
                                     torch.from_numpy(mask).to(dev), 0.125).cpu().numpy()
    assert max_rel(out, ref) <= FP32_REL
    assert not out[0, 4].any()
    assert ops.read_status(dev) == 0


@pytest.mark.parametrize("d,hq,hkv,density", [(32, 4, 4, 0.5), (64, 8, 2, 0.02), (128, 12, 1, 1.0),
                                              (256, 4, 2, 0.3), (64, 16, 4, 0.7)])
def test_masked_kernel_multi_pass(oracle, ops, d, hq, hkv, density):
    """The mask form over contexts longer than one 2048-slot compaction pass (9,000 slots: four
    full passes and a ragged one), every head-dim instantiation (D 32..256), GQA groups of 1 to 12
    (12 = two head chunks per KV head), masks from 2 % to all allowed, a fully masked row, and a
    row whose allowed slots straddle the pass boundaries; fp32, within 1e-5 relative."""
    rng = np.random.default_rng(d + hq + hkv)
    bs, NB, nq, nctx = 16, 600, 5, 9000
    kc = rng.standard_normal((1, NB, bs, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((1, NB, bs, hkv, d), dtype=np.float32)
    q = rng.standard_normal((1, hq, nq, d), dtype=np.float32)
    gs = rng.permutation(NB * bs)[:nctx].astype(np.int32)
    mask = (rng.random((1, 1, nq, nctx)) < density).astype(np.uint8)
    mask[0, 0, 1] = 0
    mask[0, 0, 3] = 0
    mask[0, 0, 3, 4080:4110] = 1
    mask[0, 0, 3, 8180:8200] = 1
    ref = oracle.paged_attention(q, kc, vc, 0, gs, mask, 1.0 / np.sqrt(d))
    dev = torch.device("cuda")
    out = ops.paged_attention_masked(torch.from_numpy(q).to(dev), torch.from_numpy(kc).to(dev),
                                     torch.from_numpy(vc).to(dev), 0, torch.from_numpy(gs).to(dev),
                                     torch.from_numpy(mask).to(dev),
                                     float(1.0 / np.sqrt(d))).cpu().numpy()
    assert np.isfinite(out).all()
    assert max_rel(out, ref) <= FP32_REL
    assert not out[0, 1].any()
    assert ops.read_status(dev) == 0


def test_prefill_config3_full_size_vs_oracle(pkg, oracle, ops):
    """Config 3 at full size, every row against the fp32 oracle: 16 prefill chunks on their
    cached prefixes + 240 decodes, 17,783 new tokens x 32 heads, as one paged_prefill call (the
    engine's mixed step).  bf16 within 2e-2 absolute of the oracle on the exactly upcast values.
    The oracle (the ragged causal form of paged_kernels.cpp:7-105) runs on every host core."""
    full = pkg.workloads.config3(seed=0)
    q, kc, vc, bt, ctx = device_batch(full, torch.bfloat16, seed=21)
    cu = torch.from_numpy(full.cu_seqlens()).cuda()
    out = ops.paged_prefill(q, kc, vc, 0, bt, cu, ctx, full.scale,
                            int(full.new_token_counts.max()), int(full.context_lens.max()))
    torch.cuda.synchronize()
    assert ops.read_status(q.device) == 0
    got = out.float().cpu().numpy()
    ref = oracle_ragged(oracle, full, q, kc, vc)
    assert got.shape == ref.shape == (17783, 32, 128)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= BF16_ABS


def test_prefill_config3_full_size_last_rows_match_decode(pkg, ops):
    """Config 3 at full size, a second, size-independent check: the last query row of each of the
    16 prefill chunks attends to its chunk's whole context, exactly what a decode query at that
    position does, so the tensor-core prefill kernel's row must equal the decode kernel's.  (The
    240 one-token sequences are left out: paged_prefill hands them to the decode kernel, so they
    would compare that kernel with itself.)  Both kernels are within 2e-2 of the fp32 oracle, hence
    within 4e-2 of each other."""
    full = pkg.workloads.config3(seed=0)
    q, kc, vc, bt, ctx = device_batch(full, torch.bfloat16, seed=21)
    cu = torch.from_numpy(full.cu_seqlens()).cuda()
    out = ops.paged_prefill(q, kc, vc, 0, bt, cu, ctx, full.scale,
                            int(full.new_token_counts.max()), int(full.context_lens.max()))
    chunks = torch.from_numpy(np.flatnonzero(full.new_token_counts > 1)).cuda()
    assert chunks.numel() == 16
    last = (cu[1:] - 1).to(torch.int32)
    dec = ops.paged_decode(q, kc, vc, 0, bt, ctx, full.scale, int(full.context_lens.max()),
                           query_rows=last)
    torch.cuda.synchronize()
    rows = last[chunks].long()
    a = out[rows].float()
    b = dec[rows].float()
    assert torch.isfinite(a).all() and torch.isfinite(b).all()
    assert (a - b).abs().max().item() <= 2 * BF16_ABS
    assert ops.read_status(q.device) == 0
