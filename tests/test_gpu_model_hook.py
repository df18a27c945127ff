"""End-to-end through the reference-shaped API: a random-init Llama from transformers, its
attention routed through ``paged_attention_forward`` (reshape_and_cache + paged kernels over the
device block pool and K4 metadata), against the same model's own eager attention over the full
sequence.  Mirrors the reference's paged-vs-generate parity tests
(tests/correctness/test_paged_attention.py:70-83) with a seeded random model in place of the
SmolLM weights, which are not available offline."""
import pytest
import torch

pytestmark = pytest.mark.gpu


class _Seq:
    def __init__(self, seq_id, prompt):
        self.seq_id = seq_id
        self.prompt_token_ids = list(prompt)
        self.output_token_ids = []
        self.block_table = None

    @property
    def total_len(self):
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    def tokens(self):
        return self.prompt_token_ids + self.output_token_ids


def _model(dtype):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=64, max_position_embeddings=1024, rms_norm_eps=1e-6)
    cfg._attn_implementation = "eager"
    return LlamaForCausalLM(cfg).to(device="cuda", dtype=dtype).eval(), cfg


def _eager_logits(model, ids):
    with torch.inference_mode():
        return model(torch.tensor([ids], device="cuda"), use_cache=False).logits[0].float()


@pytest.mark.parametrize("dtype,atol", [(torch.float32, 2e-3), (torch.bfloat16, 8e-2)])
def test_paged_hook_matches_eager_forward(pkg, dtype, atol):
    from llm_serving_b200.kv_cache import PagedKVCacheManager
    from llm_serving_b200.step_context import PagedStepContext
    from llm_serving_b200 import paged_attention as pa

    model, cfg = _model(dtype)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 17, 40)]
    # reference: greedy tokens by full recompute with the model's own eager attention
    ref_tokens, ref_logits = [], []
    for p in prompts:
        ids, toks, lgs = list(p), [], []
        for _ in range(6):
            lg = _eager_logits(model, ids)[-1]
            t = int(lg.argmax())
            toks.append(t)
            lgs.append(lg)
            ids.append(t)
        ref_tokens.append(toks)
        ref_logits.append(lgs)

    store = PagedKVCacheManager.from_model_config(cfg, total_blocks=64, block_size=16,
                                                  dtype=dtype, device="cuda", max_seqs=8)
    pa.register_paged_attention(model)
    seqs = [_Seq(i + 1, p) for i, p in enumerate(prompts)]
    for s in seqs:
        store.allocate_prefix_blocks(s)
    # step 0: prefill all three
    ctx = PagedStepContext(store, seqs, [0] * 3, [len(p) for p in prompts])
    flat = torch.tensor([[t for p in prompts for t in p]], device="cuda")
    with torch.inference_mode():
        logits = pa.run_paged_forward(model, ctx, flat)[0].float()
    for i, s in enumerate(seqs):
        lg = logits[int(ctx.cu_seqlens[i + 1]) - 1]
        assert (lg - ref_logits[i][0]).abs().max().item() < atol
        s.output_token_ids.append(ref_tokens[i][0])  # teacher forcing keeps the paths aligned
    # steps 1..5: decode; step 3 mixes a fresh prefill chunk of sequence 0 into the batch
    for step in range(1, 6):
        starts, counts, inputs = [], [], []
        for s in seqs:
            store.allocate_slot_for_next_token(s)
            starts.append(s.block_table.get_tokens_count() - 1)
            counts.append(1)
            inputs.append(s.output_token_ids[-1])
        ctx = PagedStepContext(store, seqs, starts, counts)
        assert ctx.is_decode
        with torch.inference_mode():
            logits = pa.run_paged_forward(model, ctx, torch.tensor([inputs], device="cuda"))[0]
        for i, s in enumerate(seqs):
            lg = logits[i].float()
            assert (lg - ref_logits[i][step]).abs().max().item() < atol, (step, i)
            s.output_token_ids.append(ref_tokens[i][step])
    assert pkg.paged_ops.read_status(torch.device("cuda")) == 0


def test_mixed_prefill_and_decode_step(pkg):
    """One step carrying a multi-token chunk for one sequence and single tokens for others (the
    ragged causal kernel), against eager recompute."""
    from llm_serving_b200.kv_cache import PagedKVCacheManager
    from llm_serving_b200.step_context import PagedStepContext
    from llm_serving_b200 import paged_attention as pa

    model, cfg = _model(torch.float32)
    g = torch.Generator().manual_seed(2)
    a = torch.randint(0, 512, (30,), generator=g).tolist()
    b = torch.randint(0, 512, (9,), generator=g).tolist()
    nxt = 7
    ref_a = _eager_logits(model, a)[20:]
    ref_b = _eager_logits(model, b + [nxt])[-1]
    store = PagedKVCacheManager.from_model_config(cfg, total_blocks=32, block_size=16,
                                                  dtype=torch.float32, device="cuda", max_seqs=4)
    pa.register_paged_attention(model)
    sa, sb = _Seq(1, a[:20]), _Seq(2, b)
    store.allocate_prefix_blocks(sa)
    store.allocate_prefix_blocks(sb)
    ctx = PagedStepContext(store, [sa, sb], [0, 0], [20, 9])
    with torch.inference_mode():
        pa.run_paged_forward(model, ctx, torch.tensor([a[:20] + b], device="cuda"))
    # mixed step: 10 more prompt tokens of `a` (chunked prefill) + one decode token of `b`
    sa.prompt_token_ids = a
    store.allocate_prefix_blocks(sa)
    sb.output_token_ids.append(nxt)
    store.allocate_slot_for_next_token(sb)
    ctx = PagedStepContext(store, [sa, sb], [20, 9], [10, 1])
    assert not ctx.is_decode
    with torch.inference_mode():
        logits = pa.run_paged_forward(model, ctx, torch.tensor([a[20:] + [nxt]], device="cuda"))[0]
    assert (logits[:10].float() - ref_a).abs().max().item() < 2e-3
    assert (logits[10].float() - ref_b).abs().max().item() < 2e-3
