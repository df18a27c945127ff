"""The continuous-batching engine on the GPU: greedy tokens against a dense recompute of the same
random-init model (attention by plain torch over each sequence's full history), with and without
recompute-preemption, fp32 (CUDA-core kernels) and bf16 (tensor-core kernels); the captured
decode graphs against the eager step."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dense_attend(q, k, v):
    G = q.shape[1] // k.shape[1]
    kk = k.float().repeat_interleave(G, dim=1)
    vv = v.float().repeat_interleave(G, dim=1)
    s = torch.einsum("thd,shd->hts", q.float(), kk) / (q.shape[-1] ** 0.5)
    n = q.shape[0]
    s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool, device=q.device), 1),
                      float("-inf"))
    return torch.einsum("hts,shd->thd", s.softmax(-1), vv).to(q.dtype)


def _dense_logits(model, tokens):
    ids = torch.tensor(tokens, device="cuda")
    pos = torch.arange(len(tokens), device="cuda")
    with torch.inference_mode():
        h = model.forward(ids, pos, lambda layer, q, k, v: _dense_attend(q, k, v))
        return model.logits(h[-1:])[0]


def _run(engine, prompts, max_tokens):
    seqs = [engine.add_request(p, max_tokens=m) for p, m in zip(prompts, max_tokens)]
    steps = 0
    while engine.has_unfinished_requests():
        engine.step()
        steps += 1
        assert steps < 10000
    return seqs


def _prompts(n, vocab, seed):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 70, (n,), generator=g).tolist()
    return [torch.randint(0, vocab, (L,), generator=g).tolist() for L in lens]


def test_engine_fp32_matches_dense_greedy(pkg):
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import LlamaShape
    shape = LlamaShape(2, 128, 8, 2, 32, 256, 300)
    eng = build_engine(shape, total_blocks=128, block_size=16, dtype=torch.float32, seed=1,
                       max_batch_size=8, max_model_len=256, full_init=True)
    prompts = _prompts(6, shape.vocab, 0)
    seqs = _run(eng, prompts, [7] * 6)
    for s in seqs:
        toks = list(s.prompt_token_ids)
        for t in s.output_token_ids:
            assert int(_dense_logits(eng.model, toks).argmax()) == t
            toks.append(t)
    assert eng.kv.pool.get_num_free_blocks() == 128
    assert eng.graph_steps > 0  # the pure decode steps ran as captured graphs
    assert pkg.paged_ops.read_status(torch.device("cuda")) == 0


def test_engine_graph_decode_matches_eager(pkg):
    """Captured decode graphs (bucketed batch sizes, padded rows) give the eager engine's tokens.
    Output lengths differ per request, so the decode batch shrinks through several buckets."""
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import LlamaShape
    shape = LlamaShape(2, 128, 8, 2, 32, 256, 300)
    prompts = _prompts(11, shape.vocab, 21)
    lens = [3, 20, 7, 30, 12, 25, 5, 16, 9, 28, 14]
    toks = {}
    for graphs in (False, True):
        eng = build_engine(shape, total_blocks=128, block_size=16, dtype=torch.float32, seed=6,
                           max_batch_size=16, max_model_len=256, full_init=True,
                           cuda_graphs=graphs)
        toks[graphs] = [s.output_token_ids for s in _run(eng, prompts, lens)]
        assert (eng.graph_steps > 0) == graphs
        if graphs:
            assert len(eng._graphs) >= 3
    assert toks[True] == toks[False]
    assert pkg.paged_ops.read_status(torch.device("cuda")) == 0


def test_engine_preemption_recompute_is_exact(pkg):
    """A pool too small for the batch forces recompute-preemption (scheduler.py:100-112); the
    tokens must equal those of an unconstrained run."""
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import LlamaShape
    shape = LlamaShape(2, 128, 8, 2, 32, 256, 300)
    prompts = _prompts(8, shape.vocab, 5)
    big = build_engine(shape, total_blocks=256, block_size=16, dtype=torch.float32, seed=2,
                       max_batch_size=8, max_model_len=256, full_init=True)
    ref = [s.output_token_ids for s in _run(big, prompts, [40] * 8)]
    small = build_engine(shape, total_blocks=14, block_size=16, dtype=torch.float32, seed=2,
                         max_batch_size=8, max_model_len=256, full_init=True)
    got = [s.output_token_ids for s in _run(small, prompts, [40] * 8)]
    assert small.scheduler.preemption_count > 0
    assert got == ref
    assert small.kv.pool.get_num_free_blocks() == 14


def test_engine_bf16_tensor_core_paths(pkg):
    """bf16, head_dim 64 (config-4 attention shape): decode on the mma/TMA kernel, prefill on the
    tcgen05 kernel.  Every sampled token is the dense argmax or within 0.05 of it."""
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import LlamaShape
    shape = LlamaShape(2, 512, 8, 2, 64, 1024, 1000)
    eng = build_engine(shape, total_blocks=256, block_size=16, dtype=torch.bfloat16, seed=4,
                       max_batch_size=16, max_model_len=512, full_init=True)
    prompts = _prompts(10, shape.vocab, 9)
    seqs = _run(eng, prompts, [12] * 10)
    checked = 0
    for s in seqs:
        toks = list(s.prompt_token_ids)
        for t in s.output_token_ids:
            lg = _dense_logits(eng.model, toks)
            assert lg.max().item() - lg[t].item() <= 0.05, (lg.max().item(), lg[t].item())
            toks.append(t)
            checked += 1
    assert checked == 120
    assert pkg.paged_ops.read_status(torch.device("cuda")) == 0
