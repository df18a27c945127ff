"""The reference's own engine, unchanged, on top of this package (the north star's drop-in:
"the existing Python engine API stays unchanged and calls the new kernels").

The reference's LLMEngine + Scheduler + PagedKVCacheManager (app/engine/llm_engine.py:20-260,
app/scheduler/scheduler.py, app/memory/manager.py, with its own CudaKVCacheStrategy,
app/memory/strategies.py:100-129) run a seeded random-init transformers Llama in fp32 on the GPU,
with `llm_allocator_cpp` bound to this package's drop-in module.  Twice:
  * `_BACKEND = None`: the reference's inline SDPA path (app/model/paged_attention.py:165-180);
  * `_BACKEND = NativePagedBackend()` (app/model/attention_backends.py:85-117): decode steps go
    through llm_allocator_cpp.paged_attention, i.e. the B200 kernel, and the caller's own
    torch.from_numpy(output) line; prefill steps fall back to SDPA as the reference routes them.
The greedy tokens must be identical, and the native path must actually have run.

A second test runs the same reference LLMEngine and Scheduler on this package's whole device
path: the device-pool PagedKVCacheManager, the device
PagedStepContext (step metadata on the GPU) and the layer hook, so every prefill and decode of
the step goes through this package's kernels; its tokens must equal the reference's SDPA run."""
import pytest
import torch

import reference_app

pytestmark = pytest.mark.gpu


def _model(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=4, head_dim=64,
                      max_position_embeddings=1024, rms_norm_eps=1e-5, rope_theta=10000.0)
    torch.manual_seed(seed)
    return cfg, LlamaForCausalLM(cfg).to(torch.float32).cuda().eval()


def _run(ref, cfg, model, prompts, max_tokens):
    kv = ref["PagedKVCacheManager"].from_model_config(cfg, total_blocks=96, block_size=16,
                                                     dtype=torch.float32, device="cuda")
    sched = ref["Scheduler"](kv_cache_manager=kv, max_batch_size=4, max_num_batched_tokens=512,
                             block_size=16, max_model_len=512)
    eng = ref["LLMEngine"](kv_cache_manager=kv, scheduler=sched, model=model)
    seqs = [eng.add_request(prompt_token_ids=p, max_tokens=max_tokens) for p in prompts]
    while eng.has_unfinished_requests():
        eng.step()
    return [list(s.output_token_ids) for s in seqs], kv


@pytest.mark.skipif(not reference_app.staged(),
                    reason="reference app not staged (make -C oracle ref with a reference checkout)")
def test_reference_engine_unchanged_on_the_b200_kernel(pkg):
    from llm_serving_b200 import llm_allocator_cpp as dropin
    ref = reference_app.import_reference_app(dropin)
    backends, hook = ref["backends"], ref["paged_attention"]
    assert backends.native_kernel_available()
    # kv-cache strategy chosen by the reference itself for a CUDA device
    cfg, model = _model()
    g = torch.Generator().manual_seed(5)
    # 6 prompts on a 4-sequence batch limit: admission waits, decode groups of several sizes
    prompts = [torch.randint(0, 512, (int(n),), generator=g).tolist()
               for n in (5, 40, 17, 1, 90, 33)]
    calls = []
    real = dropin.paged_attention

    def counted(*a, **k):
        out = real(*a, **k)
        calls.append(out.shape)
        return out

    try:
        hook._BACKEND = None
        sdpa_tokens, kv = _run(ref, cfg, model, prompts, 12)
        assert type(kv.strategy).__name__ == "CudaKVCacheStrategy"
        assert kv.key_cache.is_cuda
        dropin.paged_attention = counted
        hook._BACKEND = backends.NativePagedBackend()
        native_tokens, _ = _run(ref, cfg, model, prompts, 12)
    finally:
        dropin.paged_attention = real
        hook._BACKEND = None
    # every decode step of every layer went through the drop-in binding (3 layers per step)
    assert len(calls) > 0 and len(calls) % cfg.num_hidden_layers == 0
    assert all(len(s) == 4 and s[0] == 1 for s in calls)  # (1, Nq, Hq, D) numpy, as bindings.cpp
    assert native_tokens == sdpa_tokens
    assert all(len(t) == 12 for t in native_tokens)


@pytest.mark.skipif(not reference_app.staged(),
                    reason="reference app not staged (make -C oracle ref with a reference checkout)")
def test_reference_engine_on_the_device_path(pkg):
    from llm_serving_b200 import llm_allocator_cpp as dropin
    from llm_serving_b200 import paged_attention as hook
    from llm_serving_b200.kv_cache import PagedKVCacheManager
    from llm_serving_b200.step_context import PagedStepContext
    ref = reference_app.import_reference_app(dropin)
    import app.engine.llm_engine as ref_engine
    ref_pa = ref["paged_attention"]
    cfg, model = _model(seed=1)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 512, (int(n),), generator=g).tolist()
               for n in (7, 64, 1, 33, 130, 18)]
    ref_pa._BACKEND = None
    sdpa_tokens, _ = _run(ref, cfg, model, prompts, 12)
    saved = (ref_engine.PagedStepContext, ref_pa.paged_attention_forward)
    calls = {"n": 0}
    real_forward = hook.paged_attention_forward

    def counted(*a, **k):
        calls["n"] += 1
        return real_forward(*a, **k)

    try:
        # the two names the reference engine resolves for its step context and its layer hook
        ref_engine.PagedStepContext = PagedStepContext
        ref_pa.paged_attention_forward = counted
        kv = PagedKVCacheManager.from_model_config(cfg, total_blocks=96, block_size=16,
                                                   dtype=torch.float32, device="cuda",
                                                   max_seqs=64, max_blocks_per_seq=32)
        sched = ref["Scheduler"](kv_cache_manager=kv, max_batch_size=4, max_num_batched_tokens=512,
                                 block_size=16, max_model_len=512)
        eng = ref["LLMEngine"](kv_cache_manager=kv, scheduler=sched, model=model)
        seqs = [eng.add_request(prompt_token_ids=p, max_tokens=12) for p in prompts]
        while eng.has_unfinished_requests():
            eng.step()
        device_tokens = [list(s.output_token_ids) for s in seqs]
    finally:
        ref_engine.PagedStepContext, ref_pa.paged_attention_forward = saved
    assert calls["n"] > 0 and calls["n"] % cfg.num_hidden_layers == 0
    assert kv.pool.status() == 0
    assert device_tokens == sdpa_tokens
