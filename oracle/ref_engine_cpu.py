"""Throughput of the REFERENCE engine on the host CPU, for BASELINE config 4, time-boxed.

Test and measurement infrastructure, not product: it drives the reference's own LLMEngine,
Scheduler and PagedKVCacheManager (app/engine/llm_engine.py:20-260, app/scheduler/scheduler.py,
app/memory/manager.py) with a transformers Llama of the config-4 architecture (random init), its
attention routed through the reference's paged hook (app/model/paged_attention.py:138-207, the
SDPA path), on the CPU in fp32, the reference's CPU dtype.  It imports the reference tree, so it
runs only where that tree and its compiled binding are:

    make -C oracle ref
    PYTHONPATH=<reference checkout>:oracle/_ref python oracle/ref_engine_cpu.py \
        --requests 16 --seconds 300

The first `--requests` requests of the bench's seeded config-4 stream are all submitted at t=0
(the CPU engine is far slower than the 20 req/s arrivals, so pacing would change nothing), and
steps run until they finish or `--seconds` have passed.  Prints one JSON line: output tokens/s,
the thread count, steps and how many requests finished.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=16)
    ap.add_argument("--seconds", type=float, default=300.0)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    torch.set_num_threads(args.threads)

    from transformers import LlamaConfig, LlamaForCausalLM
    from app.engine.llm_engine import LLMEngine
    from app.memory.manager import PagedKVCacheManager
    from app.scheduler.scheduler import Scheduler

    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200.model import CONFIG4 as shape
    _, prompts, olens = pkg.workloads.config4_requests(args.requests, vocab=shape.vocab)

    cfg = LlamaConfig(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.ffn, num_hidden_layers=shape.num_layers,
                      num_attention_heads=shape.num_heads, num_key_value_heads=shape.num_kv_heads,
                      head_dim=shape.head_dim, max_position_embeddings=8192,
                      rms_norm_eps=shape.rms_eps, rope_theta=shape.rope_theta)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(torch.float32).eval()
    bs = 16
    blocks = sum(-(-(len(p) + int(o)) // bs) for p, o in zip(prompts, olens)) + 64
    kv = PagedKVCacheManager.from_model_config(cfg, total_blocks=blocks, block_size=bs,
                                               dtype=torch.float32, device="cpu")
    sched = Scheduler(kv_cache_manager=kv, max_batch_size=256, max_num_batched_tokens=16384,
                      block_size=bs, max_model_len=8192)
    eng = LLMEngine(kv_cache_manager=kv, scheduler=sched, model=model)
    seqs = [eng.add_request(prompt_token_ids=p, max_tokens=int(o))
            for p, o in zip(prompts, olens[:args.requests])]
    steps = 0
    t0 = time.perf_counter()
    while eng.has_unfinished_requests() and time.perf_counter() - t0 < args.seconds:
        eng.step()
        steps += 1
    elapsed = time.perf_counter() - t0
    out_tokens = sum(len(s.output_token_ids) for s in seqs)
    print(json.dumps({
        "impl": "reference engine (LLMEngine + paged hook, SDPA), CPU",
        "metric": "engine output tokens/s (config 4)", "value": round(out_tokens / elapsed, 3),
        "unit": "tokens/s", "threads": torch.get_num_threads(), "dtype": "f32",
        "requests": args.requests, "prompt_tokens": sum(len(p) for p in prompts),
        "output_tokens": out_tokens, "finished": sum(1 for s in seqs if s.is_finished()),
        "steps": steps, "elapsed_s": round(elapsed, 2), "time_box_s": args.seconds,
    }))
    return 0


if __name__ == "__main__":
    sys.exit(main())
