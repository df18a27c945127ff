"""Benchmark of the paged-attention hot path on B200.

Headline (`value`): one step = reshape_and_cache of each sequence's new token
+ paged-attention decode over the whole batch (256 sequences, lognormal contexts median 1024
clipped to [16, 4096], GQA 32/8, head_dim 128, block size 16, bf16, shuffled block pool), one
layer.  Metric: algorithmic HBM GB/s of the step (bytes every step must move: each context
token's K and V once per KV head, queries, outputs, block tables, lengths, the new K/V rows and
slots).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The same default run then adds two more legs to its JSON line:
  * `engine` -- the north star's engine target: the 8B-shape engine,
    tensor-parallel by KV head over the launched ranks (NCCL all-reduce after o_proj and
    down_proj), with its block pool at 95 % occupancy and a queue of long prompts, so the
    reference's recompute-preemption policy runs; output tokens/s over `--engine-steps` steps
    (max over ranks).  Under TP it also carries `tp_parity`: greedy tokens of a small fp32 model
    at TP N against the same engine on one GPU.
  * `prefill` (one GPU) -- the tcgen05 prefill kernel alone on the config-3 prefill chunks,
    TFLOP/s against the measured dense bf16 peak.

Multi-GPU (torchrun, one rank per GPU): for the headline, every rank runs its own independent
config-2 batch (the path partitions by sequence; no data-path collective), so scaling is weak and
`value` is the sum of all ranks' bytes over the max-over-ranks time.  The reference arm
(`--impl reference`) times the reference's own CPU kernel (oracle/_ref, compiled from the
reference's sources; the oracle's C restatement when that build is absent) on the host cores,
rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "paged-attn decode HBM GB/s (% of peak); engine tokens/s at 1/2/4/8 B200"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic(profile="paged_decode_config2.md"):
    """DRAM bytes per launch of a profiled kernel, from its committed ncu summary (or None)."""
    path = os.path.join(ROOT, "profiles", profile)
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def step_bytes(b, elem=2):
    """Algorithmic bytes of one step (decode + the new-token cache write)."""
    ctx = b.context_lens.astype(np.int64)
    kv = int(ctx.sum()) * b.num_kv_heads * b.head_dim * elem * 2
    qo = 2 * b.num_seqs * b.num_query_heads * b.head_dim * elem
    tables = int(((ctx + b.block_size - 1) // b.block_size).sum()) * 4 + b.num_seqs * 4
    write = b.num_seqs * b.num_kv_heads * b.head_dim * elem * 2 * 2 + b.num_seqs * 8
    decode = kv + qo + tables
    return decode + write, decode


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.strip().split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_sample_inputs(b, nseq, seed=1):
    """Host copies (fp32 holding bf16-rounded N(0,1) values) of the first `nseq` sequences of the
    batch, each as a compact cache with its own gather slots -- the shape of one reference call
    per sequence, the way the reference's NativePagedBackend would be driven for decode."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    seqs = []
    for s in range(nseq):
        ctx = int(b.context_lens[s])
        nb = -(-ctx // b.block_size)
        shape = (1, nb, b.block_size, b.num_kv_heads, b.head_dim)
        kc = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))).reshape(shape)
        vc = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32))).reshape(shape)
        q = O.bf16_bits_to_f32(O.f32_to_bf16_bits(
            rng.standard_normal((1, b.num_query_heads, 1, b.head_dim), dtype=np.float32))).reshape(
            1, b.num_query_heads, 1, b.head_dim)
        gs = np.arange(ctx, dtype=np.int32)
        mask = np.ones((1, 1, 1, ctx), dtype=np.uint8)
        seqs.append((q, kc, vc, gs, mask))
    return seqs


def run_cpu_kernel(b, seqs, repeats=1, min_seconds=0.0):
    """Time the reference kernel (or the oracle port) over the sample, `repeats` passes or as many
    as fill `min_seconds`; returns (GB/s, seconds per pass, kind, cores, passes)."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    if O.RefKernel.available():
        k = O.RefKernel()
        k.set_threads(cores)
        call, kind = k.paged_attention, "reference"
    else:
        os.environ["OMP_NUM_THREADS"] = str(cores)
        call, kind = O.paged_attention, "port"
    nbytes = 0
    for q, kc, vc, gs, mask in seqs:
        ctx = gs.shape[0]
        nbytes += ctx * b.num_kv_heads * b.head_dim * 2 * 2 + 2 * b.num_query_heads * b.head_dim * 2
    t0 = time.perf_counter()
    passes = 0
    while passes < repeats or time.perf_counter() - t0 < min_seconds:
        for q, kc, vc, gs, mask in seqs:
            call(q, kc, vc, 0, gs, mask, b.scale)
        passes += 1
    dt = time.perf_counter() - t0
    return nbytes * passes / dt / 1e9, dt / passes, kind, cores, passes


def cpu_mixed_sample(b, num_prefill, rows_per_chunk=256, num_decode=16, seed=2):
    """Reference-kernel calls for a bounded sample of a mixed ragged step (config 3), shaped the
    way the reference would be driven: one call per prefill chunk with a causal mask over the
    chunk's whole context (prior tokens + the chunk), one call per decode sequence.  Each chunk
    call keeps only the chunk's first `rows_per_chunk` query rows; the reference computes every
    row against the full context whatever the mask (paged_kernels.cpp:27-104), so a row costs
    the same as in the whole chunk.  Returns [(q, kc, vc, gs, mask, rows, causal_flops)]."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    Hq, Hkv, D, BS = b.num_query_heads, b.num_kv_heads, b.head_dim, b.block_size

    def bf16(shape):
        x = rng.standard_normal(shape, dtype=np.float32)
        return O.bf16_bits_to_f32(O.f32_to_bf16_bits(x)).reshape(shape)

    calls = []
    picks = list(range(num_prefill)) + list(range(num_prefill, min(b.num_seqs, num_prefill + num_decode)))
    for s in picks:
        prior, cnt = int(b.start_positions[s]), int(b.new_token_counts[s])
        ctx = prior + cnt
        rows = min(cnt, rows_per_chunk)
        nb = -(-ctx // BS)
        shape = (1, nb, BS, Hkv, D)
        pos = prior + np.arange(rows, dtype=np.int64)
        mask = (np.arange(ctx, dtype=np.int64)[None, :] <= pos[:, None]).astype(np.uint8)
        flops = 4 * Hq * D * int((pos + 1).sum())
        calls.append((bf16((1, Hq, rows, D)), bf16(shape), bf16(shape),
                      np.arange(ctx, dtype=np.int32), mask.reshape(1, 1, rows, ctx), rows, flops))
    return calls


def run_cpu_calls(calls, scale, min_seconds=0.0):
    """Run the sampled reference calls (one pass, or as many as fill `min_seconds`); returns
    (new tokens/s, causal TFLOP/s, seconds per pass, kind, cores, passes)."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    if O.RefKernel.available():
        k = O.RefKernel()
        k.set_threads(cores)
        call, kind = k.paged_attention, "reference"
    else:
        os.environ["OMP_NUM_THREADS"] = str(cores)
        call, kind = O.paged_attention, "port"
    rows = sum(c[5] for c in calls)
    flops = sum(c[6] for c in calls)
    t0 = time.perf_counter()
    passes = 0
    while passes < 1 or time.perf_counter() - t0 < min_seconds:
        for q, kc, vc, gs, mask, _, _ in calls:
            call(q, kc, vc, 0, gs, mask, scale)
        passes += 1
    dt = (time.perf_counter() - t0) / passes
    return rows / dt, flops / dt / 1e12, dt, kind, cores, passes


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import __graft_entry__
    wl = __graft_entry__.load_package().workloads
    b = wl.config2(seed=0)
    nseq = args.cpu_seqs
    seqs = cpu_sample_inputs(b, nseq)
    for _ in range(args.warmup):
        run_cpu_kernel(b, seqs[:4])
    vals, times = [], []
    for _ in range(args.steps):
        v, dt, kind, cores, _ = run_cpu_kernel(b, seqs)
        vals.append(v)
        times.append(dt)
    value = statistics.median(vals)
    sample = (f"first {nseq} of the 256 config-2 sequences (sum ctx "
              f"{int(b.context_lens[:nseq].sum())}), one reference call per sequence with bf16 "
              f"values upcast to fp32, {kind} kernel")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.median(times) * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2 decode (256 seqs, GQA 32/8, D128, BS16), CPU sample",
                   "seed": 0},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def ours_arm(args):
    import torch
    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200 import paged_ops
    import llm_serving_b200._native as N

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if args.split:
        N.lib().b200_set_decode_split_tokens(args.split)

    b = pkg.workloads.config2(seed=rank, num_seqs=args.seqs)
    total_bytes, decode_bytes = step_bytes(b)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    shape = (1, b.total_blocks, b.block_size, b.num_kv_heads, b.head_dim)
    kc = torch.randn(shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    vc = torch.randn(shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((b.num_seqs, b.num_query_heads, b.head_dim), generator=g, device=dev).to(torch.bfloat16)
    newk = torch.randn((b.num_seqs, b.num_kv_heads, b.head_dim), generator=g, device=dev).to(torch.bfloat16)
    newv = torch.randn((b.num_seqs, b.num_kv_heads, b.head_dim), generator=g, device=dev).to(torch.bfloat16)
    slots = torch.from_numpy(b.slot_mapping()).to(dev)
    bt = torch.from_numpy(b.block_tables()).to(dev)
    ctx = torch.from_numpy(b.context_lens.astype(np.int32)).to(dev)
    out = torch.empty_like(q)
    max_ctx = int(b.context_lens.max())
    stream = torch.cuda.current_stream(dev)

    def step():
        paged_ops.reshape_and_cache(newk, newv, kc, vc, slots, 0)
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, b.scale, max_ctx, out=out)

    launches_per_step = 3  # reshape_and_cache, decode plan, decode
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)

    # Clocks: nvidia-smi samples every 200 ms, longer than a timed region of a few ms, so the
    # sampler also covers ~0.6 s of the same step run back to back just before the timed steps.
    sampler = ClockSampler(local)
    sampler.start()
    t_end = time.perf_counter() + 0.6
    while time.perf_counter() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        paged_ops.reshape_and_cache(newk, newv, kc, vc, slots, 0)
        ev[i][0].record(stream)
        paged_ops.paged_decode(q, kc, vc, 0, bt, ctx, b.scale, max_ctx, out=out)
        ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    elapsed_ms = t0.elapsed_time(t1)
    decode_ms = sum(a.elapsed_time(c) for a, c in ev) / args.steps

    # e2e through the public API with host buffers: every step copies its inputs from pinned host
    # memory and reads its result back, inside the timed region.  As a serving loop would, the
    # copies run on one stream per direction with two buffer sets: step i+1's inputs go up while
    # step i decodes, and step i's output comes back while step i+1 computes.
    h_in = {"q": q.cpu().pin_memory(), "k": newk.cpu().pin_memory(),
            "v": newv.cpu().pin_memory(), "slots": slots.cpu().pin_memory(),
            "bt": bt.cpu().pin_memory(), "ctx": ctx.cpu().pin_memory()}
    h_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    bufs = [{n: torch.empty_like(t, device=dev) for n, t in h_in.items()} for _ in range(2)]
    for bset in bufs:
        bset["out"] = torch.empty_like(out)
    h2d = sum(t.numel() * t.element_size() for t in h_in.values())
    d2h = h_out[0].numel() * h_out[0].element_size()
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)  # one copy engine per direction
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    fetched = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        bset = bufs[i % 2]
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(done[i % 2])  # step i-2 has finished reading this buffer set
            for n, t in h_in.items():
                bset[n].copy_(t, non_blocking=True)
            ready[i % 2].record(up)

    def compute(i):
        bset = bufs[i % 2]
        stream.wait_event(ready[i % 2])
        if i >= 2:
            stream.wait_event(fetched[i % 2])  # step i-2's output has been read back
        paged_ops.reshape_and_cache(bset["k"], bset["v"], kc, vc, bset["slots"], 0)
        paged_ops.paged_decode(bset["q"], kc, vc, 0, bset["bt"], bset["ctx"], b.scale, max_ctx,
                               out=bset["out"])
        done[i % 2].record(stream)

    def download(i):
        with torch.cuda.stream(down):
            down.wait_event(done[i % 2])
            h_out[i % 2].copy_(bufs[i % 2]["out"], non_blocking=True)
            fetched[i % 2].record(down)

    def e2e_run(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)
            download(i)
        stream.wait_stream(up)
        stream.wait_stream(down)

    e2e_run(3)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_stream(stream)
    down.wait_stream(stream)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    e2e_ok = bool(torch.equal(h_out[(args.steps - 1) % 2], out.cpu()))

    times = torch.tensor([elapsed_ms, e2e_ms, decode_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms, decode_ms = times.tolist()
    status = paged_ops.read_status(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        seqs = cpu_sample_inputs(b, args.cpu_seqs)
        run_cpu_kernel(b, seqs[:4])  # warm-up
        v, dt, kind, cores, passes = run_cpu_kernel(b, seqs, min_seconds=args.cpu_seconds)
        cpu = {"value": round(v, 4), "unit": UNIT, "cores": cores, "kind": kind,
               "sample": f"first {args.cpu_seqs} config-2 sequences (sum ctx "
                         f"{int(b.context_lens[:args.cpu_seqs].sum())}), one call per sequence, "
                         f"bf16 values upcast to fp32; {passes} passes, {passes * dt:.1f} s"}

    # The north star's engine target (config 5, TP by KV head over these ranks, preemption
    # forced) and, under TP, the token check against one GPU; then the prefill kernel (rank 0).
    del kc, vc, bufs, h_in, h_out
    torch.cuda.empty_cache()
    engine = None
    tp_tokens = None
    if not args.no_engine:
        engine = run_engine5(args, world, rank, dev, args.engine_steps, 3, sample_clocks=True)
        if world > 1:
            tp_tokens = tp_parity_tokens(world, rank, dev)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    if tp_tokens is not None:
        ref_tokens = tp_parity_tokens(1, 0, dev)
        engine["tp_parity"] = {
            "match": tp_tokens[0] == ref_tokens[0],
            "check": f"greedy tokens of a 2-layer fp32 random-init Llama (hidden 256, 16/8 "
                     f"heads) on 4 prompts x 12 tokens at TP{world} (graph steps "
                     f"{tp_tokens[1]}) vs the same engine on one GPU, run by rank 0 after the "
                     f"process group is torn down"}
    elif engine is not None:
        engine["tp_parity"] = None
    prefill = None
    if world == 1 and not args.no_prefill:
        if args.prefill_kernel is not None:
            N.lib().b200_set_prefill_kernel(args.prefill_kernel)
        prefill = prefill_measure(dev, 20, 3,
                                  1 if args.prefill_kernel is None else args.prefill_kernel)
        prefill["kernel_selector"] = 1 if args.prefill_kernel is None else args.prefill_kernel
        prefill["long_prompts"] = prefill_long_measure(dev)
    peak, peak_kind = load_peaks()
    ms_per_step = elapsed_ms / args.steps
    value = world * total_bytes / (ms_per_step * 1e-3) / 1e9
    achieved = decode_bytes / (decode_ms * 1e-3) / 1e9
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"config2 decode step: reshape_and_cache + paged decode, "
                               f"{b.num_seqs} seqs/rank, ctx lognormal(1024,0.8) in [16,4096], "
                               f"GQA 32/8, D 128, BS 16, bf16, shuffled pool",
                   "sum_ctx_per_rank": int(b.context_lens.sum()),
                   "bytes_per_step_per_rank": total_bytes,
                   "l2": "inputs larger than L2 (KV ~%.2f GB per rank)" % (decode_bytes / 1e9),
                   "parallelism": f"independent sequence shards x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": peak_kind,
                     "kernel": "b200_paged_decode (plan + decode_tc), bytes per launch %d"
                               % decode_bytes},
        "e2e": {"value": round(world * total_bytes / (e2e_ms / args.steps * 1e-3) / 1e9, 2),
                "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipelining": "one copy stream per direction, two buffer sets: inputs of step "
                              "i+1 and output of step i-1 move while step i computes",
                "output_matches_device_run": e2e_ok},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "device_status": status,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if engine is not None:
        line["engine"] = engine
    if prefill is not None:
        line["prefill"] = prefill
    print(json.dumps(line))
    return 0


def attention_flops(b):
    """QK^T + PV flops of causal attention for every new token: 4 * Hq * D * (position + 1)."""
    tot = 0
    for st, c in zip(b.start_positions.astype(np.int64), b.new_token_counts.astype(np.int64)):
        # sum over positions st..st+c-1 of (pos + 1)
        tot += 4 * b.num_query_heads * b.head_dim * (c * st + c * (c + 1) // 2)
    return int(tot)


def config3_arm(args):
    """Mixed ragged step of BASELINE config 3 (16 prefill chunks on cached prefixes + 240 decodes):
    reshape_and_cache of all new tokens + ragged causal attention over the batch.  Reports the
    tensor-pipe fraction of the prefill chunks alone and the mixed step's tokens/s."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200 import paged_ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.prefill_kernel is not None:
        pkg._native.lib().b200_set_prefill_kernel(args.prefill_kernel)
    pkg._native.lib().b200_set_prefill_poly_exp(args.prefill_poly_exp)
    full = pkg.workloads.config3(seed=0)
    npre = 16
    pre = pkg.workloads.custom(seed=1, context_lens=full.context_lens[:npre],
                               new_token_counts=full.new_token_counts[:npre], num_query_heads=32,
                               num_kv_heads=8, head_dim=128, block_size=16)

    def setup(b, seed):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        shape = (1, b.total_blocks, b.block_size, b.num_kv_heads, b.head_dim)
        kc = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn((b.num_tokens, b.num_query_heads, b.head_dim), generator=g, device=dev).to(torch.bfloat16)
        nk = torch.randn((b.num_tokens, b.num_kv_heads, b.head_dim), generator=g, device=dev).to(torch.bfloat16)
        nv = torch.randn((b.num_tokens, b.num_kv_heads, b.head_dim), generator=g, device=dev).to(torch.bfloat16)
        return dict(kc=kc, vc=vc, q=q, nk=nk, nv=nv, out=torch.empty_like(q),
                    slots=torch.from_numpy(b.slot_mapping()).to(dev),
                    bt=torch.from_numpy(b.block_tables()).to(dev),
                    cu=torch.from_numpy(b.cu_seqlens()).to(dev),
                    ctx=torch.from_numpy(b.context_lens.astype(np.int32)).to(dev),
                    mq=int(b.new_token_counts.max()), mc=int(b.context_lens.max()))

    def attn(b, t):
        paged_ops.paged_prefill(t["q"], t["kc"], t["vc"], 0, t["bt"], t["cu"], t["ctx"], b.scale,
                                t["mq"], t["mc"], out=t["out"])

    def time_it(fn, steps, warmup):
        for _ in range(max(warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    tp = setup(pre, 5)
    ms_pre = time_it(lambda: attn(pre, tp), args.steps, args.warmup)
    f_pre = attention_flops(pre)
    tm = setup(full, 6)

    def mixed():
        paged_ops.reshape_and_cache(tm["nk"], tm["nv"], tm["kc"], tm["vc"], tm["slots"], 0)
        attn(full, tm)

    ms_mix = time_it(mixed, args.steps, args.warmup)
    peak = 1675.3
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    tflops = f_pre / (ms_pre * 1e-3) / 1e12
    line = {
        "metric": "config3 mixed ragged step: new tokens/s; prefill attention TFLOP/s",
        "value": round(full.num_tokens / (ms_mix * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_mix, 4),
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config3: 16 prefill chunks U[128,2048] on prior U[0,2048] + 240 "
                               "decodes, GQA 32/8, D 128, BS 16", "new_tokens": full.num_tokens,
                   "prefill_tokens": pre.num_tokens},
        "prefill_only": {"ms": round(ms_pre, 4), "flops": f_pre, "tflops": round(tflops, 2),
                         "roofline": {"bound": "tensor", "achieved": round(tflops, 2),
                                      "peak": peak, "unit": "TFLOP/s",
                                      "frac": round(tflops / peak, 4)}},
        "mixed_attention_tflops": round(attention_flops(full) / (ms_mix * 1e-3) / 1e12, 2),
        "prefill_kernel": {None: "library default", 0: "one query tile per item",
                           1: "two query tiles per item", 2: "two streams per CTA"}[args.prefill_kernel],
        "prefill_poly_exp_mode": args.prefill_poly_exp,
        "device_status": paged_ops.read_status(dev),
    }
    if not args.no_cpu:
        npre_s = 16
        calls = cpu_mixed_sample(full, npre_s)
        tok_s, cpu_tf, dt, kind, cores, passes = run_cpu_calls(calls, full.scale,
                                                               args.cpu_seconds)
        line["cpu_baseline"] = {
            "value": round(tok_s, 1), "unit": "tokens/s", "cores": cores, "kind": kind,
            "tflops": round(cpu_tf, 5),
            "sample": (f"the {npre_s} prefill chunks (first 256 query rows of each, causal mask "
                       f"over the chunk's whole context) and 16 of the decodes, one reference "
                       f"call each, bf16 values upcast to fp32; {passes} pass(es), "
                       f"{dt:.2f} s per pass")}
    print(json.dumps(line))
    return 0


def _dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, rank, dev


def engine4_arm(args):
    """random-init Llama (16 x 2048, 32/8 heads, D 64, FFN 8192, vocab 32000,
    bf16) under continuous batching (max 256 decoding sequences); seeded requests with Poisson
    arrivals at 20 req/s, prompts lognormal(median 512) <= 4096 tokens of uniform ids, outputs
    U[64, 512].  The first `--requests` requests of the 2000-request stream are run (the stream
    is 100 s of arrivals; the prefix keeps a bench call within minutes).  Value: output tokens/s
    over the run.  Tensor-parallel when launched with torchrun."""
    import torch
    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import CONFIG4, kv_bytes_per_token
    world, rank, dev = _dist_setup()
    # rate <= 0: every request arrives at t=0 (closed loop: the engine's capacity, not the
    # offered load); the prompts and output lengths do not depend on the rate
    arrivals, prompts, olens = pkg.workloads.config4_requests(args.requests,
                                                              args.rate if args.rate > 0 else 20.0,
                                                              CONFIG4.vocab)
    if args.rate <= 0:
        arrivals = np.zeros_like(arrivals)
    nreq = args.requests
    blocks = int(args.kv_gb * 1e9 // (kv_bytes_per_token(CONFIG4, world) * 16))
    eng = build_engine(CONFIG4, total_blocks=blocks, block_size=16, rank=rank, world=world,
                       device=dev, seed=0, max_batch_size=256, max_num_batched_tokens=16384,
                       max_model_len=8192)
    # warm-up: a few requests outside the timed run
    for i in range(4):
        eng.add_request(prompts[i][:64], max_tokens=8)
    while eng.has_unfinished_requests():
        eng.step()
    torch.cuda.synchronize(dev)
    eng.tokens_generated = 0
    if world > 1:
        dist.barrier()
    seqs = []
    admitted = 0
    flag = torch.zeros(1, dtype=torch.int64, device=dev)
    t0 = time.perf_counter()
    while admitted < nreq or eng.has_unfinished_requests():
        now = time.perf_counter() - t0
        n_new = 0
        if rank == 0:
            while admitted + n_new < nreq and arrivals[admitted + n_new] <= now:
                n_new += 1
            if n_new == 0 and not eng.has_unfinished_requests() and admitted < nreq:
                time.sleep(max(0.0, arrivals[admitted] - now))
        if world > 1:
            flag.fill_(n_new)
            dist.broadcast(flag, 0)
            n_new = int(flag.item())
        for i in range(admitted, admitted + n_new):
            seqs.append(eng.add_request(prompts[i], max_tokens=int(olens[i]),
                                        arrival=t0 + arrivals[i]))
        admitted += n_new
        if eng.has_unfinished_requests():
            eng.step()
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    out_tokens = sum(len(s.output_token_ids) for s in seqs)
    ttft = [s.first_token_time - s.arrival for s in seqs if s.first_token_time]
    tpot = [(s.finish_time - s.first_token_time) / max(1, len(s.output_token_ids) - 1)
            for s in seqs if s.finish_time and s.first_token_time]
    graph_steps = eng.graph_steps
    eng.release_graphs()  # captured graphs hold NCCL calls: release before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": "engine output tokens/s (config 4)", "value": round(out_tokens / elapsed, 1),
        "unit": "tokens/s", "n_gpus": world, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "n/a", "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config4 engine, first {nreq} of 2000 requests, "
                               + (f"Poisson({args.rate}/s) arrivals" if args.rate > 0 else
                                  "all submitted at t=0 (closed loop)")
                               + ", prompts lognormal(512) <= 4096, outputs U[64,512], "
                               "max 256 decoding sequences, random-init 16x2048 Llama",
                   "parallelism": f"tp{world}", "kv_pool_blocks": blocks},
        "elapsed_s": round(elapsed, 3), "output_tokens": out_tokens, "steps": eng.steps,
        "graph_steps": graph_steps, "preemptions": eng.scheduler.preemption_count,
        "ttft_ms_p50": round(1e3 * float(np.median(ttft)), 2) if ttft else None,
        "tpot_ms_p50": round(1e3 * float(np.median(tpot)), 3) if tpot else None,
    }
    print(json.dumps(line))
    return 0


def reference_engine4_arm(args):
    """`--workload engine4 --impl reference`: the reference's own engine on one B200, the engine
    baseline for config 4.  Its LLMEngine + Scheduler + PagedKVCacheManager (app/, staged
    unmodified into oracle/_ref by `make -C oracle ref`) with its own compiled allocator binding
    (oracle/_ref/llm_allocator_cpp*.so) and its own CudaKVCacheStrategy
    (app/memory/strategies.py:100-129); the engine is built directly, because the reference's
    configure_runtime rejects CUDA (app/config.py:35-36).  The model is a transformers Llama of
    the config-4 architecture, random init, bf16, attention through the reference's paged hook on
    its SDPA path (app/model/paged_attention.py:138-180).  The first `--requests` requests of the
    seeded config-4 stream are submitted at t=0, and steps run until they finish or `--seconds`
    pass.  Compare with `--workload engine4 --rate 0 --requests N` (this package's engine on the
    same requests).  Rank 0 only."""
    import glob
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    ref_parent = os.path.join(ROOT, "oracle", "_ref")
    binding = glob.glob(os.path.join(ref_parent, "llm_allocator_cpp*.so"))
    if not (os.path.isfile(os.path.join(ref_parent, "app", "engine", "llm_engine.py")) and binding):
        print(json.dumps({"impl": "reference", "unavailable": "the reference engine is not staged "
                          "(make -C oracle ref, which needs a reference checkout)"}))
        return 0
    import torch
    # The reference pins torch 2.13; its CudaKVCacheStrategy enters torch.cuda._device_ctx(index)
    # (app/memory/strategies.py:112,118), which this image's torch lacks: torch.cuda.device(index)
    # is the same context manager.
    if not hasattr(torch.cuda, "_device_ctx"):
        torch.cuda._device_ctx = torch.cuda.device
    sys.path.insert(0, ref_parent)
    import llm_allocator_cpp  # noqa: F401  (the compiled reference binding)
    from transformers import LlamaConfig, LlamaForCausalLM
    from app.engine.llm_engine import LLMEngine
    from app.memory.manager import PagedKVCacheManager
    from app.scheduler.scheduler import Scheduler
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200.model import CONFIG4 as shape, kv_bytes_per_token
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    _, prompts, olens = pkg.workloads.config4_requests(args.requests, 20.0, shape.vocab)
    cfg = LlamaConfig(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.ffn, num_hidden_layers=shape.num_layers,
                      num_attention_heads=shape.num_heads, num_key_value_heads=shape.num_kv_heads,
                      head_dim=shape.head_dim, max_position_embeddings=8192,
                      rms_norm_eps=shape.rms_eps, rope_theta=shape.rope_theta)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
    blocks = int(args.kv_gb * 1e9 // (kv_bytes_per_token(shape) * 16))
    kv = PagedKVCacheManager.from_model_config(cfg, total_blocks=blocks, block_size=16,
                                               dtype=torch.bfloat16, device=str(dev))
    sched = Scheduler(kv_cache_manager=kv, max_batch_size=256, max_num_batched_tokens=16384,
                      block_size=16, max_model_len=8192)
    eng = LLMEngine(kv_cache_manager=kv, scheduler=sched, model=model)
    for i in range(2):  # warm-up outside the timed run
        eng.add_request(prompt_token_ids=prompts[i][:64], max_tokens=4)
    while eng.has_unfinished_requests():
        eng.step()
    torch.cuda.synchronize(dev)
    seqs = [eng.add_request(prompt_token_ids=p, max_tokens=int(o))
            for p, o in zip(prompts, olens[:args.requests])]
    steps = 0
    t0 = time.perf_counter()
    while eng.has_unfinished_requests() and time.perf_counter() - t0 < args.seconds:
        eng.step()
        steps += 1
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    out_tokens = sum(len(s.output_token_ids) for s in seqs)
    value = out_tokens / elapsed
    line = {
        "impl": "reference", "metric": "engine output tokens/s (config 4)",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": 1, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config4 engine, first {args.requests} of 2000 requests all "
                               "submitted at t=0 (closed loop), prompts lognormal(512) <= 4096, "
                               "outputs U[64,512], max 256 decoding sequences, random-init "
                               "16x2048 Llama", "kv_pool_blocks": blocks,
                   "engine": "reference LLMEngine + Scheduler + PagedKVCacheManager "
                             "(CudaKVCacheStrategy, compiled reference allocator), transformers "
                             "Llama through the reference's paged hook (SDPA path), on the GPU"},
        "output_tokens": out_tokens, "finished": sum(1 for s in seqs if s.is_finished()),
        "requests": args.requests, "steps": steps, "elapsed_s": round(elapsed, 2),
        "time_box_s": args.seconds, "preemptions": sched.preemption_count,
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def reference_engine5_arm(args):
    """`--workload engine5 --impl reference`: the reference's own engine on one B200 on a bounded
    config-5 sample.  The reference's LLMEngine + Scheduler + PagedKVCacheManager (app/, staged
    unmodified into oracle/_ref) with its compiled allocator binding and CudaKVCacheStrategy, a
    transformers Llama of the Llama-3-8B shape (random init, bf16) through its paged hook on the
    SDPA path.  The running sequences of config 5 (contexts U[8192, 32768] at 95 % of a
    `--kv-gb` pool, free list shuffled through the reference allocator, random K/V, placed as if
    prefilled) are decoded for `--steps` timed steps after `--warmup` (at most 2) untimed ones,
    within `--seconds`.  The waiting queue is left out: admitting one of its 8k-32k-token prompts
    runs SDPA over a dense (prompt x context) mask with grouped heads, whose attention matrix
    (32 heads x 32k x 32k fp32 = 137 GB at the longest prompt) does not fit next to the model and
    the pool.  Compare with `--workload engine5 --decode-only` (this package's engine on the same
    sample).  Rank 0 only."""
    import glob
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    ref_parent = os.path.join(ROOT, "oracle", "_ref")
    binding = glob.glob(os.path.join(ref_parent, "llm_allocator_cpp*.so"))
    if not (os.path.isfile(os.path.join(ref_parent, "app", "engine", "llm_engine.py")) and binding):
        print(json.dumps({"impl": "reference", "unavailable": "the reference engine is not staged "
                          "(make -C oracle ref, which needs a reference checkout)"}))
        return 0
    import torch
    if not hasattr(torch.cuda, "_device_ctx"):   # see reference_engine4_arm
        torch.cuda._device_ctx = torch.cuda.device
    sys.path.insert(0, ref_parent)
    import llm_allocator_cpp  # noqa: F401  (the compiled reference binding)
    from transformers import LlamaConfig, LlamaForCausalLM
    from app.engine.llm_engine import LLMEngine
    from app.memory.manager import PagedKVCacheManager
    from app.scheduler.scheduler import Scheduler
    from app.scheduler.sequence import Sequence, SequenceStatus
    import __graft_entry__
    __graft_entry__.load_package()
    from llm_serving_b200.model import CONFIG5 as shape
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    bs = 16
    w5 = engine5_workload(1, args.kv_gb, bs)
    blocks, ctxs, out_lens, rng = w5["blocks"], w5["ctxs"], w5["out_lens"], w5["rng"]
    cfg = LlamaConfig(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.ffn, num_hidden_layers=shape.num_layers,
                      num_attention_heads=shape.num_heads, num_key_value_heads=shape.num_kv_heads,
                      head_dim=shape.head_dim, max_position_embeddings=ENGINE5_MAX_LEN,
                      rms_norm_eps=shape.rms_eps, rope_theta=shape.rope_theta)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    kv = PagedKVCacheManager.from_model_config(cfg, total_blocks=blocks, block_size=bs,
                                               dtype=torch.bfloat16, device=str(dev))
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    for t in (kv.key_cache, kv.value_cache):
        t.normal_(generator=g)
    sched = Scheduler(kv_cache_manager=kv, max_batch_size=32,
                      max_num_batched_tokens=ENGINE5_MAX_LEN, block_size=bs,
                      max_model_len=ENGINE5_MAX_LEN)
    eng = LLMEngine(kv_cache_manager=kv, scheduler=sched, model=model)
    # shuffled free list: filler sequences take the whole pool, released in random order
    fillers = 64
    per = blocks // fillers
    fill = [Sequence(seq_id=-1 - f, prompt_token_ids=[1] * (per * bs), max_tokens=1)
            for f in range(fillers)]
    for f in fill:
        kv.allocate_prefix_blocks(f)
    for f in rng.permutation(fillers):
        kv.free_sequence(fill[int(f)])
    seqs = []
    for c, o in zip(ctxs, out_lens):
        s = eng.add_request(prompt_token_ids=[1] * c, max_tokens=int(o))
        sched.waiting.remove(s)
        kv.allocate_prefix_blocks(s)
        s.output_token_ids.append(2)          # as if prefilled: the next step decodes
        s.status = SequenceStatus.RUNNING
        sched.running.append(s)
        seqs.append(s)
    for _ in range(max(1, min(args.warmup, 2))):
        eng.step()
    torch.cuda.synchronize(dev)
    gen0 = sum(len(s.output_token_ids) for s in seqs)
    steps = 0
    t0 = time.perf_counter()
    while steps < args.steps and time.perf_counter() - t0 < args.seconds:
        eng.step()
        steps += 1
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    toks = sum(len(s.output_token_ids) for s in seqs) - gen0
    value = toks / elapsed
    line = {
        "impl": "reference", "metric": "engine output tokens/s (config 5, decode-only sample)",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config5 decode-only sample: Llama-3-8B shape random init, bf16; "
                               "the running contexts U[8192,32768] at 95% pool occupancy "
                               "(shuffled free list), no waiting queue: every step decodes them "
                               "all", "kv_pool_blocks": blocks, "sequences": len(ctxs),
                   "sum_ctx": int(sum(ctxs)),
                   "engine": "reference LLMEngine + Scheduler + PagedKVCacheManager "
                             "(CudaKVCacheStrategy, compiled reference allocator), transformers "
                             "Llama through the reference's paged hook (SDPA path), on the GPU"},
        "output_tokens": toks, "elapsed_s": round(elapsed, 2),
        "ms_per_step": round(elapsed * 1e3 / max(steps, 1), 1), "time_box_s": args.seconds,
        "preemptions": sched.preemption_count,
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


ENGINE5_MAX_OUT = 1024
ENGINE5_MAX_LEN = 32768 + ENGINE5_MAX_OUT


def engine5_workload(world, kv_gb, bs=16, seed=5):
    """The config-5 request set at tensor-parallel size `world` (host only): the pool's block
    count for `kv_gb` per GPU, running contexts U[8192, 32768] drawn until they would exceed 95 %
    of it, their output lengths U[256, 1024], and a waiting queue of twice as many prompts
    U[8192, 32768] with their output lengths.  Also returns the generator, which the engine leg
    goes on drawing from (free-list shuffle, prompt token ids)."""
    from llm_serving_b200.model import CONFIG5, kv_bytes_per_token
    blocks = int(kv_gb * 1e9 // (kv_bytes_per_token(CONFIG5, world) * bs))
    rng = np.random.default_rng(seed)
    ctxs = []
    used = 0
    while True:
        c = int(rng.integers(8192, 32769))
        need = -(-c // bs)
        if used + need > 0.95 * blocks:
            break
        ctxs.append(c)
        used += need
    out_lens = rng.integers(256, ENGINE5_MAX_OUT + 1, size=len(ctxs))
    n_wait = 2 * len(ctxs)
    wait_lens = rng.integers(8192, 32769, size=n_wait)
    wait_outs = rng.integers(256, ENGINE5_MAX_OUT + 1, size=n_wait)
    return {"blocks": blocks, "ctxs": ctxs, "out_lens": out_lens, "wait_lens": wait_lens,
            "wait_outs": wait_outs, "rng": rng}


def run_engine5(args, world, rank, dev, steps, warmup, sample_clocks=False, queue=True):
    """BASELINE config 5 under preemption pressure, tensor-parallel by KV head over the launched
    ranks (call on every rank, inside the process group when world > 1).

    Random-init Llama-3-8B shape (32 x 4096, 32/8 heads, D 128, FFN 14336, vocab 128256, bf16).
    Running sequences with contexts U[8192, 32768] are placed in the cache (random K/V, blocks
    handed out by the device pool from a shuffled free list) until they hold 95 % of a pool of
    `--kv-gb` per GPU; behind them waits a queue of twice as many requests with prompts
    U[8192, 32768] of uniform-random token ids.  Outputs are U[256, 1024] tokens.  The reference
    scheduling policy then runs (scheduler.py:84-151): waiting requests are admitted whenever
    their whole prompt fits, which drives the pool to full, and a running sequence that needs a
    block when none is free is preempted -- its blocks freed, itself re-queued at the front and
    later recomputed from its prompt and outputs.  The per-step token budget is
    `ENGINE5_MAX_LEN * world`, so every TP size admits the same work per rank (weak scaling: TP t
    holds t times the sequences in the same bytes per GPU).  With `queue=False` the waiting queue
    is left out: every step decodes the running sequences (the sample the reference's own engine
    can run on one GPU, see reference_engine5_arm).

    Returns a dict (identical on every rank; times are the max over ranks)."""
    import torch
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from llm_serving_b200.engine import build_engine, SequenceStatus
    from llm_serving_b200.model import CONFIG5, kv_bytes_per_token
    shape = CONFIG5
    bs = 16
    w5 = engine5_workload(world, args.kv_gb, bs)
    blocks, ctxs, out_lens = w5["blocks"], w5["ctxs"], w5["out_lens"]
    wait_lens, wait_outs = w5["wait_lens"], w5["wait_outs"]
    if not queue:
        wait_lens, wait_outs = wait_lens[:0], wait_outs[:0]
    n_wait = len(wait_lens)
    rng = w5["rng"]
    eng = build_engine(shape, total_blocks=blocks, block_size=bs, rank=rank, world=world,
                       device=dev, seed=0, max_batch_size=32 * world,
                       max_num_batched_tokens=ENGINE5_MAX_LEN * world,
                       max_model_len=ENGINE5_MAX_LEN)
    kv, pool = eng.kv, eng.kv.pool
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    for t in (kv.key_cache, kv.value_cache):
        t.normal_(generator=g)
    # shuffled free list: fillers take the whole pool, released in random order (at least 64 of
    # them, and enough that none exceeds a sequence's block-table row)
    fillers = max(64, -(-blocks // pool.max_blocks_per_seq))
    per = blocks // fillers
    base_slot = pool.max_seqs - fillers
    for f in range(fillers):
        pool.append_tokens(base_slot + f, per * bs)
    pool.flush()
    for f in rng.permutation(fillers):
        pool.release(base_slot + int(f))
    pool.flush()
    for c, o in zip(ctxs, out_lens):
        s = eng.add_request([1] * c, max_tokens=int(o))
        eng.scheduler.waiting.remove(s)
        kv.allocate_prefix_blocks(s)
        s.output_token_ids.append(2)          # as if prefilled: the next step decodes
        s.status = SequenceStatus.RUNNING
        eng.scheduler.running.append(s)
    # the cache holds random K/V for every allocated token (no prefill pass for these)
    pool.flush()
    for c, o in zip(wait_lens, wait_outs):
        eng.add_request(rng.integers(0, shape.vocab, size=int(c)).tolist(), max_tokens=int(o))
    for _ in range(max(warmup, 3)):
        eng.step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    pre0 = eng.scheduler.preemption_count
    gen0, ptok0, steps0, gsteps0 = (eng.tokens_generated, eng.prefill_tokens, eng.steps,
                                    eng.graph_steps)
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) if sample_clocks else None
    if sampler:
        sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    t0 = time.perf_counter()
    for _ in range(steps):
        eng.step()
    e1.record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1)
    tt = torch.tensor([ms, wall * 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms, wall_ms = tt.tolist()
    toks = eng.tokens_generated - gen0
    res = {
        "tokens_per_s": round(toks / (ms * 1e-3), 1), "tp": world, "steps": steps,
        "ms_per_step": round(ms / steps, 3), "output_tokens": toks,
        "prefill_tokens": eng.prefill_tokens - ptok0,
        "processed_tokens_per_s": round((toks + eng.prefill_tokens - ptok0) / (ms * 1e-3), 1),
        "preemptions": eng.scheduler.preemption_count - pre0,
        "preemptions_incl_warmup": eng.scheduler.preemption_count,
        "graph_steps": eng.graph_steps - gsteps0, "eager_steps": steps - (eng.graph_steps - gsteps0),
        "sequences": len(ctxs), "waiting_at_start": n_wait,
        "running_at_end": len(eng.scheduler.running), "waiting_at_end": len(eng.scheduler.waiting),
        "sum_ctx": int(sum(ctxs)), "kv_pool_blocks_per_gpu": blocks, "kv_gb_per_gpu": args.kv_gb,
        "wall_ms_max_over_ranks": round(wall_ms, 1),
        "workload": ("config5: Llama-3-8B shape random init, bf16, TP by KV head; running "
                     "contexts U[8192,32768] at 95% pool occupancy (shuffled free list) + a queue "
                     "of twice as many prompts U[8192,32768]; outputs U[256,1024]; reference "
                     "admission and recompute-preemption policy; weak scaling (pool bytes per GPU "
                     "fixed, TP t holds t x the sequences)") if queue else
                    ("config5 decode-only sample: Llama-3-8B shape random init, bf16, TP by KV "
                     "head; the running contexts U[8192,32768] at 95% pool occupancy (shuffled "
                     "free list), no waiting queue: every step decodes them all"),
        "device_status": eng.kv.pool.status(),
    }
    if clocks is not None:
        res["clocks"] = clocks
    if world > 1:
        # the step's exchange on its own: 2 all-reduces per layer (after o_proj and down_proj) of
        # the decode batch's hidden states, bf16, timed back to back (max over ranks)
        rows = max(1, min(len(eng.scheduler.running), eng.scheduler.max_batch_size))
        x = torch.randn((rows, shape.hidden), device=dev).to(torch.bfloat16)
        n_ar = 2 * shape.num_layers
        for _ in range(3):
            dist.all_reduce(x)
        torch.cuda.synchronize(dev)
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(10 * n_ar):
            dist.all_reduce(x)
        a1.record()
        torch.cuda.synchronize(dev)
        ar = torch.tensor([a0.elapsed_time(a1) / 10], dtype=torch.float64, device=dev)
        dist.all_reduce(ar, op=dist.ReduceOp.MAX)
        ar_ms = float(ar.item())
        res["allreduce"] = {"ms_per_step": round(ar_ms, 3), "calls_per_step": n_ar,
                            "bytes_per_call": rows * shape.hidden * 2,
                            "share_of_mean_step": round(ar_ms / res["ms_per_step"], 4),
                            "how": "NCCL all-reduce of the decode batch's hidden states "
                                   "(rows x hidden, bf16), 2 per layer, timed alone back to back "
                                   "with CUDA events, max over ranks"}
        del x
    eng.release_graphs()  # captured graphs hold NCCL calls: release before the process group
    del eng, kv, pool
    torch.cuda.empty_cache()
    return res


TP_PARITY_SHAPE = dict(num_layers=2, hidden=256, num_heads=16, num_kv_heads=8, head_dim=32,
                       ffn=512, vocab=400)


def tp_parity_tokens(world, rank, dev):
    """Greedy tokens of a small fp32 random-init Llama (weights drawn whole from one seed, so every
    world size holds the same model) on 4 prompts, through the engine at tensor-parallel size
    `world` (inside the process group when world > 1): decode steps as captured graphs holding
    the all-reduces, prefill eager."""
    import torch
    import __graft_entry__
    __graft_entry__.load_package()
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import LlamaShape
    shape = LlamaShape(**TP_PARITY_SHAPE)
    eng = build_engine(shape, total_blocks=128, block_size=16, rank=rank, world=world, device=dev,
                       dtype=torch.float32, seed=3, max_batch_size=8, max_model_len=256,
                       full_init=True)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, shape.vocab, (int(n),), generator=g).tolist()
               for n in (3, 30, 17, 64)]
    seqs = [eng.add_request(p, max_tokens=12) for p in prompts]
    while eng.has_unfinished_requests():
        eng.step()
    toks = [s.output_token_ids for s in seqs]
    graphs = eng.graph_steps
    eng.release_graphs()
    del eng
    return toks, graphs


def engine5_arm(args):
    """`--workload engine5`: the config-5 engine alone (see run_engine5), one JSON line."""
    import torch.distributed as dist
    world, rank, dev = _dist_setup()
    res = run_engine5(args, world, rank, dev, args.steps, args.warmup, sample_clocks=True,
                      queue=not args.decode_only)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": ("engine output tokens/s (config 5, long context under preemption)"
                   if not args.decode_only else
                   "engine output tokens/s (config 5, decode-only sample)"),
        "value": res["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
        "config": {"workload": res["workload"], "parallelism": f"tp{world} (KV heads)"},
        "engine": res,
    }
    print(json.dumps(line))
    return 0


def _prefill_time_ms(dev, pre, steps, warmup):
    """CUDA-event time of one paged_prefill call over the workload `pre` (bf16, random K/V)."""
    import torch
    from llm_serving_b200 import paged_ops
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    shape = (1, pre.total_blocks, pre.block_size, pre.num_kv_heads, pre.head_dim)
    kc = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((pre.num_tokens, pre.num_query_heads, pre.head_dim), generator=g,
                    device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    bt = torch.from_numpy(pre.block_tables()).to(dev)
    cu = torch.from_numpy(pre.cu_seqlens()).to(dev)
    ctx = torch.from_numpy(pre.context_lens.astype(np.int32)).to(dev)
    mq, mc = int(pre.new_token_counts.max()), int(pre.context_lens.max())

    def call():
        paged_ops.paged_prefill(q, kc, vc, 0, bt, cu, ctx, pre.scale, mq, mc, out=out)

    for _ in range(max(warmup, 3)):
        call()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / steps


def _bf16_peaks():
    peak, sustained, src = 1590.0, None, "fallback"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mp = json.load(f)
        peak, src = float(mp["bf16_tflops"]), "measured"
        sustained = float(mp["bf16_tflops_sustained"]) if "bf16_tflops_sustained" in mp else None
    except Exception:
        pass
    return peak, sustained, src


PREFILL_KERNEL_NAMES = {0: "prefill_tc_kernel", 1: "prefill_q2_kernel", 2: "prefill_ds_kernel"}


def prefill_measure(dev, steps, warmup, selector=1):
    """K3 alone on the 16 prefill chunks of the config-3 step (lengths U[128,2048] on prior
    contexts U[0,2048], GQA 32/8, D 128, bf16): CUDA-event time of the paged_prefill call and
    its causal QK^T + PV flops against the measured dense bf16 peak."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    full = pkg.workloads.config3(seed=0)
    npre = 16
    pre = pkg.workloads.custom(seed=1, context_lens=full.context_lens[:npre],
                               new_token_counts=full.new_token_counts[:npre], num_query_heads=32,
                               num_kv_heads=8, head_dim=128, block_size=16)
    ms = _prefill_time_ms(dev, pre, steps, warmup)
    flops = attention_flops(pre)
    peak, _, src = _bf16_peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    return {"kernel": "b200_paged_prefill (%s, tcgen05)" % PREFILL_KERNEL_NAMES[selector],
            "workload": "the 16 prefill chunks of the config-3 step (%d new tokens)"
                        % pre.num_tokens,
            "ms": round(ms, 4), "flops": flops, "tflops": round(tflops, 2),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tflops / peak, 4),
                         "peak_source": src + " (burst bf16 GEMM)"}}


def prefill_long_measure(dev, steps=5, warmup=3):
    """K3 on the prompts config 5 recomputes after a preemption: single causal prefills of 8192,
    16384 and 32768 tokens (no cached prefix; GQA 32/8, D 128, bf16), each timed alone.  Long
    prompts make long work items, so the item changes that bound the config-3 chunks weigh
    little here.  The 32k launch runs ~8 ms back to back, so the sustained GEMM figure under
    the power cap is its fairer denominator; both fractions are given."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    peak, sustained, src = _bf16_peaks()
    rows = []
    for n in (8192, 16384, 32768):
        pre = pkg.workloads.custom(seed=1, context_lens=np.array([n]),
                                   new_token_counts=np.array([n]), num_query_heads=32,
                                   num_kv_heads=8, head_dim=128, block_size=16)
        ms = _prefill_time_ms(dev, pre, steps, warmup)
        tf = attention_flops(pre) / (ms * 1e-3) / 1e12
        row = {"tokens": n, "ms": round(ms, 4), "tflops": round(tf, 1),
               "frac_of_burst_peak": round(tf / peak, 4)}
        if sustained:
            row["frac_of_sustained_peak"] = round(tf / sustained, 4)
        rows.append(row)
    return {"workload": "config-5 recompute prompts: single causal prefills (no prefix)",
            "peak_source": src, "burst_peak": peak, "sustained_peak": sustained,
            "prompts": rows}


def swap_arm(args):
    """Whole-block copies (K6) at config-5 block geometry (32 layers, block 16, 8 KV heads, D 128,
    bf16: 1 MiB of K and 1 MiB of V per block): 512 blocks at random ids of a 2048-block device
    cache move out to a page-locked host swap space, back in to other random ids, and between
    device blocks.  GB/s = block bytes moved / CUDA-event time; the host-link reference is a
    plain 1 GiB pinned cudaMemcpyAsync in each direction timed the same way; the device copy
    counts read + write bytes against the measured HBM copy peak."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200 import paged_ops
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    Ln, nb_dev, nb_host, n = 32, 2048, 512, 512
    shape = (Ln, nb_dev, 16, 8, 128)
    kc = torch.randn(shape, device=dev).to(torch.bfloat16)
    vc = torch.randn(shape, device=dev).to(torch.bfloat16)
    hk = torch.empty((Ln, nb_host, 16, 8, 128), dtype=torch.bfloat16, pin_memory=True)
    hv = torch.empty_like(hk, pin_memory=True)
    g = torch.Generator().manual_seed(9)
    perm = torch.randperm(nb_dev, generator=g).to(torch.int32)
    dev_ids, dev_ids2 = perm[:n].to(dev), perm[n:2 * n].to(dev)  # disjoint: no block is both
    # a source and a destination of one call
    host_ids = torch.randperm(nb_host, generator=g)[:n].to(torch.int32).to(dev)
    block_bytes = Ln * 16 * 8 * 128 * 2 * 2  # K + V, all layers
    moved = n * block_bytes

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / args.steps  # ms

    ms_out = timed(lambda: paged_ops.copy_blocks(kc, vc, hk, hv, dev_ids, host_ids))
    ms_in = timed(lambda: paged_ops.copy_blocks(hk, hv, kc, vc, host_ids, dev_ids2))
    ms_dd = timed(lambda: paged_ops.copy_blocks(kc, vc, kc, vc, dev_ids, dev_ids2))
    # round trip: the swapped-in (and then device-copied) blocks equal the swapped-out ones
    ok = bool(torch.equal(kc[:, dev_ids2.long()].cpu(), hk[:, host_ids.long().cpu()]))
    big_d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    big_h = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    ms_d2h = timed(lambda: big_h.copy_(big_d, non_blocking=True))
    ms_h2d = timed(lambda: big_d.copy_(big_h, non_blocking=True))
    hbm, src = load_peaks()
    gbs = lambda b, ms: round(b / (ms * 1e-3) / 1e9, 1)
    line = {
        "metric": "KV block swap GB/s (device -> host swap out)", "unit": "GB/s",
        "value": gbs(moved, ms_out), "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "512 blocks of config-5 geometry (32 layers, BS 16, 8 KV heads, "
                               "D 128; 2 MiB per block K+V) at random ids, 2048-block device "
                               "cache, 512-block pinned host swap space",
                   "bytes_per_call": moved},
        "swap_in_gbs": gbs(moved, ms_in),
        "device_copy_gbs": gbs(2 * moved, ms_dd),
        "link_reference": {"d2h_memcpy_gbs": gbs(1 << 30, ms_d2h),
                           "h2d_memcpy_gbs": gbs(1 << 30, ms_h2d)},
        "roofline": {"swap_out_frac_of_link": round((moved / ms_out) / ((1 << 30) / ms_d2h), 3),
                     "swap_in_frac_of_link": round((moved / ms_in) / ((1 << 30) / ms_h2d), 3),
                     "device_copy_frac_of_hbm": round(gbs(2 * moved, ms_dd) / hbm, 3),
                     "hbm_peak_gbs": hbm, "peak_source": src},
        "round_trip_bit_exact": ok, "gpu_launches": 3 * args.steps,
        "device_status": paged_ops.read_status(dev),
    }
    print(json.dumps(line))
    return 0


def meta_arm(args):
    """Per-step metadata (K4) at config-3 scale: cu_seqlens, context offsets and lengths,
    position ids, slot mapping and padded block tables for 16 prefill chunks + 240 decodes, built
    on the device from the device block pool's tables (a shuffled free list).  Device latency is
    measured on a CUDA graph of one call replayed `--steps` times (the engine replays K4 inside
    its decode graphs); the eager figure adds the host cost of one Python call.  The CPU
    baseline is the numpy port of the reference's PagedStepContext + build_block_tables
    (app/model/paged_attention.py:40-90, app/memory/manager.py:236-271) on the same tables."""
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from llm_serving_b200.block_manager import DeviceBlockPool
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    b = pkg.workloads.config3(seed=0)
    S, BS = b.num_seqs, b.block_size
    nfill = 64
    per_fill = b.total_blocks // nfill
    pool = DeviceBlockPool(b.total_blocks, BS, S + nfill, max(512, per_fill), dev)
    rng = np.random.default_rng(0)
    for i in range(nfill):                      # take the pool, give it back shuffled
        pool.append_tokens(S + i, BS * per_fill)
    pool.flush()
    for i in rng.permutation(nfill):
        pool.release(S + int(i))
    pool.flush()
    starts = b.start_positions.astype(np.int32)
    counts = b.new_token_counts.astype(np.int32)
    for s in range(S):
        pool.append_tokens(s, int(starts[s] + counts[s]))
    pool.flush()
    bt_stride = max(pool.num_blocks(s) for s in range(S))
    ntok = int(counts.sum())
    nctx = int((starts + counts).sum())
    d_slots = torch.arange(S, dtype=torch.int32, device=dev)
    d_start = torch.from_numpy(starts).to(dev)
    d_count = torch.from_numpy(counts).to(dev)

    def call(gather):
        return pool.build_step_metadata(d_slots, d_start, d_count, ntok, bt_stride=bt_stride,
                                        with_gather_slots=gather, num_context_tokens=nctx)

    def device_us(gather):
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(max(args.warmup, 3)):
                call(gather)
        cur.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            md = call(gather)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e3 / args.steps, md, g

    us_engine, md, g1 = device_us(False)
    us_full, md_full, g2 = device_us(True)
    for _ in range(max(args.warmup, 3)):
        call(True)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        call(True)
    torch.cuda.synchronize(dev)
    eager_us = (time.perf_counter() - t0) * 1e6 / args.steps
    # bytes each call must move: the three per-sequence inputs and the pool's table rows read,
    # the outputs written (gather slots only in the full variant)
    base = 3 * S * 4 + S * bt_stride * 4 + 2 * (S + 1) * 8 + S * 4 + 2 * ntok * 8 + \
        S * bt_stride * 4
    line = {
        "metric": "step metadata (K4) latency, config-3 step", "value": round(us_engine, 2),
        "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": False, "dtype": "int64", "data": "synthetic",
        "config": {"workload": "config3 metadata: 16 prefill chunks + 240 decodes, BS 16, "
                               "shuffled device pool", "num_seqs": S, "new_tokens": ntok,
                   "context_tokens": nctx, "bt_stride": bt_stride},
        "device_us": {"engine_outputs": round(us_engine, 2),
                      "with_gather_slots": round(us_full, 2)},
        "eager_us_with_gather_slots": round(eager_us, 2),
        "bytes": {"engine_outputs": base, "with_gather_slots": base + nctx * 8},
        "gpu_launches": 2 * args.steps,
        "device_status": pool.status(),
    }
    if not args.no_cpu:
        from oracle import oracle as O
        tables = [pool.table(s) for s in range(S)]
        tok = (starts + counts).tolist()
        n = 0
        t0 = time.perf_counter()
        while n < 3 or time.perf_counter() - t0 < 2.0:
            ref = O.step_metadata(tables, tok, starts.tolist(), counts.tolist(), BS)
            ref_bt, _ = O.build_block_tables(tables, tok)
            n += 1
        cpu_us = (time.perf_counter() - t0) * 1e6 / n
        exact = (np.array_equal(md_full["cu_seqlens"].cpu().numpy(), ref["cu_seqlens"]) and
                 np.array_equal(md_full["cu_context_offsets"].cpu().numpy(),
                                ref["cu_context_offsets"]) and
                 np.array_equal(md_full["context_lens"].cpu().numpy(), ref["context_lens"]) and
                 np.array_equal(md_full["position_ids"].cpu().numpy(), ref["position_ids"][0]) and
                 np.array_equal(md_full["slot_mapping"].cpu().numpy(), ref["scatter_slots"]) and
                 np.array_equal(md_full["gather_slots"].cpu().numpy(), ref["gather_slots"]) and
                 np.array_equal(md_full["block_tables"].cpu().numpy(), ref_bt))
        line["bit_exact_vs_port"] = bool(exact)
        line["cpu_baseline"] = {
            "value": round(cpu_us, 1), "unit": "us", "cores": 1, "kind": "port",
            "sample": f"the whole step ({n} repetitions): numpy restatement of PagedStepContext "
                      f"(scatter and gather slots, positions, offsets) + build_block_tables"}
    del g1, g2
    print(json.dumps(line))
    return 0


def config1_inputs_np(seed=0, value_seed=1):
    """Config 1 as the reference's binding receives it: 8 decode sequences (contexts U[1,512]),
    12/12 heads, D 64, BS 16, fp32 N(0,1) values in a 512-block pool; the gather slots are each
    sequence's context slots in order and the (1, 1, 8, Nctx) mask lets query s see only its own
    sequence's slots -- what PagedStepContext builds for a decode step
    (app/model/paged_attention.py:64-69, :92-118).  Same recipe (and seeds) as the config-1
    golden fixture."""
    import __graft_entry__
    b = __graft_entry__.load_package().workloads.config1(seed)
    rng = np.random.default_rng(value_seed)
    shape = (1, b.total_blocks, b.block_size, b.num_kv_heads, b.head_dim)
    kc = rng.standard_normal(shape, dtype=np.float32)
    vc = rng.standard_normal(shape, dtype=np.float32)
    q = rng.standard_normal((1, b.num_query_heads, b.num_seqs, b.head_dim), dtype=np.float32)
    ctx = b.context_lens
    gs = np.concatenate([np.asarray(t, np.int64)[np.arange(c) // b.block_size] * b.block_size +
                         np.arange(c) % b.block_size
                         for t, c in zip(b.tables, ctx)]).astype(np.int32)
    owner = np.repeat(np.arange(b.num_seqs), ctx)
    mask = (owner[None, :] == np.arange(b.num_seqs)[:, None]).astype(np.uint8)[None, None]
    return b, q, kc, vc, gs, mask


def config1_arm(args):
    """Config 1 through the reference-signature C symbol ``paged_attention``
    (csrc/include/paged_kernels.h:22-34; the fp32 masked row kernel behind it), one call for the
    whole decode batch with the dense decode mask, the way NativePagedBackend.attend drives the
    binding (app/model/attention_backends.py:108-117).  value = useful bytes of the step (each
    sequence's K and V rows once, plus Q and O) / CUDA-event time of the call on device-resident
    inputs.  The whole cache (50 MB) fits in L2, so a 256 MB buffer is written between timed
    calls, outside the timed events.  e2e adds to every step the copy of Q, the gather slots and
    the mask from one pinned host buffer (one copy) and the read-back of the output (the cache
    stays resident, as it does in a server).  --impl reference (and the cpu_baseline leg): the reference's own
    kernel built from its sources (oracle/_ref), else the C port, on all host cores, on the same
    inputs; its output is compared with the GPU's (fp32: 1e-5 relative)."""
    import ctypes
    import torch
    b, q, kc, vc, gs, mask = config1_inputs_np()
    nq, hq, d = b.num_seqs, b.num_query_heads, b.head_dim
    useful = int(b.context_lens.sum()) * b.num_kv_heads * d * 4 * 2 + 2 * q.size * 4
    workload = ("config1: the paged_attention C symbol (fp32 masked form), 8 decode sequences, "
                "ctx U[1,512], 12/12 heads, D 64, BS 16, 512-block pool, one call per step")

    def cpu_leg(min_seconds):
        from oracle import oracle as O
        cores = os.cpu_count() or 1
        if O.RefKernel.available():
            k = O.RefKernel()
            k.set_threads(cores)
            call, kind = k.paged_attention, "reference"
        else:
            os.environ["OMP_NUM_THREADS"] = str(cores)
            call, kind = O.paged_attention, "port"
        out = call(q, kc, vc, 0, gs, mask, b.scale)
        t0 = time.perf_counter()
        n = 0
        while n < 3 or time.perf_counter() - t0 < min_seconds:
            call(q, kc, vc, 0, gs, mask, b.scale)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return useful / dt / 1e9, dt, kind, cores, n, np.asarray(out).reshape(1, nq, hq, d)

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        gbs, dt, kind, cores, n, _ = cpu_leg(max(2.0, args.cpu_seconds / 5))
        sample = f"the whole config-1 step, {n} calls ({dt * 1e3:.3f} ms each)"
        print(json.dumps({
            "impl": "reference", "metric": "paged_attention (config 1) GB/s", "value": round(gbs, 4),
            "unit": "GB/s", "n_gpus": 1, "steps": n, "warmup": 1, "higher_is_better": True,
            "dtype": "f32", "data": "synthetic", "ms_per_step": round(dt * 1e3, 4),
            "config": {"workload": workload},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return 0

    import __graft_entry__
    __graft_entry__.load_package()
    from llm_serving_b200 import _native as N
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    tk, tv = torch.from_numpy(kc).to(dev), torch.from_numpy(vc).to(dev)
    tq, tgs, tm = (torch.from_numpy(x).to(dev) for x in (q, gs, mask))
    out = torch.empty((1, nq, hq, d), dtype=torch.float32, device=dev)
    dims = N.PagedAttentionDims(hq, nq, d, kc.shape[0], kc.shape[1], kc.shape[2], kc.shape[3],
                                gs.shape[0])
    fn = N.lib().paged_attention
    stream = torch.cuda.current_stream(dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    scale = ctypes.c_float(b.scale)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def call(qp, gp, mp, op):
        fn(qp, tk.data_ptr(), tv.data_ptr(), 0, dims, gp, mp, scale, op, None, sptr)

    for _ in range(max(args.warmup, 3)):
        call(tq.data_ptr(), tgs.data_ptr(), tm.data_ptr(), out.data_ptr())
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record(stream)
        call(tq.data_ptr(), tgs.data_ptr(), tm.data_ptr(), out.data_ptr())
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / args.steps
    dev_out = out.cpu().numpy()
    # e2e: per step, Q, gather slots and mask in from one pinned host buffer (one copy; each
    # array at a 256-byte aligned offset), the output back out
    offs, total = [], 0
    for x in (q, gs, mask):
        offs.append(total)
        total += -(-x.nbytes // 256) * 256
    pin = torch.empty(total, dtype=torch.uint8).pin_memory()
    for x, o in zip((q, gs, mask), offs):
        pin[o:o + x.nbytes].copy_(torch.from_numpy(np.ascontiguousarray(x).view(np.uint8).ravel()))
    dbuf = torch.empty(total, dtype=torch.uint8, device=dev)
    dq, dgs, dm = (dbuf.data_ptr() + o for o in offs)
    hout = torch.empty((1, nq, hq, d), dtype=torch.float32).pin_memory()
    h2d = total
    d2h = hout.numel() * 4
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for e0, e1 in ev2:
        flush.zero_()
        e0.record(stream)
        dbuf.copy_(pin, non_blocking=True)
        call(dq, dgs, dm, out.data_ptr())
        hout.copy_(out, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_e2e = sum(e0.elapsed_time(e1) for e0, e1 in ev2) / args.steps
    # the same batch through the block-table decode API (b200_paged_decode); fp32 caches take the
    # CUDA-core row kernel
    from llm_serving_b200 import paged_ops
    qd = torch.from_numpy(np.ascontiguousarray(q[0].transpose(1, 0, 2))).to(dev)
    bt = torch.from_numpy(b.block_tables()).to(dev)
    cl = torch.from_numpy(b.context_lens).to(dev)
    maxc = int(b.context_lens.max())
    for _ in range(3):
        out_bt = paged_ops.paged_decode(qd, tk, tv, 0, bt, cl, b.scale, maxc)
    torch.cuda.synchronize(dev)
    ev3 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for e0, e1 in ev3:
        flush.zero_()
        e0.record(stream)
        out_bt = paged_ops.paged_decode(qd, tk, tv, 0, bt, cl, b.scale, maxc)
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_bt = sum(e0.elapsed_time(e1) for e0, e1 in ev3) / args.steps
    bt_out = out_bt.cpu().numpy()[None]
    peak, peak_kind = load_peaks()
    gbs = useful / (ms * 1e-3) / 1e9
    line = {
        "metric": "paged_attention (config 1) GB/s", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "l2": "256 MB buffer written between timed calls",
                   "useful_bytes_per_step": useful},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 3), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 5),
                     "traffic": load_traffic("paged_attention_masked_config1.md"),
                     "peak_source": peak_kind,
                     "kernel": "mask_attn_kernel: 96 CTAs (8 query rows x 12 heads), "
                               "latency-bound"},
        "e2e": {"value": round(useful / (ms_e2e * 1e-3) / 1e9, 3), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(ms_e2e, 5),
                "output_matches_device_run": bool(np.array_equal(hout.numpy(), dev_out))},
        "block_table_decode": {
            "api": "b200_paged_decode (block tables + context lengths) on the same batch",
            "kernel": "row_attn_kernel (fp32 caches)", "us": round(ms_bt * 1e3, 2),
            "gbs": round(useful / (ms_bt * 1e-3) / 1e9, 3),
            "max_rel_vs_mask_form": float(np.abs(bt_out - dev_out).max() / np.abs(dev_out).max())},
        "gpu_launches": 3 * args.steps,  # mask form device-resident and e2e, block-table decode
    }
    if not args.no_cpu:
        cgbs, dt, kind, cores, n, ref = cpu_leg(max(2.0, args.cpu_seconds / 5))
        line["cpu_baseline"] = {"value": round(cgbs, 4), "unit": "GB/s", "cores": cores,
                                "kind": kind,
                                "sample": f"the whole config-1 step, {n} calls "
                                          f"({dt * 1e3:.3f} ms each)"}
        line["max_rel_vs_cpu"] = float(np.abs(dev_out - ref).max() / np.abs(ref).max())
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seqs", type=int, default=256)
    ap.add_argument("--split", type=int, default=0, help="decode split tokens (0 = heuristic)")
    ap.add_argument("--cpu-seqs", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="minimum CPU work of the cpu_baseline leg (passes over the sample)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-engine", action="store_true",
                    help="skip the config-5 engine leg of the default run")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the prefill-kernel leg of the default run")
    ap.add_argument("--engine-steps", type=int, default=600,
                    help="timed engine steps of the config-5 leg of the default run")
    ap.add_argument("--prefill-poly-exp", type=int, default=1, choices=[0, 1, 2],
                    help="config3: share of softmax exponentials on the FMA pipe (0 none, 1 a "
                         "quarter, 2 half)")
    ap.add_argument("--prefill-kernel", type=int, default=None, choices=[0, 1, 2],
                    help="tensor-core prefill kernel (config3 and the prefill leg): 0 one query "
                         "tile per item, 1 two tiles per item, 2 two streams per CTA; default: "
                         "the library's")
    ap.add_argument("--workload", choices=["config1", "config2", "config3", "engine4", "engine5",
                                           "swap", "meta"],
                    default="config2")
    ap.add_argument("--requests", type=int, default=200, help="engine4: requests to run")
    ap.add_argument("--rate", type=float, default=20.0,
                    help="engine4: arrivals per second (<= 0: all requests at t=0)")
    ap.add_argument("--seconds", type=float, default=120.0,
                    help="engine4/engine5 --impl reference: time box of the reference engine's "
                         "run")
    ap.add_argument("--kv-gb", type=float, default=40.0, help="engine: KV pool GB per GPU")
    ap.add_argument("--decode-only", action="store_true",
                    help="engine5: leave out the waiting queue (the sample the reference's engine "
                         "runs with --impl reference)")
    args = ap.parse_args()
    if args.workload == "config1":
        return config1_arm(args)
    if args.workload == "config3":
        return config3_arm(args)
    if args.workload == "engine4":
        return reference_engine4_arm(args) if args.impl == "reference" else engine4_arm(args)
    if args.workload == "engine5":
        return reference_engine5_arm(args) if args.impl == "reference" else engine5_arm(args)
    if args.workload == "swap":
        return swap_arm(args)
    if args.workload == "meta":
        return meta_arm(args)
    if args.impl == "reference":
        return reference_arm(args)
    return ours_arm(args)


if __name__ == "__main__":
    sys.exit(main())
