"""The CPU legs of bench.py: the config-3 reference sample is the causal arithmetic of the mixed
step (its masks give the same rows as the oracle's ragged causal form) and its flop count is the
GPU arm's algorithmic count when no rows are dropped."""
import numpy as np

import bench


def _batch(pkg):
    # 2 prefill chunks (one on a cached prefix) + 2 decodes, GQA 4/2, D 16, BS 4
    return pkg.workloads.custom(seed=3, context_lens=[37, 21, 9, 14], new_token_counts=[12, 21, 1, 1],
                                num_query_heads=4, num_kv_heads=2, head_dim=16, block_size=4)


def test_mixed_sample_flops_match_the_gpu_arm_count(pkg):
    b = _batch(pkg)
    calls = bench.cpu_mixed_sample(b, num_prefill=2, rows_per_chunk=10 ** 6, num_decode=2)
    assert len(calls) == 4
    assert sum(c[5] for c in calls) == b.num_tokens
    assert sum(c[6] for c in calls) == bench.attention_flops(b)


def test_mixed_sample_masks_are_causal(pkg, oracle):
    b = _batch(pkg)
    calls = bench.cpu_mixed_sample(b, num_prefill=2, rows_per_chunk=8, num_decode=2)
    for s, (q, kc, vc, gs, mask, rows, _) in enumerate(calls):
        prior = int(b.start_positions[s])
        assert rows == min(int(b.new_token_counts[s]), 8)
        assert mask.shape == (1, 1, rows, prior + int(b.new_token_counts[s]))
        out = oracle.paged_attention(q, kc, vc, 0, gs, mask, b.scale)[0]
        ragged = oracle.paged_ragged(np.ascontiguousarray(q[0].transpose(1, 0, 2)), kc, vc, 0,
                                     np.arange(kc.shape[1], dtype=np.int32)[None, :], [prior],
                                     [rows], b.scale)
        err = np.abs(out - ragged).max() / np.abs(ragged).max()
        assert err <= 1e-5, (s, err)


def test_run_cpu_calls_reports_rates(pkg):
    b = _batch(pkg)
    calls = bench.cpu_mixed_sample(b, num_prefill=2, num_decode=2)
    tok_s, tflops, dt, kind, cores, passes = bench.run_cpu_calls(calls, b.scale)
    assert passes == 1 and dt > 0 and cores >= 1
    assert kind in ("reference", "port")
    assert tok_s > 0 and tflops > 0


def test_config4_request_stream_is_the_seeded_one(pkg):
    """The engine bench's request stream: seed 4, draws in the order arrivals, prompt lengths,
    output lengths, then the prompts' token ids."""
    import math
    arrivals, prompts, olens = pkg.workloads.config4_requests(5)
    rng = np.random.default_rng(4)
    gaps = rng.exponential(1.0 / 20.0, size=2000)
    plens = np.clip(np.rint(np.exp(rng.normal(math.log(512), 0.8, size=2000))), 1, 4096)
    expect_olens = rng.integers(64, 513, size=2000)
    assert arrivals[0] == 0.0 and np.allclose(np.diff(arrivals), gaps[1:])
    assert np.array_equal(olens, expect_olens)
    assert [len(p) for p in prompts] == plens[:5].astype(int).tolist()
    assert prompts[0] == rng.integers(0, 32000, size=int(plens[0])).tolist()
    assert 64 <= olens.min() and olens.max() <= 512 and max(map(max, prompts)) < 32000


def test_roofline_arithmetic_matches_the_quoted_figures(pkg):
    """The algorithmic bytes and flops the bench divides by measured time are the figures the
    profile summaries quote: config-2 decode 1,421,076,360 B per launch (K and V of every context
    token once per KV head, Q, O, block ids, lengths), config-3 prefill chunks 533,616,574,464
    flop (QK^T and PV over the causal region only)."""
    b2 = pkg.workloads.config2(seed=0)
    step, decode = bench.step_bytes(b2)
    assert int(b2.context_lens.sum()) == 345897
    assert decode == 1421076360
    assert step - decode == 256 * 8 * 128 * 2 * 2 * 2 + 256 * 8   # new K/V rows read + written, slots
    full = pkg.workloads.config3(seed=0)
    pre = pkg.workloads.custom(seed=1, context_lens=full.context_lens[:16],
                               new_token_counts=full.new_token_counts[:16], num_query_heads=32,
                               num_kv_heads=8, head_dim=128, block_size=16)
    assert pre.num_tokens == 17543
    assert bench.attention_flops(pre) == 533616574464


def test_config1_bench_inputs_are_the_golden_ones(golden):
    """The config-1 bench leg feeds the reference-signature symbol the golden fixture's inputs:
    the same arrays as the fixture generator, and the reference's recorded output from them."""
    from config1_inputs import config1_inputs
    b, q, kc, vc, gs, mask = bench.config1_inputs_np()
    b2, q2, kc2, vc2, gs2, mask2 = config1_inputs()
    for x, y in ((q, q2), (kc, kc2), (vc, vc2), (gs, gs2), (mask, mask2)):
        assert x.dtype == y.dtype and np.array_equal(x, y)
    assert b.scale == b2.scale and mask.shape == (1, 1, b.num_seqs, gs.shape[0])


def test_config1_reference_arm_line(capsys):
    """--workload config1 --impl reference prints one line on the reference contract."""
    import json
    import sys
    argv = sys.argv
    sys.argv = ["bench.py", "--workload", "config1", "--impl", "reference", "--cpu-seconds", "1"]
    try:
        assert bench.main() == 0
    finally:
        sys.argv = argv
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GB/s"
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
