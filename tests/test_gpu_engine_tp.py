"""Tensor-parallel engine on 2 GPUs (NCCL): KV heads split across ranks, all-reduce after o_proj
and down_proj, vocab-parallel greedy, decode steps as captured graphs holding the collectives.
The generated tokens must equal the single-GPU engine's on the same random-init model.  Skipped
on boxes with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from llm_serving_b200.engine import build_engine
    from llm_serving_b200.model import LlamaShape
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    if world > 1:
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    shape = LlamaShape(2, 256, 8, 4, 32, 512, 400)
    eng = build_engine(shape, total_blocks=96, block_size=16, rank=rank, world=world, device=dev,
                       dtype=torch.float32, seed=3, max_batch_size=8, max_model_len=256,
                       full_init=True)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 400, (int(L),), generator=g).tolist() for L in (3, 30, 17, 64)]
    seqs = [eng.add_request(p, max_tokens=10) for p in prompts]
    while eng.has_unfinished_requests():
        eng.step()
    if rank == 0:
        q.put([s.output_token_ids for s in seqs])
    assert eng.graph_steps > 0
    eng.release_graphs()  # graphs holding NCCL calls go before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_engine_matches_single_gpu(pkg):
    ctx = mp.get_context("spawn")
    out = {}
    for world in (1, 2):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
        for p in procs:
            p.start()
        out[world] = q.get(timeout=300)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    assert out[1] == out[2]
