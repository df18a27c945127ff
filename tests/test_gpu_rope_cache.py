"""GPU parity of the rotary-fused cache write (b200_rope_reshape_and_cache): bit-identical to the
unfused path it replaces -- rotate-half rotary in fp32 (the model's elementwise ops) followed by
reshape_and_cache -- for the rotated queries and for every cache slot, with padding slots skipped
and out-of-range slots flagged."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(pkg):
    from llm_serving_b200 import paged_ops
    return paged_ops


def _rope_ref(x, positions, inv_freq):
    # the unfused path: angles in fp32, cos/sin, x1*c - x2*s / x2*c + x1*s, cast back
    ang = positions.float()[:, None] * inv_freq[None, :]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    d2 = x.shape[-1] // 2
    x1, x2 = x[..., :d2].float(), x[..., d2:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hq,hkv,D", [(32, 8, 128), (8, 2, 64), (4, 4, 32)])
def test_rope_cache_bit_identical_to_unfused(ops, dtype, hq, hkv, D):
    L, NB, BS = 2, 64, 16
    n = 97
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    kc = torch.randn((L, NB, BS, hkv, D), generator=gen, device="cuda").to(dtype)
    vc = torch.randn((L, NB, BS, hkv, D), generator=gen, device="cuda").to(dtype)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    # a strided qkv view (row stride longer than the row) to check the stride handling
    row = (hq + 2 * hkv) * D
    big = torch.randn((n, row + 8), generator=gen, device="cuda").to(dtype)
    qkv = big[:, :row]
    positions = torch.randint(0, 40000, (n,), generator=gen, device="cuda", dtype=torch.int64)
    positions[:5] = torch.tensor([0, 1, 2, 8191, 32767], device="cuda")
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    slots = torch.randperm(NB * BS, generator=torch.Generator().manual_seed(4))[:n].cuda()
    slots[7] = -1  # padding: skipped
    layer = 1

    ops.read_status(torch.device("cuda"))
    q = ops.rope_reshape_and_cache(qkv, positions, inv_freq, hq, kc, vc, slots, layer)
    torch.cuda.synchronize()
    assert ops.read_status(torch.device("cuda")) == 0

    q_ref = _rope_ref(qkv[:, :hq * D].view(n, hq, D), positions, inv_freq)
    k_ref = _rope_ref(qkv[:, hq * D:(hq + hkv) * D].view(n, hkv, D), positions, inv_freq)
    v_ref = qkv[:, (hq + hkv) * D:].view(n, hkv, D)
    ops.reshape_and_cache(k_ref, v_ref, kc_ref, vc_ref, slots, layer)
    assert torch.equal(q.view(torch.int8) if dtype != torch.float32 else q,
                       q_ref.view(torch.int8) if dtype != torch.float32 else q_ref)
    assert torch.equal(kc, kc_ref)
    assert torch.equal(vc, vc_ref)


def test_rope_cache_flags_out_of_range_slot(ops):
    L, NB, BS, hq, hkv, D = 1, 8, 16, 4, 2, 64
    dev = torch.device("cuda")
    kc = torch.zeros((L, NB, BS, hkv, D), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    qkv = torch.randn((3, (hq + 2 * hkv) * D), device=dev).to(torch.bfloat16)
    positions = torch.arange(3, device=dev, dtype=torch.int64)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
    slots = torch.tensor([0, NB * BS, 5], device=dev, dtype=torch.int64)
    ops.read_status(dev)
    ops.rope_reshape_and_cache(qkv, positions, inv_freq, hq, kc, vc, slots, 0)
    torch.cuda.synchronize()
    st = ops.read_status(dev)
    from llm_serving_b200 import _native as N
    assert st & N.DEVICE_BAD_SLOT
    # the in-range tokens were still written
    assert kc.view(-1, hkv, D)[0].abs().sum() > 0 and kc.view(-1, hkv, D)[5].abs().sum() > 0


def test_rope_cache_rejects_bad_arguments(ops):
    dev = torch.device("cuda")
    kc = torch.zeros((1, 8, 16, 2, 64), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    qkv = torch.zeros((2, 8 * 64), dtype=torch.bfloat16, device=dev)
    pos = torch.zeros(2, dtype=torch.int64, device=dev)
    inv = torch.ones(32, dtype=torch.float32, device=dev)
    slots = torch.zeros(2, dtype=torch.int64, device=dev)
    with pytest.raises(ValueError):  # 3 query heads do not group over 2 kv heads
        ops.rope_reshape_and_cache(qkv, pos, inv, 3, kc, vc, slots, 0)
    with pytest.raises(ValueError):  # row too short for 4 q + 2 k + 2 v heads of 64
        ops.rope_reshape_and_cache(qkv[:, :400], pos, inv, 4, kc, vc, slots, 0)
    with pytest.raises(ValueError):
        ops.rope_reshape_and_cache(qkv, pos.int(), inv, 4, kc, vc, slots, 0)
