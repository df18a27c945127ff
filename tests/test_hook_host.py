"""The per-layer attention hook's contract on the host, with stand-ins for the store, the step
context and the backend (as the reference's own tests do, tests/unit/test_attention_backends.py):
the new K/V go to the store as (Ntok, Hkv, D) rows with the step's slots, a supported step is
routed once to the backend with the module's layer and scale, the hook returns ((1, Nq, Hq, D),
None), and an unsupported step raises instead of falling back to a host path.  Registration
routes a transformers Llama's layers through the hook."""
import pytest
import torch

HQ, HKV, D, NQ = 6, 2, 8, 5


class FakeStore:
    def __init__(self):
        self.writes = []

    def scatter_layer_kv(self, layer_idx, keys, values, slots):
        self.writes.append((layer_idx, keys.clone(), values.clone(), slots))


class FakeContext:
    def __init__(self, store):
        self.store = store
        self.scatter_slots = torch.arange(NQ, dtype=torch.long)


class RecordingBackend:
    name = "recording"

    def __init__(self, supported=True):
        self.supported, self.calls = supported, []

    def supports(self, context, num_query_tokens):
        return self.supported and num_query_tokens > 0

    def attend(self, query, store, layer_idx, context, scaling, dropout):
        self.calls.append((query.shape, layer_idx, scaling, dropout))
        return torch.zeros(1, query.shape[2], query.shape[1], query.shape[3])


class FakeModule:
    layer_idx = 3
    scaling = 0.35

    def __init__(self, context):
        self.paged_context = context


def _qkv():
    g = torch.Generator().manual_seed(0)
    return (torch.randn(1, HQ, NQ, D, generator=g), torch.randn(1, HKV, NQ, D, generator=g),
            torch.randn(1, HKV, NQ, D, generator=g))


def test_supported_step_is_written_then_routed_once(pkg, monkeypatch):
    from llm_serving_b200 import paged_attention as hook
    store, backend = FakeStore(), RecordingBackend()
    ctx = FakeContext(store)
    monkeypatch.setattr(hook, "_BACKEND", backend)
    q, k, v = _qkv()
    out, weights = hook.paged_attention_forward(FakeModule(ctx), q, k, v, None, dropout=0.0)
    assert weights is None and out.shape == (1, NQ, HQ, D)
    assert backend.calls == [((1, HQ, NQ, D), 3, 0.35, 0.0)]   # module scale when none given
    (layer, keys, values, slots), = store.writes
    assert layer == 3 and slots is ctx.scatter_slots
    assert torch.equal(keys, k[0].transpose(0, 1)) and torch.equal(values, v[0].transpose(0, 1))
    hook.paged_attention_forward(FakeModule(ctx), q, k, v, None, dropout=0.0, scaling=0.125)
    assert backend.calls[-1][2] == 0.125                        # an explicit scale wins


def test_unsupported_step_raises_without_a_fallback(pkg, monkeypatch):
    from llm_serving_b200 import paged_attention as hook
    backend = RecordingBackend(supported=False)
    monkeypatch.setattr(hook, "_BACKEND", backend)
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="does not support"):
        hook.paged_attention_forward(FakeModule(FakeContext(FakeStore())), q, k, v, None)
    assert backend.calls == []


def test_registration_routes_the_layers_through_the_hook(pkg):
    from transformers import LlamaConfig, LlamaForCausalLM
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from llm_serving_b200 import paged_attention as hook
    cfg = LlamaConfig(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2)
    model = LlamaForCausalLM(cfg)
    hook.register_paged_attention(model)
    assert model.config._attn_implementation == hook.PAGED_ATTENTION_NAME
    assert ALL_ATTENTION_FUNCTIONS[hook.PAGED_ATTENTION_NAME] is hook.paged_attention_forward
    assert all(layer.self_attn.paged_context is None for layer in model.model.layers)
