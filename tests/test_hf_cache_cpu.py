"""SagaStaticCache plumbing with a real transformers model, on CPU.

The attention function here is a CPU stand-in for the saga_b200 decode
kernels. It consumes the decode token that SagaStaticCache recorded, writes
it at the recorded device-side position itself, and runs SDPA. The test
checks the cache class and the hand-off that the fused kernel relies on:
logits and cache contents must equal a run with transformers' own
StaticCache.
"""
import pytest
import torch

transformers = pytest.importorskip("transformers")
from transformers import AttentionInterface, LlamaConfig, LlamaForCausalLM  # noqa: E402
from transformers.cache_utils import StaticCache  # noqa: E402
from transformers.integrations.sdpa_attention import sdpa_attention_forward  # noqa: E402

from saga_b200.attention.cache import SagaStaticCache, take_pending  # noqa: E402


def _stand_in(module, query, key, value, attention_mask, **kwargs):
    pend = take_pending(key)
    if pend is not None:  # what the fused kernel does: write the token, then attend
        k_new, v_new, pos = pend
        key.index_copy_(2, pos, k_new)
        value.index_copy_(2, pos, v_new)
    return sdpa_attention_forward(module, query, key, value, attention_mask, **kwargs)


AttentionInterface.register("saga_cpu_stand_in", _stand_in)


def _decode(cache_cls, steps=5):
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=256)
    cfg._attn_implementation = "saga_cpu_stand_in"
    model = LlamaForCausalLM(cfg).eval()
    cache = cache_cls(config=cfg, max_cache_len=64)
    prompt = torch.randint(0, 128, (2, 7))
    logits = []
    with torch.no_grad():
        out = model(input_ids=prompt, past_key_values=cache, use_cache=True, cache_position=torch.arange(7))
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        for s in range(steps):
            out = model(input_ids=tok, past_key_values=cache, use_cache=True,
                        cache_position=torch.tensor([7 + s]))
            logits.append(out.logits[:, -1])
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
    return torch.stack(logits), cache


def test_saga_static_cache_matches_static_cache():
    ref, ref_cache = _decode(StaticCache)
    got, cache = _decode(SagaStaticCache)
    assert torch.equal(got, ref)
    for a, b in zip(cache.layers, ref_cache.layers):
        assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)


def test_unconsumed_token_raises():
    cfg = LlamaConfig(vocab_size=32, hidden_size=32, intermediate_size=64, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=16)
    cache = SagaStaticCache(config=cfg, max_cache_len=16)
    k = torch.zeros(1, 1, 1, 16)
    cache.layers[0].update(k, k)
    with pytest.raises(RuntimeError):
        cache.layers[0].update(k, k)
    take_pending(cache.layers[0].keys)
