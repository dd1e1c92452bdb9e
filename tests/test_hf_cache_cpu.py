"""SagaStaticCache and SagaPagedCache plumbing with a real transformers
model, on CPU.

The attention functions here are CPU stand-ins for the saga_b200 decode
kernels. They consume the decode token that the cache recorded, write it
where the fused kernel would (the recorded position; for the paged cache the
page its table names), and run SDPA. The tests check the cache classes and
the hand-off that the fused kernels rely on: logits and cache contents must
equal a run with the reference's StaticCache (keys merged to one head, values
with the config's heads), and, for the paged cache with a prompt forked to
several sequences, a run with transformers' DynamicCache.
"""
import pytest
import torch

transformers = pytest.importorskip("transformers")
from transformers import AttentionInterface  # noqa: E402
from transformers.cache_utils import StaticCache  # noqa: E402
from transformers.integrations.sdpa_attention import repeat_kv  # noqa: E402

from saga_b200.attention.cache import SagaStaticCache, take_pending  # noqa: E402
from _hf_models import surgery_static_cache, tiny_llama  # noqa: E402

Hq, Hv, Hk, D = 4, 2, 1, 16


def _stand_in(module, query, key, value, attention_mask, scaling=None, **kwargs):
    pend = take_pending(key)
    if pend is not None:  # what the fused kernel does: write the token, then attend
        k_new, v_new, pos = pend
        key.index_copy_(2, pos, k_new)
        value.index_copy_(2, pos, v_new)
    k = repeat_kv(key, query.shape[1] // key.shape[1])
    v = repeat_kv(value, query.shape[1] // value.shape[1])
    mask = None if attention_mask is None else attention_mask[:, :, :, :k.shape[-2]]
    out = torch.nn.functional.scaled_dot_product_attention(query, k, v, attn_mask=mask, scale=scaling,
                                                           is_causal=mask is None and query.shape[2] > 1)
    return out.transpose(1, 2).contiguous(), None


AttentionInterface.register("saga_cpu_stand_in", _stand_in)


def _decode(make_cache, steps=5):
    cfg, model = tiny_llama("cpu", "saga_cpu_stand_in", torch.float32, Hq=Hq, Hv=Hv, Hk=Hk, D=D, vocab=128)
    cache = make_cache(cfg)
    prompt = torch.randint(0, 128, (2, 7), generator=torch.Generator().manual_seed(1))
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
    ref, ref_cache = _decode(lambda cfg: surgery_static_cache(cfg, 64, 2, Hk, Hv, "cpu", torch.float32))
    got, cache = _decode(lambda cfg: SagaStaticCache(config=cfg, max_cache_len=64))
    assert torch.equal(got, ref)
    for a, b in zip(cache.layers, ref_cache.layers):
        assert a.keys.shape[1] == Hk and a.values.shape[1] == Hv
        assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)


def test_unconsumed_token_raises():
    cfg, _ = tiny_llama("cpu", "saga_cpu_stand_in", torch.float32, Hq=2, Hv=1, Hk=1, D=16, layers=1, vocab=32)
    cache = SagaStaticCache(config=cfg, max_cache_len=16)
    k = torch.zeros(1, 1, 1, 16)
    cache.layers[0].update(k, k)
    with pytest.raises(RuntimeError):
        cache.layers[0].update(k, k)
    take_pending(cache.layers[0].keys)


def test_plain_static_cache_sizes_values_by_key_heads():
    """Why the reference rebuilds its cache: transformers' own StaticLayer
    gives the values the key-head count."""
    cfg, _ = tiny_llama("cpu", "saga_cpu_stand_in", torch.float32, Hq=Hq, Hv=Hv, Hk=Hk, D=D, layers=1, vocab=32)
    plain = StaticCache(config=cfg, max_cache_len=8)
    plain.layers[0].lazy_initialization(torch.zeros(1, Hk, 1, D), torch.zeros(1, Hv, 1, D))
    assert plain.layers[0].values.shape[1] == Hk
    ours = SagaStaticCache(config=cfg, max_cache_len=8)
    ours.layers[0].lazy_initialization(torch.zeros(1, Hk, 1, D), torch.zeros(1, Hv, 1, D))
    assert ours.layers[0].values.shape[1] == Hv


# ---------------------------------------------------------------------------
# SagaPagedCache
# ---------------------------------------------------------------------------

def _paged_stand_in(module, query, key, value, attention_mask, scaling=None, **kwargs):
    """What the paged fused kernel does, on CPU: append the token into the
    page the table names, then attend over the logical rows."""
    from saga_b200.attention.cache import take_paged
    pg = take_paged(key)
    if pg is None:
        return _stand_in(module, query, key, value, attention_mask, scaling=scaling, **kwargs)
    key, value, table, ctx = pg  # the pools behind the views
    k_new, v_new, pos = take_pending(key)
    page_len = key.shape[2]
    B = query.shape[0]
    for b in range(B):
        page = int(table[b, pos // page_len])
        key[page, :, pos % page_len] = k_new[b, :, 0]
        value[page, :, pos % page_len] = v_new[b, :, 0]
    npg = (ctx + page_len - 1) // page_len
    ids = table[:B, :npg].long()
    kc = key[ids].transpose(1, 2).reshape(B, key.shape[1], npg * page_len, -1)[:, :, :ctx]
    vc = value[ids].transpose(1, 2).reshape(B, value.shape[1], npg * page_len, -1)[:, :, :ctx]
    mask = None if attention_mask is None else attention_mask[:, :, :, :ctx]
    return _stand_in(module, query, kc, vc, mask, scaling=scaling, **kwargs)


AttentionInterface.register("saga_cpu_paged", _paged_stand_in)


def _fork_decode(make_cache, attn, fork=3, prompt_len=200, steps=70):
    """Prefill one prompt, fork it to `fork` sequences that then decode
    different tokens (crossing the 256-row page boundary)."""
    cfg, model = tiny_llama("cpu", attn, torch.float32, Hq=Hq, Hv=Hv, Hk=Hk, D=D, vocab=128)
    cache = make_cache(cfg)
    prompt = torch.randint(0, 128, (1, prompt_len), generator=torch.Generator().manual_seed(2))
    logits = []
    with torch.no_grad():
        out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
        cache.batch_repeat_interleave(fork)
        tok = out.logits[:, -1].argmax(-1, keepdim=True).repeat(fork, 1) + torch.arange(fork).unsqueeze(1)
        for s in range(steps):
            out = model(input_ids=tok % 128, past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1])
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
    return torch.stack(logits), cache


def test_saga_paged_cache_matches_dynamic_cache():
    from transformers.cache_utils import DynamicCache
    from saga_b200.attention.cache import SagaPagedCache
    ref, _ = _fork_decode(lambda cfg: DynamicCache(config=cfg), "saga_cpu_paged")
    got, cache = _fork_decode(lambda cfg: SagaPagedCache(cfg, max_cache_len=512, page_len=128, num_pages=16),
                              "saga_cpu_paged")
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
    layer = cache.layers[0]
    assert layer.keys.shape[1] == Hk and layer.values.shape[1] == Hv
    assert layer.length == 270 and layer.batch == 3
    # the prompt's first (full) page stays shared; pages 1 (copied on the
    # first append) and 2 (past the boundary) are private
    first = {row[0] for row in layer.table_host}
    assert len(first) == 1 and layer.refs[first.pop()] == 3
    own = [row[1] for row in layer.table_host] + [row[2] for row in layer.table_host]
    assert len(set(own)) == 6 and all(layer.refs[p] == 1 for p in own)
    assert sorted(layer.free) == sorted(set(range(16)) - {layer.table_host[0][0]} - set(own))
