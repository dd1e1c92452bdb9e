"""Tiny random-init transformers models in the reference's benchmark setup.

speedup.py:88-116 merges each layer's key projection to fewer heads (the
average of the merged heads' rows) while values keep the config's key/value
head count, and speedup.py:119-139 then rebuilds the StaticCache tensors by
hand with the two head counts. Both steps are restated here for the tests.
"""
import torch
from transformers import LlamaConfig, LlamaForCausalLM
from transformers.cache_utils import StaticCache


def tiny_llama(dev, attn_impl, dtype=torch.bfloat16, Hq=8, Hv=2, Hk=1, D=128, layers=2, vocab=512, seed=0):
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=Hq * D, intermediate_size=2 * Hq * D, num_hidden_layers=layers,
                      num_attention_heads=Hq, num_key_value_heads=Hv, head_dim=D, max_position_embeddings=4096)
    cfg._attn_implementation = attn_impl
    model = LlamaForCausalLM(cfg).to(device=dev, dtype=dtype).eval()
    if Hk != Hv:
        hidden = cfg.hidden_size
        for layer in model.model.layers:
            w = layer.self_attn.k_proj.weight.data                 # [Hv * D, hidden]
            merged = w.float().reshape(Hk, Hv // Hk, D, hidden).mean(1).reshape(Hk * D, hidden)
            proj = torch.nn.Linear(hidden, Hk * D, bias=False, device=dev, dtype=dtype)
            proj.weight.data.copy_(merged.to(dtype))
            layer.self_attn.k_proj = proj
    return cfg, model


def surgery_static_cache(cfg, max_len, B, Hk, Hv, dev, dtype):
    """A transformers StaticCache with Hk key heads and Hv value heads, built
    the way the reference's benchmark builds it."""
    cache = StaticCache(config=cfg, max_cache_len=max_len)
    D = cfg.head_dim
    for layer in cache.layers:
        layer.lazy_initialization(torch.zeros(B, Hk, 1, D, dtype=dtype, device=dev),
                                  torch.zeros(B, Hv, 1, D, dtype=dtype, device=dev))
        layer.values = torch.zeros(B, Hv, max_len, D, dtype=dtype, device=dev)
    return cache
