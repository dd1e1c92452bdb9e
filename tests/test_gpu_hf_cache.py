"""A transformers Llama decoding through the saga_b200 kernels, with the
decode token written into the cache by the fused kernel (SagaStaticCache)
instead of by the cache's own index_copy_ (StaticCache).

The attention dispatcher follows speedup.py:42-84 of the reference: prefill
through SDPA, the first decode step calibrates the thresholds
(approx_top_n_attention_amortized_cal), later steps run the amortized kernel.
Three runs of the same seeded model and prompt:
* StaticCache, eager: index_copy_ then the kernel;
* SagaStaticCache, eager: the kernel appends the token itself;
* SagaStaticCache with the amortized step captured once in a CUDA graph and
  replayed (speedup.py:338-380 captures its decode step the same way); the
  append position is read on the device, so every replay writes one row
  further.
All three must give the same logits and the same caches.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")
from transformers import AttentionInterface, LlamaConfig, LlamaForCausalLM  # noqa: E402
from transformers.cache_utils import StaticCache  # noqa: E402
from transformers.integrations.sdpa_attention import sdpa_attention_forward  # noqa: E402
from transformers.masking_utils import AttentionMaskInterface, sdpa_mask  # noqa: E402

P, S, TOP_N = 700, 6, 64  # prompt, decode steps, top_n_attention
_STEP = [0]


def _dispatch(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None, **kwargs):
    from saga_b200.attention import attention as A
    layer = getattr(module, "layer_idx", 0)
    if query.shape[-2] > 1:
        if layer == 0:
            _STEP[0] = 0
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, is_causal=is_causal, **kwargs)
    if layer == 0:
        _STEP[0] += 1
    mask = None if attention_mask is None else attention_mask[:, :, :, :key.shape[-2]]
    fn = A.approx_top_n_attention_amortized_cal if _STEP[0] <= 1 else A.approx_top_n_attention_amortized
    out = fn(query, key, value, mask, scaling=scaling, top_n_attention=TOP_N, layer_idx=layer)
    return out.transpose(1, 2).contiguous(), None


AttentionInterface.register("saga_hf_test", _dispatch)
AttentionMaskInterface.register("saga_hf_test", sdpa_mask)


def _model(dev):
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=1, head_dim=128,
                      max_position_embeddings=2048)
    cfg._attn_implementation = "saga_hf_test"
    model = LlamaForCausalLM(cfg).to(device=dev, dtype=torch.bfloat16).eval()
    prompt = torch.randint(0, 512, (1, P), device=dev)
    return cfg, model, prompt


def _prefill(model, cfg, cache_cls, prompt, dev):
    from saga_b200.attention import attention as A
    A.init_amortized_threshold_tensor(dev, cfg.num_hidden_layers, cfg.num_attention_heads)
    cache = cache_cls(config=cfg, max_cache_len=P + S)
    out = model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1,
                cache_position=torch.arange(P, device=dev))
    return cache, out.logits[:, -1].argmax(-1, keepdim=True)


def _eager(model, cfg, cache_cls, prompt, dev):
    cache, tok = _prefill(model, cfg, cache_cls, prompt, dev)
    logits = []
    for s in range(S):
        out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1,
                    cache_position=torch.tensor([P + s], device=dev))
        logits.append(out.logits[:, -1].float())
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
    torch.cuda.synchronize()
    return torch.stack(logits), cache


def _graphed(model, cfg, prompt, dev, ref_logits):
    """Steps 0-1 eager (calibration, then the first amortized step, which
    allocates the workspaces); steps 2.. replay one captured step. The input
    tokens are the eager run's, so the replays see the same sequence."""
    from saga_b200.attention.cache import SagaStaticCache
    cache, tok = _prefill(model, cfg, SagaStaticCache, prompt, dev)
    logits = []
    for s in range(2):
        out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1,
                    cache_position=torch.tensor([P + s], device=dev))
        logits.append(out.logits[:, -1].float())
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
    static_tok = tok.clone()
    static_pos = torch.tensor([P + 2], device=dev)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = model(input_ids=static_tok, past_key_values=cache, use_cache=True, logits_to_keep=1,
                           cache_position=static_pos).logits[:, -1].float()
    for s in range(2, S):
        static_tok.copy_(ref_logits[s - 1].argmax(-1, keepdim=True))
        static_pos.fill_(P + s)
        graph.replay()
        logits.append(static_out.clone())
    torch.cuda.synchronize()
    del graph
    return torch.stack(logits), cache


def test_llama_decode_through_saga_static_cache():
    from saga_b200 import ops
    from saga_b200 import _lib as L
    from saga_b200.attention.cache import SagaStaticCache
    dev = torch.device("cuda", 0)
    cfg, model, prompt = _model(dev)
    with torch.no_grad():
        ref, ref_cache = _eager(model, cfg, StaticCache, prompt, dev)
        got, cache = _eager(model, cfg, SagaStaticCache, prompt, dev)
        assert torch.equal(got, ref), (got - ref).abs().max().item()
        for a, b in zip(cache.layers, ref_cache.layers):
            assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)
            assert int(a.cumulative_length.item()) == P + S
        gr, gcache = _graphed(model, cfg, prompt, dev, ref)
        assert torch.equal(gr, ref), (gr - ref).abs().max().item()
        for a, b in zip(gcache.layers, ref_cache.layers):
            assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)
    assert ops.read_status(dev) & (L.STATUS_WAIT_TIMEOUT | L.STATUS_APPEND_RANGE) == 0
