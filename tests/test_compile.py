"""torch.compile(fullgraph=True) over decode steps through the torch.ops.saga ops.

The reference's harness compiles ``model.forward`` (speedup.py:620-622); its
attention functions must therefore trace without graph breaks. The custom
ops carry fake implementations, so dynamo sees them as single opaque nodes.

CPU tests trace only: a capturing backend records the FX graph and returns a
callable that raises instead of running it (nothing reaches a kernel).
GPU tests run the compiled step with the default backend and compare it with
the eager step: the ops are opaque, so the attention outputs and the
calibrated thresholds must be bit-identical.
"""
import pytest
import torch

from saga_b200.attention import attention as A

B, Hq, Hk, Hv, L, D, N = 2, 8, 1, 2, 1024, 128, 64


class _Traced(Exception):
    pass


def _capture():
    graphs = []

    def backend(gm, example_inputs):
        graphs.append(gm)

        def run(*args):
            raise _Traced()
        return run
    return graphs, backend


def _saga_nodes(gm):
    return [str(n.target) for n in gm.graph.nodes if n.op == "call_function" and "saga." in str(n.target)]


def _inputs(dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B, Hq, 1, D), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((B, Hk, L, D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((B, Hv, L, D), generator=g, device=dev).to(torch.bfloat16)
    mask = torch.zeros((B, 1, 1, L + 8), device=dev, dtype=torch.bfloat16)
    mask[:, :, :, L - 3] = float("-inf")
    return q, k, v, mask


STEPS = {
    "amortized": (lambda q, k, v, m: A.approx_top_n_attention_amortized(q, k, v, m, top_n_attention=N, layer_idx=1),
                  "saga.atopn_decode"),
    "calibrate": (lambda q, k, v, m: A.approx_top_n_attention_amortized_cal(q, k, v, m, top_n_attention=N,
                                                                           layer_idx=1),
                  "saga.atopn_calibrate"),
    "dense": (lambda q, k, v, m: A.full_einsum_forward(q, k, v, m), "saga.dense_decode"),
}


@pytest.mark.parametrize("name", sorted(STEPS))
def test_fullgraph_trace_of_one_step(name):
    fn, op = STEPS[name]
    torch._dynamo.reset()
    A.init_amortized_threshold_tensor("cpu", 2, B * Hq)
    graphs, backend = _capture()
    step = torch.compile(fn, fullgraph=True, backend=backend)
    with pytest.raises(_Traced):
        step(*_inputs("cpu"))
    assert len(graphs) == 1
    nodes = _saga_nodes(graphs[0])
    assert len(nodes) == 1 and op in nodes[0], nodes


_CALIBRATE = [False]


def _decode_dispatch(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None,
                     **kwargs):
    """Prefill through SDPA; decode through the calibration step while
    _CALIBRATE[0] is set, else the amortized Atop-N step."""
    if query.shape[-2] > 1:
        return A.sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                        scaling=scaling, is_causal=is_causal, **kwargs)
    mask = None if attention_mask is None else attention_mask[:, :, :, :key.shape[-2]]
    fn = A.approx_top_n_attention_amortized_cal if _CALIBRATE[0] else A.approx_top_n_attention_amortized
    out = fn(query, key, value, mask, scaling=scaling, top_n_attention=N, layer_idx=getattr(module, "layer_idx", 0))
    return out.transpose(1, 2).contiguous(), None


def _register():
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register("saga_compile_test", _decode_dispatch)
    AttentionMaskInterface.register("saga_compile_test", sdpa_mask)


@pytest.mark.parametrize("saga_cache", [False, True])
def test_fullgraph_trace_of_a_model_decode_step(saga_cache):
    """One decode step of a tiny merged-key Llama, the way speedup.py compiles
    model.forward: every layer's attention is one torch.ops.saga node."""
    pytest.importorskip("transformers")
    from _hf_models import surgery_static_cache, tiny_llama
    from saga_b200.attention.cache import SagaStaticCache
    _register()
    torch._dynamo.reset()
    dev, P = torch.device("cpu"), 16
    cfg, model = tiny_llama(dev, "saga_compile_test", Hq=Hq, Hv=Hv, Hk=Hk, D=D, layers=2)
    cache = (SagaStaticCache(config=cfg, max_cache_len=P + 8) if saga_cache
             else surgery_static_cache(cfg, P + 8, 1, Hk, Hv, dev, torch.bfloat16))
    A.init_amortized_threshold_tensor(dev, cfg.num_hidden_layers, Hq)
    prompt = torch.randint(0, cfg.vocab_size, (1, P))
    with torch.no_grad():
        model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1,
              cache_position=torch.arange(P))
        graphs, backend = _capture()
        fwd = torch.compile(model.forward, fullgraph=True, backend=backend)
        with pytest.raises(_Traced):
            fwd(input_ids=prompt[:, -1:], past_key_values=cache, use_cache=True, logits_to_keep=1,
                cache_position=torch.tensor([P]))
    assert len(graphs) == 1
    nodes = _saga_nodes(graphs[0])
    assert len(nodes) == cfg.num_hidden_layers and all("saga.atopn_decode" in n for n in nodes), nodes


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(STEPS))
def test_compiled_step_matches_eager(name):
    fn, _ = STEPS[name]
    dev = torch.device("cuda", 0)
    torch._dynamo.reset()
    q, k, v, m = _inputs(dev, seed=3)
    A.init_amortized_threshold_tensor(dev, 2, B * Hq)
    A.approx_top_n_attention_amortized_cal(q, k, v, m, top_n_attention=N, layer_idx=1)
    thr0 = A.AMORTIZED_THRESHOLD_TENSOR.clone()
    ref = fn(q, k, v, m)
    thr_ref = A.AMORTIZED_THRESHOLD_TENSOR.clone()
    A.AMORTIZED_THRESHOLD_TENSOR.copy_(thr0)
    out = torch.compile(fn, fullgraph=True)(q, k, v, m)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # the calibration writes the thresholds through the compiled graph too
    assert torch.equal(A.AMORTIZED_THRESHOLD_TENSOR, thr_ref)


@pytest.mark.gpu
def test_compiled_model_decode_matches_eager():
    """speedup.py:620-622 on a tiny merged-key Llama: model.forward compiled
    fullgraph. Both runs calibrate eagerly at the first decode step, then
    decode S steps fed the same tokens (the eager run's). Through dynamo and
    AOT autograd without code generation ("aot_eager") the logits must be
    bit-identical to eager; the default backend (inductor) must run the same
    graph to finite logits (it keeps the norms' and MLPs' intermediates in
    fp32 instead of rounding them to bf16 like eager torch, which moves
    this random-init bf16 model's logits by several percent)."""
    from _hf_models import tiny_llama
    from saga_b200.attention.cache import SagaStaticCache
    _register()
    torch._dynamo.reset()
    dev, P, S = torch.device("cuda", 0), 600, 4
    cfg, model = tiny_llama(dev, "saga_compile_test", Hq=Hq, Hv=Hv, Hk=Hk, D=D, layers=2)
    prompt = torch.randint(0, cfg.vocab_size, (1, P), device=dev,
                           generator=torch.Generator(device=dev).manual_seed(1))

    def run(fwd, toks):
        cache = SagaStaticCache(config=cfg, max_cache_len=P + S + 8)
        A.init_amortized_threshold_tensor(dev, cfg.num_hidden_layers, Hq)
        kw = dict(past_key_values=cache, use_cache=True, logits_to_keep=1)
        with torch.no_grad():
            out = model(input_ids=prompt, cache_position=torch.arange(P, device=dev), **kw)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            _CALIBRATE[0] = True
            out = model(input_ids=tok, cache_position=torch.tensor([P], device=dev), **kw)
            _CALIBRATE[0] = False
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            logits = []
            for s in range(S):
                o = fwd(input_ids=tok, cache_position=torch.tensor([P + 1 + s], device=dev), **kw)
                logits.append(o.logits[:, -1].float().clone())
                tok = toks[s] if toks else o.logits[:, -1].argmax(-1, keepdim=True)
        torch.cuda.synchronize()
        return torch.stack(logits)

    ref = run(model.forward, None)
    toks = [r.argmax(-1, keepdim=True) for r in ref]
    out = run(torch.compile(model.forward, fullgraph=True, backend="aot_eager"), toks)
    assert torch.equal(out, ref)
    torch._dynamo.reset()
    out = run(torch.compile(model.forward, fullgraph=True), toks)
    assert torch.isfinite(out).all()
