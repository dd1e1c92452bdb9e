"""A transformers Llama decoding through the saga_b200 kernels, in the two
callers' flows of the reference.

The model is random-init, with the key projection merged to one head and two
value heads (speedup.py:88-116's setup).

speedup.py's flow (42-84): prefill through SDPA, the first decode step
calibrates the thresholds (approx_top_n_attention_amortized_cal), later steps
run the amortized kernel. Three runs of the same seeded model and prompt:
* the reference's StaticCache, built by hand with the two head counts
  (speedup.py:119-139): index_copy_ then the kernel;
* SagaStaticCache: the kernel appends the decode token itself;
* SagaStaticCache with the amortized step captured once in a CUDA graph and
  replayed (speedup.py:338-380 captures its decode step the same way); the
  append position is read on the device, so every replay writes one row
  further.
All three must give the same logits and the same caches.

SagaPagedCache: one prompt forked to several sequences that share its
pages, against transformers' DynamicCache (which copies them).

lm_eval_saga.py's flow (152-212): a DynamicCache that grows by one position
per step, the threshold table created lazily with MAX_LAYERS rows, an exempt
layer on the dense kernel, recalibration at the first step and every 32
steps. Every kernel call is checked against the CPU oracle on the same
inputs, and the workspaces stay one per op while the length grows.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")
from transformers import AttentionInterface  # noqa: E402
from transformers.masking_utils import AttentionMaskInterface, sdpa_mask  # noqa: E402

from _hf_models import surgery_static_cache, tiny_llama  # noqa: E402

Hq, Hv, Hk = 8, 2, 1
P, S, TOP_N = 700, 6, 64  # prompt, decode steps, top_n_attention
_STEP = [0]


def _dispatch(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None, **kwargs):
    from saga_b200.attention import attention as A
    layer = getattr(module, "layer_idx", 0)
    if query.shape[-2] > 1:
        if layer == 0:
            _STEP[0] = 0
        return A.sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                        scaling=scaling, is_causal=is_causal, **kwargs)
    if layer == 0:
        _STEP[0] += 1
    mask = None if attention_mask is None else attention_mask[:, :, :, :key.shape[-2]]
    fn = A.approx_top_n_attention_amortized_cal if _STEP[0] <= 1 else A.approx_top_n_attention_amortized
    out = fn(query, key, value, mask, scaling=scaling, top_n_attention=TOP_N, layer_idx=layer)
    return out.transpose(1, 2).contiguous(), None


AttentionInterface.register("saga_hf_test", _dispatch)
AttentionMaskInterface.register("saga_hf_test", sdpa_mask)


def _setup(dev):
    cfg, model = tiny_llama(dev, "saga_hf_test", Hq=Hq, Hv=Hv, Hk=Hk)
    prompt = torch.randint(0, cfg.vocab_size, (1, P), device=dev)
    return cfg, model, prompt


def _prefill(model, cfg, cache, prompt, dev):
    from saga_b200.attention import attention as A
    A.init_amortized_threshold_tensor(dev, cfg.num_hidden_layers, Hq)
    out = model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1,
                cache_position=torch.arange(P, device=dev))
    return out.logits[:, -1].argmax(-1, keepdim=True)


def _eager(model, cfg, cache, prompt, dev):
    tok = _prefill(model, cfg, cache, prompt, dev)
    logits = []
    for s in range(S):
        out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1,
                    cache_position=torch.tensor([P + s], device=dev))
        logits.append(out.logits[:, -1].float())
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
    torch.cuda.synchronize()
    return torch.stack(logits)


def _graphed(model, cfg, cache, prompt, dev, ref_logits):
    """Steps 0-1 eager (calibration, then the first amortized step, which
    allocates the workspaces); steps 2.. replay one captured step. The input
    tokens are the eager run's, so the replays see the same sequence."""
    tok = _prefill(model, cfg, cache, prompt, dev)
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
    return torch.stack(logits)


def test_speedup_flow_static_caches():
    from saga_b200 import ops
    from saga_b200 import _lib as L
    from saga_b200.attention.cache import SagaStaticCache
    dev = torch.device("cuda", 0)
    cfg, model, prompt = _setup(dev)
    with torch.no_grad():
        ref_cache = surgery_static_cache(cfg, P + S, 1, Hk, Hv, dev, torch.bfloat16)
        ref = _eager(model, cfg, ref_cache, prompt, dev)
        cache = SagaStaticCache(config=cfg, max_cache_len=P + S)
        got = _eager(model, cfg, cache, prompt, dev)
        assert torch.equal(got, ref), (got - ref).abs().max().item()
        for a, b in zip(cache.layers, ref_cache.layers):
            assert a.keys.shape[1] == Hk and a.values.shape[1] == Hv
            assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)
            assert int(a.cumulative_length.item()) == P + S
        gcache = SagaStaticCache(config=cfg, max_cache_len=P + S)
        gr = _graphed(model, cfg, gcache, prompt, dev, ref)
        assert torch.equal(gr, ref), (gr - ref).abs().max().item()
        for a, b in zip(gcache.layers, ref_cache.layers):
            assert torch.equal(a.keys, b.keys) and torch.equal(a.values, b.values)
    assert ops.read_status(dev) & (L.STATUS_WAIT_TIMEOUT | L.STATUS_APPEND_RANGE) == 0


# ---------------------------------------------------------------------------
# lm_eval_saga.py's flow
# ---------------------------------------------------------------------------

LM_P, LM_STEPS = 300, 40
_LM = {"count": 0, "calls": []}


def _np(t):
    return t.detach().float().cpu().numpy()


def _lm_dispatch(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None, **kwargs):
    """lm_eval_saga.py:152-210 with every decode call recorded for the oracle."""
    from saga_b200.attention import attention as A
    layer = getattr(module, "layer_idx", 0)
    if query.shape[2] != 1:
        if layer == 0:
            _LM["count"] = 0
            A.reset_amortized_state()
        return A.sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                        scaling=scaling, is_causal=is_causal)
    mask = None if attention_mask is None else attention_mask[:, :, :, :key.shape[-2]]
    if layer == 0:
        _LM["count"] += 1
        if A.AMORTIZED_THRESHOLD_TENSOR is None:
            A.init_amortized_threshold_tensor(query.device, A.MAX_LAYERS, query.shape[0] * query.shape[1])
    rows = query.shape[0] * query.shape[1]
    if layer in A.EXEMPT_LAYERS:
        kind, thr = "dense", None
        out = A.full_einsum_forward(query, key, value, mask, scaling=scaling)
    elif _LM["count"] <= 1 or _LM["count"] % 32 == 1:
        kind, thr = "cal", None
        out = A.approx_top_n_attention_amortized_cal(query, key, value, mask, scaling=scaling,
                                                     top_n_attention=TOP_N, layer_idx=layer)
    else:
        kind, thr = "amortized", _np(A.AMORTIZED_THRESHOLD_TENSOR[layer, :rows])
        out = A.approx_top_n_attention_amortized(query, key, value, mask, scaling=scaling,
                                                 top_n_attention=TOP_N, layer_idx=layer)
    rec = dict(kind=kind, layer=layer, step=_LM["count"], q=_np(query), k=_np(key), v=_np(value), thr=thr,
               mask=None if mask is None else mask.cpu().numpy(), scaling=scaling, out=_np(out))
    if kind == "cal":
        rec["thr_out"] = _np(A.AMORTIZED_THRESHOLD_TENSOR[layer, :rows])
    _LM["calls"].append(rec)
    return out.transpose(1, 2).contiguous(), None


AttentionInterface.register("saga_lm_eval_test", _lm_dispatch)
AttentionMaskInterface.register("saga_lm_eval_test", sdpa_mask)


def _out_close(got, ref):
    err = float(np.abs(got - ref).max())
    rel = float(np.sqrt(np.mean((got - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-12))
    return err <= 2e-2 and rel <= 1e-2, (err, rel)


def test_lm_eval_flow_dynamic_cache():
    from oracle import atopn_oracle as O
    from saga_b200 import ops
    from saga_b200 import _lib as L
    from saga_b200.attention import attention as A
    dev = torch.device("cuda", 0)
    cfg, model = tiny_llama(dev, "saga_lm_eval_test", Hq=Hq, Hv=Hv, Hk=Hk, layers=3)
    prompt = torch.randint(0, cfg.vocab_size, (1, LM_P), device=dev)
    saved = (A.AMORTIZED_THRESHOLD_TENSOR, set(A.EXEMPT_LAYERS))
    A.AMORTIZED_THRESHOLD_TENSOR = None
    A.EXEMPT_LAYERS.clear()
    A.EXEMPT_LAYERS.add(0)
    _LM["calls"].clear()
    try:
        ops.read_status(dev)
        with torch.no_grad():
            out = model(input_ids=prompt, use_cache=True, logits_to_keep=1)
            cache, tok = out.past_key_values, out.logits[:, -1].argmax(-1, keepdim=True)
            n_ws = len(ops._WORKSPACES)
            for _ in range(LM_STEPS):
                out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
                cache, tok = out.past_key_values, out.logits[:, -1].argmax(-1, keepdim=True)
            torch.cuda.synchronize()
        # one workspace per op (dense, calibrate, amortized), not one per length
        assert len(ops._WORKSPACES) <= n_ws + 3
        assert A.AMORTIZED_THRESHOLD_TENSOR.shape == (A.MAX_LAYERS, Hq)
        st = ops.read_status(dev)
        assert st & (L.STATUS_WAIT_TIMEOUT | L.STATUS_NONFINITE_THR) == 0, st
    finally:
        A.AMORTIZED_THRESHOLD_TENSOR, ex = saved
        A.EXEMPT_LAYERS.clear()
        A.EXEMPT_LAYERS.update(ex)
    calls = _LM["calls"]
    assert len(calls) == 3 * LM_STEPS
    cal_steps = sorted({c["step"] for c in calls if c["kind"] == "cal"})
    assert cal_steps == [1, 33]
    assert all(c["kind"] == "dense" for c in calls if c["layer"] == 0)
    assert [c["k"].shape[2] for c in calls if c["layer"] == 1] == list(range(LM_P + 1, LM_P + LM_STEPS + 1))
    for c in calls:
        args = (c["q"], c["k"], c["v"])
        if c["kind"] == "dense":
            ref = O.dense_decode(*args, "bf16", scaling=c["scaling"], mask=c["mask"])
        elif c["kind"] == "cal":
            r = O.atopn_calibrate(*args, TOP_N, "bf16", scaling=c["scaling"], mask=c["mask"])
            np.testing.assert_allclose(c["thr_out"], r["thr"], rtol=1e-2)
            ref = r["out"]
        else:
            ref = O.atopn_amortized(*args, c["thr"], TOP_N, "bf16", scaling=c["scaling"], mask=c["mask"])["out"]
        ok, stats = _out_close(c["out"].reshape(ref.shape), ref)
        assert ok, (c["kind"], c["layer"], c["step"], stats)


# ---------------------------------------------------------------------------
# SagaPagedCache: a prompt forked to several sequences that share its pages
# ---------------------------------------------------------------------------

def test_paged_cache_fork_matches_dynamic_cache():
    """One prompt prefilled, forked to 4 sequences (transformers' DynamicCache
    copies the tensors per sequence; SagaPagedCache shares the pages), then
    the sequences decode different tokens across a page boundary. Same
    kernels, same rows: identical logits."""
    from transformers.cache_utils import DynamicCache
    from saga_b200 import ops
    from saga_b200 import _lib as Lb
    from saga_b200.attention import attention as A
    from saga_b200.attention.cache import SagaPagedCache
    dev = torch.device("cuda", 0)
    fork, prompt_len, steps = 4, 200, 70
    cfg, model = tiny_llama(dev, "saga_hf_test", Hq=Hq, Hv=Hv, Hk=Hk)
    prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), device=dev)

    def run(cache):
        A.init_amortized_threshold_tensor(dev, cfg.num_hidden_layers, fork * Hq)
        logits = []
        with torch.no_grad():
            out = model(input_ids=prompt, past_key_values=cache, use_cache=True, logits_to_keep=1)
            cache.batch_repeat_interleave(fork)
            tok = out.logits[:, -1].argmax(-1, keepdim=True).repeat(fork, 1)
            tok = (tok + torch.arange(fork, device=dev).unsqueeze(1)) % cfg.vocab_size
            for _ in range(steps):
                out = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
                logits.append(out.logits[:, -1].float())
                tok = out.logits[:, -1].argmax(-1, keepdim=True)
        torch.cuda.synchronize()
        return torch.stack(logits)

    ops.read_status(dev)
    ref = run(DynamicCache(config=cfg))
    cache = SagaPagedCache(cfg, max_cache_len=512, page_len=128, num_pages=16)
    got = run(cache)
    assert torch.equal(got, ref), (got - ref).abs().max().item()
    layer = cache.layers[0]
    assert layer.length == prompt_len + steps and layer.batch == fork
    assert layer.refs[layer.table_host[0][0]] == fork  # the prompt's full page is shared
    assert ops.read_status(dev) & (Lb.STATUS_WAIT_TIMEOUT | Lb.STATUS_PAGE_RANGE) == 0
