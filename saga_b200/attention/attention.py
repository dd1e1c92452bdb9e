"""Drop-in replacement of the reference's ``attention/attention.py`` (noamelata/SAGA).

Same public names, signatures, module globals and side effects, so that
``speedup.py`` and ``lm_eval_saga.py`` import it unchanged
(``from attention.attention import ...``; ``import attention.attention``).
Decode-time attention (one query position) runs on the sm_100a kernels of
``libsaga_b200.so`` through the ``torch.ops.saga`` custom ops. Prefill keeps
torch SDPA, as the reference does (attention.py:13-53).

Reference line numbers below refer to ``attention/attention.py``.
"""
import math
from typing import Optional, Tuple

import torch

from saga_b200 import ops as _ops  # loads libsaga_b200.so (ImportError if missing)

try:  # transformers is only needed for the prefill path and the registration helper
    from transformers.integrations.sdpa_attention import repeat_kv
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
except Exception:  # pragma: no cover - exercised only without transformers
    ALL_ATTENTION_FUNCTIONS = None

    def repeat_kv(hidden_states: torch.Tensor, n_rep: int) -> torch.Tensor:
        b, h, s, d = hidden_states.shape
        if n_rep == 1:
            return hidden_states
        return hidden_states[:, :, None].expand(b, h, n_rep, s, d).reshape(b, h * n_rep, s, d)


# =============================================================================
# Base SDPA (prefill in all modes) -- attention.py:13-57
# =============================================================================

def sdpa_attention_forward(
        module: torch.nn.Module,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        attention_mask: Optional[torch.Tensor],
        dropout: float = 0.0,
        scaling: Optional[float] = None,
        is_causal: Optional[bool] = None,
        **kwargs,
) -> Tuple[torch.Tensor, None]:
    """Prefill attention through torch SDPA, with K and V expanded separately
    to the query heads (attention.py:24-26). Not a decode hot path."""
    if hasattr(module, "num_key_value_groups"):
        key = repeat_kv(key, query.shape[-3] // key.shape[-3])
        value = repeat_kv(value, query.shape[-3] // value.shape[-3])
    causal_mask = attention_mask
    if attention_mask is not None:
        causal_mask = causal_mask[:, :, :, : key.shape[-2]]
    query, key, value = query.contiguous(), key.contiguous(), value.contiguous()
    if is_causal is None:
        is_causal = query.shape[2] > 1 and causal_mask is None
    if torch.jit.is_tracing() and isinstance(is_causal, torch.Tensor):
        is_causal = is_causal.item()
    attn_output = torch.nn.functional.scaled_dot_product_attention(
        query, key, value, attn_mask=causal_mask, dropout_p=dropout, scale=scaling, is_causal=is_causal)
    return attn_output.transpose(1, 2).contiguous(), None


def register_sdpa():
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa_attention_forward


def _mask(attention_mask, key):
    if attention_mask is None:
        return None
    return attention_mask[:, :, :, : key.shape[-2]]


# =============================================================================
# Dense decode -- attention.py:64-85
# =============================================================================

def _pending(key):
    """Decode token recorded by SagaStaticCache / SagaPagedCache for this key
    cache (or None). Under torch.compile the caches copy the token themselves
    (a graph cannot look tensors up by address), so there is none."""
    if torch.compiler.is_compiling():
        return None
    try:
        from .cache import take_pending
    except Exception:  # pragma: no cover - transformers missing
        return None
    return take_pending(key)


def _paged(key, attention_mask):
    """For the key view of a SagaPagedCache decode step: the key and value
    pools, the mask, and the keyword arguments of the paged fused call
    (decode token, page table, logical length); else None (always under
    torch.compile: the paged cache's address registry is eager-only)."""
    if torch.compiler.is_compiling():
        return None
    try:
        from .cache import take_paged
    except Exception:  # pragma: no cover - transformers missing
        return None
    pg = take_paged(key)
    if pg is None:
        return None
    kpool, vpool, table, ctx = pg
    k_new, v_new, pos = _pending(key)
    mask = None if attention_mask is None else attention_mask[:, :, :, :ctx]
    return kpool, vpool, mask, dict(k_new=k_new, v_new=v_new, append_pos=pos, page_table=table, context_len=ctx)


def full_einsum_forward(query, key, value, attention_mask=None, is_causal=False, scaling=None):
    """Dense GQA decode with asymmetric key/value head counts -> [B, Hq, 1, D]."""
    if query.shape[2] != 1:
        raise NotImplementedError("saga_b200 full_einsum_forward serves decode (one query position)")
    pg = _paged(key, attention_mask)
    if pg is not None:
        return _ops.dense_decode(query, pg[0], pg[1], pg[2], _ops.scaling_or_default(query, scaling), **pg[3])
    pend = _pending(key)
    if pend is not None:
        return torch.ops.saga.dense_decode_append(query, key, value, _mask(attention_mask, key),
                                                  _ops.scaling_or_default(query, scaling), *pend)
    return torch.ops.saga.dense_decode(query, key, value, _mask(attention_mask, key),
                                       _ops.scaling_or_default(query, scaling))


# =============================================================================
# Atop-N amortized attention -- attention.py:92-209
# =============================================================================

MAX_LAYERS = 128
AMORTIZED_THRESHOLD_TENSOR: Optional[torch.Tensor] = None
EXEMPT_LAYERS: set = set()


def init_amortized_threshold_tensor(device, num_layers, num_rows):
    """attention.py:97-99: the [num_layers, num_rows] fp32 softmax-space thresholds."""
    global AMORTIZED_THRESHOLD_TENSOR
    AMORTIZED_THRESHOLD_TENSOR = torch.zeros(num_layers, num_rows, device=device, dtype=torch.float32)


def reset_amortized_state():
    """attention.py:102-105."""
    global AMORTIZED_THRESHOLD_TENSOR
    if AMORTIZED_THRESHOLD_TENSOR is not None:
        AMORTIZED_THRESHOLD_TENSOR.zero_()


def _threshold_topk_triton(x: torch.Tensor, k: int, threshold: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """attention.py:108-110 (the name is kept; the kernel is CUDA, not Triton)."""
    from .triton_atopn import threshold_topk_fast
    return threshold_topk_fast(x, k, threshold)


def _compute_attn_weights(query, key, scaling, attention_mask):
    """attention.py:113-128: logits [B, Hq, Lq, L] of the reduced key heads."""
    if query.shape[2] != 1:
        raise NotImplementedError("saga_b200 computes decode logits (one query position)")
    return torch.ops.saga.attn_logits(query, key, _mask(attention_mask, key),
                                      _ops.scaling_or_default(query, scaling))


def _compute_attn_probs(query, key, scaling, attention_mask):
    """attention.py:131-133."""
    return torch.nn.functional.softmax(_compute_attn_weights(query, key, scaling, attention_mask), dim=-1)


def _transform_softmax_threshold(attn_logits, softmax_threshold, tail_size=256):
    """attention.py:136-149: softmax-space threshold -> logit-space threshold."""
    return torch.ops.saga.transform_threshold(attn_logits, softmax_threshold, int(tail_size))


def _atopn_gather_and_output(attn_weights_topk, attn_indices, value, query_shape, top_n_attention,
                              input_is_logits=False):
    """attention.py:152-170: softmax (or renormalisation) of the buffer, V gather, output."""
    b, q_h, l_q, d = query_shape
    return _ops.gather_output(attn_weights_topk, attn_indices, value, q_h, input_is_logits)


def _threshold_row(layer_idx: int, num_rows: int) -> torch.Tensor:
    if AMORTIZED_THRESHOLD_TENSOR is None:
        raise RuntimeError("call init_amortized_threshold_tensor() first")
    return AMORTIZED_THRESHOLD_TENSOR[layer_idx, :num_rows]


def approx_top_n_attention_amortized_cal(query, key, value, attention_mask=None, is_causal=False,
                                          top_n_attention: int = 256, scaling=None, layer_idx: int = 0):
    """First decode step (attention.py:173-189): full softmax + exact top-N;
    stores the N-th largest probability of every row in
    AMORTIZED_THRESHOLD_TENSOR[layer_idx]."""
    b, q_h, l_q, d = query.shape
    thr = _threshold_row(layer_idx, b * q_h)
    pg = _paged(key, attention_mask)
    if pg is not None:
        return _ops.atopn_calibrate(query, pg[0], pg[1], pg[2], thr, int(top_n_attention),
                                    _ops.scaling_or_default(query, scaling), **pg[3])
    pend = _pending(key)
    if pend is not None:
        return torch.ops.saga.atopn_calibrate_append(query, key, value, _mask(attention_mask, key), thr,
                                                     int(top_n_attention), _ops.scaling_or_default(query, scaling),
                                                     *pend)
    return torch.ops.saga.atopn_calibrate(query, key, value, _mask(attention_mask, key), thr,
                                          int(top_n_attention), _ops.scaling_or_default(query, scaling))


def approx_top_n_attention_amortized(query, key, value, attention_mask=None, is_causal=False,
                                      top_n_attention: int = 256, scaling=None, layer_idx: int = 0):
    """Later decode steps (attention.py:192-209): cached thresholds, one fused kernel."""
    b, q_h, l_q, d = query.shape
    thr = _threshold_row(layer_idx, b * q_h)
    pg = _paged(key, attention_mask)
    if pg is not None:
        return _ops.atopn_decode(query, pg[0], pg[1], pg[2], thr, int(top_n_attention),
                                 _ops.scaling_or_default(query, scaling), **pg[3])
    pend = _pending(key)
    if pend is not None:
        return torch.ops.saga.atopn_decode_append(query, key, value, _mask(attention_mask, key), thr,
                                                  int(top_n_attention), _ops.scaling_or_default(query, scaling),
                                                  *pend)
    return torch.ops.saga.atopn_decode(query, key, value, _mask(attention_mask, key), thr,
                                       int(top_n_attention), _ops.scaling_or_default(query, scaling))
