"""CPU oracle for SAGA's decode-time attention path (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the arithmetic of the reference's decode
attention: ``attention/attention.py`` and ``attention/triton_atopn.py`` of
noamelata/SAGA. It is the checker that the CUDA path is compared against. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it. The product (``saga_b200``) never calls it.

Parity is pinned by golden fixtures made by running the reference itself on
CPU. The Triton kernel runs under ``TRITON_INTERPRET=1``. The fixtures live in
``tests/golden/`` and the script that made them is ``tests/golden/make_golden.py``.

Number formats. Arrays are float32 holding values representable in the
computation dtype ("bf16", "fp16" or "fp32"). Every place where the reference
produces a low-precision tensor is rounded with ``round_to``, so the rounding
chain of the reference is replayed step by step.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

# Kept local so the oracle depends on nothing but numpy.


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def round_to(dtype: str, x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    return x


TAIL_SIZE = 256  # attention.py:136 (tail_size default)


# ---------------------------------------------------------------------------
# Q.K^T logits -- attention.py:113-128 (_compute_attn_weights)
# ---------------------------------------------------------------------------

def attn_logits(q: np.ndarray, k: np.ndarray, dtype: str, scaling: Optional[float] = None,
                mask: Optional[np.ndarray] = None) -> np.ndarray:
    """Logits [B, Hq, 1, L] of the decode query against the key cache.

    attention.py:119-121: one bmm per (batch, key head) of the G = Hq/Hk query
    heads that share the key head against all L keys. The GEMM accumulates in
    fp32 and rounds once to the tensor dtype. attention.py:122 then multiplies
    by ``scaling`` (default 1/sqrt(D), attention.py:117) in fp32 and rounds
    again. attention.py:124-126 adds the mask sliced to L. A boolean mask adds
    1.0 where True and 0.0 where False, in the logits dtype.
    """
    B, Hq, Lq, D = q.shape
    Hk, L = k.shape[1], k.shape[2]
    G = Hq // Hk
    sc = 1.0 / math.sqrt(D) if scaling is None else scaling
    qg = q.reshape(B, Hk, G * Lq, D).astype(np.float64)
    acc = np.matmul(qg, np.swapaxes(k.astype(np.float64), -1, -2))  # [B, Hk, G, L]
    lg = round_to(dtype, acc.astype(np.float32))
    lg = round_to(dtype, lg * np.float32(sc))
    lg = lg.reshape(B, Hq, Lq, L)
    if mask is not None:
        m = np.asarray(mask)[..., :L]
        addend = m.astype(np.float32)
        lg = round_to(dtype, lg + addend)
    return lg


def softmax_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """torch.softmax over the last dim for a tensor of ``dtype``.

    fp32 internally: the max, the sum of exp(x - max), and exp(x - max)/sum. The
    result is rounded to the dtype.
    """
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        mx = x.max(axis=-1, keepdims=True)
        e = np.exp(x - mx)
        s = e.sum(axis=-1, keepdims=True, dtype=np.float32)
        return round_to(dtype, e / s)


# ---------------------------------------------------------------------------
# softmax-space -> logit-space threshold -- attention.py:136-149
# ---------------------------------------------------------------------------

def transform_threshold(logits2d: np.ndarray, softmax_thr: np.ndarray, dtype: str,
                        tail: int = TAIL_SIZE) -> Tuple[np.ndarray, dict]:
    """Per-row logit threshold ``t = m + log(max(thr, 1e-30) * s)``.

    attention.py:142-143: m is the max of the last ``tail`` logits (exact).
    attention.py:145: s = exp(logits - m).sum(-1). In a low-precision dtype the
    difference and the exp are each rounded to the dtype, the sum accumulates
    in fp32 and is rounded to the dtype. attention.py:147: ``thr.clamp(1e-30)``
    times s, then log and ``+ m``, all in fp32.
    Returns (t[R] float32, {"m": m, "s": s}).
    """
    x = np.asarray(logits2d, dtype=np.float32)
    L = x.shape[-1]
    tl = min(tail, L)
    m = x[:, L - tl:].max(axis=-1)
    with np.errstate(invalid="ignore", over="ignore"):
        d = round_to(dtype, x - m[:, None])
        e = round_to(dtype, np.exp(d))
        s = round_to(dtype, e.sum(axis=-1, dtype=np.float32))
        thr = np.maximum(np.asarray(softmax_thr, dtype=np.float32), np.float32(1e-30))
        t = (m + np.log(thr * s).astype(np.float32)).astype(np.float32)
    return t, {"m": m, "s": s}


# ---------------------------------------------------------------------------
# threshold selection -- triton_atopn.py:6-53 (kernel), 59-113 (wrapper)
# ---------------------------------------------------------------------------

def threshold_select(x2d: np.ndarray, t, k: int):
    """Per row, every element with ``x > t`` (strict, fp32 compare).

    triton_atopn.py:42 selects ``x_vals > threshold``. triton_atopn.py:46-53
    compacts the passing elements into ``k`` slots per row. The reference's
    slot order follows atomic block order, and when more than k pass it keeps an
    arbitrary k of them. This oracle uses ascending index order and keeps the
    k lowest indices. Padding is vals=-inf and idx=0 (triton_atopn.py:82-84).
    Returns (vals[R,k], idx[R,k] int64, count_passing[R], count_kept[R]).
    """
    x = np.asarray(x2d, dtype=np.float32)
    R, L = x.shape
    t = np.broadcast_to(np.asarray(t, dtype=np.float32).reshape(-1, 1) if np.ndim(t) else
                        np.float32(t), (R, 1))
    with np.errstate(invalid="ignore"):
        passing = x > t
    vals = np.full((R, k), -np.inf, dtype=np.float32)
    idx = np.zeros((R, k), dtype=np.int64)
    cnt = passing.sum(axis=-1).astype(np.int64)
    kept = np.minimum(cnt, k)
    for r in range(R):
        pos = np.nonzero(passing[r])[0][:k]
        vals[r, :len(pos)] = x[r, pos]
        idx[r, :len(pos)] = pos
    return vals, idx, cnt, kept


# ---------------------------------------------------------------------------
# sparse V gather + output -- attention.py:152-170
# ---------------------------------------------------------------------------

def gather_output(weights: np.ndarray, idx: np.ndarray, v: np.ndarray, B: int, Hq: int,
                  dtype: str, input_is_logits: bool) -> np.ndarray:
    """Output [B, Hq, 1, D] from per-row buffers of weights and key positions.

    attention.py:158-161: with ``input_is_logits`` the buffer is softmaxed (the
    -inf pads get weight 0). Otherwise the weights are divided by their sum,
    clamped to 1e-12, in the dtype. attention.py:163-168: query head h reads
    value head h // (Hq/Hv) at the buffer positions. A bmm with fp32
    accumulation rounds the result to the dtype.
    """
    Hv, D = v.shape[1], v.shape[3]
    Gv = Hq // Hv
    R, K = weights.shape
    w = np.asarray(weights, dtype=np.float32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        if input_is_logits:
            p = softmax_dtype(w, dtype)
        else:
            s = round_to(dtype, w.sum(axis=-1, keepdims=True, dtype=np.float32))
            p = round_to(dtype, w / np.maximum(s, np.float32(1e-12)))
    out = np.zeros((B, Hq, 1, D), dtype=np.float32)
    for b in range(B):
        for h in range(Hq):
            r = b * Hq + h
            rows = v[b, h // Gv][idx[r]].astype(np.float64)      # [K, D]
            with np.errstate(invalid="ignore"):
                acc = p[r].astype(np.float64) @ rows
            out[b, h, 0] = round_to(dtype, acc.astype(np.float32))
    return out


# ---------------------------------------------------------------------------
# decode steps
# ---------------------------------------------------------------------------

def atopn_amortized(q, k, v, softmax_thr_row: np.ndarray, top_n: int, dtype: str,
                    scaling=None, mask=None) -> dict:
    """Steady-state Atop-N step -- attention.py:192-209.

    logits (a2) -> logit threshold (a5) -> select with K = min(2N, L) (a6) ->
    softmax over the selected logits and V gather (a8).
    """
    B, Hq, _, D = q.shape
    L = k.shape[2]
    lg = attn_logits(q, k, dtype, scaling, mask)
    R = B * Hq
    lg2 = lg.reshape(R, L)
    t, st = transform_threshold(lg2, np.asarray(softmax_thr_row, dtype=np.float32)[:R], dtype)
    buf_k = min(top_n * 2, L)
    vals, idx, cnt, kept = threshold_select(lg2, t, buf_k)
    out = gather_output(vals, idx, v, B, Hq, dtype, input_is_logits=True)
    return {"logits": lg2, "t": t, "m": st["m"], "s": st["s"], "vals": vals, "idx": idx,
            "count": cnt, "kept": kept, "buf_k": buf_k, "out": out}


def topn_threshold(probs2d: np.ndarray, n: int):
    """The n-th largest value per row and the top-n set.

    attention.py:181-185 uses ``torch.topk(probs, n)``. The stored threshold
    is the last (smallest) of the top-n values. Ties at that value are broken
    here by ascending index; torch.topk may keep other members of the tie.
    Returns (pN[R], idx[R, n] ascending, n_greater[R]).
    """
    p = np.asarray(probs2d, dtype=np.float32)
    R, L = p.shape
    pn = np.partition(p, L - n, axis=-1)[:, L - n]
    idx = np.zeros((R, n), dtype=np.int64)
    ngt = np.zeros(R, dtype=np.int64)
    for r in range(R):
        gt = np.nonzero(p[r] > pn[r])[0]
        eq = np.nonzero(p[r] == pn[r])[0]
        ngt[r] = len(gt)
        sel = np.sort(np.concatenate([gt, eq[: n - len(gt)]]))
        idx[r] = sel
    return pn, idx, ngt


def atopn_calibrate(q, k, v, top_n: int, dtype: str, scaling=None, mask=None) -> dict:
    """Calibration step -- attention.py:173-189.

    Full softmax (attention.py:131-133), exact top-N probabilities
    (attention.py:181-182). The threshold written to the table is the N-th
    largest probability (attention.py:184-187). The output renormalises the
    top-N probabilities and gathers V (attention.py:160-161, 163-168).
    """
    B, Hq, _, D = q.shape
    L = k.shape[2]
    lg = attn_logits(q, k, dtype, scaling, mask)
    R = B * Hq
    probs = softmax_dtype(lg.reshape(R, L), dtype)
    n = min(top_n, L)
    pn, idx, ngt = topn_threshold(probs, n)
    w = np.take_along_axis(probs, idx, axis=-1)
    out = gather_output(w, idx, v, B, Hq, dtype, input_is_logits=False)
    return {"logits": lg.reshape(R, L), "probs": probs, "thr": pn.astype(np.float32),
            "idx": idx, "n_greater": ngt, "out": out}


def dense_decode(q, k, v, dtype: str, scaling=None, mask=None) -> np.ndarray:
    """Dense GQA decode -- attention.py:64-85 (full_einsum_forward).

    Same logits as above; softmax over all L in the dtype (attention.py:79).
    Then one bmm per (batch, value head) of its Gv = Hq/Hv query heads'
    probabilities against the value rows (attention.py:81-83).
    """
    B, Hq, Lq, D = q.shape
    Hv, L = v.shape[1], v.shape[2]
    Gv = Hq // Hv
    lg = attn_logits(q, k, dtype, scaling, mask)
    p = softmax_dtype(lg, dtype).reshape(B, Hv, Gv * Lq, L).astype(np.float64)
    out = np.matmul(p, v.astype(np.float64))                    # [B, Hv, Gv, D]
    return round_to(dtype, out.astype(np.float32)).reshape(B, Hq, Lq, D)


def kv_append(k_cache: np.ndarray, v_cache: np.ndarray, k_new: np.ndarray, v_new: np.ndarray,
              pos: int):
    """The static-cache append of one decode token: transformers'
    ``StaticLayer.update`` does ``index_copy_`` of the new K and V rows at the
    cache position along dim 2. speedup.py:119-139 builds that cache with
    independent key and value head counts."""
    k2, v2 = k_cache.copy(), v_cache.copy()
    k2[:, :, pos] = k_new[:, :, 0]
    v2[:, :, pos] = v_new[:, :, 0]
    return k2, v2
