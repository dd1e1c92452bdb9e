"""Padded batches in the oracle: what the reference's steps give per padding side.

The amortized step's stabiliser m is the maximum of the row's last 256 logits
(attention.py:142-143). A row padded on the right, with its last 256 positions
masked, has m = -inf, so s = sum exp(l - m) is inf or NaN and the logit
threshold t = m + log(thr * s) is NaN: nothing passes x > t and the output is
NaN. A row padded on the left keeps its tail and is finite. Dense decode and
calibration take the softmax over the whole row and are finite on both sides.
The fused kernels follow the same behaviour (their GPU tests pad accordingly).
"""
import numpy as np

from oracle import atopn_oracle as O


def _case(seed=5):
    rng = np.random.default_rng(seed)
    B, Hq, Hk, Hv, D, L = 2, 4, 1, 2, 64, 1024
    q = O.bf16_round(rng.standard_normal((B, Hq, 1, D)).astype(np.float32) * 0.5)
    k = O.bf16_round(rng.standard_normal((B, Hk, L, D)).astype(np.float32) * 0.5)
    v = O.bf16_round(rng.standard_normal((B, Hv, L, D)).astype(np.float32) * 0.5)
    mask = np.zeros((B, 1, 1, L), dtype=np.float32)
    mask[0, ..., L - 300:] = -np.inf  # row 0: padded on the right
    mask[1, ..., :300] = -np.inf      # row 1: padded on the left
    return q, k, v, mask, Hq


def test_amortized_right_padding_is_nan_left_padding_finite():
    q, k, v, mask, Hq = _case()
    thr = np.full(q.shape[0] * Hq, 1e-4, dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        r = O.atopn_amortized(q, k, v, thr, 64, "bf16", mask=mask)
    assert np.all(r["m"][:Hq] == -np.inf)
    assert np.all(np.isnan(r["t"][:Hq]))
    assert np.all(r["count"][:Hq] == 0)
    assert np.all(np.isnan(r["out"][0]))
    assert np.all(np.isfinite(r["t"][Hq:]))
    assert np.all(np.isfinite(r["out"][1]))


def test_dense_and_calibration_finite_on_both_sides():
    q, k, v, mask, Hq = _case()
    out = O.dense_decode(q, k, v, "bf16", mask=mask)
    assert np.all(np.isfinite(out))
    cal = O.atopn_calibrate(q, k, v, 64, "bf16", mask=mask)
    assert np.all(np.isfinite(cal["out"]))
    assert np.all(np.isfinite(cal["thr"])) and np.all(cal["thr"] > 0)
    # masked positions carry probability 0 and are never among the top N
    L = k.shape[2]
    idx = cal["idx"].reshape(2, Hq, -1)
    assert np.all(idx[0] < L - 300) and np.all(idx[1] >= 300)
