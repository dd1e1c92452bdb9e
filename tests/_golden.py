"""Loading and comparing golden fixtures (shared by the CPU and GPU tests)."""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import numpy as np

from saga_b200.workloads import DecodeShape, make_inputs, input_digest

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@dataclass
class Golden:
    name: str
    meta: dict
    shape: DecodeShape
    data: dict

    def __getitem__(self, k):
        return self.data[k]

    def has(self, k):
        return k in self.data

    def inputs(self):
        inp = make_inputs(self.shape, self.meta["seed"])
        if input_digest(inp) != self.meta["digest"]:
            raise AssertionError(f"{self.name}: input generator changed (digest mismatch)")
        return inp

    def mask(self):
        from saga_b200.workloads import bool_decode_mask
        f = self.meta["opts"].get("mask_filled")
        return None if f is None else bool_decode_mask(self.shape.B, self.shape.L, f)

    def step1_cache(self, inp):
        """(K', V') with the new token at ``append_pos``, as in the fixture."""
        pos = self.meta["append_pos"]
        k1, v1 = inp.k.copy(), inp.v.copy()
        k1[:, :, pos] = inp.k_new[:, :, 0]
        v1[:, :, pos] = inp.v_new[:, :, 0]
        return k1, v1


def golden_names():
    return sorted(f[:-4] for f in os.listdir(GOLDEN_DIR) if f.endswith(".npz"))


def load(name: str) -> Golden:
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    data = {k: z[k] for k in z.files if k != "meta"}
    meta = json.loads(str(z["meta"]))
    return Golden(name=name, meta=meta, shape=DecodeShape(**meta["shape"]), data=data)


def ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of the number format at |x| (for x != 0)."""
    x = np.abs(np.asarray(x, dtype=np.float32))
    mant = {"bf16": 7, "fp16": 10, "fp32": 23}[dtype]
    e = np.floor(np.log2(np.maximum(x, np.float32(1e-30))))
    if dtype == "fp16":
        e = np.maximum(e, -14)
    return np.exp2(e - mant).astype(np.float32)


def near_threshold_ok(x_row: np.ndarray, t: float, diff_idx, dtype: str, n_ulps: float = 1.0):
    """True when every position in ``diff_idx`` has a logit within ``n_ulps``
    (in the logits' own format) of the threshold ``t``."""
    if len(diff_idx) == 0:
        return True
    xs = x_row[np.asarray(list(diff_idx), dtype=np.int64)]
    tol = n_ulps * np.maximum(ulp(xs, dtype), ulp(np.float32(t), dtype))
    return bool(np.all(np.abs(xs - np.float32(t)) <= tol))


def calib_row_ok(probs_row: np.ndarray, pn: float, thr: float, ours, ref, dtype: str):
    """One row of a calibration step against a checker that ran on the same
    logits. ``probs_row`` and ``pn`` are the checker's probabilities and N-th
    largest probability, ``thr`` the kernel's threshold; ``ours`` / ``ref`` are
    the kept positions. Two exp / sum implementations can round a probability
    one ulp apart, so the rule is the parity bar with no allowance beyond that:
    the thresholds are equal or one ulp apart, and every position kept by one
    side only has a probability within one ulp of pN (a tie at the threshold).
    Returns (ok, reason)."""
    pn = np.float32(pn)
    thr = np.float32(thr)
    if dtype == "fp32":
        tol = np.float32(1e-5) * abs(pn) + ulp(pn, "fp32")
    else:
        tol = ulp(pn, dtype)
    if abs(thr - pn) > tol:
        return False, f"threshold {thr!r} vs {pn!r}: more than one ulp apart"
    d = np.asarray(sorted(set(np.asarray(ours).tolist()) ^ set(np.asarray(ref).tolist())), dtype=np.int64)
    if len(d):
        off = np.abs(probs_row[d] - pn)
        if not np.all(off <= tol):
            bad = d[off > tol]
            return False, f"positions {bad[:8].tolist()} kept by one side only are not ties at pN"
    return True, ""


def amortized_set_ok(lg_ref: np.ndarray, lg_ours: np.ndarray, t: float, ours, ref, dtype: str, fp32_tol: float):
    """Selected sets of one amortized row. A position kept by one side only is
    allowed when its reference logit lies within one ulp of the threshold t (a
    tie), or when the kernel's own logit for it differs from the reference's
    (the GEMM accumulation order, bounded by the logits test) by at least the
    distance of the reference logit from t beyond that ulp. Nothing else may
    differ."""
    d = np.asarray(sorted(set(np.asarray(ours).tolist()) ^ set(np.asarray(ref).tolist())), dtype=np.int64)
    if len(d) == 0:
        return True
    xr = lg_ref[d].astype(np.float32)
    xo = lg_ours[d].astype(np.float32)
    t = np.float32(t)
    if dtype == "fp32":
        tie = np.float32(fp32_tol)
    else:
        tie = np.maximum(ulp(xr, dtype), ulp(t, dtype))
    dist = np.abs(xr - t)
    return bool(np.all(dist <= tie + np.abs(xo - xr)))


def rel_rms(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / max(np.sqrt(np.mean(b ** 2)), 1e-30))
