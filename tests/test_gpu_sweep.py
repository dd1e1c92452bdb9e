"""A sweep of kernel configurations against the CPU oracle.

dtype (bf16, fp16, fp32) x head_dim (64, 128) x head layouts (G = Hq / Hk
from 1 to 32; Hv below, equal to and above Hk) x (batch, context, N, mask).
That gives 144 seeded cases, each running the calibration step, the
amortized step on the calibrated thresholds, and dense decode. The golden
fixtures pin the reference's own shapes; this sweep covers the kernel's other
paths. These are the tensor-core and CUDA-core scorers, the tensor-core and
CUDA-core P.V, and one-batch and multi-batch value-row gathers.

Tolerances are those of the parity tests: 16-bit max-abs 2e-2, fp32 1e-4.
Thresholds must be equal (16-bit) or within 1e-6 (fp32). In calibration, a
row whose top-N set differs from the oracle's must differ only in positions
whose probability is within 4 fp32 ulps of the N-th largest. In the amortized
step, positions whose logit sits on the threshold can fall either way (the
N-th position's logit equals t up to rounding, and logits may differ from the
oracle's by an ulp): a row whose selected set differs from the oracle's must
differ only in positions within 1 ulp (16-bit) or 2e-5 (fp32) of t, and is
then not compared; every other row must match within the tolerance.
"""
import numpy as np
import pytest
import torch

from oracle import atopn_oracle as O
from _golden import near_threshold_ok

pytestmark = pytest.mark.gpu

FP32_LOGIT_TOL = 2e-5  # fp32 logits of two GEMM orders differ by ~1e-6
LAYOUTS = [(12, 1, 2), (8, 2, 4), (16, 1, 1), (20, 1, 2), (32, 1, 2), (4, 4, 4), (24, 2, 3), (6, 3, 1)]
SIZES = [(1, 300, 16, False), (3, 1700, 64, True), (2, 5000, 512, False)]


def _cases():
    for dt in ("bf16", "fp16", "fp32"):
        for d in (64, 128):
            for lay in LAYOUTS:
                yield dt, d, lay


@pytest.mark.parametrize("dt,d,lay", list(_cases()))
def test_configuration_against_oracle(dt, d, lay):
    from saga_b200 import ops
    dev = torch.device("cuda", 0)
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dt]
    hq, hk, hv = lay
    tol = 1e-4 if dt == "fp32" else 2e-2
    for b, length, n, with_mask in SIZES:
        g = torch.Generator(device=dev).manual_seed(d * 1000 + hq * 10 + length)
        q = (torch.randn((b, hq, 1, d), generator=g, device=dev) * 0.5).to(tdt)
        k = (torch.randn((b, hk, length, d), generator=g, device=dev) * 0.5).to(tdt)
        v = (torch.randn((b, hv, length, d), generator=g, device=dev) * 0.5).to(tdt)
        mask = (torch.rand((b, 1, 1, length), generator=g, device=dev) > 0.1) if with_mask else None
        qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
        mn = None if mask is None else mask.cpu().numpy()
        case = (dt, d, lay, b, length, n, with_mask)

        thr = torch.zeros(b * hq, dtype=torch.float32, device=dev)
        diag = {}
        out = ops.atopn_calibrate(q, k, v, mask, thr, n, diag=diag)
        ref = O.atopn_calibrate(qn, kn, vn, n, dt, mask=mn)
        assert np.abs(thr.cpu().numpy() - ref["thr"]).max() <= (1e-6 if dt == "fp32" else 0.0), case
        err = np.abs(out.float().cpu().numpy().reshape(b * hq, d) - ref["out"].reshape(b * hq, d)).max(-1)
        sel, nn = diag["sel_idx"].cpu().numpy(), min(n, length)
        for r in range(b * hq):
            diff = set(sel[r, :nn].tolist()) ^ set(ref["idx"][r].tolist())
            if diff:  # a tie at the N-th probability: the positions that differ sit on it
                ps = ref["probs"][r, sorted(diff)]
                assert np.all(np.abs(ps - ref["thr"][r]) <= 4 * np.spacing(np.float32(ref["thr"][r]))), (case, r)
            else:
                assert err[r] <= tol, (case, r, err[r])

        diag = {}
        out = ops.atopn_decode(q, k, v, mask, thr, n, diag=diag)
        ref = O.atopn_amortized(qn, kn, vn, thr.cpu().numpy(), n, dt, mask=mn)
        err = np.abs(out.float().cpu().numpy().reshape(b * hq, d) - ref["out"].reshape(b * hq, d)).max(-1)
        cnt, sel = diag["count"].cpu().numpy(), diag["sel_idx"].cpu().numpy()
        for r in range(b * hq):
            ours = set(sel[r, :min(int(cnt[r]), ref["buf_k"])].tolist())
            theirs = set(ref["idx"][r, :min(int(ref["count"][r]), ref["buf_k"])].tolist())
            diff = ours ^ theirs
            if diff:  # a tie at the threshold: the positions that differ sit on it
                if dt == "fp32":
                    xs = ref["logits"][r, sorted(diff)]
                    assert np.all(np.abs(xs - ref["t"][r]) <= FP32_LOGIT_TOL), (case, r)
                else:
                    assert near_threshold_ok(ref["logits"][r], ref["t"][r], diff, dt), (case, r)
            else:
                assert err[r] <= tol, (case, r, err[r])

        ref = O.dense_decode(qn, kn, vn, dt, mask=mn)
        out = ops.dense_decode(q, k, v, mask)
        assert np.abs(out.float().cpu().numpy().reshape(ref.shape) - ref).max() <= tol, case
    assert ops.read_status(dev) & 0x1 == 0


def test_wide_fp32_groups_use_the_whole_shared_memory():
    """fp32 with G = 32 at head_dim 128 does not fit two CTAs per SM: the plan
    falls back to one CTA per SM with all of its shared memory."""
    from saga_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn((2, 32, 1, 128), generator=g, device=dev) * 0.5
    k = torch.randn((2, 1, 1700, 128), generator=g, device=dev) * 0.5
    v = torch.randn((2, 2, 1700, 128), generator=g, device=dev) * 0.5
    ref = O.dense_decode(*(x.cpu().numpy() for x in (q, k, v)), "fp32")
    assert np.abs(ops.dense_decode(q, k, v).cpu().numpy() - ref).max() <= 1e-4
    thr = torch.zeros(64, dtype=torch.float32, device=dev)
    out = ops.atopn_calibrate(q, k, v, None, thr, 64)
    rc = O.atopn_calibrate(*(x.cpu().numpy() for x in (q, k, v)), 64, "fp32")
    assert np.abs(thr.cpu().numpy() - rc["thr"]).max() <= 1e-6
    assert np.isfinite(out.cpu().numpy()).all()
