"""The CPU oracle against golden vectors made by the reference itself.

The fixtures come from running noamelata/SAGA's ``attention/attention.py`` and
``attention/triton_atopn.py`` on CPU (``tests/golden/make_golden.py``). These
tests pin the oracle before it is used to check the CUDA path.
"""
import numpy as np
import pytest

from oracle import atopn_oracle as O
from _golden import load, golden_names, near_threshold_ok, rel_rms

NAMES = golden_names()
SMALL = [n for n in NAMES if n != "c2_bf16"]


@pytest.fixture(scope="module")
def cache():
    return {}


def _get(cache, name):
    if name not in cache:
        g = load(name)
        cache[name] = (g, g.inputs())
    return cache[name]


@pytest.mark.parametrize("name", SMALL)
def test_logits_match_reference(cache, name):
    g, inp = _get(cache, name)
    dt = g.shape.dtype
    lg0 = O.attn_logits(inp.q0, inp.k, dt, mask=g.mask()).reshape(g.shape.rows, -1)
    ref = g["logits0"]
    if dt == "fp32":
        np.testing.assert_allclose(lg0, ref, rtol=1e-5, atol=1e-5)
    else:
        d = lg0 != ref
        # GEMM accumulation order may move the fp32 dot product across a rounding
        # boundary (1 ulp of the raw product); the second rounding after
        # ``* scaling`` can turn that into up to 2 ulps of the final logit.
        assert d.mean() < 1e-3, d.mean()
        from _golden import ulp
        assert np.all(np.abs(lg0 - ref)[d] <= 2 * ulp(ref[d], dt) * 1.0001)


@pytest.mark.parametrize("name", SMALL)
def test_threshold_transform_and_selection(cache, name):
    """Given the reference's own logits, the oracle's logit threshold and its
    selected set equal the reference's."""
    g, _ = _get(cache, name)
    dt = g.shape.dtype
    lg1 = g["logits1"]
    t, _ = O.transform_threshold(lg1, g["thr_used"], dt)
    np.testing.assert_allclose(t, g["t1"], rtol=2e-6, atol=0)
    buf_k = g.meta["buf_k"]
    vals, idx, cnt, kept = O.threshold_select(lg1, g["t1"], buf_k)
    np.testing.assert_array_equal(cnt, g["passing"])
    np.testing.assert_array_equal(kept, g["sel_kept"])
    for r in range(g.shape.rows):
        ref = g["sel_idx"][r, :g["sel_kept"][r]].astype(np.int64)
        if g["passing"][r] <= buf_k:
            np.testing.assert_array_equal(idx[r, :kept[r]], ref)
        else:
            # Overflow: the reference keeps an arbitrary buf_k of the passing set.
            assert len(set(ref.tolist())) == buf_k
            assert np.all(lg1[r, ref] > g["t1"][r])


@pytest.mark.parametrize("name", SMALL)
def test_amortized_output(cache, name):
    g, inp = _get(cache, name)
    dt = g.shape.dtype
    k1, v1 = g.step1_cache(inp)
    R, D = g.shape.rows, g.shape.D
    lg1 = g["logits1"]
    kk = g.meta["buf_k"]
    # Gather on the reference's own selection: must agree to rounding.
    sel = g["sel_idx"].astype(np.int64)
    vals = np.full((R, kk), -np.inf, np.float32)
    for r in range(R):
        n = g["sel_kept"][r]
        vals[r, :n] = lg1[r, sel[r, :n]]
    out = O.gather_output(vals, sel, v1, g.shape.B, g.shape.Hq, dt, True).reshape(R, D)
    tol = 1e-5 if dt == "fp32" else 1e-2
    assert np.nanmax(np.abs(out - g["out1"])) <= tol
    # The whole oracle step from the inputs.
    res = O.atopn_amortized(inp.q1, k1, v1, g["thr_used"], g.shape.N, dt, mask=g.mask())
    if name != "overflow_bf16":
        assert np.abs(res["out"].reshape(R, D) - g["out1"]).max() <= (1e-4 if dt == "fp32" else 2e-2)


@pytest.mark.parametrize("name", SMALL)
def test_calibration(cache, name):
    g, inp = _get(cache, name)
    dt = g.shape.dtype
    R, D = g.shape.rows, g.shape.D
    cal = O.atopn_calibrate(inp.q0, inp.k, inp.v, g.shape.N, dt, mask=g.mask())
    if dt == "fp32":
        np.testing.assert_allclose(cal["thr"], g["thr"], rtol=1e-4)
    else:
        assert (cal["thr"] == g["thr"]).mean() >= 0.95
    # Output on the reference's own top-N set matches to rounding.
    ref_idx = g["ref_top_idx"].astype(np.int64)
    probs = O.softmax_dtype(g["logits0"], dt) if g.has("logits0") else cal["probs"]
    w = np.take_along_axis(probs, ref_idx, axis=-1)
    out = O.gather_output(w, ref_idx, inp.v, g.shape.B, g.shape.Hq, dt, False).reshape(R, D)
    assert np.abs(out - g["out0"]).max() <= (1e-5 if dt == "fp32" else 1e-2)
    # The oracle breaks ties at the N-th probability by ascending index (as a
    # GPU radix top-k does); CPU torch.topk keeps another subset of the tie.
    # Rows with the same set match the reference's output; rows that differ
    # may differ only in members of the tie.
    if dt == "fp32":
        return
    ours_out = cal["out"].reshape(R, D)
    for r in range(R):
        a, b = set(cal["idx"][r].tolist()), set(ref_idx[r].tolist())
        if a == b:
            assert np.abs(ours_out[r] - g["out0"][r]).max() <= 1e-2
        else:
            sym = np.array(sorted(a ^ b))
            assert np.all(cal["probs"][r, sym] == cal["thr"][r]), r


@pytest.mark.parametrize("name", SMALL)
def test_dense(cache, name):
    g, inp = _get(cache, name)
    dt = g.shape.dtype
    k1, v1 = g.step1_cache(inp)
    out = O.dense_decode(inp.q1, k1, v1, dt, mask=g.mask()).reshape(g.shape.rows, g.shape.D)
    assert np.abs(out - g["dense"]).max() <= (1e-5 if dt == "fp32" else 1e-2)


def test_config2_full_pipeline(cache):
    """Config 2 (B=8, L=32768, bf16): the oracle from the inputs alone against
    the reference's threshold table, logit thresholds, selections and outputs."""
    g, inp = _get(cache, "c2_bf16")
    dt = "bf16"
    R, D, N = g.shape.rows, g.shape.D, g.shape.N
    cal = O.atopn_calibrate(inp.q0, inp.k, inp.v, N, dt)
    assert (cal["thr"] == g["thr"]).mean() >= 0.95
    assert np.abs(cal["out"].reshape(R, D) - g["out0"]).max() <= 2e-2
    k1, v1 = g.step1_cache(inp)
    res = O.atopn_amortized(inp.q1, k1, v1, g["thr_used"], N, dt)
    np.testing.assert_allclose(res["t"], g["t1"], rtol=1e-5)
    lg1 = res["logits"]
    for r in range(R):
        ours = set(res["idx"][r, :res["kept"][r]].tolist())
        ref = set(g["sel_idx"][r, :g["sel_kept"][r]].astype(np.int64).tolist())
        assert near_threshold_ok(lg1[r], g["t1"][r], ours ^ ref, dt), r
    out = res["out"].reshape(R, D)
    assert np.abs(out - g["out1"]).max() <= 2e-2
    assert rel_rms(out, g["out1"]) <= 1e-2
