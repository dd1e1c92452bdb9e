"""ops.DecodeStep (a decode op bound to fixed buffers) against the per-call functions.

The bound step runs the same kernels with the same arguments, so its outputs
and calibrated thresholds must be bit-identical to ``atopn_decode`` /
``atopn_calibrate`` / ``dense_decode`` on the same inputs, including after the
query buffer is refilled in place, and with the decode token appended.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

B, Hq, Hk, Hv, L, D, N = 4, 12, 1, 2, 6000, 128, 128


def _inputs(dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B, Hq, 1, D), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((B, Hk, L, D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((B, Hv, L, D), generator=g, device=dev).to(torch.bfloat16)
    kn = torch.randn((B, Hk, 1, D), generator=g, device=dev).to(torch.bfloat16)
    vn = torch.randn((B, Hv, 1, D), generator=g, device=dev).to(torch.bfloat16)
    return q, k, v, kn, vn


def test_bound_steps_match_the_per_call_functions():
    from saga_b200 import ops
    dev = torch.device("cuda", 0)
    q, k, v, kn, vn = _inputs(dev, 5)
    q2 = _inputs(dev, 6)[0]
    thr_ref = torch.zeros(B * Hq, dtype=torch.float32, device=dev)
    thr = torch.zeros_like(thr_ref)
    ref_c = ops.atopn_calibrate(q, k, v, None, thr_ref, N)
    qbuf = q.clone()
    cal = ops.DecodeStep("calibrate", qbuf, k, v, threshold=thr, top_n=N)
    out_c = cal()
    torch.cuda.synchronize()
    assert torch.equal(out_c, ref_c) and torch.equal(thr, thr_ref)

    step = ops.DecodeStep("atopn", qbuf, k, v, threshold=thr, top_n=N)
    dense = ops.DecodeStep("dense", qbuf, k, v)
    for qi in (q, q2, q):
        qbuf.copy_(qi)
        assert torch.equal(step().clone(), ops.atopn_decode(qi, k, v, None, thr, N))
        assert torch.equal(dense().clone(), ops.dense_decode(qi, k, v))
    assert ops.read_status(dev) & 0x1 == 0

    # the fused append of the decode token at a position held on the device
    k1, v1, k2, v2 = k.clone(), v.clone(), k.clone(), v.clone()
    pos = torch.tensor([L - 1], dtype=torch.int64, device=dev)
    app = ops.DecodeStep("atopn", qbuf, k1, v1, threshold=thr, top_n=N, k_new=kn, v_new=vn, append_pos=pos)
    o1 = app().clone()
    o2 = ops.atopn_decode(qbuf, k2, v2, None, thr, N, k_new=kn, v_new=vn, append_pos=L - 1)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(k1, k2) and torch.equal(v1, v2)


def test_bound_step_checks_its_buffers():
    from saga_b200 import ops
    dev = torch.device("cuda", 0)
    q, k, v, _, _ = _inputs(dev, 7)
    with pytest.raises(ValueError):
        ops.DecodeStep("topk", q, k, v)
    with pytest.raises(ValueError):
        ops.DecodeStep("atopn", q, k, v)  # no threshold
    with pytest.raises(ValueError):
        ops.DecodeStep("dense", q, k, v, out=torch.empty((B, Hq, 2, D), dtype=q.dtype, device=dev))
