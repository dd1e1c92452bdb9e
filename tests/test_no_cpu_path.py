"""The product path has no CPU fallback: every op refuses host tensors.

The decode ops and the drop-in attention functions (attention.py:64-85,
173-209 of the reference) are served only by the CUDA library; given CPU
tensors they raise instead of computing a result some other way.
"""
import pytest
import torch


def _inputs():
    g = torch.Generator().manual_seed(3)
    q = torch.randn((1, 4, 1, 64), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 1, 256, 64), generator=g).to(torch.bfloat16)
    v = torch.randn((1, 2, 256, 64), generator=g).to(torch.bfloat16)
    thr = torch.zeros(4, dtype=torch.float32)
    return q, k, v, thr


@pytest.mark.parametrize("op", ["dense", "atopn", "calibrate", "logits"])
def test_ops_refuse_host_tensors(op):
    from saga_b200 import ops
    q, k, v, thr = _inputs()
    call = {"dense": lambda: ops.dense_decode(q, k, v),
            "atopn": lambda: ops.atopn_decode(q, k, v, None, thr, 16),
            "calibrate": lambda: ops.atopn_calibrate(q, k, v, None, thr, 16),
            "logits": lambda: ops.attn_logits(q, k)}[op]
    with pytest.raises(ValueError, match="no CPU path"):
        call()


@pytest.mark.parametrize("fn", ["full_einsum_forward", "approx_top_n_attention_amortized",
                                "approx_top_n_attention_amortized_cal"])
def test_dropin_functions_refuse_host_tensors(fn):
    from saga_b200.attention import attention as A
    q, k, v, _ = _inputs()
    saved = A.AMORTIZED_THRESHOLD_TENSOR
    try:
        A.init_amortized_threshold_tensor("cpu", 1, q.shape[0] * q.shape[1])
        with pytest.raises(ValueError, match="no CPU path"):
            getattr(A, fn)(q, k, v, None)
    finally:
        A.AMORTIZED_THRESHOLD_TENSOR = saved


@pytest.mark.parametrize("op", ["dense", "atopn", "calibrate"])
def test_decode_step_refuses_host_tensors(op):
    from saga_b200 import ops
    q, k, v, thr = _inputs()
    with pytest.raises(ValueError, match="no CPU path"):
        ops.DecodeStep(op, q, k, v, threshold=thr, top_n=16)
