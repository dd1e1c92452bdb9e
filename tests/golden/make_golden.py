"""Generate golden fixtures by running the reference's own decode attention.

Runs ``attention/attention.py`` and ``attention/triton_atopn.py`` of
noamelata/SAGA on CPU. The Triton kernel runs under ``TRITON_INTERPRET=1``. The
inputs come from ``saga_b200.workloads.make_inputs`` (seeded numpy PCG64), so a
fixture stores the seed, the shape and a digest of the inputs, not the inputs.

The protocol of one case:
  step 0 (calibration) on (q0, K, V):
      approx_top_n_attention_amortized_cal -> out0 and the threshold table row
  step 1 (amortized) on (q1, K', V'), where K', V' have the new token at L-1:
      _compute_attn_weights -> logits1, _transform_softmax_threshold -> t1,
      threshold_topk_fast -> selected positions,
      approx_top_n_attention_amortized -> out1
  dense: full_einsum_forward(q1, K', V') -> out_dense

Usage: python tests/golden/make_golden.py [--reference PATH] [--only NAME]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"   # before any triton import

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402

from saga_b200.workloads import (DecodeShape, CONFIG1, CONFIG2, make_inputs,  # noqa: E402
                                 input_digest, to_torch, bool_decode_mask)

# name -> (shape, seed, options)
CASES = {
    "c1_fp32": (CONFIG1, 0, {}),
    "c2_bf16": (CONFIG2, 0, {"save_logits": False}),
    "odd_bf16": (DecodeShape(B=2, L=3000, Hq=12, Hk=1, Hv=2, D=128, N=256, dtype="bf16",
                             scale=0.5, plant=32), 1, {}),
    "mask_hk2_bf16": (DecodeShape(B=2, L=2000, Hq=8, Hk=2, Hv=4, D=64, N=128, dtype="bf16",
                                  scale=0.5, plant=16), 2, {"mask_filled": 1900}),
    "tiny_bf16": (DecodeShape(B=1, L=100, Hq=4, Hk=1, Hv=2, D=64, N=64, dtype="bf16",
                              scale=0.5, plant=4), 3, {}),
    "overflow_bf16": (DecodeShape(B=1, L=4096, Hq=6, Hk=1, Hv=3, D=128, N=64, dtype="bf16",
                                  scale=0.5, plant=8), 4, {"thr_scale": 1e-3}),
    "fp16": (DecodeShape(B=1, L=2048, Hq=8, Hk=1, Hv=2, D=128, N=128, dtype="fp16",
                         scale=0.5, plant=16), 5, {}),
    "hv_lt_hk_bf16": (DecodeShape(B=1, L=1536, Hq=8, Hk=4, Hv=2, D=64, N=96, dtype="bf16",
                                  scale=0.5, plant=8), 6, {}),
}


def _f32(t):
    return t.detach().float().numpy()


def run_case(A, tt, name, shape, seed, opts):
    import torch
    inp = make_inputs(shape, seed)
    dt = shape.dtype
    R, L = shape.rows, shape.L
    q0, q1 = to_torch(inp.q0, dt), to_torch(inp.q1, dt)
    k, v = to_torch(inp.k, dt), to_torch(inp.v, dt)
    # step-1 cache: new token appended at position L-1 (StaticLayer.update's index_copy_)
    pos = L - 1
    k1, v1 = k.clone(), v.clone()
    k1.index_copy_(2, torch.tensor([pos]), to_torch(inp.k_new, dt))
    v1.index_copy_(2, torch.tensor([pos]), to_torch(inp.v_new, dt))
    mask = None
    if "mask_filled" in opts:
        mask = torch.from_numpy(bool_decode_mask(shape.B, L, opts["mask_filled"]))

    A.init_amortized_threshold_tensor("cpu", A.MAX_LAYERS, R)
    out0 = A.approx_top_n_attention_amortized_cal(q0, k, v, mask, top_n_attention=shape.N,
                                                  layer_idx=0)
    thr = A.AMORTIZED_THRESHOLD_TENSOR[0, :R].clone()
    probs0 = A._compute_attn_probs(q0, k, None, mask)
    n = min(shape.N, L)
    _, topi = torch.topk(probs0, n, dim=-1)
    topi = np.sort(topi.reshape(R, n).numpy(), axis=-1)
    if "thr_scale" in opts:
        A.AMORTIZED_THRESHOLD_TENSOR[0, :R] *= opts["thr_scale"]
    thr_used = A.AMORTIZED_THRESHOLD_TENSOR[0, :R].clone()

    logits1 = A._compute_attn_weights(q1, k1, None, mask)
    t1 = A._transform_softmax_threshold(logits1, thr_used)
    buf_k = min(2 * shape.N, L)
    vals, idx = tt.threshold_topk_fast(logits1, buf_k, t1)
    vals = _f32(vals).reshape(R, buf_k)
    idx = idx.reshape(R, buf_k).numpy()
    kept = (vals > -np.inf).sum(-1)
    sel = np.zeros((R, buf_k), dtype=np.int64)
    for r in range(R):
        sel[r, :kept[r]] = np.sort(idx[r, :kept[r]])
    lg1 = _f32(logits1).reshape(R, L)
    passing = (lg1 > _f32(t1)[:, None]).sum(-1)
    out1 = A.approx_top_n_attention_amortized(q1, k1, v1, mask, top_n_attention=shape.N,
                                              layer_idx=0)
    dense = A.full_einsum_forward(q1, k1, v1, mask)

    meta = {"name": name, "shape": shape.as_dict(), "seed": seed, "opts": opts,
            "digest": input_digest(inp), "append_pos": pos, "buf_k": buf_k, "top_n_k": n,
            "torch": torch.__version__}
    try:
        import transformers
        meta["transformers"] = transformers.__version__
    except Exception:
        pass
    idx_dtype = np.uint16 if L <= 65535 else np.int32
    data = {
        "meta": np.array(json.dumps(meta)),
        "thr": _f32(thr),
        "thr_used": _f32(thr_used),
        "ref_top_idx": topi.astype(idx_dtype),
        "out0": _f32(out0).reshape(R, shape.D),
        "t1": _f32(t1),
        "sel_idx": sel.astype(idx_dtype),
        "sel_kept": kept.astype(np.int32),
        "passing": passing.astype(np.int32),
        "out1": _f32(out1).reshape(R, shape.D),
        "dense": _f32(dense).reshape(R, shape.D),
    }
    if opts.get("save_logits", True):
        data["logits0"] = _f32(A._compute_attn_weights(q0, k, None, mask)).reshape(R, L)
        data["logits1"] = lg1
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **data)
    print(f"{name}: wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB) "
          f"passing[:4]={passing[:4].tolist()} kept[:4]={kept[:4].tolist()}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SAGA_REFERENCE"),
                    help="checkout of noamelata/SAGA (or set SAGA_REFERENCE)")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    if not a.reference:
        ap.error("pass --reference <SAGA checkout> or set SAGA_REFERENCE")
    sys.path.insert(0, a.reference)
    import torch
    torch.manual_seed(0)
    import attention.attention as A          # the reference module
    import attention.triton_atopn as tt      # the reference Triton kernel (interpreted)
    assert os.path.abspath(os.path.dirname(A.__file__)).startswith(os.path.abspath(a.reference))
    for name, (shape, seed, opts) in CASES.items():
        if a.only and name != a.only:
            continue
        run_case(A, tt, name, shape, seed, opts)


if __name__ == "__main__":
    main()
