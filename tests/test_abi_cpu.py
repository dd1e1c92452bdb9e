"""Host-side checks of the C ABI that need no GPU.

* libsaga_b200.so loads and exports every function include/saga_b200.h declares;
* the ctypes mirror of SagaAttnArgs has the C layout (checked against gcc);
* invalid requests are rejected on the host with SAGA_ERR_* and a message,
  before any CUDA call.
"""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from saga_b200 import _lib as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "saga_b200.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"SAGA_API\s+[\w\s\*]+?\b(saga_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L.lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    assert set(names) <= exported
    assert set(L.SIGNATURES) == set(names)


def test_version():
    assert "sm_100a" in L.version()


def test_struct_layout_matches_c():
    fields = [f for f, _ in L.SagaAttnArgs._fields_]
    prog = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
            'printf("%zu\\n", sizeof(SagaAttnArgs));']
    prog += [f'printf("%zu\\n", offsetof(SagaAttnArgs, {f}));' for f in fields]
    prog += ["return 0;}"]
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(c, "w").write("\n".join(prog))
        subprocess.run(["gcc", "-std=c99", c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(L.SagaAttnArgs)
    for f, off in zip(fields, vals[1:]):
        assert getattr(L.SagaAttnArgs, f).offset == off, f


def _args(**kw):
    a = L.SagaAttnArgs()
    base = dict(dtype=L.SAGA_BF16, B=1, Hq=12, Hk=1, Hv=2, D=128, L=1024, q=16, k=16, v=16, q_sb=12 * 128,
                q_sh=128, k_sb=1024 * 128, k_sh=1024 * 128, k_sl=128, v_sb=2 * 1024 * 128, v_sh=1024 * 128,
                v_sl=128, scaling=0.088, top_n=64, thr_in=16, out=16, o_sb=12 * 128, o_sh=128, append_pos=-1)
    base.update(kw)
    for k_, v_ in base.items():
        setattr(a, k_, v_)
    return a


@pytest.mark.parametrize("kw,code,needle", [
    (dict(Hk=5), L.SAGA_ERR_INVALID, "multiple of Hk"),
    (dict(Hv=5), L.SAGA_ERR_INVALID, "multiple of Hv"),
    (dict(D=96), L.SAGA_ERR_UNSUPPORTED, "head_dim"),
    (dict(dtype=7), L.SAGA_ERR_INVALID, "dtype"),
    (dict(k_sl=100), L.SAGA_ERR_INVALID, "16 bytes"),
    (dict(q=None), L.SAGA_ERR_INVALID, "non-NULL"),
    (dict(thr_in=None), L.SAGA_ERR_INVALID, "thr_in"),
    (dict(top_n=0), L.SAGA_ERR_INVALID, "top_n"),
    (dict(k=8), L.SAGA_ERR_INVALID, "aligned"),
    (dict(Hq=64, Hk=1, Hv=2, q_sb=64 * 128), L.SAGA_ERR_UNSUPPORTED, "32 query heads"),
    (dict(k_new=16, v_new=16, append_pos=1024), L.SAGA_ERR_INVALID, "append_pos"),
])
def test_invalid_requests_rejected_on_host(kw, code, needle):
    a = _args(**kw)
    rc = L.lib.saga_atopn_decode(ctypes.byref(a), None)
    assert rc == code
    assert needle in L.lib.saga_last_error().decode()


def test_unfused_entry_points_validate():
    rc = L.lib.saga_threshold_select(L.SAGA_BF16, 16, 100, 4, 100, 0, 16, 1, 16, 16, None, None)
    assert rc == L.SAGA_ERR_INVALID and "k" in L.lib.saga_last_error().decode()
    rc = L.lib.saga_kv_append(L.SAGA_BF16, 1, 1, 2, 128, 100, 100, 16, 0, 0, 128, 16, 0, 0, 128, 16, 0, 0, 16, 0,
                              0, None)
    assert rc == L.SAGA_ERR_INVALID and "pos" in L.lib.saga_last_error().decode()
    rc = L.lib.saga_transform_threshold(9, 16, 10, 1, 10, 16, 256, 16, None, None, None)
    assert rc == L.SAGA_ERR_INVALID


def test_workspace_query_rejects_bad_shapes():
    a = _args(Hk=5)
    assert L.lib.saga_workspace_bytes(ctypes.byref(a), L.SAGA_OP_ATOPN_DECODE) == 0
    assert "multiple" in L.lib.saga_last_error().decode()


def test_dropin_module_surface():
    """The names speedup.py:18-26 / 427-428 and lm_eval_saga.py:9-17 import."""
    import saga_b200.attention.attention as A
    import saga_b200.attention.triton_atopn as T
    for n in ["sdpa_attention_forward", "full_einsum_forward", "approx_top_n_attention_amortized_cal",
              "approx_top_n_attention_amortized", "init_amortized_threshold_tensor", "reset_amortized_state",
              "MAX_LAYERS", "AMORTIZED_THRESHOLD_TENSOR", "EXEMPT_LAYERS", "register_sdpa",
              "_compute_attn_weights", "_compute_attn_probs", "_transform_softmax_threshold",
              "_atopn_gather_and_output", "_threshold_topk_triton"]:
        assert hasattr(A, n), n
    assert A.MAX_LAYERS == 128
    assert isinstance(T._BUFFER_CACHE, dict) and callable(T.threshold_topk_fast)
    import inspect
    src = inspect.getsource(T)
    assert "import triton" not in src
