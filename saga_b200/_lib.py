"""ctypes binding of libsaga_b200.so (the C ABI declared in include/saga_b200.h).

The library must have been built (``python -m saga_b200.build``); importing
this module without it raises ImportError. The product has no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsaga_b200.so")

SAGA_BF16, SAGA_FP16, SAGA_FP32, SAGA_BOOL, SAGA_INT64 = 0, 1, 2, 3, 4
SAGA_OK, SAGA_ERR_INVALID, SAGA_ERR_UNSUPPORTED, SAGA_ERR_WORKSPACE, SAGA_ERR_CUDA = 0, -1, -2, -3, -4
SAGA_OP_ATOPN_DECODE, SAGA_OP_ATOPN_CALIBRATE, SAGA_OP_DENSE_DECODE, SAGA_OP_LOGITS = 0, 1, 2, 3

STATUS_WAIT_TIMEOUT = 0x1
STATUS_NONFINITE_THR = 0x2
STATUS_OVERFLOW = 0x4
STATUS_EMPTY_ROW = 0x8
STATUS_APPEND_RANGE = 0x10
STATUS_PAGE_RANGE = 0x20

_i32, _i64, _f32, _vp, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class SagaAttnArgs(ctypes.Structure):
    """Mirror of ``SagaAttnArgs`` in include/saga_b200.h (same field order)."""
    _fields_ = [
        ("dtype", _i32), ("B", _i32), ("Hq", _i32), ("Hk", _i32), ("Hv", _i32), ("D", _i32), ("L", _i32),
        ("q", _vp), ("q_sb", _i64), ("q_sh", _i64),
        ("k", _vp), ("k_sb", _i64), ("k_sh", _i64), ("k_sl", _i64),
        ("v", _vp), ("v_sb", _i64), ("v_sh", _i64), ("v_sl", _i64),
        ("mask", _vp), ("mask_dtype", _i32), ("m_sb", _i64), ("m_sh", _i64), ("m_sl", _i64),
        ("scaling", _f32), ("top_n", _i32), ("thr_in", _vp), ("thr_out", _vp),
        ("out", _vp), ("o_sb", _i64), ("o_sh", _i64),
        ("k_new", _vp), ("kn_sb", _i64), ("kn_sh", _i64),
        ("v_new", _vp), ("vn_sb", _i64), ("vn_sh", _i64),
        ("append_pos", _i32),
        ("logit_thr_out", _vp), ("count_out", _vp), ("sel_idx_out", _vp), ("sel_ld", _i32),
        ("logits_out", _vp), ("lo_ld", _i64),
        ("workspace", _vp), ("workspace_bytes", _sz),
        ("status", _vp),
        ("trace", _vp),
        ("nsel", _i32), ("pos_offset", _i32), ("shards", _i32), ("shard", _i32),
        ("shard_workspaces", _vp * 8),
        ("append_pos_dev", _vp),
        ("page_table", _vp), ("pt_sb", _i64), ("page_len", _i32), ("num_pages", _i32),
    ]


# (name, restype, argtypes) of every exported function
SIGNATURES = {
    "saga_workspace_bytes": (_sz, [ctypes.POINTER(SagaAttnArgs), _i32]),
    "saga_atopn_decode": (_i32, [ctypes.POINTER(SagaAttnArgs), _vp]),
    "saga_atopn_calibrate": (_i32, [ctypes.POINTER(SagaAttnArgs), _vp]),
    "saga_atopn_decode_noalloc": (_i32, [ctypes.POINTER(SagaAttnArgs), _vp]),
    "saga_noalloc_scratch_bytes": (_sz, []),
    "saga_dense_decode": (_i32, [ctypes.POINTER(SagaAttnArgs), _vp]),
    "saga_attn_logits": (_i32, [ctypes.POINTER(SagaAttnArgs), _vp]),
    "saga_transform_threshold": (_i32, [_i32, _vp, _i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp]),
    "saga_threshold_select": (_i32, [_i32, _vp, _i64, _i32, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp]),
    "saga_gather_output": (_i32, [_i32, _vp, _vp, _i32, _i32, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _i32,
                                  _i32, _vp, _i64, _i64, _vp]),
    "saga_kv_append": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _i64, _i64, _vp, _i64, _i64,
                              _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp]),
    "saga_ipc_handle": (_i32, [_vp, _vp, ctypes.POINTER(_sz)]),
    "saga_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "saga_ipc_close": (_i32, [_vp]),
    "saga_last_error": (ctypes.c_char_p, []),
    "saga_version": (ctypes.c_char_p, []),
    "saga_last_launches": (ctypes.c_char_p, []),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m saga_b200.build` "
            "(the CUDA library is required; there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class SagaError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, code: int, fn: str):
        msg = lib.saga_last_error().decode(errors="replace")
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


def check(code: int, fn: str) -> None:
    if code != SAGA_OK:
        raise SagaError(code, fn)


def last_launches() -> list:
    s = lib.saga_last_launches().decode()
    return [x for x in s.split(",") if x]


def version() -> str:
    return lib.saga_version().decode()
