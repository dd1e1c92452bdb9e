"""Torch-facing host layer over the C ABI (libsaga_b200.so).

Each function takes torch CUDA tensors, fills a C descriptor with their
pointers and element strides, and enqueues the kernel on the current CUDA
stream. No host synchronisation happens, and after the first call for a
shape no memory is allocated except the outputs, so the calls can be captured
in CUDA graphs. The same functions are registered as torch custom ops
(``torch.ops.saga.*``) with fake implementations, so ``torch.compile``
traces through them.

Workspaces come from torch's caching allocator. They are zero-filled when
created, and each kernel leaves them zeroed. A workspace is cached per
(device, op, shapes), the way the reference caches its buffers per shape
(triton_atopn.py:56, 74-84): callers on one device must run on one stream at
a time.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib as L

_DT = {torch.bfloat16: L.SAGA_BF16, torch.float16: L.SAGA_FP16, torch.float32: L.SAGA_FP32}

_WORKSPACES: dict = {}
_STATUS: dict = {}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype} (bf16, fp16 or fp32)") from None


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("saga_b200 ops take CUDA tensors (there is no CPU path)")


def status_tensor(device) -> torch.Tensor:
    """The int32 device status word the kernels OR their SAGA_STATUS_* bits into."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def read_status(device="cuda", reset: bool = True) -> int:
    """Read (and by default clear) the status word. Synchronises the device."""
    t = status_tensor(device)
    v = int(t.item())
    if reset and v:
        t.zero_()
        if v & L.STATUS_WAIT_TIMEOUT:
            # a wait gave up: counters may be left non-zero, rebuild workspaces
            for k in [k for k in _WORKSPACES if k[0] == t.device.index]:
                _WORKSPACES[k][0].zero_()
    return v


def clear_workspaces():
    _WORKSPACES.clear()


def _workspace(args: L.SagaAttnArgs, op: int, device: torch.device) -> torch.Tensor:
    key = (device.index, op, args.dtype, args.B, args.Hq, args.Hk, args.Hv, args.D)
    ent = _WORKSPACES.get(key)
    if ent is not None and ent[1] == args.L:  # same shapes as the last call: nothing to size
        return ent[0]
    nbytes = L.lib.saga_workspace_bytes(ctypes.byref(args), op)
    if nbytes == 0:
        raise L.SagaError(L.SAGA_ERR_INVALID, "saga_workspace_bytes")
    # One workspace per (device, op, dtype, batch, heads, head_dim). Its layout
    # also depends on the context length, so a call with another length than
    # the previous one zero-fills it first (enqueued on the current stream):
    # a cache that grows by one position per step (transformers' DynamicCache)
    # reuses one buffer, as the reference's buffer cache does once L >= 2N
    # (triton_atopn.py:74-80), instead of keeping one per length.
    if ent is None or ent[0].numel() < nbytes:
        size = nbytes if ent is None else max(nbytes, ent[0].numel() * 5 // 4)
        ent = [torch.zeros(size, dtype=torch.uint8, device=device), args.L]
        _WORKSPACES[key] = ent
    elif ent[1] != args.L:
        ent[0].zero_()
        ent[1] = args.L
    return ent[0]


def _attn_args(q, k, v, attention_mask, scaling, page_table=None, context_len=None) -> L.SagaAttnArgs:
    """Kernel arguments. With ``page_table`` (int32 [B, max_pages] on the
    device), ``k`` and ``v`` are page pools [pages, H, page_len, D] and
    ``context_len`` is the logical length L of every sequence."""
    _require_cuda(q, k, v, attention_mask, page_table)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("query, key and value must be 4-D [B, H, L, D]")
    B, Hq, Lq, D = q.shape
    if Lq != 1:
        raise ValueError(f"decode kernels take one query position (got {Lq})")
    Hk, Hv = k.shape[1], v.shape[1]
    if page_table is None:
        Lk = k.shape[2]
        if k.shape[0] != B or v.shape[0] != B or k.shape[3] != D or v.shape[3] != D or v.shape[2] != Lk:
            raise ValueError("query/key/value shapes disagree")
    else:
        page_len = k.shape[2]
        if v.shape[2] != page_len or k.shape[3] != D or v.shape[3] != D:
            raise ValueError("key/value page pools disagree with the query")
        if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.stride(1) != 1:
            raise ValueError("page_table must be an int32 [B, max_pages] tensor with unit column stride")
        if page_table.shape[0] < B:
            raise ValueError("page_table has fewer rows than the batch")
        if context_len is None or not 1 <= int(context_len) <= page_table.shape[1] * page_len:
            raise ValueError("context_len in [1, max_pages * page_len] is required with a page table")
        Lk = int(context_len)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("query, key and value must share a dtype")
    for name, t in (("query", q), ("key", k), ("value", v)):
        if t.stride(3) != 1:
            raise ValueError(f"{name} needs a unit stride along head_dim")
    a = L.SagaAttnArgs()
    a.dtype = _dt(q)
    a.B, a.Hq, a.Hk, a.Hv, a.D, a.L = B, Hq, Hk, Hv, D, Lk
    a.q, a.q_sb, a.q_sh = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_sb, a.k_sh, a.k_sl = k.data_ptr(), k.stride(0), k.stride(1), k.stride(2)
    a.v, a.v_sb, a.v_sh, a.v_sl = v.data_ptr(), v.stride(0), v.stride(1), v.stride(2)
    if attention_mask is not None:
        m = attention_mask[..., :Lk]
        if m.dim() != 4 or m.shape[-1] != Lk:
            raise ValueError("mask must be [B|1, 1|Hq, 1, >=L]")
        m = m.expand(B, Hq, 1, Lk)
        if m.dtype == torch.bool:
            a.mask_dtype = L.SAGA_BOOL
        elif m.dtype == q.dtype:
            a.mask_dtype = _dt(q)
        else:
            raise TypeError("mask must be bool or the logits dtype")
        a.mask, a.m_sb, a.m_sh, a.m_sl = m.data_ptr(), m.stride(0), m.stride(1), m.stride(3)
    a.scaling = float(1.0 / math.sqrt(D) if scaling is None else scaling)
    a.append_pos = -1
    if page_table is not None:
        a.page_table, a.pt_sb = page_table.data_ptr(), page_table.stride(0)
        a.page_len, a.num_pages = k.shape[2], min(k.shape[0], v.shape[0])
    return a


def _set_append(a, k_new, v_new, append_pos):
    if k_new is None and v_new is None:
        return
    if k_new is None or v_new is None:
        raise ValueError("k_new and v_new go together")
    _require_cuda(k_new, v_new)
    if k_new.stride(-1) != 1 or v_new.stride(-1) != 1:
        raise ValueError("k_new / v_new need a unit stride along head_dim")
    a.k_new, a.kn_sb, a.kn_sh = k_new.data_ptr(), k_new.stride(0), k_new.stride(1)
    a.v_new, a.vn_sb, a.vn_sh = v_new.data_ptr(), v_new.stride(0), v_new.stride(1)
    if isinstance(append_pos, torch.Tensor):
        # read on the device by the kernel (a CUDA graph can replay an advancing position)
        if not append_pos.is_cuda or append_pos.dtype != torch.int64 or append_pos.numel() < 1:
            raise ValueError("a tensor append position must be a CUDA int64 tensor")
        a.append_pos = 0
        a.append_pos_dev = append_pos.data_ptr()
    else:
        a.append_pos = int(append_pos)


def _out_like(q):
    B, Hq, _, D = q.shape
    return torch.empty((B, Hq, 1, D), dtype=q.dtype, device=q.device)


def _diag_buffers(a, q, K, diag):
    if diag is None:
        return
    R = a.B * a.Hq
    diag["logit_thr"] = torch.full((R,), float("nan"), dtype=torch.float32, device=q.device)
    diag["count"] = torch.full((R,), -1, dtype=torch.int32, device=q.device)
    diag["sel_idx"] = torch.full((R, max(K, 1)), -1, dtype=torch.int32, device=q.device)
    a.logit_thr_out = diag["logit_thr"].data_ptr()
    a.count_out = diag["count"].data_ptr()
    a.sel_idx_out = diag["sel_idx"].data_ptr()
    a.sel_ld = max(K, 1)


def _run(fn_name, a, op, device, diag=None):
    ws = _workspace(a, op, device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.status = status_tensor(device).data_ptr()
    if diag is not None and diag.get("trace"):
        diag["trace"] = torch.zeros((1024, 128), dtype=torch.int64, device=device)
        a.trace = diag["trace"].data_ptr()
    rc = getattr(L.lib, fn_name)(ctypes.byref(a), _stream(device))
    L.check(rc, fn_name)
    if diag is not None:
        diag["launches"] = L.last_launches()


# ---------------------------------------------------------------------------
# public host functions
# ---------------------------------------------------------------------------

def atopn_decode(query, key, value, attention_mask=None, threshold=None, top_n: int = 256,
                 scaling=None, k_new=None, v_new=None, append_pos: int = -1, diag: Optional[dict] = None,
                 page_table=None, context_len=None):
    """Steady-state Atop-N step (attention.py:192-209) in one fused kernel.

    ``threshold`` holds the softmax-space threshold of each (batch, query head)
    row, e.g. ``AMORTIZED_THRESHOLD_TENSOR[layer, :B*Hq]``. With
    ``k_new``/``v_new`` the token is first written at ``append_pos`` of the
    caches. ``diag``, if a dict, receives per-row logit thresholds, passing
    counts and the kept positions. With ``page_table``, key and value are
    page pools (see ``_attn_args``).
    """
    a = _attn_args(query, key, value, attention_mask, scaling, page_table, context_len)
    if threshold is None or threshold.dtype != torch.float32 or not threshold.is_contiguous():
        raise ValueError("threshold must be a contiguous float32 tensor with B*Hq entries")
    if threshold.numel() < a.B * a.Hq:
        raise ValueError("threshold has fewer than B*Hq entries")
    a.top_n = int(top_n)
    a.thr_in = threshold.data_ptr()
    _set_append(a, k_new, v_new, append_pos)
    out = _out_like(query)
    a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
    _diag_buffers(a, query, min(2 * int(top_n), a.L), diag)
    _run("saga_atopn_decode", a, L.SAGA_OP_ATOPN_DECODE, query.device, diag)
    return out


def atopn_calibrate(query, key, value, attention_mask=None, threshold_out=None, top_n: int = 256,
                    scaling=None, k_new=None, v_new=None, append_pos: int = -1, diag: Optional[dict] = None,
                    page_table=None, context_len=None):
    """Calibration step (attention.py:173-189): writes the N-th largest
    probability of each row into ``threshold_out`` and returns the output of
    the renormalised top-N probabilities."""
    a = _attn_args(query, key, value, attention_mask, scaling, page_table, context_len)
    if threshold_out is None or threshold_out.dtype != torch.float32 or not threshold_out.is_contiguous():
        raise ValueError("threshold_out must be a contiguous float32 tensor with B*Hq entries")
    if threshold_out.numel() < a.B * a.Hq:
        raise ValueError("threshold_out has fewer than B*Hq entries")
    a.top_n = int(top_n)
    a.thr_out = threshold_out.data_ptr()
    _set_append(a, k_new, v_new, append_pos)
    out = _out_like(query)
    a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
    _diag_buffers(a, query, min(int(top_n), a.L), diag)
    _run("saga_atopn_calibrate", a, L.SAGA_OP_ATOPN_CALIBRATE, query.device, diag)
    return out


def dense_decode(query, key, value, attention_mask=None, scaling=None, k_new=None, v_new=None,
                 append_pos: int = -1, diag: Optional[dict] = None, page_table=None, context_len=None):
    """Dense GQA decode (attention.py:64-85) for one query position."""
    a = _attn_args(query, key, value, attention_mask, scaling, page_table, context_len)
    _set_append(a, k_new, v_new, append_pos)
    out = _out_like(query)
    a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
    _run("saga_dense_decode", a, L.SAGA_OP_DENSE_DECODE, query.device, diag)
    return out


class DecodeStep:
    """One decode op bound to fixed tensors, for serving loops.

    The descriptor is built and validated once, here; every call is then a
    single C-ABI call that reads the tensors' current contents (refill the
    query and decode-token buffers in place, e.g. by a copy from pinned host
    memory) and writes ``self.out``. The same kernels and arguments as
    ``atopn_decode`` / ``atopn_calibrate`` / ``dense_decode`` with these
    tensors. The step owns its workspace, so it never shares exchange state
    with the per-call functions; steps must not overlap in time with each
    other on one workspace (one stream at a time). ``op`` is "atopn",
    "calibrate" or "dense"; ``threshold`` is read (atopn) or written
    (calibrate).
    """

    _FN = {"atopn": ("saga_atopn_decode", L.SAGA_OP_ATOPN_DECODE),
           "calibrate": ("saga_atopn_calibrate", L.SAGA_OP_ATOPN_CALIBRATE),
           "dense": ("saga_dense_decode", L.SAGA_OP_DENSE_DECODE)}

    def __init__(self, op: str, query, key, value, attention_mask=None, threshold=None, top_n: int = 256,
                 scaling=None, k_new=None, v_new=None, append_pos=-1, out=None, page_table=None,
                 context_len=None):
        if op not in self._FN:
            raise ValueError(f"op must be one of {sorted(self._FN)}")
        fn_name, code = self._FN[op]
        a = _attn_args(query, key, value, attention_mask, scaling, page_table, context_len)
        if op != "dense":
            if threshold is None or threshold.dtype != torch.float32 or not threshold.is_contiguous():
                raise ValueError("threshold must be a contiguous float32 tensor with B*Hq entries")
            if threshold.numel() < a.B * a.Hq:
                raise ValueError("threshold has fewer than B*Hq entries")
            a.top_n = int(top_n)
            if op == "atopn":
                a.thr_in = threshold.data_ptr()
            else:
                a.thr_out = threshold.data_ptr()
        _set_append(a, k_new, v_new, append_pos)
        if out is None:
            out = _out_like(query)
        elif out.shape != (a.B, a.Hq, 1, a.D) or out.dtype != query.dtype or out.stride(3) != 1 or not out.is_cuda:
            raise ValueError("out must be a CUDA [B, Hq, 1, D] tensor of the query dtype, unit stride along D")
        a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
        nbytes = L.lib.saga_workspace_bytes(ctypes.byref(a), code)
        if nbytes == 0:
            raise L.SagaError(L.SAGA_ERR_INVALID, "saga_workspace_bytes")
        self.device = query.device
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
        a.status = status_tensor(self.device).data_ptr()
        self.out = out
        self._args = a
        self._ref = ctypes.byref(a)
        self._fn = getattr(L.lib, fn_name)
        self._name = fn_name
        # the bound tensors stay alive as long as the step
        self._tensors = (query, key, value, attention_mask, threshold, k_new, v_new, append_pos, page_table)

    def __call__(self, stream: Optional[int] = None) -> torch.Tensor:
        """Enqueue the step on ``stream`` (a cudaStream_t as int; default:
        the device's current torch stream) and return ``self.out``."""
        rc = self._fn(self._ref, _stream(self.device) if stream is None else stream)
        if rc:
            L.check(rc, self._name)
        return self.out


def attn_logits(query, key, attention_mask=None, scaling=None):
    """Logits [B, Hq, 1, L] (attention.py:113-128)."""
    a = _attn_args(query, key, key[:, :1].expand(key.shape[0], 1, key.shape[2], key.shape[3]),
                   attention_mask, scaling)
    a.Hv = a.Hq  # the value cache is not read; any divisor of Hq passes validation
    a.v, a.v_sb, a.v_sh, a.v_sl = key.data_ptr(), key.stride(0), 0, key.stride(2)
    B, Hq, _, _ = query.shape
    out = torch.empty((B, Hq, 1, a.L), dtype=query.dtype, device=query.device)
    a.logits_out, a.lo_ld = out.data_ptr(), a.L
    a.status = status_tensor(query.device).data_ptr()
    L.check(L.lib.saga_attn_logits(ctypes.byref(a), _stream(query.device)), "saga_attn_logits")
    return out


def transform_threshold(attn_logits: torch.Tensor, softmax_threshold: torch.Tensor, tail_size: int = 256,
                        return_stats: bool = False):
    """Logit-space threshold per row (attention.py:136-149)."""
    _require_cuda(attn_logits, softmax_threshold)
    Lk = attn_logits.shape[-1]
    x = attn_logits.reshape(-1, Lk)
    if x.stride(-1) != 1:
        x = x.contiguous()
    R = x.shape[0]
    thr = softmax_threshold.reshape(-1).to(torch.float32).contiguous()
    if thr.numel() < R:
        raise ValueError("softmax_threshold has fewer entries than rows")
    t = torch.empty(R, dtype=torch.float32, device=x.device)
    m = torch.empty(R, dtype=torch.float32, device=x.device) if return_stats else None
    s = torch.empty(R, dtype=torch.float32, device=x.device) if return_stats else None
    L.check(L.lib.saga_transform_threshold(_dt(x), x.data_ptr(), x.stride(0), R, Lk, thr.data_ptr(),
                                           int(tail_size), t.data_ptr(), m.data_ptr() if m is not None else None,
                                           s.data_ptr() if s is not None else None, _stream(x.device)),
            "saga_transform_threshold")
    return (t, m, s) if return_stats else t


def threshold_select(x: torch.Tensor, k: int, threshold: torch.Tensor, vals=None, idx=None, counts=None):
    """Every x[r, i] > threshold[r] in ascending i, at most k per row
    (triton_atopn.py:6-53, 59-113). Returns (vals, idx, counts)."""
    _require_cuda(x, threshold)
    Lk = x.shape[-1]
    xf = x.reshape(-1, Lk)
    if xf.stride(-1) != 1:
        xf = xf.contiguous()
    R = xf.shape[0]
    thr = threshold.reshape(-1)
    if thr.dtype != torch.float32 or not thr.is_contiguous():
        thr = thr.to(torch.float32).contiguous()
    if vals is None:
        vals = torch.empty((R, k), dtype=x.dtype, device=x.device)
    if idx is None:
        idx = torch.empty((R, k), dtype=torch.int64, device=x.device)
    if counts is None:
        counts = torch.empty(R, dtype=torch.int32, device=x.device)
    L.check(L.lib.saga_threshold_select(_dt(xf), xf.data_ptr(), xf.stride(0), R, Lk, int(k), thr.data_ptr(),
                                        thr.numel(), vals.data_ptr(), idx.data_ptr(), counts.data_ptr(),
                                        _stream(x.device)), "saga_threshold_select")
    return vals, idx, counts


def gather_output(weights: torch.Tensor, indices: torch.Tensor, value: torch.Tensor, num_q_heads: int,
                  input_is_logits: bool) -> torch.Tensor:
    """Output [B, Hq, 1, D] from a [B, Hq, 1, K] buffer of weights and
    positions (attention.py:152-170)."""
    _require_cuda(weights, indices, value)
    B, Hv, Lk, D = value.shape
    K = weights.shape[-1]
    w = weights.reshape(-1, K).contiguous()
    ix = indices.reshape(-1, K).to(torch.int64).contiguous()
    out = torch.empty((B, num_q_heads, 1, D), dtype=value.dtype, device=value.device)
    L.check(L.lib.saga_gather_output(_dt(value), w.data_ptr(), ix.data_ptr(), K, int(bool(input_is_logits)),
                                     value.data_ptr(), value.stride(0), value.stride(1), value.stride(2), B,
                                     num_q_heads, Hv, D, Lk, out.data_ptr(), out.stride(0), out.stride(1),
                                     _stream(value.device)), "saga_gather_output")
    return out


def kv_append(k_cache, v_cache, k_new, v_new, pos: int) -> None:
    """Write one decode token into the asymmetric static cache at ``pos``."""
    _require_cuda(k_cache, v_cache, k_new, v_new)
    B, Hk, Lk, D = k_cache.shape
    Hv = v_cache.shape[1]
    if k_new.shape != (B, Hk, 1, D) or v_new.shape != (B, Hv, 1, D):
        raise ValueError("k_new [B, Hk, 1, D] and v_new [B, Hv, 1, D] expected")
    L.check(L.lib.saga_kv_append(_dt(k_cache), B, Hk, Hv, D, Lk, int(pos), k_cache.data_ptr(),
                                 k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), v_cache.data_ptr(),
                                 v_cache.stride(0), v_cache.stride(1), v_cache.stride(2), k_new.data_ptr(),
                                 k_new.stride(0), k_new.stride(1), v_new.data_ptr(), v_new.stride(0),
                                 v_new.stride(1), _stream(k_cache.device)), "saga_kv_append")


# ---------------------------------------------------------------------------
# torch custom ops (opaque to torch.compile, capturable in CUDA graphs)
# ---------------------------------------------------------------------------

@torch.library.custom_op("saga::atopn_decode", mutates_args=())
def _op_atopn_decode(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     attention_mask: Optional[torch.Tensor], threshold: torch.Tensor, top_n: int,
                     scaling: float) -> torch.Tensor:
    return atopn_decode(query, key, value, attention_mask, threshold, top_n, scaling)


@_op_atopn_decode.register_fake
def _(query, key, value, attention_mask, threshold, top_n, scaling):
    return query.new_empty((query.shape[0], query.shape[1], 1, query.shape[3]))


@torch.library.custom_op("saga::atopn_calibrate", mutates_args=("threshold_out",))
def _op_atopn_calibrate(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                        attention_mask: Optional[torch.Tensor], threshold_out: torch.Tensor, top_n: int,
                        scaling: float) -> torch.Tensor:
    return atopn_calibrate(query, key, value, attention_mask, threshold_out, top_n, scaling)


@_op_atopn_calibrate.register_fake
def _(query, key, value, attention_mask, threshold_out, top_n, scaling):
    return query.new_empty((query.shape[0], query.shape[1], 1, query.shape[3]))


@torch.library.custom_op("saga::dense_decode", mutates_args=())
def _op_dense_decode(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     attention_mask: Optional[torch.Tensor], scaling: float) -> torch.Tensor:
    return dense_decode(query, key, value, attention_mask, scaling)


@_op_dense_decode.register_fake
def _(query, key, value, attention_mask, scaling):
    return query.new_empty((query.shape[0], query.shape[1], 1, query.shape[3]))


@torch.library.custom_op("saga::attn_logits", mutates_args=())
def _op_attn_logits(query: torch.Tensor, key: torch.Tensor, attention_mask: Optional[torch.Tensor],
                    scaling: float) -> torch.Tensor:
    return attn_logits(query, key, attention_mask, scaling)


@_op_attn_logits.register_fake
def _(query, key, attention_mask, scaling):
    return query.new_empty((query.shape[0], query.shape[1], 1, key.shape[2]))


@torch.library.custom_op("saga::transform_threshold", mutates_args=())
def _op_transform_threshold(attn_logits: torch.Tensor, softmax_threshold: torch.Tensor,
                            tail_size: int) -> torch.Tensor:
    return transform_threshold(attn_logits, softmax_threshold, tail_size)


@_op_transform_threshold.register_fake
def _(attn_logits, softmax_threshold, tail_size):
    return attn_logits.new_empty((attn_logits.numel() // attn_logits.shape[-1],), dtype=torch.float32)


@torch.library.custom_op("saga::kv_append", mutates_args=("k_cache", "v_cache"))
def _op_kv_append(k_cache: torch.Tensor, v_cache: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                  pos: int) -> None:
    kv_append(k_cache, v_cache, k_new, v_new, pos)


@_op_kv_append.register_fake
def _(k_cache, v_cache, k_new, v_new, pos):
    return None


# The same steps with the decode token's key/value rows appended in the fused
# kernel (the caches are written in place at the device-side position `pos`).
@torch.library.custom_op("saga::atopn_decode_append", mutates_args=("key", "value"))
def _op_atopn_decode_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                            attention_mask: Optional[torch.Tensor], threshold: torch.Tensor, top_n: int,
                            scaling: float, k_new: torch.Tensor, v_new: torch.Tensor,
                            pos: torch.Tensor) -> torch.Tensor:
    return atopn_decode(query, key, value, attention_mask, threshold, top_n, scaling, k_new=k_new, v_new=v_new,
                        append_pos=pos)


@_op_atopn_decode_append.register_fake
def _(query, key, value, attention_mask, threshold, top_n, scaling, k_new, v_new, pos):
    return query.new_empty((query.shape[0], query.shape[1], 1, query.shape[3]))


@torch.library.custom_op("saga::atopn_calibrate_append", mutates_args=("key", "value", "threshold_out"))
def _op_atopn_calibrate_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                               attention_mask: Optional[torch.Tensor], threshold_out: torch.Tensor, top_n: int,
                               scaling: float, k_new: torch.Tensor, v_new: torch.Tensor,
                               pos: torch.Tensor) -> torch.Tensor:
    return atopn_calibrate(query, key, value, attention_mask, threshold_out, top_n, scaling, k_new=k_new,
                           v_new=v_new, append_pos=pos)


@_op_atopn_calibrate_append.register_fake
def _(query, key, value, attention_mask, threshold_out, top_n, scaling, k_new, v_new, pos):
    return query.new_empty((query.shape[0], query.shape[1], 1, query.shape[3]))


@torch.library.custom_op("saga::dense_decode_append", mutates_args=("key", "value"))
def _op_dense_decode_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                            attention_mask: Optional[torch.Tensor], scaling: float, k_new: torch.Tensor,
                            v_new: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    return dense_decode(query, key, value, attention_mask, scaling, k_new=k_new, v_new=v_new, append_pos=pos)


@_op_dense_decode_append.register_fake
def _(query, key, value, attention_mask, scaling, k_new, v_new, pos):
    return query.new_empty((query.shape[0], query.shape[1], 1, query.shape[3]))


def scaling_or_default(query: torch.Tensor, scaling) -> float:
    return float(1.0 / math.sqrt(query.size(-1)) if scaling is None else scaling)
