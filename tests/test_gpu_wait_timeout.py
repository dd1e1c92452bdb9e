"""The bounded waits of the fused kernel end, with a status, when a partner
never arrives; the device stays usable.

One launch of a sequence-sharded call (shards = 2) on a single GPU, whose
partner shard is never launched: its exchange slots and completion ticket are
a zero-filled buffer that nothing writes. Every wait of the call on the
partner gives up after its limit (0.5 s each), sets SAGA_STATUS_WAIT_TIMEOUT
and returns; no thread hangs and no memory outside the two buffers is
touched. The next ordinary call on the same device must give the same output
as before. No fault is involved: the failure is a flag that nothing sets.
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

B, L, HQ, HK, HV, D, N = 1, 4096, 12, 1, 2, 128, 128


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(5)
    q = (torch.randn((B, HQ, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, HK, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, HV, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q, k, v


def test_partner_never_launched_times_out_and_device_recovers():
    from saga_b200 import _lib as Lib
    from saga_b200 import ops
    from saga_b200.seqpar import shard_layout, shard_cache
    dev = torch.device("cuda", 0)
    q, k, v = _inputs(dev)
    thr = torch.zeros(B * HQ, dtype=torch.float32, device=dev)
    ops.atopn_calibrate(q, k, v, None, thr, N)
    before = ops.atopn_decode(q, k, v, None, thr, N)
    torch.cuda.synchronize()
    assert not ops.read_status(dev) & Lib.STATUS_WAIT_TIMEOUT

    lay = shard_layout(L, 2, 0)  # shard 0 of 2: own half plus the tail replica
    kl, vl = shard_cache(k, lay), shard_cache(v, lay)
    a = ops._attn_args(q, kl, vl, None, None)
    a.nsel, a.pos_offset, a.shards, a.shard = lay.own, lay.offset, 2, 0
    a.top_n, a.thr_in = N, thr.data_ptr()
    nbytes = Lib.lib.saga_workspace_bytes(ctypes.byref(a), Lib.SAGA_OP_ATOPN_DECODE)
    assert nbytes > 0
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    absent = torch.zeros(nbytes, dtype=torch.uint8, device=dev)  # the partner that never comes
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    a.shard_workspaces[0], a.shard_workspaces[1] = ws.data_ptr(), absent.data_ptr()
    out = torch.empty_like(q)
    a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    a.status = status.data_ptr()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    Lib.check(Lib.lib.saga_atopn_decode(ctypes.byref(a), ctypes.c_void_p(ops._stream(dev))), "saga_atopn_decode")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) & Lib.STATUS_WAIT_TIMEOUT
    # a handful of sequential waits on the partner, 0.5 s each at most
    assert elapsed < 10.0, elapsed
    assert torch.count_nonzero(absent).item() == 0  # nothing wrote into the absent partner

    after = ops.atopn_decode(q, k, v, None, thr, N)
    torch.cuda.synchronize()
    assert not ops.read_status(dev) & Lib.STATUS_WAIT_TIMEOUT
    assert torch.equal(after, before)
