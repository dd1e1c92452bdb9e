"""Sequence-sharded decode on 2 GPUs against the unsharded kernel.

One process per GPU (spawned here); gloo exchanges the workspaces' IPC
handles. Every rank builds the same seeded full caches, runs the unsharded
fused kernel on them as the reference, then the sharded step on its shard.
The sharded and unsharded outputs must agree, with the same tolerances as
the parity tests against the oracle, and the per-row counts must be equal.
Cases:
* the planted-key inputs, with the selected sets merged over the ranks;
* the sharded calibration step: thresholds, kept sets and outputs;
* a zero threshold, so that every position passes and the global K cap
  decides which shard keeps what;
* the fused append of a decode token at the last global position.
Skipped with fewer than 2 GPUs.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = (1, 8192, 12, 1, 2, 128, 256)  # B, L, Hq, Hk, Hv, D, N


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(dev):
    B, L, Hq, Hk, Hv, D, N = SHAPE
    g = torch.Generator(device=dev).manual_seed(11)
    q = (torch.randn((B, Hq, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hk, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    pos = torch.randperm(L, generator=g, device=dev)[:32]
    qd = q[0, 0, 0].float()
    k[0, 0, pos] += (4.0 * qd / qd.norm()).to(torch.bfloat16)
    kn = (torch.randn((B, Hk, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    vn = (torch.randn((B, Hv, 1, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q, k, v, kn, vn


def _close(a, b):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    rel = ((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt().clamp_min(1e-12)).item()
    return err <= 2e-2 and rel <= 1e-2, (err, rel)


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from saga_b200 import ops
        from saga_b200.seqpar import ShardedDecode, shard_cache
        B, L, Hq, Hk, Hv, D, N = SHAPE
        q, k, v, kn, vn = _inputs(dev)
        thr = torch.zeros(B * Hq, dtype=torch.float32, device=dev)
        ops.atopn_calibrate(q, k, v, None, thr, N)
        sd = ShardedDecode(dist.group.WORLD, dev, B, L, Hq, Hk, Hv, D)
        res = {}
        for name, t in (("planted", thr), ("zero_threshold", torch.zeros_like(thr))):
            dref, dsh = {}, {}
            ref = ops.atopn_decode(q, k, v, None, t, N, diag=dref)
            o = sd(q, shard_cache(k, sd.lay), shard_cache(v, sd.lay), t, N, diag=dsh)
            torch.cuda.synchronize()
            ok, stats = _close(o, ref)
            res[name] = (ok, stats, torch.equal(dsh["count"].cpu(), dref["count"].cpu()))
        # fused append of the decode token at the last global position
        k2, v2 = k.clone(), v.clone()
        ref = ops.atopn_decode(q, k2, v2, None, thr, N, k_new=kn, v_new=vn, append_pos=L - 1)
        kl, vl = shard_cache(k, sd.lay), shard_cache(v, sd.lay)
        o = sd(q, kl, vl, thr, N, k_new=kn, v_new=vn, append_pos=L - 1)
        torch.cuda.synchronize()
        ok, stats = _close(o, ref)
        res["append"] = (ok, stats, torch.equal(kl[:, :, -1], kn[:, :, 0]))
        # the selected sets: every rank writes its own chunks' positions at their
        # global ranks; merged over the ranks they must be the unsharded sets
        dref, dsh = {}, {}
        ops.atopn_decode(q, k, v, None, thr, N, diag=dref)
        sd(q, shard_cache(k, sd.lay), shard_cache(v, sd.lay), thr, N, diag=dsh)
        torch.cuda.synchronize()
        parts = [None] * world
        dist.all_gather_object(parts, dsh["sel_idx"].cpu())
        res["amortized_sets"] = (torch.stack(parts).amax(0), dref["sel_idx"].cpu(), dref["count"].cpu(),
                                 dref["logit_thr"].cpu(), dsh["count"].cpu(), dsh["logit_thr"].cpu(),
                                 [(p >= 0).sum(1).tolist() for p in parts])
        # sharded calibration against the unsharded one
        sdc = ShardedDecode(dist.group.WORLD, dev, B, L, Hq, Hk, Hv, D, op="calibrate")
        thr_u = torch.zeros(B * Hq, dtype=torch.float32, device=dev)
        thr_s = torch.zeros_like(thr_u)
        du, ds = {}, {}
        ref_c = ops.atopn_calibrate(q, k, v, None, thr_u, N, diag=du)
        out_c = sdc(q, shard_cache(k, sd.lay), shard_cache(v, sd.lay), thr_s, N, diag=ds)
        torch.cuda.synchronize()
        parts = [None] * world
        dist.all_gather_object(parts, ds["sel_idx"].cpu())
        ok, stats = _close(out_c, ref_c)
        res["calibrate"] = (ok, stats, thr_s.cpu(), thr_u.cpu(), torch.stack(parts).amax(0), du["sel_idx"].cpu(),
                            ops.attn_logits(q, k).float().cpu())
        res["status"] = ops.read_status(dev)
        dist.barrier()  # every rank is done with the peers' workspaces
        sd.close()
        sdc.close()
        dist.barrier()
        out[rank] = res
    finally:
        dist.destroy_process_group()


def test_sharded_decode_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
        res = dict(out)
    from saga_b200 import _lib as L
    for rank in range(world):
        r = res[rank]
        assert r["status"] & L.STATUS_WAIT_TIMEOUT == 0, r
        for name in ("planted", "zero_threshold"):
            ok, stats, counts_equal = r[name]
            assert ok, (rank, name, stats)
            assert counts_equal, (rank, name)
        ok, stats, appended = r["append"]
        assert ok and appended, (rank, stats)
        # amortized sets: equal, except positions whose logit lies within one
        # ulp of the threshold (the devices sum the exp-sums in another order)
        import numpy as np
        from _golden import near_threshold_ok, calib_row_ok
        from oracle import atopn_oracle as O
        sel_sh, sel_ref, cnt, t, cnt_sh, t_sh, written = r["amortized_sets"]
        B, Lk, Hq, Hk, Hv, D, N = SHAPE
        lg = r["calibrate"][6].numpy().reshape(B * Hq, Lk)
        for row in range(B * Hq):
            kept = min(int(cnt_sh[row]), 2 * N)
            a_, b_ = set(sel_sh[row, :kept].tolist()), set(sel_ref[row, :min(int(cnt[row]), 2 * N)].tolist())
            holes = (sel_sh[row, :kept] < 0).nonzero().flatten().tolist()
            assert not holes, (rank, row, int(cnt[row]), int(cnt_sh[row]), float(t[row]), float(t_sh[row]),
                               [w[row] for w in written], holes[:16])
            assert near_threshold_ok(lg[row], float(t[row]), a_ ^ b_, "bf16"), (rank, row, a_ ^ b_)
        # calibration: every row's threshold equal or one ulp apart, sets equal
        # except ties at the N-th probability, outputs within the parity bar
        ok, stats, thr_s, thr_u, csel_sh, csel_ref, _ = r["calibrate"]
        assert ok, (rank, "calibrate", stats)
        probs = O.softmax_dtype(lg, "bf16")
        for row in range(B * Hq):
            okr, why = calib_row_ok(probs[row], float(thr_u[row]), float(thr_s[row]), csel_sh[row, :N].numpy(),
                                    csel_ref[row, :N].numpy(), "bf16")
            assert okr, (rank, row, why)
