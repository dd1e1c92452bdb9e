"""Host logic of the sequence-sharded decode on CPU (gloo, world size 2).

Checked here:
* the shard layout covers every global position exactly once;
* every shard keeps the 256-row tail replica;
* appended positions map to the right local rows.
* Exactness: with the exp-sums and counts of all shards combined, and the
  partial outputs merged by log-sum-exp, the sharded algorithm (numpy oracle
  per shard) gives the unsharded oracle's output. The partials cross ranks
  through gloo, as they cross devices through peer memory on the GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from saga_b200.seqpar import TAIL, shard_cache, shard_layout
from oracle import atopn_oracle as O


def test_layout_covers_every_position_once():
    L = 4096
    for P in (1, 2, 4, 8):
        seen = np.zeros(L, dtype=int)
        for r in range(P):
            lay = shard_layout(L, P, r)
            seen[lay.offset:lay.offset + lay.own] += 1
            if P > 1 and r < P - 1:
                assert lay.local_len == lay.own + TAIL
                assert lay.local_position(L - 1) == lay.local_len - 1  # appended token hits the replica
            else:
                assert lay.local_len == lay.own
        assert (seen == 1).all()


def test_shard_cache_rows():
    L, P = 2048, 4
    cache = torch.arange(L, dtype=torch.float32).view(1, 1, L, 1).expand(1, 2, L, 3).contiguous()
    for r in range(P):
        lay = shard_layout(L, P, r)
        loc = shard_cache(cache, lay)
        assert loc.shape[2] == lay.local_len
        assert torch.equal(loc[0, 0, :lay.own, 0], torch.arange(lay.offset, lay.offset + lay.own, dtype=torch.float32))
        if lay.replica:
            assert torch.equal(loc[0, 0, lay.own:, 0], torch.arange(L - TAIL, L, dtype=torch.float32))


def test_shard_cache_never_aliases_the_full_cache():
    # B = H = 1: the last shard's slice is already contiguous; an append into
    # the shard must still leave the full cache as it was
    L, P = 2048, 2
    cache = torch.arange(L, dtype=torch.float32).view(1, 1, L, 1).expand(1, 1, L, 4).contiguous()
    before = cache.clone()
    for r in range(P):
        loc = shard_cache(cache, shard_layout(L, P, r))
        assert loc.is_contiguous()
        loc.fill_(-1.0)
    assert torch.equal(cache, before)


def test_layout_rejects_uneven_or_tiny_shards():
    with pytest.raises(ValueError):
        shard_layout(1000, 3, 0)
    with pytest.raises(ValueError):
        shard_layout(256, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(5)
    B, L, Hq, Hk, Hv, D, N = 1, 2048, 4, 1, 2, 64, 64
    q = rng.standard_normal((B, Hq, 1, D)).astype(np.float32)
    k = rng.standard_normal((B, Hk, L, D)).astype(np.float32)
    v = rng.standard_normal((B, Hv, L, D)).astype(np.float32)
    k[0, 0, rng.choice(L, 16, replace=False)] += 4 * q[0, 0, 0] / np.linalg.norm(q[0, 0, 0])
    return q, k, v, N


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, N = _inputs()
        B, Hq, _, D = q.shape
        Lg = k.shape[2]
        thr = np.full((B * Hq,), 1e-3, dtype=np.float32)
        lay = shard_layout(Lg, world, rank)
        logits = O.attn_logits(q, k, "fp32").reshape(B * Hq, Lg)  # every shard can score the tail
        m = logits[:, Lg - TAIL:].max(axis=1)
        own = logits[:, lay.offset:lay.offset + lay.own]
        s_part = np.exp(own - m[:, None]).sum(axis=1).astype(np.float64)
        s_all = torch.tensor(s_part)
        dist.all_reduce(s_all)                                   # the exp-sum exchange
        t = m + np.log(np.maximum(thr, 1e-30) * s_all.numpy())
        passing = own > t[:, None]
        cnt = torch.tensor(passing.sum(axis=1))
        counts = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(counts, cnt)                             # the count exchange
        prefix = sum(c for c in counts[:rank]).numpy() if rank else np.zeros_like(cnt.numpy())
        K = min(2 * N, Lg)
        R = logits.shape[0]
        Gv = Hq // v.shape[1]
        mloc = np.full(R, -np.inf)
        lloc = np.zeros(R)
        oloc = np.zeros((R, D))
        for r_ in range(R):
            idx = np.nonzero(passing[r_])[0][:max(0, K - int(prefix[r_]))]   # the global K cap
            if len(idx):
                x = own[r_, idx]
                mloc[r_] = x.max()
                w = np.exp(x - mloc[r_])
                lloc[r_] = w.sum()
                oloc[r_] = w @ v[0, r_ // Gv, lay.offset + idx]
        parts = [None] * world
        dist.all_gather_object(parts, (mloc, lloc, oloc))        # the partial-output exchange
        M = np.max([p_[0] for p_ in parts], axis=0)
        num = sum(np.exp(p_[0] - M)[:, None] * p_[2] for p_ in parts)
        den = sum(np.exp(p_[0] - M) * p_[1] for p_ in parts)
        out[rank] = num / den[:, None]
    finally:
        dist.destroy_process_group()


def test_sharded_algorithm_matches_unsharded_oracle():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
        res = dict(out)
    q, k, v, N = _inputs()
    D = q.shape[-1]
    thr = np.full((q.shape[1],), 1e-3, dtype=np.float32)
    ref = O.atopn_amortized(q, k, v, thr, N, "fp32")["out"].reshape(-1, D)
    for rank in range(world):
        np.testing.assert_allclose(res[rank], ref, atol=1e-4, rtol=1e-4)
