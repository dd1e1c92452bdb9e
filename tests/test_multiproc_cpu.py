"""Multi-process host logic of the replica bench on CPU (gloo, world size 2).

On a GPU box, `bench.py --gpus N` runs one replica per rank, each decoding its
own batch, with no collective on the data path. Here two gloo ranks check the
parts that do not need a GPU:
  * the per-rank input seeds differ;
  * the reported step time is the slowest rank's;
  * the whole-job throughput counts every rank's sequences.
"""
import importlib.util
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(HERE, "..", "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b = _bench()
        local_ms = 0.05 + 0.01 * rank  # rank 1 is the slower one
        ms = b.max_over_ranks(torch, dist, local_ms, torch.device("cpu"), world)
        seeds = [b.replica_seed(rank, c) for c in range(4)]
        gathered = [None] * world
        dist.all_gather_object(gathered, seeds)
        out[rank] = (ms, gathered)
    finally:
        dist.destroy_process_group()


def test_replica_host_logic_two_ranks():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
        res = dict(out)
    for rank in range(world):
        ms, seeds = res[rank]
        assert ms == pytest.approx(0.06)  # every rank reports the slowest rank's time
        assert set(seeds[0]).isdisjoint(seeds[1])  # each rank decodes its own inputs
    b = _bench()
    assert b.job_throughput(8, 2, 0.06) == pytest.approx(16 / 0.06e-3)


def test_reference_arm_compaction_matches_the_oracle_selection():
    """bench.torch_threshold_topk, the torch stand-in for the reference's
    Triton selection in the CPU reference arm, keeps x > t in ascending
    position order with -inf / 0 padding, exactly as the oracle's restatement
    of triton_atopn.py does (the K lowest positions on overflow)."""
    import numpy as np
    from oracle import atopn_oracle as O
    b = _bench()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(7, 3000, generator=g).to(torch.bfloat16)
    t = torch.randn(7, generator=g) * 0.4 + 1.2
    t[3] = -10.0  # every position passes: overflow, the 64 lowest kept
    vals, idx = b.torch_threshold_topk(x, 64, t)
    ov, oi, _, _ = O.threshold_select(x.float().numpy(), t.numpy(), 64)
    np.testing.assert_array_equal(idx.numpy(), oi)
    np.testing.assert_array_equal(vals.float().numpy(), ov)
