#!/usr/bin/env python
"""SAGA Atop-N decode-attention benchmark (one process per GPU).

Default workload (config 2): one attention layer of a SAGA model, batch 8,
context 32768, 12 query heads, 1 key head, 2 value heads, head_dim 128,
N = 512, bf16 KV cache. One step = one amortized Atop-N decode step:
append of the new token, logits over the reduced key head, threshold
transform, selection and the sparse V gather, as a single fused kernel.

  value      decode tokens/s of the layer, whole job (sum over ranks): B * N_gpus / step time
  e2e        the same through the serving API (saga_b200.ops.DecodeStep: the
             step's arguments bound once, one C-ABI call per step), with the
             step's inputs copied from pinned host memory and its output
             copied back, inside the timed region, the copies on two side
             streams under the neighbouring steps' kernels; "e2e_serial" the
             same with every copy and step in order on one stream, and
             "e2e_per_call" that through the per-call functions
             (saga_b200.ops.atopn_decode)
  roofline   algorithmic HBM bytes of one step / step time, against the
             measured copy bandwidth (MEASURED_PEAKS.json)

Inputs are synthetic (seeded, on the device); 4 rotating KV-cache copies
(4 x 192 MiB > L2) so that no step reads a cache that is still in L2.

--impl reference times the reference's own implementation of the step on the
host cores (its attention.py, installed unmodified into baseline/_ref by
baseline/install_reference.sh, with its Triton selection replaced by a torch
compaction), the whole batch per step, with all torch threads; it falls back to
the numpy port of its algorithm (oracle/) when the reference is not installed.
The default line also reports, on the GPU, the reference's own torch + Triton
step and calibration, this library's calibration step with its roofline, and
dense GQA decode (this library's kernel and the reference's torch bmm) under
"gpu_baselines".
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

WORKLOADS = {
    # name: (B, L, Hq, Hk, Hv, D, N, plant)
    "config1": (1, 4096, 15, 1, 5, 64, 128, 16),  # fp32, the reference's CPU-runnable case
    "config2": (8, 32768, 12, 1, 2, 128, 512, 64),
    "config4": (1, 131072, 12, 1, 2, 128, 1024, 256),
    # the same model with its unmerged key heads, for the dense-GQA baseline (--mode dense)
    "config2_gqa": (8, 32768, 12, 2, 2, 128, 512, 64),
    "config3_layer": (16, 16384 + 128, 15, 1, 5, 64, 256, 64),
    "config5_layer": (64, 65536 + 64, 12, 1, 4, 128, 512, 128),
}
L2_BYTES = 126 * 1024 * 1024

# Model-level workloads, decoded through the reference's own harness
# (speedup.measure_decode_latency) with this package as its attention module:
# name: (family, layers, hidden, q heads, value heads, head_dim, mlp, vocab,
#        batch, prefilled context, new tokens, N, key heads of the dense model)
MODELS = {
    "config3": ("llama", 32, 960, 15, 5, 64, 2560, 49152, 16, 16384, 128, 256, 5),
    "config5": ("qwen2", 28, 1536, 12, 4, 128, 8960, 151936, 64, 65536, 64, 512, 2),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="saga_b200", choices=["saga_b200", "reference"])
    ap.add_argument("--workload", default="config2", choices=sorted(WORKLOADS) + sorted(MODELS))
    ap.add_argument("--iterations", type=int, default=3, help="model workloads: measured generations")
    ap.add_argument("--compile", action="store_true", help="model workloads: torch.compile(model.forward)")
    ap.add_argument("--mode", default="atopn", choices=["atopn", "dense", "calibrate"])
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-config4", action="store_true", help="skip the sequence-sharded config-4 leg (N > 1)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

# ---------------------------------------------------------------------------
# multi-GPU host logic: replicas, one per rank, each on its own batch
# ---------------------------------------------------------------------------

def replica_seed(rank: int, copy: int) -> int:
    """Seed of a rank's input copy: every rank decodes its own batch."""
    return 1000 * rank + copy


def max_over_ranks(torch, dist, value: float, device, world: int) -> float:
    """The slowest rank's time: every rank takes part, in the same order."""
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(batch_per_rank: int, world: int, ms_per_step: float) -> float:
    """Whole-job tokens/s: all ranks' sequences per step over the slowest rank's step time."""
    return batch_per_rank * world / (ms_per_step * 1e-3)


def ncu_traffic(workload: str, mode: str):
    """DRAM bytes (read + write) of one launch of the timed kernel, from the
    committed ncu summary of this workload (profiles/), or None."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                        f"saga_decode_kernel_{'amortized' if mode == 'atopn' else mode}_{workload}.md")
    try:
        for line in open(path):
            if line.startswith("| traffic (read + write) per launch |"):
                return int(float(line.split("|")[2].split()[0]) * 1e6)
    except (OSError, ValueError, IndexError):
        pass
    return None


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons (read-only)."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str, enabled=True):
        self.gpu_id, self.enabled, self.proc, self.path = gpu_id, enabled, None, None

    def start(self):
        if not self.enabled:
            return
        import tempfile
        self.path = tempfile.mktemp(suffix=".csv")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for ln in f:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) == 7:
                    try:
                        rows.append((float(parts[0]), float(parts[1]), parts[3:]))
                    except ValueError:
                        pass
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, x in enumerate(r) if x.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def make_device_inputs(torch, shape, device, seed):
    """Seeded synthetic tensors on the device: q0, q1, K, V, k_new, v_new."""
    B, L, Hq, Hk, Hv, D, N, plant = shape
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    bf = torch.bfloat16
    s = 0.5
    q0 = torch.randn(B, Hq, 1, D, generator=g, device=device) * s
    q1 = 0.9 * q0 + math.sqrt(1 - 0.81) * torch.randn(B, Hq, 1, D, generator=g, device=device) * s
    k = (torch.randn(B, Hk, L, D, generator=g, device=device) * s)
    G = Hq // Hk
    for kk in range(Hk):
        qh = q0[:, kk * G, 0]
        qhat = qh / qh.norm(dim=-1, keepdim=True)
        pos = torch.randint(0, L, (B, plant), generator=g, device=device)
        k[torch.arange(B, device=device)[:, None], kk, pos] += 4.0 * qhat[:, None, :]
    k = k.to(bf)
    v = torch.empty(B, Hv, L, D, device=device, dtype=bf)
    for h in range(Hv):  # chunked to keep the fp32 temporary small
        v[:, h] = (torch.randn(B, L, D, generator=g, device=device) * s).to(bf)
    kn = (torch.randn(B, Hk, 1, D, generator=g, device=device) * s).to(bf)
    vn = (torch.randn(B, Hv, 1, D, generator=g, device=device) * s).to(bf)
    return q0.to(bf), q1.to(bf), k, v, kn, vn


def algorithmic_bytes(shape, union_rows: int, mode: str) -> int:
    """HBM bytes one step must move (bf16): the key cache, the value rows the
    step needs, q, out, the appended token and the per-row thresholds."""
    B, L, Hq, Hk, Hv, D, N, _ = shape
    e = 2
    kv = B * Hk * L * D * e
    if mode == "dense":
        vb = B * Hv * L * D * e
    else:
        vb = union_rows * D * e
    return kv + vb + 2 * B * Hq * D * e + 2 * B * (Hk + Hv) * D * e + B * Hq * 4


# ---------------------------------------------------------------------------
# The reference itself (noamelata/SAGA, installed unmodified into
# baseline/_ref by baseline/install_reference.sh)
# ---------------------------------------------------------------------------

REF_DIR = os.path.join(REPO, "baseline", "_ref")


def load_reference():
    """The reference's attention module from baseline/_ref, or None when the
    reference is not installed. Its Triton selection kernel is replaced by
    torch_threshold_topk (the Triton kernel needs a GPU); everything else is
    the reference's own code."""
    if not os.path.exists(os.path.join(REF_DIR, "attention", "attention.py")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import importlib
    A = importlib.import_module("attention.attention")
    if os.path.abspath(os.path.dirname(A.__file__)) != os.path.join(REF_DIR, "attention"):
        raise RuntimeError(f"attention.attention resolved to {A.__file__}, not the installed reference")
    return A


def torch_threshold_topk(x, k: int, threshold):
    """torch restatement of the reference's threshold_topk_fast
    (triton_atopn.py:59-113) for CPU tensors: per row, the elements with
    x > threshold (strict, fp32 compare, triton_atopn.py:42) compacted into k
    slots in ascending position order; padding vals = -inf, idx = 0
    (triton_atopn.py:82-84). When more than k pass, the k lowest positions are
    kept (the Triton kernel keeps an arbitrary k)."""
    import torch
    shape = x.shape
    L = shape[-1]
    xf = x.reshape(-1, L)
    R = xf.shape[0]
    t = threshold.reshape(-1).to(torch.float32)
    if t.numel() != R:
        t = t.repeat((R + t.numel() - 1) // t.numel())[:R]
    passing = xf.to(torch.float32) > t[:, None]
    rank = passing.cumsum(-1) - 1
    keep = passing & (rank < k)
    rows, cols = keep.nonzero(as_tuple=True)
    vals = torch.full((R, k), float("-inf"), dtype=x.dtype)
    idx = torch.zeros((R, k), dtype=torch.int64)
    slot = rank[rows, cols]
    vals[rows, slot] = xf[rows, cols]
    idx[rows, slot] = cols
    return vals.reshape(shape[:-1] + (k,)), idx.reshape(shape[:-1] + (k,))


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def make_cpu_inputs(shape, seed: int, dtype_name: str):
    """The workload's seeded synthetic tensors on the host (torch CPU)."""
    import torch
    B, L, Hq, Hk, Hv, D, N, plant = shape
    g = torch.Generator().manual_seed(seed)
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32}[dtype_name]
    s = 0.5 if dtype_name == "bf16" else 1.0
    q0 = torch.randn(B, Hq, 1, D, generator=g) * s
    q1 = 0.9 * q0 + math.sqrt(1 - 0.81) * torch.randn(B, Hq, 1, D, generator=g) * s
    k = torch.randn(B, Hk, L, D, generator=g) * s
    G = Hq // Hk
    for kk in range(Hk):
        qh = q0[:, kk * G, 0]
        qhat = qh / qh.norm(dim=-1, keepdim=True)
        pos = torch.randint(0, L, (B, plant), generator=g)
        k[torch.arange(B)[:, None], kk, pos] += 4.0 * qhat[:, None, :]
    v = torch.randn(B, Hv, L, D, generator=g) * s
    return q0.to(dt), q1.to(dt), k.to(dt), v.to(dt)


def reference_cpu(shape, steps: int, warmup: int, dtype_name: str = "bf16", budget_s: float = 60.0):
    """Time the reference's own amortized step (attention.py:192-209) on the
    host cores, all torch threads, on the whole batch of the workload per step.
    Returns the cpu_baseline dict, or None when the reference is absent."""
    import torch
    A = load_reference()
    if A is None:
        return None
    A._threshold_topk_triton = torch_threshold_topk
    B, L, Hq, Hk, Hv, D, N, plant = shape
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    q0, q1, k, v = make_cpu_inputs(shape, 0, dtype_name)
    with torch.no_grad():
        A.init_amortized_threshold_tensor("cpu", A.MAX_LAYERS, B * Hq)
        A.approx_top_n_attention_amortized_cal(q0, k, v, None, top_n_attention=N, layer_idx=0)
        for _ in range(max(1, warmup)):
            A.approx_top_n_attention_amortized(q1, k, v, None, top_n_attention=N, layer_idx=0)
        times = []
        t_start = time.perf_counter()
        for _ in range(max(1, steps)):
            t0 = time.perf_counter()
            A.approx_top_n_attention_amortized(q1, k, v, None, top_n_attention=N, layer_idx=0)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > budget_s:
                break
    t = statistics.median(times)
    return {"value": B / t, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
            "ms_per_step": round(t * 1e3, 3), "os_cpu_count": cores, "torch_threads": torch.get_num_threads(),
            "cpu_model": cpu_model(),
            "sample": f"the whole batch ({B} sequences) per step, {len(times)} steps, median; the reference's "
                      f"approx_top_n_attention_amortized from baseline/_ref in {dtype_name} on CPU tensors, "
                      f"its Triton selection replaced by a torch compaction (bench.torch_threshold_topk)"}


def graph_ms(torch, stream, fns, steps: int) -> float:
    """Device ms per call of the step functions `fns` (already warmed up),
    replayed from one CUDA graph that holds one call of each."""
    with torch.cuda.stream(stream):
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for f in fns:
                f()
        for _ in range(3):
            graph.replay()
        stream.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = max(1, steps // len(fns))
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * len(fns))
    del graph
    return ms


def gpu_baselines(torch, ops, shape, dev, caches, steps: int):
    """On this GPU, beside the timed step: the reference's own GPU path (its
    attention.py with the Triton selection kernel, from baseline/_ref) on the
    same caches, and dense GQA decode of the same model with its unmerged key
    heads (Hk = Hv) by this library's dense kernel and by the reference's
    full_einsum_forward (torch bmm). Every step replays from a CUDA graph over
    rotating caches larger than L2; no torch.compile."""
    B, L, Hq, Hk, Hv, D, N, _ = shape
    out = {}
    stream = torch.cuda.Stream(device=dev)
    A = load_reference()
    if A is not None:
        try:
            copies = len(caches)
            with torch.cuda.stream(stream):
                A.init_amortized_threshold_tensor(dev, A.MAX_LAYERS, B * Hq)
                for c in range(copies):
                    A.approx_top_n_attention_amortized_cal(caches[c][0], caches[c][2], caches[c][3], None,
                                                           top_n_attention=N, layer_idx=c)
                fns = [(lambda c=c: A.approx_top_n_attention_amortized(caches[c][1], caches[c][2], caches[c][3], None,
                                                                      top_n_attention=N, layer_idx=c))
                       for c in range(copies)]
                for f in fns:  # Triton compiles here
                    f()
            out["reference_atopn_us"] = round(1e3 * graph_ms(torch, stream, fns, steps), 3)
        except Exception as e:  # the reference's GPU path is a reported baseline only
            out["reference_atopn_error"] = f"{type(e).__name__}: {e}"[:300]
    # the calibration step (first decode step of a generation) on the same
    # caches, with its algorithmic bytes: the key cache, and the value rows of
    # the union of the top-N sets of the heads sharing a value head
    copies = len(caches)
    thr_c = [torch.zeros(B * Hq, dtype=torch.float32, device=dev) for _ in range(copies)]
    d = {}
    ops.atopn_calibrate(caches[0][1], caches[0][2], caches[0][3], None, thr_c[0], N, diag=d)
    torch.cuda.synchronize()
    sel = d["sel_idx"].cpu()
    Gv = Hq // Hv
    union = 0
    for b in range(B):
        for vh in range(Hv):
            rows = set()
            for h in range(vh * Gv, (vh + 1) * Gv):
                rows.update(sel[b * Hq + h, :N].tolist())
            rows.discard(-1)
            union += len(rows)
    with torch.cuda.stream(stream):
        fns = [(lambda c=c: ops.atopn_calibrate(caches[c][1], caches[c][2], caches[c][3], None, thr_c[c], N))
               for c in range(copies)]
        for f in fns:
            f()
    cal_ms = graph_ms(torch, stream, fns, steps)
    cal_bytes = B * Hk * L * D * 2 + union * D * 2
    peak, peak_kind = measured_peaks()
    out["calibrate_us"] = round(1e3 * cal_ms, 3)
    out["calibrate_roofline"] = {"bound": "hbm", "achieved": round(cal_bytes / (cal_ms * 1e-3) / 1e9, 1), "peak": peak,
                                 "unit": "GB/s", "frac": round(cal_bytes / (cal_ms * 1e-3) / 1e9 / peak, 4),
                                 "peak_kind": peak_kind, "algorithmic_bytes_per_step": cal_bytes,
                                 "value_rows_union_per_step": union}
    if A is not None:
        try:
            with torch.cuda.stream(stream):
                fns = [(lambda c=c: A.approx_top_n_attention_amortized_cal(caches[c][1], caches[c][2], caches[c][3], None,
                                                                          top_n_attention=N, layer_idx=c))
                       for c in range(copies)]
                for f in fns:
                    f()
            out["reference_calibrate_us"] = round(1e3 * graph_ms(torch, stream, fns, steps), 3)
        except Exception as e:
            out["reference_calibrate_error"] = f"{type(e).__name__}: {e}"[:300]
    # dense GQA of the unmerged model (the reference's baseline, eval.md:60-65)
    gshape = (B, L, Hq, Hv, Hv, D, N, 0)
    gq = [make_device_inputs(torch, gshape, dev, seed=100 + c) for c in range(2)]
    with torch.cuda.stream(stream):
        fns = [(lambda c=c: ops.dense_decode(gq[c][1], gq[c][2], gq[c][3], None)) for c in range(2)]
        for f in fns:
            f()
    out["dense_gqa_us"] = round(1e3 * graph_ms(torch, stream, fns, steps), 3)
    if A is not None:
        with torch.cuda.stream(stream):
            fns = [(lambda c=c: A.full_einsum_forward(gq[c][1], gq[c][2], gq[c][3], None)) for c in range(2)]
            for f in fns:
                f()
        out["reference_dense_gqa_us"] = round(1e3 * graph_ms(torch, stream, fns, steps), 3)
    out["dense_gqa_heads"] = [Hq, Hv, Hv]
    out["how"] = ("CUDA graphs of the steps over rotating caches (> L2); the reference from baseline/_ref "
                  "(attention.py + triton_atopn.py), its amortized step on this line's caches, without "
                  "torch.compile and without the KV append")
    del gq
    torch.cuda.synchronize()
    return out


def config4_leg(torch, dist, ops, dev, rank: int, world: int, steps: int):
    """Config 4 sequence-sharded over the job's ranks (one process per GPU),
    beside the replica line: batch 1, context 131072, Hq 12 / Hk 1 / Hv 2,
    head_dim 128, N 1024. Every rank holds its shard of the same sequence
    (plus the 256-row tail replica); the calibration step and the amortized
    step each run as one launch per device, exchanging through peer-mapped
    workspaces. Timed as the max over ranks of device events over rotating
    shard copies whose bytes exceed twice L2. Checked against the unsharded
    kernel on the full cache, on this box: outputs (max-abs / relative RMS),
    thresholds (equal or one ulp apart) and selected sets (merged over the
    ranks; equal except positions within one ulp of the threshold)."""
    from saga_b200.seqpar import ShardedDecode, shard_cache, shard_layout
    shape = WORKLOADS["config4"]
    B, L, Hq, Hk, Hv, D, N, _ = shape
    lay = shard_layout(L, world, rank)
    per_copy = (Hk + Hv) * lay.local_len * D * 2 * B
    copies = max(2, math.ceil(2 * L2_BYTES / per_copy))
    shards, full0 = [], None
    for c in range(copies):  # the same sequences on every rank (seed c), sharded
        q0, q1, k, v, kn, vn = make_device_inputs(torch, shape, dev, seed=500 + c)
        shards.append((q0, q1, shard_cache(k, lay), shard_cache(v, lay)))
        if c == 0:
            full0 = (q0, q1, k, v)
        else:
            del k, v
    sdc = ShardedDecode(dist.group.WORLD, dev, B, L, Hq, Hk, Hv, D, op="calibrate")
    sda = ShardedDecode(dist.group.WORLD, dev, B, L, Hq, Hk, Hv, D, op="atopn")
    thrs = [torch.zeros(B * Hq, dtype=torch.float32, device=dev) for _ in range(copies)]
    stream = torch.cuda.Stream(device=dev)

    def run(fns, reps):
        # every rank launches the same steps in the same order: warm-up, then
        # one CUDA graph of one step per copy, replayed reps times
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for f in fns:
                f()
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for f in fns:
                    f()
            graph.replay()
            stream.synchronize()
            dist.barrier()
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        del graph
        return max_over_ranks(torch, dist, e0.elapsed_time(e1) / (reps * len(fns)), dev, world)

    reps = max(1, steps // copies)
    cal_ms = run([(lambda c=c: sdc(shards[c][0], shards[c][2], shards[c][3], thrs[c], N)) for c in range(copies)],
                 max(1, reps // 4))
    amo_ms = run([(lambda c=c: sda(shards[c][1], shards[c][2], shards[c][3], thrs[c], N)) for c in range(copies)], reps)
    # the check: this rank's sharded result against the unsharded kernel on copy 0
    q0, q1, k, v = full0
    thr_u = torch.zeros(B * Hq, dtype=torch.float32, device=dev)
    thr_s = torch.zeros_like(thr_u)
    du, ds = {}, {}
    ref_c = ops.atopn_calibrate(q0, k, v, None, thr_u, N)
    out_c = sdc(q0, shards[0][2], shards[0][3], thr_s, N)
    ref_a = ops.atopn_decode(q1, k, v, None, thr_u, N, diag=du)
    out_a = sda(q1, shards[0][2], shards[0][3], thr_u, N, diag=ds)
    torch.cuda.synchronize()
    parts = [None] * world
    dist.all_gather_object(parts, ds["sel_idx"].cpu())
    check = None
    if rank == 0:
        def close(a, b):
            a, b = a.float(), b.float()
            return (round((a - b).abs().max().item(), 6),
                    round(((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt().clamp_min(1e-12)).item(), 6))
        merged = torch.stack(parts).amax(0)
        ref_sel, cnt, t = du["sel_idx"].cpu(), du["count"].cpu(), du["logit_thr"].cpu()
        lg = ops.attn_logits(q1, k).float().cpu().reshape(B * Hq, L)
        sets_ok, diff = True, 0
        for r in range(B * Hq):
            kept = min(int(cnt[r]), 2 * N)
            a_, b_ = set(merged[r, :kept].tolist()), set(ref_sel[r, :kept].tolist())
            d = a_ ^ b_
            diff += len(d)
            if -1 in a_:
                sets_ok = False
            for pos in d:  # a difference must be a tie: within one bf16 ulp of t
                x, tt = float(lg[r, pos]), float(t[r])
                ulp = 2.0 ** (math.floor(math.log2(max(abs(tt), 1e-30))) - 7)
                if abs(x - tt) > ulp:
                    sets_ok = False
        thr_ulps = []
        for a_, b_ in zip(thr_s.cpu().tolist(), thr_u.cpu().tolist()):
            ulp = 2.0 ** (math.floor(math.log2(max(abs(b_), 1e-30))) - 7)
            thr_ulps.append(abs(a_ - b_) / ulp)
        check = {"amortized_max_abs_rel_rms": close(out_a, ref_a), "calibrate_max_abs_rel_rms": close(out_c, ref_c),
                 "sets_equal_except_ties": sets_ok, "set_positions_differing": diff,
                 "thresholds_max_ulps": max(thr_ulps), "rows": B * Hq}
        am, cm = check["amortized_max_abs_rel_rms"], check["calibrate_max_abs_rel_rms"]
        check["passed"] = bool(sets_ok and check["thresholds_max_ulps"] <= 1.0 and am[0] <= 2e-2 and am[1] <= 1e-2
                               and cm[0] <= 2e-2 and cm[1] <= 1e-2)
    st = ops.read_status(dev)
    dist.barrier()
    sdc.close()
    sda.close()
    dist.barrier()
    return {"workload": f"config4: batch {B}, context {L}, Hq {Hq} / Hk {Hk} / Hv {Hv}, head_dim {D}, N {N}, "
                        f"sequence-sharded over {world} GPUs", "us_per_step": round(amo_ms * 1e3, 3),
            "tokens_per_s": round(B / (amo_ms * 1e-3), 1), "calibrate_us_per_step": round(cal_ms * 1e3, 3),
            "copies": copies, "status": st, "check": check,
            "exchange": "peer-mapped workspaces over NVLink (system-scope slots, histogram atomics and barriers); "
                        "no collective on the data path"}


def reference_harness():
    """The reference's benchmark module (speedup.py, from baseline/_ref,
    unchanged) with this package standing in for its `attention` package:
    speedup's `from attention.attention import ...` and
    `from attention.triton_atopn import _BUFFER_CACHE` resolve to
    saga_b200.attention, as they would with this package ahead on sys.path."""
    import importlib
    import saga_b200.attention as SP
    import saga_b200.attention.attention as SA
    import saga_b200.attention.triton_atopn as ST
    if not os.path.exists(os.path.join(REF_DIR, "speedup.py")):
        raise RuntimeError("the reference is not installed (bash baseline/install_reference.sh)")
    sys.modules["attention"] = SP
    sys.modules["attention.attention"] = SA
    sys.modules["attention.triton_atopn"] = ST
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    sp = importlib.import_module("speedup")
    assert sp.approx_top_n_attention_amortized is SA.approx_top_n_attention_amortized
    if not getattr(sp, "_saga_cache_fix", False):
        # Compatibility with the installed transformers (5.5; the reference pins
        # 5.3): its StaticLayer keeps a cumulative_length tensor that only its
        # own lazy initialisation moves to the device. speedup.py:119-139 marks
        # the hand-built layers initialised itself, so the counter stays on the
        # host and the model's position arithmetic mixes devices. The wrapper
        # moves it; the caches and everything else are the reference's.
        import torch
        orig = sp.initialize_kv_cache

        def initialize_kv_cache(model, max_cache_len, num_key_heads=None, device="cuda", dtype=torch.float32):
            cache = orig(model, max_cache_len, num_key_heads=num_key_heads, device=device, dtype=dtype)
            for layer in getattr(cache, "layers", []):
                cl = getattr(layer, "cumulative_length", None)
                if isinstance(cl, torch.Tensor) and getattr(layer, "is_initialized", False):
                    layer.cumulative_length = cl.to(device)
            return cache

        sp.initialize_kv_cache = initialize_kv_cache
        sp._saga_cache_fix = True
    return sp


def build_model(torch, family, layers, hidden, heads, kv_heads, head_dim, mlp, vocab, ctx, dev):
    """A random-init model of the named family's shape: bf16 weights ~ N(0, 0.02)."""
    from transformers import AutoModelForCausalLM, LlamaConfig, Qwen2Config
    kw = dict(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=head_dim,
              intermediate_size=mlp, vocab_size=vocab, num_hidden_layers=layers, max_position_embeddings=ctx,
              initializer_range=0.02, attn_implementation="sdpa")
    cfg = LlamaConfig(tie_word_embeddings=True, **kw) if family == "llama" else Qwen2Config(**kw)
    torch.manual_seed(0)
    with torch.device(dev):
        model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16)
    return model.eval()


def decode_graph_ms(torch, sp, model, input_ids, new_heads, new_tokens: int, iterations: int, atopn: bool):
    """Per-token decode time of one generation of `new_tokens`, by the protocol
    of the reference's speedup.measure_decode_latency with use_cuda_graph
    (speedup.py:197-291, 293-440): prefill at batch 1 and repeat over the batch
    (its own prefill()), the decode step captured in CUDA graphs (for Atop-N
    one calibration graph for the first token, one amortized graph for the
    rest), then replayed with the argmax token fed back, the threshold table
    reset before every generation. Restated rather than called: with the
    installed transformers a StaticLayer ignores the cache position and
    advances its own device counter on every update, so the harness's
    warm-up forwards and replays would write past the cache's end. Here each
    captured step first sets every layer's counter back to the prefilled
    length, so every replay writes the same position, which is what the
    harness intends ("the graph always writes to the same cache_position").
    Device time of the replays (CUDA events)."""
    dev = input_ids.device
    with torch.no_grad():
        if atopn:
            sp._AMORTIZED_STEP_COUNT = 0
        past_kv, next_token = sp.prefill(model, input_ids, new_heads, dtype=torch.bfloat16, num_new_tokens=new_tokens)
        if atopn:
            sp.init_amortized_threshold_tensor(dev, sp.MAX_LAYERS, next_token.shape[0] * model.config.num_attention_heads)
        seen = int(past_kv.layers[0].cumulative_length.item())
        position_ids = torch.arange(seen, seen + 1, device=dev, dtype=torch.long).unsqueeze(0)
        batch = past_kv.layers[0].keys.shape[0]
        static_input = torch.empty_like(next_token)
        static_logits = torch.empty(batch, 1, model.config.vocab_size, device=dev, dtype=torch.bfloat16)
        counters = [layer.cumulative_length for layer in past_kv.layers]

        def step():
            for c in counters:  # every replay writes the decode token at `seen`
                c.fill_(seen)
            # the causal mask is built inside the step from the counter (the
            # installed transformers takes no precomputed per-type mask dict)
            out = model(static_input, past_key_values=past_kv, use_cache=True, position_ids=position_ids)
            static_logits.copy_(out.logits[:, -1:, :])

        static_input.copy_(next_token)
        if dev.type != "cuda":  # host dry run of the same steps (no graphs, no timing)
            for i in range(new_tokens):
                sp._AMORTIZED_STEP_COUNT = 0 if (atopn and i == 0) else 2
                step()
                static_input.copy_(static_logits.argmax(dim=-1))
            return float("nan")
        graphs = {}
        for name, count in ((("cal", 0), ("fast", 2)) if atopn else (("fast", 2),)):
            sp._AMORTIZED_STEP_COUNT = count
            step()  # warm-up outside the capture (lazy set-up, workspaces)
            torch.cuda.synchronize()
            sp._AMORTIZED_STEP_COUNT = count
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                step()
            graphs[name] = gr
        times = []
        for it in range(iterations + 1):  # the first generation is a warm-up
            if atopn:
                sp.reset_amortized_state()
            tok = next_token
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(new_tokens):
                static_input.copy_(tok)
                graphs["cal" if (atopn and i == 0) else "fast"].replay()
                tok = static_logits.argmax(dim=-1)
            e1.record()
            torch.cuda.synchronize()
            if it > 0:
                times.append(e0.elapsed_time(e1) / new_tokens)
        del graphs, past_kv
    return statistics.median(times)


def model_bench(args, world: int, rank: int, local_rank: int):
    """Decode tokens/s of a whole random-init model, decoded by the protocol
    of the reference's speedup.measure_decode_latency (decode_graph_ms) with
    this package's attention module standing in for the reference's, the
    reference's own dispatcher (speedup.sdpa_attention_forward_dispatch),
    prefill and key-head merge. The SAGA model (key projection merged to one
    head, Atop-N with the calibration at the first decode step) is reported
    next to the same model with its unmerged key heads and dense attention: the
    reference's "full" mode (this package's dense kernel) and plain SDPA.
    Batch-sharded: every rank decodes batch / ranks sequences of its own; the
    job's rate uses the slowest rank's time."""
    import torch
    import torch.distributed as dist
    family, layers, hidden, heads, vh, hd, mlp, vocab, B, ctx, new, N, dense_kv = MODELS[args.workload]
    if B % world:
        raise SystemExit(f"batch {B} does not split over {world} ranks")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800), device_id=dev)
    sp = reference_harness()
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sp.sdpa_attention_forward_dispatch
    b_rank = B // world
    g = torch.Generator().manual_seed(1000 + rank)
    input_ids = torch.randint(0, vocab, (b_rank, ctx), generator=g, dtype=torch.long).to(dev)
    runs = {}

    def measure(name, kv_heads, mode, merge):
        model = build_model(torch, family, layers, hidden, heads, kv_heads, hd, mlp, vocab, ctx + new + 8, dev)
        if merge:
            model = sp.merge_key_projection_heads(model, new_heads=1)
        if args.compile:
            model.forward = torch.compile(model.forward)
        sp.ATTENTION_MODE = mode
        sp.TOP_N_ATTENTION = N if mode == "atopn" else None
        err = None
        try:
            ms = decode_graph_ms(torch, sp, model, input_ids, 1 if merge else None, new, args.iterations,
                                 mode == "atopn")
        except torch.cuda.OutOfMemoryError:
            ms, err = float("inf"), "out of memory"
        del model
        import gc
        gc.collect()
        torch.cuda.empty_cache()
        from saga_b200 import ops
        st = ops.read_status(dev)
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        runs[name] = {"ms_per_token": round(ms, 4) if ms != float("inf") else None,
                      "tokens_per_s": round(B / (ms * 1e-3), 1) if ms != float("inf") else None,
                      "key_heads": 1 if merge else kv_heads, "value_heads": kv_heads, "attention": mode,
                      "status": st}
        if err:
            runs[name]["error"] = err

    measure("saga_atopn", vh, "atopn", True)
    measure("dense_full", dense_kv, "full", False)
    measure("dense_sdpa", dense_kv, "vanilla", False)
    if rank == 0:
        saga, dense = runs["saga_atopn"], [runs["dense_full"], runs["dense_sdpa"]]
        best = min([d["ms_per_token"] for d in dense if d["ms_per_token"]] or [float("nan")])
        line = {"metric": f"decode tokens/s of the whole model ({args.workload}: {family}-shaped SAGA model)",
                "value": saga["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.iterations * new,
                "warmup": new, "ms_per_step": saga["ms_per_token"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random token ids)",
                "config": {"workload": f"{args.workload}: {layers} layers, hidden {hidden}, {heads} query heads, "
                                       f"1 key head / {vh} value heads, head_dim {hd}, MLP {mlp}, vocab {vocab}, "
                                       f"batch {B}, context {ctx}, {new} new tokens, N {N}",
                           "parallelism": f"replicas x{world} (batch-sharded, no collective)",
                           "harness": "the protocol of the reference's measure_decode_latency with CUDA graphs "
                                      "(its prefill, merge and dispatcher); device time of the replays" +
                                      (", torch.compile(model.forward)" if args.compile else "")},
                "runs": runs,
                "atopn_speedup_vs_faster_dense": round(best / saga["ms_per_token"], 3) if saga["ms_per_token"] else None}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference's algorithm)
# ---------------------------------------------------------------------------

def cpu_baseline(shape, steps: int, budget_s: float = 20.0):
    """Time the numpy oracle's amortized step on one sequence of the workload."""
    import numpy as np
    from oracle import atopn_oracle as O
    from saga_b200.workloads import DecodeShape, make_inputs
    B, L, Hq, Hk, Hv, D, N, plant = shape
    sh = DecodeShape(B=1, L=L, Hq=Hq, Hk=Hk, Hv=Hv, D=D, N=N, dtype="bf16", scale=0.5, plant=plant)
    inp = make_inputs(sh, seed=7)
    cal = O.atopn_calibrate(inp.q0, inp.k, inp.v, N, "bf16")
    times = []
    t_start = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        O.atopn_amortized(inp.q1, inp.k, inp.v, cal["thr"], N, "bf16")
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    t = statistics.median(times)
    cores = os.cpu_count() or 1
    return {"value": 1.0 / t, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"1 of {B} sequences of the workload per step, {len(times)} steps, median {t * 1e3:.1f} ms; "
                      f"numpy oracle (BLAS threads up to {cores} for the logits GEMM, other ops 1 thread)"}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def main():
    args = parse()
    if args.workload in MODELS:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "model workloads run the reference's harness "
                                  "with this package as its attention module; the reference's own model decode "
                                  "needs its Triton kernel on a GPU and is not a CPU baseline"}))
            return
        return model_bench(args, world, int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")))
    shape = WORKLOADS[args.workload]
    B, L, Hq, Hk, Hv, D, N, _ = shape
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    # config 4 runs one long sequence sharded over the ranks (strong scaling);
    # the other workloads run one replica per rank (weak scaling)
    sharded = args.workload == "config4" and world > 1 and args.mode in ("atopn", "dense")
    config = {"workload": f"{args.workload}: one SAGA attention layer, batch {B}, context {L}, "
                          f"Hq {Hq} / Hk {Hk} / Hv {Hv}, head_dim {D}, N {N}, mode {args.mode}",
              "batch_per_gpu": B, "seq_len": L, "heads": [Hq, Hk, Hv], "head_dim": D, "top_n": N,
              "parallelism": (f"sequence-sharded x{world} (one fused launch per device; exchanges through "
                              f"peer-mapped workspaces over NVLink, no collective on the data path)") if sharded
              else f"replicas x{world} (batch-sharded, no collective)",
              "l2": "rotating KV-cache copies, each step reads a cache not in L2"}
    metric = "decode tokens/s of one Atop-N attention layer (config 2 shapes)"
    if args.mode != "atopn" or args.workload != "config2":
        metric = f"decode tokens/s of one attention layer, {args.mode} ({args.workload} shapes)"
    unit = "tokens/s"

    if args.impl == "reference":
        if rank != 0:
            return
        dtn = "fp32" if args.workload == "config1" else "bf16"
        cb = reference_cpu(shape, args.steps, args.warmup, dtn, budget_s=max(60.0, 3.0 * args.steps))
        if cb is None:  # the reference is not installed: the numpy port of its algorithm
            cb = cpu_baseline(shape, args.steps, budget_s=max(20.0, 0.5 * args.steps))
        line = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": unit, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * B / cb["value"] if cb["kind"] == "reference"
                else 1e3 / cb["value"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtn,
                "data": "synthetic", "config": config, "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if args.workload != "config1":  # the CPU-runnable case beside it
            c1 = reference_cpu(WORKLOADS["config1"], 20, 3, "fp32", budget_s=20.0)
            if c1 is not None:
                line["config1_cpu"] = c1
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist
    from saga_b200 import ops
    from saga_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    copies = 4 if (B * Hk * L * D * 2) < 2 * L2_BYTES else 1
    caches = [make_device_inputs(torch, shape, dev, seed=c if sharded else replica_seed(rank, c))
              for c in range(copies)]
    q1 = caches[0][1]
    thrs = []
    for c in range(copies):
        q0c, _, kc, vc, _, _ = caches[c]
        t = torch.zeros(B * Hq, dtype=torch.float32, device=dev)
        ops.atopn_calibrate(q0c, kc, vc, None, t, N)
        thrs.append(t)
    torch.cuda.synchronize()

    # union of the value rows the step needs (for the algorithmic bytes)
    diag = {}
    ops.atopn_decode(q1, caches[0][2], caches[0][3], None, thrs[0], N, diag=diag)
    torch.cuda.synchronize()
    sel = diag["sel_idx"].cpu()
    cnt = diag["count"].cpu().clamp(max=min(2 * N, L))
    union = 0
    Gv = Hq // Hv
    for b in range(B):
        for vh in range(Hv):
            s = set()
            for h in range(vh * Gv, (vh + 1) * Gv):
                r = b * Hq + h
                s.update(sel[r, :int(cnt[r])].tolist())
            union += len(s)
    overflow_rows = int((diag["count"].cpu() > min(2 * N, L)).sum())
    if args.mode != "atopn":  # the launches of the timed mode
        d2 = {}
        if args.mode == "dense":
            ops.dense_decode(q1, caches[0][2], caches[0][3], None, diag=d2)
        else:
            ops.atopn_calibrate(q1, caches[0][2], caches[0][3], None, thrs[0].clone(), N, diag=d2)
        diag["launches"] = d2["launches"]
    launches_per_step = len(diag["launches"])
    ops.read_status(dev)

    sd = None
    if sharded:
        from saga_b200.seqpar import ShardedDecode, shard_cache
        sd = ShardedDecode(dist.group.WORLD, dev, B, L, Hq, Hk, Hv, D, op=args.mode)
        # keep only this rank's shard (+ tail replica) of every cache copy
        caches = [(c[0], c[1], shard_cache(c[2], sd.lay), shard_cache(c[3], sd.lay), c[4], c[5]) for c in caches]
        torch.cuda.synchronize()

    def step(i, q):
        _, _, kc, vc, kn, vn = caches[i % copies]
        if sd is not None:
            return sd(q, kc, vc, thrs[i % copies], N, k_new=kn, v_new=vn, append_pos=L - 1)
        if args.mode == "atopn":
            return ops.atopn_decode(q, kc, vc, None, thrs[i % copies], N, k_new=kn, v_new=vn, append_pos=L - 1)
        if args.mode == "dense":
            return ops.dense_decode(q, kc, vc, None, k_new=kn, v_new=vn, append_pos=L - 1)
        return ops.atopn_calibrate(q, kc, vc, None, thrs[i % copies], N)

    # CUDA graph of one step per cache copy (device timing without host gaps)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup)):
            step(i, q1)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                step(i, q1)
    reps = max(1, math.ceil(args.steps / copies))
    steps_timed = reps * copies

    props = torch.cuda.get_device_properties(dev)
    gpu_id = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local_rank)
    sampler = ClockSampler(gpu_id, enabled=not args.no_clocks)
    sampler.start()
    with torch.cuda.stream(stream):
        if sharded:
            # the shards of a step run together: every rank replays the same
            # number of steps (a rank with an extra launch would wait for a
            # partner launch that never comes)
            for _ in range(max(1, 2000 // copies)):
                graph.replay()
            stream.synchronize()
        else:
            t_soak = time.perf_counter()
            while time.perf_counter() - t_soak < 0.5:   # untimed soak so the clocks settle
                graph.replay()
                stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replays and events on the same stream
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = max_over_ranks(torch, dist, e0.elapsed_time(e1) / steps_timed, dev, world)
    status = ops.read_status(dev)

    # End to end with host buffers. Every step copies one pinned host block
    # (the query and the decode token's key/value rows) into the device block
    # the step reads, runs the step, and copies the output back to pinned
    # host memory. Two API levels are timed: the serving API (ops.DecodeStep,
    # arguments bound once, one C-ABI call per step) as "e2e", and the
    # per-call functions the reference's module API goes through
    # (ops.atopn_decode & co., arguments built every call) as "e2e_per_call".
    nq, nk, nv = B * Hq * D, B * Hk * D, B * Hv * D
    hin = torch.empty(nq + nk + nv, dtype=torch.bfloat16, pin_memory=True)
    hin[:nq].copy_(q1.reshape(-1).cpu())
    hin[nq:nq + nk].copy_(caches[0][4].reshape(-1).cpu())
    hin[nq + nk:].copy_(caches[0][5].reshape(-1).cpu())
    din = torch.empty(hin.shape, dtype=hin.dtype, device=dev)
    qd = din[:nq].view(B, Hq, 1, D)
    knd = din[nq:nq + nk].view(B, Hk, 1, D)
    vnd = din[nq + nk:].view(B, Hv, 1, D)
    hout = torch.empty((B, Hq, 1, D), dtype=torch.bfloat16, pin_memory=True)
    h2d = hin.numel() * 2
    d2h = hout.numel() * 2
    ne = max(copies, args.e2e_steps)
    bound = None
    if sd is None:
        bound = []
        for c in range(copies):
            _, _, kc, vc, _, _ = caches[c]
            if args.mode == "calibrate":
                bound.append(ops.DecodeStep("calibrate", qd, kc, vc, threshold=thrs[c], top_n=N))
            else:
                bound.append(ops.DecodeStep(args.mode, qd, kc, vc, threshold=thrs[c] if args.mode == "atopn" else None,
                                            top_n=N, k_new=knd, v_new=vnd, append_pos=L - 1))

    def per_call(i):
        _, _, kc, vc, _, _ = caches[i % copies]
        if sd is not None:
            return sd(qd, kc, vc, thrs[i % copies], N, k_new=knd, v_new=vnd, append_pos=L - 1)
        if args.mode == "atopn":
            return ops.atopn_decode(qd, kc, vc, None, thrs[i % copies], N, k_new=knd, v_new=vnd, append_pos=L - 1)
        if args.mode == "dense":
            return ops.dense_decode(qd, kc, vc, None, k_new=knd, v_new=vnd, append_pos=L - 1)
        return ops.atopn_calibrate(qd, kc, vc, None, thrs[i % copies], N)

    def e2e_ms(run):
        def e2e_step(i):
            din.copy_(hin, non_blocking=True)
            hout.copy_(run(i), non_blocking=True)
        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        f0.record()
        for i in range(ne):
            e2e_step(i)
        f1.record()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(torch, dist, f0.elapsed_time(f1) / ne, dev, world)

    def e2e_pipelined_ms():
        """The serving loop: the bound steps of two slots (device input block,
        output), the host-to-device copies on one stream, the steps on
        another, the device-to-host copies on a third. Step i's input copy
        waits only for step i-2 (the last reader of its slot), so it runs
        under step i-1's kernel, and step i's output copy under step i+1's."""
        dins = [din, torch.empty_like(din)]
        outs = [torch.empty((B, Hq, 1, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        houts = [hout, torch.empty_like(hout).pin_memory()]
        slots = []
        for s_ in range(2):
            qs = dins[s_][:nq].view(B, Hq, 1, D)
            kns = dins[s_][nq:nq + nk].view(B, Hk, 1, D)
            vns = dins[s_][nq + nk:].view(B, Hv, 1, D)
            row = []
            for c in range(copies):
                _, _, kc, vc, _, _ = caches[c]
                if args.mode == "calibrate":
                    row.append(ops.DecodeStep("calibrate", qs, kc, vc, threshold=thrs[c], top_n=N, out=outs[s_]))
                else:
                    row.append(ops.DecodeStep(args.mode, qs, kc, vc,
                                              threshold=thrs[c] if args.mode == "atopn" else None, top_n=N,
                                              k_new=kns, v_new=vns, append_pos=L - 1, out=outs[s_]))
            slots.append(row)
        comp = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_k = [torch.cuda.Event() for _ in range(2)]
        ev_dr = [torch.cuda.Event() for _ in range(2)]
        comp_h = comp.cuda_stream

        def submit(i):
            s_ = i & 1
            s_in.wait_event(ev_k[s_])
            with torch.cuda.stream(s_in):
                dins[s_].copy_(hin, non_blocking=True)
            ev_in[s_].record(s_in)
            comp.wait_event(ev_in[s_])
            comp.wait_event(ev_dr[s_])
            slots[s_][i % copies](comp_h)
            ev_k[s_].record(comp)
            s_out.wait_event(ev_k[s_])
            with torch.cuda.stream(s_out):
                houts[s_].copy_(outs[s_], non_blocking=True)
            ev_dr[s_].record(s_out)

        def run(n):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(comp)
            for e in ev_k + ev_dr:  # every wait of the first steps is on work after `start`
                e.record(comp)
            for i in range(n):
                submit(i)
            for e in ev_dr:
                comp.wait_event(e)
            end.record(comp)
            return start, end

        run(4)
        torch.cuda.synchronize()
        barrier()
        f0, f1 = run(ne)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(torch, dist, f0.elapsed_time(f1) / ne, dev, world)

    ms_e2e_call = e2e_ms(per_call)
    call_api = "seqpar.ShardedDecode" if sd is not None else \
        {"atopn": "ops.atopn_decode", "dense": "ops.dense_decode", "calibrate": "ops.atopn_calibrate"}[args.mode]
    ms_e2e_serial = e2e_ms(lambda i: bound[i % copies]()) if bound is not None else ms_e2e_call
    ms_e2e = e2e_pipelined_ms() if bound is not None else ms_e2e_call

    baselines = None
    if world == 1 and args.workload in ("config2", "config3_layer", "config5_layer") and args.mode == "atopn":
        baselines = gpu_baselines(torch, ops, shape, dev, caches, min(400, max(40, args.steps)))
    c4 = None
    if world > 1 and not sharded and args.mode == "atopn" and not args.no_config4:
        c4 = config4_leg(torch, dist, ops, dev, rank, world, min(400, max(40, args.steps)))
    if sd is not None:  # unmap the peers' workspaces once every rank is done with them
        barrier()
        sd.close()
        barrier()
    peak, peak_kind = measured_peaks()
    abytes = algorithmic_bytes(shape, union, args.mode)
    # per device: a sharded step spreads the job's bytes over the ranks
    achieved = abytes / (world if sharded else 1) / (ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "frac_of_8TBs_nominal": round(achieved / 8000.0, 4),
                "traffic": ncu_traffic(args.workload, args.mode), "algorithmic_bytes_per_step": abytes,
                "kernel": "saga_decode_kernel<amortized>" if args.mode == "atopn" else f"saga_decode_kernel<{args.mode}>"}
    if rank == 0:
        ranks_b = 1 if sharded else world  # a sharded job decodes one batch per step over all ranks
        line = {"metric": metric, "value": round(job_throughput(B, ranks_b, ms), 1), "unit": unit, "n_gpus": world,
                "steps": steps_timed, "warmup": args.warmup, "ms_per_step": round(ms, 5),
                "us_per_layer_step": round(ms * 1e3, 3),
                "higher_is_better": True, "scaling": "strong" if sharded else "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic", "config": config,
                "e2e": {"value": round(job_throughput(B, ranks_b, ms_e2e), 1), "unit": unit, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 5),
                        "api": ("ops.DecodeStep, copies on two side streams overlapping the steps" if bound is not None
                                else "seqpar.ShardedDecode")},
                "e2e_serial": {"value": round(job_throughput(B, ranks_b, ms_e2e_serial), 1), "unit": unit,
                               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                               "ms_per_step": round(ms_e2e_serial, 5),
                               "api": "ops.DecodeStep" if bound is not None else call_api},
                "e2e_per_call": {"value": round(job_throughput(B, ranks_b, ms_e2e_call), 1), "unit": unit,
                                 "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                                 "ms_per_step": round(ms_e2e_call, 5),
                                 "api": call_api},
                "roofline": roofline, "clocks": clocks,
                "gpu_launches": steps_timed * launches_per_step,
                "kernels_per_step": diag["launches"], "status": status,
                "overflow_rows": overflow_rows, "rows": B * Hq,
                "value_rows_union_per_step": union}
        if c4 is not None:
            line["config4_sharded"] = c4
        if baselines is not None:
            baselines["atopn_us"] = round(ms * 1e3, 3)
            dense = min([x for x in (baselines.get("dense_gqa_us"), baselines.get("reference_dense_gqa_us")) if x])
            baselines["atopn_speedup_vs_faster_dense"] = round(dense / (ms * 1e3), 3)
            if baselines.get("reference_atopn_us"):
                baselines["speedup_vs_reference_gpu"] = round(baselines["reference_atopn_us"] / (ms * 1e3), 3)
            line["gpu_baselines"] = baselines
        if not args.no_cpu_baseline:
            cb = reference_cpu(shape, 3, 1, "bf16", budget_s=30.0)
            line["cpu_baseline"] = cb if cb is not None else cpu_baseline(shape, steps=3)
        print(json.dumps(line))
    if world > 1:
        del graph
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
