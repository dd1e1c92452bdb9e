"""Phase trace of the fused decode kernel (diagnostics).

The kernel stamps the time at which each CTA reaches the phases of a step
when the library is built with the trace compiled in:

    SAGA_PHASE_TRACE=1 python -m saga_b200.build --force
    python -m saga_b200.phase_trace --B 8 --L 32768 --Hq 12 --Hk 1 --Hv 2 --D 128 --N 512 --mode calibrate
    python -m saga_b200.build --force          # back to the product build

and prints, as one JSON object, the median over CTAs (and launches) of
* p<k>: global-timer stamps in microseconds from the first CTA's entry
  (comparable across SMs): p0 item start, p1 scoring done, p2 exp-sums
  exchanged, p8 logit threshold, p9 selection, p5 lists built, p3 value rows
  issued, p4 counts exchanged, p10/p11 prefix and diagnostics, p12-p14 the
  P.V passes and the published partials, p15 merged, p6/p7 item end;
* s<k>: SM-clock sub-stamps of thread 0, in microseconds from its item start
  at the nominal 1965 MHz: s0-s6 list building, s10-s14 the P.V, s15-s23 the
  calibration's radix passes (histogram, push, exchange, bin search; pass 0
  then 1), s36-s38 and s27-s30 its selection, ties and trim, s34 its final
  masks, s21/s24-s26 the merge.
The trace costs time of its own (the stamp sites), so its totals run a few
microseconds above the product build's.
"""
from __future__ import annotations

import argparse
import json
import math
import statistics

import torch

from . import ops


def _inputs(B, L, Hq, Hk, Hv, D, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q0 = torch.randn(B, Hq, 1, D, generator=g, device=dev) * 0.5
    q1 = 0.9 * q0 + math.sqrt(1 - 0.81) * 0.5 * torch.randn(B, Hq, 1, D, generator=g, device=dev)
    k = (torch.randn(B, Hk, L, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = torch.empty(B, Hv, L, D, device=dev, dtype=torch.bfloat16)
    for h in range(Hv):
        v[:, h] = (torch.randn(B, L, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    kn = (torch.randn(B, Hk, 1, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    vn = (torch.randn(B, Hv, 1, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q0.to(torch.bfloat16), q1.to(torch.bfloat16), k, v, kn, vn


def main():
    ap = argparse.ArgumentParser()
    for name, default in (("B", 8), ("L", 32768), ("Hq", 12), ("Hk", 1), ("Hv", 2), ("D", 128), ("N", 512)):
        ap.add_argument(f"--{name}", type=int, default=default)
    ap.add_argument("--mode", default="atopn", choices=["atopn", "calibrate", "dense"])
    ap.add_argument("--copies", type=int, default=4, help="rotating caches (more than L2 together)")
    ap.add_argument("--launches", type=int, default=12)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    caches = [_inputs(a.B, a.L, a.Hq, a.Hk, a.Hv, a.D, dev, seed=c) for c in range(a.copies)]
    thrs = []
    for c in caches:
        t = torch.zeros(a.B * a.Hq, dtype=torch.float32, device=dev)
        ops.atopn_calibrate(c[0], c[2], c[3], None, t, a.N)
        thrs.append(t)
    torch.cuda.synchronize()
    res = {}
    nct = 148
    for rep in range(a.launches):
        c = rep % a.copies
        q0, q1, k, v, kn, vn = caches[c]
        diag = {"trace": True}
        if a.mode == "atopn":
            ops.atopn_decode(q1, k, v, None, thrs[c], a.N, k_new=kn, v_new=vn, append_pos=a.L - 1, diag=diag)
        elif a.mode == "dense":
            ops.dense_decode(q1, k, v, None, k_new=kn, v_new=vn, append_pos=a.L - 1, diag=diag)
        else:
            ops.atopn_calibrate(q1, k, v, None, thrs[c], a.N, diag=diag)
        torch.cuda.synchronize()
        if rep < min(4, a.launches - 1):
            continue
        tr = diag["trace"].cpu()
        ent = tr[:nct, 120]
        valid = ent > 0
        if not bool(valid.any()):
            raise SystemExit("no trace stamps: build the library with SAGA_PHASE_TRACE=1")
        t0 = int(ent[valid].min())
        for k in range(16):
            vals = sorted((int(x) - t0) / 1e3 for x in tr[:nct, 64 + k][valid] if int(x) > 0)
            if vals:
                res.setdefault(f"p{k}", []).append(statistics.median(vals))
        col = tr[:nct, 122]
        vals = [(int(x) - t0) / 1e3 for x in col[valid] if int(x) > 0]
        if vals:
            res.setdefault("exit_med", []).append(statistics.median(vals))
            res.setdefault("exit_max", []).append(max(vals))
        base = tr[:nct, 0]
        for k in range(40):
            vals = [(int(x) - int(b)) / 1965.0 for x, b in zip(tr[:nct, 80 + k][valid], base[valid])
                    if int(x) > 0 and int(b) > 0]
            if vals:
                res.setdefault(f"s{k}", []).append(statistics.median(vals))
    out = {k: round(statistics.median(v), 2) for k, v in sorted(res.items(), key=lambda kv: statistics.median(kv[1]))}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
