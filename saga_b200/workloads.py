"""Seeded synthetic decode workloads (no datasets, no checkpoints).

The shapes follow the single-layer decode configurations this library is
benchmarked on: a query ``q[B, Hq, 1, D]``, a key cache ``k[B, Hk, L, D]`` with
few key heads and a value cache ``v[B, Hv, L, D]`` with more value heads.

Values are drawn with numpy's PCG64 generator. This keeps every input the same
bit for bit on any host with the same numpy, so golden fixtures can store a
seed instead of tensors. ``plant`` high-score keys per (batch, key head) get
``k += gain * q_hat``. Here ``q_hat`` is the unit vector of the first query
head of that key group, so attention on that head is peaked, as in the
reference's latency setup.
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict
from typing import Optional

import numpy as np


@dataclass(frozen=True)
class DecodeShape:
    B: int
    L: int
    Hq: int
    Hk: int
    Hv: int
    D: int
    N: int                      # top_n_attention
    dtype: str = "bf16"         # "bf16" | "fp16" | "fp32"
    scale: float = 1.0          # std of q, k, v
    plant: int = 16             # planted keys per (batch, key head)
    gain: float = 4.0

    def check(self) -> None:
        if self.Hq % self.Hk or self.Hq % self.Hv:
            raise ValueError("Hq must be a multiple of Hk and of Hv")

    @property
    def rows(self) -> int:
        return self.B * self.Hq

    def as_dict(self) -> dict:
        return asdict(self)


# The single-layer configurations of the benchmark plan.
CONFIG1 = DecodeShape(B=1, L=4096, Hq=15, Hk=1, Hv=5, D=64, N=128, dtype="fp32",
                      scale=1.0, plant=16, gain=4.0)
CONFIG2 = DecodeShape(B=8, L=32768, Hq=12, Hk=1, Hv=2, D=128, N=512, dtype="bf16",
                      scale=0.5, plant=64, gain=4.0)
CONFIG4 = DecodeShape(B=1, L=131072, Hq=12, Hk=1, Hv=2, D=128, N=1024, dtype="bf16",
                      scale=0.5, plant=256, gain=4.0)
# One attention layer of the two model-shaped configurations.
CONFIG3_LAYER = DecodeShape(B=16, L=16384 + 128, Hq=15, Hk=1, Hv=5, D=64, N=256,
                            dtype="bf16", scale=0.5, plant=64, gain=4.0)
CONFIG5_LAYER = DecodeShape(B=64, L=65536 + 64, Hq=12, Hk=1, Hv=4, D=128, N=512,
                            dtype="bf16", scale=0.5, plant=128, gain=4.0)


def bf16_round_np(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000))
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def fp16_round_np(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(dtype: str, x: np.ndarray) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round_np(x)
    if dtype == "fp16":
        return fp16_round_np(x)
    return np.asarray(x, dtype=np.float32)


@dataclass
class DecodeInputs:
    shape: DecodeShape
    q0: np.ndarray              # [B, Hq, 1, D] float32 holding dtype-representable values
    q1: np.ndarray              # next-step query, correlated with q0
    k: np.ndarray               # [B, Hk, L, D]
    v: np.ndarray               # [B, Hv, L, D]
    k_new: np.ndarray           # [B, Hk, 1, D] token appended at `append_pos`
    v_new: np.ndarray           # [B, Hv, 1, D]
    planted: np.ndarray         # [B, Hk, plant] planted positions
    extra: dict = field(default_factory=dict)


def make_inputs(shape: DecodeShape, seed: int = 0, rho: float = 0.9) -> DecodeInputs:
    """Build the seeded inputs of one decode step.

    ``q1 = rho * q0 + sqrt(1 - rho^2) * noise`` stands in for the next decode
    step's query. All arrays are float32, already rounded to ``shape.dtype``.
    """
    shape.check()
    B, L, Hq, Hk, Hv, D = shape.B, shape.L, shape.Hq, shape.Hk, shape.Hv, shape.D
    G = Hq // Hk
    rng = np.random.Generator(np.random.PCG64(seed))
    s = np.float32(shape.scale)
    q0 = rng.standard_normal((B, Hq, 1, D), dtype=np.float32) * s
    k = rng.standard_normal((B, Hk, L, D), dtype=np.float32)
    k *= s
    v = rng.standard_normal((B, Hv, L, D), dtype=np.float32)
    v *= s
    nplant = min(shape.plant, L)
    planted = np.zeros((B, Hk, nplant), dtype=np.int64)
    for b in range(B):
        for kk in range(Hk):
            pos = rng.permutation(L)[:nplant]
            planted[b, kk] = np.sort(pos)
            qh = q0[b, kk * G, 0].astype(np.float64)
            qhat = (qh / np.linalg.norm(qh)).astype(np.float32)
            k[b, kk, pos] += np.float32(shape.gain) * qhat
    noise = rng.standard_normal((B, Hq, 1, D), dtype=np.float32) * s
    q1 = np.float32(rho) * q0 + np.float32(np.sqrt(1.0 - rho * rho)) * noise
    k_new = rng.standard_normal((B, Hk, 1, D), dtype=np.float32) * s
    v_new = rng.standard_normal((B, Hv, 1, D), dtype=np.float32) * s
    dt = shape.dtype
    return DecodeInputs(shape=shape, q0=round_to(dt, q0), q1=round_to(dt, q1),
                        k=round_to(dt, k), v=round_to(dt, v),
                        k_new=round_to(dt, k_new), v_new=round_to(dt, v_new),
                        planted=planted)


def bool_decode_mask(B: int, L: int, filled: int) -> np.ndarray:
    """The [B, 1, 1, L] boolean decode mask of a static cache: True on the
    ``filled`` valid slots, False on the unfilled tail."""
    m = np.zeros((B, 1, 1, L), dtype=bool)
    m[..., :filled] = True
    return m


def input_digest(inp: DecodeInputs) -> str:
    """A short content hash of the generated inputs, stored in fixtures so a
    test can tell a generator change from a kernel change."""
    import hashlib
    h = hashlib.sha256()
    for a in (inp.q0, inp.q1, inp.k, inp.v, inp.k_new, inp.v_new):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def to_torch(a: np.ndarray, dtype: str, device=None):
    """float32 array -> torch tensor of ``dtype`` (exact: values are representable)."""
    import torch
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    if device is not None:
        t = t.to(device)
    return t.to(tdt)
