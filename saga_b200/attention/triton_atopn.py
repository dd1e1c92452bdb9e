"""Drop-in replacement of the reference's ``attention/triton_atopn.py``.

The module keeps its name and its two public names, because
``speedup.py:427-428`` does ``from attention.triton_atopn import _BUFFER_CACHE``
and ``.clear()``s it. The selection kernel is the CUDA ``select_kernel`` of
``libsaga_b200.so``; Triton is not imported.

Behaviour follows triton_atopn.py:59-113. Output buffers are cached per
(rows, k, device, dtype) and reused across calls, so that a captured CUDA
graph keeps its addresses; slots are filled with -inf / 0 before selection.
One difference is deliberate: passing positions are written in ascending
order, and when more than k pass, the k lowest positions are kept. The
reference's order and its kept subset depend on atomics.
"""
import torch

from saga_b200 import ops as _ops

_BUFFER_CACHE = {}


def threshold_topk_fast(
    x: torch.Tensor,
    k: int,
    threshold: torch.Tensor,
    block_size: int = 1024,
) -> tuple:
    """Select, per row of ``x[..., D]``, every element > threshold (strict).

    ``threshold`` may hold one value per row, a single value, or a shorter
    vector repeated over the rows (triton_atopn.py:86-96). Returns
    ``(values[..., k], indices[..., k])`` with -inf / 0 in unused slots.
    ``block_size`` is accepted for signature compatibility.
    """
    original_shape = x.shape
    D = original_shape[-1]
    x_flat = x.reshape(-1, D)
    N = x_flat.shape[0]
    cache_key = (N, k, x.device, x.dtype)
    if cache_key not in _BUFFER_CACHE:
        _BUFFER_CACHE[cache_key] = (
            torch.empty(N, k, device=x.device, dtype=x.dtype),
            torch.empty(N, k, device=x.device, dtype=torch.int64),
            torch.empty(N, device=x.device, dtype=torch.int32),
        )
    out_values, out_indices, counts = _BUFFER_CACHE[cache_key]
    # Row r uses threshold[r % numel]: per-row (numel == N), scalar (numel == 1)
    # and the reference's repeat-to-N-rows rule (triton_atopn.py:94-96) alike.
    thr = threshold.reshape(-1)[:N] if threshold.numel() > N else threshold.reshape(-1)
    _ops.threshold_select(x_flat, k, thr, out_values, out_indices, counts)
    new_shape = original_shape[:-1] + (k,)
    return out_values.reshape(new_shape), out_indices.reshape(new_shape)
