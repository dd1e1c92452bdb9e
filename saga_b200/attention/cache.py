"""Static KV cache whose decode-token append runs inside the fused kernel.

HF calls `past_key_values.update(k_new, v_new, layer)` before the attention
function. For a static cache this is two `index_copy_` launches per layer
(transformers' StaticLayer.update). SagaStaticLayer instead records the decode
token: its key/value rows and a device tensor with its position. The
saga_b200 attention functions then pass the token to the fused kernel,
which writes the rows into the cache and scores them in the same launch.
Prefill (more than one new position) goes through the normal update.

The position stays on the device (copied from the cache's running length),
so that CUDA-graph replays of the decode step append at the advancing
position. Use this cache only with the saga_b200 attention functions: a
recorded token that no attention call consumes raises on the next update.

Key and value heads may differ (a model whose key projection was merged to
fewer heads, speedup.py:88-116): each cache is sized from the states it first
receives. transformers' StaticLayer sizes the values with the key-head count,
which is why the reference rebuilds the cache tensors by hand
(speedup.py:119-139); this cache needs no such step.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
from transformers.cache_utils import StaticCache, StaticLayer

# keys tensor (data_ptr) -> (k_new, v_new, position tensor) of the pending decode token
_PENDING: Dict[int, Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}


def take_pending(key: torch.Tensor) -> Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """The decode token recorded for this key cache, if any (and forget it)."""
    return _PENDING.pop(key.data_ptr(), None)


class SagaStaticLayer(StaticLayer):
    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        super().lazy_initialization(key_states, value_states)
        hv = value_states.shape[1]
        if self.values.shape[1] != hv:
            self.values = torch.zeros((self.max_batch_size, hv, self.max_cache_len, self.v_head_dim),
                                      dtype=self.dtype, device=self.device)
            if not torch.compiler.is_compiling():
                torch._dynamo.mark_static_address(self.values)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if key_states.shape[-2] != 1:
            return super().update(key_states, value_states, *args, **kwargs)
        if self.keys.data_ptr() in _PENDING:
            raise RuntimeError("the previous decode token of this layer was never appended: "
                               "SagaStaticCache needs the saga_b200 attention functions")
        if getattr(self, "_saga_pos", None) is None:
            self._saga_pos = torch.zeros(1, dtype=torch.int64, device=self.keys.device)
        self._saga_pos.copy_(self.cumulative_length.reshape(1).to(torch.int64))
        self.cumulative_length.add_(1)
        _PENDING[self.keys.data_ptr()] = (key_states, value_states, self._saga_pos)
        return self.keys, self.values


class SagaStaticCache(StaticCache):
    """transformers' StaticCache whose full-attention layers append decode
    tokens in the fused saga_b200 kernel (SagaStaticLayer)."""

    def __init__(self, config, max_cache_len: int, **kwargs):
        super().__init__(config=config, max_cache_len=max_cache_len, **kwargs)
        self.layers = [SagaStaticLayer(max_cache_len=max_cache_len) if type(layer) is StaticLayer else layer
                       for layer in self.layers]
