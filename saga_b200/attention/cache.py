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
from transformers.cache_utils import Cache, CacheLayerMixin, StaticCache, StaticLayer

# keys tensor (data_ptr) -> (k_new, v_new, position: device tensor or int) of the pending decode token
_PENDING: Dict[int, tuple] = {}


def take_pending(key: torch.Tensor) -> Optional[tuple]:
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
        if key_states.shape[-2] != 1 or torch.compiler.is_compiling():
            # prefill; and decode under torch.compile, where the token is
            # copied in the graph (the pending-token registry is eager-only)
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


# ---------------------------------------------------------------------------
# Paged cache
# ---------------------------------------------------------------------------

# keys pool (data_ptr) -> (keys pool, values pool, page table, logical length)
# of the pending decode step
_PAGED: Dict[int, tuple] = {}


def take_paged(key: torch.Tensor) -> Optional[tuple]:
    """(keys pool, values pool, page table, logical length) recorded for the
    decode step whose key view is `key`, if any."""
    return _PAGED.pop(key.data_ptr(), None)


class SagaPagedLayer(CacheLayerMixin):
    """One layer's keys and values in page pools [pages, H, page_len, D]
    (key and value head counts taken from the states), a device page table
    [batch, pages per sequence] and host-side page reference counts.

    Sequences of a batch advance together. Pages can be shared between
    sequences (``batch_repeat_interleave``, which transformers' ``generate``
    calls to expand a batch, shares them instead of copying the tensors); a
    sequence gets its own copy of a shared page before its first append
    there. Decode tokens are appended by the fused kernel.

    A decode step returns zero-stride views [B, H, length, D] of the pools:
    callers that cut the mask to ``key.shape[-2]`` (speedup.py:47,
    lm_eval_saga.py:171) see the logical length, and the attention functions
    find the pools and the page table from the view's address.
    """

    is_compileable = False
    is_sliding = False

    def __init__(self, max_cache_len: int, page_len: int = 128, num_pages: Optional[int] = None):
        super().__init__()
        if page_len < 128 or page_len & (page_len - 1):
            raise ValueError("page_len must be a power of two and at least 128")
        self.max_cache_len = max_cache_len
        self.page_len = page_len
        self.max_pages = (max_cache_len + page_len - 1) // page_len
        self.num_pages = num_pages
        self.length = 0

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        self.batch = key_states.shape[0]
        if self.num_pages is None:
            self.num_pages = self.batch * self.max_pages
        kshape = (self.num_pages, key_states.shape[1], self.page_len, key_states.shape[-1])
        vshape = (self.num_pages, value_states.shape[1], self.page_len, value_states.shape[-1])
        self.keys = torch.zeros(kshape, dtype=self.dtype, device=self.device)
        self.values = torch.zeros(vshape, dtype=self.dtype, device=self.device)
        self.table_host = [[-1] * self.max_pages for _ in range(self.batch)]
        self.page_table = torch.zeros((self.batch, self.max_pages), dtype=torch.int32, device=self.device)
        self.refs = [0] * self.num_pages
        self.free = list(range(self.num_pages - 1, -1, -1))
        self.is_initialized = True

    # -- page bookkeeping (host) -------------------------------------------------
    def _alloc(self) -> int:
        if not self.free:
            raise RuntimeError("SagaPagedCache is out of pages; pass a larger num_pages")
        pg = self.free.pop()
        self.refs[pg] = 1
        return pg

    def _release(self, pg: int) -> None:
        self.refs[pg] -= 1
        if self.refs[pg] == 0:
            self.free.append(pg)

    def _sync_table(self) -> None:
        self.page_table = torch.tensor(self.table_host, dtype=torch.int32, device=self.device)

    def _own_page(self, b: int, idx: int) -> bool:
        """Make page idx of sequence b present and private; True if the
        table changed."""
        pg = self.table_host[b][idx]
        if pg >= 0 and self.refs[pg] == 1:
            return False
        new = self._alloc()
        if pg >= 0:  # copy on write of a shared page
            self.keys[new].copy_(self.keys[pg])
            self.values[new].copy_(self.values[pg])
            self._release(pg)
        self.table_host[b][idx] = new
        return True

    def _write(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        """Prompt rows [length, length + n) of every sequence into pages."""
        n = key_states.shape[-2]
        start, end = self.length, self.length + n
        if end > self.max_pages * self.page_len:
            raise RuntimeError("SagaPagedCache is full (max_cache_len)")
        changed = False
        for b in range(self.batch):
            for idx in range(start // self.page_len, (end - 1) // self.page_len + 1):
                changed |= self._own_page(b, idx)
        if changed:
            self._sync_table()
        if start % self.page_len == 0:  # whole pages from the start: one scatter per tensor
            npg = (n + self.page_len - 1) // self.page_len
            ids = self.page_table[:, start // self.page_len:start // self.page_len + npg].reshape(-1).long()
            for pool, st in ((self.keys, key_states), (self.values, value_states)):
                pad = npg * self.page_len - n
                x = torch.nn.functional.pad(st, (0, 0, 0, pad)) if pad else st
                B, H, _, D = x.shape
                x = x.reshape(B, H, npg, self.page_len, D).transpose(1, 2).reshape(B * npg, H, self.page_len, D)
                pool.index_copy_(0, ids, x.to(pool.dtype))
        else:
            for b in range(self.batch):
                for pos in range(start, end):
                    pg, r = self.table_host[b][pos // self.page_len], pos % self.page_len
                    self.keys[pg, :, r] = key_states[b, :, pos - start]
                    self.values[pg, :, r] = value_states[b, :, pos - start]

    def _contiguous(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """The cached rows as [B, H, length, D] tensors (prefill after decode)."""
        npg = (self.length + self.page_len - 1) // self.page_len
        ids = self.page_table[:, :npg].long()
        out = []
        for pool in (self.keys, self.values):
            x = pool[ids]  # [B, npg, H, page_len, D]
            B, _, H, _, D = x.shape
            out.append(x.transpose(1, 2).reshape(B, H, npg * self.page_len, D)[:, :, :self.length])
        return out[0], out[1]

    # -- transformers' layer interface -------------------------------------------
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        n = key_states.shape[-2]
        if n != 1:  # prefill: rows into pages; attention reads contiguous states
            was_empty = self.length == 0
            self._write(key_states, value_states)
            self.length += n
            if was_empty:
                return key_states, value_states
            return self._contiguous()
        if self.keys.data_ptr() in _PENDING:
            raise RuntimeError("the previous decode token of this layer was never appended: "
                               "SagaPagedCache needs the saga_b200 attention functions")
        if self.length >= self.max_pages * self.page_len:
            raise RuntimeError("SagaPagedCache is full (max_cache_len)")
        idx = self.length // self.page_len
        changed = False
        for b in range(self.batch):
            changed |= self._own_page(b, idx)
        if changed:
            self._sync_table()
        pos = self.length
        self.length += 1
        _PENDING[self.keys.data_ptr()] = (key_states, value_states, pos)
        _PAGED[self.keys.data_ptr()] = (self.keys, self.values, self.page_table, self.length)
        kv = self.keys[:1, :, :1].expand(self.batch, self.keys.shape[1], self.length, self.keys.shape[3])
        vv = self.values[:1, :, :1].expand(self.batch, self.values.shape[1], self.length, self.values.shape[3])
        return kv, vv

    def get_mask_sizes(self, query_length: int) -> tuple:
        return self.length + query_length, 0

    def get_seq_length(self) -> int:
        return self.length

    def get_max_cache_shape(self) -> int:
        return self.max_cache_len

    def batch_repeat_interleave(self, repeats: int) -> None:
        """Each sequence becomes `repeats` sequences sharing its pages."""
        if not self.is_initialized:
            return
        rows = []
        for row in self.table_host:
            for _ in range(repeats):
                rows.append(list(row))
                for pg in row:
                    if pg >= 0:
                        self.refs[pg] += 1
            for pg in row:
                if pg >= 0:
                    self._release(pg)
        self.table_host = rows
        self.batch = len(rows)
        self._sync_table()

    def reset(self) -> None:
        if self.is_initialized:
            self.table_host = [[-1] * self.max_pages for _ in range(self.batch)]
            self.refs = [0] * self.num_pages
            self.free = list(range(self.num_pages - 1, -1, -1))
            self._sync_table()
        self.length = 0


class SagaPagedCache(Cache):
    """transformers cache whose layers keep keys and values in page pools
    (SagaPagedLayer) and append decode tokens in the fused saga_b200 kernel.
    Use it with the saga_b200 attention functions. page_len: a power of two,
    at least 128; num_pages: pages per layer pool (default: enough for every
    sequence without sharing)."""

    def __init__(self, config, max_cache_len: int, page_len: int = 128, num_pages: Optional[int] = None):
        cfg = config.get_text_config(decoder=True) if hasattr(config, "get_text_config") else config
        layers = [SagaPagedLayer(max_cache_len, page_len, num_pages) for _ in range(cfg.num_hidden_layers)]
        super().__init__(layers=layers)
