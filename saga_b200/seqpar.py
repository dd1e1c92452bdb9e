"""Sequence-sharded Atop-N decode: one sequence's positions over several devices.

Config 4 of the reference's benchmarks: batch 1, context 131072, sharded over
1/2/4/8 B200s, one process per device. Shard r owns global positions
[r * Ls, (r + 1) * Ls), Ls = L / P. Every shard but the last also keeps a
replica of the sequence's last 256 key rows, for the tail max of
attention.py:142-143.

Each decode step is one launch of the fused kernel on every device. Its
exchanges run between the devices through peer-mapped workspaces (NVLink):
* the exp-sums and counts, in chunk order;
* the global K = min(2N, L) cap;
* the partial outputs, merged by log-sum-exp;
* the completion ticket.
The calibration step (attention.py:173-189) is sharded the same way: every
device adds its chunks' 256-bin logit-key histograms into shard 0's (system-
scope atomics over NVLink), the chunks meet at system-scope barriers on shard
0's counters, and every device reads all chunks' maxima, exp-sums and counts
from the peers' workspaces; so every shard computes the exact global N-th
largest probability, the threshold of the whole row.
No collective library is on the data path; torch.distributed only exchanges
the workspaces' IPC handles once, at set-up. Every shard ends with the full
output.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as Lib
from . import ops

TAIL = 256  # attention.py:136, tail_size of the max estimate


@dataclass(frozen=True)
class ShardLayout:
    """Where shard `rank` of `shards` keeps its part of an L-position sequence."""
    L: int          # global context length
    shards: int
    rank: int
    own: int        # positions this shard owns (Ls)
    offset: int     # global position of its first own position
    local_len: int  # rows of its cache: own positions (+ the tail replica)

    @property
    def replica(self) -> bool:
        return self.local_len > self.own

    def local_position(self, global_pos: int) -> int:
        """Local row of a global position this shard holds, or -1."""
        if self.offset <= global_pos < self.offset + self.own:
            return global_pos - self.offset
        if self.replica and global_pos >= self.L - TAIL:
            return self.own + (global_pos - (self.L - TAIL))
        return -1


def shard_layout(L: int, shards: int, rank: int) -> ShardLayout:
    if shards < 1 or not 0 <= rank < shards:
        raise ValueError("need 0 <= rank < shards")
    if L % shards:
        raise ValueError(f"context {L} must split evenly over {shards} shards")
    own = L // shards
    if shards > 1 and own < TAIL:
        raise ValueError(f"each shard needs at least {TAIL} positions")
    last = rank == shards - 1
    return ShardLayout(L=L, shards=shards, rank=rank, own=own, offset=rank * own,
                       local_len=own if (last or shards == 1) else own + TAIL)


def shard_cache(cache: torch.Tensor, lay: ShardLayout) -> torch.Tensor:
    """This shard's rows of a [B, H, L, D] cache: its own positions, then the
    tail replica when it is not the last shard (a new contiguous tensor)."""
    own = cache[:, :, lay.offset:lay.offset + lay.own]
    if not lay.replica:
        # a copy even when the slice is already contiguous (B = H = 1): an
        # append into the shard must not write through to `cache`
        return own.clone(memory_format=torch.contiguous_format)
    return torch.cat([own, cache[:, :, lay.L - TAIL:]], dim=2).contiguous()


class ShardedDecode:
    """Per-process handle of a sequence-sharded decode group.

    Construct it on every rank of `group` with the same shapes. Only this
    device's memory is passed in; the peers' workspaces are mapped once here.
    """

    def __init__(self, group, device, B: int, L: int, Hq: int, Hk: int, Hv: int, D: int,
                 dtype=torch.bfloat16, op: str = "atopn"):
        import torch.distributed as dist
        self.group = group
        self.shards = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.lay = shard_layout(L, self.shards, self.rank)
        self.shape = (B, Hq, Hk, Hv, D)
        self.dtype = dtype
        self.op = {"atopn": Lib.SAGA_OP_ATOPN_DECODE, "dense": Lib.SAGA_OP_DENSE_DECODE,
                   "calibrate": Lib.SAGA_OP_ATOPN_CALIBRATE}[op]
        probe = self._probe_args()
        nbytes = Lib.lib.saga_workspace_bytes(ctypes.byref(probe), self.op)
        if nbytes == 0:
            raise Lib.SagaError(Lib.SAGA_ERR_INVALID, "saga_workspace_bytes")
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)
        # Map every shard's workspace into THIS device (CUDA IPC with peer
        # access), through the library: the handle of the allocation that
        # holds the workspace, the workspace's offset in it, and an open on
        # the current device.
        hbuf = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t()
        Lib.check(Lib.lib.saga_ipc_handle(ctypes.c_void_p(self.workspace.data_ptr()), hbuf, ctypes.byref(off)),
                  "saga_ipc_handle")
        mine = (hbuf.raw, int(off.value))
        handles = [None] * self.shards
        dist.all_gather_object(handles, mine, group=group)
        self._opened = []
        self.peer_ptrs = []
        for s, (h, off) in enumerate(handles):
            if s == self.rank:
                self.peer_ptrs.append(self.workspace.data_ptr())
                continue
            base = ctypes.c_void_p()
            Lib.check(Lib.lib.saga_ipc_open(ctypes.c_char_p(h), ctypes.byref(base)), "saga_ipc_open")
            self._opened.append(base.value)
            self.peer_ptrs.append(base.value + off)
        dist.barrier(group=group)

    def close(self):
        """Unmap the peers' workspaces (every rank, before any rank frees its own)."""
        for ptr in self._opened:
            Lib.lib.saga_ipc_close(ctypes.c_void_p(ptr))
        self._opened = []

    def _probe_args(self):
        """Shapes-only arguments of this shard, for saga_workspace_bytes."""
        B, Hq, Hk, Hv, D = self.shape
        a = Lib.SagaAttnArgs()
        a.dtype = ops._DT[self.dtype]
        a.B, a.Hq, a.Hk, a.Hv, a.D, a.L = B, Hq, Hk, Hv, D, self.lay.local_len
        ll = self.lay.local_len
        a.q_sb, a.q_sh = Hq * D, D
        a.k_sb, a.k_sh, a.k_sl = Hk * ll * D, ll * D, D
        a.v_sb, a.v_sh, a.v_sl = Hv * ll * D, ll * D, D
        a.scaling = D ** -0.5
        a.nsel = self.lay.own
        a.pos_offset = self.lay.offset
        a.shards = self.shards
        a.shard = self.rank
        a.top_n = 1
        return a

    def __call__(self, q, k_local, v_local, threshold=None, top_n: int = 256, scaling=None,
                 k_new=None, v_new=None, append_pos: int = -1, diag=None):
        """One decode step on this shard. k_local / v_local: [B, H, local_len, D]
        from shard_cache(). append_pos is global. Returns the full [B, Hq, 1, D].
        For the amortized op `threshold` holds the rows' softmax-space
        thresholds; for the calibration op it receives them (every shard
        writes its own copy of the whole row set). With `diag`, this shard
        writes the kept positions of its own chunks (global positions) at their
        global ranks; the other ranks' slots stay -1."""
        a = ops._attn_args(q, k_local, v_local, None, scaling)
        a.nsel = self.lay.own
        a.pos_offset = self.lay.offset
        a.shards = self.shards
        a.shard = self.rank
        for s, ptr in enumerate(self.peer_ptrs):
            a.shard_workspaces[s] = ptr
        if self.op == Lib.SAGA_OP_ATOPN_DECODE:
            a.top_n = top_n
            a.thr_in = threshold.data_ptr()
        elif self.op == Lib.SAGA_OP_ATOPN_CALIBRATE:
            a.top_n = top_n
            a.thr_out = threshold.data_ptr()
        if k_new is not None:
            lp = self.lay.local_position(append_pos)
            if lp < 0:
                raise ValueError("the appended position is neither owned nor in the tail replica")
            ops._set_append(a, k_new, v_new, lp)
        out = ops._out_like(q)
        a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
        a.workspace, a.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()
        a.status = ops.status_tensor(self.device).data_ptr()
        if diag is not None:
            kk = top_n if self.op == Lib.SAGA_OP_ATOPN_CALIBRATE else 2 * top_n
            ops._diag_buffers(a, q, min(kk, self.lay.L), diag)
        fn = {Lib.SAGA_OP_ATOPN_DECODE: "saga_atopn_decode", Lib.SAGA_OP_DENSE_DECODE: "saga_dense_decode",
              Lib.SAGA_OP_ATOPN_CALIBRATE: "saga_atopn_calibrate"}[self.op]
        Lib.check(getattr(Lib.lib, fn)(ctypes.byref(a), ctypes.c_void_p(ops._stream(q.device))), fn)
        return out
