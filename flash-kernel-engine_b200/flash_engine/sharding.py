"""Spreading the attention hot path over the GPUs of one node (one process per GPU).

The reference is single-GPU and has no distributed code; these are the two ways the
work is partitioned here:

* Head sharding (prefill, paged decode). Rank r owns KV heads
  [r*Hkv/N, (r+1)*Hkv/N) and the query heads that read them; every rank runs the
  ordinary single-GPU operator on its slice. No communication.
* KV-range sharding (long-context decode). Rank r owns the token window
  [r*ceil(M/N), (r+1)*ceil(M/N)) of every sequence, rounded to whole cache blocks:
  the split rule of python/flash_engine/ops.py:112-121 applied across GPUs. Each
  rank computes one (O, m, l) partial per (sequence, query head) over its window,
  the partials are all-gathered (NCCL over NVLink), and every rank combines them
  with the log-sum-exp merge of src/flash_decoding.cu:151-223.

The exchange step (``allgather_merge``) takes the local-partial and merge functions
as arguments, so the same protocol runs with the CUDA kernels on NCCL ranks and
with the CPU oracle on gloo ranks in the tests.

``KVRangeExchange`` is the fused form used on NVLink-connected GPUs: the decode
kernel itself stores each partial row into every rank's exchange buffer (peer
memory mapped through CUDA IPC) and raises a per-rank step flag; a small merge
kernel waits for all flags (bounded) and combines. No NCCL call on the data path.
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist


def head_shard_bounds(num_heads: int, num_kv_heads: int, world: int, rank: int):
    """(kv_lo, kv_hi, q_lo, q_hi) owned by `rank` under KV-head sharding."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads cannot be split over {world} ranks")
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    per = num_kv_heads // world
    g = num_heads // num_kv_heads
    kv_lo, kv_hi = rank * per, (rank + 1) * per
    return kv_lo, kv_hi, kv_lo * g, kv_hi * g


def kv_range_bounds(max_context_len: int, world: int, rank: int, block_size: int = 16):
    """Token window [begin, end) of `rank` under KV-range sharding: split size
    ceil(M / N) (ops.py:112), rounded up to whole blocks so that no cache block is
    shared by two GPUs. The last rank's window ends at max_context_len; a rank whose
    window is empty (few tokens, many ranks) gets (0, 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    per = math.ceil(max(max_context_len, 1) / world)
    per = math.ceil(per / block_size) * block_size
    begin = min(rank * per, max_context_len)
    end = max_context_len if rank == world - 1 else min((rank + 1) * per, max_context_len)
    if end <= begin:
        return 0, 0
    return begin, end


def _gather(t: torch.Tensor, group, world: int) -> torch.Tensor:
    """[world, *t.shape] stack of every rank's tensor."""
    t = t.contiguous()
    out = t.new_empty((world,) + tuple(t.shape))
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t, group=group)
    return out


def allgather_merge(local_out: torch.Tensor, local_stats: torch.Tensor, merge, group=None):
    """All-gather every rank's partial (O [rows, d], stats [rows, 2]) and merge them.

    ``merge(gathered_out [world, rows, d], gathered_stats [world, rows, 2], world)``
    returns the combined output. Every rank performs the same collective steps in the
    same order (one all-gather of O, one of the stats)."""
    world = dist.get_world_size(group)
    go = _gather(local_out, group, world)
    gs = _gather(local_stats, group, world)
    return merge(go, gs, world)


def paged_decode_kv_range(query, key_cache, value_cache, block_tables, context_lens,
                          max_context_len: int, block_size: int = 16, scale=None,
                          group=None, out_dtype: str = "bf16", workspace=None):
    """KV-range-sharded paged decode (bf16 cache) on this rank's GPU.

    ``key_cache`` / ``value_cache`` hold this rank's blocks; ``block_tables`` maps the
    global logical blocks of this rank's window to them (entries outside the window
    are never read). Returns the full [S, H, d] output on every rank."""
    from . import ops

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    tb, te = kv_range_bounds(max_context_len, world, rank, block_size)
    o, st = ops.paged_decode_partials(query, key_cache, value_cache, block_tables,
                                      context_lens, tb, te, block_size, scale, workspace)
    S, H, d = query.shape

    def merge(go, gs, w):
        return ops.merge_partials(go.view(w, S * H, 1, d), gs.view(w, S * H, 1, 2), w, 1,
                                  out_dtype).view(S, H, d)

    return allgather_merge(o.view(S * H, d), st.view(S * H, 2), merge, group)


class KVRangeExchange:
    """Peer-memory exchange buffers of KV-range-sharded decode for one process group
    (one process per GPU, all GPUs of one node, at most 8 ranks).

    Each rank allocates one buffer (``fe_kv_exchange_alloc``), all-gathers the CUDA IPC
    handles over the group and maps the peers' buffers. ``decode`` then runs one step:
    ``ops.paged_decode_kv_exchange`` over this rank's token window. Every rank must call
    ``decode`` the same number of times; ``close`` (collective) releases the buffers.
    """

    def __init__(self, max_rows: int, head_dim: int, group=None):
        from . import _lib

        self._lib = _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the exchange supports at most 8 ranks")
        self.max_rows, self.head_dim = int(max_rows), int(head_dim)
        L = _lib.lib
        nbytes = int(L.fe_kv_exchange_bytes(self.world, self.max_rows, self.head_dim))
        if nbytes == 0:
            raise ValueError("bad exchange shape")
        own = ctypes.c_void_p()
        _lib.check(L.fe_kv_exchange_alloc(nbytes, ctypes.byref(own)), "fe_kv_exchange_alloc")
        self._own = own.value
        handle = (ctypes.c_ubyte * 64)()
        _lib.check(L.fe_kv_exchange_ipc_handle(self._own, handle), "fe_kv_exchange_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        self.ptrs = []
        for r in range(self.world):
            if r == self.rank:
                self.ptrs.append(self._own)
                continue
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r])
            p = ctypes.c_void_p()
            _lib.check(L.fe_kv_exchange_ipc_open(hb, ctypes.byref(p)), "fe_kv_exchange_ipc_open")
            self._opened.append(p.value)
            self.ptrs.append(p.value)
        dist.barrier(group=group)

    def decode(self, query, key_cache, value_cache, block_tables, context_lens,
               max_context_len: int, block_size: int = 16, scale=None, workspace=None,
               out=None):
        """One KV-range-sharded decode step; returns the full [S, H, d] bf16 output."""
        from . import ops

        tb, te = kv_range_bounds(max_context_len, self.world, self.rank, block_size)
        return ops.paged_decode_kv_exchange(query, key_cache, value_cache, block_tables,
                                            context_lens, tb, te, self.ptrs, self.rank,
                                            self.max_rows, block_size, scale, workspace, out)

    def prepare(self, query, key_cache, value_cache, block_tables, context_lens,
                max_context_len: int, block_size: int = 16, scale=None, workspace=None,
                out=None):
        """``decode`` with its arguments checked and converted once: returns a function
        of no arguments that runs one step (on the stream current at this call) into
        ``out`` and returns it. Every rank must call the returned function the same number
        of times, interleaved with its ``decode`` calls in the same order."""
        from . import ops

        tb, te = kv_range_bounds(max_context_len, self.world, self.rank, block_size)
        return ops.paged_decode_kv_exchange_prepared(query, key_cache, value_cache,
                                                     block_tables, context_lens, tb, te,
                                                     self.ptrs, self.rank, self.max_rows,
                                                     block_size, scale, workspace, out)

    def close(self):
        """Collective: unmap the peers' buffers and free this rank's own."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        L = self._lib.lib
        for p in self._opened:
            L.fe_kv_exchange_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        L.fe_kv_exchange_free(self._own)
        self._own = None
