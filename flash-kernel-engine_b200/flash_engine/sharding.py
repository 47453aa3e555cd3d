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
"""

from __future__ import annotations

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
    shared by two GPUs. The last rank's window ends at max_context_len."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    per = math.ceil(max(max_context_len, 1) / world)
    per = math.ceil(per / block_size) * block_size
    begin = min(rank * per, max_context_len)
    end = max_context_len if rank == world - 1 else min((rank + 1) * per, max_context_len)
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
