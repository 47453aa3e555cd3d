"""KV-head and KV-range sharding protocols on CPU ranks (gloo, world size 2 and 3),
with the oracle computing each rank's share: the exchange and merge code paths of
flash_engine.sharding without a GPU."""
import ast
import os
import socket
import time

import pytest
import torch.multiprocessing as mp

import dist_workers
from flash_engine import sharding


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world, tmp_path, join_timeout=120):
    path = str(tmp_path / "res")
    ctx = mp.start_processes(fn, args=(world, _port(), path), nprocs=world, join=False,
                             start_method="spawn")
    deadline = time.time() + join_timeout
    while not ctx.join(timeout=1) and time.time() < deadline:
        pass  # join() returns after each process exit; wait for all of them
    for proc in ctx.processes:
        if proc.is_alive():  # give up on a stuck rank: kill exactly the processes we started
            proc.kill()
    out = []
    for r in range(world):
        fp = f"{path}.{r}"
        out.append(ast.literal_eval(open(fp).read()) if os.path.exists(fp) else None)
    return out


def test_bounds():
    assert sharding.kv_range_bounds(131072, 8, 0) == (0, 16384)
    assert sharding.kv_range_bounds(131072, 8, 7) == (114688, 131072)
    # rounding to blocks: 100 tokens over 3 ranks -> 48-token (3-block) windows
    assert [sharding.kv_range_bounds(100, 3, r) for r in range(3)] == [(0, 48), (48, 96),
                                                                       (96, 100)]
    # more ranks than blocks: the ranks past the end get an empty window
    assert [sharding.kv_range_bounds(20, 8, r) for r in range(4)] == [(0, 16), (16, 20), (0, 0),
                                                                      (0, 0)]
    assert sharding.head_shard_bounds(32, 8, 4, 3) == (6, 8, 24, 32)
    with pytest.raises(ValueError):
        sharding.head_shard_bounds(32, 8, 3, 0)


@pytest.mark.parametrize("world", [2, 3])
def test_kv_range_allgather_merge_gloo(tmp_path, world):
    res = _run(dist_workers.kv_range_worker, world, tmp_path)
    assert all(r is not None for r in res), res
    assert res[0][0] == 0 and res[-1][1] == 1017
    for tb, te, err in res:
        assert err < 1e-5


def test_head_shard_gloo(tmp_path):
    res = _run(dist_workers.head_shard_worker, 2, tmp_path)
    assert all(r is not None for r in res), res
    assert [r[:2] for r in res] == [(0, 8), (8, 16)]
    assert all(r[2] < 1e-6 for r in res)


def test_rank_dropout_ends_in_error_not_hang(tmp_path):
    res = _run(dist_workers.dropout_worker, 2, tmp_path, join_timeout=60)
    assert res[0] is not None, "rank 0 did not finish"
    status, seconds = res[0]
    assert status != "no-error"
    assert seconds < 30
