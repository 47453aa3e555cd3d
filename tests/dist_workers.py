"""Worker bodies for the multi-process (gloo, CPU) tests of flash_engine.sharding.
Run by torch.multiprocessing with the spawn start method."""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for p in (ROOT, os.path.join(ROOT, "flash-kernel-engine_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _init(rank, world, port, timeout_s=60):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _problem():
    from oracle import attention_oracle as O
    lens = [0, 7, 64, 250, 1000, 1017]
    return O.make_paged_problem(12, len(lens), 16, 4, 64, lens, bf16=False)


def kv_range_worker(rank, world, port, result_path):
    import torch
    from flash_engine import sharding
    from oracle import attention_oracle as O
    dist = _init(rank, world, port)
    p = _problem()
    M = int(max(p["context_lens"]))
    tb, te = sharding.kv_range_bounds(M, world, rank, 16)
    o, m, l = O.kv_range_partials(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                  p["context_lens"], tb, te)
    S, H, d = p["q"].shape
    lo = torch.from_numpy(o.reshape(S * H, d))
    ls = torch.from_numpy(np.stack([m.reshape(-1), l.reshape(-1)], 1))

    def merge(go, gs, w):
        outs = [go[i].numpy() for i in range(w)]
        ms = [gs[i, :, 0].numpy() for i in range(w)]
        ls_ = [gs[i, :, 1].numpy() for i in range(w)]
        return O.lse_merge(outs, ms, ls_).reshape(S, H, d)

    out = sharding.allgather_merge(lo, ls, merge)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    err = float(np.abs(out - ref).max())
    dist.barrier()
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr((tb, te, err)))


def head_shard_worker(rank, world, port, result_path):
    import torch
    from flash_engine import sharding
    from oracle import attention_oracle as O
    dist = _init(rank, world, port)
    p = _problem()
    S, H, d = p["q"].shape
    Hkv = p["k_cache"].shape[1]
    kv_lo, kv_hi, q_lo, q_hi = sharding.head_shard_bounds(H, Hkv, world, rank)
    part = O.paged_attention_gqa(p["q"][:, q_lo:q_hi], p["k_cache"][:, kv_lo:kv_hi],
                                 p["v_cache"][:, kv_lo:kv_hi], p["block_tables"],
                                 p["context_lens"])
    t = torch.from_numpy(np.ascontiguousarray(part))
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    full = torch.cat(parts, dim=1).numpy()
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    err = float(np.abs(full - ref).max())
    dist.barrier()
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr((q_lo, q_hi, err)))


def dropout_worker(rank, world, port, result_path):
    """Rank 1 leaves before the exchange (between steps); rank 0 must get an error
    from its collective within the short process-group timeout, not hang."""
    import time

    import torch
    from flash_engine import sharding
    dist = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(0)  # leaves without joining the all-gather
    t0 = time.time()
    status = "no-error"
    try:
        sharding.allgather_merge(torch.zeros(4, 8), torch.zeros(4, 2),
                                 lambda go, gs, w: go.sum(0))
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        status = type(e).__name__
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr((status, time.time() - t0)))
    os._exit(0)


def nccl_kv_range_worker(rank, world, port, result_path):
    """KV-range-sharded paged decode on `world` GPUs over NCCL (each rank holds the
    blocks of its own window), checked against the oracle's single-pass result."""
    import torch
    import torch.distributed as dist
    import flash_engine
    from flash_engine import sharding
    from oracle import attention_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    lens = [0, 5, 16, 300, 1500, 2047]
    p = O.make_paged_problem(21, len(lens), 32, 8, 128, lens)
    M = int(max(lens))
    dev = torch.device("cuda", rank)
    q, kc, vc = (torch.from_numpy(p[x]).to(dev).to(torch.bfloat16)
                 for x in ("q", "k_cache", "v_cache"))
    bt = torch.from_numpy(p["block_tables"]).to(dev)
    cl = torch.from_numpy(p["context_lens"]).to(dev)
    out = sharding.paged_decode_kv_range(q, kc, vc, bt, cl, M, 16)
    errs = flash_engine.device_errors()
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    err = float(np.abs(out.float().cpu().numpy() - ref).max())
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr((err, errs)))


def nccl_graph_worker(rank, world, port, result_path):
    """The KV-range-sharded decode step, NCCL all-gather included, captured once in
    a CUDA graph and replayed on new query tokens."""
    import torch
    import torch.distributed as dist
    from flash_engine import graph, sharding
    from oracle import attention_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    lens = [9, 300, 1024, 2000]
    p = O.make_paged_problem(51, len(lens), 32, 8, 128, lens)
    dev = torch.device("cuda", rank)
    q, kc, vc = (torch.from_numpy(p[x]).to(dev).to(torch.bfloat16)
                 for x in ("q", "k_cache", "v_cache"))
    bt = torch.from_numpy(p["block_tables"]).to(dev)
    cl = torch.from_numpy(p["context_lens"]).to(dev)
    g = graph.DecodeGraph(lambda: sharding.paged_decode_kv_range(q, kc, vc, bt, cl, 2000, 16))
    errs = []
    for seed in (52, 53):
        q2 = O.make_paged_problem(seed, len(lens), 32, 8, 128, lens)["q"]
        q.copy_(torch.from_numpy(q2).to(dev).to(torch.bfloat16))
        out = g.replay()
        torch.cuda.synchronize()
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        errs.append(float(np.abs(out.float().cpu().numpy() - ref).max()))
    del g
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr(max(errs)))


def p2p_exchange_worker(rank, world, port, result_path):
    """KV-range decode with the all-gather done by the decode kernel over peer memory
    (KVRangeExchange): three eager steps on new query tokens, two replays of the step
    captured in a CUDA graph, then two prepared steps, each checked against the oracle."""
    import torch
    import torch.distributed as dist
    import flash_engine
    from flash_engine import graph, sharding
    from oracle import attention_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    lens = [0, 5, 16, 300, 1500, 2047]
    S, H, Hkv, d = len(lens), 32, 8, 128
    p = O.make_paged_problem(61, S, H, Hkv, d, lens)
    M = int(max(lens))
    dev = torch.device("cuda", rank)
    q, kc, vc = (torch.from_numpy(p[x]).to(dev).to(torch.bfloat16)
                 for x in ("q", "k_cache", "v_cache"))
    bt = torch.from_numpy(p["block_tables"]).to(dev)
    cl = torch.from_numpy(p["context_lens"]).to(dev)
    ws = torch.zeros(flash_engine.paged_attention_workspace_floats(H, Hkv, d),
                     dtype=torch.float32, device=dev)
    ex = sharding.KVRangeExchange(S * H, d)
    errs = []

    def check(seed):
        q2 = O.make_paged_problem(seed, S, H, Hkv, d, lens)["q"]
        q.copy_(torch.from_numpy(q2).to(dev).to(torch.bfloat16))
        return q2

    for seed in (62, 63, 64):
        q2 = check(seed)
        out = ex.decode(q, kc, vc, bt, cl, M, 16, workspace=ws)
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        errs.append(float(np.abs(out.float().cpu().numpy() - ref).max()))
    g = graph.DecodeGraph(lambda: ex.decode(q, kc, vc, bt, cl, M, 16, workspace=ws))
    for seed in (65, 66):
        q2 = check(seed)
        out = g.replay()
        torch.cuda.synchronize()
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        errs.append(float(np.abs(out.float().cpu().numpy() - ref).max()))
    step = ex.prepare(q, kc, vc, bt, cl, M, 16, workspace=ws)
    for seed in (67, 68):
        q2 = check(seed)
        out = step()
        torch.cuda.synchronize()
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        errs.append(float(np.abs(out.float().cpu().numpy() - ref).max()))
    dev_errs = flash_engine.device_errors()
    del g
    ex.close()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr((max(errs), dev_errs)))


def nccl_c_entry_worker(rank, world, port, result_path):
    """The C entry that takes an NCCL communicator (fe_paged_decode_kv_range_nccl_bf16):
    the communicator is made by the library from a unique id that rank 0 creates and
    the process group broadcasts; every rank decodes its KV range of the same cache."""
    import ctypes
    import torch
    import torch.distributed as dist
    import flash_engine
    from flash_engine import _lib
    from oracle import attention_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    L = _lib.lib
    uid = (ctypes.c_ubyte * 128)()
    if rank == 0:
        assert L.fe_nccl_unique_id(uid) == 0
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
    comm = ctypes.c_void_p()
    assert L.fe_nccl_comm_init(ctypes.byref(comm), world, uid, rank) == 0
    lens = [0, 5, 16, 300, 1500, 2047]
    S, H, Hkv, d = len(lens), 32, 8, 128
    p = O.make_paged_problem(71, S, H, Hkv, d, lens)
    dev = torch.device("cuda", rank)
    q, kc, vc = (torch.from_numpy(p[x]).to(dev).to(torch.bfloat16)
                 for x in ("q", "k_cache", "v_cache"))
    bt = torch.from_numpy(p["block_tables"]).to(dev)
    cl = torch.from_numpy(p["context_lens"]).to(dev)
    ws = torch.zeros(flash_engine.paged_attention_workspace_floats(H, Hkv, d), dtype=torch.float32,
                     device=dev)
    scratch = torch.empty(L.fe_kv_range_nccl_scratch_floats(world, S, H, d), dtype=torch.float32,
                          device=dev)
    out = torch.empty_like(q)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.fe_paged_decode_kv_range_nccl_bf16(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), cl.data_ptr(), S, H, Hkv, d, 16,
        bt.shape[1], kc.shape[0], 0.0, int(max(lens)), ws.data_ptr(), ws.numel(), comm, rank,
        world, scratch.data_ptr(), scratch.numel(), out.data_ptr(), st)
    torch.cuda.synchronize()
    errs = flash_engine.device_errors()
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    err = float(np.abs(out.float().cpu().numpy() - ref).max()) if rc == 0 else float("inf")
    L.fe_nccl_comm_destroy(comm)
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(repr((rc, err, errs)))
