#!/usr/bin/env python
"""Benchmark of the inference-attention hot path on B200.

Default workload: paged decode, bf16, batch 64, 32 query /
8 KV heads, head_dim 128, block size 16, context lengths uniform in [512, 4096]
(seed 0), physical blocks a random permutation of the pool. One step = one
``flash_engine.paged_attention`` call (split-KV kernel + log-sum-exp merge) over
the whole batch. With N GPUs (torchrun, one rank per GPU) the KV heads are
sharded: rank r owns KV heads [r*8/N, (r+1)*8/N) and their query heads; no
communication is needed (strong scaling, total work fixed).

Metric: paged-decode KV bandwidth in GB/s = algorithmic bytes per step (K and V
rows of every context token of every KV head, plus q, out, block-table entries and
context lengths) / step time, whole job. ``--workload prefill`` measures BASELINE
config 2 (FA2 bf16 causal [4, 32, 4096, 128], heads sharded over ranks) in TFLOP/s.

``--impl reference`` times the reference's CPU implementation of the same path
(the NumPy port in oracle/, all host threads) on a bounded sample per step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "flash-kernel-engine_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

L2_BYTES = 126 * 1024 * 1024


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "prefill"], default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            return json.load(f)
    except Exception:
        return None


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) every 5 ms."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self, t0, t1):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        window = "timed"
        if len(inside) < 3:
            inside, window = self.samples, "warmup+timed"
        mhz = statistics.median(s[1] for s in inside)
        bits = 0
        for s in inside:
            bits |= s[2]
        reasons = [n for b, n in self.REASONS.items() if bits & b and b != 0x1]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(inside), "window": window}


# --------------------------------------------------------------------------- distributed
def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _init_pg(ws, backend):
    if ws > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))


def _max_over_ranks(x, ws, device):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(ws, device=None):
    if ws > 1:
        import torch.distributed as dist
        if device is not None:
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


# --------------------------------------------------------------------------- decode workload
CFG3 = dict(num_seqs=64, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16)


def decode_bytes(lens, Hkv, H, d, bs, elt=2):
    """Algorithmic bytes of one decode call: K+V rows of every context token of
    every KV head, plus q and out, block-table entries and context lengths."""
    tokens = int(np.sum(np.maximum(lens, 0)))
    pages = int(np.sum((np.maximum(lens, 0) + bs - 1) // bs))
    S = len(lens)
    return tokens * Hkv * d * 2 * elt + 2 * S * H * d * elt + pages * 4 + S * 4


def bench_decode_ours(a, ws, rank, local):
    import torch
    import flash_engine
    from oracle.attention_oracle import config3_context_lens

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _init_pg(ws, "nccl")
    c = CFG3
    S, H, Hkv, d, bs = c["num_seqs"], c["num_heads"], c["num_kv_heads"], c["head_dim"], c["block_size"]
    if Hkv % ws:
        raise SystemExit(f"--gpus {ws} must divide the {Hkv} KV heads")
    hkv_l, h_l = Hkv // ws, H // ws
    lens = config3_context_lens(a.seed)
    nblk = (lens + bs - 1) // bs
    pool = int(nblk.sum())
    step_bytes_rank = decode_bytes(lens, hkv_l, h_l, d, bs)
    # Disjoint block sets rotated between steps so that consecutive steps never
    # hit L2 (>= 4 x L2 of distinct KV bytes in flight over the rotation).
    kv_bytes_set = pool * hkv_l * bs * d * 2 * 2
    R = max(1, math.ceil(4 * L2_BYTES / kv_bytes_set))
    rng = np.random.default_rng(a.seed + 1)
    perm = rng.permutation(pool * R).astype(np.int32)
    maxb = int(nblk.max())
    bts = []
    for r in range(R):
        bt = np.zeros((S, maxb), np.int32)
        off = r * pool
        for s in range(S):
            bt[s, :nblk[s]] = perm[off:off + nblk[s]]
            off += nblk[s]
        bts.append(torch.from_numpy(bt).to(dev))
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + a.seed * 17 + rank)
    kc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    vc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((S, h_l, d), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    lens_t = torch.from_numpy(lens).to(dev)
    out = torch.empty_like(q)
    max_ctx = int(lens.max())
    splits = flash_engine.paged_attention_splits(S, h_l, hkv_l, d, bs, max_ctx)
    ws_out = torch.empty(S * h_l * splits * d, dtype=torch.float32, device=dev)
    ws_st = torch.empty(S * h_l * splits * 2, dtype=torch.float32, device=dev)

    def step(i):
        flash_engine.paged_attention(q, kc, vc, bts[i % R], lens_t, bs, max_context_len=max_ctx,
                                     num_splits=splits, out=out, workspace=(ws_out, ws_st))

    sampler = ClockSampler(local)
    sampler.start()
    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(ws, dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record(st)
    for i in range(a.steps):
        step(i)
    e1.record(st)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    _barrier(ws, dev)
    sampler.stop()
    ms_rank = e0.elapsed_time(e1) / a.steps
    ms = _max_over_ranks(ms_rank, ws, dev)
    assert flash_engine.device_errors() == 0
    total_bytes = decode_bytes(lens, Hkv, H, d, bs)
    value = total_bytes / (ms * 1e-3) / 1e9
    achieved = step_bytes_rank / (ms_rank * 1e-3) / 1e9

    # ---- end to end through the public API: per-step inputs (q, block table,
    # context lengths) from pinned host memory, the output back to pinned host.
    q_h = q.cpu().pin_memory()
    bt_h = [b.cpu().pin_memory() for b in bts]
    lens_h = lens_t.cpu().pin_memory()
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_d, lens_d = torch.empty_like(q), torch.empty_like(lens_t)
    bt_d = torch.empty_like(bts[0])

    def e2e_step(i):
        q_d.copy_(q_h, non_blocking=True)
        bt_d.copy_(bt_h[i % R], non_blocking=True)
        lens_d.copy_(lens_h, non_blocking=True)
        o = flash_engine.paged_attention(q_d, kc, vc, bt_d, lens_d, bs, max_context_len=max_ctx,
                                         num_splits=splits, workspace=(ws_out, ws_st))
        out_h.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(min(a.warmup, 5)):
        e2e_step(i)
    _barrier(ws, dev)
    n_e2e = max(1, min(a.steps, 200))
    te0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    te1 = time.perf_counter()
    e2e_ms = _max_over_ranks((te1 - te0) * 1e3 / n_e2e, ws, dev)
    h2d = q_h.numel() * 2 + bt_h[0].numel() * 4 + lens_h.numel() * 4
    d2h = out_h.numel() * 2

    peak_hbm, _, peak_src = _peaks()
    prof = _traffic("paged_decode_config3_traffic.json")
    traffic = None
    if prof and ws == 1:
        traffic = prof.get("dram_bytes_per_launch")

    res = {
        "metric": "paged decode KV GB/s (config 3: B64, 32q/8kv, d128, bs16, ctx U[512,4096])",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 K/V/q; lens U[512,4096] seed %d)" % a.seed,
        "config": {
            "workload": "paged_decode_config3",
            "num_seqs": S, "num_heads": H, "num_kv_heads": Hkv, "head_dim": d,
            "block_size": bs, "total_context_tokens": int(lens.sum()),
            "bytes_per_step": total_bytes, "num_splits": splits,
            "parallelism": f"kv-head shard x{ws}",
            "l2": f"{R} disjoint block sets rotated per step ({R * kv_bytes_set / 2**20:.0f} MiB)",
        },
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 2), "peak": peak_hbm, "unit": "GB/s",
            "frac": round(achieved / peak_hbm, 4), "peak_source": peak_src,
            "traffic": traffic,
            "kernel": "paged_decode_kernel + merge_kernel (one step)",
        },
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": 2 * a.steps,
        "clocks": sampler.summary(t0, t1),
    }
    if rank == 0 and ws == 1 and not a.no_cpu_baseline:
        res["cpu_baseline"] = cpu_decode_baseline(lens, a.seed, budget_s=15.0)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return res if rank == 0 else None


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_decode_baseline(lens, seed, budget_s=15.0, steps=1):
    """The NumPy port of the reference's paged_attention (per KV-head group), timed
    on the host over a bounded prefix of config 3's sequences."""
    from oracle import attention_oracle as O
    c = CFG3
    # size the sample to the budget: time one sequence first
    p1 = O.make_paged_problem(seed, 1, c["num_heads"], c["num_kv_heads"], c["head_dim"],
                              lens[:1])
    t = time.perf_counter()
    O.paged_attention_gqa(p1["q"], p1["k_cache"], p1["v_cache"], p1["block_tables"],
                          p1["context_lens"])
    per_tok = (time.perf_counter() - t) / max(1, int(lens[0]))
    n = 1
    while n < len(lens) and per_tok * int(lens[:n + 1].sum()) * steps < budget_s:
        n += 1
    sub = lens[:n]
    p = O.make_paged_problem(seed, n, c["num_heads"], c["num_kv_heads"], c["head_dim"], sub)
    t = time.perf_counter()
    for _ in range(steps):
        O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                              p["context_lens"])
    dt = (time.perf_counter() - t) / steps
    b = decode_bytes(sub, c["num_kv_heads"], c["num_heads"], c["head_dim"], c["block_size"], elt=2)
    return {"value": round(b / dt / 1e9, 4), "unit": "GB/s", "cores": _cpu_threads(),
            "kind": "port",
            "sample": f"first {n} of {len(lens)} config-3 sequences ({int(sub.sum())} tokens), "
                      f"{dt:.2f} s per pass; bytes counted as bf16 like the GPU metric"}


def bench_decode_reference(a, ws, rank):
    """--impl reference: the reference's CPU implementation (NumPy port) only."""
    if rank != 0:
        return None
    from oracle.attention_oracle import config3_context_lens
    lens = config3_context_lens(a.seed)
    total_budget = 120.0
    per_step = max(0.05, total_budget / max(1, a.steps + a.warmup))
    from oracle import attention_oracle as O
    c = CFG3
    p1 = O.make_paged_problem(a.seed, 1, c["num_heads"], c["num_kv_heads"], c["head_dim"], lens[:1])
    t = time.perf_counter()
    O.paged_attention_gqa(p1["q"], p1["k_cache"], p1["v_cache"], p1["block_tables"],
                          p1["context_lens"])
    per_tok = (time.perf_counter() - t) / max(1, int(lens[0]))
    n = 1
    while n < len(lens) and per_tok * int(lens[:n + 1].sum()) < per_step:
        n += 1
    sub = lens[:n]
    p = O.make_paged_problem(a.seed, n, c["num_heads"], c["num_kv_heads"], c["head_dim"], sub)
    args = (p["q"], p["k_cache"], p["v_cache"], p["block_tables"], p["context_lens"])
    for _ in range(a.warmup):
        O.paged_attention_gqa(*args)
    t = time.perf_counter()
    for _ in range(a.steps):
        O.paged_attention_gqa(*args)
    dt = (time.perf_counter() - t) / max(1, a.steps)
    b = decode_bytes(sub, c["num_kv_heads"], c["num_heads"], c["head_dim"], c["block_size"])
    v = round(b / dt / 1e9, 4)
    return {
        "impl": "reference",
        "metric": "paged decode KV GB/s (config 3: B64, 32q/8kv, d128, bs16, ctx U[512,4096])",
        "value": v, "unit": "GB/s", "n_gpus": ws, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (bf16-rounded inputs)", "data": "synthetic",
        "config": {"workload": "paged_decode_config3", "sample_seqs": n},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": _cpu_threads(), "kind": "port",
                         "sample": f"first {n} of 64 config-3 sequences per step"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- prefill workload
CFG2 = dict(batch=4, heads=32, seq=4096, head_dim=128, causal=True)


def prefill_flops(B, H, N, d, causal=True):
    """4*B*H*N^2*d, halved for causal: the reference's convention
    (benchmarks/bench_attention.cu:48-49)."""
    f = 4.0 * B * H * N * N * d
    return f / 2 if causal else f


def bench_prefill_ours(a, ws, rank, local, init_pg=True, steps=None, warmup=None):
    import torch
    import flash_engine

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if init_pg:
        _init_pg(ws, "nccl")
    c = CFG2
    B, H, N, d = c["batch"], c["heads"], c["seq"], c["head_dim"]
    if H % ws:
        raise SystemExit(f"--gpus {ws} must divide the {H} heads")
    h_l = H // ws
    steps = a.steps if steps is None else steps
    warmup = a.warmup if warmup is None else warmup
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + a.seed * 31 + rank)
    q, k, v = (torch.randn((B, h_l, N, d), generator=g, device=dev, dtype=torch.float32)
               .to(torch.bfloat16) for _ in range(3))
    out = torch.empty_like(q)

    def step():
        return flash_engine.flash_attention(q, k, v, True)

    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(ws, dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    _barrier(ws, dev)
    sampler.stop()
    assert flash_engine.device_errors() == 0
    ms_rank = e0.elapsed_time(e1) / steps
    ms = _max_over_ranks(ms_rank, ws, dev)
    flops_rank = prefill_flops(B, h_l, N, d)
    total = prefill_flops(B, H, N, d)
    tflops = total / (ms * 1e-3) / 1e12
    achieved = flops_rank / (ms_rank * 1e-3) / 1e12
    _, peak, src = _peaks()
    return {
        "metric": "FA2 prefill TFLOP/s (config 2: bf16 causal [4, 32, 4096, 128])",
        "value": round(tflops, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "flops_per_step": total,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "peak_source": src + " bf16 burst",
                     "kernel": "fa_prefill_kernel<bf16,128>"},
        "clocks": sampler.summary(t0, t1),
        "gpu_launches": steps,
    }


def main():
    a = _args()
    ws, rank, local = _dist()
    if a.impl == "reference":
        res = bench_decode_reference(a, ws, rank)
    elif a.workload == "prefill":
        pr = bench_prefill_ours(a, ws, rank, local)
        res = None
        if rank == 0:
            res = dict(pr)
            res.update({"n_gpus": ws, "steps": a.steps, "warmup": a.warmup,
                        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 Q/K/V)",
                        "config": {"workload": "fa2_prefill_config2", "batch": 4, "heads": 32,
                                   "seq_len": 4096, "head_dim": 128, "causal": True,
                                   "parallelism": f"head shard x{ws}",
                                   "l2": "inputs 384 MiB > L2"}})
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    else:
        res = bench_decode_ours(a, ws, rank, local)
    if res is not None and rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
