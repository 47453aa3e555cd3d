#!/usr/bin/env python
"""Benchmark of the inference-attention hot path on B200 (one process per GPU).

Headline (``value``): benchmark config 3, paged decode bf16 -- batch 64, 32 query /
8 KV heads, head_dim 128, block size 16, context lengths U[512, 4096] (seed 0),
physical blocks a random permutation of the pool. One step = one
``flash_engine.paged_attention`` call over the whole batch (one persistent split-KV
kernel with the log-sum-exp merge fused in), replayed from CUDA graphs of 10 steps.
With N GPUs (torchrun) the KV heads are sharded: rank r owns KV heads
[r*8/N, (r+1)*8/N) and their query heads; no communication (strong scaling). Metric:
KV GB/s = algorithmic bytes per step (K and V rows of every context token and KV head,
q, out, block-table entries, context lengths) / step time, whole job; ``roofline``
against the measured HBM copy peak.

``secondary`` reports the other benchmark configs measured in the same run:
  config 2 -- FA2 prefill bf16 causal [4, 32, 4096, 128], heads sharded (TFLOP/s);
  config 4 -- split-KV decode, 131072-token context, KV range sharded over the
              ranks; the decode kernel stores its (O, m, l) partials into every
              rank's exchange buffer over NVLink and a merge kernel combines them
              (``--kv-exchange nccl``: an NCCL all-gather instead) (KV GB/s);
  config 5 -- serving-mix paged decode, 256 seqs, 64q/8kv, lognormal contexts,
              KV-head sharded (KV GB/s);
  config 1 -- FA2 forward fp32 [1, 8, 512, 64], non-causal (3xTF32 tensor-core
              kernel), heads sharded (TFLOP/s);
  paged_fp32 -- the reference's fp32 paged entry on config 3's shapes with an fp32
              cache (KV GB/s).
``--workload`` makes any of them the headline instead. ``--impl reference`` times the
reference's CPU implementation of the path (the NumPy port in oracle/, all host
threads) on a bounded sample per step.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
import traceback

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "flash-kernel-engine_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
WORKLOADS = ("decode", "serving", "splitkv", "prefill", "prefill_fp32", "paged_fp32")


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=WORKLOADS, default="decode")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--num-seqs", type=int, default=0,
                    help="paged_fp32 only: use the first N sequences of config 3 (a small "
                         "case for profiler captures); 0 = all 64")
    ap.add_argument("--kv-exchange", choices=["p2p", "nccl"], default="p2p",
                    help="KV-range all-gather at N > 1: the decode kernel's own peer stores "
                         "(p2p) or NCCL all-gather + merge kernel (nccl)")
    return ap.parse_args()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def _traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) every 5 ms."""

    REASONS = {
        0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
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
        return self

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
        reasons = [n for b, n in self.REASONS.items() if bits & b]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(inside), "window": window}


# --------------------------------------------------------------------------- distributed
def _dist():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _max_over_ranks(x, ws, device):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(ws, device):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])


def _time_steps(step, steps, warmup, ws, dev):
    """Warm up, then time `steps` back-to-back calls with CUDA events on the current
    stream between barriers; returns (ms_per_step on this rank, t0, t1)."""
    import torch
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    _barrier(ws, dev)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(st)
    for i in range(steps):
        step(i)
    e1.record(st)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    _barrier(ws, dev)
    return e0.elapsed_time(e1) / steps, t0, t1


# --------------------------------------------------------------------------- paged decode
CFG3 = dict(name="paged_decode_config3", num_seqs=64, num_heads=32, num_kv_heads=8,
            head_dim=128, block_size=16,
            metric="paged decode KV GB/s (config 3: B64, 32q/8kv, d128, bs16, ctx U[512,4096])")
CFG5 = dict(name="paged_decode_config5_serving", num_seqs=256, num_heads=64, num_kv_heads=8,
            head_dim=128, block_size=16,
            metric="serving-mix paged decode KV GB/s (config 5: B256, 64q/8kv, d128, bs16, "
                   "ctx lognormal(med 1024, sigma 1) in [16, 32768])")


def _lens(cfg, seed):
    from oracle import attention_oracle as O
    if cfg is CFG5:
        return O.config5_context_lens(seed)
    return O.config3_context_lens(seed)


def decode_bytes(lens, Hkv, H, d, bs, elt=2):
    """Algorithmic bytes of one decode call: K+V rows of every context token of
    every KV head, plus q and out, block-table entries and context lengths."""
    lens = np.maximum(np.asarray(lens), 0)
    tokens = int(lens.sum())
    pages = int(((lens + bs - 1) // bs).sum())
    S = len(lens)
    return tokens * Hkv * d * 2 * elt + 2 * S * H * d * elt + pages * 4 + S * 4


def bench_paged(a, ws, rank, local, cfg, with_cpu, steps, warmup):
    import torch
    import flash_engine

    dev = torch.device("cuda", local)
    S, H, Hkv, d, bs = (cfg[k] for k in ("num_seqs", "num_heads", "num_kv_heads", "head_dim",
                                         "block_size"))
    if Hkv % ws:
        raise ValueError(f"{ws} ranks cannot split {Hkv} KV heads")
    hkv_l, h_l = Hkv // ws, H // ws
    lens = _lens(cfg, a.seed)
    nblk = (lens + bs - 1) // bs
    pool = int(nblk.sum())
    # Disjoint block sets rotated between steps: >= 4 x L2 of distinct KV over a cycle.
    kv_set = pool * hkv_l * bs * d * 2 * 2
    R = max(1, math.ceil(4 * L2_BYTES / kv_set))
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
    kc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((S, h_l, d), generator=g, device=dev).to(torch.bfloat16)
    lens_t = torch.from_numpy(lens).to(dev)
    out = torch.empty_like(q)
    max_ctx = int(lens.max())
    wsp = torch.zeros(flash_engine.paged_attention_workspace_floats(h_l, hkv_l, d, bs),
                      dtype=torch.float32, device=dev)

    def call(i):
        flash_engine.paged_attention(q, kc, vc, bts[i % R], lens_t, bs, max_context_len=max_ctx,
                                     out=out, workspace=wsp)

    # A decode step is one call of the public API. The calls are captured GSTEPS at a
    # time into CUDA graphs (one per starting block set) and replayed back to back, as a
    # serving loop replays its captured decode steps. The decode kernel is launched with
    # programmatic dependent launch, so inside a graph each call's CTAs are placed as
    # the previous call's CTAs retire (they wait for its results before reading
    # anything). One graph per call measured 26.8 us a step on the N = 8 shard, 24.4 us
    # with 10 calls per graph.
    GSTEPS = 10 if steps % 10 == 0 and warmup >= 3 else 1
    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    graphs = []
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        for r in range(R):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=cap):
                for j in range(GSTEPS):
                    call(r + j)
            graphs.append(gr)
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()

    def step(i):  # GSTEPS decode steps, starting at step i * GSTEPS
        graphs[(i * GSTEPS) % R].replay()

    sampler = ClockSampler(local).start()
    ms_rank, t0, t1 = _time_steps(step, steps // GSTEPS, max(1, -(-warmup // GSTEPS)), ws, dev)
    ms_rank /= GSTEPS
    sampler.stop()
    assert flash_engine.device_errors() == 0
    ms = _max_over_ranks(ms_rank, ws, dev)
    total = decode_bytes(lens, Hkv, H, d, bs)
    rank_bytes = decode_bytes(lens, hkv_l, h_l, d, bs)

    # End to end through the public API: the step's q, block table and context lengths
    # from pinned host memory, the output back to pinned host memory, wall clock.
    q_h = q.cpu().pin_memory()
    bt_h = [b.cpu().pin_memory() for b in bts]
    lens_h = lens_t.cpu().pin_memory()
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_d, lens_d, bt_d = torch.empty_like(q), torch.empty_like(lens_t), torch.empty_like(bts[0])

    def e2e_step(i):
        q_d.copy_(q_h, non_blocking=True)
        bt_d.copy_(bt_h[i % R], non_blocking=True)
        lens_d.copy_(lens_h, non_blocking=True)
        o = flash_engine.paged_attention(q_d, kc, vc, bt_d, lens_d, bs, max_context_len=max_ctx,
                                         workspace=wsp)
        out_h.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(3):
        e2e_step(i)
    _barrier(ws, dev)
    n_e2e = max(1, min(steps, 200))
    te0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    te1 = time.perf_counter()
    e2e_serial_ms = _max_over_ranks((te1 - te0) * 1e3 / n_e2e, ws, dev)

    # The same steps two deep, as a serving loop runs them: step i+1's inputs are copied
    # in (one copy stream) while step i decodes, and step i's output is copied out (a
    # second copy stream) while step i+1 decodes; the host reads step i's output before
    # it reuses that step's buffers two steps later. Every step still moves its own
    # inputs in and its own output out.
    comp = torch.cuda.current_stream()
    in_s, out_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    qb = [torch.empty_like(q) for _ in range(2)]
    btb = [torch.empty_like(bts[0]) for _ in range(2)]
    lb = [torch.empty_like(lens_t) for _ in range(2)]
    ob = [torch.empty_like(out) for _ in range(2)]
    ohb = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_pipelined(n):
        for i in range(n):
            b = i % 2
            if i >= 2:
                ev_done[b].synchronize()  # step i-2's output is on the host
            with torch.cuda.stream(in_s):
                if i >= 2:
                    in_s.wait_event(ev_used[b])
                qb[b].copy_(q_h, non_blocking=True)
                btb[b].copy_(bt_h[i % R], non_blocking=True)
                lb[b].copy_(lens_h, non_blocking=True)
                ev_in[b].record(in_s)
            comp.wait_event(ev_in[b])
            flash_engine.paged_attention(qb[b], kc, vc, btb[b], lb[b], bs, max_context_len=max_ctx,
                                         out=ob[b], workspace=wsp)
            ev_used[b].record(comp)
            with torch.cuda.stream(out_s):
                out_s.wait_event(ev_used[b])
                ohb[b].copy_(ob[b], non_blocking=True)
                ev_done[b].record(out_s)
        torch.cuda.synchronize()

    e2e_pipelined(4)
    _barrier(ws, dev)
    te0 = time.perf_counter()
    e2e_pipelined(n_e2e)
    te1 = time.perf_counter()
    e2e_ms = _max_over_ranks((te1 - te0) * 1e3 / n_e2e, ws, dev)
    del graphs

    peak_hbm, _, _, src = _peaks()
    res = {
        "metric": cfg["metric"], "value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(ms, 5),
        "config": {"workload": cfg["name"], "num_seqs": S, "num_heads": H, "num_kv_heads": Hkv,
                   "head_dim": d, "block_size": bs, "total_context_tokens": int(lens.sum()),
                   "bytes_per_step": total, "workspace_floats": int(wsp.numel()),
                   "parallelism": f"kv-head shard x{ws}",
                   "l2": f"{R} disjoint block sets rotated per step "
                         f"({R * kv_set / 2**20:.0f} MiB per rank)"},
        "roofline": {"bound": "hbm", "achieved": round(rank_bytes / (ms_rank * 1e-3) / 1e9, 2),
                     "peak": peak_hbm, "unit": "GB/s",
                     "frac": round(rank_bytes / (ms_rank * 1e-3) / 1e9 / peak_hbm, 4),
                     "peak_source": src, "kernel": "paged_decode_kernel (merge fused)",
                     "traffic": _traffic("paged_decode_config3_traffic.json")
                     if cfg is CFG3 and ws == 1 else None},
        "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": int(q_h.numel() * 2 + bt_h[0].numel() * 4 + lens_h.numel() * 4),
                "d2h_bytes_per_step": int(out_h.numel() * 2),
                "mode": "two steps in flight (copies overlap the neighbouring steps' decode)",
                "serial_value": round(total / (e2e_serial_ms * 1e-3) / 1e9, 2),
                "serial_ms_per_step": round(e2e_serial_ms, 4)},
        "gpu_launches": steps,
        "clocks": sampler.summary(t0, t1),
    }
    if with_cpu and rank == 0 and ws == 1:
        res["cpu_baseline"] = cpu_paged_baseline(cfg, lens, a.seed, budget_s=12.0)
    return res


def bench_paged_fp32(a, ws, rank, local, steps, warmup):
    """The reference's fp32 paged entry (launch_paged_attention_v1_fp32) on config 3's
    shapes with an fp32 cache: one step = one flash_engine.paged_attention call (512-token
    split kernel + merge). KV heads sharded over the ranks as in config 3."""
    import torch
    import flash_engine

    dev = torch.device("cuda", local)
    c = CFG3
    H, Hkv, d, bs = c["num_heads"], c["num_kv_heads"], c["head_dim"], c["block_size"]
    if Hkv % ws:
        raise ValueError(f"{ws} ranks cannot split {Hkv} KV heads")
    hkv_l, h_l = Hkv // ws, H // ws
    lens = _lens(c, a.seed)
    if a.num_seqs > 0:
        lens = lens[:a.num_seqs]
    S = len(lens)
    nblk = (lens + bs - 1) // bs
    pool = int(nblk.sum())
    kv_set = pool * hkv_l * bs * d * 4 * 2
    R = max(1, math.ceil(2 * L2_BYTES / kv_set))
    rng = np.random.default_rng(a.seed + 1)
    perm = rng.permutation(pool * R).astype(np.int32)
    maxb = int(nblk.max())
    bts = []
    for r in range(R):
        bt = np.zeros((S, maxb), np.int32)
        off = r * pool
        for s_ in range(S):
            bt[s_, :nblk[s_]] = perm[off:off + nblk[s_]]
            off += nblk[s_]
        bts.append(torch.from_numpy(bt).to(dev))
    g = torch.Generator(device=dev)
    g.manual_seed(3000 + a.seed * 17 + rank)
    kc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev)
    vc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev)
    q = torch.randn((S, h_l, d), generator=g, device=dev)
    lens_t = torch.from_numpy(lens).to(dev)
    out = torch.empty_like(q)

    def step(i):
        flash_engine.paged_attention(q, kc, vc, bts[i % R], lens_t, bs, out=out)

    sampler = ClockSampler(local).start()
    ms_rank, t0, t1 = _time_steps(step, steps, max(3, warmup), ws, dev)
    sampler.stop()
    assert flash_engine.device_errors() == 0
    ms = _max_over_ranks(ms_rank, ws, dev)
    total = decode_bytes(lens, Hkv, H, d, bs, elt=4)
    rank_bytes = decode_bytes(lens, hkv_l, h_l, d, bs, elt=4)

    # End to end through the public API: q, block table and lengths in from pinned host
    # memory, the output back, one step at a time on the wall clock.
    q_h, lens_h = q.cpu().pin_memory(), lens_t.cpu().pin_memory()
    bt_h = [b.cpu().pin_memory() for b in bts]
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_d, lens_d, bt_d = torch.empty_like(q), torch.empty_like(lens_t), torch.empty_like(bts[0])

    def e2e_step(i):
        q_d.copy_(q_h, non_blocking=True)
        bt_d.copy_(bt_h[i % R], non_blocking=True)
        lens_d.copy_(lens_h, non_blocking=True)
        out_h.copy_(flash_engine.paged_attention(q_d, kc, vc, bt_d, lens_d, bs), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(3):
        e2e_step(i)
    _barrier(ws, dev)
    n_e2e = max(1, min(steps, 50))
    te0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    e2e_ms = _max_over_ranks((time.perf_counter() - te0) * 1e3 / n_e2e, ws, dev)
    peak_hbm, _, _, src = _peaks()
    return {
        "metric": "paged decode fp32 KV GB/s (the reference's v1 fp32 entry on config 3 shapes)",
        "value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(ms, 5),
        "config": {"workload": "paged_decode_fp32_config3", "num_seqs": S, "num_heads": H,
                   "num_kv_heads": Hkv, "head_dim": d, "block_size": bs,
                   "total_context_tokens": int(lens.sum()), "bytes_per_step": total,
                   "parallelism": f"kv-head shard x{ws}",
                   "l2": f"{R} block set(s) of {kv_set / 2**20:.0f} MiB per rank used in turn"},
        "roofline": {"bound": "hbm", "achieved": round(rank_bytes / (ms_rank * 1e-3) / 1e9, 2),
                     "peak": peak_hbm, "unit": "GB/s",
                     "frac": round(rank_bytes / (ms_rank * 1e-3) / 1e9 / peak_hbm, 4),
                     "peak_source": src,
                     "kernel": "paged_split_fp32_kernel (512-token splits) + merge_kernel",
                     "traffic": None},
        "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": int(q_h.numel() * 4 + bt_h[0].numel() * 4 + lens_h.numel() * 4),
                "d2h_bytes_per_step": int(out_h.numel() * 4)},
        "gpu_launches": 2 * steps,
        "clocks": sampler.summary(t0, t1),
    }


def cpu_paged_baseline(cfg, lens, seed, budget_s=12.0, steps=1):
    """The NumPy port of the reference's paged_attention (per KV-head group), timed on
    the host over a bounded prefix of the workload's sequences."""
    from oracle import attention_oracle as O
    H, Hkv, d, bs = cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"], cfg["block_size"]
    p1 = O.make_paged_problem(seed, 1, H, Hkv, d, lens[:1])
    t = time.perf_counter()
    O.paged_attention_gqa(p1["q"], p1["k_cache"], p1["v_cache"], p1["block_tables"],
                          p1["context_lens"])
    per_tok = (time.perf_counter() - t) / max(1, int(lens[0]))
    n = 1
    while n < len(lens) and per_tok * int(lens[:n + 1].sum()) * steps < budget_s:
        n += 1
    sub = lens[:n]
    p = O.make_paged_problem(seed, n, H, Hkv, d, sub)
    t = time.perf_counter()
    for _ in range(steps):
        O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                              p["context_lens"])
    dt = (time.perf_counter() - t) / steps
    b = decode_bytes(sub, Hkv, H, d, bs)
    return {"value": round(b / dt / 1e9, 4), "unit": "GB/s", "cores": _cpu_threads(),
            "kind": "port",
            "sample": f"first {n} of {len(lens)} sequences of {cfg['name']} "
                      f"({int(sub.sum())} tokens), {dt:.2f} s per pass; bytes counted as bf16"}


# --------------------------------------------------------------------------- split-KV (config 4)
CFG4 = dict(name="splitkv_decode_config4", batch=4, num_heads=32, num_kv_heads=8, head_dim=128,
            block_size=16, context=131072,
            metric="split-KV decode KV GB/s (config 4: B4, 32q/8kv, d128, ctx 131072, bs16)")


def bench_splitkv(a, ws, rank, local, steps, warmup):
    import torch
    import flash_engine
    from flash_engine import sharding

    dev = torch.device("cuda", local)
    c = CFG4
    B, H, Hkv, d, bs, M = (c[k] for k in ("batch", "num_heads", "num_kv_heads", "head_dim",
                                          "block_size", "context"))
    tb, te = sharding.kv_range_bounds(M, ws, rank, bs)
    nloc = (te - tb + bs - 1) // bs           # blocks this rank holds per sequence
    maxb = (M + bs - 1) // bs
    pool = B * nloc
    rng = np.random.default_rng(a.seed + 7)
    perm = rng.permutation(pool).astype(np.int32)
    bt = np.zeros((B, maxb), np.int32)
    for s in range(B):
        bt[s, tb // bs: tb // bs + nloc] = perm[s * nloc:(s + 1) * nloc]
    g = torch.Generator(device=dev)
    g.manual_seed(3000 + rank)
    kc = torch.randn((pool, Hkv, bs, d), generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn((pool, Hkv, bs, d), generator=g, device=dev).to(torch.bfloat16)
    q_all = torch.randn((B, H, d), generator=g, device=dev).to(torch.bfloat16)
    if ws > 1:
        import torch.distributed as dist
        dist.broadcast(q_all, 0)        # every rank decodes the same query tokens
    bt_t = torch.from_numpy(bt).to(dev)
    lens_t = torch.full((B,), M, dtype=torch.int32, device=dev)
    wsp = torch.zeros(flash_engine.paged_attention_workspace_floats(H, Hkv, d, bs),
                      dtype=torch.float32, device=dev)

    ex = sharding.KVRangeExchange(B * H, d) if ws > 1 and a.kv_exchange == "p2p" else None

    def call(i, qq=q_all, bb=bt_t, ll=lens_t):
        if ws == 1:
            return flash_engine.paged_attention(qq, kc, vc, bb, ll, bs, max_context_len=M,
                                                version="v2", workspace=wsp)
        if ex is not None:
            return ex.decode(qq, kc, vc, bb, ll, M, bs, workspace=wsp)
        return sharding.paged_decode_kv_range(qq, kc, vc, bb, ll, M, bs, workspace=wsp)

    # A step (decode, all-gather and merge at N > 1) is one CUDA-graph replay, except
    # with the peer-memory exchange: its two launches are not CPU-bound, and replaying
    # them as a graph measured slower at N = 8 (88 vs 70 us a step), so they are issued
    # directly.
    from flash_engine.graph import DecodeGraph
    graph = DecodeGraph(lambda: call(0)) if ex is None else None

    def step(i):
        if graph is not None:
            graph.replay()
        else:
            call(i)

    sampler = ClockSampler(local).start()
    ms_rank, t0, t1 = _time_steps(step, steps, warmup, ws, dev)
    sampler.stop()
    assert flash_engine.device_errors() == 0
    ms = _max_over_ranks(ms_rank, ws, dev)
    kv_total = B * M * Hkv * d * 2 * 2
    kv_rank = B * (te - tb) * Hkv * d * 2 * 2
    # end to end: q, block table and lengths from pinned host, output back to host
    q_h, bt_h, l_h = q_all.cpu().pin_memory(), bt_t.cpu().pin_memory(), lens_t.cpu().pin_memory()
    out_h = torch.empty(q_all.shape, dtype=q_all.dtype).pin_memory()
    q_d, bt_d, l_d = torch.empty_like(q_all), torch.empty_like(bt_t), torch.empty_like(lens_t)

    def e2e(i):
        q_d.copy_(q_h, non_blocking=True)
        bt_d.copy_(bt_h, non_blocking=True)
        l_d.copy_(l_h, non_blocking=True)
        out_h.copy_(call(i, q_d, bt_d, l_d), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(3):
        e2e(i)
    _barrier(ws, dev)
    n = max(1, min(steps, 100))
    te0 = time.perf_counter()
    for i in range(n):
        e2e(i)
    e2e_ms = _max_over_ranks((time.perf_counter() - te0) * 1e3 / n, ws, dev)
    del graph
    if ex is not None:
        ex.close()
    peak_hbm, _, _, src = _peaks()
    return {
        "metric": c["metric"], "value": round(kv_total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(ms, 5),
        "config": {"workload": c["name"], "batch": B, "num_heads": H, "num_kv_heads": Hkv,
                   "head_dim": d, "context": M, "block_size": bs,
                   "parallelism": f"kv-range shard x{ws} + all-gather of (O,m,l) partials"
                                  + ("" if ws == 1 else
                                     " by the decode kernel's peer stores" if ex is not None
                                     else " by NCCL"),
                   "l2": f"{kv_rank / 2**20:.0f} MiB of KV per rank"},
        "roofline": {"bound": "hbm", "achieved": round(kv_rank / (ms_rank * 1e-3) / 1e9, 2),
                     "peak": peak_hbm, "unit": "GB/s",
                     "frac": round(kv_rank / (ms_rank * 1e-3) / 1e9 / peak_hbm, 4),
                     "peak_source": src},
        "e2e": {"value": round(kv_total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(q_h.numel() * 2 + bt_h.numel() * 4 + l_h.numel() * 4),
                "d2h_bytes_per_step": int(out_h.numel() * 2)},
        "clocks": sampler.summary(t0, t1),
    }


# --------------------------------------------------------------------------- prefill (config 2)
def prefill_flops(B, H, N, d, causal=True):
    """4*B*H*N^2*d, halved for causal (the reference's convention,
    benchmarks/bench_attention.cu:48-49)."""
    f = 4.0 * B * H * N * N * d
    return f / 2 if causal else f


def bench_prefill(a, ws, rank, local, steps, warmup, fp32=False):
    import torch
    import flash_engine

    dev = torch.device("cuda", local)
    if fp32:   # config 1: fp32, non-causal, [1, 8, 512, 64]
        B, H, N, d, causal, dt = 1, 8, 512, 64, False, torch.float32
        name = "fa2_prefill_fp32_config1"
        metric = "FA2 forward fp32 TFLOP/s (config 1: [1, 8, 512, 64], non-causal)"
    else:
        B, H, N, d, causal, dt = 4, 32, 4096, 128, True, torch.bfloat16
        name = "fa2_prefill_config2"
        metric = "FA2 prefill TFLOP/s (config 2: bf16 causal [4, 32, 4096, 128])"
    if H % ws:
        raise ValueError(f"{ws} ranks cannot split {H} heads")
    h_l = H // ws
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + a.seed * 31 + rank)
    # Enough input sets, used in turn, that consecutive steps never find their Q/K/V/O
    # in L2 (>= 2 x L2 over a cycle; one set at N = 1, several for small shards).
    set_bytes = 4 * B * h_l * N * d * (4 if fp32 else 2)
    nsets = max(1, math.ceil(2 * L2_BYTES / set_bytes))
    sets = [tuple(torch.randn((B, h_l, N, d), generator=g, device=dev).to(dt) for _ in range(3))
            for _ in range(nsets)]
    outs = [torch.empty_like(sets[0][0]) for _ in range(nsets)]
    q, k, v = sets[0]

    def call(i):
        qq, kk, vv = sets[i % nsets]
        return flash_engine.flash_attention(qq, kk, vv, causal, out=outs[i % nsets])

    # config 1 (fp32) runs for about as long as the host takes to issue one call, so its
    # steps are replayed from CUDA graphs of GSTEPS calls (one graph per starting input
    # set), as a serving loop replays captured work; the bf16 steps are long enough to
    # be issued one at a time.
    GSTEPS = 10 if fp32 and steps % 10 == 0 and warmup >= 3 else 1
    graphs = []
    if GSTEPS > 1:
        for i in range(3):
            call(i)
        torch.cuda.synchronize()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            for r in range(nsets):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=cap):
                    for j in range(GSTEPS):
                        call(r + j)
                graphs.append(gr)
        torch.cuda.current_stream().wait_stream(cap)
        torch.cuda.synchronize()

    def step(i):  # GSTEPS calls, starting at call i * GSTEPS
        if GSTEPS > 1:
            graphs[(i * GSTEPS) % nsets].replay()
        else:
            call(i)

    sampler = ClockSampler(local).start()
    ms_rank, t0, t1 = _time_steps(step, steps // GSTEPS, max(1, -(-warmup // GSTEPS)), ws, dev)
    ms_rank /= GSTEPS
    sampler.stop()
    del graphs
    assert flash_engine.device_errors() == 0
    ms = _max_over_ranks(ms_rank, ws, dev)
    total = prefill_flops(B, H, N, d, causal)
    rank_flops = prefill_flops(B, h_l, N, d, causal)
    achieved = rank_flops / (ms_rank * 1e-3) / 1e12

    # End to end through the public API: Q, K, V from pinned host memory and O back,
    # every step (the host link, not the kernel, bounds this number).
    q_h, k_h, v_h = (x.cpu().pin_memory() for x in (q, k, v))
    o_h = torch.empty(q.shape, dtype=dt).pin_memory()
    qd, kd, vd = (torch.empty_like(x) for x in (q, k, v))

    def e2e_step(i):
        qd.copy_(q_h, non_blocking=True)
        kd.copy_(k_h, non_blocking=True)
        vd.copy_(v_h, non_blocking=True)
        o_h.copy_(flash_engine.flash_attention(qd, kd, vd, causal), non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step(0)
    _barrier(ws, dev)
    n_e2e = max(1, min(steps, 5 if not fp32 else 100))
    te0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    e2e_ms = _max_over_ranks((time.perf_counter() - te0) * 1e3 / n_e2e, ws, dev)
    elt = 4 if fp32 else 2
    _, peak, peak_sus, src = _peaks()
    # fp32 runs on the tensor core as 3xTF32 (three TF32 products per fp32 product, TF32 at
    # half the bf16 rate): its ceiling in fp32 FLOP/s is the bf16 peak / 6.
    pk, pk_sus = (peak / 6, peak_sus / 6) if fp32 else (peak, peak_sus)
    return {
        "metric": metric, "value": round(total / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
        "ms_per_step": round(ms, 4),
        "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": int(3 * q.numel() * elt),
                "d2h_bytes_per_step": int(q.numel() * elt)},
        "config": {"workload": name, "batch": B, "heads": H, "seq_len": N, "head_dim": d,
                   "causal": causal, "parallelism": f"head shard x{ws}",
                   "flops_per_step": total,
                   "l2": f"{nsets} input set(s) of {set_bytes / 2**20:.0f} MiB used in turn",
                   "steps_per_graph": GSTEPS},
        "roofline": {"bound": "tensor",
                     "achieved": round(achieved, 3), "peak": round(pk, 1),
                     "unit": "TFLOP/s", "frac": round(achieved / pk, 4),
                     "frac_of_sustained": round(achieved / pk_sus, 4),
                     "peak_source": src + (" bf16 burst / 6: TF32 runs at half the bf16 rate "
                                           "and each fp32 product takes 3 TF32 products"
                                           if fp32 else " bf16 burst"),
                     "kernel": "fa_tf32_kernel (3xTF32 tcgen05)" if fp32 else "fa_prefill_kernel",
                     "traffic": None if fp32 or ws > 1 else _traffic("fa_prefill_config2_traffic.json")},
        "clocks": sampler.summary(t0, t1),
        "gpu_launches": steps,
    }


# --------------------------------------------------------------------------- reference arm
def bench_reference(a, ws, rank):
    """--impl reference: the reference's CPU implementation (its NumPy paged_attention,
    ported to oracle/) on the host cores, over a bounded prefix of config 3."""
    if rank != 0:
        return None
    from oracle import attention_oracle as O
    c = CFG3
    lens = _lens(c, a.seed)
    per_step = max(0.05, 120.0 / max(1, a.steps + a.warmup))
    H, Hkv, d, bs = c["num_heads"], c["num_kv_heads"], c["head_dim"], c["block_size"]
    p1 = O.make_paged_problem(a.seed, 1, H, Hkv, d, lens[:1])
    t = time.perf_counter()
    O.paged_attention_gqa(p1["q"], p1["k_cache"], p1["v_cache"], p1["block_tables"],
                          p1["context_lens"])
    per_tok = (time.perf_counter() - t) / max(1, int(lens[0]))
    n = 1
    while n < len(lens) and per_tok * int(lens[:n + 1].sum()) < per_step:
        n += 1
    sub = lens[:n]
    p = O.make_paged_problem(a.seed, n, H, Hkv, d, sub)
    args = (p["q"], p["k_cache"], p["v_cache"], p["block_tables"], p["context_lens"])
    for _ in range(a.warmup):
        O.paged_attention_gqa(*args)
    t = time.perf_counter()
    for _ in range(a.steps):
        O.paged_attention_gqa(*args)
    dt = (time.perf_counter() - t) / max(1, a.steps)
    v = round(decode_bytes(sub, Hkv, H, d, bs) / dt / 1e9, 4)
    return {
        "impl": "reference", "metric": c["metric"], "value": v, "unit": "GB/s", "n_gpus": ws,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 (bf16-rounded inputs)", "data": "synthetic",
        "config": {"workload": c["name"], "sample_seqs": n},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": _cpu_threads(), "kind": "port",
                         "sample": f"first {n} of 64 config-3 sequences per step"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- main
def run_workload(name, a, ws, rank, local, primary):
    steps = a.steps if primary else min(a.steps, 30)
    warmup = a.warmup if primary else min(a.warmup, 3)
    if name == "decode":
        return bench_paged(a, ws, rank, local, CFG3, primary and not a.no_cpu_baseline, steps,
                           warmup)
    if name == "serving":
        return bench_paged(a, ws, rank, local, CFG5, primary and not a.no_cpu_baseline, steps,
                           warmup)
    if name == "splitkv":
        return bench_splitkv(a, ws, rank, local, steps, warmup)
    if name == "prefill":
        return bench_prefill(a, ws, rank, local, steps, warmup)
    if name == "paged_fp32":
        return bench_paged_fp32(a, ws, rank, local, steps, warmup)
    return bench_prefill(a, ws, rank, local, steps, warmup, fp32=True)


def main():
    a = _args()
    ws, rank, local = _dist()
    if a.impl == "reference":
        res = bench_reference(a, ws, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    import torch
    torch.cuda.set_device(local)
    if ws > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    res = run_workload(a.workload, a, ws, rank, local, True)
    res.update({"n_gpus": ws, "steps": a.steps, "warmup": a.warmup, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,1) bf16 inputs; benchmark config shapes)"})
    if a.workload in ("prefill_fp32", "paged_fp32"):
        res["dtype"] = "f32"
    if not a.no_secondary:
        sec = {}
        for name in ("prefill", "splitkv", "serving", "prefill_fp32", "paged_fp32"):
            if name == a.workload:
                continue
            try:
                r = run_workload(name, a, ws, rank, local, False)
                sec[name] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step",
                                               "roofline", "config", "e2e") if k in r}
            except Exception as e:  # recorded, never silently dropped
                sec[name] = {"error": f"{type(e).__name__}: {e}"}
                if rank == 0:
                    traceback.print_exc()
        res["secondary"] = sec
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
