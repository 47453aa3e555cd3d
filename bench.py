#!/usr/bin/env python
"""Benchmark of the inference-attention hot path on B200 (one process per GPU).

Headline (the LAST line printed): benchmark config 3, paged decode bf16 -- batch 64,
32 query / 8 KV heads, head_dim 128, block size 16, context lengths U[512, 4096]
(seed 0), physical blocks a random permutation of the pool. One step = one
``flash_engine.paged_attention`` call over the whole batch (one persistent split-KV
kernel with the log-sum-exp merge fused in), replayed from CUDA graphs of 10 steps.
With N GPUs (torchrun) the KV heads are sharded: rank r owns KV heads
[r*8/N, (r+1)*8/N) and their query heads; no communication. Metric: KV GB/s =
algorithmic bytes per step (K and V rows of every context token and KV head, q, out,
block-table entries, context lengths) / step time, whole job; ``roofline`` against the
measured HBM copy peak (and the nominal 8 TB/s).

Before the headline, one JSON line per other benchmark config measured in the same run
(``"secondary": true``):
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
Every line carries ``parity``: after the timed steps each rank checks a seeded sample of
its output rows against the CPU oracle (the NumPy restatement of the reference's
attention) and the worst error over the ranks is reported with the tolerance (bf16:
2e-2 absolute; fp32: 1e-3 relative). At N = 1, rank 0 also times the oracle on the host
cores for every config (``cpu_baseline``). ``--workload`` makes any config the headline.
``--impl reference`` times the reference's CPU implementation of the path (the NumPy
port in oracle/, all host threads) on a bounded sample per step.
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
WORKLOADS = ("decode", "serving", "splitkv", "prefill", "prefill_fp32", "paged_fp32",
             "prefill_rope")
NOMINAL_HBM_GBS = 8000.0       # B200 HBM3e (DGX figure)
NOMINAL_BF16_TFLOPS = 2250.0   # B200 dense bf16 tensor
BF16_ATOL = 2e-2
FP32_RTOL = 1e-3


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=WORKLOADS, default="decode")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
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
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary
    (profiles/<name>), with its source; (None, None) if there is none."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            d = json.load(f)
        return d.get("dram_bytes_per_launch"), (
            f"profiles/{name}: dram__bytes_read.sum + dram__bytes_write.sum of one ncu "
            f"capture of this kernel on this config (committed; not measured in this run)")
    except Exception:
        return None, None


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def _hbm_roofline(rank_bytes, ms_rank, kernel, traffic_file=None):
    peak, _, _, src = _peaks()
    ach = rank_bytes / (ms_rank * 1e-3) / 1e9
    traffic, tsrc = _traffic(traffic_file) if traffic_file else (None, None)
    r = {"bound": "hbm", "achieved": round(ach, 2), "peak": peak, "unit": "GB/s",
         "frac": round(ach / peak, 4), "peak_source": src,
         "frac_nominal": round(ach / NOMINAL_HBM_GBS, 4),
         "peak_nominal": NOMINAL_HBM_GBS, "kernel": kernel, "traffic": traffic}
    if tsrc:
        r["traffic_source"] = tsrc
    return r


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) every 0.5 ms."""

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
            time.sleep(0.0005)

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


# --------------------------------------------------------------------------- parity
def _parity(err, tol, kind, sample, ws, dev):
    """Worst error over the ranks against the tolerance (kind "abs" or "rel")."""
    e = _max_over_ranks(float(err), ws, dev)
    return {"max_err": float(f"{e:.4g}"), "tol": tol, "kind": kind, "ok": bool(e <= tol),
            "ranks": ws, "sample": sample}


def _err(got, ref, rel):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if not np.isfinite(got).all():
        return float("inf")
    e = float(np.abs(got - ref).max()) if ref.size else 0.0
    if rel:
        e /= float(np.abs(ref).max()) or 1.0
    return e


def _sample_seqs(lens, seed, n=6):
    """Seeded sample of sequence indices, with the longest and the shortest."""
    rng = np.random.default_rng(seed + 12345)
    S = len(lens)
    pick = set(int(x) for x in rng.choice(S, size=min(n, S), replace=False))
    pick.add(int(np.argmax(lens)))
    pick.add(int(np.argmin(lens)))
    return sorted(pick)


def _paged_oracle_rows(q, kc, vc, bt, lens, sel, bs):
    """Oracle rows (the reference's paged_attention per KV-head group) of sequences `sel`:
    their pages are copied to the host as a compact cache and the block table is
    remapped onto it (same gather rule: token t -> block bt[s, t // bs], row t % bs)."""
    import torch
    from oracle import attention_oracle as O
    bt_np = bt[sel].cpu().numpy()
    ls = np.asarray(lens)[sel].astype(np.int32)
    nb = (np.maximum(ls, 0) + bs - 1) // bs
    used = np.concatenate([bt_np[i, :nb[i]] for i in range(len(sel))] + [np.zeros(1, np.int32)])
    blocks = np.unique(used)
    idx = torch.from_numpy(blocks.astype(np.int64)).to(kc.device)
    kc_h = kc.index_select(0, idx).float().cpu().numpy()
    vc_h = vc.index_select(0, idx).float().cpu().numpy()
    bt_sub = np.zeros_like(bt_np)
    for i in range(len(sel)):
        bt_sub[i, :nb[i]] = np.searchsorted(blocks, bt_np[i, :nb[i]])
    q_h = q[sel].float().cpu().numpy()
    return O.paged_attention_gqa(q_h, kc_h, vc_h, bt_sub, ls, bs)


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


def _block_sets(lens, bs, R, seed):
    """R disjoint block tables over a pool of R * sum(ceil(ctx / bs)) blocks."""
    nblk = (lens + bs - 1) // bs
    pool = int(nblk.sum())
    rng = np.random.default_rng(seed + 1)
    perm = rng.permutation(pool * R).astype(np.int32)
    maxb = int(nblk.max())
    bts = []
    for r in range(R):
        bt = np.zeros((len(lens), maxb), np.int32)
        off = r * pool
        for s in range(len(lens)):
            bt[s, :nblk[s]] = perm[off:off + nblk[s]]
            off += nblk[s]
        bts.append(bt)
    return pool, bts


def _e2e_decode(q, kc, vc, bts, lens_t, bs, max_ctx, wsp, R, steps, ws, dev, elt):
    """End to end through the public API with host buffers. Every step moves that step's
    q, block table and context lengths in from pinned host memory as ONE packed copy,
    runs the decode (flash_engine.paged_attention) and copies its output back to pinned
    host memory. Steps are pipelined over three device buffer sets: the CUDA graph of
    step k runs the decode of step k and, on two forked streams, the input copy of step
    k+1 and the output copy of step k-1 (as a serving loop overlaps its transfers with
    the running step); the host replays one graph per step and waits for the graph of
    step k-2 before it replays step k. The timed region includes the first step's input
    copy and the last step's output copy. Also returned: the same three operations
    issued eagerly from Python, one step at a time (no overlap).
    Returns (pipelined_ms, eager_ms, h2d_bytes, d2h_bytes) per step on this rank."""
    import torch
    import flash_engine

    S = q.shape[0]
    nq = q.numel() * q.element_size()
    nbt = bts[0].numel() * 4
    nl = S * 4

    def al(x):
        return (x + 255) // 256 * 256
    o_bt, o_l = al(nq), al(nq) + al(nbt)
    total = o_l + al(nl)
    stage_h = []
    for r in range(R):
        h = torch.zeros(total, dtype=torch.uint8).pin_memory()
        h[:nq].copy_(q.detach().cpu().contiguous().view(-1).view(torch.uint8))
        h[o_bt:o_bt + nbt].copy_(bts[r].cpu().contiguous().view(-1).view(torch.uint8))
        h[o_l:o_l + nl].copy_(lens_t.cpu().contiguous().view(torch.uint8))
        stage_h.append(h)
    NB = 3
    in_d = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(NB)]
    views = [(sd[:nq].view(q.dtype).view(q.shape), sd[o_bt:o_bt + nbt].view(torch.int32)
              .view(bts[0].shape), sd[o_l:o_l + nl].view(torch.int32)) for sd in in_d]
    out_d = [torch.empty_like(q) for _ in range(NB)]
    out_h = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(NB)]
    evs = [torch.cuda.Event() for _ in range(NB)]

    def decode(b):
        qv, btv, lv = views[b]
        flash_engine.paged_attention(qv, kc, vc, btv, lv, bs, max_context_len=max_ctx,
                                     out=out_d[b], workspace=wsp)

    # one graph per (buffer set of step k, block set of step k+1)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    for b in range(NB):
        in_d[b].copy_(stage_h[0])
        decode(b)
    torch.cuda.synchronize()
    graphs = {}
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        for b in range(NB):
            for rn in range(R):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=cap):
                    s_in.wait_stream(cap)
                    s_out.wait_stream(cap)
                    with torch.cuda.stream(s_in):
                        in_d[(b + 1) % NB].copy_(stage_h[rn], non_blocking=True)
                    with torch.cuda.stream(s_out):
                        out_h[(b - 1) % NB].copy_(out_d[(b - 1) % NB], non_blocking=True)
                    decode(b)
                    cap.wait_stream(s_in)
                    cap.wait_stream(s_out)
                graphs[(b, rn)] = g
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()

    def pipelined(n):
        in_d[0].copy_(stage_h[0], non_blocking=True)
        for k in range(n):
            b = k % NB
            if k >= 2:
                evs[(k - 2) % NB].synchronize()
            graphs[(b, (k + 1) % R)].replay()
            evs[b].record()
        lb = (n - 1) % NB
        out_h[lb].copy_(out_d[lb], non_blocking=True)
        torch.cuda.synchronize()

    def eager(n):
        for k in range(n):
            b = k % NB
            in_d[b].copy_(stage_h[k % R], non_blocking=True)
            decode(b)
            out_h[b].copy_(out_d[b], non_blocking=True)
            evs[b].record()
            evs[b].synchronize()

    n = max(4, min(steps, 200))
    res = []
    for fn in (pipelined, eager):
        fn(4)
        _barrier(ws, dev)
        t0 = time.perf_counter()
        fn(n)
        res.append(_max_over_ranks((time.perf_counter() - t0) * 1e3 / n, ws, dev))
    # the outputs that came back are the decode's
    for b in range(NB):
        assert torch.equal(out_h[b].to(dev), out_d[b])
    del graphs
    return res[0], res[1], nq + nbt + nl, nq


def bench_paged(a, ws, rank, local, cfg, steps, warmup, fp32=False):
    """Config 3 / config 5 paged decode (bf16), or the reference's fp32 paged entry on
    config 3's shapes with an fp32 cache (``fp32``)."""
    import torch
    import flash_engine

    dev = torch.device("cuda", local)
    S, H, Hkv, d, bs = (cfg[k] for k in ("num_seqs", "num_heads", "num_kv_heads", "head_dim",
                                         "block_size"))
    if Hkv % ws:
        raise ValueError(f"{ws} ranks cannot split {Hkv} KV heads")
    hkv_l, h_l = Hkv // ws, H // ws
    lens = _lens(cfg, a.seed)
    if fp32 and a.num_seqs > 0:
        lens = lens[:a.num_seqs]
    S = len(lens)
    elt = 4 if fp32 else 2
    dt = torch.float32 if fp32 else torch.bfloat16
    nblk = (lens + bs - 1) // bs
    pool1 = int(nblk.sum())
    # Disjoint block sets used in turn: >= 4 x L2 (2 x L2 for fp32) of distinct KV over a
    # cycle, so no step finds its KV in L2.
    kv_set = pool1 * hkv_l * bs * d * elt * 2
    R = max(1, math.ceil((2 if fp32 else 4) * L2_BYTES / kv_set))
    pool, bts_np = _block_sets(lens, bs, R, a.seed)
    bts = [torch.from_numpy(b).to(dev) for b in bts_np]
    g = torch.Generator(device=dev)
    g.manual_seed((3000 if fp32 else 1000) + a.seed * 17 + rank)
    kc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev).to(dt)
    vc = torch.randn((pool * R, hkv_l, bs, d), generator=g, device=dev).to(dt)
    q = torch.randn((S, h_l, d), generator=g, device=dev).to(dt)
    lens_t = torch.from_numpy(lens).to(dev)
    out = torch.empty_like(q)
    max_ctx = int(lens.max())
    wsp = torch.zeros(flash_engine.paged_attention_workspace_floats(h_l, hkv_l, d, bs),
                      dtype=torch.float32, device=dev)

    def call(i, o=out):
        flash_engine.paged_attention(q, kc, vc, bts[i % R], lens_t, bs, max_context_len=max_ctx,
                                     out=o, workspace=wsp)

    # A decode step is one call of the public API. The calls are captured GSTEPS at a
    # time into CUDA graphs (one per starting block set) and replayed back to back, as a
    # serving loop replays its captured decode steps. The decode kernel is launched with
    # programmatic dependent launch, so inside a graph each call's CTAs are placed as
    # the previous call's CTAs retire (they wait for its results before reading
    # anything).
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
    del graphs
    ms = _max_over_ranks(ms_rank, ws, dev)
    total = decode_bytes(lens, Hkv, H, d, bs, elt)
    rank_bytes = decode_bytes(lens, hkv_l, h_l, d, bs, elt)

    gms, ems, h2d, d2h = _e2e_decode(q, kc, vc, bts, lens_t, bs, max_ctx, wsp, R, steps, ws,
                                     dev, elt)
    parity = None
    if not a.no_parity:
        call(0)
        torch.cuda.synchronize()
        sel = _sample_seqs(lens, a.seed)
        ref = _paged_oracle_rows(q, kc, vc, bts[0], lens, sel, bs)
        err = _err(out[sel].float().cpu().numpy(), ref, rel=fp32)
        parity = _parity(err, FP32_RTOL if fp32 else BF16_ATOL, "rel" if fp32 else "abs",
                         f"{len(sel)} sequences (seeded, incl. longest and shortest), all "
                         f"{h_l} query heads of each rank, vs the CPU oracle", ws, dev)
    if fp32:
        metric = "paged decode fp32 KV GB/s (the reference's v1 fp32 entry on config 3 shapes)"
        name = "paged_decode_fp32_config3"
        kernel = "paged_decode_kernel<float> (fp32 CUDA-core consumer, merge fused)"
        tfile = "paged_decode_fp32_config3_traffic.json" if ws == 1 else None
    else:
        metric, name = cfg["metric"], cfg["name"]
        kernel = "paged_decode_kernel (merge fused)"
        tfile = ({"paged_decode_config3": "paged_decode_config3_traffic.json",
                  "paged_decode_config5_serving": "paged_decode_config5_traffic.json"}[name]
                 if ws == 1 else None)
    res = {
        "metric": metric, "value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(ms, 5),
        "config": {"workload": name, "num_seqs": S, "num_heads": H, "num_kv_heads": Hkv,
                   "head_dim": d, "block_size": bs, "total_context_tokens": int(lens.sum()),
                   "bytes_per_step": total, "workspace_floats": int(wsp.numel()),
                   "parallelism": f"kv-head shard x{ws}",
                   "l2": f"{R} disjoint block sets rotated per step "
                         f"({R * kv_set / 2**20:.0f} MiB per rank)"},
        "roofline": _hbm_roofline(rank_bytes, ms_rank, kernel, tfile),
        "e2e": {"value": round(total / (gms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(gms, 4), "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "mode": "per step: one packed H2D copy of q, block table and lengths from "
                        "pinned memory, the public paged_attention call, one D2H copy of "
                        "the output; one CUDA graph per step (decode of step k, input copy "
                        "of step k+1 and output copy of step k-1 on forked streams), "
                        "replayed by the host every step",
                "eager_value": round(total / (ems * 1e-3) / 1e9, 2),
                "eager_ms_per_step": round(ems, 4),
                "eager_mode": "the same three operations issued from Python, one step at a "
                              "time"},
        "gpu_launches": steps,
        "clocks": sampler.summary(t0, t1),
    }
    if parity:
        res["parity"] = parity
    return res


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
    # with the peer-memory exchange: replaying its two launches as a graph measured slower
    # at N = 8 (88 vs 70 us a step), so they are issued directly, through the exchange's
    # prepared step (arguments checked and converted once; issuing through the checking
    # wrapper cost as much host time as the step's GPU work at N = 8).
    from flash_engine.graph import DecodeGraph
    graph = DecodeGraph(lambda: call(0)) if ex is None else None
    fast = ex.prepare(q_all, kc, vc, bt_t, lens_t, M, bs, workspace=wsp) if ex is not None else None

    def step(i):
        if graph is not None:
            graph.replay()
        elif fast is not None:
            fast()
        else:
            call(i)

    sampler = ClockSampler(local).start()
    ms_rank, t0, t1 = _time_steps(step, steps, warmup, ws, dev)
    sampler.stop()
    assert flash_engine.device_errors() == 0
    ms = _max_over_ranks(ms_rank, ws, dev)
    kv_total = B * M * Hkv * d * 2 * 2
    kv_rank = B * (te - tb) * Hkv * d * 2 * 2
    # end to end: q, block table and lengths from pinned host as one packed copy, the
    # output back to pinned host, every step, on the step's stream. Two buffer sets: the
    # host issues step k once step k - 2 (the last user of its buffers) has completed,
    # so it issues a step while the previous one runs instead of after a synchronize.
    nq, nbt, nl = q_all.numel() * 2, bt_t.numel() * 4, B * 4
    stage_h = torch.zeros(nq + nbt + nl, dtype=torch.uint8).pin_memory()
    stage_h[:nq].copy_(q_all.cpu().view(-1).view(torch.uint8))
    stage_h[nq:nq + nbt].copy_(bt_t.cpu().view(-1).view(torch.uint8))
    stage_h[nq + nbt:].copy_(lens_t.cpu().view(torch.uint8))
    NB = 2
    stage_d = [torch.empty_like(stage_h, device=dev) for _ in range(NB)]
    views = [(sd[:nq].view(torch.bfloat16).view(q_all.shape),
              sd[nq:nq + nbt].view(torch.int32).view(bt_t.shape),
              sd[nq + nbt:].view(torch.int32)) for sd in stage_d]
    out_h = [torch.empty(q_all.shape, dtype=q_all.dtype).pin_memory() for _ in range(NB)]
    done = [torch.cuda.Event() for _ in range(NB)]
    # with the peer-memory exchange, prepared steps bound to the staged tensors
    fast_e2e = ([ex.prepare(qv, kc, vc, bv, lv, M, bs, workspace=wsp) for qv, bv, lv in views]
                if ex is not None else None)

    def e2e(i):
        b = i % NB
        done[b].synchronize()  # step i - NB: its output has reached the host
        stage_d[b].copy_(stage_h, non_blocking=True)
        out_h[b].copy_(fast_e2e[b]() if fast_e2e is not None else call(i, *views[b]),
                       non_blocking=True)
        done[b].record()

    for i in range(3):
        e2e(i)
    torch.cuda.current_stream().synchronize()
    _barrier(ws, dev)
    n = max(1, min(steps, 100))
    te0 = time.perf_counter()
    for i in range(n):
        e2e(i)
    torch.cuda.current_stream().synchronize()
    e2e_ms = _max_over_ranks((time.perf_counter() - te0) * 1e3 / n, ws, dev)

    parity = None
    if not a.no_parity:
        out = call(0)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        parity = _splitkv_parity(q_all, kc, vc, bt, tb, te, M, bs, got, ws, dev)
    del graph
    if ex is not None:
        ex.close()
    res = {
        "metric": c["metric"], "value": round(kv_total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(ms, 5),
        "config": {"workload": c["name"], "batch": B, "num_heads": H, "num_kv_heads": Hkv,
                   "head_dim": d, "context": M, "block_size": bs,
                   "parallelism": f"kv-range shard x{ws} + all-gather of (O,m,l) partials"
                                  + ("" if ws == 1 else
                                     " by the decode kernel's peer stores" if ex is not None
                                     else " by NCCL"),
                   "l2": f"{kv_rank / 2**20:.0f} MiB of KV per rank"},
        "roofline": _hbm_roofline(kv_rank, ms_rank, "paged_decode_kernel (partials / exchange "
                                  "mode) + merge" if ws > 1 else "paged_decode_kernel (merge "
                                  "fused)", "splitkv_decode_config4_traffic.json"
                                  if ws == 1 else None),
        "e2e": {"value": round(kv_total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": int(nq + nbt + nl),
                "d2h_bytes_per_step": int(out_h[0].numel() * 2),
                "mode": "per step one packed H2D copy, the step and one D2H copy on the step's "
                        "stream; two buffer sets, the host issues step k once step k - 2 "
                        "has completed"},
        "gpu_launches": steps * (1 if ws == 1 else 2),
        "clocks": sampler.summary(t0, t1),
    }
    if parity:
        res["parity"] = parity
    return res


def _splitkv_parity(q_all, kc, vc, bt, tb, te, M, bs, got, ws, dev):
    """Each rank computes the oracle's split-KV stage 1 (ops.py:117-131) over its own
    token window for two sequences and the query heads of two KV heads (the first and
    the last), the partials of all ranks are gathered and merged with the oracle's
    log-sum-exp combine (ops.py:133-143), and every rank compares the result with its
    output rows."""
    import torch
    from oracle import attention_oracle as O
    sel = [0, q_all.shape[0] - 1]
    H, d = q_all.shape[1], q_all.shape[2]
    Hkv = kc.shape[1]
    G = H // Hkv
    kvs = [0, Hkv - 1]
    heads = [g * G + j for g in kvs for j in range(G)]
    nb0, nb1 = tb // bs, (te + bs - 1) // bs
    if te > tb:
        blocks = np.unique(bt[sel, nb0:nb1])
        idx = torch.from_numpy(blocks.astype(np.int64)).to(kc.device)
        kh = torch.tensor(kvs, device=kc.device)
        kc_h = kc.index_select(0, idx).index_select(1, kh).float().cpu().numpy()
        vc_h = vc.index_select(0, idx).index_select(1, kh).float().cpu().numpy()
        bt_sub = np.zeros((len(sel), bt.shape[1]), np.int32)
        bt_sub[:, nb0:nb1] = np.searchsorted(blocks, bt[sel, nb0:nb1])
        qs = q_all[sel][:, heads].float().cpu().numpy()
        Op, mp, lp = O.kv_range_partials(qs, kc_h, vc_h, bt_sub,
                                         np.full(len(sel), M, np.int32), tb, te, bs)
    else:
        Op, mp, lp = (np.zeros((len(sel), len(heads), d)), np.full((len(sel), len(heads)),
                      -np.inf), np.zeros((len(sel), len(heads))))
    parts = [(Op, mp, lp)]
    if ws > 1:
        import torch.distributed as dist
        parts = [None] * ws
        dist.all_gather_object(parts, (Op, mp, lp))
    ref = O.lse_merge([p[0] for p in parts], [p[1] for p in parts], [p[2] for p in parts])
    err = _err(got[sel][:, heads], ref, rel=False)
    return _parity(err, BF16_ATOL, "abs",
                   f"sequences {sel}, the {len(heads)} query heads of KV heads {kvs}: "
                   f"per-rank oracle partials over each rank's window, gathered and merged "
                   f"by the oracle's LSE combine", ws, dev)


# --------------------------------------------------------------------------- prefill
def prefill_flops(B, H, N, d, causal=True):
    """4*B*H*N^2*d, halved for causal (the reference's convention,
    benchmarks/bench_attention.cu:48-49)."""
    f = 4.0 * B * H * N * N * d
    return f / 2 if causal else f


def bench_prefill(a, ws, rank, local, steps, warmup, fp32=False, rope=False):
    """Config 1 (fp32) or config 2 (bf16); with rope, config 2 with Q and K rotated
    (the RoPE pass for both, then the attention) inside every step."""
    import torch
    import flash_engine

    dev = torch.device("cuda", local)
    if fp32:   # config 1: fp32, non-causal, [1, 8, 512, 64]
        B, H, N, d, causal, dt = 1, 8, 512, 64, False, torch.float32
        name = "fa2_prefill_fp32_config1"
        metric = "FA2 forward fp32 TFLOP/s (config 1: [1, 8, 512, 64], non-causal)"
    elif rope:
        B, H, N, d, causal, dt = 4, 32, 4096, 128, True, torch.bfloat16
        name = "fa2_prefill_rope_config2"
        metric = ("FA2 prefill with RoPE on Q and K, attention TFLOP/s (config 2: bf16 causal "
                  "[4, 32, 4096, 128])")
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
    tabs, krot = None, None
    if rope:
        # cos / sin [N, d/2] of angle p * 10000^(-2i/d), made on the device
        inv = 10000.0 ** (-2.0 * torch.arange(d // 2, dtype=torch.float64, device=dev) / d)
        ang = torch.arange(N, dtype=torch.float64, device=dev)[:, None] * inv[None, :]
        tabs = (torch.cos(ang).float().contiguous(), torch.sin(ang).float().contiguous())
        krot = [torch.empty_like(sets[0][1]) for _ in range(nsets)]

    def call(i):
        qq, kk, vv = sets[i % nsets]
        if rope:
            return flash_engine.flash_attention(qq, kk, vv, causal, out=outs[i % nsets],
                                                rope=tabs, k_rotated=krot[i % nsets])
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

    # End to end through the public API: Q, K, V from pinned host memory (one packed
    # copy) and O back, every step. Two buffer sets and three streams: the input copy
    # of step k runs on its own stream, the call on the current one once that copy is in,
    # and the output copy on a third once the call is done; the host issues step k once
    # step k - 2 has reached the host, so step k's input copy overlaps the output copy
    # of step k - 1 (the host link carries both directions at once) and the calls.
    elt = 4 if fp32 else 2
    nb = q.numel() * elt
    stage_h = torch.empty(3 * nb, dtype=torch.uint8).pin_memory()
    for j, x in enumerate((q, k, v)):
        stage_h[j * nb:(j + 1) * nb].copy_(x.cpu().view(-1).view(torch.uint8))
    NB = 2
    stage_d = [torch.empty_like(stage_h, device=dev) for _ in range(NB)]
    views = [tuple(sd[j * nb:(j + 1) * nb].view(dt).view(q.shape) for j in range(3))
             for sd in stage_d]
    o_d = [torch.empty_like(q) for _ in range(NB)]
    o_h = [torch.empty(q.shape, dtype=dt).pin_memory() for _ in range(NB)]
    main = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in, ev_call, done = ([torch.cuda.Event() for _ in range(NB)] for _ in range(3))

    def e2e_step(i):
        b = i % NB
        done[b].synchronize()  # step i - 2 is on the host: buffer set b is free
        with torch.cuda.stream(s_in):
            stage_d[b].copy_(stage_h, non_blocking=True)
            ev_in[b].record(s_in)
        main.wait_event(ev_in[b])
        qd, kd, vd = views[b]
        if rope:
            flash_engine.flash_attention(qd, kd, vd, causal, out=o_d[b], rope=tabs)
        else:
            flash_engine.flash_attention(qd, kd, vd, causal, out=o_d[b])
        ev_call[b].record(main)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_call[b])
            o_h[b].copy_(o_d[b], non_blocking=True)
            done[b].record(s_out)

    def e2e_drain():
        for st in (s_in, main, s_out):
            st.synchronize()

    e2e_step(0)
    e2e_drain()
    _barrier(ws, dev)
    n_e2e = max(1, min(steps, 5 if not fp32 else 100))
    te0 = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    e2e_drain()
    e2e_ms = _max_over_ranks((time.perf_counter() - te0) * 1e3 / n_e2e, ws, dev)
    assert torch.equal(o_h[(n_e2e - 1) % NB].to(dev), o_d[(n_e2e - 1) % NB])

    parity = None
    if not a.no_parity:
        from oracle import attention_oracle as O
        o = call(0)
        torch.cuda.synchronize()
        if fp32:
            ref = O.flash_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), causal)
            err = _err(o.cpu().numpy(), ref, rel=True)
            smp = f"all {h_l} heads of each rank"
        else:
            rng = np.random.default_rng(a.seed + 99 + rank)
            pairs = [(int(rng.integers(B)), int(rng.integers(h_l))) for _ in range(2)]
            err = 0.0
            for b, h in pairs:
                sl = (slice(b, b + 1), slice(h, h + 1))
                qs, ks = q[sl].float().cpu().numpy(), k[sl].float().cpu().numpy()
                if rope:
                    cs, sn = (t.cpu().numpy() for t in tabs)
                    qs = O.bf16_round(O.rope_rotate(qs, cs, sn, np.arange(N)).astype(np.float32))
                    ks = O.bf16_round(O.rope_rotate(ks, cs, sn, np.arange(N)).astype(np.float32))
                ref = O.flash_attention(qs, ks, v[sl].float().cpu().numpy(), causal)
                err = max(err, _err(o[sl].float().cpu().numpy(), ref, rel=False))
            smp = "2 seeded (batch, head) slices of each rank, all 4096 rows"
            if rope:
                smp += ", Q and K rotated by the oracle's RoPE"
        parity = _parity(err, FP32_RTOL if fp32 else BF16_ATOL, "rel" if fp32 else "abs",
                         smp + ", vs the CPU oracle", ws, dev)

    _, peak, peak_sus, src = _peaks()
    # fp32 runs on the tensor core as 3xTF32 (three TF32 products per fp32 product, TF32 at
    # half the bf16 rate): its ceiling in fp32 FLOP/s is the bf16 peak / 6.
    pk, pk_sus, pk_nom = ((peak / 6, peak_sus / 6, NOMINAL_BF16_TFLOPS / 6) if fp32
                          else (peak, peak_sus, NOMINAL_BF16_TFLOPS))
    tfile = None if fp32 or rope or ws > 1 else "fa_prefill_config2_traffic.json"
    traffic, tsrc = _traffic(tfile) if tfile else (None, None)
    roof = {"bound": "tensor", "achieved": round(achieved, 3), "peak": round(pk, 1),
            "unit": "TFLOP/s", "frac": round(achieved / pk, 4),
            "frac_of_sustained": round(achieved / pk_sus, 4),
            "frac_nominal": round(achieved / pk_nom, 4), "peak_nominal": round(pk_nom, 1),
            "peak_source": src + (" bf16 burst / 6: TF32 runs at half the bf16 rate "
                                  "and each fp32 product takes 3 TF32 products"
                                  if fp32 else " bf16 burst"),
            "kernel": ("fa_tf32_kernel (3xTF32 tcgen05)" if fp32 else
                       "rope_row_kernel + fa_prefill_kernel (step time; FLOPs of the attention)"
                       if rope else "fa_prefill_kernel"),
            "traffic": traffic}
    if tsrc:
        roof["traffic_source"] = tsrc
    res = {
        "metric": metric, "value": round(total / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
        "ms_per_step": round(ms, 4),
        "e2e": {"value": round(total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": int(3 * nb), "d2h_bytes_per_step": int(nb),
                "mode": "per step one packed H2D copy of Q, K, V, the call and one D2H copy "
                        "of O, each on its own stream; two buffer sets, the host issues step "
                        "k once step k - 2 is on the host"},
        "config": {"workload": name, "batch": B, "heads": H, "seq_len": N, "head_dim": d,
                   "causal": causal, "parallelism": f"head shard x{ws}",
                   "flops_per_step": total,
                   "l2": f"{nsets} input set(s) of {set_bytes / 2**20:.0f} MiB used in turn",
                   "steps_per_graph": GSTEPS},
        "roofline": roof,
        "clocks": sampler.summary(t0, t1),
        "gpu_launches": steps * (2 if rope else 1),
    }
    if parity:
        res["parity"] = parity
    return res


# --------------------------------------------------------------------------- CPU baselines
def cpu_baseline(name, a, budget_s):
    """The reference's CPU implementation of the workload (the NumPy port in oracle/),
    timed on this host's cores over a bounded sample; returns the cpu_baseline object."""
    from oracle import attention_oracle as O
    if name in ("decode", "serving", "paged_fp32"):
        cfg = CFG5 if name == "serving" else CFG3
        lens = _lens(cfg, a.seed)
        H, Hkv, d, bs = cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"], cfg["block_size"]
        elt = 4 if name == "paged_fp32" else 2
        p1 = O.make_paged_problem(a.seed, 1, H, Hkv, d, lens[:1], bf16=elt == 2)
        t = time.perf_counter()
        O.paged_attention_gqa(p1["q"], p1["k_cache"], p1["v_cache"], p1["block_tables"],
                              p1["context_lens"])
        per_tok = (time.perf_counter() - t) / max(1, int(lens[0]))
        n = 1
        while n < len(lens) and per_tok * int(lens[:n + 1].sum()) < budget_s:
            n += 1
        sub = lens[:n]
        p = O.make_paged_problem(a.seed, n, H, Hkv, d, sub, bf16=elt == 2)
        t = time.perf_counter()
        O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                              p["context_lens"])
        dt = time.perf_counter() - t
        b = decode_bytes(sub, Hkv, H, d, bs, elt)
        return {"value": round(b / dt / 1e9, 4), "unit": "GB/s", "cores": _cpu_threads(),
                "kind": "port",
                "sample": f"first {n} of {len(lens)} sequences of {cfg['name']} "
                          f"({int(sub.sum())} tokens), {dt:.2f} s; bytes counted as "
                          f"{'fp32' if elt == 4 else 'bf16'}"}
    if name == "splitkv":
        c = CFG4
        H, Hkv, d, bs, M = (c[k] for k in ("num_heads", "num_kv_heads", "head_dim",
                                           "block_size", "context"))
        # one sequence, KV heads taken one at a time until the budget is spent
        tok = M
        p = O.make_paged_problem(a.seed, 1, H // Hkv, 1, d, [tok])
        t = time.perf_counter()
        done = 0
        while True:
            O.paged_flash_decoding_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                       p["context_lens"], 1, bs)
            done += 1
            if time.perf_counter() - t > budget_s / 2 or done >= 4:
                break
        dt = (time.perf_counter() - t) / done
        b = tok * d * 2 * 2
        return {"value": round(b / dt / 1e9, 4), "unit": "GB/s", "cores": _cpu_threads(),
                "kind": "port",
                "sample": f"one (sequence, KV head) of config 4 ({tok} tokens, {H // Hkv} query "
                          f"heads) per pass, {done} passes of {dt:.2f} s; bytes counted as bf16"}
    if name in ("prefill", "prefill_fp32", "prefill_rope"):
        fp32 = name == "prefill_fp32"
        rope = name == "prefill_rope"
        B, H, N, d, causal = (1, 8, 512, 64, False) if fp32 else (4, 32, 4096, 128, True)
        rng = np.random.default_rng(a.seed)
        q, k, v = (rng.standard_normal((1, 1, N, d), dtype=np.float32) for _ in range(3))
        cs, sn = O.rope_tables(N, d) if rope else (None, None)
        t = time.perf_counter()
        done = 0
        while True:
            if rope:  # the reference's fused RoPE on Q and K, then the attention
                pos = np.arange(N)
                O.flash_attention(O.rope_rotate(q, cs, sn, pos), O.rope_rotate(k, cs, sn, pos),
                                  v, causal)
            else:
                O.flash_attention(q, k, v, causal)
            done += 1
            if time.perf_counter() - t > budget_s or done >= (8 if fp32 else 4):
                break
        dt = (time.perf_counter() - t) / done
        f = prefill_flops(1, 1, N, d, causal)
        return {"value": round(f / dt / 1e12, 6), "unit": "TFLOP/s", "cores": _cpu_threads(),
                "kind": "port",
                "sample": f"one (batch, head) slice [{N}, {d}] of the config per pass"
                          f"{' (RoPE of Q and K included)' if rope else ''} "
                          f"({done} passes of {dt * 1e3:.1f} ms), FLOPs counted as on the GPU"}
    raise ValueError(name)


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
        return bench_paged(a, ws, rank, local, CFG3, steps, warmup)
    if name == "serving":
        return bench_paged(a, ws, rank, local, CFG5, steps, warmup)
    if name == "paged_fp32":
        return bench_paged(a, ws, rank, local, CFG3, steps, warmup, fp32=True)
    if name == "splitkv":
        return bench_splitkv(a, ws, rank, local, steps, warmup)
    if name == "prefill":
        return bench_prefill(a, ws, rank, local, steps, warmup)
    if name == "prefill_rope":
        return bench_prefill(a, ws, rank, local, steps, warmup, rope=True)
    return bench_prefill(a, ws, rank, local, steps, warmup, fp32=True)


def _common(res, a, ws, name):
    # every config keeps its total work fixed as N grows (heads or the KV range are
    # divided over the ranks): strong scaling
    res.update({"n_gpus": ws, "steps": a.steps, "warmup": a.warmup, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "f32" if name in ("prefill_fp32", "paged_fp32") else "bf16",
                "data": "synthetic (seeded N(0,1) inputs; benchmark config shapes)"})
    return res


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
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    head = _common(run_workload(a.workload, a, ws, rank, local, True), a, ws, a.workload)
    lines = []
    if not a.no_secondary:
        for name in ("prefill", "splitkv", "serving", "prefill_fp32", "paged_fp32", "decode"):
            if name == a.workload:
                continue
            try:
                r = _common(run_workload(name, a, ws, rank, local, False), a, ws, name)
                r["secondary"] = True
                r["steps"] = min(a.steps, 30)
                r["warmup"] = min(a.warmup, 3)
            except Exception as e:  # recorded, never silently dropped
                r = {"workload": name, "secondary": True, "error": f"{type(e).__name__}: {e}"}
                if rank == 0:
                    traceback.print_exc()
            lines.append((name, r))
    # CPU baselines (the reference's NumPy path on the host cores), rank 0 at N = 1,
    # after all GPU timing
    if ws == 1 and rank == 0 and not a.no_cpu_baseline:
        for name, r in [(a.workload, head)] + lines:
            if "error" in r:
                continue
            try:
                r["cpu_baseline"] = cpu_baseline(name, a, 12.0 if r is head else 4.0)
            except Exception as e:
                r["cpu_baseline"] = {"error": f"{type(e).__name__}: {e}"}
    if ws > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        for _, r in lines:
            print(json.dumps(r), flush=True)
        print(json.dumps(head), flush=True)


if __name__ == "__main__":
    main()
