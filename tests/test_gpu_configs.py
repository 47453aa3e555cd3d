"""Parity at the benchmark configurations' full shapes (4, 5).

The caches are drawn on the GPU (seeded torch generator, bf16 or fp32) and copied to
the host once; the oracle is the NumPy restatement of the reference's
paged_attention (python/flash_engine/ops.py:59-101, per KV-head group for GQA) and of
its split-KV stage 1 + log-sum-exp merge (ops.py:103-143) for the KV-range shards.
Tolerances: 2e-2 absolute for bf16, 1e-3 relative (max |err| / max |ref|) for fp32.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, assert_fp32_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _problem(seed, lens, H, Hkv, d, bs=16, dtype=torch.bfloat16):
    """Paged problem with the cache drawn on the GPU: block tables are a seeded random
    permutation of a pool sized to the total, as in the benchmark configs."""
    lens = np.asarray(lens, dtype=np.int32)
    nblk = (lens + bs - 1) // bs
    pool = int(nblk.sum())
    rng = np.random.default_rng(seed)
    perm = rng.permutation(pool).astype(np.int32)
    maxb = int(nblk.max())
    bt = np.zeros((len(lens), maxb), np.int32)
    off = 0
    for s, n in enumerate(nblk):
        bt[s, :n] = perm[off:off + n]
        off += n
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    kc = torch.randn((pool, Hkv, bs, d), generator=g, device="cuda").to(dtype)
    vc = torch.randn((pool, Hkv, bs, d), generator=g, device="cuda").to(dtype)
    q = torch.randn((len(lens), H, d), generator=g, device="cuda").to(dtype)
    return dict(q=q, kc=kc, vc=vc, bt=bt, lens=lens, bt_d=cuda(bt), lens_d=cuda(lens),
                H=H, Hkv=Hkv, d=d, bs=bs)


def _oracle(p, sel=None):
    """Oracle rows of the sequences in `sel` (all by default)."""
    sel = np.arange(len(p["lens"])) if sel is None else np.asarray(sel)
    kc = host(p["kc"])
    vc = host(p["vc"])
    return O.paged_attention_gqa(host(p["q"])[sel], kc, vc, p["bt"][sel], p["lens"][sel],
                                 p["bs"])


# --------------------------------------------------------------------------- config 4
C4 = dict(B=4, H=32, Hkv=8, d=128, ctx=131072)


@pytest.fixture(scope="module")
def config4():
    p = _problem(404, [C4["ctx"]] * C4["B"], C4["H"], C4["Hkv"], C4["d"])
    p["ref"] = _oracle(p)
    return p


def test_config4_full_shape_single_gpu(config4):
    """Benchmark config 4 at its real shape (B4, 32q/8kv, d128, 131072-token contexts,
    8192 blocks a sequence, a permuted pool of 32768 blocks) through the split-KV
    decode on one GPU: every (sequence, head) row against the oracle."""
    import flash_engine
    p = config4
    for version in ("v2", "v1"):
        out = flash_engine.paged_attention(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"], 16,
                                           max_context_len=C4["ctx"], version=version)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out), p["ref"])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config4_kv_range_partials_merge(config4, world):
    """Config 4's KV-range sharding emulated on one GPU: rank r decodes its token
    window (the ceil(M / world) rule of ops.py:112-121, rounded to whole blocks), the
    world partials are stacked as the all-gather would and merged by log-sum-exp."""
    import flash_engine
    from flash_engine import sharding
    p = config4
    outs, stats = [], []
    for r in range(world):
        tb, te = sharding.kv_range_bounds(C4["ctx"], world, r, 16)
        o, s = flash_engine.paged_decode_partials(p["q"], p["kc"], p["vc"], p["bt_d"],
                                                  p["lens_d"], tb, te)
        outs.append(o)
        stats.append(s)
    final = flash_engine.merge_partials(torch.stack(outs), torch.stack(stats), world, 1, "bf16")
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(final).reshape(p["ref"].shape), p["ref"])


@pytest.mark.parametrize("world", [2, 8])
def test_config4_kv_exchange_emulated(config4, world):
    """The fused KV-range step (the decode kernel stores its partials into every rank's
    exchange buffer, the merge kernel combines them) with `world` ranks emulated on one
    GPU over config 4's full cache: phase 1 of every rank, then phase 2 of every rank,
    for two steps (both slot generations)."""
    import ctypes
    import flash_engine
    from flash_engine import _lib, ops, sharding
    p = config4
    S, H, d = C4["B"], C4["H"], C4["d"]
    L = _lib.lib
    nbytes = L.fe_kv_exchange_bytes(world, S * H, d)
    bufs = []
    for _ in range(world):
        b = ctypes.c_void_p()
        assert L.fe_kv_exchange_alloc(nbytes, ctypes.byref(b)) == 0
        bufs.append(b.value)
    wss = [torch.zeros(flash_engine.paged_attention_workspace_floats(H, C4["Hkv"], d),
                       dtype=torch.float32, device="cuda") for _ in range(world)]
    try:
        for _step in range(2):
            outs = [torch.full_like(p["q"], float("nan")) for _ in range(world)]
            for r in range(world):
                tb, te = sharding.kv_range_bounds(C4["ctx"], world, r, 16)
                ops.paged_decode_kv_exchange(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"],
                                             tb, te, bufs, r, S * H, workspace=wss[r],
                                             out=outs[r], phases=1)
            for r in range(world):
                ops.paged_decode_kv_exchange(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"],
                                             0, 0, bufs, r, S * H, workspace=wss[r],
                                             out=outs[r], phases=2)
            torch.cuda.synchronize()
            assert flash_engine.device_errors() == 0
            for r in range(world):
                assert_bf16_close(host(outs[r]), p["ref"])
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            L.fe_kv_exchange_free(b)


# --------------------------------------------------------------------------- config 5
def test_config5_full_batch():
    """Benchmark config 5 at its real shape: 256 sequences, 64q/8kv, d128, lognormal
    context lengths (median 1024, sigma 1, clipped to [16, 32768], seed 0); every row
    of the split-KV (v2) and single-pass (v1) decode against the oracle."""
    import flash_engine
    lens = O.config5_context_lens(0)
    p = _problem(505, lens, 64, 8, 128)
    ref = _oracle(p)
    for version in ("v2", "v1"):
        out = flash_engine.paged_attention(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"], 16,
                                           version=version)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out), ref)


# --------------------------------------------------------------------------- config 3 fp32
def test_config3_full_batch_fp32():
    """The reference's fp32 paged entry on benchmark config 3's full shape (64
    sequences, 32q/8kv, d128, ctx U[512, 4096]) with an fp32 cache: the persistent
    split-KV decode with CUDA-core fp32 arithmetic, every row within 1e-3 relative."""
    import flash_engine
    lens = O.config3_context_lens(0)
    p = _problem(303, lens, 32, 8, 128, dtype=torch.float32)
    ref = _oracle(p)
    for version in ("v2", "v1"):
        out = flash_engine.paged_attention(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"], 16,
                                           version=version)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_fp32_close(host(out), ref)


@pytest.mark.parametrize("H,Hkv,d,bs", [(64, 8, 128, 16), (8, 8, 64, 32), (16, 1, 128, 32),
                                        (6, 3, 64, 16)])
def test_fp32_persistent_decode_shapes(H, Hkv, d, bs):
    """The fp32 persistent decode over its head-group widths (4 or 8 query heads a CTA,
    padded for G < 4, several chunks for G > 8), both block sizes and ragged contexts
    that cut pages at arbitrary tokens."""
    import flash_engine
    lens = [0, 1, bs - 1, bs + 1, 777, 3001, 64, 2500]
    p = _problem(600 + H + d + bs, lens, H, Hkv, d, bs=bs, dtype=torch.float32)
    ref = _oracle(p)
    for version in ("v2", "v1"):
        out = flash_engine.paged_attention(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"], bs,
                                           version=version)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_fp32_close(host(out), ref)


def test_fp32_decode_fused_query_rope():
    """RoPE of the query token at position context_len - 1 in the fp32 decode prologue,
    against the oracle rotating q first."""
    import flash_engine
    lens = [1, 33, 700, 2000]
    p = _problem(71, lens, 32, 8, 128, dtype=torch.float32)
    cos, sin = O.rope_tables(4096, 128)
    pos = np.maximum(np.asarray(lens) - 1, 0)
    q_rot = O.rope_rotate(host(p["q"]), cos, sin, pos[:, None]).astype(np.float32)
    ref = O.paged_attention_gqa(q_rot, host(p["kc"]), host(p["vc"]), p["bt"], p["lens"])
    out = flash_engine.paged_attention(p["q"], p["kc"], p["vc"], p["bt_d"], p["lens_d"], 16,
                                       rope=(cuda(cos), cuda(sin)))
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    assert_fp32_close(host(out), ref)
