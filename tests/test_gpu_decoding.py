"""Split-KV decoding on the GPU: the dense fp32 reference entry, the paged
partials + log-sum-exp merge used for KV-range sharding, against the oracle."""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, assert_fp32_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def test_flash_decoding_fp32_golden(golden):
    import flash_engine
    g = golden("decoding")
    out = flash_engine.flash_decoding(cuda(g["q"]), cuda(g["k"]), cuda(g["v"]),
                                      int(g["num_splits"]))
    assert_fp32_close(host(out), g["out"])


@pytest.mark.parametrize("B,H,M,d,S", [(2, 4, 512, 64, 8), (1, 3, 1000, 128, 16),
                                       (2, 2, 7, 32, 8), (1, 1, 33, 256, 4)])
def test_flash_decoding_fp32_random(B, H, M, d, S):
    import flash_engine
    rng = np.random.default_rng(B * 100 + M)
    q = rng.standard_normal((B, H, 1, d), dtype=np.float32)
    k = rng.standard_normal((B, H, M, d), dtype=np.float32)
    v = rng.standard_normal((B, H, M, d), dtype=np.float32)
    ref = O.flash_decoding(q, k, v, S)
    out = flash_engine.flash_decoding(cuda(q), cuda(k), cuda(v), S)
    assert_fp32_close(host(out), ref)


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_kv_range_partials_merge(ranks):
    """KV-range sharding emulated on one GPU: each 'rank' computes the merged
    partial of its token window, the partials are stacked as an all-gather would
    and merged; the result must match single-pass attention."""
    import flash_engine
    lens = [0, 5, 16, 300, 1024, 2047]
    S, H, Hkv, d, bs = len(lens), 32, 8, 128, 16
    p = O.make_paged_problem(4, S, H, Hkv, d, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
    bt, cl = cuda(p["block_tables"]), cuda(p["context_lens"])
    M = 2048
    per = -(-M // ranks)
    per = -(-per // bs) * bs
    outs, stats = [], []
    for r in range(ranks):
        o, s = flash_engine.paged_decode_partials(q, kc, vc, bt, cl, r * per, (r + 1) * per)
        outs.append(o)
        stats.append(s)
    go = torch.stack(outs)  # [ranks, S, H, d]
    gs = torch.stack(stats)
    final = flash_engine.merge_partials(go, gs, ranks, 1, "bf16")
    out = host(final).reshape(S, H, d)
    assert flash_engine.device_errors() == 0
    assert_bf16_close(out, ref)


def test_partials_match_oracle_partials():
    import flash_engine
    lens = [0, 40, 100]
    p = O.make_paged_problem(8, 3, 8, 2, 64, lens)
    o, s = flash_engine.paged_decode_partials(*(cuda(p[x], torch.bfloat16)
                                                for x in ("q", "k_cache", "v_cache")),
                                              cuda(p["block_tables"]), cuda(p["context_lens"]),
                                              32, 96)
    O_ref, m_ref, l_ref = O.kv_range_partials(p["q"], p["k_cache"], p["v_cache"],
                                              p["block_tables"], p["context_lens"], 32, 96)
    o, s = host(o), host(s)
    assert np.all(s[0, :, 1] == 0) and np.all(np.isneginf(s[0, :, 0]))
    # compare normalised partial outputs and the log-sum-exp of each row
    for seq in (1, 2):
        lse_gpu = s[seq, :, 0] * np.log(2) + np.log(s[seq, :, 1])
        lse_ref = m_ref[seq] + np.log(l_ref[seq])
        np.testing.assert_allclose(lse_gpu, lse_ref, atol=2e-3)
        assert_bf16_close(o[seq] / s[seq, :, 1:2], O_ref[seq] / l_ref[seq][:, None])


@pytest.mark.parametrize("world", [1, 2, 4])
def test_kv_exchange_emulated_ranks_one_gpu(world):
    """The peer-memory KV-range exchange with its ranks emulated on one GPU: every
    rank's exchange buffer lives here, phase 1 (decode + stores into every buffer) runs
    for all ranks before phase 2 (wait for all flags + merge) of any. Two steps use the
    two slot generations; every rank's output must match the oracle."""
    import ctypes
    import flash_engine
    from flash_engine import _lib, ops, sharding
    lens = [0, 1, 40, 333, 1024, 2047]
    S, H, Hkv, d = len(lens), 32, 8, 128
    p = O.make_paged_problem(70 + world, S, H, Hkv, d, lens)
    kc, vc = (cuda(p[x], torch.bfloat16) for x in ("k_cache", "v_cache"))
    bt, cl = cuda(p["block_tables"]), cuda(p["context_lens"])
    M = int(max(lens))
    L = _lib.lib
    nbytes = L.fe_kv_exchange_bytes(world, S * H, d)
    bufs = []
    for _ in range(world):
        b = ctypes.c_void_p()
        assert L.fe_kv_exchange_alloc(nbytes, ctypes.byref(b)) == 0
        bufs.append(b.value)
    wss = [torch.zeros(flash_engine.paged_attention_workspace_floats(H, Hkv, d),
                       dtype=torch.float32, device="cuda") for _ in range(world)]
    try:
        for step in range(2):
            q_np = O.make_paged_problem(80 + step, S, H, Hkv, d, lens)["q"]
            q = cuda(q_np, torch.bfloat16)
            ref = O.paged_attention_gqa(q_np, p["k_cache"], p["v_cache"], p["block_tables"],
                                        p["context_lens"])
            outs = [torch.full_like(q, float("nan")) for _ in range(world)]
            for r in range(world):
                tb, te = sharding.kv_range_bounds(M, world, r, 16)
                ops.paged_decode_kv_exchange(q, kc, vc, bt, cl, tb, te, bufs, r, S * H,
                                             workspace=wss[r], out=outs[r], phases=1)
            for r in range(world):
                ops.paged_decode_kv_exchange(q, kc, vc, bt, cl, 0, 0, bufs, r, S * H,
                                             workspace=wss[r], out=outs[r], phases=2)
            torch.cuda.synchronize()
            assert flash_engine.device_errors() == 0
            for r in range(world):
                assert_bf16_close(host(outs[r]), ref)
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            L.fe_kv_exchange_free(b)


def test_partials_captured_first_on_library_scratch():
    """A KV-range step (partials of two windows + merge) captured into a CUDA graph with
    no workspace given: on the capture stream nothing may be allocated, so the partials
    run on the stream's slot of the library scratch; replays on new queries match the
    oracle."""
    import flash_engine
    from flash_engine.graph import DecodeGraph
    lens = [9, 300, 1024, 2000]
    S, H, Hkv, d = len(lens), 32, 8, 128
    p = O.make_paged_problem(54, S, H, Hkv, d, lens)
    q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
    bt, cl = cuda(p["block_tables"]), cuda(p["context_lens"])

    def step():
        parts = [flash_engine.paged_decode_partials(q, kc, vc, bt, cl, tb, te)
                 for tb, te in ((0, 1008), (1008, 2000))]
        return flash_engine.merge_partials(torch.stack([o for o, _ in parts]),
                                           torch.stack([s for _, s in parts]), 2, 1, "bf16")

    g = DecodeGraph(step, warmup=0)
    for seed in (55, 56):
        q2 = O.make_paged_problem(seed, S, H, Hkv, d, lens)["q"]
        q.copy_(cuda(q2, torch.bfloat16))
        out = g.replay()
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        assert_bf16_close(host(out).reshape(S, H, d), ref)
