"""Paged decode on the GPU (C-ABI through flash_engine.ops) against the CPU oracle
and the reference-generated golden vectors."""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, assert_fp32_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _run(p, dtype, version="auto", bs=16):
    import flash_engine
    q = cuda(p["q"], dtype)
    kc = cuda(p["k_cache"], dtype)
    vc = cuda(p["v_cache"], dtype)
    bt = cuda(p["block_tables"])
    lens = cuda(p["context_lens"])
    out = flash_engine.paged_attention(q, kc, vc, bt, lens, bs, version=version)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    return host(out)


def test_paged_fp32_reference_case(golden):
    g = golden("paged_fp32")
    out = _run({"q": g["q"], "k_cache": g["k_cache"], "v_cache": g["v_cache"],
                "block_tables": g["block_tables"], "context_lens": g["context_lens"]},
               torch.float32)
    assert_fp32_close(out, g["out"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_paged_kat_constant_inputs(golden, dtype):
    g = golden("paged_kat")
    out = _run(g, dtype)
    np.testing.assert_array_equal(out, np.full_like(out, 0.25))


@pytest.mark.parametrize("version", ["v1", "v2"])
def test_paged_bf16_golden_gqa(golden, version):
    g = golden("paged_gqa_bf16")
    out = _run(g, torch.bfloat16, version)
    assert_bf16_close(out, g["out"])
    assert np.all(out[3] == 0)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("H,Hkv", [(8, 8), (32, 8), (64, 8), (16, 1), (48, 2)])
@pytest.mark.parametrize("version", ["v1", "v2"])
def test_paged_bf16_random(d, bs, H, Hkv, version):
    lens = [0, 1, bs - 1, bs, bs + 1, 3 * bs + 7, 300, 1000]
    p = O.make_paged_problem(11 + d + bs + H, len(lens), H, Hkv, d, lens, block_size=bs,
                             extra_blocks=5)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"], bs)
    out = _run(p, torch.bfloat16, version, bs=bs)
    assert_bf16_close(out, ref)


@pytest.mark.parametrize("H,Hkv", [(8, 8), (32, 8)])
def test_paged_fp16_random(H, Hkv):
    lens = [0, 17, 64, 555]
    p = O.make_paged_problem(5, len(lens), H, Hkv, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    out = _run(p, torch.float16)
    assert_bf16_close(out, ref, atol=5e-3)


@pytest.mark.parametrize("H,Hkv,d", [(8, 2, 64), (32, 8, 128), (12, 4, 96)])
def test_paged_fp32_random(H, Hkv, d):
    lens = [0, 1, 16, 33, 300]
    p = O.make_paged_problem(9, len(lens), H, Hkv, d, lens, bf16=False)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    out = _run(p, torch.float32)
    assert_fp32_close(out, ref)


@pytest.mark.parametrize("H,Hkv,d", [(8, 2, 64), (32, 8, 128), (12, 4, 96), (64, 8, 128),
                                     (4, 4, 256)])
def test_paged_fp32_long_contexts_split(H, Hkv, d):
    """Long fp32 contexts (boundaries around 512 tokens): head_dim 64 and 128 run the
    persistent split-KV decode, which cuts long sequences over several CTAs and merges
    the pieces; head_dim 96 and 256 run the generic single-pass fp32 kernel."""
    lens = [0, 1, 511, 512, 513, 1500, 2049]
    p = O.make_paged_problem(19 + d, len(lens), H, Hkv, d, lens, bf16=False)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    out = _run(p, torch.float32)
    assert_fp32_close(out, ref)


def test_paged_fp32_misaligned_cache_generic_decoder():
    """An fp32 cache that is only 4-byte aligned cannot take the persistent decode's bulk
    page copies or the vectorised decoder's 128-bit loads: the generic single-pass
    kernel runs."""
    import flash_engine
    for lens in ([900, 40, 1], [300, 17]):
        p = O.make_paged_problem(31, len(lens), 32, 8, 128, lens, bf16=False)
        ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        caches = []
        for name in ("k_cache", "v_cache"):
            x = p[name]
            flat = torch.empty(x.size + 4, dtype=torch.float32, device="cuda")
            t = flat[1:1 + x.size].view(x.shape)
            t.copy_(torch.from_numpy(np.ascontiguousarray(x)))
            assert t.data_ptr() % 16 == 4
            caches.append(t)
        out = flash_engine.paged_attention(cuda(p["q"]), caches[0], caches[1],
                                           cuda(p["block_tables"]), cuda(p["context_lens"]), 16)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_fp32_close(host(out), ref)


def test_paged_fp32_split_in_graph_capture():
    """fp32 paged decode inside a CUDA-graph capture: on a fresh stream (no cached
    workspace yet) the Python operator runs the split-KV kernel on the stream's slot of
    the library scratch, after an eager call on that stream on the stream's cached
    workspace; both replays match the oracle."""
    import flash_engine
    lens = [700, 1300, 64, 2000]
    p = O.make_paged_problem(77, len(lens), 16, 4, 128, lens, bf16=False)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    q, kc, vc = (cuda(p[k], torch.float32) for k in ("q", "k_cache", "v_cache"))
    bt, ln = cuda(p["block_tables"]), cuda(p["context_lens"])
    for eager_first in (False, True):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            if eager_first:
                flash_engine.paged_attention(q, kc, vc, bt, ln, 16)
            out = torch.empty_like(q)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                flash_engine.paged_attention(q, kc, vc, bt, ln, 16, out=out)
            out.zero_()
            g.replay()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_fp32_close(host(out), ref)


def test_paged_fp32_context_past_block_row_is_flagged():
    """A context longer than max_blocks_per_seq * block_size is a bad input: flagged in
    the device error word, no read past the row."""
    import flash_engine
    lens = [600, 40]
    p = O.make_paged_problem(5, len(lens), 8, 2, 64, lens, bf16=False)
    ln = cuda(np.array([600 + 16 * 5, 40], dtype=np.int32))
    flash_engine.paged_attention(cuda(p["q"], torch.float32), cuda(p["k_cache"], torch.float32),
                                 cuda(p["v_cache"], torch.float32), cuda(p["block_tables"]),
                                 ln, 16)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() != 0


@pytest.mark.parametrize("version", ["v1", "v2"])
def test_block_table_gather_is_bit_exact(version):
    """One-hot attention: token j of each sequence carries a key that dominates by
    e^45, so the output row must equal V[token j] bit for bit. Checks the
    (block table, block offset, KV head) address of every selected row."""
    rng = np.random.default_rng(1)
    S, H, Hkv, d, bs = 24, 32, 8, 128, 16
    lens = rng.integers(1, 700, size=S).astype(np.int32)
    p = O.make_paged_problem(2, S, H, Hkv, d, lens, extra_blocks=7)
    kc = np.zeros_like(p["k_cache"])
    q = np.zeros_like(p["q"])
    q[:, :, 0] = 8.0
    sel = np.array([rng.integers(0, c) for c in lens])
    for s in range(S):
        j = sel[s]
        kc[p["block_tables"][s, j // bs], :, j % bs, 0] = 64.0
    p2 = dict(p, q=q, k_cache=kc)
    out = _run(p2, torch.bfloat16, version)
    for s in range(S):
        j = sel[s]
        vrow = p["v_cache"][p["block_tables"][s, j // bs], :, j % bs, :]  # [Hkv, d]
        expect = np.repeat(vrow, H // Hkv, axis=0)
        np.testing.assert_array_equal(out[s], expect)


def test_bad_block_index_is_flagged_not_read():
    import flash_engine
    lens = [40, 40]
    p = O.make_paged_problem(3, 2, 8, 2, 128, lens)
    nb = p["k_cache"].shape[0]
    bt = p["block_tables"].copy()
    bt[1, 1] = nb + 1000  # outside the pool
    q = cuda(p["q"], torch.bfloat16)
    kc = cuda(p["k_cache"], torch.bfloat16)
    vc = cuda(p["v_cache"], torch.bfloat16)
    flash_engine.paged_attention(q, kc, vc, cuda(bt), cuda(p["context_lens"]), 16,
                                 version="v1")
    assert flash_engine.device_errors() & 2
    assert flash_engine.device_errors() == 0  # cleared by the read


def test_config3_shape_parity():
    """Benchmark config 3 shape (B64, 32q/8kv, d128, ctx U[512,4096], bs 16), on a
    seeded subset of 8 sequences for oracle speed, with the full split logic."""
    lens = O.config3_context_lens(0)[:8]
    p = O.make_paged_problem(0, 8, 32, 8, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    out = _run(p, torch.bfloat16)
    assert_bf16_close(out, ref)


def test_config3_full_batch():
    """All 64 sequences of benchmark config 3 (seed 0) against the oracle, through the
    single-pass kernel and the split-KV kernel (whose flat chunking cuts sequences
    at arbitrary pages)."""
    import flash_engine
    lens = O.config3_context_lens(0)
    p = O.make_paged_problem(0, 64, 32, 8, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
    bt, cl = cuda(p["block_tables"]), cuda(p["context_lens"])
    for version in ("v1", "v2"):
        out = flash_engine.paged_attention(q, kc, vc, bt, cl, 16, version=version)
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out), ref)


def test_serving_mix_long_tail():
    """Config-5-like lognormal context lengths (a few very long sequences among many
    short ones): the flat chunking spreads the long ones over many CTAs."""
    import flash_engine
    lens = O.config5_context_lens(3)[:48]
    lens[5] = 20000
    p = O.make_paged_problem(5, len(lens), 64, 8, 128, lens)
    sel = [0, 5, 17, 47]
    ref = O.paged_attention_gqa(p["q"][sel], p["k_cache"], p["v_cache"],
                                p["block_tables"][sel], p["context_lens"][sel])
    q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
    out = flash_engine.paged_attention(q, kc, vc, cuda(p["block_tables"]),
                                       cuda(p["context_lens"]), 16)
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(out)[sel], ref)


def test_workspace_counters_left_zero_across_shapes():
    """One zero-filled workspace serves split-KV calls of several head configurations
    back to back: every call leaves the arrival counters (the first 1024 floats) at
    zero. The long sequences make the kernel split them and merge the pieces."""
    import flash_engine
    shapes = [(32, 8, 128), (64, 8, 128), (8, 1, 64), (16, 2, 128)]
    n = max(flash_engine.paged_attention_workspace_floats(H, Hkv, d) for H, Hkv, d in shapes)
    ws = torch.zeros(n, dtype=torch.float32, device="cuda")
    lens = [3000, 1, 0, 700, 4096, 17]
    for seed, (H, Hkv, d) in enumerate(shapes):
        p = O.make_paged_problem(40 + seed, len(lens), H, Hkv, d, lens)
        ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
        out = flash_engine.paged_attention(q, kc, vc, cuda(p["block_tables"]),
                                           cuda(p["context_lens"]), 16, workspace=ws)
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out), ref)
        assert int(torch.count_nonzero(ws[:1024].view(torch.int32))) == 0


def test_single_long_sequence_many_pieces():
    """One KV head and one 60k-token sequence: its pages are cut over every CTA, so
    the CTA of the last piece merges a few hundred partials (more than one 32-part
    pass of the combine)."""
    import flash_engine
    lens = [60000, 5]
    p = O.make_paged_problem(51, 2, 8, 1, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    for version in ("v2", "v1"):
        out = _run(p, torch.bfloat16, version)
        assert_bf16_close(out, ref)


@pytest.mark.parametrize("n_seqs", [16, 24])
def test_sequences_cut_into_9_to_32_pieces(n_seqs):
    """One KV head, n_seqs sequences of 4096 tokens: the flat split gives each
    sequence 9-32 pieces on 148 SMs (16 seqs: about 19; 24 seqs: about 13), so the
    combine takes its multi-batch path (stats of every part in the first round trip,
    O rows 8 at a time)."""
    lens = [4096] * n_seqs
    p = O.make_paged_problem(60 + n_seqs, n_seqs, 4, 1, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    assert_bf16_close(_run(p, torch.bfloat16, "v2"), ref)


def test_nonzero_workspace_counters_are_flagged():
    """A workspace whose counters were not zero-filled is reported through the device
    error word (bit 3) instead of being trusted silently."""
    import flash_engine
    lens = [4096] * 6
    p = O.make_paged_problem(52, len(lens), 32, 8, 128, lens)
    q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
    n = flash_engine.paged_attention_workspace_floats(32, 8, 128)
    ws = torch.zeros(n, dtype=torch.float32, device="cuda")
    ws[:1024].view(torch.int32).fill_(100000)
    flash_engine.paged_attention(q, kc, vc, cuda(p["block_tables"]), cuda(p["context_lens"]), 16,
                                 workspace=ws)
    assert flash_engine.device_errors() & 8
    assert flash_engine.device_errors() == 0


def _to_vllm(kc, vc):
    """[nb, Hkv, bs, d] -> vLLM K [nb, Hkv, d/8, bs, 8] and V [nb, Hkv, d, bs]."""
    nb, hkv, bs, d = kc.shape
    kx = np.ascontiguousarray(kc.reshape(nb, hkv, bs, d // 8, 8).transpose(0, 1, 3, 2, 4))
    vx = np.ascontiguousarray(vc.transpose(0, 1, 3, 2))
    return kx, vx


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("version", ["v1", "v2"])
@pytest.mark.parametrize("H,Hkv,d", [(32, 8, 128), (64, 4, 64), (8, 8, 128)])
def test_paged_vllm_layout(dtype, version, H, Hkv, d):
    import flash_engine
    lens = [0, 1, 15, 16, 17, 250, 1500]
    p = O.make_paged_problem(61 + H + d, len(lens), H, Hkv, d, lens, extra_blocks=3)
    kc, vc = p["k_cache"], p["v_cache"]
    if dtype == torch.float16:
        kc, vc = kc.astype(np.float16).astype(np.float32), vc.astype(np.float16).astype(np.float32)
    ref = O.paged_attention_gqa(p["q"], kc, vc, p["block_tables"], p["context_lens"])
    kx, vx = _to_vllm(kc, vc)
    out = flash_engine.paged_attention(cuda(p["q"], dtype), cuda(kx, dtype), cuda(vx, dtype),
                                       cuda(p["block_tables"]), cuda(p["context_lens"]), 16,
                                       version=version, kv_layout="vllm")
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(out), ref, atol=2e-2 if dtype == torch.bfloat16 else 5e-3)


def test_fp16_reference_entry_takes_vllm_layout(golden):
    """fe_paged_attention_v1_fp16 follows the layout the reference's header declares
    for it; the constant known-answer case gives 0.25."""
    from flash_engine import _lib
    g = golden("paged_kat")
    kx, vx = _to_vllm(g["k_cache"], g["v_cache"])
    q, kc, vc = cuda(g["q"], torch.float16), cuda(kx, torch.float16), cuda(vx, torch.float16)
    out = torch.empty_like(q)
    bt, cl = cuda(g["block_tables"]), cuda(g["context_lens"])
    S, H, d = g["q"].shape
    rc = _lib.lib.fe_paged_attention_v1_fp16(q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                             out.data_ptr(), bt.data_ptr(), cl.data_ptr(), S, H,
                                             H, d, 16, 64, bt.shape[1], 0, 0.0,
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(out), np.full((S, H, d), 0.25, np.float32))


@pytest.mark.parametrize("version", ["v1", "v2"])
@pytest.mark.parametrize("kv_layout", ["flat", "vllm"])
def test_paged_decode_fused_query_rope(version, kv_layout):
    """RoPE of the query token at position context_len - 1, applied in the kernel
    prologue, against the oracle rotating q first."""
    import flash_engine
    lens = [1, 33, 700, 2000]
    p = O.make_paged_problem(71, len(lens), 32, 8, 128, lens)
    cos, sin = O.rope_tables(4096, 128)
    pos = np.maximum(np.asarray(lens) - 1, 0)
    q_rot = O.bf16_round(O.rope_rotate(p["q"], cos, sin, pos[:, None]).astype(np.float32))
    ref = O.paged_attention_gqa(q_rot, p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    kc, vc = p["k_cache"], p["v_cache"]
    if kv_layout == "vllm":
        kc, vc = _to_vllm(kc, vc)
    out = flash_engine.paged_attention(cuda(p["q"], torch.bfloat16), cuda(kc, torch.bfloat16),
                                       cuda(vc, torch.bfloat16), cuda(p["block_tables"]),
                                       cuda(p["context_lens"]), 16, version=version,
                                       kv_layout=kv_layout, rope=(cuda(cos), cuda(sin)))
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(out), ref)


def _v1_bf16(lib, x, out, stream):
    S = x["q"].shape[0]
    return lib.fe_paged_attention_v1_bf16(
        x["q"].data_ptr(), x["kc"].data_ptr(), x["vc"].data_ptr(), out.data_ptr(),
        x["bt"].data_ptr(), x["lens"].data_ptr(), S, x["H"], x["Hkv"], x["d"], 16,
        x["max_ctx"], x["bt"].shape[1], x["kc"].shape[0], 0.0, stream)


def test_v1_c_entry_splits_on_library_scratch_and_in_capture():
    """The reference's v1 calling convention (no scratch): the library runs the
    split-KV kernel on the stream's slot of its static scratch, which needs no
    allocation, so a first call captured into a CUDA graph on a new stream splits too;
    both match the oracle."""
    import ctypes
    from flash_engine import _lib
    lens = [4096, 1, 0, 3000, 700, 2049]
    p = O.make_paged_problem(90, len(lens), 32, 8, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    x = dict(q=cuda(p["q"], torch.bfloat16), kc=cuda(p["k_cache"], torch.bfloat16),
             vc=cuda(p["v_cache"], torch.bfloat16), bt=cuda(p["block_tables"]),
             lens=cuda(p["context_lens"]), H=32, Hkv=8, d=128, max_ctx=max(lens))
    lib = _lib.lib
    # eager, twice (the second call reuses the stream's workspace)
    for _ in range(2):
        out = torch.full_like(x["q"], float("nan"))
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        assert _v1_bf16(lib, x, out, st) == 0
        torch.cuda.synchronize()
        assert _lib.device_errors() == 0
        assert_bf16_close(host(out), ref)
    # first call on a new stream happens inside a capture
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    out = torch.full_like(x["q"], float("nan"))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        assert _v1_bf16(lib, x, out, ctypes.c_void_p(side.cuda_stream)) == 0
    g.replay()
    torch.cuda.synchronize()
    assert _lib.device_errors() == 0
    assert_bf16_close(host(out), ref)


def test_more_sequences_than_one_launch():
    """More sequences than one kernel launch takes (4096): the library issues several
    launches that share one workspace; every row must match the oracle."""
    import flash_engine
    rng = np.random.default_rng(91)
    S = 4300
    lens = rng.integers(0, 48, size=S).astype(np.int32)
    lens[7] = 700  # one longer sequence among many short ones
    lens[4200] = 900
    p = O.make_paged_problem(92, S, 8, 2, 64, lens)
    sel = np.array([0, 7, 100, 4095, 4096, 4200, S - 1])
    ref = O.paged_attention_gqa(p["q"][sel], p["k_cache"], p["v_cache"], p["block_tables"][sel],
                                p["context_lens"][sel])
    q, kc, vc = (cuda(p[x], torch.bfloat16) for x in ("q", "k_cache", "v_cache"))
    bt, cl = cuda(p["block_tables"]), cuda(p["context_lens"])
    for version in ("v2", "v1"):
        out = flash_engine.paged_attention(q, kc, vc, bt, cl, 16, version=version)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out)[sel], ref)


def _v1_fp32(lib, x, out, stream):
    S = x["q"].shape[0]
    return lib.fe_paged_attention_v1_fp32(
        x["q"].data_ptr(), x["kc"].data_ptr(), x["vc"].data_ptr(), out.data_ptr(),
        x["bt"].data_ptr(), x["lens"].data_ptr(), S, x["H"], x["Hkv"], x["d"], 16,
        x["max_ctx"], x["bt"].shape[1], x["kc"].shape[0], 0.0, stream)


@pytest.mark.parametrize("d", [64, 128])
def test_v1_fp32_c_entry_capture_first_and_replay(d):
    """The reference's fp32 v1 entry (launch_paged_attention_v1_fp32: no scratch
    argument) on a stream whose first call is inside a CUDA-graph capture: the
    persistent split-KV decode runs on the library's static scratch slot, so nothing is
    allocated; the replays and a later eager call on the same stream match the oracle."""
    import ctypes
    from flash_engine import _lib
    lens = [4096, 1, 0, 3000, 700, 2049, 513]
    p = O.make_paged_problem(93 + d, len(lens), 32, 8, d, lens, bf16=False)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    x = dict(q=cuda(p["q"]), kc=cuda(p["k_cache"]), vc=cuda(p["v_cache"]),
             bt=cuda(p["block_tables"]), lens=cuda(p["context_lens"]), H=32, Hkv=8, d=d,
             max_ctx=max(lens))
    lib = _lib.lib
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    out = torch.full_like(x["q"], float("nan"))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        assert _v1_fp32(lib, x, out, ctypes.c_void_p(side.cuda_stream)) == 0
    for _ in range(2):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert _lib.device_errors() == 0
        assert_fp32_close(host(out), ref)
    out2 = torch.full_like(x["q"], float("nan"))
    with torch.cuda.stream(side):
        assert _v1_fp32(lib, x, out2, ctypes.c_void_p(side.cuda_stream)) == 0
    torch.cuda.synchronize()
    assert _lib.device_errors() == 0
    assert_fp32_close(host(out2), ref)
    del g


def test_v1_entries_on_many_streams():
    """More streams than the library has scratch slots call the v1 bf16 entry: the
    first streams run the split-KV decode on their own slot, the rest the single-pass
    kernel; all results match the oracle, and the slots' counters stay consistent
    when the first stream is used again."""
    import ctypes
    from flash_engine import _lib
    lens = [3000, 17, 2500, 0, 4096]
    p = O.make_paged_problem(95, len(lens), 32, 8, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    x = dict(q=cuda(p["q"], torch.bfloat16), kc=cuda(p["k_cache"], torch.bfloat16),
             vc=cuda(p["v_cache"], torch.bfloat16), bt=cuda(p["block_tables"]),
             lens=cuda(p["context_lens"]), H=32, Hkv=8, d=128, max_ctx=max(lens))
    lib = _lib.lib
    streams = [torch.cuda.Stream() for _ in range(6)]
    outs = [torch.full_like(x["q"], float("nan")) for _ in streams]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    for rep in range(2):
        for s, o in zip(streams, outs):
            assert _v1_bf16(lib, x, o, ctypes.c_void_p(s.cuda_stream)) == 0
        torch.cuda.synchronize()
        assert _lib.device_errors() == 0
        for o in outs:
            assert_bf16_close(host(o), ref)


@pytest.mark.parametrize("dtype,kv_layout", [(torch.bfloat16, "flat"), (torch.bfloat16, "vllm"),
                                             (torch.float16, "flat"), (torch.float32, "flat")])
def test_kv_append_with_rope_then_decode(dtype, kv_layout):
    """One decode step with RoPE on Q and K: the new token's key is rotated at position
    ctx - 1 and written with its value into the paged cache (fe_paged_kv_append), then
    the decode rotates the query at the same position. The cache's earlier keys were
    stored rotated by earlier steps. Against the oracle with Q and every key rotated."""
    import flash_engine
    lens = [1, 17, 700, 2000, 0]
    S, H, Hkv, d = len(lens), 32, 8, 128
    p = O.make_paged_problem(81, S, H, Hkv, d, lens, bf16=dtype != torch.float32)
    cos, sin = O.rope_tables(4096, d)
    rnd = (lambda x: O.bf16_round(x.astype(np.float32))) if dtype == torch.bfloat16 else \
        (lambda x: x.astype(np.float16).astype(np.float32)) if dtype == torch.float16 else \
        (lambda x: x.astype(np.float32))
    kc, vc = rnd(p["k_cache"]), rnd(p["v_cache"])
    rng = np.random.default_rng(82)
    k_new = rnd(rng.standard_normal((S, Hkv, d), dtype=np.float32))
    v_new = rnd(rng.standard_normal((S, Hkv, d), dtype=np.float32))
    # what the cache must hold after the append: the new key rotated at ctx - 1
    kc_ref, vc_ref = kc.copy(), vc.copy()
    for s, c in enumerate(lens):
        if c <= 0:
            continue
        blk, off = p["block_tables"][s, (c - 1) // 16], (c - 1) % 16
        kc_ref[blk, :, off] = rnd(O.rope_rotate(k_new[s], cos, sin, c - 1))
        vc_ref[blk, :, off] = v_new[s]
    pos = np.maximum(np.asarray(lens) - 1, 0)
    q = rnd(p["q"])
    q_rot = rnd(O.rope_rotate(q, cos, sin, pos[:, None]))
    ref = O.paged_attention_gqa(q_rot, kc_ref, vc_ref, p["block_tables"], p["context_lens"])
    kd, vd = kc, vc
    if kv_layout == "vllm":
        kd, vd = _to_vllm(kc, vc)
    kd, vd = cuda(kd, dtype), cuda(vd, dtype)
    bt, cl = cuda(p["block_tables"]), cuda(p["context_lens"])
    tabs = (cuda(cos), cuda(sin))
    flash_engine.paged_kv_append(cuda(k_new, dtype), cuda(v_new, dtype), kd, vd, bt, cl, 16,
                                 kv_layout=kv_layout, rope=tabs)
    out = flash_engine.paged_attention(cuda(q, dtype), kd, vd, bt, cl, 16, kv_layout=kv_layout,
                                       rope=tabs)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    if dtype == torch.float32:
        assert_fp32_close(host(out), ref)
    else:
        assert_bf16_close(host(out), ref, atol=2e-2 if dtype == torch.bfloat16 else 5e-3)
    # the appended rows landed where the oracle put them (flat layout): V bit for bit, K
    # within one rounding of the cache type (fp32 products in the kernel, fp64 here)
    if kv_layout == "flat":
        np.testing.assert_array_equal(host(vd), host(cuda(vc_ref, dtype)))
        tol = {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10, torch.float32: 1e-6}[dtype]
        np.testing.assert_allclose(host(kd), kc_ref, rtol=tol, atol=tol)
