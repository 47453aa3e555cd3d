"""The CPU oracle against the golden vectors produced by the reference's own
ops.py (tests/golden/make_golden.py), plus self-consistency of its wrappers."""
import math

import numpy as np
import pytest

from oracle import attention_oracle as O

ATTN_CASES = ["attn_d64", "attn_d64_causal", "attn_d64_nm", "attn_d64_nm_causal", "attn_d32",
              "attn_d128"]


@pytest.mark.parametrize("name", ATTN_CASES)
def test_flash_attention_matches_reference(golden, name):
    g = golden(name)
    out = O.flash_attention(g["q"], g["k"], g["v"], bool(g["is_causal"]))
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-7)


def test_paged_attention_matches_reference(golden):
    g = golden("paged_fp32")
    out = O.paged_attention(g["q"], g["k_cache"], g["v_cache"], g["block_tables"],
                            g["context_lens"], 16)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-6)


def test_paged_kat_is_quarter(golden):
    g = golden("paged_kat")
    out = O.paged_attention(g["q"], g["k_cache"], g["v_cache"], g["block_tables"],
                            g["context_lens"], 16)
    np.testing.assert_allclose(out, g["out"], atol=1e-6)
    np.testing.assert_allclose(out, 0.25, atol=1e-6)


def test_paged_gqa_wrapper_matches_reference(golden):
    g = golden("paged_gqa_bf16")
    out = O.paged_attention_gqa(g["q"], g["k_cache"], g["v_cache"], g["block_tables"],
                                g["context_lens"], 16)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-6)
    assert np.all(out[3] == 0)  # context_len 0 -> zero row, as ops.py:74-78


def test_flash_decoding_matches_reference(golden):
    g = golden("decoding")
    out = O.flash_decoding(g["q"], g["k"], g["v"], int(g["num_splits"]))
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1e-7)
    # the reference test's own pin: split-KV agrees with full attention (< 1e-4)
    assert np.abs(out - g["out_full"]).max() < 1e-4


def test_bf16_round_matches_torch():
    import torch
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1e-40, 3.0e38, np.inf, -np.inf], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    got = O.bf16_round(x)
    np.testing.assert_array_equal(got, ref)
    assert np.isnan(O.bf16_round(np.array([np.nan], np.float32)))[0]
    bits = O.to_bf16_bits(x)
    np.testing.assert_array_equal(O.from_bf16_bits(bits), ref)


def test_paged_split_kv_equals_single_pass():
    p = O.make_paged_problem(3, 4, 8, 2, 64, [1, 31, 100, 257])
    a = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                              p["context_lens"])
    for splits in (1, 3, 8):
        b = O.paged_flash_decoding_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                       p["context_lens"], splits)
        assert np.abs(a - b).max() < 1e-5


def test_kv_range_partials_merge_to_full():
    p = O.make_paged_problem(5, 4, 8, 2, 32, [0, 20, 64, 150])
    full = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                 p["context_lens"])
    bounds = [0, 48, 96, 10 ** 9]
    parts = [O.kv_range_partials(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                 p["context_lens"], bounds[i], bounds[i + 1])
             for i in range(3)]
    merged = O.lse_merge([x[0] for x in parts], [x[1] for x in parts], [x[2] for x in parts])
    assert np.abs(merged - full).max() < 1e-5
    assert np.all(merged[0] == 0)


def test_config_generators():
    c3 = O.config3_context_lens(0)
    assert c3.shape == (64,) and c3.min() >= 512 and c3.max() <= 4096
    c5 = O.config5_context_lens(0)
    assert c5.shape == (256,) and c5.min() >= 16 and c5.max() <= 32768
    assert abs(np.median(c5) - 1024) < 300
    p = O.make_paged_problem(0, 4, 8, 2, 64, [5, 16, 17, 0])
    # the physical blocks are a permutation of the pool
    used = np.concatenate([p["block_tables"][s, :(int(c) + 15) // 16]
                           for s, c in enumerate(p["context_lens"])])
    assert len(set(used.tolist())) == len(used) == p["k_cache"].shape[0]


def test_rope_rotation_is_the_reference_formula():
    cos, sin = O.rope_tables(64, 8)
    x = np.arange(16, dtype=np.float32).reshape(2, 8)
    pos = np.array([3, 40])
    got = O.rope_rotate(x, cos, sin, pos)
    for r in range(2):
        for i in range(4):
            c, s = float(cos[pos[r], i]), float(sin[pos[r], i])
            x0, x1 = float(x[r, 2 * i]), float(x[r, 2 * i + 1])
            assert abs(got[r, 2 * i] - (x0 * c - x1 * s)) < 1e-6
            assert abs(got[r, 2 * i + 1] - (x0 * s + x1 * c)) < 1e-6
    # a rotation keeps pair norms
    assert np.allclose(np.linalg.norm(got.reshape(2, 4, 2), axis=-1),
                       np.linalg.norm(x.reshape(2, 4, 2), axis=-1))
