"""Prefill forward on the GPU against the reference-generated golden vectors and
the oracle."""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, assert_fp32_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

ATTN_CASES = ["attn_d64", "attn_d64_causal", "attn_d64_nm", "attn_d64_nm_causal", "attn_d32",
              "attn_d128"]


@pytest.mark.parametrize("name", ATTN_CASES)
@pytest.mark.parametrize("kind", ["flash", "naive"])
def test_fp32_golden(golden, name, kind):
    import flash_engine
    g = golden(name)
    fn = flash_engine.flash_attention if kind == "flash" else flash_engine.naive_attention
    out = fn(cuda(g["q"]), cuda(g["k"]), cuda(g["v"]), bool(g["is_causal"]))
    assert_fp32_close(host(out), g["out"])


def test_fp32_config1():
    """fp32, non-causal, [1, 8, 512, 64], N(0,1) inputs, seed 42."""
    import flash_engine
    rng = np.random.default_rng(42)
    q, k, v = (rng.standard_normal((1, 8, 512, 64), dtype=np.float32) for _ in range(3))
    ref = O.flash_attention(q, k, v, False)
    out = flash_engine.flash_attention(cuda(q), cuda(k), cuda(v), False)
    assert_fp32_close(host(out), ref)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("N,M,d", [(1, 1, 64), (65, 130, 32), (200, 77, 128), (128, 128, 100)])
def test_fp32_shapes(causal, N, M, d):
    import flash_engine
    rng = np.random.default_rng(N + M + d)
    q = rng.standard_normal((2, 3, N, d), dtype=np.float32)
    k = rng.standard_normal((2, 3, M, d), dtype=np.float32)
    v = rng.standard_normal((2, 3, M, d), dtype=np.float32)
    ref = O.flash_attention(q, k, v, causal)
    out = flash_engine.flash_attention(cuda(q), cuda(k), cuda(v), causal)
    assert_fp32_close(host(out), ref)
