"""The reference extension-module names (``flash_engine_cuda``, the reference's
python/bindings.cpp:10-57) on the GPU: results against the oracle, the binding's
argument checks, and the output allocated like ``torch::empty_like(q)``."""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, assert_fp32_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_forward(dtype, causal):
    import flash_engine_cuda
    rng = np.random.default_rng(11 + causal)
    q, k, v = (rng.standard_normal((1, 2, 200, 64), dtype=np.float32) for _ in range(3))
    if dtype == torch.float16:
        q, k, v = (x.astype(np.float16).astype(np.float32) for x in (q, k, v))
    out = flash_engine_cuda.flash_attention_forward(cuda(q, dtype), cuda(k, dtype),
                                                    cuda(v, dtype), causal)
    torch.cuda.synchronize()
    assert out.dtype == dtype and out.shape == (1, 2, 200, 64) and out.is_contiguous()
    ref = O.flash_attention(q, k, v, causal)
    if dtype == torch.float32:
        assert_fp32_close(host(out), ref)
    else:
        assert_bf16_close(host(out), ref)


def test_flash_attention_forward_checks():
    import flash_engine_cuda
    q = torch.zeros((1, 2, 64, 64), device="cuda")
    with pytest.raises(RuntimeError, match="K must be contiguous"):
        flash_engine_cuda.flash_attention_forward(q, q.transpose(2, 3), q, False)
    with pytest.raises(RuntimeError, match="Unsupported scalar type"):
        x = q.to(torch.float64)
        flash_engine_cuda.flash_attention_forward(x, x, x, False)


def test_paged_attention_forward():
    import flash_engine_cuda
    lens = [1, 37, 300, 1000]
    p = O.make_paged_problem(12, len(lens), 8, 2, 128, lens)
    ref = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                p["context_lens"])
    out = flash_engine_cuda.paged_attention_forward(
        cuda(p["q"], torch.bfloat16), cuda(p["k_cache"], torch.bfloat16),
        cuda(p["v_cache"], torch.bfloat16), cuda(p["block_tables"]), cuda(p["context_lens"]))
    torch.cuda.synchronize()
    assert_bf16_close(host(out), ref)
    with pytest.raises(RuntimeError, match="must be int32"):
        flash_engine_cuda.paged_attention_forward(
            cuda(p["q"], torch.bfloat16), cuda(p["k_cache"], torch.bfloat16),
            cuda(p["v_cache"], torch.bfloat16), cuda(p["block_tables"]).long(),
            cuda(p["context_lens"]))
