"""The no-allocation split-KV decode entry point (fe_paged_attention_v2_bf16_noalloc).

Some callers cannot allocate device memory: plugin hosts that own every device
buffer and pass a library only its inputs and outputs, and serving loops that may
not call cudaMalloc because it synchronises the device. This entry point keeps its
split partials in a fixed array inside the library. The test calls it through the
C ABI twice in a row, on two different problems, and compares each result with the
scratch-taking entry point (fe_paged_attention_v2_bf16) on the same inputs.

The file name sorts last so that a run stopping at the first failure has already
run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(seed, lens, H=32, Hkv=8, d=128):
    p = O.make_paged_problem(seed, len(lens), H, Hkv, d, lens)
    return dict(q=cuda(p["q"], torch.bfloat16), kc=cuda(p["k_cache"], torch.bfloat16),
                vc=cuda(p["v_cache"], torch.bfloat16), bt=cuda(p["block_tables"]),
                lens=cuda(p["context_lens"]), H=H, Hkv=Hkv, d=d,
                max_ctx=int(max(lens)), ref=p)


def _noalloc(lib, x, out, d=None):
    S = x["q"].shape[0]
    return lib.fe_paged_attention_v2_bf16_noalloc(
        x["q"].data_ptr(), x["kc"].data_ptr(), x["vc"].data_ptr(), out.data_ptr(),
        x["bt"].data_ptr(), x["lens"].data_ptr(), S, x["H"], x["Hkv"], d or x["d"], 16,
        x["max_ctx"], x["bt"].shape[1], x["kc"].shape[0], 0.0,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_scratch_entry_on_two_calls():
    import flash_engine
    from flash_engine import _lib
    lib = _lib.lib
    problems = [_inputs(21, [0, 1, 300, 4000, 2049, 16]),
                _inputs(22, [700, 33, 1, 1500], H=64, Hkv=4, d=64)]
    for x in problems:
        ref = flash_engine.paged_attention(x["q"], x["kc"], x["vc"], x["bt"], x["lens"], 16,
                                           version="v2")
        out = torch.full_like(x["q"], float("nan"))
        assert _noalloc(lib, x, out) == 0
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out), host(ref))
        # and against the CPU oracle on the same inputs
        p = x["ref"]
        oracle = O.paged_attention_gqa(p["q"], p["k_cache"], p["v_cache"], p["block_tables"],
                                       p["context_lens"])
        assert_bf16_close(host(out), oracle)


def test_noalloc_limit_and_rejection():
    """The library-owned scratch covers every supported head configuration on this
    GPU; shapes the kernel does not support are refused before any GPU work."""
    from flash_engine import _lib
    lib = _lib.lib
    limit = 4 * 1024 * 1024  # FE_NOALLOC_SCRATCH_FLOATS
    for H, Hkv in ((32, 8), (64, 8), (64, 4), (16, 1)):
        for d in (64, 128):
            need = lib.fe_paged_attention_v2_workspace_floats(H, Hkv, d, 16)
            assert 0 < need <= limit, (H, Hkv, d, need)
    x = _inputs(23, [64, 64])
    out = torch.empty_like(x["q"])
    assert _noalloc(lib, x, out, d=96) == 1
    assert _noalloc(lib, x, out) == 0
    torch.cuda.synchronize()
    assert np.isfinite(host(out)).all()
