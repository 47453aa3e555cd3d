"""The C-ABI shared library: loads, exports every symbol include/flash_engine_c.h
declares, and rejects unsupported arguments before touching the GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "flash_engine_c.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fe_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from flash_engine import _lib
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(_lib.lib, n), n
    assert set(_lib.EXPORTED) <= set(names)
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    for n in names:
        assert re.search(rf"\bT {n}\b", out), n


def test_version():
    import flash_engine
    assert flash_engine.get_version().startswith("1.2.0")


def test_rejects_unsupported_arguments_without_launch():
    from flash_engine import _lib
    L = _lib.lib
    # head_dim 96 / block_size 8 are not supported by the tensor-core decode
    assert L.fe_paged_attention_v1_bf16(None, None, None, None, None, None, 1, 8, 2, 96, 16,
                                        16, 1, 0, 0.0, None) == 1
    assert L.fe_paged_attention_v1_bf16(None, None, None, None, None, None, 1, 8, 2, 128, 8,
                                        16, 1, 0, 0.0, None) == 1
    # heads not a multiple of kv heads
    assert L.fe_paged_attention_v1_fp32(None, None, None, None, None, None, 1, 6, 4, 64, 16,
                                        16, 1, 0, 0.0, None) == 1
    # split count < 1
    assert L.fe_flash_decoding_forward_fp32(None, None, None, None, None, None, 1, 1, 16, 64, 0,
                                            0.0, None) == 1
    # merge: bad dtype code
    assert L.fe_merge_partials(None, None, 1, 1, 1, 64, None, None, 7, None) == 1
    # KV-range exchange: bad world / phases; buffer size of a bad shape is 0
    assert L.fe_kv_exchange_bytes(9, 128, 128) == 0
    assert L.fe_kv_exchange_bytes(2, 128, 128) == 256 + 8 * 2 * 2 * 128 * (128 + 2)
    for world, rank, phases in ((9, 0, 3), (2, 2, 3), (2, 0, 0), (2, 0, 4)):
        assert L.fe_paged_decode_kv_exchange_bf16(None, None, None, None, None, 1, 8, 2, 128,
                                                  16, 1, 0, 0.0, 0, 16, None, 0, None, world,
                                                  rank, 8, None, phases, None) == 1
    # KV range over NCCL: scratch size, and rejection before any NCCL or GPU work
    assert L.fe_kv_range_nccl_scratch_floats(4, 6, 32, 128) == 5 * 6 * 32 * 130
    assert L.fe_kv_range_nccl_scratch_floats(0, 6, 32, 128) == 0
    assert L.fe_paged_decode_kv_range_nccl_bf16(None, None, None, None, None, 1, 8, 2, 128, 16,
                                                1, 0, 0.0, 16, None, 0, None, 0, 2, None, 0,
                                                None, None) == 1
    # empty problems are a no-op success
    assert L.fe_flash_attention_forward_fp32(None, None, None, None, 0, 4, 16, 16, 64, 0, 0.0,
                                             None) == 0


def test_ops_have_no_cpu_fallback():
    import numpy as np
    import torch
    import flash_engine
    q = torch.zeros(1, 1, 4, 64)
    with pytest.raises(TypeError):
        flash_engine.flash_attention(q, q, q)
    with pytest.raises(TypeError):
        flash_engine.flash_attention(np.zeros((1, 1, 4, 64), np.float32), q, q)
    # the reference binding's checks (TORCH_CHECK raises RuntimeError with these messages)
    import flash_engine_cuda
    with pytest.raises(RuntimeError, match="Q must be a CUDA tensor"):
        flash_engine_cuda.flash_attention_forward(q, q, q, False)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        flash_engine_cuda.paged_attention_forward(q, q, q, q, q)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        flash_engine_cuda.fused_rmsnorm_forward(q, q, 1e-5)
