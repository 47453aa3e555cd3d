"""Helpers shared by the GPU parity tests (numpy <-> torch CUDA tensors)."""
import numpy as np
import torch

BF16_ATOL = 2e-2     # bf16 tolerance (absolute), as stated for this path
FP32_RTOL = 1e-3     # fp32 tolerance: max|err| / max|ref|


def cuda(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def host(t):
    return t.float().cpu().numpy()


def assert_bf16_close(got, ref, atol=BF16_ATOL):
    err = float(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64)).max()) \
        if np.asarray(ref).size else 0.0
    assert np.isfinite(np.asarray(got)).all(), "non-finite output"
    assert err <= atol, f"max abs err {err} > {atol}"
    return err


def assert_fp32_close(got, ref, rtol=FP32_RTOL):
    ref = np.asarray(ref, np.float64)
    err = float(np.abs(np.asarray(got, np.float64) - ref).max())
    scale = float(np.abs(ref).max()) or 1.0
    assert np.isfinite(np.asarray(got)).all(), "non-finite output"
    assert err <= rtol * scale, f"max abs err {err} > {rtol} * {scale}"
    return err / scale
