"""``flash_engine_cuda`` -- the extension module of the reference's
``python/bindings.cpp:135-140``, served by libflash_engine_b200.so.

Each entry keeps the binding's contract (``bindings.cpp:10-57``): CUDA and contiguity
checks that raise ``RuntimeError`` with the binding's messages (as ``TORCH_CHECK``
does), the output allocated like ``torch::empty_like(q)``, and the launch on the
current stream. It adds what the binding lacks: bf16 inputs (besides fp32 and fp16) and
a checked launch status. ``paged_attention_forward`` and ``flash_decoding_forward`` are
entries for the two decode operators the reference only has in NumPy.
``fused_rmsnorm_forward`` / ``fused_swiglu_forward`` exist because the reference's
``ops.py`` calls them whenever the extension imports; those kernels are not part of
this attention library, so after the binding's checks they raise NotImplementedError.
"""

import torch

from flash_engine import ops as _ops

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_cuda_contiguous(**tensors):
    for name, t in tensors.items():
        _check(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")
    for name, t in tensors.items():
        _check(t.is_contiguous(), f"{name} must be contiguous")


def flash_attention_forward(q, k, v, is_causal):
    """O = softmax(Q K^T / sqrt(d) [+ causal mask]) V for [B, H, N|M, d] tensors."""
    _check_cuda_contiguous(Q=q, K=k, V=v)
    _check(q.dtype in _DTYPES and k.dtype == q.dtype and v.dtype == q.dtype,
           "Unsupported scalar type for FlashAttention: only Float, Half and BFloat16 "
           "are supported")
    out = torch.empty_like(q)
    return _ops.flash_attention(q, k, v, bool(is_causal), out=out)


def paged_attention_forward(query, key_cache, value_cache, block_tables, context_lens,
                            block_size=16, scale=None):
    """vLLM-style paged decode: query [S, H, d], caches [blocks, Hkv, block_size, d]."""
    _check_cuda_contiguous(query=query, key_cache=key_cache, value_cache=value_cache,
                           block_tables=block_tables, context_lens=context_lens)
    _check(query.dtype in _DTYPES, "Unsupported scalar type for paged attention: only "
           "Float, Half and BFloat16 are supported")
    _check(block_tables.dtype == torch.int32 and context_lens.dtype == torch.int32,
           "block_tables and context_lens must be int32")
    out = torch.empty_like(query)
    return _ops.paged_attention(query, key_cache, value_cache, block_tables, context_lens,
                                block_size, scale, out=out)


def flash_decoding_forward(query, key, value, num_splits=4, scale=None):
    """Split-KV decoding with the log-sum-exp combine over a dense cache."""
    _check_cuda_contiguous(query=query, key=key, value=value)
    return _ops.flash_decoding(query, key, value, num_splits, scale)


def fused_rmsnorm_forward(x, gamma, eps):
    _check_cuda_contiguous(x=x, gamma=gamma)
    raise NotImplementedError("fused RMSNorm is not part of the B200 attention library")


def fused_swiglu_forward(gate, up):
    _check_cuda_contiguous(gate=gate, up=up)
    raise NotImplementedError("fused SwiGLU is not part of the B200 attention library")
