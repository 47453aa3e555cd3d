"""``flash_engine_cuda`` -- the extension-module names of the reference's
``python/bindings.cpp:135-140``, served by libflash_engine_b200.so.

``flash_attention_forward(q, k, v, is_causal)`` keeps the binding's contract
(CUDA + contiguous checks raising, output allocated like ``torch::empty_like``,
current-stream launch) and adds what the binding lacks: bf16 inputs and a
checked launch status. ``paged_attention_forward`` and ``flash_decoding_forward``
are new entries for the two decode operators the reference only has in NumPy.
``fused_rmsnorm_forward`` / ``fused_swiglu_forward`` exist because the reference's
``ops.py`` calls them whenever the extension imports; those kernels are not part
of this attention library, so they raise NotImplementedError.
"""

from flash_engine import ops as _ops


def flash_attention_forward(q, k, v, is_causal):
    return _ops.flash_attention(q, k, v, bool(is_causal))


def paged_attention_forward(query, key_cache, value_cache, block_tables, context_lens,
                            block_size=16, scale=None):
    return _ops.paged_attention(query, key_cache, value_cache, block_tables, context_lens,
                                block_size, scale)


def flash_decoding_forward(query, key, value, num_splits=4, scale=None):
    return _ops.flash_decoding(query, key, value, num_splits, scale)


def fused_rmsnorm_forward(x, gamma, eps):
    raise NotImplementedError("fused RMSNorm is not part of the B200 attention library")


def fused_swiglu_forward(gate, up):
    raise NotImplementedError("fused SwiGLU is not part of the B200 attention library")
