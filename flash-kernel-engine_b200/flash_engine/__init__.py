"""FlashKernel-Engine inference attention for NVIDIA B200 (sm_100a).

Drop-in for the attention part of the reference's ``flash_engine`` package
(``python/flash_engine/__init__.py``): ``flash_attention``, ``paged_attention`` and
``flash_decoding`` with the same names and arguments, implemented by
``libflash_engine_b200.so`` (hand-written sm_100a kernels behind a C ABI).
"""

from .ops import (  # noqa: F401
    device_errors,
    flash_attention,
    flash_decoding,
    get_version,
    merge_partials,
    naive_attention,
    paged_attention,
    paged_attention_workspace_floats,
    paged_decode_partials,
    paged_kv_append,
    rope,
)

__version__ = "1.2.0"

__all__ = [
    "flash_attention",
    "paged_attention",
    "flash_decoding",
    "naive_attention",
    "paged_decode_partials",
    "paged_kv_append",
    "rope",
    "merge_partials",
    "paged_attention_workspace_floats",
    "device_errors",
    "get_version",
]
