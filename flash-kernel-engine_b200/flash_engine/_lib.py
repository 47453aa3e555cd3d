"""ctypes binding of libflash_engine_b200.so (the C ABI in include/flash_engine_c.h).

The library is required: importing this module raises ImportError when the shared
object is missing, and every wrapper raises RuntimeError on a non-zero status. There
is no CPU fallback anywhere in the package.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# FLASH_ENGINE_LIB may point at another build of the same library (e.g. one
# compiled with -DFE_DEBUG_CHECKS, which adds device-side bounds checks).
LIB_PATH = os.environ.get("FLASH_ENGINE_LIB") or os.path.join(_HERE, "lib",
                                                              "libflash_engine_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"libflash_engine_b200.so not found at {LIB_PATH}; build it with "
        "`make -C flash-kernel-engine_b200/csrc` (or __graft_entry__.build())")

lib = ctypes.CDLL(LIB_PATH)

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_LL = ctypes.c_longlong

_SIGS = {
    "fe_get_version": ([], ctypes.c_char_p),
    "fe_print_device_info": ([_I], _I),
    "fe_get_device_errors": ([ctypes.POINTER(ctypes.c_uint)], _I),
    "fe_flash_attention_forward_fp32": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P], _I),
    "fe_flash_attention_forward_fp16": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P], _I),
    "fe_flash_attention_forward_bf16": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P], _I),
    "fe_naive_attention_forward_fp32": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P], _I),
    "fe_flash_attention_forward_ex": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _I, _P, _P, _I,
                                       _P, _P, _P], _I),
    "fe_rope_forward": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "fe_paged_attention_v1_fp32": ([_P, _P, _P, _P, _P, _P] + [_I] * 8 + [_F, _P], _I),
    "fe_paged_attention_v1_fp16": ([_P, _P, _P, _P, _P, _P] + [_I] * 8 + [_F, _P], _I),
    "fe_paged_attention_v1_bf16": ([_P, _P, _P, _P, _P, _P] + [_I] * 8 + [_F, _P], _I),
    "fe_paged_attention_v2_bf16": ([_P] * 6 + [_I] * 8 + [_F, _P, ctypes.c_size_t, _P], _I),
    "fe_paged_attention_v2_workspace_floats": ([_I] * 4, ctypes.c_size_t),
    "fe_paged_kv_append": ([_P] * 6 + [_I] * 8 + [_P, _P, _I, _P], _I),
    "fe_paged_attention_ex": ([_P] * 6 + [_I] * 7 + [_F, _I, _I, _P, _P, _I, _P,
                                                     ctypes.c_size_t, _P], _I),
    "fe_paged_attention_v2_bf16_noalloc": ([_P] * 6 + [_I] * 8 + [_F, _P], _I),
    "fe_flash_decoding_forward_fp32": ([_P] * 6 + [_I] * 5 + [_F, _P], _I),
    "fe_paged_decode_partials_bf16": ([_P] * 5 + [_I] * 7 + [_F, _I, _I, _P, ctypes.c_size_t,
                                                              _P, _P, _P], _I),
    "fe_merge_partials": ([_P, _P, _I, _I, _I, _I, _P, _P, _I, _P], _I),
    "fe_kv_exchange_bytes": ([_I, _I, _I], ctypes.c_size_t),
    "fe_kv_exchange_alloc": ([ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)], _I),
    "fe_kv_exchange_free": ([_P], _I),
    "fe_kv_exchange_ipc_handle": ([_P, _P], _I),
    "fe_kv_exchange_ipc_open": ([_P, ctypes.POINTER(ctypes.c_void_p)], _I),
    "fe_kv_exchange_ipc_close": ([_P], _I),
    "fe_paged_decode_kv_exchange_bf16": ([_P] * 5 + [_I] * 7 + [_F, _I, _I, _P, ctypes.c_size_t,
                                                                 _P, _I, _I, _I, _P, _I, _P],
                                         _I),
    "fe_nccl_unique_id": ([_P], _I),
    "fe_nccl_comm_init": ([ctypes.POINTER(ctypes.c_void_p), _I, _P, _I], _I),
    "fe_nccl_comm_destroy": ([_P], _I),
    "fe_kv_range_nccl_scratch_floats": ([_I, _I, _I, _I], ctypes.c_size_t),
    "fe_paged_decode_kv_range_nccl_bf16": ([_P] * 5 + [_I] * 7 + [_F, _I, _P, ctypes.c_size_t,
                                                                   _P, _I, _I, _P, ctypes.c_size_t,
                                                                   _P, _P], _I),
    "fe_graph_capture": ([None, _P, _P, ctypes.POINTER(ctypes.c_void_p)], _I),
    "fe_graph_launch": ([_P, _P], _I),
    "fe_graph_destroy": ([_P], None),
}

# void record(void* stream, void* user): the step recorded by fe_graph_capture
RECORD_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_void_p)

for _name, (_args, _res) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = [RECORD_FN if a is None else a for a in _args]
    _fn.restype = _res

EXPORTED = tuple(_SIGS)

_CUDA_ERRORS = {
    1: "cudaErrorInvalidValue (unsupported arguments)",
    2: "cudaErrorMemoryAllocation",
    3: "cudaErrorInitializationError",
    9: "cudaErrorInvalidConfiguration",
    98: "cudaErrorInvalidDeviceFunction",
    209: "cudaErrorNoKernelImageForDevice",
    400: "cudaErrorInvalidResourceHandle",
    801: "cudaErrorNotSupported",
}


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"{what} failed: CUDA error {status} "
                           f"({_CUDA_ERRORS.get(status, 'see cudaError_t')})")


def device_errors() -> int:
    """Synchronise and return (and clear) the library's device error word."""
    v = ctypes.c_uint(0)
    check(lib.fe_get_device_errors(ctypes.byref(v)), "fe_get_device_errors")
    return int(v.value)


ERR_WAIT_TIMEOUT = 1
ERR_BAD_BLOCK = 2
ERR_TMEM = 4
ERR_WORKSPACE = 8
