"""Inference-attention operators over CUDA tensors -- the B200 counterpart of the
reference's ``python/flash_engine/ops.py:15-143``.

Same function names, argument order and meaning as the reference:

* ``flash_attention(q, k, v, is_causal=False, scale=None)``       (ops.py:15-57)
* ``paged_attention(query, key_cache, value_cache, block_tables,
  context_lens, block_size=16, scale=None)``                       (ops.py:59-101)
* ``flash_decoding(query, key, value, num_splits=4, scale=None)`` (ops.py:103-143)

Differences, all deliberate:

* Inputs must be CUDA tensors; there is no NumPy/torch fallback (the reference's
  CPU code is the test oracle under ``oracle/``). Non-CUDA inputs raise TypeError.
* ``paged_attention`` supports GQA (num_heads a multiple of num_kv_heads, query
  head h reading KV head h // (H / Hkv), as src/paged_attention.cu:33-35) and
  bf16 / fp16 / fp32 caches.
* Every kernel runs on the current torch CUDA stream; tensors must be contiguous.
"""

from __future__ import annotations

import contextlib
import math

import torch

from . import _lib

_lib_c = _lib.lib


def _on(device):
    """Context that makes `device` current, or nothing when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _stream():
    return ctypes_stream(torch.cuda.current_stream())


def ctypes_stream(s) -> int:
    return int(s.cuda_stream)


def _ptr(t: torch.Tensor) -> int:
    return int(t.data_ptr())


def _require_cuda(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise TypeError("flash_engine operators take CUDA tensors; the CPU reference "
                            "implementation is test infrastructure, not a fallback")
        if not t.is_contiguous():
            raise ValueError("tensors must be contiguous")


def _scale_arg(scale, d):
    return float(scale) if scale is not None else 1.0 / math.sqrt(d)


# --------------------------------------------------------------------------- prefill
def rope(x, cos, sin, out=None):
    """Rotary position embedding of x [B, H, seq, d] (float32, bfloat16 or float16): row
    (b, h, i) is rotated at position i, pairs (2j, 2j+1) -> (x0 c - x1 s, x0 s + x1 c) with
    the float32 tables cos/sin [>= seq, d/2] (the reference's fused RoPE kernel,
    src/fused_rope.cu:13-45). ``out`` may be x (in place). Returns out."""
    _require_cuda(x, cos, sin)
    B, H, N, d = x.shape
    if cos.dtype != torch.float32 or cos.shape != sin.shape or cos.dim() != 2 or \
            cos.shape[1] != d // 2 or cos.shape[0] < N:
        raise ValueError("rope tables must be float32 [max_pos >= seq, d/2]")
    dt = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}.get(x.dtype)
    if dt is None:
        raise TypeError(f"unsupported dtype {x.dtype}")
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor like x")
    with _on(x.device):
        _lib.check(_lib_c.fe_rope_forward(_ptr(x), _ptr(cos), _ptr(sin), _ptr(out), B, H, N, d,
                                          dt, _stream()), "rope")
    return out


def flash_attention(q, k, v, is_causal: bool = False, scale: float | None = None, *,
                    out=None, rope=None, k_rotated=None):
    """FA2 forward: softmax(q k^T * scale [+ top-left causal mask]) v.

    q: [B, H, N, d]; k, v: [B, H, M, d]; dtype float32, bfloat16 or float16. ``out``
    (optional, new): a contiguous tensor like q to write into. ``rope=(cos, sin)``
    (optional, new; bf16/fp16): float32 CUDA tables [max_pos, d/2] with max_pos >= N, M;
    query row i and key row j are rotated at positions i and j (the reference's fused
    RoPE arithmetic, applied to Q and K) by the streaming RoPE pass into a temporary
    like q and into ``k_rotated`` (a tensor like k, made here if not given; it then holds
    the rotated keys a KV cache stores), which the attention kernel reads.
    """
    _require_cuda(q, k, v)
    B, H, N, d = q.shape
    M = k.shape[2]
    if k.shape != (B, H, M, d) or v.shape != k.shape:
        raise ValueError("k and v must be [B, H, M, d] matching q")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share a dtype")
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor like q")
    if rope is not None:
        if q.dtype not in (torch.bfloat16, torch.float16):
            raise TypeError("rope is supported for bfloat16 / float16 attention")
        rcos, rsin = rope
        _require_cuda(rcos, rsin)
        if rcos.dtype != torch.float32 or rcos.shape != rsin.shape or rcos.dim() != 2 or \
                rcos.shape[1] != d // 2 or rcos.shape[0] < max(N, M):
            raise ValueError("rope tables must be float32 [max_pos >= max(N, M), d/2]")
        if k_rotated is None:
            k_rotated = torch.empty_like(k)
        elif k_rotated.shape != k.shape or k_rotated.dtype != k.dtype or \
                not k_rotated.is_contiguous():
            raise ValueError("k_rotated must be a contiguous tensor like k")
        with _on(q.device):
            _lib.check(_lib_c.fe_flash_attention_forward_ex(
                _ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, N, M, d, int(bool(is_causal)),
                _scale_arg(scale, d), 0 if q.dtype == torch.bfloat16 else 1, _ptr(rcos),
                _ptr(rsin), rcos.shape[0], _ptr(torch.empty_like(q)), _ptr(k_rotated),
                _stream()), "flash_attention")
        return out
    fn = {torch.float32: _lib_c.fe_flash_attention_forward_fp32,
          torch.bfloat16: _lib_c.fe_flash_attention_forward_bf16,
          torch.float16: _lib_c.fe_flash_attention_forward_fp16}.get(q.dtype)
    if fn is None:
        raise TypeError(f"unsupported dtype {q.dtype}")
    with _on(q.device):
        _lib.check(fn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, N, M, d, int(bool(is_causal)),
                      _scale_arg(scale, d), _stream()), "flash_attention")
    return out


def naive_attention(q, k, v, is_causal: bool = False, scale: float | None = None):
    """Row-per-thread fp32 attention (the reference's naive baseline kernel)."""
    _require_cuda(q, k, v)
    if q.dtype != torch.float32:
        raise TypeError("naive_attention is fp32 only")
    B, H, N, d = q.shape
    M = k.shape[2]
    out = torch.empty_like(q)
    with _on(q.device):
        _lib.check(_lib_c.fe_naive_attention_forward_fp32(
            _ptr(q), _ptr(k), _ptr(v), _ptr(out), B, H, N, M, d, int(bool(is_causal)),
            _scale_arg(scale, d), _stream()), "naive_attention")
    return out


# --------------------------------------------------------------------------- paged
def _paged_shapes(query, key_cache, value_cache, block_tables, context_lens, block_size,
                  kv_layout="flat"):
    S, H, d = query.shape
    if kv_layout == "flat":
        nb, Hkv, bs, d2 = key_cache.shape
        ok = bs == block_size and d2 == d and value_cache.shape == key_cache.shape
    elif kv_layout == "vllm":
        nb, Hkv, dx, bs, x = key_cache.shape
        ok = (bs == block_size and dx * x == d and x == 8
              and tuple(value_cache.shape) == (nb, Hkv, d, bs))
    else:
        raise ValueError("kv_layout must be 'flat' or 'vllm'")
    if not ok:
        raise ValueError("cache shape does not match the layout: flat K/V [num_blocks, Hkv, "
                         "block_size, d]; vllm K [num_blocks, Hkv, d/8, block_size, 8], "
                         "V [num_blocks, Hkv, d, block_size]")
    if H % Hkv:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise TypeError("block_tables and context_lens must be int32")
    if block_tables.dim() != 2 or block_tables.shape[0] != S or context_lens.shape != (S,):
        raise ValueError("block_tables [S, max_blocks] and context_lens [S] expected")
    return S, H, Hkv, d, nb, block_tables.shape[1]


def paged_attention_workspace_floats(num_heads, num_kv_heads, head_dim, block_size=16) -> int:
    """Float32 elements of workspace the split-KV decode needs on the current device
    for this head configuration (independent of batch, context lengths and dtype).

    Allocate it zero-filled (``torch.zeros``): its first 4 KiB hold arrival counters
    that must be zero when a call starts, and every call leaves them at zero, so one
    workspace serves any number of calls and head configurations (one stream at a
    time)."""
    n = int(_lib_c.fe_paged_attention_v2_workspace_floats(num_heads, num_kv_heads, head_dim,
                                                          block_size))
    if n == 0:
        raise ValueError("unsupported head configuration for the split-KV decode")
    return n


# One zero-filled workspace per (device, stream), made on the first call without a
# caller workspace and kept for the life of the process: it is sized for every
# supported head configuration, so it is never replaced (a CUDA graph that captured it
# keeps a valid buffer), and calls on one stream are ordered, so they can share it.
_WS_CACHE: dict = {}
_WS_MAX: dict = {}
# workspace_floats that asks the library for the stream's slot of its own scratch
# (FE_WORKSPACE_LIBRARY of flash_engine_c.h, with a NULL workspace)
WORKSPACE_LIBRARY = (1 << 64) - 1


def _max_workspace_floats(device_index: int) -> int:
    n = _WS_MAX.get(device_index)
    if n is None:
        n = max(int(_lib_c.fe_paged_attention_v2_workspace_floats(h, 1, d, bs))
                for h in (1, 16) for d in (64, 128) for bs in (16, 32))
        _WS_MAX[device_index] = n
    return n


def _workspace(query, H, Hkv, d, bs, workspace):
    """(workspace tensor, floats), or (None, WORKSPACE_LIBRARY) while the stream is being
    captured before it has a cached workspace: nothing may be allocated and zero-filled
    then, so the call uses the stream's slot of the library's own scratch."""
    if workspace is None:
        stream = torch.cuda.current_stream(query.device)
        key = (query.device.index, int(stream.cuda_stream))
        ws = _WS_CACHE.get(key)
        if ws is None:
            if torch.cuda.is_current_stream_capturing():
                return None, WORKSPACE_LIBRARY
            with _on(query.device):
                n = _max_workspace_floats(query.device.index)
                ws = torch.zeros(n, dtype=torch.float32, device=query.device)
            _WS_CACHE[key] = ws
        return ws, ws.numel()
    n = paged_attention_workspace_floats(H, Hkv, d, bs)
    if workspace.dtype != torch.float32 or workspace.numel() < n or not workspace.is_cuda:
        raise ValueError(f"workspace must be a CUDA float32 tensor of >= {n} elements")
    return workspace, workspace.numel()


def _persistent_decode_ok(query, key_cache, value_cache, out, d, block_size, kv_layout):
    """Shapes the persistent split-KV decode takes (else the generic fp32 kernel)."""
    if d not in (64, 128) or block_size not in (16, 32):
        return False
    if query.dtype == torch.float32:
        return (kv_layout == "flat" and key_cache.data_ptr() % 16 == 0
                and value_cache.data_ptr() % 16 == 0
                and query.data_ptr() % (16 if d == 128 else 8) == 0)
    return True


def paged_attention(query, key_cache, value_cache, block_tables, context_lens,
                    block_size: int = 16, scale: float | None = None, *,
                    max_context_len: int | None = None, out=None, workspace=None,
                    version: str = "auto", kv_layout: str = "flat", rope=None):
    """Paged-KV decode attention (one query token per sequence).

    query [S, H, d]; block_tables [S, max_blocks] int32; context_lens [S] int32.
    Returns [S, H, d]. Cache layouts (``kv_layout``):
      "flat" -- K and V [num_blocks, Hkv, block_size, d] (the reference's fp32 layout);
      "vllm" -- K [num_blocks, Hkv, d/8, block_size, 8], V [num_blocks, Hkv, d,
                block_size] (vLLM's x-packed layout; bf16/fp16, block_size 16).
    The persistent split-KV kernel runs bf16, fp16 and fp32 caches (``version``
    "auto"/"v2"; fp32 with head_dim 64 or 128, block size 16 or 32, 16-byte aligned
    caches) on a zero-filled float32 ``workspace`` of
    ``paged_attention_workspace_floats(...)`` elements. Without one, the call uses a
    workspace cached for the current (device, stream), made on the first such call.
    A first call on a stream that is being captured into a CUDA graph uses the stream's
    slot of the library's own scratch instead (nothing is allocated during a capture).
    ``version="v1"`` runs the single-pass kernel (no workspace). Other fp32 shapes run
    the generic single-pass fp32 kernel.

    ``rope=(cos, sin)`` (bf16/fp16): float32 CUDA tables [max_pos, d/2]; each query is
    rotated at position context_len - 1 inside the kernel (pairs (2i, 2i+1), the
    arithmetic of the reference's fused RoPE). Cached keys are taken as already rotated.
    """
    _require_cuda(query, key_cache, value_cache, block_tables, context_lens)
    S, H, Hkv, d, nb, maxb = _paged_shapes(query, key_cache, value_cache, block_tables,
                                           context_lens, block_size, kv_layout)
    if out is None:
        out = torch.empty_like(query)
    sc = _scale_arg(scale, d)
    if max_context_len is None:
        max_context_len = maxb * block_size
    if query.dtype == torch.float32 and kv_layout != "flat":
        raise ValueError("the fp32 decode takes the flat cache layout")
    with _on(query.device):
        if query.dtype == torch.float32 and not _persistent_decode_ok(
                query, key_cache, value_cache, out, d, block_size, kv_layout):
            if rope is not None:
                raise ValueError("rope with an fp32 cache needs head_dim 64/128, block size "
                                 "16/32 and 16-byte aligned tensors")
            _lib.check(_lib_c.fe_paged_attention_v1_fp32(
                _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(out), _ptr(block_tables),
                _ptr(context_lens), S, H, Hkv, d, block_size, int(max_context_len), maxb, nb, sc,
                _stream()), "paged_attention")
        elif query.dtype in (torch.bfloat16, torch.float16, torch.float32):
            dt = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[query.dtype]
            lay = 0 if kv_layout == "flat" else 1
            if version == "v1":
                ws, n = None, 0
            else:
                ws, n = _workspace(query, H, Hkv, d, block_size, workspace)
            rc, rs, rmax = None, None, 0
            if rope is not None:
                rcos, rsin = rope
                _require_cuda(rcos, rsin)
                if rcos.dtype != torch.float32 or rcos.shape != rsin.shape or \
                        rcos.dim() != 2 or rcos.shape[1] != d // 2:
                    raise ValueError("rope tables must be float32 [max_pos, d/2]")
                rc, rs, rmax = _ptr(rcos), _ptr(rsin), rcos.shape[0]
            _lib.check(_lib_c.fe_paged_attention_ex(
                _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(out), _ptr(block_tables),
                _ptr(context_lens), S, H, Hkv, d, block_size, maxb, nb, sc, dt, lay, rc, rs, rmax,
                _ptr(ws) if ws is not None else None, n, _stream()), "paged_attention")
        else:
            raise TypeError(f"unsupported dtype {query.dtype}")
    return out


def paged_kv_append(k_new, v_new, key_cache, value_cache, block_tables, context_lens,
                    block_size: int = 16, *, kv_layout: str = "flat", rope=None):
    """Writes the decode step's new token into the paged cache: K and V rows
    k_new / v_new [S, Hkv, d] of sequence s go to position context_lens[s] - 1 (block
    block_tables[s, pos // block_size], row pos % block_size). ``rope=(cos, sin)``: float32
    CUDA tables [max_pos, d/2]; the key is rotated at that position first (the reference's
    fused RoPE arithmetic), so with the same tables passed to ``paged_attention`` both the
    query and the keys carry the embedding. Returns the caches."""
    _require_cuda(k_new, v_new, key_cache, value_cache, block_tables, context_lens)
    S, Hkv, d = k_new.shape
    if v_new.shape != k_new.shape or k_new.dtype != key_cache.dtype or \
            v_new.dtype != key_cache.dtype:
        raise ValueError("k_new / v_new must be [S, Hkv, d] of the cache dtype")
    dummy_q = k_new.new_empty((S, Hkv, d))
    _, _, Hkv2, d2, nb, maxb = _paged_shapes(dummy_q, key_cache, value_cache, block_tables,
                                             context_lens, block_size, kv_layout)
    if Hkv2 != Hkv or d2 != d:
        raise ValueError("k_new does not match the cache's KV heads / head_dim")
    dt = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}.get(k_new.dtype)
    if dt is None:
        raise TypeError(f"unsupported dtype {k_new.dtype}")
    rc, rs, rmax = None, None, 0
    if rope is not None:
        rcos, rsin = rope
        _require_cuda(rcos, rsin)
        if rcos.dtype != torch.float32 or rcos.shape != rsin.shape or rcos.dim() != 2 or \
                rcos.shape[1] != d // 2:
            raise ValueError("rope tables must be float32 [max_pos, d/2]")
        rc, rs, rmax = _ptr(rcos), _ptr(rsin), rcos.shape[0]
    with _on(k_new.device):
        _lib.check(_lib_c.fe_paged_kv_append(
            _ptr(k_new), _ptr(v_new), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
            _ptr(context_lens), S, Hkv, d, block_size, maxb, nb, dt,
            0 if kv_layout == "flat" else 1, rc, rs, rmax, _stream()), "paged_kv_append")
    return key_cache, value_cache


def paged_decode_partials(query, key_cache, value_cache, block_tables, context_lens,
                          token_begin: int, token_end: int, block_size: int = 16,
                          scale: float | None = None, workspace=None, out=None, out_stats=None):
    """Partial attention of every (sequence, query head) over the token window
    [token_begin, token_end) (bf16 cache; token_begin a multiple of block_size).

    Returns (O [S, H, d] f32 unnormalised, stats [S, H, 2] f32 = (m log2, l)); an
    empty window gives (0, (-inf, 0)). ``workspace`` as for ``paged_attention``."""
    _require_cuda(query, key_cache, value_cache, block_tables, context_lens)
    S, H, Hkv, d, nb, maxb = _paged_shapes(query, key_cache, value_cache, block_tables,
                                           context_lens, block_size)
    dev = query.device
    ws, n = _workspace(query, H, Hkv, d, block_size, workspace)
    if out is None:
        out = torch.empty((S, H, d), dtype=torch.float32, device=dev)
    if out_stats is None:
        out_stats = torch.empty((S, H, 2), dtype=torch.float32, device=dev)
    with _on(dev):
        _lib.check(_lib_c.fe_paged_decode_partials_bf16(
            _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
            _ptr(context_lens), S, H, Hkv, d, block_size, maxb, nb, _scale_arg(scale, d),
            int(token_begin), int(token_end), _ptr(ws) if ws is not None else None, n,
            _ptr(out), _ptr(out_stats),
            _stream()), "paged_decode_partials")
    return out, out_stats


def paged_decode_kv_exchange(query, key_cache, value_cache, block_tables, context_lens,
                             token_begin: int, token_end: int, xbufs, rank: int, max_rows: int,
                             block_size: int = 16, scale: float | None = None, workspace=None,
                             out=None, phases: int = 3):
    """KV-range decode step with the all-gather done over peer memory (bf16 cache).

    ``xbufs``: device addresses (ints) of every rank's exchange buffer as mapped in
    this process (``xbufs[rank]`` is this rank's own), each of
    ``fe_kv_exchange_bytes(len(xbufs), max_rows, d)`` bytes, zero-filled at creation
    (``sharding.KVRangeExchange`` manages them). ``phases`` 1: decode the window
    [token_begin, token_end) and store this rank's partial rows into every buffer;
    2: wait for every rank's rows and merge them into ``out`` [S, H, d] bf16; 3: both.
    Returns ``out``."""
    import ctypes

    _require_cuda(query, key_cache, value_cache, block_tables, context_lens)
    if query.dtype != torch.bfloat16:
        raise TypeError("the KV-range exchange decode takes bf16")
    S, H, Hkv, d, nb, maxb = _paged_shapes(query, key_cache, value_cache, block_tables,
                                           context_lens, block_size)
    ws, n = _workspace(query, H, Hkv, d, block_size, workspace)
    if out is None:
        out = torch.empty_like(query)
    arr = (ctypes.c_void_p * len(xbufs))(*[int(x) for x in xbufs])
    with _on(query.device):
        _lib.check(_lib_c.fe_paged_decode_kv_exchange_bf16(
            _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
            _ptr(context_lens), S, H, Hkv, d, block_size, maxb, nb, _scale_arg(scale, d),
            int(token_begin), int(token_end), _ptr(ws) if ws is not None else None, n, arr,
            len(xbufs), int(rank),
            int(max_rows), _ptr(out), int(phases), _stream()), "paged_decode_kv_exchange")
    return out


def paged_decode_kv_exchange_prepared(query, key_cache, value_cache, block_tables,
                                      context_lens, token_begin: int, token_end: int, xbufs,
                                      rank: int, max_rows: int, block_size: int = 16,
                                      scale: float | None = None, workspace=None, out=None):
    """``paged_decode_kv_exchange`` (both phases) with its arguments checked and converted
    once: returns a function of no arguments that runs one step on the stream current at
    this call and returns ``out``. For loops that decode into the same tensors step after
    step (their data may change, not their shapes or storage), where the per-call checks
    and argument conversion would cost as much host time as the step's GPU work."""
    import ctypes

    _require_cuda(query, key_cache, value_cache, block_tables, context_lens)
    if query.dtype != torch.bfloat16:
        raise TypeError("the KV-range exchange decode takes bf16")
    S, H, Hkv, d, nb, maxb = _paged_shapes(query, key_cache, value_cache, block_tables,
                                           context_lens, block_size)
    ws, n = _workspace(query, H, Hkv, d, block_size, workspace)
    if out is None:
        out = torch.empty_like(query)
    arr = (ctypes.c_void_p * len(xbufs))(*[int(x) for x in xbufs])
    with _on(query.device):
        stream = _stream()
    fn = _lib_c.fe_paged_decode_kv_exchange_bf16
    args = [_ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(block_tables),
            _ptr(context_lens), S, H, Hkv, d, block_size, maxb, nb, _scale_arg(scale, d),
            int(token_begin), int(token_end), _ptr(ws) if ws is not None else None, n, arr,
            len(xbufs), int(rank), int(max_rows), _ptr(out), 3, stream]
    # convert once to the declared ctypes argument types
    cargs = tuple(a if isinstance(a, ctypes.Array) or a is None else t(a)
                  for a, t in zip(args, fn.argtypes))
    keep = (query, key_cache, value_cache, block_tables, context_lens, ws, out, arr)

    def step():
        _ = keep
        st = fn(*cargs)
        if st != 0:
            _lib.check(st, "paged_decode_kv_exchange")
        return out

    return step


def merge_partials(part_out, part_stats, ranks: int, parts_per_rank: int, out_dtype: str = "bf16",
                   out=None, out_stats=None):
    """Log-sum-exp combine of partials laid out [ranks, rows, parts_per_rank, d]
    (and [..., 2] stats). out_dtype: "fp32" | "bf16" | "fp16" (final output rows
    [rows, d]) or "partial" (returns (O, stats) merged partials)."""
    _require_cuda(part_out, part_stats)
    d = part_out.shape[-1]
    rows = part_out.numel() // (d * ranks * parts_per_rank)
    code = {"fp32": 0, "bf16": 1, "partial": 2, "fp16": 3}[out_dtype]
    dt = {0: torch.float32, 1: torch.bfloat16, 2: torch.float32, 3: torch.float16}[code]
    if out is None:
        out = torch.empty((rows, d), dtype=dt, device=part_out.device)
    if code == 2 and out_stats is None:
        out_stats = torch.empty((rows, 2), dtype=torch.float32, device=part_out.device)
    with _on(part_out.device):
        _lib.check(_lib_c.fe_merge_partials(
            _ptr(part_out), _ptr(part_stats), rows, ranks, parts_per_rank, d, _ptr(out),
            _ptr(out_stats) if out_stats is not None else None, code, _stream()),
            "merge_partials")
    return (out, out_stats) if code == 2 else out


# --------------------------------------------------------------------------- decoding
def flash_decoding(query, key, value, num_splits: int = 4, scale: float | None = None,
                   scratch=None):
    """Two-stage split-KV decoding over a dense cache (fp32).

    query [B, H, 1, d]; key/value [B, H, M, d]. Returns [B, H, 1, d]. Split s
    covers [s*ceil(M/S), min(M, (s+1)*ceil(M/S))) (ops.py:112-121).
    """
    _require_cuda(query, key, value)
    B, H, one, d = query.shape
    M = key.shape[2]
    if one != 1 or key.shape != (B, H, M, d) or value.shape != key.shape:
        raise ValueError("query [B,H,1,d] and key/value [B,H,M,d] expected")
    if query.dtype != torch.float32:
        raise TypeError("flash_decoding takes float32 tensors (as the reference's kernel)")
    out = torch.empty_like(query)
    if scratch is None:
        so = torch.empty((B, H, num_splits, d), dtype=torch.float32, device=query.device)
        ss = torch.empty((B, H, num_splits, 2), dtype=torch.float32, device=query.device)
    else:
        so, ss = scratch
    with _on(query.device):
        _lib.check(_lib_c.fe_flash_decoding_forward_fp32(
            _ptr(query), _ptr(key), _ptr(value), _ptr(out), _ptr(so), _ptr(ss), B, H, M, d,
            int(num_splits), _scale_arg(scale, d), _stream()), "flash_decoding")
    return out


def device_errors() -> int:
    """Synchronise, then return and clear the device error word (0 = no error)."""
    return _lib.device_errors()


def get_version() -> str:
    return _lib_c.fe_get_version().decode()
