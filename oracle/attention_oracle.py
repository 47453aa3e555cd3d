"""CPU oracle for the inference-attention hot path.

TEST INFRASTRUCTURE ONLY. This module is the parity checker: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it. The product path (``flash_engine`` and the
``libflash_engine_b200.so`` C-ABI) never calls into it and has no CPU fallback.

What it restates (NumPy, float64/float32 exactly as the reference does):

* ``flash_attention``  -- the NumPy branch of ``python/flash_engine/ops.py:48-57``
  (scores = Q K^T * scale; additive causal mask ``triu(full(N, M, -1e30), 1)``,
  top-left aligned; max-subtracted softmax; P V).
* ``paged_attention``  -- ``python/flash_engine/ops.py:59-101`` (per sequence:
  gather ``ceil(ctx/block_size)`` physical blocks through the block table,
  concatenate along the token axis, slice to ``ctx``, softmax attention; a
  sequence with ``ctx <= 0`` leaves its output row at zero).
* ``flash_decoding``   -- ``python/flash_engine/ops.py:103-143`` (split size
  ``ceil(M / S)``, empty splits skipped, per-split (O_s, m_s, l_s), then the
  log-sum-exp combine ``O = sum O_s e^{m_s-g} / sum l_s e^{m_s-g}``).

and adds the wrappers the reference's functions lack (none of which change the
arithmetic):

* GQA: ``ops.paged_attention`` broadcasts only for Hkv == 1 or Hkv == H. The
  kernel mapping is ``kv_head = head // (H / Hkv)`` (``src/paged_attention.cu:33-35``),
  so the wrapper calls the reference function once per KV-head group with
  ``query[:, g*G:(g+1)*G]`` and ``cache[:, g:g+1]``.
* Paged split-KV: gather through the block table (same rule as
  ``ops.py:80-90``) then ``flash_decoding`` per KV-head group.
* bf16: NumPy has no bf16, so inputs are rounded to bf16 (round to nearest
  even, the conversion ``__float2bfloat16_rn`` performs) and fed as float32.

Parity is pinned by ``tests/golden/*.npz``, produced by running the reference's
own ``ops.py`` (see ``tests/golden/make_golden.py``) and checked in
``tests/test_oracle.py``.
"""

from __future__ import annotations

import math

import numpy as np

NEG_MASK = -1e30  # the reference's additive mask value (ops.py:51)


# --------------------------------------------------------------------------
# bf16 helpers
# --------------------------------------------------------------------------

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); return float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding_bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding_bias) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    # NaN must stay NaN (the addition above could carry into the exponent).
    return np.where(np.isnan(x), x, out).astype(np.float32)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns (round to nearest even)."""
    r = bf16_round(x)
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32."""
    return (b.astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------
# Reference algorithms (restated)
# --------------------------------------------------------------------------

def flash_attention(q, k, v, is_causal: bool = False, scale: float | None = None):
    """Dense attention, NumPy branch of ``python/flash_engine/ops.py:33-57``.

    q: [B, H, N, d]; k, v: [B, H, M, d]. Returns [B, H, N, d].
    """
    B, H, N, d = q.shape
    M = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    scores = np.matmul(q, np.swapaxes(k, -2, -1)) * scale
    if is_causal:
        scores = scores + np.triu(np.full((N, M), NEG_MASK), k=1)
    m = np.max(scores, axis=-1, keepdims=True)
    e = np.exp(scores - m)
    probs = e / np.sum(e, axis=-1, keepdims=True)
    return np.matmul(probs, v)


def flash_attention_sliced(q, k, v, is_causal: bool = False, scale: float | None = None,
                           heads=None):
    """``flash_attention`` evaluated one (b, h) slice at a time.

    Same arithmetic per slice; used where the full [B, H, N, M] score tensor would
    not fit in host memory (the Llama-2-7B prefill shape). ``heads`` optionally
    restricts the evaluation to a list of (b, h) pairs; other rows stay zero.
    """
    B, H, N, d = q.shape
    out = np.zeros(q.shape, dtype=np.result_type(q, k, v))
    pairs = heads if heads is not None else [(b, h) for b in range(B) for h in range(H)]
    for b, h in pairs:
        out[b, h] = flash_attention(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                    v[b:b + 1, h:h + 1], is_causal, scale)[0, 0]
    return out


def paged_attention(query, key_cache, value_cache, block_tables, context_lens,
                    block_size: int = 16, scale: float | None = None):
    """PagedAttention v1, ``python/flash_engine/ops.py:59-101``.

    query: [S, H, d]; key_cache/value_cache: [num_blocks, Hkv, block_size, d];
    block_tables: [S, max_blocks] int32; context_lens: [S] int32.
    Valid for Hkv == H or Hkv == 1 (NumPy broadcasting), exactly like the reference.
    """
    num_seqs, num_heads, head_dim = query.shape
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    output = np.zeros_like(query)
    for b in range(num_seqs):
        ctx_len = int(context_lens[b])
        if ctx_len <= 0:
            continue
        nblk = (ctx_len + block_size - 1) // block_size
        k_chunks = [key_cache[block_tables[b, i]] for i in range(nblk)]
        v_chunks = [value_cache[block_tables[b, i]] for i in range(nblk)]
        k_seq = np.concatenate(k_chunks, axis=1)[:, :ctx_len, :]
        v_seq = np.concatenate(v_chunks, axis=1)[:, :ctx_len, :]
        q_b = query[b][:, np.newaxis, :]
        scores = np.matmul(q_b, np.swapaxes(k_seq, -2, -1)) * scale
        m = np.max(scores, axis=-1, keepdims=True)
        p = np.exp(scores - m)
        probs = p / np.sum(p, axis=-1, keepdims=True)
        output[b] = np.matmul(probs, v_seq).squeeze(1)
    return output


def flash_decoding(query, key, value, num_splits: int = 4, scale: float | None = None):
    """Two-stage split-KV decoding, ``python/flash_engine/ops.py:103-143``.

    query: [B, H, 1, d]; key/value: [B, H, M, d]. Returns [B, H, 1, d].
    """
    B, H, _, d = query.shape
    M = key.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    split_size = (M + num_splits - 1) // num_splits
    outs, maxs, sums = [], [], []
    for s in range(num_splits):
        start = s * split_size
        end = min(start + split_size, M)
        if start >= M:
            continue
        scores = np.matmul(query, np.swapaxes(key[:, :, start:end, :], -2, -1)) * scale
        m_s = np.max(scores, axis=-1, keepdims=True)
        p_s = np.exp(scores - m_s)
        outs.append(np.matmul(p_s, value[:, :, start:end, :]))
        maxs.append(m_s)
        sums.append(np.sum(p_s, axis=-1, keepdims=True))
    global_m = np.maximum.reduce(maxs)
    global_sum = np.zeros_like(sums[0])
    global_out = np.zeros_like(outs[0])
    for out_s, m_s, l_s in zip(outs, maxs, sums):
        rescale = np.exp(m_s - global_m)
        global_sum += l_s * rescale
        global_out += out_s * rescale
    return global_out / global_sum


# --------------------------------------------------------------------------
# Wrappers that close the reference's gaps (GQA, paged split-KV)
# --------------------------------------------------------------------------

def paged_attention_gqa(query, key_cache, value_cache, block_tables, context_lens,
                        block_size: int = 16, scale: float | None = None):
    """GQA paged decode: ``paged_attention`` per KV-head group.

    Query head h reads KV head ``h // (H // Hkv)`` (``src/paged_attention.cu:33-35``).
    """
    S, H, d = query.shape
    Hkv = key_cache.shape[1]
    if H % Hkv != 0:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    G = H // Hkv
    out = np.zeros_like(query)
    for g in range(Hkv):
        out[:, g * G:(g + 1) * G] = paged_attention(
            query[:, g * G:(g + 1) * G], key_cache[:, g:g + 1], value_cache[:, g:g + 1],
            block_tables, context_lens, block_size, scale)
    return out


def gather_paged(cache, block_tables, context_lens, seq: int, block_size: int = 16):
    """Dense [Hkv, ctx, d] view of one sequence's cache (``ops.py:80-90`` gather rule):
    logical token t lives at ``cache[block_tables[seq, t // bs], :, t % bs, :]``."""
    ctx = int(context_lens[seq])
    nblk = (ctx + block_size - 1) // block_size
    chunks = [cache[block_tables[seq, i]] for i in range(nblk)]
    return np.concatenate(chunks, axis=1)[:, :ctx, :]


def paged_flash_decoding_gqa(query, key_cache, value_cache, block_tables, context_lens,
                             num_splits: int, block_size: int = 16, scale: float | None = None):
    """Paged split-KV decode: gather each sequence, then ``flash_decoding`` per
    KV-head group (all sequences of one call must share one context length per
    ``flash_decoding``'s dense contract; sequences are processed one at a time)."""
    S, H, d = query.shape
    Hkv = key_cache.shape[1]
    G = H // Hkv
    out = np.zeros_like(query)
    for s in range(S):
        if int(context_lens[s]) <= 0:
            continue
        kd = gather_paged(key_cache, block_tables, context_lens, s, block_size)
        vd = gather_paged(value_cache, block_tables, context_lens, s, block_size)
        for g in range(Hkv):
            q = query[s, g * G:(g + 1) * G][None, :, None, :]           # [1, G, 1, d]
            kk = np.broadcast_to(kd[g][None, None], (1, G) + kd[g].shape)
            vv = np.broadcast_to(vd[g][None, None], (1, G) + vd[g].shape)
            out[s, g * G:(g + 1) * G] = flash_decoding(q, kk, vv, num_splits, scale)[0, :, 0, :]
    return out


def kv_range_partials(query, key_cache, value_cache, block_tables, context_lens,
                      token_begin: int, token_end: int, block_size: int = 16,
                      scale: float | None = None):
    """Stage-1 partial of one KV range for every (seq, q-head): returns
    (O_unnormalised [S, H, d], m [S, H] (natural-log units), l [S, H]).

    This is ``flash_decoding``'s per-split body (``ops.py:117-131``) over the
    token range [token_begin, min(token_end, ctx)); an empty range gives
    (0, -inf, 0). Used to check the multi-GPU KV-range sharding on CPU ranks.
    """
    S, H, d = query.shape
    Hkv = key_cache.shape[1]
    G = H // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    O = np.zeros((S, H, d), dtype=np.float64)
    m = np.full((S, H), -np.inf)
    l = np.zeros((S, H))
    for s in range(S):
        ctx = int(context_lens[s])
        b, e = token_begin, min(token_end, ctx)
        if e <= b:
            continue
        kd = gather_paged(key_cache, block_tables, context_lens, s, block_size)[:, b:e]
        vd = gather_paged(value_cache, block_tables, context_lens, s, block_size)[:, b:e]
        for h in range(H):
            sc = (kd[h // G].astype(np.float64) @ query[s, h].astype(np.float64)) * scale
            mm = sc.max()
            p = np.exp(sc - mm)
            O[s, h] = p @ vd[h // G].astype(np.float64)
            m[s, h] = mm
            l[s, h] = p.sum()
    return O, m, l


def lse_merge(outs, maxs, sums):
    """Stage-2 combine (``ops.py:133-143``) over a list of partials
    (O [.., d], m [..], l [..]); splits with m = -inf and l = 0 contribute nothing."""
    g = np.maximum.reduce([np.asarray(x) for x in maxs])
    L = np.zeros_like(np.asarray(sums[0], dtype=np.float64))
    O = np.zeros_like(np.asarray(outs[0], dtype=np.float64))
    for o, mm, ll in zip(outs, maxs, sums):
        w = np.where(np.isneginf(mm), 0.0, np.exp(np.where(np.isneginf(mm), 0.0, mm - g)))
        L = L + ll * w
        O = O + o * w[..., None]
    with np.errstate(invalid="ignore", divide="ignore"):
        res = O / L[..., None]
    return np.where(L[..., None] > 0, res, 0.0)


# --------------------------------------------------------------------------
# Seeded input generators for the benchmark configurations
# --------------------------------------------------------------------------

def make_paged_problem(seed: int, num_seqs: int, num_heads: int, num_kv_heads: int,
                       head_dim: int, context_lens, block_size: int = 16,
                       extra_blocks: int = 0, bf16: bool = True):
    """Random paged-decode problem: q, K/V ~ N(0,1) (bf16-rounded if ``bf16``),
    physical blocks a random permutation of a pool sized to the total.

    Returns dict(q [S,H,d] f32, k_cache/v_cache [P,Hkv,bs,d] f32, block_tables
    [S,maxb] i32, context_lens [S] i32). ``max_blocks`` = ceil(max ctx / bs)
    (at least 1); table slots past a sequence's last block hold 0.
    """
    rng = np.random.default_rng(seed)
    context_lens = np.asarray(context_lens, dtype=np.int32)
    nblk = [(int(c) + block_size - 1) // block_size if c > 0 else 0 for c in context_lens]
    pool = int(sum(nblk)) + int(extra_blocks)
    pool = max(pool, 1)
    maxb = max(1, max(nblk) if nblk else 1)
    perm = rng.permutation(pool).astype(np.int32)
    bt = np.zeros((num_seqs, maxb), dtype=np.int32)
    off = 0
    for s, n in enumerate(nblk):
        bt[s, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((num_seqs, num_heads, head_dim), dtype=np.float32)
    kc = rng.standard_normal((pool, num_kv_heads, block_size, head_dim), dtype=np.float32)
    vc = rng.standard_normal((pool, num_kv_heads, block_size, head_dim), dtype=np.float32)
    if bf16:
        q, kc, vc = bf16_round(q), bf16_round(kc), bf16_round(vc)
    return dict(q=q, k_cache=kc, v_cache=vc, block_tables=bt, context_lens=context_lens)


def config3_context_lens(seed: int = 0, num_seqs: int = 64):
    """Config 3: context lengths uniform in [512, 4096]."""
    rng = np.random.default_rng(seed)
    return rng.integers(512, 4096, size=num_seqs, endpoint=True).astype(np.int32)


def config5_context_lens(seed: int = 0, num_seqs: int = 256):
    """Config 5: lognormal (median 1024, sigma 1.0), rounded, clipped to [16, 32768]."""
    rng = np.random.default_rng(seed)
    x = rng.lognormal(mean=math.log(1024.0), sigma=1.0, size=num_seqs)
    return np.clip(np.round(x), 16, 32768).astype(np.int32)


# --------------------------------------------------------------------------
# Rotary position embedding (the arithmetic of src/fused_rope.cu:29-43)
# --------------------------------------------------------------------------

def rope_tables(max_pos: int, head_dim: int, base: float = 10000.0):
    """cos/sin tables [max_pos, head_dim/2] (float32) for pair i at position p:
    angle = p * base^(-2i/head_dim) (RoPEConfig's theta_base, include/fused_rope.cuh:13)."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    inv = base ** (-2.0 * i / head_dim)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope_rotate(x, cos, sin, pos):
    """Rotate adjacent pairs (2i, 2i+1) of x[..., d] by cos/sin[pos, i]:
    (x0 c - x1 s, x0 s + x1 c) -- src/fused_rope.cu:33-43. `pos` broadcasts over the
    leading dimensions of x: cos[pos] must broadcast against x[..., 0::2]."""
    x = np.asarray(x, dtype=np.float64)
    c = np.asarray(cos, np.float64)[pos]
    s = np.asarray(sin, np.float64)[pos]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out
