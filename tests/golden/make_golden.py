"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container where the upstream FlashKernel-Engine checkout is mounted
(``--ref`` points at its root); the GPU box does not have it, so the outputs are
committed as ``tests/golden/*.npz``:

    python tests/golden/make_golden.py --ref <path-to-flash-kernel-engine>

Every expected output below is produced by the reference's own
``python/flash_engine/ops.py`` (imported from the checkout, unmodified). The
inputs follow the reference's tests where they exist:

* ``attn_*``      -- ``python/tests/test_correctness.py:27-47`` recipe
  (``np.random.seed(42)``, randn * 0.1), at smaller shapes plus N != M and
  head_dim 32 / 128 variants.
* ``paged_fp32``  -- ``python/tests/test_correctness.py:49-67`` exactly
  (2 seqs, 4 heads, d=64, block 16, 8 blocks, block tables
  ``[[3,7,1,0],[2,5,4,6]]``, lens ``[48,64]``).
* ``paged_kat``   -- the constant-input known-answer case of
  ``tests/test_paged_attention.cu:20-53`` (Q=1, K=0.5, V=0.25; tables
  ``[3,7,1,9]`` / ``[5,2,8,4]``; lens 48 / 64); the answer is 0.25 everywhere.
* ``paged_gqa_bf16`` -- a GQA case (8 q heads / 2 KV heads, d=128), bf16-rounded
  inputs, ragged lengths 1 / 17 / 50 / 0, evaluated with the reference's
  ``paged_attention`` once per KV-head group.
* ``decoding``    -- ``python/tests/test_correctness.py:69-86`` recipe at
  B,H,d,M = 1,2,64,100 with 8 splits (``flash_decoding``), plus the
  ``flash_attention`` result it must agree with.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
from oracle.attention_oracle import bf16_round  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the upstream checkout")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "python"))
    from flash_engine import ops  # the reference implementation, unmodified

    out = {}

    # ---- dense attention (fp32) --------------------------------------------
    for name, (B, H, N, M, d, causal) in {
        "attn_d64": (1, 2, 64, 64, 64, False),
        "attn_d64_causal": (1, 2, 64, 64, 64, True),
        "attn_d64_nm": (1, 2, 40, 72, 64, False),
        "attn_d64_nm_causal": (1, 2, 72, 40, 64, True),
        "attn_d32": (2, 1, 33, 33, 32, True),
        "attn_d128": (1, 1, 72, 72, 128, True),
    }.items():
        np.random.seed(42)
        q = np.random.randn(B, H, N, d).astype(np.float32) * 0.1
        k = np.random.randn(B, H, M, d).astype(np.float32) * 0.1
        v = np.random.randn(B, H, M, d).astype(np.float32) * 0.1
        o = ops.flash_attention(q, k, v, is_causal=causal)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=q, k=k, v=v, out=o,
                 is_causal=np.array(causal))
        out[name] = o

    # ---- paged fp32: the reference test case --------------------------------
    np.random.seed(42)
    S, Hh, d, bs, nb = 2, 4, 64, 16, 8
    q = np.random.randn(S, Hh, d).astype(np.float32)
    kc = np.random.randn(nb, Hh, bs, d).astype(np.float32)
    vc = np.random.randn(nb, Hh, bs, d).astype(np.float32)
    bt = np.array([[3, 7, 1, 0], [2, 5, 4, 6]], dtype=np.int32)
    lens = np.array([48, 64], dtype=np.int32)
    o = ops.paged_attention(q, kc, vc, bt, lens, bs)
    np.savez_compressed(os.path.join(HERE, "paged_fp32.npz"), q=q, k_cache=kc, v_cache=vc,
             block_tables=bt, context_lens=lens, out=o)

    # ---- paged KAT: constant inputs -----------------------------------------
    S, Hh, d, bs, nb, maxb = 2, 4, 64, 16, 16, 8
    q = np.full((S, Hh, d), 1.0, np.float32)
    kc = np.full((nb, Hh, bs, d), 0.5, np.float32)
    vc = np.full((nb, Hh, bs, d), 0.25, np.float32)
    bt = np.zeros((S, maxb), np.int32)
    bt[0, :4] = [3, 7, 1, 9]
    bt[1, :4] = [5, 2, 8, 4]
    lens = np.array([48, 64], np.int32)
    o = ops.paged_attention(q, kc, vc, bt, lens, bs)
    np.savez_compressed(os.path.join(HERE, "paged_kat.npz"), q=q, k_cache=kc, v_cache=vc,
             block_tables=bt, context_lens=lens, out=o)

    # ---- paged GQA, bf16-rounded inputs, ragged lengths ----------------------
    rng = np.random.default_rng(7)
    S, Hh, Hkv, d, bs = 4, 8, 2, 128, 16
    lens = np.array([1, 17, 50, 0], np.int32)
    nblk = [(int(c) + bs - 1) // bs for c in lens]
    pool = sum(nblk) + 3
    perm = rng.permutation(pool).astype(np.int32)
    bt = np.zeros((S, max(nblk)), np.int32)
    off = 0
    for s, n in enumerate(nblk):
        bt[s, :n] = perm[off:off + n]
        off += n
    q = bf16_round(rng.standard_normal((S, Hh, d), dtype=np.float32))
    kc = bf16_round(rng.standard_normal((pool, Hkv, bs, d), dtype=np.float32))
    vc = bf16_round(rng.standard_normal((pool, Hkv, bs, d), dtype=np.float32))
    G = Hh // Hkv
    o = np.zeros_like(q)
    for g in range(Hkv):
        o[:, g * G:(g + 1) * G] = ops.paged_attention(
            q[:, g * G:(g + 1) * G], kc[:, g:g + 1], vc[:, g:g + 1], bt, lens, bs)
    np.savez_compressed(os.path.join(HERE, "paged_gqa_bf16.npz"), q=q, k_cache=kc, v_cache=vc,
             block_tables=bt, context_lens=lens, out=o)

    # ---- split-KV flash decoding --------------------------------------------
    np.random.seed(42)
    B, Hh, d, M = 1, 2, 64, 100
    q = np.random.randn(B, Hh, 1, d).astype(np.float32) * 0.1
    k = np.random.randn(B, Hh, M, d).astype(np.float32) * 0.1
    v = np.random.randn(B, Hh, M, d).astype(np.float32) * 0.1
    od = ops.flash_decoding(q, k, v, num_splits=8)
    oa = ops.flash_attention(q, k, v, is_causal=False)
    np.savez_compressed(os.path.join(HERE, "decoding.npz"), q=q, k=k, v=v, out=od, out_full=oa,
             num_splits=np.array(8))

    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
