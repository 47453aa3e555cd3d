"""Prefill forward on the GPU against the reference-generated golden vectors and
the oracle."""
import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, assert_fp32_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

ATTN_CASES = ["attn_d64", "attn_d64_causal", "attn_d64_nm", "attn_d64_nm_causal", "attn_d32",
              "attn_d128"]


@pytest.mark.parametrize("name", ATTN_CASES)
@pytest.mark.parametrize("kind", ["flash", "naive"])
def test_fp32_golden(golden, name, kind):
    import flash_engine
    g = golden(name)
    fn = flash_engine.flash_attention if kind == "flash" else flash_engine.naive_attention
    out = fn(cuda(g["q"]), cuda(g["k"]), cuda(g["v"]), bool(g["is_causal"]))
    assert_fp32_close(host(out), g["out"])


def test_fp32_config1():
    """Benchmark config 1: fp32, non-causal, [1, 8, 512, 64], N(0,1) inputs, seed 42."""
    import flash_engine
    rng = np.random.default_rng(42)
    q, k, v = (rng.standard_normal((1, 8, 512, 64), dtype=np.float32) for _ in range(3))
    ref = O.flash_attention(q, k, v, False)
    out = flash_engine.flash_attention(cuda(q), cuda(k), cuda(v), False)
    assert_fp32_close(host(out), ref)


def test_fp32_config1_cuda_core_kernel():
    """Head dims 32 and 64 run on the 3xTF32 tensor-core kernel; FE_FP32_SIMT=1 selects
    the CUDA-core kernel instead. Both must match the oracle (run in a child process,
    since the switch is read once per process)."""
    import os
    import subprocess
    import sys
    code = (
        "import numpy as np, torch, flash_engine\n"
        "from gpu_util import assert_fp32_close, cuda, host\n"
        "from oracle import attention_oracle as O\n"
        "rng = np.random.default_rng(42)\n"
        "q, k, v = (rng.standard_normal((1, 8, 512, 64), dtype=np.float32) for _ in range(3))\n"
        "for causal in (False, True):\n"
        "    out = flash_engine.flash_attention(cuda(q), cuda(k), cuda(v), causal)\n"
        "    assert_fp32_close(host(out), O.flash_attention(q, k, v, causal))\n"
        "    a, b, c = (x[..., :32].copy() for x in (q, k, v))\n"
        "    out = flash_engine.flash_attention(cuda(a), cuda(b), cuda(c), causal)\n"
        "    assert_fp32_close(host(out), O.flash_attention(a, b, c, causal))\n"
        "assert flash_engine.device_errors() == 0\n")
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, FE_FP32_SIMT="1",
               PYTHONPATH=os.pathsep.join([here, os.path.dirname(here),
                                           os.path.join(os.path.dirname(here),
                                                        "flash-kernel-engine_b200"),
                                           os.environ.get("PYTHONPATH", "")]))
    r = subprocess.run([sys.executable, "-c", code], env=env, cwd=here, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr


def _misaligned(x):
    """A contiguous CUDA copy of x whose data pointer is 4 bytes past a 16-byte boundary."""
    flat = torch.empty(x.size + 4, dtype=torch.float32, device="cuda")
    t = flat[1:1 + x.size].view(x.shape)
    t.copy_(torch.from_numpy(np.ascontiguousarray(x)))
    assert t.data_ptr() % 16 == 4
    return t


@pytest.mark.parametrize("d", [32, 64, 128])
def test_fp32_misaligned_tensors_take_cuda_core_kernel(d):
    """Tensors that are only 4-byte aligned cannot be read by TMA: the fp32 entry takes
    the CUDA-core kernel (scalar loads) and must still match the oracle."""
    import flash_engine
    rng = np.random.default_rng(d)
    q, k, v = (rng.standard_normal((1, 2, 150, d), dtype=np.float32) for _ in range(3))
    for causal in (False, True):
        out = flash_engine.flash_attention(_misaligned(q), _misaligned(k), _misaligned(v), causal,
                                           out=_misaligned(np.zeros_like(q)))
        torch.cuda.synchronize()
        assert_fp32_close(host(out), O.flash_attention(q, k, v, causal))


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("N,M,d", [(1, 1, 64), (65, 130, 32), (200, 77, 128), (128, 128, 100),
                                   (100, 300, 64), (100, 300, 50), (70, 1000, 32), (1, 700, 128),
                                   (1000, 1000, 64), (129, 700, 64), (300, 900, 128),
                                   (129, 33, 128)])
def test_fp32_shapes(causal, N, M, d):
    import flash_engine
    rng = np.random.default_rng(N + M + d)
    q = rng.standard_normal((2, 3, N, d), dtype=np.float32)
    k = rng.standard_normal((2, 3, M, d), dtype=np.float32)
    v = rng.standard_normal((2, 3, M, d), dtype=np.float32)
    ref = O.flash_attention(q, k, v, causal)
    out = flash_engine.flash_attention(cuda(q), cuda(k), cuda(v), causal)
    assert_fp32_close(host(out), ref)


def _bf16_case(B, H, N, M, d, causal, seed, dtype=torch.bfloat16):
    import flash_engine
    rng = np.random.default_rng(seed)
    q = O.bf16_round(rng.standard_normal((B, H, N, d), dtype=np.float32))
    k = O.bf16_round(rng.standard_normal((B, H, M, d), dtype=np.float32))
    v = O.bf16_round(rng.standard_normal((B, H, M, d), dtype=np.float32))
    if dtype == torch.float16:
        q, k, v = (x.astype(np.float16).astype(np.float32) for x in (q, k, v))
    ref = O.flash_attention_sliced(q, k, v, causal)
    out = flash_engine.flash_attention(cuda(q, dtype), cuda(k, dtype), cuda(v, dtype), causal)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    return host(out), ref


@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("N,M", [(128, 128), (256, 256), (300, 300), (1, 1), (77, 200),
                                 (200, 77), (512, 384)])
def test_bf16_tcgen05_shapes(d, causal, N, M):
    out, ref = _bf16_case(1, 2, N, M, d, causal, N * 7 + M + d)
    assert_bf16_close(out, ref)


def test_fp16_tcgen05():
    out, ref = _bf16_case(2, 2, 384, 384, 128, True, 3, torch.float16)
    assert_bf16_close(out, ref, atol=5e-3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_head_dim_32_reference_dispatch(dtype):
    """head_dim 32, which the reference's fp16 launcher dispatches
    (src/flash_attention.cu:514-521): the d = 64 tensor-core kernel loads 64-column
    boxes over the 32 real columns (zero-filled by TMA) and stores 32 columns."""
    out, ref = _bf16_case(2, 3, 640, 520, 32, True, 32, dtype)
    assert_bf16_close(out, ref, atol=5e-3 if dtype == torch.float16 else 2e-2)


def test_bf16_config2_shape_slice():
    """Benchmark config 2 shape (causal, seq 4096, d 128) on 2 heads: the oracle runs
    per (b, h) slice."""
    out, ref = _bf16_case(1, 2, 4096, 4096, 128, True, 42)
    assert_bf16_close(out, ref)


def test_bf16_reference_scale_inputs(golden):
    """The reference test recipe (N(0,1) * 0.1 inputs), bf16-rounded."""
    import flash_engine
    g = golden("attn_d64_causal")
    q, k, v = (O.bf16_round(g[x]) for x in ("q", "k", "v"))
    ref = O.flash_attention(q, k, v, True)
    out = flash_engine.flash_attention(cuda(q, torch.bfloat16), cuda(k, torch.bfloat16),
                                       cuda(v, torch.bfloat16), True)
    assert_bf16_close(host(out), ref)


def _heads_case(B, H, N, d, seed):
    rng = np.random.default_rng(seed)
    q, k, v = (O.bf16_round(rng.standard_normal((B, H, N, d), dtype=np.float32))
               for _ in range(3))
    return q, k, v


def test_bf16_many_heads_ragged():
    """Many (batch, head)s over several head groups of the longest-first schedule, a
    ragged sequence length, two calls in a row."""
    import flash_engine
    B, H, N, d = 2, 40, 1000, 128
    q, k, v = _heads_case(B, H, N, d, 7)
    sel = [(0, 0), (0, 17), (1, 39)]
    for _ in range(2):
        out = flash_engine.flash_attention(cuda(q, torch.bfloat16), cuda(k, torch.bfloat16),
                                           cuda(v, torch.bfloat16), True)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        o = host(out)
        for b, h in sel:
            ref = O.flash_attention_sliced(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                           v[b:b + 1, h:h + 1], True)
            assert_bf16_close(o[b:b + 1, h:h + 1], ref)


def test_bf16_first_call_inside_graph_capture():
    """The prefill captured into a CUDA graph as the first call on a new stream; the
    replay matches the oracle."""
    import flash_engine
    B, H, N, d = 1, 24, 700, 64
    q, k, v = _heads_case(B, H, N, d, 8)
    qd, kd, vd = (cuda(x, torch.bfloat16) for x in (q, k, v))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        out = flash_engine.flash_attention(qd, kd, vd, True)
    g.replay()
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    o = host(out)
    for h in (0, 11, 23):
        ref = O.flash_attention_sliced(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], True)
        assert_bf16_close(o[:, h:h + 1], ref)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("N,M", [(300, 300), (520, 200), (256, 700)])
def test_bf16_many_pairs_repeated_and_second_stream(d, causal, N, M):
    """More query-tile pairs than SMs (several waves of CTAs, longest-first over head
    groups). N = 300 leaves the last pair without its second tile. Three launches in a
    row and one on a second stream; every (batch, head) against the oracle."""
    import flash_engine
    B, H = 3, 56
    rng = np.random.default_rng(N * 3 + M + d + causal)
    q = O.bf16_round(rng.standard_normal((B, H, N, d), dtype=np.float32))
    k = O.bf16_round(rng.standard_normal((B, H, M, d), dtype=np.float32))
    v = O.bf16_round(rng.standard_normal((B, H, M, d), dtype=np.float32))
    ref = O.flash_attention(q, k, v, causal)
    qd, kd, vd = (cuda(x, torch.bfloat16) for x in (q, k, v))
    for _ in range(3):
        out = flash_engine.flash_attention(qd, kd, vd, causal)
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        assert_bf16_close(host(out), ref)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = flash_engine.flash_attention(qd, kd, vd, causal)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(out), ref)


def test_bf16_many_pairs_graph_replays():
    """More query-tile pairs than SMs, captured into a CUDA graph as the first call on a
    new stream and replayed three times (the output zeroed before each replay)."""
    import flash_engine
    B, H, N, d = 2, 48, 1100, 64
    q, k, v = _heads_case(B, H, N, d, 9)
    qd, kd, vd = (cuda(x, torch.bfloat16) for x in (q, k, v))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        out = flash_engine.flash_attention(qd, kd, vd, True)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert flash_engine.device_errors() == 0
        o = host(out)
        for b, h in ((0, 0), (1, 47), (0, 30)):
            ref = O.flash_attention_sliced(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                           v[b:b + 1, h:h + 1], True)
            assert_bf16_close(o[b:b + 1, h:h + 1], ref)


@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("N,M", [(300, 300), (128, 520), (640, 200)])
def test_bf16_fused_rope_q_and_k(d, causal, N, M):
    """RoPE of Q (row i at position i) and K (row j at position j) by the streaming RoPE
    pass, then the tensor-core prefill, against the oracle rotating Q and K first (the
    reference's fused RoPE arithmetic, src/fused_rope.cu:33-43) then attending; k_rotated
    returns the rotated keys."""
    import flash_engine
    rng = np.random.default_rng(N + M + d)
    q = O.bf16_round(rng.standard_normal((2, 3, N, d), dtype=np.float32))
    k = O.bf16_round(rng.standard_normal((2, 3, M, d), dtype=np.float32))
    v = O.bf16_round(rng.standard_normal((2, 3, M, d), dtype=np.float32))
    cos, sin = O.rope_tables(max(N, M) + 7, d)
    qr = O.bf16_round(O.rope_rotate(q, cos, sin, np.arange(N)).astype(np.float32))
    kr = O.bf16_round(O.rope_rotate(k, cos, sin, np.arange(M)).astype(np.float32))
    ref = O.flash_attention_sliced(qr, kr, v, causal)
    k_rot = torch.empty((2, 3, M, d), dtype=torch.bfloat16, device="cuda")
    out = flash_engine.flash_attention(cuda(q, torch.bfloat16), cuda(k, torch.bfloat16),
                                       cuda(v, torch.bfloat16), causal,
                                       rope=(cuda(cos), cuda(sin)), k_rotated=k_rot)
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(out), ref)
    # the rotated keys a KV cache would store
    np.testing.assert_allclose(host(k_rot), kr, rtol=2 ** -7, atol=2 ** -7)


def test_fp16_fused_rope_config2_slice():
    """RoPE + prefill on the config 2 shape (causal, 4096 rows, d 128) in fp16, 2 heads."""
    import flash_engine
    rng = np.random.default_rng(7)
    N, d = 4096, 128
    q, k, v = (rng.standard_normal((1, 2, N, d), dtype=np.float32).astype(np.float16)
               .astype(np.float32) for _ in range(3))
    cos, sin = O.rope_tables(N, d)
    pos = np.arange(N)
    qr = O.rope_rotate(q, cos, sin, pos).astype(np.float16).astype(np.float32)
    kr = O.rope_rotate(k, cos, sin, pos).astype(np.float16).astype(np.float32)
    ref = O.flash_attention_sliced(qr, kr, v, True)
    out = flash_engine.flash_attention(cuda(q, torch.float16), cuda(k, torch.float16),
                                       cuda(v, torch.float16), True,
                                       rope=(cuda(cos), cuda(sin)))
    torch.cuda.synchronize()
    assert flash_engine.device_errors() == 0
    assert_bf16_close(host(out), ref, atol=5e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [64, 128, 6])
def test_rope_forward(dtype, d):
    """The dense RoPE pass (the reference's fused_rope_kernel_fp32 rule: row (b, h, i)
    rotated at position i with the caller's tables), vector path (d % 8 == 0) and the
    per-pair path (d = 6), out of place and in place."""
    import flash_engine
    rng = np.random.default_rng(d)
    x = rng.standard_normal((2, 3, 77, d), dtype=np.float32)
    rnd = (lambda a: O.bf16_round(a.astype(np.float32))) if dtype == torch.bfloat16 else \
        (lambda a: a.astype(np.float16).astype(np.float32)) if dtype == torch.float16 else \
        (lambda a: a.astype(np.float32))
    x = rnd(x)
    cos, sin = O.rope_tables(100, d)
    ref = rnd(O.rope_rotate(x, cos, sin, np.arange(77)))
    xt = cuda(x, dtype)
    out = flash_engine.rope(xt, cuda(cos), cuda(sin))
    flash_engine.rope(xt, cuda(cos), cuda(sin), out=xt)   # in place
    torch.cuda.synchronize()
    tol = {torch.float32: 1e-6, torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10}[dtype]
    np.testing.assert_allclose(host(out), ref, rtol=tol, atol=tol)
    np.testing.assert_array_equal(host(xt), host(out))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [64, 128])
def test_rope_forward_many_passes(dtype, d):
    """The row path of the dense RoPE pass when each thread covers several rows of a
    grid-wide pass (50k rows of an odd sequence length, so that positions wrap inside a
    pass), out of place and in place."""
    import flash_engine
    rng = np.random.default_rng(d + 1)
    x = rng.standard_normal((3, 50, 333, d), dtype=np.float32)
    rnd = (lambda a: O.bf16_round(a.astype(np.float32))) if dtype == torch.bfloat16 else \
        (lambda a: a.astype(np.float16).astype(np.float32)) if dtype == torch.float16 else \
        (lambda a: a.astype(np.float32))
    x = rnd(x)
    cos, sin = O.rope_tables(400, d)
    ref = rnd(O.rope_rotate(x, cos, sin, np.arange(333)))
    xt = cuda(x, dtype)
    out = flash_engine.rope(xt, cuda(cos), cuda(sin))
    flash_engine.rope(xt, cuda(cos), cuda(sin), out=xt)   # in place
    torch.cuda.synchronize()
    tol = {torch.float32: 1e-6, torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10}[dtype]
    np.testing.assert_allclose(host(out), ref, rtol=tol, atol=tol)
    np.testing.assert_array_equal(host(xt), host(out))
