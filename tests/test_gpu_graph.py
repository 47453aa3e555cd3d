"""CUDA-graph capture of decode steps: the C++ runner through the C ABI and the
torch-graph helper; replays must reproduce eager results on updated inputs."""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_bf16_close, cuda, host
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _problem(seed):
    lens = [3, 100, 777, 2048]
    p = O.make_paged_problem(seed, len(lens), 32, 8, 128, lens)
    return p, {k: cuda(p[k], torch.bfloat16) for k in ("q", "k_cache", "v_cache")}, \
        cuda(p["block_tables"]), cuda(p["context_lens"])


def test_cpp_graph_runner_replays_decode():
    import flash_engine
    from flash_engine import _lib, graph
    p, t, bt, cl = _problem(31)
    S, H, d = p["q"].shape
    out = torch.empty_like(t["q"])
    n = flash_engine.paged_attention_workspace_floats(32, 8, 128)
    ws = torch.zeros(n, dtype=torch.float32, device="cuda")

    def record(stream):
        rc = _lib.lib.fe_paged_attention_v2_bf16(
            t["q"].data_ptr(), t["k_cache"].data_ptr(), t["v_cache"].data_ptr(), out.data_ptr(),
            bt.data_ptr(), cl.data_ptr(), S, H, 8, d, 16, 2048, bt.shape[1],
            t["k_cache"].shape[0], 0.0, ws.data_ptr(), n, stream)
        assert rc == 0

    stream = torch.cuda.Stream()
    # the first (uncaptured) call performs the per-device set-up
    flash_engine.paged_attention(t["q"], t["k_cache"], t["v_cache"], bt, cl, 16, workspace=ws)
    torch.cuda.synchronize()
    runner = graph.CUDAGraphRunner()
    runner.capture(record, stream)
    assert runner.is_captured()
    for seed in (32, 33):
        q2 = O.make_paged_problem(seed, S, 32, 8, 128, p["context_lens"])["q"]
        t["q"].copy_(cuda(q2, torch.bfloat16))
        runner.launch(stream)
        stream.synchronize()
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        assert_bf16_close(host(out), ref)
    runner.reset()
    assert not runner.is_captured()


def test_decode_graph_helper():
    import flash_engine
    from flash_engine import graph
    p, t, bt, cl = _problem(41)
    g = graph.DecodeGraph(lambda: flash_engine.paged_attention(
        t["q"], t["k_cache"], t["v_cache"], bt, cl, 16))
    for seed in (42, 43):
        q2 = O.make_paged_problem(seed, len(p["context_lens"]), 32, 8, 128,
                                  p["context_lens"])["q"]
        t["q"].copy_(cuda(q2, torch.bfloat16))
        out = g.replay()
        torch.cuda.synchronize()
        ref = O.paged_attention_gqa(q2, p["k_cache"], p["v_cache"], p["block_tables"],
                                    p["context_lens"])
        assert_bf16_close(host(out), ref)
    assert flash_engine.device_errors() == 0
