"""KV-range sharding over NCCL on 2 GPUs (skipped with fewer GPUs): the partials of
each rank's token window are all-gathered and merged; every rank must reproduce the
single-pass attention of the oracle."""
import pytest
import torch

import dist_workers
from test_sharding_gloo import _run

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_kv_range_nccl_two_gpus(tmp_path):
    res = _run(dist_workers.nccl_kv_range_worker, 2, tmp_path, join_timeout=180)
    assert all(r is not None for r in res), res
    for err, dev_errors in res:
        assert dev_errors == 0
        assert err <= 2e-2


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_graph_captured_kv_range_step_two_gpus(tmp_path):
    res = _run(dist_workers.nccl_graph_worker, 2, tmp_path, join_timeout=180)
    assert all(r is not None for r in res), res
    assert all(e <= 2e-2 for e in res)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_kv_range_peer_exchange_two_gpus(tmp_path):
    """The fused KV-range step: the decode kernel stores its partials into both GPUs'
    exchange buffers over NVLink, the merge kernel waits for both flags. Eager steps
    and CUDA-graph replays must all match the oracle."""
    res = _run(dist_workers.p2p_exchange_worker, 2, tmp_path, join_timeout=180)
    assert all(r is not None for r in res), res
    for err, dev_errors in res:
        assert dev_errors == 0
        assert err <= 2e-2


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_kv_range_c_entry_with_nccl_communicator_two_gpus(tmp_path):
    """The C/C++ multi-GPU entry that takes an ncclComm_t: decode, all-gather and merge
    on every rank must match the oracle."""
    res = _run(dist_workers.nccl_c_entry_worker, 2, tmp_path, join_timeout=180)
    assert all(r is not None for r in res), res
    for rc, err, dev_errors in res:
        assert rc == 0
        assert dev_errors == 0
        assert err <= 2e-2
