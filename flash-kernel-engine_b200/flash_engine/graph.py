"""CUDA-graph capture of decode steps.

* ``CUDAGraphRunner`` -- the reference's C++ runner (include/cuda_graph_runner.h:10-35)
  through the C ABI (fe_graph_capture / fe_graph_launch): ``capture(record)`` calls
  ``record(stream_handle)`` once under stream capture, ``launch()`` replays it.
* ``DecodeGraph`` -- captures a Python decode step (a single-GPU ``paged_attention``
  call, or the KV-range-sharded step with its NCCL all-gather) with
  torch.cuda.CUDAGraph; ``replay()`` reruns it on the same device buffers and returns
  the step's output tensor. Update inputs in place between replays.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


class CUDAGraphRunner:
    def __init__(self):
        self._g = ctypes.c_void_p()
        self._cb = None

    def capture(self, record_func, stream=None):
        """record_func(stream_handle: int) enqueues the step on that stream."""
        self.reset()
        s = stream if stream is not None else torch.cuda.current_stream()
        handle = int(s.cuda_stream)

        def _record(st, user):
            record_func(int(st or 0))

        self._cb = _lib.RECORD_FN(_record)
        _lib.check(_lib.lib.fe_graph_capture(self._cb, None, handle, ctypes.byref(self._g)),
                   "fe_graph_capture")

    def launch(self, stream=None):
        if not self._g:
            raise RuntimeError("CUDAGraphRunner: Cannot launch uncaptured graph.")
        s = stream if stream is not None else torch.cuda.current_stream()
        _lib.check(_lib.lib.fe_graph_launch(self._g, int(s.cuda_stream)), "fe_graph_launch")

    def is_captured(self) -> bool:
        return bool(self._g)

    def reset(self):
        if self._g:
            _lib.lib.fe_graph_destroy(self._g)
            self._g = ctypes.c_void_p()

    def __del__(self):
        try:
            self.reset()
        except Exception:
            pass


class DecodeGraph:
    def __init__(self, step_fn, warmup: int = 2):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                step_fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = step_fn()

    def replay(self):
        self.graph.replay()
        return self.out
