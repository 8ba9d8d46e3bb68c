"""CUDA-graph capture of a fixed number of steps -- the drop-in for ``ipc_tilelang.cuda_graph``.

Same contract as ``src/ipc_tilelang/cuda_graph.py:6-36``: the trainer's
buffers keep stable addresses, ``precompile()`` runs outside the capture,
then ``steps`` calls of ``step_initialized`` are captured once and replayed.
On the net path each captured step is a single kernel node.
"""
from __future__ import annotations

import torch


class IPCGraphRunner:
    def __init__(self, model, steps: int):
        if steps < 1:
            raise ValueError("steps must be >= 1")
        self.model = model
        self.steps = steps
        self.graph = torch.cuda.CUDAGraph()
        self._captured = False

    def capture(self) -> None:
        torch.cuda.synchronize()
        self.model.precompile()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for _ in range(self.steps):
                self.model.step_initialized(collect_metrics=False)
        torch.cuda.synchronize()
        self._captured = True

    def replay(self) -> None:
        if not self._captured:
            raise RuntimeError("Graph has not been captured")
        self.graph.replay()
