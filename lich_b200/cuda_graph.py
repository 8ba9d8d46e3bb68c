"""Steady-state CUDA graphs of the iPC step (the ``ipc_tilelang.cuda_graph`` entry point).

``IPCGraphRunner(model, steps)`` records ``steps`` calls of
``model.step_initialized()`` once and replays them with one
``cudaGraphLaunch`` (the reference's interface, ``src/ipc_tilelang/
cuda_graph.py:6-36``: construct, ``capture()``, ``replay()``).  What is
recorded depends on the path the model takes:

* persistent-kernel path: a single kernel node -- one ``ipc_net_train``
  launch that runs all ``steps`` steps with the weights resident on chip
  (the same arithmetic as ``steps`` separate ``step_initialized`` calls);
* operator path: the fused P / I / W launches of every step, in order.

Before recording, one step runs on a side stream with the model state saved
and restored (``model.precompile``): every kernel's one-time setup (function
attributes, tensor-map encoders, the first cudaMalloc of a workspace) then
happens outside the capture.  The graph allocates from a private memory pool
(``pool``; pass one runner's ``pool`` to another to share it), and the
model's buffers keep stable addresses, so a replay reads and writes the same
tensors the model exposes (``model.x`` / ``.e`` / ``.w``).
"""
from __future__ import annotations

import torch


class IPCGraphRunner:
    """A captured block of ``steps`` iPC steps of one ``TileLangIPC``; see the module docstring."""

    def __init__(self, model, steps: int, *, pool=None):
        if int(steps) < 1:
            raise ValueError("steps must be >= 1")
        self.model = model
        self.steps = int(steps)
        self.pool = pool if pool is not None else torch.cuda.graph_pool_handle()
        self.graph: torch.cuda.CUDAGraph | None = None
        self.single_node = False

    @property
    def captured(self) -> bool:
        return self.graph is not None

    def _record(self) -> None:
        m = self.model
        B = int(m.x[-1].shape[1])
        if m.net_kernel_eligible(B):
            # one persistent launch for the whole block (T = 1, no forward sweep, no batch pool: exactly
            # `steps` applications of the reference step to the resident state)
            m._net_run(steps=self.steps, T=1, forward_init=False, update_weights=True)
            m.steps_done += self.steps
            self.single_node = True
        else:
            for _ in range(self.steps):
                m.step_initialized(collect_metrics=False)

    def capture(self) -> "IPCGraphRunner":
        m = self.model
        if m.x is None:
            raise RuntimeError("Call initialize_batch before capturing a graph")
        dev = m.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            m.precompile()  # one step outside the capture, state restored afterwards
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        done = m.steps_done
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self.pool):
            self._record()
        m.steps_done = done  # recording ran nothing; replays count the steps
        self.graph = graph
        return self

    def replay(self) -> None:
        if self.graph is None:
            raise RuntimeError("Graph has not been captured")
        self.graph.replay()
        self.model.steps_done += self.steps

    def release(self) -> None:
        """Drop the graph (its memory returns to the pool)."""
        self.graph = None
