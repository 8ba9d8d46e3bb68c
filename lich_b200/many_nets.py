"""Many independent small iPC networks trained together (the batched form of the hidden-64 step).

``ManyNetIPC`` holds ``nets`` networks of the same dims as stacked tensors --
``w[l]`` is ``[nets, d_l, d_{l+1}]``, ``x[l]`` and ``e[l]`` are ``[nets, d_l, B]`` --
and trains all of them in one launch of the persistent kernel
(``ipc_net_train`` with ``nets > 1``): network n runs on its own cluster of CTAs
and nothing is shared between networks, so a network's result is the same
whether it is trained alone or among thousands.  Each network follows the
reference step (forward-init sweep, T inference iterations, one weight update;
``src/ipc_tilelang/trainer.py:509-516,601-679``).

Across GPUs the networks are sharded with no collective: ``shard(nets, world,
rank)`` is the contiguous slice of networks a rank owns.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _native as N
from .activations import get_activation
from .trainer import IPCConfig


def shard(nets: int, world: int, rank: int) -> range:
    """Networks owned by ``rank`` of ``world``: contiguous, sizes differ by at most one."""
    if nets < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad shard request nets={nets} world={world} rank={rank}")
    base, extra = divmod(nets, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


class ManyNetIPC:
    """``nets`` independent networks of ``cfg.dims`` with batch ``batch`` each (16-bit storage)."""

    def __init__(self, cfg: IPCConfig, nets: int, batch: int, *, device: torch.device):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("ManyNetIPC requires a CUDA device")
        if cfg.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("ManyNetIPC runs the persistent kernel: dtype must be float16 or bfloat16")
        if nets < 1:
            raise ValueError("nets must be >= 1")
        self.cfg, self.nets, self.B, self.device = cfg, int(nets), int(batch), device
        self.act = get_activation(cfg.activation)
        d = tuple(int(v) for v in cfg.dims)
        self.L = len(d) - 1
        dt = cfg.dtype
        self.w = [torch.zeros((nets, d[l], d[l + 1]), device=device, dtype=dt) for l in range(self.L)]
        self.x = [torch.zeros((nets, d[l], batch), device=device, dtype=dt) for l in range(self.L + 1)]
        self.e = [torch.zeros((nets, d[l], batch), device=device, dtype=dt) for l in range(self.L)]
        self._desc = N.IpcNet()
        self._desc.L = self.L
        for l, v in enumerate(d):
            self._desc.dims[l] = v
        self._desc.B, self._desc.nets = self.B, self.nets
        for l in range(self.L):
            self._desc.w[l] = self.w[l].data_ptr()
            self._desc.e[l] = self.e[l].data_ptr()
        for l in range(self.L + 1):
            self._desc.x[l] = self.x[l].data_ptr()
        plan = N.net_plan(d, self.B, nets=self.nets, cluster=int(cfg.net_cluster))
        if plan is None:
            raise ValueError(f"dims {d} with batch {batch} do not fit the persistent kernel: "
                             f"{N.load().ipc_last_error().decode()}")
        self.cluster, self.smem_bytes = plan
        self.steps_done = 0

    def set_network_weights(self, n: int, weights: Sequence[torch.Tensor]) -> None:
        """Copy one network's weights (``[d_l, d_{l+1}]`` each) into slab ``n``."""
        for l, w in enumerate(weights):
            self.w[l][n].copy_(w)

    def network_weights(self, n: int) -> list[torch.Tensor]:
        return [w[n] for w in self.w]

    def _run(self, pool_x, pool_y, *, steps, T, first_batch, energy):
        run = N.IpcNetRun()
        run.pool_x, run.pool_y = pool_x.data_ptr(), pool_y.data_ptr()
        run.pool_batches, run.first_batch = int(pool_x.shape[0]), int(first_batch)
        run.steps, run.T = int(steps), int(T)
        run.forward_init, run.update_weights, run.recompute = 1, 1, 1
        run.alpha, run.gamma = float(self.cfg.alpha), float(self.cfg.gamma)
        run.act, run.dtype = self.act.code, N.dtype_code(self.cfg.dtype)
        run.cluster = int(self.cluster)
        if energy is not None:
            run.energy = energy.data_ptr()
        N.check(N.load().ipc_net_train(self._desc, run, N.stream_handle(self.device)))

    @torch.no_grad()
    def train_pool(self, pool_x: torch.Tensor, pool_y: torch.Tensor, *, steps: int, T: int = 4,
                   first_batch: int = 0, energy: torch.Tensor | None = None) -> None:
        """``steps`` training steps of every network over a device batch pool.

        ``pool_x [P, nets, d_L, B]``, ``pool_y [P, nets, d_0, B]`` (contiguous, model dtype, on the
        device); step ``s`` of network ``n`` trains on ``pool[(first_batch + s) % P, n]``.  ``energy``
        (float32, ``>= steps * nets`` elements) receives ``[step, net]`` of ``sum_l mean(e[l]^2)``."""
        d = self.cfg.dims
        if pool_x.ndim != 4 or pool_y.ndim != 4:
            raise ValueError("pool_x / pool_y must be [P, nets, features, batch]")
        P = pool_x.shape[0]
        if tuple(pool_x.shape[1:]) != (self.nets, d[-1], self.B) or tuple(pool_y.shape) != (P, self.nets, d[0], self.B):
            raise ValueError("pool shapes do not match [P, nets, d, B] of this model")
        for t in (pool_x, pool_y):
            if t.device != self.device or t.dtype != self.cfg.dtype or not t.is_contiguous():
                raise ValueError("pool tensors must be contiguous, on the model device, in the model dtype")
        if energy is not None and (energy.dtype != torch.float32 or not energy.is_contiguous()
                                   or energy.numel() < steps * self.nets or energy.device != self.device):
            raise ValueError("energy must be a contiguous float32 tensor with >= steps * nets elements on the device")
        if steps <= 0:
            return
        self._run(pool_x, pool_y, steps=steps, T=T, first_batch=first_batch, energy=energy)
        self.steps_done += int(steps)

    def train_step(self, x: torch.Tensor, y: torch.Tensor, *, T: int = 4) -> None:
        """One training step of every network on ``x [nets, d_L, B]``, ``y [nets, d_0, B]``."""
        self.train_pool(x.unsqueeze(0), y.unsqueeze(0), steps=1, T=T)
