"""Host-side logic of the batch-sharded data-parallel step on 2 CPU ranks (gloo).

The GPU kernels are replaced by the CPU oracle behind the same hooks the
product uses (``_delta`` for a rank's dW, ``_apply`` / ``_apply_slice`` for
W += dW), so the test checks the orchestration that runs on the GPUs: local
forward sweep and T iterations, then per layer either one all-reduce and an
identical apply on every rank, or a reduce-scatter, the apply of this rank's
slice and an all-gather of the updated weights -- and that the sharded step
equals the oracle's full-batch step in both forms.
"""
import os
import socket
from dataclasses import dataclass

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ipc_oracle as O

DIMS = (6, 8, 8, 12)
ACT, ALPHA, GAMMA, T, B = "tanh", 0.05, 0.5, 3, 16


@dataclass
class _Cfg:
    dims: tuple = DIMS
    alpha: float = ALPHA
    gamma: float = GAMMA
    activation: str = ACT
    dtype: torch.dtype = torch.float32


class _OracleModel:
    """The attributes / methods of TileLangIPC the data-parallel step touches, on the CPU oracle."""

    def __init__(self, w):
        self.cfg = _Cfg()
        self.w = [t.clone() for t in w]
        self.x = self.e = None
        self._ac = None
        self.device = torch.device("cpu")
        self.steps_done = 0

    def initialize_batch(self, x_in, y):
        self.x = O.forward_init(x_in, y, self.w, ACT)

    def step_initialized(self, *, update_weights=True):
        assert not update_weights
        self.x, _, self.e, _ = O.ipc_step(self.x, self.w, act=ACT, alpha=ALPHA, gamma=GAMMA, update_weights=False)


def _worker(rank, world, port, data, out, reduce):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lich_b200.data_parallel import DataParallelIPC

        class _DP(DataParallelIPC):
            def _delta(self, l, dw):
                m = self.model
                dw.copy_(ALPHA * (m.e[l] @ O.act_forward(ACT, m.x[l + 1]).T))

            def _apply(self, l, dw):
                self.model.w[l] += dw
                caps.append(("apply", l))

            def _apply_slice(self, l, lo, hi):
                self.model.w[l].view(-1)[lo:hi] += self._dw[l].view(-1)[lo:hi]
                caps.append(("apply", l))

            def _cap(self, leave):
                caps.append(("cap", leave))

            def _sms(self):
                return 148

        caps = []

        w0, x, y = data
        cols = slice(rank * B // world, (rank + 1) * B // world)
        model = _OracleModel(w0 if rank == 0 else [torch.zeros_like(t) for t in w0])  # rank 0 broadcasts
        dp = _DP(_Cfg(), device=torch.device("cpu"), model=model, reduce=reduce)
        dp.train_step(x[:, cols].contiguous(), y[:, cols].contiguous(), T=T)
        out[rank] = ([t.clone() for t in dp.model.w], [t.clone() for t in dp.model.x], caps)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(120)
@pytest.mark.parametrize("reduce", ["rs_ag", "allreduce"])
def test_sharded_step_equals_full_batch_step(reduce):
    torch.manual_seed(0)
    w0 = [torch.randn(a, b) / b ** 0.5 for a, b in zip(DIMS[:-1], DIMS[1:])]
    x = torch.rand(DIMS[-1], B)
    y = O.one_hot(torch.randint(0, DIMS[0], (B,)), DIMS[0], dtype=torch.float32)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, _free_port(), (w0, x, y), out, reduce), nprocs=2, join=True,
                           start_method="spawn")
        res = dict(out)
    x_ref, w_ref, _, _ = O.train_step(x, y, w0, act=ACT, alpha=ALPHA, gamma=GAMMA, T=T)
    for rank in range(2):
        w_got, x_got, caps = res[rank]
        # the delta GEMMs after the first reduction leave SMs to it; each layer is applied once, behind
        # the next layer's delta GEMM, and only the last layer's apply follows the lifted cap
        assert caps[0] == ("cap", 24), caps
        lift = caps.index(("cap", 0))
        assert [k for k, _ in caps[lift + 1:]] == ["apply"] and caps[lift - 1][0] == "apply", caps
        assert all(c == ("cap", 24) for c in caps[:lift] if c[0] == "cap"), caps
        assert sorted(l for k, l in caps if k == "apply") == list(range(len(w0))), caps
        for l in range(len(w_ref)):
            assert O.rel_inf(w_got[l], w_ref[l]) <= 1e-5, (rank, "w", l)
        cols = slice(rank * B // 2, (rank + 1) * B // 2)
        for l in range(len(x_ref)):
            assert O.rel_inf(x_got[l], x_ref[l][:, cols]) <= 1e-5, (rank, "x", l)
    # the weight change is real (alpha large enough to see)
    assert max((a - b).abs().max().item() for a, b in zip(res[0][0], w0)) > 1e-3


def test_single_process_allreduce_is_identity():
    from lich_b200.data_parallel import allreduce_deltas
    d = [torch.ones(3)]
    assert allreduce_deltas(d) == [] and torch.equal(d[0], torch.ones(3))


def test_delta_cap_saves_waves():
    """comm_sms_min < comm_sms: a delta GEMM takes the extra CTAs only where they save a wave of
    256 x 256 output tiles (148 SMs: 4096^2 = 256 tiles, 5 waves on 62 pairs, 4 on 64)."""
    from lich_b200.data_parallel import DataParallelIPC

    m = _OracleModel([torch.zeros(a, b) for a, b in zip(DIMS[:-1], DIMS[1:])])
    m.cfg = _Cfg(dims=(1000, 4096, 4096, 300))
    dp = DataParallelIPC(m.cfg, device=torch.device("cpu"), model=m, comm_sms=24, comm_sms_min=16)
    dp._sms = lambda: 148
    assert dp._leave_for(1) == 20          # 256 tiles: 64 pairs -> 4 waves
    assert dp._leave_for(0) == 20          # 4 x 16 = 64 tiles: one wave on 64 pairs
    assert dp._leave_for(2) == 24          # 16 x 2 = 32 tiles: one wave already
    fixed = DataParallelIPC(m.cfg, device=torch.device("cpu"), model=m, comm_sms=24, comm_sms_min=24)
    assert fixed._leave_for(1) == 24
    default = DataParallelIPC(m.cfg, device=torch.device("cpu"), model=m, comm_sms=8)
    assert default.comm_sms_min == 8
    with pytest.raises(ValueError):
        DataParallelIPC(m.cfg, device=torch.device("cpu"), model=m, comm_sms=24, comm_sms_min=30)
