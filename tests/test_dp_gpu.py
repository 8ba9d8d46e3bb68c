"""GPU tests of the batch-sharded data-parallel step (lich_b200.data_parallel).

One GPU: DataParallelIPC with a single rank is exactly TileLangIPC.train_step.
Two GPUs (skipped with fewer): two NCCL ranks, each with half of the batch,
end with the same weights as the full batch on one GPU (1e-2, 16-bit gate)
and bit-identical replicas, with the all-reduce update and with the
reduce-scatter / sliced apply / all-gather update.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DIMS = (104, 256, 256, 256, 512)
B = 256


def _cfg():
    from lich_b200.trainer import IPCConfig
    return IPCConfig(dims=DIMS, alpha=1e-3, gamma=0.5, activation="tanh", dtype=torch.bfloat16)


def _data():
    from lich_b200 import synthetic as S
    w0 = S.fan_in_normal(DIMS, seed=41)
    (x, y), = S.batch_pool(DIMS[-1], DIMS[0], B, count=1, seed=42)
    return w0, x, y


def _full_batch_reference(dev):
    from lich_b200.trainer import TileLangIPC
    w0, x, y = _data()
    m = TileLangIPC(_cfg(), device=dev)
    for dst, src in zip(m.w, w0):
        dst.copy_(src.to(dev, torch.bfloat16))
    m.train_step(x.to(dev, torch.bfloat16), y.to(dev, torch.bfloat16), T=4)
    return [w.float().cpu() for w in m.w]


def test_single_rank_equals_trainer_step():
    from lich_b200.data_parallel import DataParallelIPC
    dev = torch.device("cuda", 0)
    w0, x, y = _data()
    dp = DataParallelIPC(_cfg(), device=dev)
    for dst, src in zip(dp.model.w, w0):
        dst.copy_(src.to(dev, torch.bfloat16))
    dp.train_step(x.to(dev, torch.bfloat16), y.to(dev, torch.bfloat16), T=4)
    ref = _full_batch_reference(dev)
    for a, b in zip(dp.model.w, ref):
        assert O.rel_inf(a.float().cpu(), b) <= 1e-2


def _worker(rank, world, port, out, reduce):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from lich_b200.data_parallel import DataParallelIPC
        w0, x, y = _data()
        dp = DataParallelIPC(_cfg(), device=dev, reduce=reduce)
        for dst, src in zip(dp.model.w, w0):
            dst.copy_(src.to(dev, torch.bfloat16))
        cols = slice(rank * B // world, (rank + 1) * B // world)
        dp.train_step(x[:, cols].contiguous().to(dev, torch.bfloat16),
                      y[:, cols].contiguous().to(dev, torch.bfloat16), T=4)
        torch.cuda.synchronize(dev)
        out[rank] = [w.float().cpu() for w in dp.model.w]
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
@pytest.mark.parametrize("reduce", ["rs_ag", "allreduce"])
def test_two_ranks_match_full_batch(reduce):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, port, out, reduce), nprocs=2, join=True, start_method="spawn")
        res = dict(out)
    ref = _full_batch_reference(torch.device("cuda", 0))
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)  # replicas identical
    for a, b in zip(res[0], ref):
        assert O.rel_inf(a, b) <= 1e-2
