"""GPU tests of the batch-sharded data-parallel step (lich_b200.data_parallel).

Both against the CPU oracle's full-batch training step (reference
``reference.py:42-59``): the bf16 weights within 1e-2 of the fp32 oracle, and
the fp32 weight delta ``alpha * sum_b e f(x)^T`` within 1e-2 of the oracle
with the reference kernels' bf16 storage rounding.
One GPU: DataParallelIPC with a single rank, and equality with
TileLangIPC.train_step.  Two GPUs (skipped with fewer): two NCCL ranks, each
with half of the batch, with the all-reduce update and with the
reduce-scatter / sliced apply / all-gather update; the replicas end
bit-identical.
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


def _oracle():
    """Full-batch oracle step: the new W of the fp32 oracle, and the weight delta per layer of the oracle
    with the reference kernels' bf16 storage rounding (``train_step_storage``).  The delta of the
    deepest layer the T = 4 iterations reach comes from errors of a few bf16 ulps of the states, so the
    states' bf16 storage alone moves it 1.3e-2 away from the fp32 oracle's; the storage oracle has the
    same rounding points as the GPU step."""
    w0, x, y = _data()
    dt = torch.bfloat16
    wq = [w.to(dt).float() for w in w0]
    xo, wo, eo, _ = O.train_step(x.to(dt).float(), y.to(dt).float(), wq, act="tanh", alpha=1e-3, gamma=0.5, T=4)
    xs, _, es = O.train_step_storage(x, y, w0, act="tanh", alpha=1e-3, gamma=0.5, T=4, sdt=dt)
    dws = [1e-3 * (es[l].double() @ O.act_forward("tanh", xs[l + 1].double()).to(dt).double().T)
           for l in range(len(wq))]
    return wo, dws


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
    wo, dws = _oracle()
    for l in range(len(wo)):
        assert O.rel_inf(dp.model.w[l].cpu(), wo[l]) <= 1e-2, ("w", l)
        assert O.rel_inf(dp._dw[l].cpu(), dws[l]) <= 1e-2, ("dW", l)


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
        # the summed fp32 delta this rank holds: its slice (reduce-scatter) or all of it (all-reduce)
        dws = []
        for l, dw in enumerate(dp._dw):
            n = dw.numel() // world
            dws.append((rank * n, (rank + 1) * n) if dp._sliced(l) else (0, dw.numel()))
            dws[-1] = dws[-1] + (dw.view(-1)[dws[-1][0]:dws[-1][1]].cpu(),)
        out[rank] = ([w.float().cpu() for w in dp.model.w], dws)
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
    wo, dws = _oracle()
    for a, b in zip(res[0][0], res[1][0]):
        assert torch.equal(a, b)  # replicas identical
    for l, a in enumerate(res[0][0]):
        assert O.rel_inf(a, wo[l]) <= 1e-2, ("w", l)
    for l in range(len(wo)):
        got = torch.zeros(dws[l].numel(), dtype=torch.float64)
        for r in range(2):
            lo, hi, part = res[r][1][l]
            got[lo:hi] = part.double()
        assert O.rel_inf(got.view_as(dws[l]), dws[l]) <= 1e-2, ("dW", l)


# the fused dW + NVSwitch reduction (reduce="nvls") needs tensor-core weight deltas at the local batch
DIMS2 = (104, 512, 512, 1024)
B2 = 1024


def _data2():
    from lich_b200 import synthetic as S
    w0 = S.fan_in_normal(DIMS2, seed=43)
    (x, y), = S.batch_pool(DIMS2[-1], DIMS2[0], B2, count=1, seed=44)
    return w0, x, y


def _worker_nvls(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from lich_b200.data_parallel import DataParallelIPC
        from lich_b200.trainer import IPCConfig
        w0, x, y = _data2()
        cfg = IPCConfig(dims=DIMS2, alpha=1e-3, gamma=0.5, activation="tanh", dtype=torch.bfloat16)
        dp = DataParallelIPC(cfg, device=dev, reduce="nvls", keep_delta=True)
        for dst, src in zip(dp.model.w, w0):
            dst.copy_(src.to(dev, torch.bfloat16))
        cols = slice(rank * B2 // world, (rank + 1) * B2 // world)
        xs, ys = x[:, cols].contiguous().to(dev, torch.bfloat16), y[:, cols].contiguous().to(dev, torch.bfloat16)
        dws, ws = [], []
        for step in range(3):  # both multicast buffers, and the first one again after its zeroing
            for dst, src in zip(dp.model.w, w0):
                dst.copy_(src.to(dev, torch.bfloat16))
            dp.train_step(xs, ys, T=4)
            torch.cuda.synchronize(dev)
            dws.append([d.cpu() for d in dp._dw])
            ws.append([w.float().cpu() for w in dp.model.w])
        out[rank] = (dp.reduce, ws, dws)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
def test_two_ranks_nvls_match_full_batch():
    """The delta GEMMs add into a multicast buffer on both GPUs (IPC_FLAG_MULTIMEM_RED): the summed dW on
    each rank within 1e-2 of the storage oracle's full-batch delta, the new W within 1e-2 of the fp32
    oracle, replicas identical, and the same result on three consecutive steps (both buffers, and one
    reused after its zeroing)."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker_nvls, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
        res = dict(out)
    if res[0][0] != "nvls":
        pytest.skip("no NVLS multicast on these GPUs (the step fell back to the reduce-scatter form)")
    w0, x, y = _data2()
    dt = torch.bfloat16
    wq = [w.to(dt).float() for w in w0]
    _, wo, _, _ = O.train_step(x.to(dt).float(), y.to(dt).float(), wq, act="tanh", alpha=1e-3, gamma=0.5, T=4)
    xs, _, es = O.train_step_storage(x, y, w0, act="tanh", alpha=1e-3, gamma=0.5, T=4, sdt=dt)
    dws = [1e-3 * (es[l].double() @ O.act_forward("tanh", xs[l + 1].double()).to(dt).double().T)
           for l in range(len(wq))]
    for step in range(3):
        for a, b in zip(res[0][1][step], res[1][1][step]):
            assert torch.equal(a, b)  # replicas identical
        for l in range(len(wo)):
            assert O.rel_inf(res[0][1][step][l], wo[l]) <= 1e-2, ("w", step, l)
            for r in range(2):
                assert O.rel_inf(res[r][2][step][l], dws[l]) <= 1e-2, ("dW", r, step, l)
