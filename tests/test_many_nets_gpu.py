"""GPU tests of ManyNetIPC (many independent hidden-64 networks in one persistent-kernel launch).

* Every network of a multi-network launch is bit-identical to the same network
  trained alone (``TileLangIPC.train_pool``, one network per launch): the
  networks share nothing, and slab n of every stacked buffer is network n.
* The last network of the stack (the highest slab offsets) against the fp32
  oracle on storage-rounded inputs: the 1e-2 gate on x and W after T = 4
  inference iterations and one weight update per step.
* Several (batch, cluster) plans: 8 CTAs x 16 columns at B = 128, 4 x 16 and 8 x 8 at
  B = 64, 4 x 8 at B = 32.
"""
import pytest
import torch

from oracle import ipc_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
DIMS = (10, 64, 64, 64, 784)


def _cfg(dtype, cluster=0):
    from lich_b200.trainer import IPCConfig
    return IPCConfig(dims=DIMS, alpha=1e-4, gamma=0.5, activation="tanh", dtype=dtype, net_cluster=cluster)


def _setup(nets, B, P, dtype, cluster=0):
    from lich_b200 import synthetic as S
    from lich_b200.many_nets import ManyNetIPC
    m = ManyNetIPC(_cfg(dtype, cluster), nets, B, device=DEV)
    ws = [S.fan_in_normal(DIMS, seed=100 + n) for n in range(nets)]
    for n in range(nets):
        m.set_network_weights(n, [w.to(DEV, dtype) for w in ws[n]])
    px, py = S.stacked_pool(DIMS[-1], DIMS[0], B, count=P, nets=nets, seed=7, dtype=dtype)
    return m, ws, px.to(DEV), py.to(DEV)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,cluster", [(128, 8), (64, 4), (64, 8), (32, 4)])
def test_each_network_equals_training_it_alone(dtype, B, cluster):
    from lich_b200.trainer import TileLangIPC
    nets, P, steps = 5, 3, 4
    m, ws, px, py = _setup(nets, B, P, dtype, cluster)
    energy = torch.zeros(steps * nets, device=DEV, dtype=torch.float32)
    m.train_pool(px, py, steps=steps, T=4, energy=energy)
    torch.cuda.synchronize()
    assert m.cluster == cluster
    for n in (0, 2, nets - 1):
        solo = TileLangIPC(_cfg(dtype, cluster), device=DEV)
        for dst, src in zip(solo.w, ws[n]):
            dst.copy_(src.to(DEV, dtype))
        e_solo = torch.zeros(steps, device=DEV, dtype=torch.float32)
        solo.train_pool(px[:, n].contiguous(), py[:, n].contiguous(), steps=steps, T=4, energy=e_solo)
        torch.cuda.synchronize()
        for l in range(len(DIMS) - 1):
            assert torch.equal(m.w[l][n], solo.w[l]), ("w", n, l)
        for l in range(len(DIMS)):
            assert torch.equal(m.x[l][n], solo.x[l]), ("x", n, l)
        # energy is summed with float atomics across the cluster: equal up to summation order
        assert torch.allclose(energy.view(steps, nets)[:, n], e_solo, rtol=1e-5, atol=0), ("energy", n)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_last_network_matches_oracle(dtype):
    nets, B, P = 6, 128, 2
    m, ws, px, py = _setup(nets, B, P, dtype)
    m.train_pool(px, py, steps=1, T=4)
    torch.cuda.synchronize()
    n = nets - 1
    wq = [w.to(dtype).float() for w in ws[n]]
    batches = [(px[b, n].float().cpu(), py[b, n].float().cpu()) for b in range(P)]
    x, w, _, _ = O.train(batches, wq, act="tanh", alpha=1e-4, gamma=0.5, T=4, steps=1)
    for l in range(len(w)):
        assert O.rel_inf(m.w[l][n].cpu(), w[l]) <= 1e-2, ("w", l)
    for l in range(len(x)):
        assert O.rel_inf(m.x[l][n].cpu(), x[l]) <= 1e-2, ("x", l)


def test_pool_shape_checks():
    from lich_b200.many_nets import ManyNetIPC
    m = ManyNetIPC(_cfg(torch.float16), 2, 64, device=DEV)
    bad = torch.zeros((1, 3, DIMS[-1], 64), device=DEV, dtype=torch.float16)
    y = torch.zeros((1, 3, DIMS[0], 64), device=DEV, dtype=torch.float16)
    with pytest.raises(ValueError):
        m.train_pool(bad, y, steps=1)
