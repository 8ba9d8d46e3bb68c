"""Pin the CPU oracle (oracle/ipc_oracle.py) to the reference's own outputs.

The golden vectors were produced by the reference's ``ipc_step``
(``src/ipc_tilelang/reference.py:42-59``) via ``tests/golden/make_golden.py``.
"""
import pytest
import torch

from oracle import ipc_oracle as O
from tests.golden_io import cases, load, load_init


@pytest.mark.parametrize("name", cases())
def test_oracle_matches_reference_golden(name):
    meta, w_in, batches, w_out, x_out = load(name)
    torch.set_num_threads(1)
    if meta["single_step_no_w"]:
        xb, yb = batches[0]
        x = O.forward_init(xb, yb, w_in, meta["activation"])
        x, w, e, m = O.ipc_step(x, w_in, act=meta["activation"], alpha=meta["alpha"], gamma=meta["gamma"],
                                update_weights=False)
    else:
        x, w, e, m = O.train(batches, w_in, act=meta["activation"], alpha=meta["alpha"], gamma=meta["gamma"],
                             T=meta["T"], steps=meta["steps"])
    for l, (got, ref) in enumerate(zip(w, w_out)):
        assert O.rel_inf(got, ref) <= 1e-6, (name, "w", l)
    for l, (got, ref) in enumerate(zip(x, x_out)):
        assert O.rel_inf(got, ref) <= 1e-6, (name, "x", l)
    assert abs(m["energy"] - meta["energy"]) <= 1e-5 * max(1.0, abs(meta["energy"]))
    assert abs(m["max_abs_error"] - meta["max_abs_error"]) <= 1e-5 * max(1.0, abs(meta["max_abs_error"]))


def test_weight_delta_nonzero_in_large_alpha_cases():
    """The small golden cases use alpha=0.05 so that W actually moves; guard that."""
    meta, w_in, batches, w_out, x_out = load("small_tanh")
    assert max((a - b).abs().max().item() for a, b in zip(w_in, w_out)) > 1e-3


def test_no_w_case_keeps_weights():
    meta, w_in, batches, w_out, x_out = load("small_tanh_no_w")
    for a, b in zip(w_in, w_out):
        assert torch.equal(a, b)


def test_kernel_ops_reduce_to_whole_step():
    """The single-operator restatements (fp32 storage) compose to one reference step."""
    meta, w_in, batches, w_out, x_out = load("small_gelu")
    xb, yb = batches[0]
    act = meta["activation"]
    x = O.forward_init(xb, yb, w_in, act)
    x_ref, w_ref, e_ref, _ = O.ipc_step(x, w_in, act=act, alpha=meta["alpha"], gamma=meta["gamma"])
    L = len(w_in)
    f64 = torch.float64
    e = [O.pred_err_op(x[l + 1], w_in[l], x[l], act=act, sdt=f64) for l in range(L)]
    xn = list(x)
    for l in range(1, L):
        xn[l], _ = O.infer_update_op(x[l], e[l], w_in[l - 1], e[l - 1], act=act, gamma=meta["gamma"], sdt=f64)
    wn = [O.weight_update_op(w_in[l], e[l], xn[l + 1], act=act, alpha=meta["alpha"], sdt=f64) for l in range(L)]
    for l in range(L):
        assert O.rel_inf(e[l], e_ref[l]) < 1e-5
        assert O.rel_inf(wn[l], w_ref[l]) < 1e-6
    for l in range(1, L):
        assert O.rel_inf(xn[l], x_ref[l]) < 1e-6


def test_oracle_init_matches_reference_init():
    """oracle.init_weights draws the reference's init_weights values (CPU generator, same seeds)."""
    for dims, seed, ref in load_init():
        got = O.init_weights(dims, dtype=torch.float32, device="cpu", seed=seed)
        assert len(got) == len(ref)
        for a, b in zip(got, ref):
            assert torch.equal(a, b), (dims, seed)


def test_optim_step_matches_torch_optim():
    """oracle.optim_step follows torch.optim.SGD / AdamW step for step (CPU, float64)."""
    g0 = torch.Generator().manual_seed(3)
    w0 = torch.randn(7, 5, generator=g0, dtype=torch.float64)
    grads = [torch.randn(7, 5, generator=g0, dtype=torch.float64) for _ in range(4)]
    cases = [("adamw", dict(lr=1e-2, weight_decay=0.1, betas=(0.8, 0.95), eps=1e-6),
              lambda p: torch.optim.AdamW([p], lr=1e-2, weight_decay=0.1, betas=(0.8, 0.95), eps=1e-6)),
             ("sgd", dict(lr=5e-2, momentum=0.9, weight_decay=0.01),
              lambda p: torch.optim.SGD([p], lr=5e-2, momentum=0.9, weight_decay=0.01)),
             ("sgd", dict(lr=5e-2), lambda p: torch.optim.SGD([p], lr=5e-2))]
    for kind, kw, make in cases:
        p = torch.nn.Parameter(w0.clone())
        opt = make(p)
        w, state = w0.clone(), {}
        for g in grads:
            p.grad = g.clone()
            opt.step()
            w = O.optim_step(w, g, state, kind=kind, **kw)
            assert torch.allclose(w, p.detach(), rtol=1e-12, atol=1e-12), (kind, kw)


def test_plain_sgd_step_is_the_ipc_update():
    """SGD without momentum or decay at lr = alpha is the reference weight update W += alpha E A^T."""
    meta, w_in, batches, w_out, x_out = load("small_tanh")
    xb, yb = batches[0]
    x, w, e = O.train_step_opt(xb, yb, w_in, [{} for _ in w_in], act="tanh", gamma=meta["gamma"], T=meta["T"],
                               kind="sgd", lr=meta["alpha"])
    x2, w2, e2, _ = O.train_step(xb, yb, w_in, act="tanh", alpha=meta["alpha"], gamma=meta["gamma"], T=meta["T"])
    for a, b in zip(w, w2):
        assert O.rel_inf(a, b) <= 1e-6
