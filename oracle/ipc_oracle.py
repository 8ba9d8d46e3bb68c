"""CPU oracle for the iPC step -- TEST INFRASTRUCTURE, never the product path.

This module restates, in plain PyTorch on the CPU, the algorithm of the
reference's pure-PyTorch iPC implementation (laghzen/Lich,
``src/ipc_tilelang/reference.py`` and ``src/ipc_tilelang/activations.py``)
together with the element-wise semantics of its three fused GPU operators
(``src/ipc_tilelang/tilelang_kernels.py``).  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it, and only as the checker.  The product (``lich_b200``) never
imports it and has no CPU fallback.

Pinning: ``tests/test_oracle_golden.py`` checks this restatement against
golden vectors produced by running the reference's own ``ipc_step`` in this
container (``tests/golden/make_golden.py``), so parity is pinned to the
reference, not to this file.

Conventions (reference ``README.md:43-50``): every activation tensor is
feature-major ``[features, batch]``; ``W[l]`` is ``[d_l, d_{l+1}]`` and maps
``f(x[l+1]) -> x[l]``; ``x[0]`` is the one-hot target and ``x[L]`` the input.
"""
from __future__ import annotations

from typing import Sequence

import torch

ACTIVATIONS = ("relu", "tanh", "sigmoid", "silu", "gelu", "identity")

_GELU_C = 0.044715
_GELU_K = 0.7978845608028654


def act_forward(name: str, x: torch.Tensor) -> torch.Tensor:
    """f(x); reference ``activations.py:9-15`` (identity: ``weight_update_specialization.py:86``)."""
    if name == "relu":
        return torch.relu(x)
    if name == "tanh":
        return torch.tanh(x)
    if name == "sigmoid":
        return torch.sigmoid(x)
    if name == "silu":
        return torch.nn.functional.silu(x)
    if name == "gelu":
        return torch.nn.functional.gelu(x, approximate="tanh")
    if name == "identity":
        return x
    raise ValueError(f"Unsupported activation: {name}")


def act_derivative(name: str, x: torch.Tensor) -> torch.Tensor:
    """f'(x); reference ``activations.py:16-29``."""
    if name == "relu":
        return (x > 0).to(x.dtype)
    if name == "tanh":
        y = torch.tanh(x)
        return 1 - y * y
    if name == "sigmoid":
        y = torch.sigmoid(x)
        return y * (1 - y)
    if name == "silu":
        s = torch.sigmoid(x)
        return s * (1 + x * (1 - s))
    if name == "gelu":
        u = _GELU_K * (x + _GELU_C * x * x * x)
        t = torch.tanh(u)
        du = _GELU_K * (1 + 3 * _GELU_C * x * x)
        return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * du
    if name == "identity":
        return torch.ones_like(x)
    raise ValueError(f"Unsupported activation: {name}")


def one_hot(labels: torch.Tensor, num_classes: int, *, dtype: torch.dtype) -> torch.Tensor:
    """``[C, B]`` one-hot target; reference ``reference.py:12-13``."""
    return torch.nn.functional.one_hot(labels, num_classes=num_classes).to(dtype=dtype).T.contiguous()


def init_weights(dims: Sequence[int], *, dtype: torch.dtype, device, seed: int = 0) -> list[torch.Tensor]:
    """``W[l] ~ kaiming_uniform_(a=sqrt(5))`` = U(-1/sqrt(fan_in), 1/sqrt(fan_in)), drawn in layer order
    from ONE generator of ``device`` seeded with ``seed``; reference ``reference.py:15-22`` (the trainer
    consumes the generator in the same order, ``trainer.py:97-108``)."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    out = []
    for n_l, n_u in zip(dims[:-1], dims[1:]):
        w = torch.empty((n_l, n_u), device=device, dtype=dtype)
        torch.nn.init.kaiming_uniform_(w, a=5 ** 0.5, generator=g)
        out.append(w)
    return out


# --------------------------------------------------------------------------
# Whole-network step (reference.py)
# --------------------------------------------------------------------------

def forward_init(x_input: torch.Tensor, y_target: torch.Tensor, w: Sequence[torch.Tensor], act: str) -> list[torch.Tensor]:
    """Hidden states from one forward prediction sweep.

    Follows ``scripts/validate_reference.py:27-30`` and the trainer's
    ``initialize_batch`` (``trainer.py:509-516``): ``x[L] = input``;
    ``x[l] = W[l] @ f(x[l+1])`` for ``l = L-1 .. 1``; ``x[0] = target``.
    (The reference ``initialize_state`` leaves hidden states at zero,
    ``reference.py:31-32``; the trainer and the validation script do not.)
    """
    L = len(w)
    B = x_input.shape[1]
    dims = [wi.shape[0] for wi in w] + [w[-1].shape[1]]
    x = [torch.zeros((d, B), dtype=x_input.dtype) for d in dims]
    x[L] = x_input.clone()
    for l in reversed(range(L)):
        pred = w[l] @ act_forward(act, x[l + 1])
        if l > 0:
            x[l] = pred
    x[0] = y_target.clone()
    return x


def prediction_errors(x: Sequence[torch.Tensor], w: Sequence[torch.Tensor], act: str) -> list[torch.Tensor]:
    """``e[l] = x[l] - W[l] @ f(x[l+1])`` for ``l = 0..L-1``; reference ``reference.py:35-40``.

    ``e[L]`` is left as zeros of x[L]'s shape (the reference allocates it with
    ``empty_like`` and never writes it)."""
    L = len(w)
    e = [torch.zeros_like(xi) for xi in x]
    for l in range(L):
        e[l] = x[l] - w[l] @ act_forward(act, x[l + 1])
    return e


def ipc_step(x: Sequence[torch.Tensor], w: Sequence[torch.Tensor], *, act: str, alpha: float, gamma: float,
             update_weights: bool = True):
    """One iPC step; reference ``reference.py:42-59``.

    Returns ``(new_x, new_w, e, metrics)``.  The state update uses x/W/e of the
    same logical time (``:47-49``), the endpoints stay fixed (``:50``) and the
    weight update consumes the *updated* x (``:52-57``).
    """
    L = len(w)
    e = prediction_errors(x, w, act)
    new_x = [v.clone() for v in x]
    for l in range(1, L):
        signal = w[l - 1].T @ e[l - 1]
        new_x[l] = x[l] + gamma * (-e[l] + act_derivative(act, x[l]) * signal)
    new_w = [v.clone() for v in w]
    if update_weights:
        for l in range(L):
            a_new = act_forward(act, new_x[l + 1])
            new_w[l] = w[l] + alpha * (e[l] @ a_new.T)
    energy = sum((q.float() ** 2).mean() for q in e[:-1])
    max_abs = max(q.float().abs().max() for q in e[:-1])
    return new_x, new_w, e, {"energy": float(energy), "max_abs_error": float(max_abs)}


def train_step(x_input: torch.Tensor, y_target: torch.Tensor, w: Sequence[torch.Tensor], *, act: str,
               alpha: float, gamma: float, T: int):
    """One training step of the "T inference iterations + 1 weight update" schedule.

    ``for t in range(T): ipc_step(..., update_weights=(t == T-1))`` after a
    forward-init sweep of the batch -- the weight update uses the errors of the
    last iteration and the states it produced.  Returns ``(x, w, e, metrics)``.
    """
    x = forward_init(x_input, y_target, w, act)
    e = None
    metrics = {}
    for t in range(T):
        x, w, e, metrics = ipc_step(x, w, act=act, alpha=alpha, gamma=gamma, update_weights=(t == T - 1))
    return x, list(w), e, metrics


def train(batches: Sequence[tuple[torch.Tensor, torch.Tensor]], w: Sequence[torch.Tensor], *, act: str,
          alpha: float, gamma: float, T: int, steps: int, first_batch: int = 0):
    """``steps`` training steps; step ``s`` uses ``batches[(first_batch + s) % len(batches)]``."""
    w = [wi.clone() for wi in w]
    x = e = None
    metrics = {}
    for s in range(steps):
        xi, yi = batches[(first_batch + s) % len(batches)]
        x, w, e, metrics = train_step(xi, yi, w, act=act, alpha=alpha, gamma=gamma, T=T)
    return x, w, e, metrics


# --------------------------------------------------------------------------
# Single fused operators (tilelang_kernels.py), with the storage-dtype
# rounding points of the reference kernels.  ``sdt`` is the storage dtype
# (float16 / bfloat16 / float32); arithmetic is done in float64 so the only
# rounding the oracle adds is the storage rounding the reference kernels do.
# --------------------------------------------------------------------------

def _rnd(t: torch.Tensor, sdt: torch.dtype) -> torch.Tensor:
    return t.to(sdt).to(torch.float64)


def pred_err_op(x_up, w, x_lo, *, act: str, sdt: torch.dtype) -> torch.Tensor:
    """``E = cast(X_lo) - cast(W @ f(X_up))``; reference ``tilelang_kernels.py:159-173``.

    f is applied to the storage-dtype X_up and rounded to the storage dtype
    (``a_shared`` is a storage-dtype buffer, ``:143,163``); the product is
    accumulated wide, rounded to the storage dtype, then subtracted and
    rounded again (``:173``)."""
    a = _rnd(act_forward(act, x_up.double()), sdt)
    mu = _rnd(w.double() @ a, sdt)
    return (x_lo.double() - mu).to(sdt)


def infer_update_op(x, e, w_low, e_low, *, act: str, gamma: float, sdt: torch.dtype, save_activation: bool = False):
    """``X += gamma*(-E + f'(X) * W_low^T @ E_low)``; reference ``tilelang_kernels.py:219-231,251-262``.

    Returns ``(x_new, a_out)``; ``a_out = f(x_new)`` from the wide x_new when
    ``save_activation`` (``:231``), else None."""
    xd = x.double()
    acc = w_low.double().T @ e_low.double()
    x_new = xd + gamma * (-e.double() + act_derivative(act, xd) * acc)
    a_out = act_forward(act, x_new).to(sdt) if save_activation else None
    return x_new.to(sdt), a_out


def weight_update_op(w, e, x_up, *, act: str, alpha: float, sdt: torch.dtype, recompute_activation: bool = True):
    """``W = cast(W + alpha * E @ A^T)``; reference ``tilelang_kernels.py:304-320,337-346``.

    ``A = cast(f(X_up))`` when ``recompute_activation``, else ``X_up`` is the
    saved activation itself."""
    a = _rnd(act_forward(act, x_up.double()), sdt) if recompute_activation else x_up.double()
    acc = e.double() @ a.T
    return (w.double() + alpha * acc).to(sdt)


def weight_delta_op(e, x_up, *, act: str, alpha: float, sdt: torch.dtype, recompute_activation: bool = True):
    """``alpha * E @ A^T`` in float64, before the storage rounding of W."""
    a = _rnd(act_forward(act, x_up.double()), sdt) if recompute_activation else x_up.double()
    return alpha * (e.double() @ a.T)


def rel_inf(got: torch.Tensor, ref: torch.Tensor) -> float:
    """``max|got - ref| / max|ref|`` -- the norm-wise relative error the parity gates use."""
    g = got.double()
    r = ref.double()
    den = r.abs().max().item()
    num = (g - r).abs().max().item()
    if den == 0.0:
        return num
    return num / den


# --------------------------------------------------------------------------
# The whole training step with the reference GPU path's storage rounding.
#
# The reference trainer runs the fused operators on storage-dtype tensors
# (trainer.py:601-674) after an eager storage-dtype forward sweep
# (trainer.py:509-516).  Composing the single-operator restatements above in
# that order gives the same rounding points, so a discontinuous f' (relu)
# sees the same rounded states as the GPU kernels do.
# --------------------------------------------------------------------------

def inference_storage(x_input, y_target, w, *, act: str, gamma: float, T: int, sdt: torch.dtype):
    """Forward sweep and T x (P, I) in storage dtype; returns ``(x, e)`` of the last iteration (e computed
    before its state update, x after it -- the operands of the weight update)."""
    L = len(w)
    w = [wi.to(sdt) for wi in w]
    dims = [wi.shape[0] for wi in w] + [w[-1].shape[1]]
    B = x_input.shape[1]
    x = [torch.zeros((d, B), dtype=sdt) for d in dims]
    x[L] = x_input.to(sdt)
    for l in reversed(range(1, L)):
        a = _rnd(act_forward(act, x[l + 1].double()), sdt)
        x[l] = (w[l].double() @ a).to(sdt)
    x[0] = y_target.to(sdt)
    e = None
    for _ in range(T):
        e = [pred_err_op(x[l + 1], w[l], x[l], act=act, sdt=sdt) for l in range(L)]
        new_x = list(x)
        for l in range(1, L):
            new_x[l], _ = infer_update_op(x[l], e[l], w[l - 1], e[l - 1], act=act, gamma=gamma, sdt=sdt)
        x = new_x
    return x, e


def train_step_storage(x_input, y_target, w, *, act: str, alpha: float, gamma: float, T: int, sdt: torch.dtype):
    """One training step (forward sweep, T x (P, I), W with the last iteration's e) in storage dtype.

    Inputs are CPU tensors; returns ``(x, w, e)`` as storage-dtype tensors."""
    x, e = inference_storage(x_input, y_target, w, act=act, gamma=gamma, T=T, sdt=sdt)
    w = [weight_update_op(w[l].to(sdt), e[l], x[l + 1], act=act, alpha=alpha, sdt=sdt) for l in range(len(w))]
    return x, w, e


def train_storage(batches, w, *, act: str, alpha: float, gamma: float, T: int, steps: int, sdt: torch.dtype,
                  first_batch: int = 0):
    x = e = None
    for s in range(steps):
        xi, yi = batches[(first_batch + s) % len(batches)]
        x, w, e = train_step_storage(xi, yi, w, act=act, alpha=alpha, gamma=gamma, T=T, sdt=sdt)
    return x, w, e


# --------------------------------------------------------------------------
# Optimizer steps on the weight update (no reference counterpart: the
# reference lists fused SGD / AdamW epilogues as future work, README.md:168,
# PERFORMANCE_CHECKLIST.md:103-104).  Restated from the published algorithms
# as torch.optim documents them (SGD: dampening 0, no Nesterov, buffer
# started at zero; AdamW: Loshchilov & Hutter, decoupled weight decay,
# bias-corrected moments).  The gradient of the energy sum_l |e_l|^2 / 2 with
# respect to W[l] is g = -e[l] @ f(x[l+1])^T (summed over the batch).
# --------------------------------------------------------------------------

def optim_step(w, g, state: dict, *, kind: str, lr: float, momentum: float = 0.0, weight_decay: float = 0.0,
               betas=(0.9, 0.999), eps: float = 1e-8):
    """One step on float64 copies; ``state`` holds ``m`` / ``v`` / ``t`` and is updated.  Returns new w."""
    w = w.double()
    g = g.double()
    if kind == "adamw":
        b1, b2 = betas
        t = state.get("t", 0) + 1
        m = state.get("m", torch.zeros_like(w)) * b1 + (1 - b1) * g
        v = state.get("v", torch.zeros_like(w)) * b2 + (1 - b2) * g * g
        state.update(t=t, m=m, v=v)
        w = w * (1 - lr * weight_decay)
        return w - (lr / (1 - b1 ** t)) * m / (v.sqrt() / (1 - b2 ** t) ** 0.5 + eps)
    if kind == "sgd":
        g = g + weight_decay * w
        if momentum != 0.0:
            g = state.get("m", torch.zeros_like(w)) * momentum + g
            state["m"] = g
        return w - lr * g
    raise ValueError(f"unknown optimizer {kind!r}")


def train_step_opt(x_input, y_target, w, states, *, act: str, gamma: float, T: int, **opt):
    """One training step whose weight update is an optimizer step: forward sweep, T inference iterations,
    then ``optim_step`` per layer with g = -e f(x_new)^T of the last iteration.  ``states``: one dict per
    layer, updated.  Returns ``(x, w, e)``."""
    x = forward_init(x_input, y_target, w, act)
    e = None
    for _ in range(T):
        x, _, e, _ = ipc_step(x, w, act=act, alpha=0.0, gamma=gamma, update_weights=False)
    new_w = []
    for l in range(len(w)):
        g = -(e[l].double() @ act_forward(act, x[l + 1].double()).T)
        new_w.append(optim_step(w[l], g, states[l], **opt).to(w[l].dtype))
    return x, new_w, e


def train_step_opt_storage(x_input, y_target, w, states, *, act: str, gamma: float, T: int, sdt: torch.dtype, **opt):
    """``train_step_opt`` with the reference kernels' storage rounding (``inference_storage``; the gradient
    from the stored e and cast(f(x))).  Returns ``(x, w, e)`` with w in ``sdt``."""
    x, e = inference_storage(x_input, y_target, w, act=act, gamma=gamma, T=T, sdt=sdt)
    new_w = []
    for l in range(len(w)):
        g = -(e[l].double() @ _rnd(act_forward(act, x[l + 1].double()), sdt).T)
        new_w.append(optim_step(w[l].to(sdt), g, states[l], **opt).to(sdt))
    return x, new_w, e
