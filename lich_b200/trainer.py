"""iPC trainer -- the drop-in for ``ipc_tilelang.trainer`` (``IPCConfig``, ``TileLangIPC``, ``prepare_batch``).

Same constructor, attributes and methods as the reference
(``src/ipc_tilelang/trainer.py:28-846``); the step runs on sm_100a kernels:

* **net path** (16-bit storage, every width except the input <= 64, B a
  multiple of 8 up to 256, recompute mode): one launch of the persistent
  multi-layer kernel (``ipc_net_train``) per call -- ``step_initialized`` is
  one launch instead of the reference's 3L-1, and a whole training step
  (forward-init sweep, T inference iterations, weight update) is also one
  launch (``train_step`` / ``train_pool``);
* **operator path** (anything else: fp32, wide layers, save-activation
  mode): the fused P / I / W operators in the reference's phase order
  (``trainer.py:609-674``), with grid.z layer batching of square internal
  layers (``layer_batching.find_internal_square_groups``).

Additions (no reference counterpart): ``step_initialized(update_weights=)``
for the "T inference iterations + 1 weight update" schedule,
``train_step`` / ``train_pool`` / ``run_inference``, and
``state_dict`` / ``load_state_dict``.

Tuning (``lich_b200.tuning``), consulted as the reference does
(``trainer.py:180-215,268-345``): per operator shape the execution policy's
kernel rows (``hierarchical_policy_path``, when ``hierarchical_policy_auto``),
then ``tuning_table`` (a ``TuningTable`` or a path; ``None`` on a B200 means
the table measured on B200 that ships with the package), then ``cfg.kernel``.
With ``grid_z_auto`` the grid.z layer cap for a batch comes from the execution
policy or ``grid_z_policy_path`` (default ``grid_z_max_layers``), and the
weights are regrouped before the first step of that batch.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field, replace
from typing import Sequence

import torch

from . import _native as N
from .activations import get_activation
from .layer_batching import (
    LayerBatchGroup,
    build_forward_batched,
    build_inference_update_batched,
    build_prediction_error_batched,
    build_weight_update_batched,
    find_internal_square_groups,
)
from .tilelang_kernels import (
    KernelConfig,
    build_forward,
    build_inference_update,
    build_prediction_error,
    build_weight_update,
)
from .tuning import ExecutionPolicy, TuningTable, default_table, lookup_grid_z_cap
from .weight_update_specialization import SmallBWeightPolicy, SmallBWeightUpdater

TARGET_CAPABILITY = (10, 0)


def one_hot(labels: torch.Tensor, num_classes: int, *, dtype: torch.dtype) -> torch.Tensor:
    """``[C, B]`` one-hot target on the labels' device (reference ``reference.py:12-13``)."""
    y = torch.zeros((num_classes, labels.numel()), dtype=dtype, device=labels.device)
    y.scatter_(0, labels.reshape(1, -1).long(), 1.0)
    return y


@dataclass(frozen=True)
class IPCConfig:
    dims: tuple[int, ...]
    alpha: float = 1e-4
    gamma: float = 0.5
    activation: str = "relu"
    dtype: torch.dtype = torch.float16
    kernel: KernelConfig = KernelConfig()
    recompute_activation: bool = True
    tuning_table: TuningTable | str | None = None
    use_grid_z: bool = True
    grid_z_max_layers: int = 2
    grid_z_auto: bool = True
    grid_z_policy_path: str = "results/gridz_policy.json"
    hierarchical_policy_auto: bool = True
    hierarchical_policy_path: str = "results/hierarchical_policy.json"
    steady_state_graph_auto: bool = True
    steady_state_graph_default: bool = False
    weight_update_mode: str = "gemm"
    weight_update_policy_path: str = "results/weight_update_policy.json"
    weight_update_outer_max_batch: int = 16
    # sm_100a additions
    use_net_kernel: bool = True
    net_cluster: int = 0
    # optimizer of the weight update, fused where the product meets W (no gradient tensor): "sgd" with
    # momentum = weight_decay = 0 is the reference update W += alpha E f(x)^T; "adamw" / momentum / weight
    # decay follow torch.optim.AdamW / SGD with lr = alpha and gradient -E f(x)^T
    optimizer: str = "sgd"
    momentum: float = 0.0
    weight_decay: float = 0.0
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8


class TileLangIPC:
    """iPC MLP trainer on one B200; see the module docstring."""

    def __init__(self, cfg: IPCConfig, *, device: torch.device, seed: int = 0):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("TileLangIPC requires a CUDA device")
        cap = torch.cuda.get_device_capability(device)
        if cap != TARGET_CAPABILITY:
            raise ValueError(f"lich_b200 is built for sm_100a (B200); got capability {cap}")
        if len(cfg.dims) < 2:
            raise ValueError("dims needs at least two entries")
        self.cfg = cfg
        self.device = device
        self.act = get_activation(cfg.activation)
        N.dtype_code(cfg.dtype)
        self._runtime_recompute_activation = bool(cfg.recompute_activation)
        self._tuning = TuningTable.load(cfg.tuning_table)
        if self._tuning is None:
            self._tuning = default_table()
        self._policy: ExecutionPolicy | None = None
        if cfg.hierarchical_policy_auto:
            try:
                pol = ExecutionPolicy(cfg.hierarchical_policy_path)
                self._policy = pol if pol.exists else None
            except (OSError, ValueError):
                self._policy = None
        self._kcfg_cache: dict = {}
        self._predict_bufs: dict = {}
        if str(cfg.optimizer).lower() not in N.OPT_KINDS:
            raise ValueError(f"unknown optimizer {cfg.optimizer!r} (sgd or adamw)")
        self._opt_state: list | None = None  # per layer (m, v) fp32, allocated at the first update
        self._opt_steps = 0
        self._opt_ws: torch.Tensor | None = None
        self._grid_z_batch: int | None = None
        self._grid_z_cap = max(0, int(cfg.grid_z_max_layers))
        self._layer_groups: tuple[LayerBatchGroup, ...] = (
            find_internal_square_groups(tuple(cfg.dims), max_group_count=self._grid_z_cap)
            if cfg.use_grid_z and self._grid_z_cap >= 2 else ()
        )
        self._edge_to_group = {l: gi for gi, g in enumerate(self._layer_groups) for l in g.edge_indices}

        # Weight init: kaiming_uniform_(a=sqrt(5)) in layer order from one device generator,
        # grouped layers stored in one [G, D, D] tensor (reference trainer.py:88-108).
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        self.w: list[torch.Tensor] = [None] * (len(cfg.dims) - 1)  # type: ignore[list-item]
        self._w_grouped = [torch.empty((gr.count, gr.width, gr.width), device=device, dtype=cfg.dtype)
                           for gr in self._layer_groups]
        for l, (n_l, n_u) in enumerate(zip(cfg.dims[:-1], cfg.dims[1:])):
            gi = self._edge_to_group.get(l)
            w = (torch.empty((n_l, n_u), device=device, dtype=cfg.dtype) if gi is None
                 else self._w_grouped[gi][l - self._layer_groups[gi].start])
            torch.nn.init.kaiming_uniform_(w, a=5 ** 0.5, generator=g)
            self.w[l] = w

        self.x: list[torch.Tensor] | None = None
        self.e: list[torch.Tensor] | None = None
        self.a: list[torch.Tensor | None] | None = None
        self._x_grouped: list[torch.Tensor] = []
        self._e_grouped: list[torch.Tensor] = []
        self._a_grouped: list[torch.Tensor] | None = None
        # activation cache of the 16-bit operator path: ac[l] = cast(f(x[l])), written by the forward
        # sweep and the state-update epilogues, read as the stored operand of P / W (tensor-core GEMMs)
        self._ac: list[torch.Tensor] | None = None
        self._splitk_ws: torch.Tensor | None = None
        self._net_sync: torch.Tensor | None = None
        self._net_acache: list | None = None
        self._ac_grouped: list[torch.Tensor] = []
        self._runtime_plan_key: tuple | None = None
        self._pred_singleton_kernels: list[object | None] = []
        self._inf_singleton_kernels: list[object | None] = []
        self._weight_singleton_kernels: list[object | None] = []
        self._fwd_singleton_kernels: list[object | None] = []
        self._pred_singleton_ops: tuple = ()
        self._inf_singleton_ops: tuple = ()
        self._weight_singleton_ops: tuple = ()
        self._pred_group_kernels: tuple = ()
        self._inf_group_kernels: tuple = ()
        self._weight_group_kernels: tuple = ()
        self._weight_singleton_outer_ops: tuple = ()
        self._weight_group_outer_ops: tuple = ()
        self._steady_state_runner = None
        self._steady_state_graph_key: tuple | None = None
        self._steady_state_graph_steps: int | None = None
        self._graph_pool = None  # private memory pool shared by this model's captured graphs
        self._net_desc = None
        self._net_keep = None
        self.steps_done = 0
        self._weight_update_policy: SmallBWeightPolicy | None = None
        self._small_b_updater = SmallBWeightUpdater(alpha=float(cfg.alpha))
        if str(cfg.weight_update_mode).lower() == "auto":
            try:
                self._weight_update_policy = SmallBWeightPolicy(cfg.weight_update_policy_path)
            except Exception:
                self._weight_update_policy = None

    # ------------------------------------------------------------------ info
    @property
    def L(self) -> int:
        return len(self.w)

    @property
    def recompute_activation(self) -> bool:
        return bool(self._runtime_recompute_activation)

    @property
    def dtype_name(self) -> str:
        return str(self.cfg.dtype).split(".")[-1]

    @property
    def fused_optimizer(self) -> bool:
        """Whether the weight update is an optimizer step (AdamW, momentum or weight decay) rather than the
        reference update; such models take the operator path."""
        c = self.cfg
        return str(c.optimizer).lower() == "adamw" or float(c.momentum) != 0.0 or float(c.weight_decay) != 0.0

    def net_kernel_eligible(self, batch: int | None = None) -> bool:
        """Whether ``step_initialized`` / ``train_pool`` run as one persistent-kernel launch."""
        d = self.cfg.dims
        ok = (self.cfg.use_net_kernel and self.cfg.dtype in (torch.float16, torch.bfloat16)
              and not self.fused_optimizer
              and self.recompute_activation and 1 <= self.L <= N.NET_MAX_LAYERS)
        if not ok:
            return False
        if batch is None:  # without a batch size: whether the small-width (cluster) kernel applies
            return all(int(v) <= 64 for v in d[:-1])
        # small widths: one cluster per network; wide layers at B <= 16: the cooperative small-batch kernel
        return N.net_plan(d, int(batch), 1, int(self.cfg.net_cluster)) is not None

    def recommended_use_cuda_graph(self, batch: int | None = None, *, default: bool = False) -> bool:
        """The execution policy's choice for this network and batch, else ``default`` (the net path is one
        launch per block of steps already)."""
        if self._policy is None or batch is None:
            return bool(default)
        return bool(self._policy.selected("use_cuda_graph", bool(default), **self._policy_key(int(batch))))

    # ----------------------------------------------------------------- tuning
    def _policy_key(self, batch: int) -> dict:
        sigs = ["sm100a-v1"] + ([self._tuning.signature()] if self._tuning is not None else [])
        return {"dims": tuple(self.cfg.dims), "batch": int(batch), "activation": self.cfg.activation,
                "dtype": self.cfg.dtype, "signatures": sigs}

    def _kernel_config(self, kind: str, M: int, K: int, B: int) -> KernelConfig:
        """Kernel config of one operator shape: execution-policy row, tuning-table row, or ``cfg.kernel``."""
        key = (kind, int(M), int(K), int(B))
        kc = self._kcfg_cache.get(key)
        if kc is None:
            q = dict(kind=kind, M=M, K=K, B=B, activation=self.cfg.activation, dtype=self.cfg.dtype)
            kc = ((self._policy.lookup_kernel(**q) if self._policy is not None else None)
                  or (self._tuning.lookup(**q) if self._tuning is not None else None) or self.cfg.kernel)
            self._kcfg_cache[key] = kc
        return kc

    def _apply_grid_z_policy(self, batch: int) -> None:
        """grid.z layer cap for this batch (execution policy, then the grid.z policy file); regroups the
        weights when it changes (before the batch's buffers are built)."""
        if not (self.cfg.use_grid_z and self.cfg.grid_z_auto) or self._grid_z_batch == int(batch):
            return
        self._grid_z_batch = int(batch)
        cap = None
        if self._policy is not None:
            row = self._policy.lookup_execution(**self._policy_key(batch))
            best = (row or {}).get("best") or {}
            cap = best.get("grid_z_max_layers")
        if cap is None:
            try:
                cap = lookup_grid_z_cap(self.cfg.grid_z_policy_path, device_name=torch.cuda.get_device_name(self.device),
                                        capability=torch.cuda.get_device_capability(self.device), dims=self.cfg.dims,
                                        batch=batch, activation=self.cfg.activation, dtype=self.cfg.dtype,
                                        default=int(self.cfg.grid_z_max_layers))
            except (OSError, ValueError):
                cap = int(self.cfg.grid_z_max_layers)
        cap = max(0, int(cap))
        if cap != self._grid_z_cap:
            self._regroup(cap)

    def _regroup(self, cap: int) -> None:
        """Store the square internal layers in grid.z groups of at most ``cap`` layers (values kept)."""
        old = [w.clone() for w in self.w]
        self._grid_z_cap = cap
        self._layer_groups = (find_internal_square_groups(tuple(self.cfg.dims), max_group_count=cap)
                              if cap >= 2 else ())
        self._edge_to_group = {l: gi for gi, g in enumerate(self._layer_groups) for l in g.edge_indices}
        self._w_grouped = [torch.stack([old[l] for l in g.edge_indices]) for g in self._layer_groups]
        for l in range(len(old)):
            gi = self._edge_to_group.get(l)
            self.w[l] = old[l] if gi is None else self._w_grouped[gi][l - self._layer_groups[gi].start]
        self.x = self.e = self.a = None
        self._runtime_plan_key = None
        self._net_desc = None
        self._invalidate_steady_state_graph()

    def runtime_plan_ready(self) -> bool:
        return self._runtime_plan_key is not None

    def _grouped_edge_indices(self) -> frozenset[int]:
        return frozenset(self._edge_to_group)

    # ---------------------------------------------------------------- buffers
    def _invalidate_steady_state_graph(self) -> None:
        self._steady_state_runner = None
        self._steady_state_graph_key = None
        self._steady_state_graph_steps = None

    def _ensure_buffers(self, B: int) -> None:
        if self.x is not None and self.x[0].shape[1] == B:
            return
        self._apply_grid_z_policy(B)
        self._invalidate_steady_state_graph()
        self._net_desc = None
        dims = self.cfg.dims
        dt, dev = self.cfg.dtype, self.device
        self.x = [None] * len(dims)  # type: ignore[list-item]
        self.e = [None] * len(dims)  # type: ignore[list-item]
        self._x_grouped, self._e_grouped = [], []
        self.a = None if self.recompute_activation else [None] * len(dims)
        self._a_grouped = None if self.recompute_activation else []
        use_ac = self._acache_path(B)
        self._ac = [None] * len(dims) if use_ac else None  # type: ignore[list-item]
        self._ac_grouped = []
        # fp32 scratch of the split-K weight update (narrow layers, long batches); shared by all layers,
        # whose updates are ordered on one stream
        self._splitk_ws = (torch.empty(N.SPLITK_WORKSPACE_BYTES // 4, device=dev, dtype=torch.float32)
                           if use_ac else None)
        grouped_states = set()
        for gi, gr in enumerate(self._layer_groups):
            xbuf = torch.zeros((gr.state_count, gr.width, B), device=dev, dtype=dt)
            ebuf = torch.zeros_like(xbuf)
            self._x_grouped.append(xbuf)
            self._e_grouped.append(ebuf)
            if self._a_grouped is not None:
                self._a_grouped.append(torch.zeros_like(xbuf))
            if use_ac:
                self._ac_grouped.append(torch.zeros_like(xbuf))
            for z, layer in enumerate(gr.state_indices):
                grouped_states.add(layer)
                self.x[layer] = xbuf[z]
                self.e[layer] = ebuf[z]
                if self.a is not None:
                    self.a[layer] = self._a_grouped[gi][z]
                if use_ac:
                    self._ac[layer] = self._ac_grouped[gi][z]
        for layer, d in enumerate(dims):
            if layer in grouped_states:
                continue
            self.x[layer] = torch.zeros((d, B), device=dev, dtype=dt)
            self.e[layer] = torch.zeros_like(self.x[layer])
            if self.a is not None:
                self.a[layer] = torch.zeros_like(self.x[layer])
            if use_ac:
                self._ac[layer] = torch.zeros_like(self.x[layer])
        self._runtime_plan_key = None

    def _acache_path(self, B: int) -> bool:
        """16-bit recompute mode off the persistent kernel: P / W read a cached f(cast(x)) so their GEMMs
        take stored operands (the tensor-core kernel); numerically the recompute semantics."""
        return (self.cfg.dtype in (torch.float16, torch.bfloat16) and self.recompute_activation
                and not self.net_kernel_eligible(B))

    _KIND = {N.MODE_PRED: "prediction", N.MODE_INFER: "inference", N.MODE_WEIGHT: "weight",
             N.MODE_WDELTA: "weight", N.MODE_FORWARD: "forward"}

    def _fg(self, mode, a, b, out, aux=None, aux2=None, *, M, K, B, groups=1, scale=0.0, flags=0):
        ws = self._splitk_ws if mode in (N.MODE_WEIGHT, N.MODE_WDELTA) else None
        kc = self._kernel_config(self._KIND[mode], M, K, B)
        N.fused_gemm(mode, a, b, out, aux, aux2, M=M, K=K, B=B, groups=groups, scale=scale, flags=flags,
                     act=self.cfg.activation, dtype=self.cfg.dtype, algo=getattr(kc, "backend", "auto"),
                     device=self.device, workspace=ws, tune=kc.tune())

    def _prepare_runtime_plan(self, batch: int) -> None:
        """Build the kernel-call plan once per (dims, batch, activation, dtype, mode)."""
        key = (tuple(int(d) for d in self.cfg.dims), int(batch), self.cfg.activation, self.dtype_name,
               self.recompute_activation, self._grid_z_cap)
        if key == self._runtime_plan_key:
            return
        B = int(batch)
        d = self.cfg.dims
        act, dt = self.cfg.activation, self.dtype_name
        kc = self._kernel_config
        grouped = self._grouped_edge_indices()
        grouped_inf = {l for gr in self._layer_groups for l in range(gr.start + 1, gr.end + 2)}
        pred = [None] * self.L
        inf = [None] * self.L
        wgt = [None] * self.L
        fwd = [None] * self.L
        outer_single = []
        for l in range(self.L):
            fwd[l] = build_forward(d[l], d[l + 1], B, act, dt, kc("forward", d[l], d[l + 1], B))
            if l not in grouped:
                pred[l] = build_prediction_error(d[l], d[l + 1], B, act, dt, kc("prediction", d[l], d[l + 1], B))
                M, K = d[l], d[l + 1]
                if self._outer_weight_enabled(M, K, B):
                    op = self._small_b_updater.make_singleton(M=M, K=K, B=B, activation=act, dtype=self.cfg.dtype)
                    if op is not None:
                        outer_single.append((l, op))
                        continue
                wgt[l] = build_weight_update(d[l], d[l + 1], B, act, dt, kc("weight", d[l], d[l + 1], B),
                                             self.cfg.alpha, self.recompute_activation)
        for l in range(1, self.L):
            if l not in grouped_inf:
                inf[l] = build_inference_update(d[l], d[l - 1], B, act, dt, kc("inference", d[l], d[l - 1], B),
                                                self.cfg.gamma, not self.recompute_activation)
        pg, ig, wg, og = [], [], [], []
        for gr in self._layer_groups:
            w_ = gr.width
            pg.append(build_prediction_error_batched(w_, w_, B, gr.count, act, dt, kc("prediction", w_, w_, B)))
            ig.append(build_inference_update_batched(w_, w_, B, gr.count, act, dt, kc("inference", w_, w_, B),
                                                     self.cfg.gamma, not self.recompute_activation))
            outer = None
            if self._outer_weight_enabled(gr.width, gr.width, B, gr.count):
                outer = self._small_b_updater.make_grouped(count=gr.count, M=gr.width, K=gr.width, B=B,
                                                           activation=act, dtype=self.cfg.dtype)
            og.append(outer)
            wg.append(None if outer is not None else build_weight_update_batched(
                w_, w_, B, gr.count, act, dt, kc("weight", w_, w_, B), self.cfg.alpha, self.recompute_activation))
        self._pred_singleton_kernels, self._inf_singleton_kernels = pred, inf
        self._weight_singleton_kernels, self._fwd_singleton_kernels = wgt, fwd
        self._weight_singleton_outer_ops = tuple(outer_single)
        self._pred_singleton_ops = tuple((l, k) for l, k in enumerate(pred) if k is not None)
        self._inf_singleton_ops = tuple((l, k) for l, k in enumerate(inf) if k is not None)
        self._weight_singleton_ops = tuple((l, k) for l, k in enumerate(wgt) if k is not None)
        self._pred_group_kernels, self._inf_group_kernels = tuple(pg), tuple(ig)
        self._weight_group_kernels, self._weight_group_outer_ops = tuple(wg), tuple(og)
        self._runtime_plan_key = key

    def _outer_weight_enabled(self, M: int, K: int, B: int, count: int = 1) -> bool:
        mode = str(self.cfg.weight_update_mode).lower()
        if mode == "outer":
            return True
        if mode != "auto" or int(B) > int(self.cfg.weight_update_outer_max_batch):
            return False
        if self._weight_update_policy is None:
            return True  # measured crossover on B200: the outer kernel wins for B <= 16
        return self._weight_update_policy.backend(M=M, K=K, B=B, activation=self.cfg.activation,
                                                  dtype=self.cfg.dtype, count=count) == "outer"

    # ------------------------------------------------------------ net kernel
    def _net(self):
        if self._net_desc is None:
            desc = N.IpcNet()
            desc.L = self.L
            for l, dv in enumerate(self.cfg.dims):
                desc.dims[l] = int(dv)
            desc.B = int(self.x[0].shape[1])
            desc.nets = 1
            for l in range(self.L):
                desc.w[l] = self.w[l].data_ptr()
                desc.e[l] = self.e[l].data_ptr()
            for l in range(self.L + 1):
                desc.x[l] = self.x[l].data_ptr()
            plan = N.net_plan(self.cfg.dims, desc.B, 1, int(self.cfg.net_cluster))
            if plan is not None and plan[0] == 0:
                # the wide small-batch kernel: activation cache a[l] = cast(f(x[l])) written where x is
                # produced, so every CTA stages f(x) without recomputing it
                self._net_acache = [None] + [torch.empty_like(self.x[l]) for l in range(1, self.L + 1)]
                for l in range(1, self.L + 1):
                    desc.a[l] = self._net_acache[l].data_ptr()
            self._net_desc = desc
        return self._net_desc

    def _net_run(self, *, steps: int, T: int, forward_init: bool, update_weights: bool,
                 pool_x: torch.Tensor | None = None, pool_y: torch.Tensor | None = None, first_batch: int = 0,
                 energy: torch.Tensor | None = None):
        run = N.IpcNetRun()
        if energy is not None:
            if energy.dtype != torch.float32 or energy.numel() < steps or not energy.is_contiguous() \
                    or energy.device != self.device:
                raise ValueError("energy must be a contiguous float32 tensor with >= steps elements on the model device")
            run.energy = energy.data_ptr()
        run.pool_x = None if pool_x is None else pool_x.data_ptr()
        run.pool_y = None if pool_y is None else pool_y.data_ptr()
        run.pool_batches = 0 if pool_x is None else int(pool_x.shape[0])
        run.first_batch = int(first_batch)
        run.steps, run.T = int(steps), int(T)
        run.forward_init, run.update_weights = int(forward_init), int(update_weights)
        run.recompute = 1
        run.alpha, run.gamma = float(self.cfg.alpha), float(self.cfg.gamma)
        run.act, run.dtype = self.act.code, N.dtype_code(self.cfg.dtype)
        run.cluster = int(self.cfg.net_cluster)
        if self._net_sync is None:  # grid-barrier words of the wide small-batch kernel (zeroed per launch)
            self._net_sync = torch.zeros(N.NET_SYNC_BYTES // 4, device=self.device, dtype=torch.int32)
        run.sync = self._net_sync.data_ptr()
        N.check(N.load().ipc_net_train(self._net(), run, N.stream_handle(self.device)))

    # ----------------------------------------------------------------- steps
    def initialize_batch(self, x_input: torch.Tensor, y_target: torch.Tensor) -> None:
        """Reset endpoints and initialise hidden states by a forward prediction (reference :453-516)."""
        if x_input.ndim != 2 or y_target.ndim != 2:
            raise ValueError("Inputs must be [features, batch]")
        B = int(x_input.shape[1])
        if x_input.shape[0] != self.cfg.dims[-1] or y_target.shape[0] != self.cfg.dims[0]:
            raise ValueError("Batch dimensions do not match network dims")
        if y_target.shape[1] != B:
            raise ValueError("input and target batch sizes differ")
        self._ensure_buffers(B)
        self._prepare_runtime_plan(B)
        self.x[-1].copy_(x_input)
        if self.a is not None:
            self.a[-1].copy_(self.act.forward(self.x[-1]))
        d = self.cfg.dims
        if self._ac is not None:
            N.check(N.load().ipc_activate(N.ptr(self._ac[-1]), N.ptr(self.x[-1]), self.x[-1].numel(), self.act.code,
                                          N.dtype_code(self.cfg.dtype), N.stream_handle(self.device)))
            for l in reversed(range(1, self.L)):
                self._fg(N.MODE_FORWARD, self.w[l], self._ac[l + 1], self.x[l], None, self._ac[l],
                         M=d[l], K=d[l + 1], B=B)
        else:
            for l in reversed(range(1, self.L)):
                self._fwd_singleton_kernels[l](self.x[l + 1], self.w[l], self.x[l])
        self.x[0].copy_(y_target)

    @torch.no_grad()
    def step_initialized(self, *, collect_metrics: bool = False, update_weights: bool = True) -> dict[str, float]:
        """P for all layers, I for the hidden layers, then (by default) W for all layers
        (reference ``trainer.py:601-679``); one launch on the net path."""
        if self.x is None or self.e is None:
            raise RuntimeError("Call initialize_batch before step_initialized")
        B = int(self.x[-1].shape[1])
        if self._runtime_plan_key is None:
            self._prepare_runtime_plan(B)
        if self.net_kernel_eligible(B):
            self._net_run(steps=1, T=1, forward_init=False, update_weights=update_weights)
        else:
            self._phase_p()
            self._phase_i()
            if update_weights:
                self._phase_w()
        if update_weights:
            self.steps_done += 1
        if collect_metrics:
            return self.metrics()
        return {}

    def _phase_p(self):
        if self._ac is not None:
            B, d = int(self.x[0].shape[1]), self.cfg.dims
            for gi, gr in enumerate(self._layer_groups):
                xs, es = self._x_grouped[gi], self._e_grouped[gi]
                self._fg(N.MODE_PRED, self._w_grouped[gi], self._ac_grouped[gi][1:], es[:-1], xs[:-1],
                         M=gr.width, K=gr.width, B=B, groups=gr.count)
            for l, _ in self._pred_singleton_ops:
                self._fg(N.MODE_PRED, self.w[l], self._ac[l + 1], self.e[l], self.x[l], M=d[l], K=d[l + 1], B=B)
            return
        for gi, gr in enumerate(self._layer_groups):
            xs, es = self._x_grouped[gi], self._e_grouped[gi]
            self._pred_group_kernels[gi](xs[1:], self._w_grouped[gi], xs[:-1], es[:-1])
        for l, k in self._pred_singleton_ops:
            k(self.x[l + 1], self.w[l], self.x[l], self.e[l])

    def _phase_i(self):
        if self._ac is not None:
            B, d = int(self.x[0].shape[1]), self.cfg.dims
            g = self.cfg.gamma
            for gi, gr in enumerate(self._layer_groups):
                xs, es, ws = self._x_grouped[gi], self._e_grouped[gi], self._w_grouped[gi]
                self._fg(N.MODE_INFER, ws, es[:-1], xs[1:], es[1:], self._ac_grouped[gi][1:], M=gr.width, K=gr.width,
                         B=B, groups=gr.count, scale=g, flags=N.FLAG_AOUT_STORED)
            for l, _ in self._inf_singleton_ops:
                self._fg(N.MODE_INFER, self.w[l - 1], self.e[l - 1], self.x[l], self.e[l], self._ac[l], M=d[l],
                         K=d[l - 1], B=B, scale=g, flags=N.FLAG_AOUT_STORED)
            return
        for gi, gr in enumerate(self._layer_groups):
            xs, es, ws = self._x_grouped[gi], self._e_grouped[gi], self._w_grouped[gi]
            if self.a is None:
                self._inf_group_kernels[gi](xs[1:], es[1:], ws, es[:-1])
            else:
                self._inf_group_kernels[gi](xs[1:], es[1:], ws, es[:-1], self._a_grouped[gi][1:])
        for l, k in self._inf_singleton_ops:
            if self.a is None:
                k(self.x[l], self.e[l], self.w[l - 1], self.e[l - 1])
            else:
                k(self.x[l], self.e[l], self.w[l - 1], self.e[l - 1], self.a[l])

    def _phase_w(self):
        if self.fused_optimizer:
            self._phase_w_optimizer()
            return
        if self._ac is not None:
            B, d = int(self.x[0].shape[1]), self.cfg.dims
            al = self.cfg.alpha
            for gi, gr in enumerate(self._layer_groups):
                self._fg(N.MODE_WEIGHT, self._e_grouped[gi][:-1], self._ac_grouped[gi][1:], self._w_grouped[gi],
                         M=gr.width, K=gr.width, B=B, groups=gr.count, scale=al)
            for l in range(self.L):
                if l not in self._edge_to_group:
                    self._fg(N.MODE_WEIGHT, self.e[l], self._ac[l + 1], self.w[l], M=d[l], K=d[l + 1], B=B, scale=al)
            return
        for gi, gr in enumerate(self._layer_groups):
            es, ws = self._e_grouped[gi], self._w_grouped[gi]
            src = self._x_grouped[gi][1:] if self.a is None else self._a_grouped[gi][1:]
            op = self._weight_group_outer_ops[gi] if self._weight_group_outer_ops else None
            (op if op is not None else self._weight_group_kernels[gi])(ws, es[:-1], src)
        for l, op in self._weight_singleton_outer_ops:
            op(self.w[l], self.e[l], self.x[l + 1] if self.a is None else self.a[l + 1])
        for l, k in self._weight_singleton_ops:
            k(self.w[l], self.e[l], self.x[l + 1] if self.a is None else self.a[l + 1])

    def _phase_w_optimizer(self):
        """Weight update as an optimizer step per layer (``ipc_weight_update_opt``): the state stays in fp32
        beside W, the step is applied where E f(x)^T meets W."""
        d, B, c = self.cfg.dims, int(self.x[0].shape[1]), self.cfg
        kind = str(c.optimizer).lower()
        if self._opt_state is None:
            adam = kind == "adamw"
            self._opt_state = [(torch.zeros(w.shape, device=self.device, dtype=torch.float32)
                                if (adam or c.momentum != 0.0) else None,
                                torch.zeros(w.shape, device=self.device, dtype=torch.float32) if adam else None)
                               for w in self.w]
        need = max(max(d[l] * d[l + 1] * 4, (d[l + 1] * B * 2 + 255) // 256 * 256 + N.SPLITK_WORKSPACE_BYTES)
                   for l in range(self.L))
        if self._opt_ws is None or self._opt_ws.numel() * 4 < need:
            self._opt_ws = torch.empty((need + 3) // 4, device=self.device, dtype=torch.float32)
        self._opt_steps += 1
        for l in range(self.L):
            if self._ac is not None:
                src, rec = self._ac[l + 1], False
            elif self.a is not None:
                src, rec = self.a[l + 1], False
            else:
                src, rec = self.x[l + 1], True
            m, v = self._opt_state[l]
            kc = self._kernel_config("weight", d[l], d[l + 1], B)
            N.weight_update_opt(self.w[l], self.e[l], src, M=d[l], K=d[l + 1], B=B, kind=kind, lr=c.alpha,
                                momentum=c.momentum, weight_decay=c.weight_decay, betas=c.betas, eps=c.eps,
                                step=self._opt_steps, m=m, v=v, recompute=rec, act=c.activation, dtype=c.dtype,
                                algo=kc.backend, workspace=self._opt_ws, device=self.device)

    def metrics(self) -> dict[str, float]:
        """``max |e[l]|`` over ``l < L`` (reference ``trainer.py:676-678``); synchronises."""
        return {"max_abs_error": float(max(v.float().abs().max().item() for v in self.e[:-1]))}

    @torch.no_grad()
    def step(self, x_input: torch.Tensor, y_target: torch.Tensor) -> dict[str, float]:
        self.initialize_batch(x_input, y_target)
        return self.step_initialized(collect_metrics=True)

    @torch.no_grad()
    def run_inference(self, T: int) -> None:
        """T inference iterations (P + I) without a weight update."""
        for _ in range(int(T)):
            self.step_initialized(update_weights=False)

    @torch.no_grad()
    def train_step(self, x_input: torch.Tensor, y_target: torch.Tensor, *, T: int = 4,
                   collect_metrics: bool = False) -> dict[str, float]:
        """One training step: forward-init sweep, T inference iterations, one weight update
        with the last iteration's errors and states (the oracle schedule
        ``for t in range(T): ipc_step(update_weights=(t == T-1))``)."""
        B = int(x_input.shape[1])
        if T < 1:
            raise ValueError("T must be >= 1")
        if self.net_kernel_eligible(B):
            if x_input.shape[0] != self.cfg.dims[-1] or y_target.shape[0] != self.cfg.dims[0]:
                raise ValueError("Batch dimensions do not match network dims")
            self._ensure_buffers(B)
            self._prepare_runtime_plan(B)
            self.x[-1].copy_(x_input)
            self.x[0].copy_(y_target)
            self._net_run(steps=1, T=T, forward_init=True, update_weights=True)
            self.steps_done += 1
        else:
            self.initialize_batch(x_input, y_target)
            for t in range(T):
                self.step_initialized(update_weights=(t == T - 1))
        return self.metrics() if collect_metrics else {}

    @torch.no_grad()
    def train_pool(self, pool_x: torch.Tensor, pool_y: torch.Tensor, *, steps: int, T: int = 4,
                   first_batch: int = 0, energy: torch.Tensor | None = None) -> None:
        """``steps`` training steps over a device-resident batch pool.

        ``pool_x [P, d_L, B]`` and ``pool_y [P, d_0, B]`` (contiguous, model dtype, on the
        model's device); step ``s`` trains on batch ``(first_batch + s) % P``.  On the net
        path this is a single kernel launch.  ``energy`` (float32, >= steps elements, net
        path only) receives each step's ``sum_l mean(e[l]^2)`` of its last iteration."""
        if pool_x.ndim != 3 or pool_y.ndim != 3:
            raise ValueError("pool_x / pool_y must be [P, features, batch]")
        P, dL, B = pool_x.shape
        if dL != self.cfg.dims[-1] or pool_y.shape[1] != self.cfg.dims[0] or pool_y.shape[0] != P \
                or pool_y.shape[2] != B:
            raise ValueError("pool shapes do not match network dims")
        for t in (pool_x, pool_y):
            if t.device != self.device or t.dtype != self.cfg.dtype or not t.is_contiguous():
                raise ValueError("pool tensors must be contiguous, on the model device, in the model dtype")
        if steps <= 0:
            return
        if self.net_kernel_eligible(B):
            self._ensure_buffers(int(B))
            self._prepare_runtime_plan(int(B))
            self._net_run(steps=steps, T=T, forward_init=True, update_weights=True, pool_x=pool_x, pool_y=pool_y,
                          first_batch=first_batch, energy=energy)
            self.steps_done += int(steps)
        else:
            if energy is not None:
                raise ValueError("per-step energy output needs the persistent-kernel path")
            for s in range(int(steps)):
                b = (first_batch + s) % P
                self.train_step(pool_x[b], pool_y[b], T=T)

    # ---------------------------------------------------------- steady state
    # One batch stays loaded and the reference step (P, I, W) is applied to it over and over -- the
    # reference's latency benchmark (trainer.py:686-826).  Here a block of steps is either a captured
    # graph (IPCGraphRunner) or, on the persistent-kernel path, a single launch.

    def steady_state_graph_ready(self, steps: int) -> bool:
        return (self._steady_state_runner is not None
                and self._steady_state_graph_key == (self._runtime_plan_key, int(steps)))

    def prepare_steady_state(self, x_input: torch.Tensor, y_target: torch.Tensor, *, steps: int = 1,
                             use_graph: bool | None = None) -> bool:
        """Load the batch; if graphs are wanted, make sure a captured block of ``steps`` steps matches the
        current plan.  Returns whether ``run_prepared_steady_state`` will replay a graph."""
        self.initialize_batch(x_input, y_target)
        want = bool(self.cfg.steady_state_graph_default) if use_graph is None else bool(use_graph)
        if want and not self.steady_state_graph_ready(steps):
            self._steady_state_runner = self.capture_graph(max(1, int(steps)))
            self._steady_state_graph_key = (self._runtime_plan_key, max(1, int(steps)))
            self._steady_state_graph_steps = max(1, int(steps))
        return want

    @torch.no_grad()
    def run_prepared_steady_state(self, *, steps: int | None = None, repeats: int = 1,
                                  use_graph: bool | None = None, collect_metrics: bool = False) -> dict[str, float]:
        """``repeats`` blocks of ``steps`` reference steps on the loaded batch, then a device sync.

        With a graph: one replay per block.  Without one, on the persistent-kernel path all
        ``steps * repeats`` steps run in one launch (the same arithmetic as separate launches); on the
        operator path the steps are launched one after another."""
        if self.x is None or self._runtime_plan_key is None:
            raise RuntimeError("Call prepare_steady_state/initialize_batch first")
        block = int(steps) if steps is not None else (self._steady_state_graph_steps or 1)
        block, repeats = max(1, block), max(1, int(repeats))
        graph = self.steady_state_graph_ready(block) if use_graph is None else bool(use_graph)
        if graph:
            if not self.steady_state_graph_ready(block):
                raise RuntimeError("Requested graph replay without a matching captured graph")
            for _ in range(repeats):
                self._steady_state_runner.replay()
        elif self.net_kernel_eligible(int(self.x[-1].shape[1])):
            self._net_run(steps=block * repeats, T=1, forward_init=False, update_weights=True)
            self.steps_done += block * repeats
        else:
            for _ in range(block * repeats):
                self.step_initialized()
        torch.cuda.synchronize(self.device)
        return self.metrics() if collect_metrics else {}

    def reset_steady_state(self) -> None:
        self._invalidate_steady_state_graph()

    @property
    def steady_state_uses_graph(self) -> bool:
        return self._steady_state_runner is not None

    def run_steady_state_batch(self, x_input, y_target, *, steps: int = 1, repeats: int = 1,
                               use_graph: bool | None = None, collect_metrics: bool = False) -> dict[str, float]:
        graph = self.prepare_steady_state(x_input, y_target, steps=steps, use_graph=use_graph)
        return self.run_prepared_steady_state(steps=steps, repeats=repeats, use_graph=graph,
                                              collect_metrics=collect_metrics)

    def precompile(self) -> None:
        """Apply one step to a snapshot of the live tensors and put them back, so every kernel's
        first-launch setup (function attributes, tensor maps, workspaces) happens now and not inside a
        later stream capture (reference ``trainer.py:783-818``)."""
        if self.x is None:
            raise RuntimeError("Call initialize_batch before precompile")
        self._prepare_runtime_plan(int(self.x[-1].shape[1]))
        live = [t for group in (self.w, self.x, self.e, self.a or [], self._ac or []) for t in group if t is not None]
        snapshot = torch.cat([t.reshape(-1).float() for t in live])
        steps = self.steps_done
        self.step_initialized()
        off = 0
        for t in live:
            t.copy_(snapshot[off:off + t.numel()].view(t.shape))
            off += t.numel()
        self.steps_done = steps
        torch.cuda.synchronize(self.device)

    def capture_graph(self, steps: int):
        """A captured block of ``steps`` reference steps on the loaded batch (``IPCGraphRunner``)."""
        from .cuda_graph import IPCGraphRunner
        if self.x is None:
            raise RuntimeError("Call initialize_batch before capture_graph")
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        return IPCGraphRunner(self, steps, pool=self._graph_pool).capture()

    @torch.no_grad()
    def predict(self, x_input: torch.Tensor) -> torch.Tensor:
        """``h = W[l] @ f(h)`` for ``l = L-1..0`` (reference ``trainer.py:828-833``).

        Networks the persistent kernel holds (widths <= 64) predict in one launch: its forward sweep
        gives x[1..L-1], and its first prediction-error pass against a zero target gives
        ``e[0] = -cast(W[0] f(x[1]))`` (negation is exact), on scratch states -- the model's own states
        and weights are not written.  Other networks run one fused forward operator per layer."""
        h = x_input.contiguous()
        B = int(h.shape[1])
        if h.shape[0] != self.cfg.dims[-1]:
            raise ValueError("input features do not match dims[-1]")
        if h.dtype == self.cfg.dtype and self._predict_net_ok(B):
            return self._predict_net(h)
        for l in reversed(range(self.L)):
            out = torch.empty((self.cfg.dims[l], B), device=self.device, dtype=self.cfg.dtype)
            build_forward(self.cfg.dims[l], self.cfg.dims[l + 1], B, self.cfg.activation, self.dtype_name,
                          self._kernel_config("forward", self.cfg.dims[l], self.cfg.dims[l + 1], B))(h, self.w[l], out)
            h = out
        return h

    def _predict_net_ok(self, B: int) -> bool:
        if not (self.cfg.use_net_kernel and self.cfg.dtype in (torch.float16, torch.bfloat16)
                and 1 <= self.L <= N.NET_MAX_LAYERS):
            return False
        plan = N.net_plan(self.cfg.dims, int(B), 1, int(self.cfg.net_cluster))
        return plan is not None and plan[0] > 0  # the small-width cluster kernel

    def _predict_net(self, x_input: torch.Tensor) -> torch.Tensor:
        B = int(x_input.shape[1])
        d, dt = self.cfg.dims, self.cfg.dtype
        bufs = self._predict_bufs.get(B)
        if bufs is None:  # scratch states of the prediction launch, per batch size
            xs = [torch.zeros((dv, B), device=self.device, dtype=dt) for dv in d]
            es = [torch.zeros((dv, B), device=self.device, dtype=dt) for dv in d]
            bufs = self._predict_bufs[B] = (xs, es)
        xs, es = bufs
        xs[0].zero_()
        xs[-1].copy_(x_input)
        desc = N.IpcNet()
        desc.L, desc.B, desc.nets = self.L, B, 1
        for l, dv in enumerate(d):
            desc.dims[l] = int(dv)
            desc.x[l] = xs[l].data_ptr()
        for l in range(self.L):
            desc.w[l] = self.w[l].data_ptr()
            desc.e[l] = es[l].data_ptr()
        run = N.IpcNetRun()
        run.steps, run.T, run.forward_init, run.update_weights, run.recompute = 1, 1, 1, 0, 1
        run.alpha, run.gamma = float(self.cfg.alpha), float(self.cfg.gamma)
        run.act, run.dtype, run.cluster = self.act.code, N.dtype_code(dt), int(self.cfg.net_cluster)
        N.check(N.load().ipc_net_train(desc, run, N.stream_handle(self.device)))
        return -es[0]

    @torch.no_grad()
    def evaluate(self, x_input: torch.Tensor, labels: torch.Tensor, *,
                 counter: torch.Tensor | None = None) -> torch.Tensor:
        """Correct predictions of a batch, counted on the device: ``predict`` (the forward sweep), then per
        column the argmax over the ``d_0`` outputs against ``labels`` (``ipc_count_correct``).  Returns an
        int32 tensor of one element (``counter``, accumulated, if given) without synchronising; the
        reference takes the argmax on the host (``scripts/train_mnist.py:80-81``)."""
        B = int(x_input.shape[1])
        if labels.numel() != B:
            raise ValueError("labels must have one entry per batch column")
        logits = self.predict(x_input)
        cnt = counter if counter is not None else torch.zeros(1, dtype=torch.int32, device=self.device)
        if cnt.dtype != torch.int32 or cnt.device != self.device:
            raise ValueError("counter must be an int32 tensor on the model device")
        lab = labels.to(self.device, torch.int64).contiguous()
        N.check(N.load().ipc_count_correct(logits.data_ptr(), int(self.cfg.dims[0]), B, lab.data_ptr(),
                                           cnt.data_ptr(), N.dtype_code(self.cfg.dtype),
                                           N.stream_handle(self.device)))
        return cnt

    def accuracy(self, x_input: torch.Tensor, labels: torch.Tensor) -> float:
        """Fraction of correct predictions of a batch (synchronises)."""
        return int(self.evaluate(x_input, labels).item()) / max(1, int(x_input.shape[1]))

    # ---------------------------------------------------------- checkpoints
    def state_dict(self) -> dict:
        opt = None
        if self._opt_state is not None:
            opt = {"steps": int(self._opt_steps),
                   "m": [None if m is None else m.clone() for m, _ in self._opt_state],
                   "v": [None if v is None else v.clone() for _, v in self._opt_state]}
        return {"dims": tuple(self.cfg.dims), "w": [w.detach().clone() for w in self.w],
                "steps_done": int(self.steps_done), "optimizer": opt,
                "config": {k: (str(v) if k in ("dtype", "kernel") else v)
                           for k, v in asdict(replace(self.cfg, tuning_table=None)).items() if k != "tuning_table"}}

    def load_state_dict(self, state: dict) -> None:
        if tuple(state["dims"]) != tuple(self.cfg.dims):
            raise ValueError(f"checkpoint dims {state['dims']} != model dims {self.cfg.dims}")
        for dst, src in zip(self.w, state["w"]):
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError("checkpoint weight shape mismatch")
            dst.copy_(src.to(device=self.device, dtype=self.cfg.dtype))
        self.steps_done = int(state.get("steps_done", 0))
        opt = state.get("optimizer")
        if opt is not None:
            self._opt_steps = int(opt["steps"])
            self._opt_state = [(None if m is None else m.to(self.device, torch.float32).contiguous(),
                                None if v is None else v.to(self.device, torch.float32).contiguous())
                               for m, v in zip(opt["m"], opt["v"])]


def prepare_batch(images: torch.Tensor, labels: torch.Tensor, *, device: torch.device, dtype: torch.dtype,
                  num_classes: int) -> tuple[torch.Tensor, torch.Tensor]:
    """A host batch in the trainer's layout (reference ``trainer.py:836-846``): images ``[B, ...]``
    (NCHW for MNIST) become the input ``[features, B]``, labels ``[B]`` the one-hot target ``[C, B]``.

    The images cross PCIe in their own layout and dtype (one contiguous copy); the transpose to
    feature-major and the cast to ``dtype`` run on the device.  ``BatchPipeline``
    (``lich_b200.input_pipeline``) does the same from pinned memory on a copy stream, double-buffered."""
    if images.ndim < 2 or labels.ndim != 1 or labels.shape[0] != images.shape[0]:
        raise ValueError("images must be [B, ...] and labels [B]")
    rows = images.reshape(images.shape[0], -1).to(device, non_blocking=True)
    x = torch.empty((rows.shape[1], rows.shape[0]), device=device, dtype=dtype)
    x.copy_(rows.t())
    y = one_hot(labels.to(device, non_blocking=True), num_classes, dtype=dtype)
    return x, y
