"""Batch-sharded data-parallel iPC training (one process per GPU, torch.distributed / NCCL).

Prediction errors and state updates are column-local, so each rank runs the
forward sweep and the T inference iterations on its own slice of the batch
with no communication.  The only coupling is the weight update, a sum over
all batch columns:

    W[l] += alpha * sum_ranks E_r[l] f(x_r[l+1])^T

Each rank forms its fp32 partial ``dW_r[l]`` (``ipc_weight_delta`` /
``IPC_MODE_WDELTA``, tensor cores for wide layers), the partials are summed
with one reduction per layer (issued as soon as that layer's partial is
ready, so the reductions of earlier layers overlap the GEMMs of later ones),
and every rank applies the same sum (``ipc_weight_apply``), keeping the
replicas identical.  While reductions are in flight the persistent GEMMs
leave ``comm_sms`` SMs free (``ipc_set_max_ctas``): with every SM taken by a
GEMM CTA, the collective's kernels would wait for the GEMM and the overlap
would be lost.  Each layer's sum is applied as soon as its own reduction is
done: layer l's apply is queued behind the next layer's delta GEMM, which its
reduction runs beside, so only the last layer's reduction and apply follow the
last GEMM.

``reduce="rs_ag"`` (the default when a layer's size divides by the world)
splits the all-reduce into its halves around the apply: a reduce-scatter of
the fp32 deltas gives each rank the summed delta of 1/world of the weights,
the rank applies it to that slice only, and an all-gather of the updated
16-bit slices rebuilds the replicas.  NVLink carries 4 + 2 bytes per weight
element instead of 4 + 4, the apply touches 1/world of W, and every element
of W is computed once, so the replicas stay identical by construction.  The reference is single-GPU; this is the scaling path of
the wide configuration (batch 65536 over 1/2/4/8 B200s).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _native as N
from .trainer import IPCConfig, TileLangIPC


def allreduce_deltas(deltas: list[torch.Tensor], group=None, *, async_op: bool = True):
    """Sum-all-reduce each tensor of ``deltas`` in place (one collective per tensor, in list order).

    Returns the work handles (empty if ``async_op`` is False or there is one rank)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return []
    handles = []
    for d in deltas:
        h = dist.all_reduce(d, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
        if async_op:
            handles.append(h)
    return handles


class DataParallelIPC:
    """Replicated weights, batch shards, one fp32 dW reduction per layer per training step."""

    def __init__(self, cfg: IPCConfig, *, device: torch.device, group=None, seed: int = 0,
                 model: TileLangIPC | None = None, comm_sms: int = 24, comm_sms_min: int | None = None,
                 reduce: str = "rs_ag", keep_delta: bool = False):
        """comm_sms: SMs the delta GEMMs leave to the reductions they overlap (world > 1).
        comm_sms_min: a delta GEMM may leave as few as this many SMs (default min(16, comm_sms)) when the
        extra CTAs save it a wave of output tiles (e.g. 4096 x 4096 = 256 tiles of 256 x 256: 5 waves on
        62 CTA pairs, 4 on 64; measured at 2 GPUs on configs[4]: 1.8 % faster steps than a fixed 24).
        reduce: "rs_ag" (reduce-scatter, sliced apply, all-gather), "allreduce", or "nvls": the delta
        GEMMs add their fp32 dW straight into a multicast buffer on every GPU through the NVSwitch
        (IPC_FLAG_MULTIMEM_RED), a one-word collective orders the ranks, and every rank applies the
        whole sum -- no NCCL traffic and no SMs held back; it falls back to "rs_ag" on every rank when
        any rank has no multicast support or a layer is not a tensor-core weight delta.
        keep_delta: "nvls" only -- also copy each step's summed fp32 dW into ``_dw`` (one extra pass
        over it; the other forms leave their part of the sum there anyway)."""
        if comm_sms < 0:
            raise ValueError("comm_sms must be >= 0")
        comm_sms_min = min(16, comm_sms) if comm_sms_min is None else int(comm_sms_min)
        if not 0 <= comm_sms_min <= comm_sms:
            raise ValueError("comm_sms_min must be in [0, comm_sms]")
        if reduce not in ("rs_ag", "allreduce", "nvls"):
            raise ValueError(f"unknown reduce {reduce!r}")
        self.group = group
        self.comm_sms = int(comm_sms)
        self.comm_sms_min = comm_sms_min
        self.reduce = reduce
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.model = model if model is not None else TileLangIPC(cfg, device=device, seed=seed)
        self.cfg = self.model.cfg
        if self.world > 1:
            for w in self.model.w:  # identical replicas to start from
                dist.broadcast(w, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        self._dw = self._alloc_deltas()
        self.keep_delta = bool(keep_delta)
        self._mc = None          # "nvls": two (symmetric tensor, handle) pairs, alternated per step
        self._mc_step = 0
        self._mc_ok: dict = {}   # local batch -> every rank can take the multicast path
        if self.reduce == "nvls" and self.world > 1 and not self._setup_multicast():
            self.reduce = "rs_ag"

    def _agree(self, ok: bool) -> bool:
        """True on every rank iff ``ok`` on every rank (a MIN all-reduce of one word)."""
        dev = self.model.w[0].device
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        return bool(flag.item())

    def _setup_multicast(self) -> bool:
        """Two fp32 dW buffers in symmetric memory, each with an NVLS multicast mapping, zeroed on every
        GPU; False (on every rank) when any rank cannot have them."""
        bufs = []
        try:
            import torch.distributed._symmetric_memory as symm_mem
            n = sum(t.numel() for t in self._dw)
            grp = self.group if self.group is not None else dist.group.WORLD
            for _ in range(2):
                t = symm_mem.empty(n, dtype=torch.float32, device=self.model.w[0].device)
                h = symm_mem.rendezvous(t, grp)
                bufs.append((t, h))
            ok = all(int(h.multicast_ptr) != 0 for _, h in bufs)
        except Exception:  # no symmetric memory / multicast on this device or backend
            ok = False
        if not self._agree(ok):
            return False
        for t, _ in bufs:
            t.zero_()
        torch.cuda.synchronize(self.model.w[0].device)
        dist.barrier(group=self.group)
        self._mc = bufs
        self._offsets = []
        off = 0
        for t in self._dw:
            self._offsets.append(off)
            off += t.numel()
        self._sync_word = torch.zeros(1, dtype=torch.float32, device=self.model.w[0].device)
        return True

    def _multicast_ok(self, B: int) -> bool:
        """Whether every layer's delta is a tensor-core weight delta on every rank at local batch B."""
        if B not in self._mc_ok:
            m, d = self.model, self.cfg.dims
            ok = m._ac is not None and self.cfg.dtype in (torch.float16, torch.bfloat16) and all(
                N.tc_eligible(N.MODE_WDELTA, d[l], d[l + 1], B, self.cfg.dtype) for l in range(len(d) - 1))
            self._mc_ok[B] = self._agree(ok)
        return self._mc_ok[B]

    def _deltas_multicast(self, order, B: int) -> torch.Tensor:
        """Every layer's dW added into this step's multicast buffer on every GPU; returns the local copy."""
        m, d = self.model, self.cfg.dims
        t, h = self._mc[self._mc_step & 1]
        base = int(h.multicast_ptr)
        for l in order:
            kc = m._kernel_config("weight", d[l], d[l + 1], B)
            N.fused_gemm(N.MODE_WDELTA, m.e[l], m._ac[l + 1], base + 4 * self._offsets[l], M=d[l], K=d[l + 1],
                         B=B, scale=self.cfg.alpha, flags=N.FLAG_MULTIMEM_RED, act=self.cfg.activation,
                         dtype=self.cfg.dtype, device=m.device, tune=kc.tune())
        return t

    def _alloc_deltas(self) -> list[torch.Tensor]:
        d = self.cfg.dims
        flat = torch.zeros(sum(d[l] * d[l + 1] for l in range(len(d) - 1)), dtype=torch.float32,
                           device=self.model.w[0].device)
        out, off = [], 0
        for l in range(len(d) - 1):
            n = d[l] * d[l + 1]
            out.append(flat[off:off + n].view(d[l], d[l + 1]))
            off += n
        return out

    # -- the two kernel calls of the update (overridable for host-side tests) --
    def _delta(self, l: int, dw: torch.Tensor) -> None:
        """dw = alpha * E[l] f(x[l+1])^T over this rank's columns, fp32."""
        m = self.model
        d = self.cfg.dims
        B = int(m.x[0].shape[1])
        if m._ac is not None:  # cached activation: a stored operand (tensor-core kernel when wide)
            kc = m._kernel_config("weight", d[l], d[l + 1], B)
            N.fused_gemm(N.MODE_WDELTA, m.e[l], m._ac[l + 1], dw, M=d[l], K=d[l + 1], B=B, scale=self.cfg.alpha,
                         act=self.cfg.activation, dtype=self.cfg.dtype, algo=kc.backend, device=m.device,
                         workspace=m._splitk_ws, tune=kc.tune())
        else:
            N.fused_gemm(N.MODE_WDELTA, m.e[l], m.x[l + 1], dw, M=d[l], K=d[l + 1], B=B, scale=self.cfg.alpha,
                         flags=N.FLAG_ACTIVATE_B, act=self.cfg.activation, dtype=self.cfg.dtype, device=m.device)

    def _sms(self) -> int:
        return torch.cuda.get_device_properties(self.model.w[0].device).multi_processor_count

    def _leave_for(self, l: int) -> int:
        """SMs the delta GEMM of layer l leaves to the reductions in flight: comm_sms, or fewer (down to
        comm_sms_min) where the CTAs gained finish the layer's 256 x 256 output tiles in fewer waves (the
        persistent GEMM takes ceil(tiles / CTA pairs) tile times); the most SMs among the fewest waves."""
        if self.comm_sms_min >= self.comm_sms:
            return self.comm_sms
        d = self.cfg.dims
        tiles = -(-d[l] // 256) * -(-d[l + 1] // 256)
        sms = self._sms()
        best = None
        for leave in range(self.comm_sms, self.comm_sms_min - 1, -1):
            waves = -(-tiles // max(1, (sms - leave) // 2))
            if best is None or waves < best[0]:
                best = (waves, leave)
        return best[1]

    def _cap(self, leave: int) -> None:
        """Leave `leave` SMs free of persistent GEMM CTAs (0 lifts the cap)."""
        if leave <= 0:
            N.set_max_ctas(0)
            return
        N.set_max_ctas(max(1, self._sms() - leave))

    def _apply(self, l: int, dw: torch.Tensor) -> None:
        w = self.model.w[l]
        N.check(N.load().ipc_weight_apply(w.data_ptr(), dw.data_ptr(), w.numel(), N.dtype_code(w.dtype),
                                          N.stream_handle(w.device)))

    def _apply_slice(self, l: int, lo: int, hi: int) -> None:
        """W[l].flat[lo:hi] = cast(W[l].flat[lo:hi] + dW[l].flat[lo:hi])."""
        w, dw = self.model.w[l].view(-1), self._dw[l].view(-1)
        N.check(N.load().ipc_weight_apply(w[lo:hi].data_ptr(), dw[lo:hi].data_ptr(), hi - lo,
                                          N.dtype_code(w.dtype), N.stream_handle(w.device)))

    # -- the two collectives of the sliced update (overridable for backends without them) --
    def _reduce_scatter(self, l: int, lo: int, hi: int):
        """dW[l].flat[lo:hi] = sum over ranks of dW[l].flat[lo:hi] (this rank's slice), async."""
        flat = self._dw[l].view(-1)
        return dist.reduce_scatter_tensor(flat[lo:hi], flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)

    def _all_gather(self, l: int, lo: int, hi: int):
        """Every rank's updated slice of W[l] into every replica, async."""
        flat = self.model.w[l].view(-1)
        return dist.all_gather_into_tensor(flat, flat[lo:hi], group=self.group, async_op=True)

    def _sliced(self, l: int) -> bool:
        return self.world > 1 and self.reduce == "rs_ag" and self._dw[l].numel() % self.world == 0

    @torch.no_grad()
    def train_step(self, x_local: torch.Tensor, y_local: torch.Tensor, *, T: int = 4,
                   phases: list | None = None) -> None:
        """Forward sweep + T inference iterations on the local shard, then the all-reduced weight update
        with the last iteration's errors and states (the oracle schedule, full batch = all shards).

        ``phases``: if a list is given, CUDA events (on the current stream) are appended as
        ``(name, event)`` at the start, after the inference iterations, after the last delta GEMM was
        issued and at the end; ``phase_times`` turns them into milliseconds."""
        if T < 1:
            raise ValueError("T must be >= 1")
        m = self.model

        def mark(name):
            if phases is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                phases.append((name, ev))

        mark("start")
        m.initialize_batch(x_local, y_local)
        for _ in range(T):
            m.step_initialized(update_weights=False)
        mark("inference")
        L = len(self.cfg.dims) - 1
        order = sorted(range(L), key=lambda l: -self._dw[l].numel())  # biggest reductions start first
        B = int(m.x[0].shape[1])
        if self._mc is not None and self._multicast_ok(B):
            t = self._deltas_multicast(order, B)
            mark("deltas")
            # every rank's adds are in every copy: one stream-ordered word all-reduce (its kernels start
            # after this rank's delta kernels, whose adds were fenced at system scope)
            dist.all_reduce(self._sync_word, group=self.group)
            for l in order:
                off = self._offsets[l]
                self._apply(l, t[off:off + self._dw[l].numel()].view_as(self._dw[l]))
            if self.keep_delta:
                for l in order:
                    off = self._offsets[l]
                    self._dw[l].view(-1).copy_(t[off:off + self._dw[l].numel()])
            t.zero_()  # reused two steps on, after every rank has passed the next step's word all-reduce
            self._mc_step += 1
            mark("end")
            m.steps_done += 1
            return
        handles, gathers, pending = {}, [], []

        def finish(l):
            # the stream waits for layer l's reduction, applies it and (sliced) starts its all-gather
            if l in handles:
                handles.pop(l).wait()
            if self._sliced(l):
                n = self._dw[l].numel() // self.world
                lo, hi = self.rank * n, (self.rank + 1) * n
                self._apply_slice(l, lo, hi)
                gathers.append(self._all_gather(l, lo, hi))
            else:
                self._apply(l, self._dw[l])

        capped = False
        try:
            for l in order:
                if capped:
                    self._cap(self._leave_for(l))
                self._delta(l, self._dw[l])
                if self._sliced(l):
                    n = self._dw[l].numel() // self.world
                    handles[l] = self._reduce_scatter(l, self.rank * n, (self.rank + 1) * n)
                else:
                    hs = allreduce_deltas([self._dw[l]], self.group, async_op=True)
                    if hs:
                        handles[l] = hs[0]
                # the previous layer's reduction ran beside this layer's GEMM: apply it now, so its
                # all-gather overlaps the next GEMM instead of queueing behind the last one
                if pending:
                    finish(pending.pop(0))
                pending.append(l)
                if l in handles and not capped and self.comm_sms > 0:
                    capped = True
        finally:
            if capped:
                self._cap(0)
        mark("deltas")
        for l in pending:
            finish(l)
        for h in gathers:
            h.wait()
        mark("end")
        m.steps_done += 1

    @staticmethod
    def phase_times(phases: list) -> dict:
        """Milliseconds between consecutive marks of ``train_step(phases=...)`` (synchronises)."""
        torch.cuda.synchronize()
        return {f"{a[0]}->{b[0]}": a[1].elapsed_time(b[1]) for a, b in zip(phases, phases[1:])}

    def state_dict(self) -> dict:
        return self.model.state_dict()
