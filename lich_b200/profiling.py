"""Per-operator CUDA-event timing inside running training steps.

``operator_times(step, steps)`` runs ``step()`` ``steps`` times with every call of the fused GEMM
entry point (``_native.fused_gemm``: P, I, W, ΔW and forward launches of the operator path) bracketed
by CUDA events on the current stream, and groups the launches by operator and shape.  The kernels run
back to back as in training, under the same clocks and power cap, so the rows add up to the step and
show which operator falls behind the others (a wave-quantised grid, an epilogue-bound short
reduction).  Event records between launches cost nothing measurable against millisecond kernels.

    python -m lich_b200.profiling --config c5 [--batch 65536] [--steps 5]
    python -m lich_b200.profiling --gemm inference:4096:1000:65536 [--launches 3]
    python -m lich_b200.profiling --net-launches

The first prints one row per (operator, M, K, B, groups) for the wide data-parallel step of
configs[4] (dims (1000, 4096 x 6, 4096), bf16, tanh, T = 4) on one GPU; the second times single
launches of one operator on seeded operands (the case to give ncu); the third splits the hidden-64
persistent kernel's launch time into a fixed part and a per-step part.
"""
from __future__ import annotations

import argparse
import collections
import statistics

import torch

from . import _native as N

KIND = {N.MODE_PRED: "P", N.MODE_INFER: "I", N.MODE_WEIGHT: "W", N.MODE_WDELTA: "WD", N.MODE_FORWARD: "F"}


def operator_times(step, steps: int = 5, warmup: int = 2) -> dict:
    """Run ``warmup`` untimed and ``steps`` timed calls of ``step()``; return the step time and per
    (operator, M, K, B, groups) the launches per step, median launch time, TFLOP/s and ms per step."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    rec = []
    orig = N.fused_gemm

    def timed(mode, *a, **k):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        orig(mode, *a, **k)
        e1.record()
        rec.append(((mode, k.get("M"), k.get("K"), k.get("B"), k.get("groups", 1)), e0, e1))

    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    N.fused_gemm = timed
    try:
        s0.record()
        for _ in range(steps):
            step()
        s1.record()
        torch.cuda.synchronize()
    finally:
        N.fused_gemm = orig
    by = collections.defaultdict(list)
    for key, e0, e1 in rec:
        by[key].append(e0.elapsed_time(e1))
    rows = []
    for (mode, M, K, B, G), ts in by.items():
        med = statistics.median(ts)
        rows.append({"op": KIND.get(mode, str(mode)), "M": M, "K": K, "B": B, "groups": G,
                     "per_step": len(ts) / steps, "median_ms": round(med, 4),
                     "tflops": round(2.0 * M * K * B * G / (med * 1e-3) / 1e12, 1),
                     "ms_per_step": round(sum(ts) / steps, 3)})
    rows.sort(key=lambda r: -r["ms_per_step"])
    return {"step_ms": round(s0.elapsed_time(s1) / steps, 3),
            "gemm_ms": round(sum(r["ms_per_step"] for r in rows), 3), "rows": rows}


def _c5(batch: int):
    from . import synthetic as S
    from .data_parallel import DataParallelIPC
    from .trainer import IPCConfig

    dev = torch.device("cuda", 0)
    dims = (1000,) + (4096,) * 6 + (4096,)
    dt = torch.bfloat16
    dp = DataParallelIPC(IPCConfig(dims=dims, alpha=1e-4, gamma=0.5, activation="tanh", dtype=dt), device=dev)
    w0 = [w.to(dev, dt) for w in S.fan_in_normal(dims, seed=1)]
    g = torch.Generator(device=dev).manual_seed(100)
    x = torch.rand((dims[-1], batch), generator=g, device=dev).to(dt)
    y = torch.zeros((dims[0], batch), device=dev, dtype=dt)
    y.scatter_(0, torch.randint(0, dims[0], (1, batch), generator=g, device=dev), 1.0)

    def step():
        for w, s in zip(dp.model.w, w0):
            w.copy_(s)
        dp.train_step(x, y, T=4)
    return step


def gemm_launches(kind: str, M: int, K: int, B: int, *, launches: int = 3, dtype=torch.bfloat16,
                  act: str = "tanh") -> list[float]:
    """Run one operator of the trainer's operator path (stored activations) ``launches`` times on seeded
    operands and return each launch's milliseconds: a single-kernel case for ncu captures."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + K + B)

    def r(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)
    mode = {"prediction": N.MODE_PRED, "inference": N.MODE_INFER, "weight": N.MODE_WEIGHT,
            "wdelta": N.MODE_WDELTA, "forward": N.MODE_FORWARD}[kind]
    if mode == N.MODE_PRED:
        ops = (r(M, K, scale=K ** -0.5), r(K, B), r(M, B, scale=0.0), r(M, B), None)  # a, b, out, aux, aux2
    elif mode == N.MODE_FORWARD:
        ops = (r(M, K, scale=K ** -0.5), r(K, B), r(M, B, scale=0.0), None, r(M, B, scale=0.0))
    elif mode == N.MODE_INFER:
        ops = (r(K, M, scale=M ** -0.5), r(K, B, scale=0.5), r(M, B), r(M, B, scale=0.5), r(M, B, scale=0.0))
    elif mode == N.MODE_WEIGHT:
        ops = (r(M, B, scale=0.5), r(K, B), r(M, K, scale=0.05), None, None)
    else:
        ops = (r(M, B, scale=0.5), r(K, B), torch.zeros(M, K, device=dev), None, None)
    a, b, out, aux, aux2 = ops
    scale = 0.5 if mode == N.MODE_INFER else 1e-4
    flags = N.FLAG_AOUT_STORED if mode == N.MODE_INFER else 0
    times = []
    for _ in range(launches):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        N.fused_gemm(mode, a, b, out, aux, aux2, M=M, K=K, B=B, scale=scale, flags=flags, act=act, dtype=dtype,
                     device=dev)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    if N.device_status() != 0:
        raise RuntimeError("device-side wait timed out")
    return times


def net_launch_costs(depth: int = 6, sizes=(1, 2, 4, 8, 20, 50, 100, 500), reps: int = 7) -> dict:
    """The persistent kernel's cost per launch: median CUDA-event time of ``train_pool`` launches of
    ``sizes`` steps (configs[1]: dims (10, 64 x depth, 784), B = 128, fp16, tanh, T = 4), each queued
    behind a 200-step launch so the GPU is busy when it starts, the least-squares fit
    fixed + per-step, and a 20-step launch that starts on an idle GPU (after a synchronize)."""
    from . import synthetic as S
    from .trainer import IPCConfig, TileLangIPC

    dev = torch.device("cuda", 0)
    dims = S.paper_dims(depth)
    B, T, dt = 128, 4, torch.float16
    m = TileLangIPC(IPCConfig(dims=dims, alpha=1e-4, gamma=0.5, activation="tanh", dtype=dt), device=dev)
    w0 = [w.to(dev, dt) for w in S.fan_in_normal(dims, seed=1)]
    g = torch.Generator(device=dev).manual_seed(5)
    P = 256
    px = torch.rand((P, dims[-1], B), generator=g, device=dev).to(dt)
    lab = torch.randint(0, dims[0], (P, B), generator=g, device=dev)
    py = torch.zeros((P, dims[0], B), device=dev, dtype=dt)
    py.scatter_(1, lab.unsqueeze(1), 1.0)

    def restore():
        for d, s0 in zip(m.w, w0):
            d.copy_(s0)

    def timed(steps, idle, rep):
        restore()
        m.train_pool(px, py, steps=200, T=T)
        if idle:
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        m.train_pool(px, py, steps=steps, T=T, first_batch=rep)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3

    for _ in range(3):
        timed(500, False, 0)
    busy = {n: statistics.median(timed(n, False, r) for r in range(reps)) for n in sizes}
    xs, ys = list(busy), list(busy.values())
    mx, my = sum(xs) / len(xs), sum(ys) / len(ys)
    per = sum((a - mx) * (b - my) for a, b in zip(xs, ys)) / sum((a - mx) ** 2 for a in xs)
    idle20 = statistics.median(timed(20, True, r) for r in range(reps))
    return {"busy_us": {n: round(v, 1) for n, v in busy.items()}, "fixed_us": round(my - per * mx, 1),
            "per_step_us": round(per, 2), "idle_20_step_launch_us": round(idle20, 1),
            "busy_20_step_launch_us": busy.get(20)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--config", choices=["c5"], default="c5")
    ap.add_argument("--batch", type=int, default=65536)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--gemm", default="", help="kind:M:K:B -- time one operator's launches instead of a step")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--net-launches", action="store_true",
                    help="configs[1]: cost per persistent-kernel launch (fixed + per step, idle vs busy GPU)")
    args = ap.parse_args(argv)
    if args.net_launches:
        res = net_launch_costs()
        for n, v in res["busy_us"].items():
            print(f"{n:4d} steps per launch: {v:9.1f} us ({v / n:6.2f} us/step)")
        print(f"fit: {res['fixed_us']} us per launch + {res['per_step_us']} us per step; 20-step launch "
              f"on an idle GPU {res['idle_20_step_launch_us']} us, behind a busy one {res['busy_20_step_launch_us']} us")
        return
    if args.gemm:
        kind, M, K, B = args.gemm.split(":")
        M, K, B = int(M), int(K), int(B)
        ts = gemm_launches(kind, M, K, B, launches=args.launches)
        for t in ts:
            print(f"{kind} {M} x {K} x {B}: {t:.4f} ms, {2.0 * M * K * B / (t * 1e-3) / 1e12:.1f} TF/s")
        return
    res = operator_times(_c5(args.batch), steps=args.steps, warmup=args.warmup)
    print(f"{'op':3s} {'M':>5s} {'K':>5s} {'B':>6s} {'G':>2s} {'/step':>5s} {'median ms':>9s} {'TF/s':>7s} {'ms/step':>8s}")
    for r in res["rows"]:
        print(f"{r['op']:3s} {r['M']:5d} {r['K']:5d} {r['B']:6d} {r['groups']:2d} {r['per_step']:5.0f} "
              f"{r['median_ms']:9.3f} {r['tflops']:7.1f} {r['ms_per_step']:8.2f}")
    print(f"step {res['step_ms']:.2f} ms, of which fused GEMM launches {res['gemm_ms']:.2f} ms")


if __name__ == "__main__":
    main()
