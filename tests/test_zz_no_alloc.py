"""GPU test of ``ipc_weight_update_noalloc`` (split-K weight update, static scratch).

Called through the C ABI (ctypes on the built library).  Two calls in a row
must each match the existing entry point ``ipc_fused_gemm`` on the same
operands: fp32 deltas within 1e-3 and 16-bit weights within 1e-2 of
``max|ref|`` (the tolerances of the tcgen05 parity tests).  After the first
call, calls change the device's free memory by nothing.  Requests beyond the
scratch limit, and modes other than the weight update, return IPC_ERR_ARG.
The file is named to be collected last; it also passes alone.
"""
import gc

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
CASES = [(1, 64, 64, 65536), (1, 256, 256, 16384), (1, 1024, 1024, 8192), (3, 128, 192, 8192)]


def _N():
    from lich_b200 import _native as N
    return N


def _rand(shape, seed, scale, dt):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(dt)


def _rel(got, ref):
    return ((got.double() - ref.double()).abs().max() / ref.double().abs().max()).item()


def _noalloc(mode, e, a, out, G, M, K, B, alpha, dt, flags=0):
    N = _N()
    return N.load().ipc_weight_update_noalloc(mode, N.ptr(e), N.ptr(a), N.ptr(out), M, K, B, G, alpha, flags,
                                              N.act_code("identity"), N.dtype_code(dt), N.ALGO_CODES["auto"],
                                              N.stream_handle(DEV))


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
def test_noalloc_matches_existing_entry_point_twice(case, dt):
    N = _N()
    G, M, K, B = case
    lead = (G,) if G > 1 else ()
    e = _rand(lead + (M, B), 1, 0.5, dt)
    a = _rand(lead + (K, B), 2, 1.0, dt)
    w0 = _rand(lead + (M, K), 3, 0.05, dt)
    alpha = 1e-3
    for mode, tol in ((N.MODE_WDELTA, 1e-3), (N.MODE_WEIGHT, 1e-2)):
        fresh = (lambda: torch.zeros(lead + (M, K), dtype=torch.float32, device=DEV)) if mode == N.MODE_WDELTA \
            else (lambda: w0.clone())
        ref = fresh()
        N.fused_gemm(mode, e, a, ref, M=M, K=K, B=B, groups=G, scale=alpha, dtype=dt, device=DEV)
        outs = []
        for call in range(2):
            out = fresh()
            # garbage of earlier tests collected inside the measured window would free memory there
            gc.collect()
            gc.disable()
            try:
                torch.cuda.synchronize()
                free0 = torch.cuda.mem_get_info(DEV)[0]
                alloc0 = torch.cuda.memory_allocated(DEV)
                n0 = N.launch_count()
                rc = _noalloc(mode, e, a, out, G, M, K, B, alpha, dt)
                assert rc == N.IPC_OK, N.load().ipc_last_error().decode()
                torch.cuda.synchronize()
                assert N.launch_count() - n0 == 2  # the split GEMM and its reduce pass, nothing else
                assert torch.cuda.memory_allocated(DEV) == alloc0  # nothing through torch's allocator
                if call == 1:  # the first call may load the scratch; later calls allocate nothing
                    assert torch.cuda.mem_get_info(DEV)[0] == free0
            finally:
                gc.enable()
            outs.append(out)
        assert N.device_status() == 0
        for out in outs:
            assert _rel(out, ref) <= tol
        assert torch.equal(outs[0], outs[1])


def test_noalloc_accumulate_flag():
    N = _N()
    M, K, B, dt = 128, 64, 16384, torch.bfloat16
    e = _rand((M, B), 4, 0.5, dt)
    a = _rand((K, B), 5, 1.0, dt)
    base = _rand((M, K), 6, 0.01, torch.float32)
    ref = base.clone()
    N.fused_gemm(N.MODE_WDELTA, e, a, ref, M=M, K=K, B=B, scale=1e-3, flags=N.FLAG_ACCUMULATE, dtype=dt, device=DEV)
    for _ in range(2):
        out = base.clone()
        assert _noalloc(N.MODE_WDELTA, e, a, out, 1, M, K, B, 1e-3, dt, flags=N.FLAG_ACCUMULATE) == N.IPC_OK
        torch.cuda.synchronize()
        assert _rel(out, ref) <= 1e-3


def test_noalloc_rejects_sizes_beyond_the_scratch_limit_and_other_modes():
    N = _N()
    dt = torch.float16
    e = torch.zeros(1, dtype=dt, device=DEV)
    lib = N.load()
    # groups*M*K above IPC_NOALLOC_MAX_OUT_ELEMS (2**20): refused before any launch
    rc = _noalloc(N.MODE_WDELTA, e, e, e, 1, 1024, 1032, 64, 1.0, dt)
    assert rc == N.IPC_ERR_ARG
    assert b"IPC_NOALLOC_MAX_OUT_ELEMS" in lib.ipc_last_error()
    rc = _noalloc(N.MODE_WEIGHT, e, e, e, 2, 1024, 520, 64, 1.0, dt)
    assert rc == N.IPC_ERR_ARG
    rc = _noalloc(N.MODE_PRED, e, e, e, 1, 64, 64, 64, 1.0, dt)
    assert rc == N.IPC_ERR_ARG
