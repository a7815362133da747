"""The allocation-free SISO backward, m3_siso_scan_bwd_noalloc, called through the C ABI.

Some callers may not allocate device memory when they run the backward (for example a
host framework that owns a fixed device-memory budget and forbids side allocations by
extensions). For them the library keeps the backward's workspace in a fixed device array
of its own. This file checks, on the GPU, that two calls in a row give the same gradients
as m3_siso_scan_bwd with a caller-provided workspace (the same tolerances as the other
parity tests: rel 1e-4 for fp32, 2e-2 for bf16), and that a request larger than the fixed
array is refused with an error instead of running.
"""

import ctypes

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed, Bn, L, H, P, D, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(Bn, L, H, P, generator=g).to(dtype)
    Bm = torch.randn(Bn, L, H, D, generator=g).to(dtype)
    C = torch.randn(Bn, L, H, D, generator=g).to(dtype)
    dt = torch.nn.functional.softplus(torch.randn(Bn, L, H, generator=g) * 0.5 - 3).clamp(1e-3, 0.1)
    ADT = -torch.rand(H, generator=g) * 8 * dt
    trap = torch.randn(Bn, L, H, generator=g)
    Dw = torch.randn(H, generator=g)
    dy = torch.randn(Bn, L, H, P, generator=g).to(dtype)
    return [t.to(DEV) for t in (x, Bm, C, ADT, dt, trap, Dw, dy)]


def _grads_like(x, Bm, C, ADT, H):
    return [torch.empty_like(x), torch.empty_like(Bm), torch.empty_like(C), torch.empty_like(ADT),
            torch.empty_like(ADT), torch.empty_like(ADT), torch.empty(H, device=DEV)]


def _call(fn_name, ins, outs, workspace=None):
    from mamba3_ssm import _lib as L
    lib = L.load()
    x, Bm, C, ADT, DT, trap, Dw, dy = ins
    views = [L.tensor(t) for t in (x, Bm, C, ADT, DT, trap, Dw, None, None, dy, *outs, None, None)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    refs = [ctypes.byref(v) for v in views]
    if workspace is None:
        rc = getattr(lib, fn_name)(*refs, stream)
    else:
        rc = getattr(lib, fn_name)(*refs, ctypes.c_void_p(workspace.data_ptr()), workspace.numel(), stream)
    return rc, lib.m3_last_error_string().decode()


@pytest.mark.parametrize("shape,dtype,tol", [((2, 150, 3, 32, 64), torch.float32, 1e-4),
                                             ((2, 300, 4, 64, 128), torch.bfloat16, 2e-2)])
def test_noalloc_backward_matches_workspace_backward_twice(shape, dtype, tol):
    from mamba3_ssm import _lib as L
    Bn, Ln, H, P, D = shape
    ins = _inputs(3, Bn, Ln, H, P, D, dtype)
    x, Bm, C, ADT = ins[:4]
    ref = _grads_like(x, Bm, C, ADT, H)
    nbytes = L.load().m3_siso_scan_bwd_workspace_size(Bn, Ln, H, P, D)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc, msg = _call("m3_siso_scan_bwd", ins, ref, ws)
    assert rc == 0, msg
    for call in range(2):
        got = _grads_like(x, Bm, C, ADT, H)
        rc, msg = _call("m3_siso_scan_bwd_noalloc", ins, got)
        assert rc == 0, msg
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert rel_err(a.float().cpu().numpy(), b.float().cpu().numpy()) < tol, call


def test_noalloc_backward_refuses_oversize_requests():
    limit = 2 * 1024 * 1024
    Bn, Ln, H, P, D = 1, limit // 4 + 1, 4, 16, 16
    x = torch.empty(Bn, Ln, H, P, device=DEV)
    Bm = torch.empty(Bn, Ln, H, D, device=DEV)
    s = torch.empty(Bn, Ln, H, device=DEV)
    ins = [x, Bm, Bm, s, s, s, torch.empty(H, device=DEV), x]
    rc, msg = _call("m3_siso_scan_bwd_noalloc", ins, _grads_like(x, Bm, Bm, s, H))
    assert rc == 4  # M3_ERR_WORKSPACE
    assert "exceeds the fixed scratch" in msg
