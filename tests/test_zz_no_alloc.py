"""The allocation-free SISO backward, m3_siso_scan_bwd_noalloc, called through the C ABI.

Some callers may not allocate device memory when they run the backward (for example a
host framework that owns a fixed device-memory budget and forbids side allocations by
extensions). For them the library keeps the backward's workspace in a fixed device array
of its own (8 MiB). This file checks, on the GPU:

* two calls in a row give the gradients of m3_siso_scan_bwd with a caller-provided
  workspace and of the float64 oracle (rel 1e-4 for fp32, 2e-2 for bf16, every gradient),
  with a call on other inputs and another shape in between, so stale scratch from an
  earlier call cannot pass for a correct result;
* a bf16 shape whose tensor-core workspace does not fit the fixed array (it then runs the
  CUDA-core backward) against m3_siso_scan_bwd with a full workspace (tensor-core path);
* a request larger than the fixed array is refused with an error instead of running.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
KEYS = ("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD")


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


def _workspace_grads(ins, shape):
    from mamba3_ssm import _lib as L
    Bn, Ln, H, P, D = shape
    ref = _grads_like(*ins[:4], H)
    nbytes = L.load().m3_siso_scan_bwd_workspace_size(Bn, Ln, H, P, D)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc, msg = _call("m3_siso_scan_bwd", ins, ref, ws)
    assert rc == 0, msg
    torch.cuda.synchronize()
    return ref


def _npy(t):
    return t.detach().double().cpu().numpy()


@pytest.mark.parametrize("shape,dtype,tol", [((2, 150, 3, 32, 64), torch.float32, 1e-4),
                                             ((2, 300, 4, 64, 128), torch.bfloat16, 2e-2)])
def test_noalloc_backward_matches_workspace_backward_twice(shape, dtype, tol):
    Bn, Ln, H, P, D = shape
    ins = _inputs(3, Bn, Ln, H, P, D, dtype)
    ref = _workspace_grads(ins, shape)
    oracle = O.siso_scan_bwd(*[_npy(t) for t in ins[:7]], _npy(ins[7]))
    # other inputs and another shape (a longer sequence) between the two checked calls
    other_shape = (1, 700, 3, P, D)
    other = _inputs(4, *other_shape, dtype)
    for call in range(2):
        got = _grads_like(*ins[:4], H)
        rc, msg = _call("m3_siso_scan_bwd_noalloc", ins, got)
        assert rc == 0, msg
        torch.cuda.synchronize()
        for k, a, b in zip(KEYS, got, ref):
            assert rel_err(_npy(a), _npy(b)) < tol, (call, k)
            assert rel_err(_npy(a), oracle[k]) < tol, (call, k, "oracle")
        if call == 0:
            junk = _grads_like(*other[:4], other_shape[2])
            rc, msg = _call("m3_siso_scan_bwd_noalloc", other, junk)
            assert rc == 0, msg


def test_noalloc_backward_above_tensor_core_threshold():
    """bf16, headdim 64, d_state 128 at 1 x 2048 x 32 = 65536 positions: the tensor-core
    workspace (about 140 bytes per position) no longer fits the 8 MiB array, so the
    allocation-free call runs the CUDA-core backward; it must agree with the tensor-core
    backward that m3_siso_scan_bwd runs with a full caller workspace, within the bf16 bar."""
    shape = (1, 2048, 32, 64, 128)
    ins = _inputs(5, *shape, torch.bfloat16)
    ref = _workspace_grads(ins, shape)
    got = _grads_like(*ins[:4], shape[2])
    rc, msg = _call("m3_siso_scan_bwd_noalloc", ins, got)
    assert rc == 0, msg
    torch.cuda.synchronize()
    for k, a, b in zip(KEYS, got, ref):
        assert np.isfinite(_npy(a)).all(), k
        assert rel_err(_npy(a), _npy(b)) < 2e-2, k


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
