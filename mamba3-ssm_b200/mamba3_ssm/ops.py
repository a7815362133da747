"""Scan entry points of the B200 build, with the signatures of the reference's
``mamba3_ssm/ops.py`` (``ssm_scan_siso`` ops.py:126-134, ``ssm_scan_mimo`` ops.py:184-194,
``RMSNorm`` ops.py:96-104, ``apply_rope`` ops.py:116-119).

``ssm_scan_siso`` / ``ssm_scan_mimo`` run on sm_100a kernels through the C ABI of
libmamba3_b200.so (forward and backward, registered as autograd Functions). As in the
reference, ``trap`` is a logit and the op applies the sigmoid itself (ops.py:148), ``ADT``
is exponentiated inside (ops.py:146), and the result has the dtype of ``x``. Unlike the
reference there is no TorchScript or Python-loop tier: CPU tensors raise RuntimeError.
"""

import torch
import torch.nn as nn

from . import _lib as L

__all__ = ["RMSNorm", "apply_rope", "build_rope_freqs", "ssm_scan_siso", "ssm_scan_mimo",
           "ssm_scan_siso_states"]

_PAIRS = {(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32),
          (torch.float32, torch.bfloat16), (torch.float16, torch.float16), (torch.float16, torch.float32)}


class RMSNorm(nn.Module):
    """x / sqrt(mean(x^2) + eps) * weight, computed in fp32 and returned in x.dtype: the
    m3_rmsnorm kernel for inference, the eager formula when autograd needs a graph."""

    def __init__(self, d: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if torch.is_grad_enabled() and (x.requires_grad or self.weight.requires_grad):
            # training: the reference's own formula, differentiated by autograd
            xf = x.float()
            rms = xf.pow(2).mean(dim=-1, keepdim=True).add(self.eps).sqrt()
            return (xf / rms * self.weight).to(x.dtype)
        return rmsnorm(x, self.weight, self.eps)


def _rows_view(t: torch.Tensor) -> bool:
    """Innermost stride 1 and the leading dims collapse into rows of one stride."""
    st, sh = t.stride(), t.shape
    if t.dim() and sh[-1] > 1 and st[-1] != 1:
        return False
    return all(sh[i] <= 1 or st[i] == st[i + 1] * sh[i + 1] for i in range(t.dim() - 2))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor = None,
            residual_out: torch.Tensor = None) -> torch.Tensor:
    """RMSNorm (ops.py:94-102) on the m3_rmsnorm kernel. With ``residual``, normalises
    h = x + residual (rounded to x.dtype) and, when ``residual_out`` is given, writes h
    there (it may be x itself). Returns the normalised tensor in x.dtype."""
    if not x.is_cuda:
        raise RuntimeError("rmsnorm: the B200 build runs on CUDA tensors only (no CPU path)")
    if not _rows_view(x):
        x = x.contiguous()
    if residual is not None and not _rows_view(residual):
        residual = residual.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    lib = L.load()
    a = L.pack(x, residual, weight, out, residual_out)
    with torch.cuda.device(x.device):
        rc = lib.m3_rmsnorm(a.ptrs[0], a.ptrs[1], a.ptrs[2], float(eps), a.ptrs[3], a.ptrs[4],
                            torch.cuda.current_stream(x.device).cuda_stream)
    L.check(rc, "m3_rmsnorm")
    return out


def argmax_rows(logits: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """logits.argmax(-1) as int64 (first index of the maximum, NaN as the maximum) through
    m3_argmax_rows; ``out`` (contiguous int64, one element per row) receives it in place."""
    _require_cuda("argmax_rows", logits)
    logits = _inner(logits)
    if out is None:
        out = torch.empty(logits.shape[:-1], dtype=torch.int64, device=logits.device)
    lib = L.load()
    a = L.pack(logits, out)
    with torch.cuda.device(logits.device):
        L.check(lib.m3_argmax_rows(a.ptrs[0], a.ptrs[1], torch.cuda.current_stream(logits.device).cuda_stream),
                "m3_argmax_rows")
    return out


def build_rope_freqs(num_angles: int, device=None) -> torch.Tensor:
    i = torch.arange(num_angles, device=device, dtype=torch.float32)
    return 1.0 / (10000.0 ** (i / num_angles))


def apply_rope(x: torch.Tensor, angles: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (x[..., 0::2], x[..., 1::2]) by ``angles``."""
    c, s = torch.cos(angles), torch.sin(angles)
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack((x1 * c - x2 * s, x1 * s + x2 * c), dim=-1).flatten(-2)


def _require_cuda(name, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name}: the B200 build runs on CUDA tensors only (no CPU path); got a "
                               f"{t.device} tensor")


def _inner(t):
    return t if (t.dim() == 0 or t.shape[-1] <= 1 or t.stride(-1) == 1) else t.contiguous()


def _bc_dtype(x, B, C):
    if (x.dtype, B.dtype) not in _PAIRS:
        B = B.float()
    if C.dtype != B.dtype:
        C = C.to(B.dtype)
    return B, C


def _empty(shape, dtype, dev):
    return torch.empty(tuple(shape), dtype=dtype, device=dev)


def _siso_fwd_raw(x, B, C, ADT, DT, trap, D, h0=None, bx0=None, want_state=False, keep_states=False):
    """SISO forward on the C ABI. Returns (y, h_last, bx_last, kstates): the final states
    with ``want_state``; with ``keep_states`` and when the chunked kernels cover the shape,
    the forward's bf16 chunk-start states for the tensor-core backward (else None)."""
    lib = L.load()
    Bn, Ln, H, P = x.shape
    Ds = B.shape[-1]
    y = _empty(x.shape, x.dtype, x.device)
    hl = bl = None
    if want_state:
        hl = _empty((Bn, H, P, Ds), torch.float32, x.device)
        bl = _empty((Bn, H, P, Ds), torch.float32, x.device)
    a = L.pack(x, B, C, ADT, DT, trap, D, h0, bx0, y, hl, bl)
    ks = None
    if keep_states:
        nb = lib.m3_siso_scan_kstates_size(Bn, Ln, H, P, Ds, L._DTYPE_CODE.get(x.dtype, -1),
                                           L._DTYPE_CODE.get(B.dtype, -1))
        if nb:
            ks = torch.empty(int(nb), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        if ks is not None:
            rc = lib.m3_siso_scan_fwd_kstates(*a.ptrs, ks.data_ptr(), ks.numel(), L.stream_of(x))
            if rc == L.M3_ERR_UNSUPPORTED:
                ks = None  # e.g. unaligned strided views: the plain forward below
            else:
                L.check(rc, "m3_siso_scan_fwd_kstates")
        if ks is None:
            L.check(lib.m3_siso_scan_fwd(*a.ptrs, L.stream_of(x)), "m3_siso_scan_fwd")
    return y, hl, bl, ks


def _siso_bwd_raw(x, B, C, ADT, DT, trap, D, h0, bx0, ks, dy, need_h0=False, need_bx0=False):
    """SISO backward on the C ABI: the tensor-core pair when ``ks`` holds the forward's chunk
    states, else m3_siso_scan_bwd. Returns dx, dB, dC, dADT, dDT, dtrap, dD, dh0, dbx0."""
    lib = L.load()
    Bn, Ln, H, P = x.shape
    Ds = B.shape[-1]
    dev = x.device
    dy = _inner(dy.to(x.dtype))
    dx = _empty(x.shape, x.dtype, dev)
    dB = _empty(B.shape, B.dtype, dev)
    dC = _empty(C.shape, C.dtype, dev)
    dADT = _empty(ADT.shape, torch.float32, dev)
    dDT = _empty(DT.shape, torch.float32, dev)
    dtrap = _empty(trap.shape, torch.float32, dev)
    dD = _empty((H,), torch.float32, dev)
    dh0 = _empty(h0.shape, torch.float32, dev) if (h0 is not None and need_h0) else None
    dbx0 = _empty(bx0.shape, torch.float32, dev) if (bx0 is not None and need_bx0) else None
    a = L.pack(x, B, C, ADT, DT, trap, D, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD, dh0, dbx0)
    with torch.cuda.device(dev):
        rc = None
        if ks is not None:
            nbytes = lib.m3_siso_scan_bwd_kstates_workspace_size(Bn, Ln, H)
            ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)
            rc = lib.m3_siso_scan_bwd_kstates(*a.ptrs, ks.data_ptr(), ks.numel(), ws.data_ptr(), ws.numel(),
                                              L.stream_of(x))
            if rc != L.M3_ERR_UNSUPPORTED:  # e.g. an unaligned dy view: the general path
                L.check(rc, "m3_siso_scan_bwd_kstates")
            del ws
        if ks is None or rc == L.M3_ERR_UNSUPPORTED:
            nbytes = lib.m3_siso_scan_bwd_workspace_size(Bn, Ln, H, P, Ds)
            ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)
            L.check(lib.m3_siso_scan_bwd(*a.ptrs, ws.data_ptr(), ws.numel(), L.stream_of(x)), "m3_siso_scan_bwd")
    return dx, dB, dC, dADT, dDT, dtrap, dD, dh0, dbx0


def _mimo_fwd_raw(x, B, C, ADT, DT, trap, D, mx, mo, h0=None, bx0=None, want_state=False, keep_ws=False):
    """MIMO forward (chunk-parallel kernels) on the C ABI. Returns (y, h_last, bx_last), and
    with keep_ws also the workspace (its published chunk-end states serve the backward)."""
    lib = L.load()
    Bn, Ln, H, P = x.shape
    Ds = B.shape[-1]
    y = _empty(x.shape, x.dtype, x.device)
    hl = bl = None
    if want_state:
        hl = _empty((Bn, H, Ds), torch.float32, x.device)
        bl = _empty((Bn, H, Ds), torch.float32, x.device)
    a = L.pack(x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0, y, hl, bl)
    nbytes = lib.m3_mimo_scan_fwd_workspace_size(Bn, Ln, H, Ds)
    ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        L.check(lib.m3_mimo_scan_fwd_ws(*a.ptrs, ws.data_ptr(), ws.numel(), L.stream_of(x)), "m3_mimo_scan_fwd_ws")
    if keep_ws:
        return y, hl, bl, ws
    return y, hl, bl


def _mimo_bwd_raw(x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0, dy, need_h0=False, need_bx0=False, fwd_ws=None):
    """MIMO backward on the C ABI, from the forward's workspace when given (the single-pass
    pair). Returns dx, dB, dC, dADT, dDT, dtrap, dD, dmimo_x, dmimo_o, dh0, dbx0."""
    lib = L.load()
    Bn, Ln, H, P = x.shape
    R, Ds = B.shape[2], B.shape[-1]
    dev = x.device
    dy = _inner(dy.to(x.dtype))
    dx = _empty(x.shape, x.dtype, dev)
    dB = _empty(B.shape, B.dtype, dev)
    dC = _empty(C.shape, C.dtype, dev)
    dADT = _empty(ADT.shape, torch.float32, dev)
    dDT = _empty(DT.shape, torch.float32, dev)
    dtrap = _empty(trap.shape, torch.float32, dev)
    dD = _empty((H,), torch.float32, dev)
    dmx = _empty((H, R, P), torch.float32, dev)
    dmo = _empty((H, R, P), torch.float32, dev)
    dh0 = _empty(h0.shape, torch.float32, dev) if (h0 is not None and need_h0) else None
    dbx0 = _empty(bx0.shape, torch.float32, dev) if (bx0 is not None and need_bx0) else None
    a = L.pack(x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0, dy, dx, dB, dC, dADT, dDT, dtrap, dD, dmx, dmo,
               dh0, dbx0)
    with torch.cuda.device(dev):
        if fwd_ws is not None:
            nbytes = lib.m3_mimo_scan_bwd_ws_workspace_size(Bn, Ln, H, P, Ds, R)
            ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)
            L.check(lib.m3_mimo_scan_bwd_ws(*a.ptrs, fwd_ws.data_ptr(), fwd_ws.numel(), ws.data_ptr(), ws.numel(),
                                            L.stream_of(x)), "m3_mimo_scan_bwd_ws")
        else:
            nbytes = lib.m3_mimo_scan_bwd_workspace_size(Bn, Ln, H, P, Ds, R)
            ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)
            L.check(lib.m3_mimo_scan_bwd(*a.ptrs, ws.data_ptr(), ws.numel(), L.stream_of(x)), "m3_mimo_scan_bwd")
    return dx, dB, dC, dADT, dDT, dtrap, dD, dmx, dmo, dh0, dbx0


class _SisoScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, B, C, ADT, DT, trap, D, h0, bx0, want_state):
        # when gradients will be needed and the chunked kernels cover the shape, keep the
        # chunk-start states of the forward for the backward instead of recomputing them
        y, hl, bl, ks = _siso_fwd_raw(x, B, C, ADT, DT, trap, D, h0, bx0, want_state,
                                      keep_states=any(ctx.needs_input_grad[:9]))
        ctx.kstates = ks
        ctx.save_for_backward(x, B, C, ADT, DT, trap, D, h0, bx0)
        ctx.mark_non_differentiable(*[t for t in (hl, bl) if t is not None])
        return y, hl, bl

    @staticmethod
    def backward(ctx, dy, _dh, _dbx):
        x, B, C, ADT, DT, trap, D, h0, bx0 = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(x)
        ks = ctx.kstates
        ctx.kstates = None
        g = _siso_bwd_raw(x, B, C, ADT, DT, trap, D, h0, bx0, ks, dy, ctx.needs_input_grad[7],
                          ctx.needs_input_grad[8])
        return (*g, None)


class _MimoScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0, want_state):
        # when gradients will be needed, keep the forward's workspace (its chunk-end states)
        # for the single-pass backward
        keep = any(ctx.needs_input_grad[:11])
        out = _mimo_fwd_raw(x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0, want_state, keep_ws=keep)
        y, hl, bl = out[:3]
        ctx.fwd_ws = out[3] if keep else None
        ctx.save_for_backward(x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0)
        ctx.mark_non_differentiable(*[t for t in (hl, bl) if t is not None])
        return y, hl, bl

    @staticmethod
    def backward(ctx, dy, _dh, _dbx):
        x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0 = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(x)
        fws = ctx.fwd_ws
        ctx.fwd_ws = None
        g = _mimo_bwd_raw(x, B, C, ADT, DT, trap, D, mx, mo, h0, bx0, dy, ctx.needs_input_grad[9],
                          ctx.needs_input_grad[10], fwd_ws=fws)
        return (*g, None)


def _prep_siso(x, B_proj, C_proj, ADT, DT, trap, D):
    _require_cuda("ssm_scan_siso", x, B_proj, C_proj, ADT, DT, trap, D)
    if x.dim() != 4 or B_proj.dim() != 4 or C_proj.dim() != 4:
        raise ValueError("ssm_scan_siso: x is (B, L, H, P) and B_proj, C_proj are (B, L, H, D)")
    B_proj, C_proj = _bc_dtype(x, B_proj, C_proj)
    return (_inner(x), _inner(B_proj), _inner(C_proj), ADT.float(), DT.float(), trap.float(),
            D.float())


def ssm_scan_siso(x, B_proj, C_proj, ADT, DT, trap, D):
    """SISO scan (reference ops.py:126-177). x (B,L,H,P); B_proj, C_proj (B,L,H,D);
    ADT, DT, trap (B,L,H) with trap a logit; D (H). Returns y (B,L,H,P) in x.dtype."""
    args = _prep_siso(x, B_proj, C_proj, ADT, DT, trap, D)
    y, _, _ = _SisoScanFn.apply(*args, None, None, False)
    return y


def ssm_scan_siso_states(x, B_proj, C_proj, ADT, DT, trap, D, ssm_state=None, bx_prev=None):
    """SISO scan that starts from a decode cache (ssm_state, bx_prev: (B,H,P,D) fp32, as
    Mamba3.allocate_inference_cache returns) and also returns the cache after the last
    token: (y, ssm_state, bx_prev). Equivalent to feeding the tokens one by one through
    the recurrence of Mamba3.step."""
    args = _prep_siso(x, B_proj, C_proj, ADT, DT, trap, D)
    h0 = ssm_state.float().contiguous() if ssm_state is not None else None
    b0 = bx_prev.float().contiguous() if bx_prev is not None else None
    return _SisoScanFn.apply(*args, h0, b0, True)


def ssm_scan_mimo(x, B_proj, C_proj, ADT, DT, trap, D, mimo_x, mimo_o):
    """MIMO scan (reference ops.py:184-242). x (B,L,H,P); B_proj, C_proj (B,L,R,H,D);
    mimo_x, mimo_o (H,R,P). Returns y (B,L,H,P) in x.dtype."""
    _require_cuda("ssm_scan_mimo", x, B_proj, C_proj, ADT, DT, trap, D, mimo_x, mimo_o)
    if x.dim() != 4 or B_proj.dim() != 5 or C_proj.dim() != 5:
        raise ValueError("ssm_scan_mimo: x is (B, L, H, P) and B_proj, C_proj are (B, L, R, H, D)")
    B_proj, C_proj = _bc_dtype(x, B_proj, C_proj)
    y, _, _ = _MimoScanFn.apply(_inner(x), _inner(B_proj), _inner(C_proj), ADT.float(), DT.float(),
                                trap.float(), D.float(), _inner(mimo_x.float()), _inner(mimo_o.float()),
                                None, None, False)
    return y
