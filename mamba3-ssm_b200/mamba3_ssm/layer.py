"""Mamba3 mixer with the constructor, parameters (names, shapes, init order), forward,
step and allocate_inference_cache of the reference's ``mamba3_ssm/layer.py`` (:61-412).

* ``forward`` runs in_proj and out_proj (cuBLAS) around fused kernels for everything between
  them (softplus / clamp, RMSNorm + bias + RoPE of B / C, the angle cumsum, the scan, the silu
  gate), with their backward kernels under autograd; a one-group MIMO layer's inference
  forward forms B / C inside the scan (``m3_mimo_layer_scan_fwd``). Continuing from, or
  returning, a decode cache under autograd keeps the reference's PyTorch prologue around the
  scan kernels.
* ``step`` runs everything between in_proj and out_proj of one decode step
  (layer.py:298-371) as a single fused kernel (``m3_siso_step`` / ``m3_mimo_step``).
  Like the reference it returns new state tensors and leaves its inputs untouched.
"""

import ctypes
import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib as L
from .ops import (RMSNorm, _bc_dtype, _inner, _mimo_bwd_raw, _mimo_fwd_raw, _MimoScanFn, _siso_bwd_raw,
                  _siso_fwd_raw, apply_rope, ssm_scan_mimo, ssm_scan_siso, ssm_scan_siso_states)


class _StepNoGrad(torch.autograd.Function):
    """Marks the outputs of the fused decode step: running it under grad mode is fine
    (generation loops often do), but differentiating through it is not supported."""

    @staticmethod
    def forward(ctx, runner, *tensors):
        return runner()

    @staticmethod
    def backward(ctx, *grads):
        raise RuntimeError("Mamba3.step is inference-only in the B200 build: its fused kernel has no "
                           "backward. Differentiate through Mamba3.forward instead.")


def _f32(t):
    return None if t is None else t.detach().float().contiguous()


class _LayerCoreFn(torch.autograd.Function):
    """Everything Mamba3.forward does between in_proj and out_proj (layer.py:180-262), for
    training, on the fused kernels. Forward: m3_layer_prologue (dt / decay / trap, RMSNorm +
    bias + RoPE of B and C per head, the angle cumsum), the scan (the SISO tensor-core pair
    keeps its chunk states), m3_silu_gate. Backward: m3_silu_gate_bwd, the scan backward
    and m3_layer_prologue_bwd, which together fill the gradient of the in_proj output and
    of every mixer parameter. Returns the gated output (B, L, H, P) in zx's dtype."""

    @staticmethod
    def forward(ctx, zx, dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, Dskip, mimo_x, mimo_o, layer):
        lib = L.load()
        batch, Ln, _ = zx.shape
        R, Ds, H, P, S, di = (layer.mimo_rank, layer.d_state, layer.nheads, layer.headdim, layer.num_rope_angles,
                              layer.d_inner)
        dev = zx.device
        dims = layer._dims()
        pb = [_f32(t) for t in (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w)]
        op = torch.bfloat16 if zx.dtype == torch.bfloat16 else torch.float32
        Bp = torch.empty(batch, Ln, R, H, Ds, dtype=op, device=dev)
        Cp = torch.empty(batch, Ln, R, H, Ds, dtype=op, device=dev)
        ADT, DT, trap = (torch.empty(batch, Ln, H, dtype=torch.float32, device=dev) for _ in range(3))
        ang = torch.empty(batch, Ln, H, S, dtype=torch.float32, device=dev)
        a = L.pack(zx, *pb, None, Bp, Cp, ADT, DT, trap, ang)
        with torch.cuda.device(dev):
            L.check(lib.m3_layer_prologue(ctypes.byref(dims), *a.ptrs, L.stream_of(zx)), "m3_layer_prologue")
        z = zx[..., :di].unflatten(-1, (H, P))
        x = zx[..., di:2 * di].unflatten(-1, (H, P))
        Dv = _f32(Dskip)
        ks = None
        mx = mo = None
        if layer.is_mimo:
            mx, mo = _f32(mimo_x), _f32(mimo_o)
            y, _, _, ks = _mimo_fwd_raw(x, Bp, Cp, ADT, DT, trap, Dv, mx, mo, keep_ws=True)
        else:
            y, _, _, ks = _siso_fwd_raw(x, Bp[:, :, 0], Cp[:, :, 0], ADT, DT, trap, Dv, keep_states=True)
        g = torch.empty(batch, Ln, H, P, dtype=zx.dtype, device=dev)
        a = L.pack(y, z, g)
        with torch.cuda.device(dev):
            L.check(lib.m3_silu_gate(*a.ptrs, L.stream_of(zx)), "m3_silu_gate")
        ctx.save_for_backward(zx, Bp, Cp, ADT, DT, trap, ang, y, Dv, *pb, mx, mo)
        ctx.ks = ks
        ctx.layer = layer
        ctx.dtypes = [None if t is None else t.dtype for t in (dt_bias, B_bias, C_bias, B_norm_w, C_norm_w, Dskip,
                                                               mimo_x, mimo_o)]
        return g

    @staticmethod
    def backward(ctx, dg):
        zx, Bp, Cp, ADT, DT, trap, ang, y, Dv, dtb, Bb, Cb, Bw, Cw, mx, mo = ctx.saved_tensors
        layer = ctx.layer
        lib = L.load()
        H, P, di = layer.nheads, layer.headdim, layer.d_inner
        dev = zx.device
        dzx = torch.empty_like(zx)
        z = zx[..., :di].unflatten(-1, (H, P))
        x = zx[..., di:2 * di].unflatten(-1, (H, P))
        dg = _inner(dg.to(zx.dtype))
        dy = torch.empty_like(y)
        a = L.pack(y, z, dg, dy, dzx[..., :di].unflatten(-1, (H, P)))
        with torch.cuda.device(dev):
            L.check(lib.m3_silu_gate_bwd(*a.ptrs, L.stream_of(zx)), "m3_silu_gate_bwd")
        dmx = dmo = None
        if layer.is_mimo:
            fws = ctx.ks
            ctx.ks = None
            dx, dBp, dCp, dADT, dDT, dtrap, dD, dmx, dmo, _, _ = _mimo_bwd_raw(x, Bp, Cp, ADT, DT, trap, Dv, mx, mo,
                                                                             None, None, dy, fwd_ws=fws)
        else:
            ks = ctx.ks
            ctx.ks = None
            dx, dB, dC, dADT, dDT, dtrap, dD, _, _ = _siso_bwd_raw(x, Bp[:, :, 0], Cp[:, :, 0], ADT, DT, trap, Dv,
                                                                   None, None, ks, dy)
            dBp, dCp = dB.unsqueeze(2), dC.unsqueeze(2)
        dzx[..., di:2 * di].copy_(dx.flatten(-2))
        grads = [torch.empty(t.shape, dtype=torch.float32, device=dev) for t in (dtb, Bb, Cb, Bw, Cw)]
        dims = layer._dims()
        nbytes = lib.m3_layer_prologue_bwd_workspace_size(ctypes.byref(dims), zx.shape[0], zx.shape[1])
        ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)
        a = L.pack(zx, dtb, Bb, Cb, Bw, Cw, DT, ang, dBp, dCp, dADT, dDT, dtrap, dzx, *grads)
        with torch.cuda.device(dev):
            L.check(lib.m3_layer_prologue_bwd(ctypes.byref(dims), *a.ptrs, ws.data_ptr(), ws.numel(),
                                              L.stream_of(zx)), "m3_layer_prologue_bwd")
        out = grads + [dD, dmx, dmo]
        out = [None if (gv is None or dt is None) else gv.to(dt) for gv, dt in zip(out, ctx.dtypes)]
        return (dzx, *out, None)


class Mamba3(nn.Module):
    def __init__(self, d_model: int, d_state: int = 128, expand: int = 2, headdim: int = 64,
                 ngroups: int = 1, rope_fraction: float = 0.5, dt_min: float = 0.001,
                 dt_max: float = 0.1, dt_init_floor: float = 1e-4, A_floor: float = 1e-4,
                 is_mimo: bool = False, mimo_rank: int = 4, device=None, dtype=None):
        factory_kwargs = {"device": device, "dtype": dtype}
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.expand = expand
        self.headdim = headdim
        self.A_floor = A_floor
        self.is_mimo = is_mimo
        self.mimo_rank = mimo_rank if is_mimo else 1
        self.num_bc_heads = ngroups
        self.d_inner = int(expand * d_model)
        assert self.d_inner % headdim == 0, f"d_inner ({self.d_inner}) must be divisible by headdim ({headdim})"
        self.nheads = self.d_inner // headdim
        assert rope_fraction in (0.5, 1.0), "rope_fraction must be 0.5 or 1.0"
        split = int(d_state * rope_fraction)
        self.split_tensor_size = split - (split % 2)
        self.num_rope_angles = self.split_tensor_size // 2
        assert self.num_rope_angles > 0
        d_in_proj = (2 * self.d_inner + 2 * d_state * ngroups * self.mimo_rank + 3 * self.nheads
                     + self.num_rope_angles)
        # Parameter creation order matches the reference (in_proj init, then one
        # torch.rand(nheads) draw for dt_bias, then out_proj init), so the same seed gives
        # the same weights.
        self.in_proj = nn.Linear(d_model, d_in_proj, bias=False, **factory_kwargs)
        dt = torch.exp(torch.rand(self.nheads, dtype=torch.float32) * (math.log(dt_max) - math.log(dt_min))
                       + math.log(dt_min)).clamp(min=dt_init_floor)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))  # inverse softplus
        self.dt_bias._no_weight_decay = True
        self.B_bias = nn.Parameter(torch.ones(self.nheads, self.mimo_rank, d_state, dtype=torch.float32))
        self.C_bias = nn.Parameter(torch.ones(self.nheads, self.mimo_rank, d_state, dtype=torch.float32))
        self.B_bias._no_weight_decay = True
        self.C_bias._no_weight_decay = True
        self.B_norm = RMSNorm(d_state)
        self.C_norm = RMSNorm(d_state)
        if self.is_mimo:
            self.mimo_x = nn.Parameter(torch.ones(self.nheads, self.mimo_rank, headdim, **factory_kwargs)
                                       / self.mimo_rank)
            self.mimo_o = nn.Parameter(torch.ones(self.nheads, self.mimo_rank, headdim, **factory_kwargs)
                                       / self.mimo_rank)
        self.D = nn.Parameter(torch.ones(self.nheads, **factory_kwargs))
        self.D._no_weight_decay = True
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=False, **factory_kwargs)
        if device is not None:
            # the fp32 parameters above are drawn and filled on the CPU (same RNG stream as the
            # reference); place them on the requested device
            for mod in (self, self.B_norm, self.C_norm):
                for name, prm in list(mod._parameters.items()):
                    if prm is not None and prm.device != torch.device(device):
                        mod._parameters[name] = nn.Parameter(prm.data.to(device), requires_grad=prm.requires_grad)
            for prm_name in ("dt_bias", "B_bias", "C_bias", "D"):
                getattr(self, prm_name)._no_weight_decay = True
        self._splits = [self.d_inner, self.d_inner, d_state * ngroups * self.mimo_rank,
                        d_state * ngroups * self.mimo_rank, self.nheads, self.nheads, self.nheads,
                        self.num_rope_angles]
        self._f32_cache = None

    # ------------------------------------------------------------------------------
    def _bc(self, raw, norm, bias):
        """RMSNorm over d_state, broadcast groups to heads, add the per-head bias."""
        n = norm(raw.float())
        n = n.expand(*n.shape[:-2], self.nheads, self.d_state)
        return n + bias.transpose(0, 1)  # (H,R,D) -> (R,H,D)

    def forward(self, u: torch.Tensor, cache=None, return_cache: bool = False):
        """Mamba3.forward of the reference (layer.py:168-266) for ``forward(u)``.

        Not in the reference (whose generate prefills one step() per prompt token): with
        ``cache`` (an (angle, ssm, bx_prev) triple as allocate_inference_cache returns) the
        sequence continues from that decode state, and with ``return_cache`` the call returns
        ``(out, cache)``, the cache after the last token, from the chunked scan. Feeding a
        prompt through forward(..., return_cache=True) then decoding with step() reproduces
        stepping through the prompt token by token."""
        want = return_cache or cache is not None
        if not (torch.is_grad_enabled() and (u.requires_grad or any(p.requires_grad for p in self.parameters()))):
            out, new = self._forward_fused(u, cache, want)
        else:
            out, new = self._forward_autograd(u, cache, want)
        return (out, new) if return_cache else out

    def _forward_fused(self, u: torch.Tensor, cache=None, want_cache: bool = False):
        """Inference forward: in_proj, then for a one-group MIMO layer the scalar prologue and
        the group-row scan with the gate fused (_forward_mimo_rows); otherwise the fused
        prologue kernel (m3_layer_prologue: dt / decay / trap, RMSNorm + bias + RoPE of B and C
        per head, the angle cumsum), the scan and the fused silu gate (m3_silu_gate); out_proj.
        bf16 layers give the scan bf16 B / C (the tensor-core path); other dtypes keep them in
        fp32."""
        batch, Ln, _ = u.shape
        R, Ds, H, P, S = self.mimo_rank, self.d_state, self.nheads, self.headdim, self.num_rope_angles
        zx = self.in_proj(u)
        if not zx.is_cuda:
            raise RuntimeError("Mamba3.forward: the B200 build runs on CUDA tensors only (no CPU path)")
        if zx.stride(-1) != 1:
            zx = zx.contiguous()
        vals = self._step_params()
        dims = self._f32_cache[3]
        if self.is_mimo and self.num_bc_heads == 1:
            r = self._forward_mimo_rows(zx, vals, dims, cache, want_cache)
            if r is not None:
                return r
        dev = zx.device
        op = torch.bfloat16 if zx.dtype == torch.bfloat16 else torch.float32
        Bp = torch.empty(batch, Ln, R, H, Ds, dtype=op, device=dev)
        Cp = torch.empty(batch, Ln, R, H, Ds, dtype=op, device=dev)
        ADT, DT, trap = (torch.empty(batch, Ln, H, dtype=torch.float32, device=dev) for _ in range(3))
        ang = torch.empty(batch, Ln, H, S, dtype=torch.float32, device=dev)
        ang0 = cache[0].float().contiguous() if cache is not None else None
        lib = L.load()
        a = L.pack(zx, *vals[:5], ang0, Bp, Cp, ADT, DT, trap, ang)
        with torch.cuda.device(dev):
            rc = lib.m3_layer_prologue(ctypes.byref(dims), *a.ptrs, torch.cuda.current_stream(dev).cuda_stream)
        L.check(rc, "m3_layer_prologue")
        di = self.d_inner
        z = zx[..., :di].unflatten(-1, (H, P))
        x = zx[..., di:2 * di].unflatten(-1, (H, P))
        y, new = self._scan(x, Bp, Cp, ADT, DT, trap, ang, cache, want_cache)
        g = torch.empty(batch, Ln, H, P, dtype=zx.dtype, device=dev)
        a = L.pack(y, z, g)
        with torch.cuda.device(dev):
            rc = lib.m3_silu_gate(*a.ptrs, torch.cuda.current_stream(dev).cuda_stream)
        L.check(rc, "m3_silu_gate")
        return self.out_proj(g.flatten(-2)), new

    def _forward_mimo_rows(self, zx, vals, dims, cache, want_cache):
        """Inference forward of a one-group MIMO layer without per-head B / C tensors:
        m3_layer_prologue writes only the step scalars and angles, and
        m3_mimo_layer_scan_fwd forms B / C from the group rows inside the scan and gates its
        output. None (after the scalar prologue, nothing else launched) when that kernel does
        not apply to this layout; the caller then runs the prologue with B / C and the scan."""
        batch, Ln, _ = zx.shape
        Ds, H, P, S = self.d_state, self.nheads, self.headdim, self.num_rope_angles
        dev = zx.device
        ADT, DT, trap = (torch.empty(batch, Ln, H, dtype=torch.float32, device=dev) for _ in range(3))
        ang = torch.empty(batch, Ln, H, S, dtype=torch.float32, device=dev)
        ang0 = cache[0].float().contiguous() if cache is not None else None
        lib = L.load()
        stream = torch.cuda.current_stream(dev).cuda_stream
        a = L.pack(zx, *vals[:5], ang0, None, None, ADT, DT, trap, ang)
        with torch.cuda.device(dev):
            rc = lib.m3_layer_prologue(ctypes.byref(dims), *a.ptrs, stream)
        L.check(rc, "m3_layer_prologue")
        h0 = b0 = hl = bl = None
        if want_cache:
            if cache is not None:
                h0 = cache[1].float().contiguous()
                b0 = cache[2].float().contiguous()
            hl = torch.empty(batch, H, Ds, dtype=torch.float32, device=dev)
            bl = torch.empty(batch, H, Ds, dtype=torch.float32, device=dev)
        g = torch.empty(batch, Ln, H, P, dtype=zx.dtype, device=dev)
        ws = torch.empty(lib.m3_mimo_scan_fwd_workspace_size(batch, Ln, H, Ds), dtype=torch.uint8, device=dev)
        a = L.pack(zx, ADT, DT, trap, ang, vals[1], vals[2], vals[3], vals[4], vals[5], vals[6], vals[7], h0, b0)
        o = L.pack(g, hl, bl)
        with torch.cuda.device(dev):
            rc = lib.m3_mimo_layer_scan_fwd(ctypes.byref(dims), *a.ptrs, 1, *o.ptrs, ws.data_ptr(), ws.numel(),
                                            stream)
        if rc == L.M3_ERR_UNSUPPORTED:
            return None
        L.check(rc, "m3_mimo_layer_scan_fwd")
        new = None
        if want_cache:
            if Ln > 0:
                a_last = ang[:, -1].contiguous()
            elif cache is not None:
                a_last = cache[0].float().clone()
            else:
                a_last = torch.zeros(batch, H, S, device=dev)
            new = (a_last, hl, bl)
        return self.out_proj(g.flatten(-2)), new

    def _scan(self, x, Bp, Cp, ADT, DT, trap, ang, cache, want_cache):
        """The scan of forward; with ``want_cache`` it starts from ``cache`` (or zeros) and
        also returns the cache after the last token (angle state = the last angles)."""
        if not want_cache:
            if self.is_mimo:
                return ssm_scan_mimo(x, Bp, Cp, ADT, DT, trap, self.D, self.mimo_x, self.mimo_o), None
            return ssm_scan_siso(x, Bp[:, :, 0], Cp[:, :, 0], ADT, DT, trap, self.D), None
        h0 = b0 = None
        if cache is not None:
            h0 = cache[1].float().contiguous()
            b0 = cache[2].float().contiguous()
        if self.is_mimo:
            B_, C_ = _bc_dtype(x, Bp, Cp)
            y, hl, bl = _MimoScanFn.apply(_inner(x), _inner(B_), _inner(C_), ADT.float(), DT.float(), trap.float(),
                                          self.D.float(), _inner(self.mimo_x.float()), _inner(self.mimo_o.float()),
                                          h0, b0, True)
        else:
            y, hl, bl = ssm_scan_siso_states(x, Bp[:, :, 0], Cp[:, :, 0], ADT, DT, trap, self.D, h0, b0)
        if ang.shape[1] > 0:
            a_last = ang[:, -1].float().contiguous()
        elif cache is not None:
            a_last = cache[0].float().clone()
        else:
            a_last = torch.zeros(x.shape[0], self.nheads, self.num_rope_angles, device=x.device)
        return y, (a_last, hl, bl)

    def _forward_autograd(self, u: torch.Tensor, cache=None, want_cache: bool = False):
        """Training forward. Without a decode cache: in_proj, the fused prologue / scan / gate
        with their backward kernels (_LayerCoreFn), out_proj. With one (continuing from, or
        returning, decode states): the reference's PyTorch prologue, differentiated by
        autograd, around the scan kernels."""
        if cache is None and not want_cache:
            zx = self.in_proj(u)
            if not zx.is_cuda:
                raise RuntimeError("Mamba3.forward: the B200 build runs on CUDA tensors only (no CPU path)")
            if zx.stride(-1) != 1:
                zx = zx.contiguous()
            g = _LayerCoreFn.apply(zx, self.dt_bias, self.B_bias, self.C_bias, self.B_norm.weight, self.C_norm.weight,
                                   self.D, self.mimo_x if self.is_mimo else None,
                                   self.mimo_o if self.is_mimo else None, self)
            return self.out_proj(g.flatten(-2)), None
        batch, Ln, _ = u.shape
        R, G, Ds, H, P = self.mimo_rank, self.num_bc_heads, self.d_state, self.nheads, self.headdim
        z, x, B_raw, C_raw, dd_dt, dd_A, trap_raw, angle_raw = torch.split(self.in_proj(u), self._splits, dim=-1)
        z = z.unflatten(-1, (H, P))
        x = x.unflatten(-1, (H, P))
        B_raw = B_raw.unflatten(-1, (R, G, Ds))
        C_raw = C_raw.unflatten(-1, (R, G, Ds))
        A = -F.softplus(dd_A.float()).clamp(max=-self.A_floor)
        DT = F.softplus(dd_dt.float() + self.dt_bias)
        ADT = A * DT
        Bh = self._bc(B_raw, self.B_norm, self.B_bias)
        Ch = self._bc(C_raw, self.C_norm, self.C_bias)
        ang_h = torch.cumsum(angle_raw.float().unsqueeze(2) * DT.unsqueeze(-1), dim=1)  # (B,L,H,S)
        if cache is not None:
            ang_h = ang_h + cache[0].float().unsqueeze(1)
        ang = ang_h.unsqueeze(2).expand(batch, Ln, R, H, self.num_rope_angles)
        k = self.split_tensor_size
        B_proj = torch.cat([apply_rope(Bh[..., :k], ang), Bh[..., k:]], dim=-1)
        C_proj = torch.cat([apply_rope(Ch[..., :k], ang), Ch[..., k:]], dim=-1)
        y, new = self._scan(x, B_proj, C_proj, ADT, DT, trap_raw.float(), ang_h, cache, want_cache)
        y = y * F.silu(z.float())
        return self.out_proj(y.flatten(-2).to(x.dtype)), new

    # ------------------------------------------------------------------------------
    def _dims(self):
        d = L.M3LayerDims()
        d.d_model, d.d_inner, d.nheads, d.headdim = self.d_model, self.d_inner, self.nheads, self.headdim
        d.d_state, d.ngroups, d.mimo_rank = self.d_state, self.num_bc_heads, self.mimo_rank
        d.num_rope_angles, d.rope_split = self.num_rope_angles, self.split_tensor_size
        d.A_floor, d.norm_eps = float(self.A_floor), float(self.B_norm.eps)
        return d

    def _step_params(self):
        """fp32 contiguous views of the per-head parameters the step kernel reads, cached
        until a parameter changes (in-place update, new tensor or new device)."""
        ps = [self.dt_bias, self.B_bias, self.C_bias, self.B_norm.weight, self.C_norm.weight, self.D]
        if self.is_mimo:
            ps += [self.mimo_x, self.mimo_o]
        key = tuple((p.data_ptr(), p._version, p.dtype, p.device) for p in ps)
        if self._f32_cache is None or self._f32_cache[0] != key:
            with torch.no_grad():
                vals = [p.detach().float().contiguous() for p in ps]
            self._f32_cache = (key, vals, L.pack(*vals), self._dims())
        return self._f32_cache[1]

    def _fused_step(self, zxbcdt, ang_in, ssm_in, bx_in, ang_out, ssm_out, bx_out, y):
        """One decode step of the fused kernel (m3_siso_step / m3_mimo_step). Outputs may
        alias inputs (in-place state update)."""
        self._step_params()
        _, _, pp, dims = self._f32_cache
        lib = L.load()
        fn, name = (lib.m3_mimo_step, "m3_mimo_step") if self.is_mimo else (lib.m3_siso_step, "m3_siso_step")
        dyn = L.pack(zxbcdt, ang_in, ssm_in, bx_in, ang_out, ssm_out, bx_out, y)
        dev = zxbcdt.device
        with torch.cuda.device(dev):
            rc = fn(ctypes.byref(dims), dyn.ptrs[0], *pp.ptrs, *dyn.ptrs[1:],
                    torch.cuda.current_stream(dev).cuda_stream)
        L.check(rc, name)

    def step(self, u: torch.Tensor, angle_state: torch.Tensor, ssm_state: torch.Tensor,
             bx_prev_state: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        zxbcdt = self.in_proj(u)
        if not zxbcdt.is_cuda:
            raise RuntimeError("Mamba3.step: the B200 build runs on CUDA tensors only (no CPU path)")
        if zxbcdt.stride(-1) != 1:
            zxbcdt = zxbcdt.contiguous()
        batch = zxbcdt.shape[0]
        ang_in = angle_state.float().contiguous()
        ssm_in = ssm_state.float().contiguous()
        bx_in = bx_prev_state.float().contiguous()

        def run():
            ang_out = torch.empty_like(ang_in)
            ssm_out = torch.empty_like(ssm_in)
            bx_out = torch.empty_like(bx_in)
            y = torch.empty((batch, self.d_inner), dtype=zxbcdt.dtype, device=zxbcdt.device)
            self._fused_step(zxbcdt, ang_in, ssm_in, bx_in, ang_out, ssm_out, bx_out, y)
            return y, ang_out, ssm_out, bx_out

        if torch.is_grad_enabled() and zxbcdt.requires_grad:
            y, ang_out, ssm_out, bx_out = _StepNoGrad.apply(run, zxbcdt)
        else:
            y, ang_out, ssm_out, bx_out = run()
        out = self.out_proj(y.to(u.dtype))
        return out, ang_out, ssm_out, bx_out

    def step_inplace(self, u: torch.Tensor, angle_state: torch.Tensor, ssm_state: torch.Tensor,
                     bx_prev_state: torch.Tensor) -> torch.Tensor:
        """Like step(), but updates the (fp32, contiguous) state tensors in place and returns
        only the output; allocation-stable, so it can be recorded in a CUDA graph."""
        zxbcdt = self.in_proj(u)
        if zxbcdt.stride(-1) != 1:
            zxbcdt = zxbcdt.contiguous()
        y = torch.empty((zxbcdt.shape[0], self.d_inner), dtype=zxbcdt.dtype, device=zxbcdt.device)
        self._fused_step(zxbcdt, angle_state, ssm_state, bx_prev_state, angle_state, ssm_state, bx_prev_state, y)
        return self.out_proj(y.to(u.dtype))

    def allocate_inference_cache(self, batch_size: int, device=None, dtype=None):
        """Zero decode states (layer.py:380-412): angle (B,H,S), ssm and bx_prev
        (B,H,P,D) for SISO or (B,H,D) for MIMO, all fp32."""
        device = device or self.in_proj.weight.device
        angle_state = torch.zeros(batch_size, self.nheads, self.num_rope_angles, device=device, dtype=torch.float32)
        shape = (batch_size, self.nheads, self.d_state) if self.is_mimo else \
            (batch_size, self.nheads, self.headdim, self.d_state)
        return (angle_state, torch.zeros(shape, device=device, dtype=torch.float32),
                torch.zeros(shape, device=device, dtype=torch.float32))

    def extra_repr(self) -> str:
        return (f"d_model={self.d_model}, d_state={self.d_state}, d_inner={self.d_inner}, "
                f"nheads={self.nheads}, headdim={self.headdim}, is_mimo={self.is_mimo}, "
                f"mimo_rank={self.mimo_rank}")
