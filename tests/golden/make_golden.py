"""Generate the golden fixtures under tests/golden/ by running the reference itself.

This script imports the upstream ``mamba3_ssm`` package (Aiyoniganmaaiya/mamba3-ssm
v0.2.1) from a read-only checkout and records, on the CPU, the outputs of its own
scan loops (``mamba3_ssm/ops.py:160-177`` SISO, ``ops.py:221-242`` MIMO), of autograd
through those loops, of ``Mamba3.forward`` / ``Mamba3.step`` (``mamba3_ssm/layer.py``)
and of ``MambaLMHeadModel.forward`` / ``step`` (``mamba3_ssm/block.py``).

The fixtures are small ``.npz`` files. bf16 tensors are stored as their raw 16-bit
patterns (``uint16`` arrays); every other array keeps its own dtype.

Usage (run in the build container, where the checkout exists)::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [--ref /root/reference]

Nothing at test time imports the reference; only the committed ``.npz`` files are read.
"""

import argparse
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    import torch
    if t is None:
        return None
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        # raw bf16 bits; the test loader turns uint16 arrays back into bf16 tensors
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def scan_inputs(gen, B, L, H, P, D, dtype, mimo_rank=None, rope=True):
    """Seeded scan-op inputs with the long-context distribution:
    x, B, C ~ N(0,1); dt = clamp(softplus(N(-3, 0.5)), 1e-3, 0.1);
    A_h = -exp(U(0, ln 16)); ADT = A*dt; trap = sigmoid(N(0,1)) (passed as the
    op's logit argument, so the op applies the sigmoid a second time);
    RoPE with theta_i = 10000^(-2i/D) on the first D/2 state dims."""
    import torch
    import torch.nn.functional as F
    from mamba3_ssm.ops import apply_rope
    R = mimo_rank
    bc_shape = (B, L, H, D) if R is None else (B, L, R, H, D)
    x = torch.randn(B, L, H, P, generator=gen)
    Bp = torch.randn(*bc_shape, generator=gen)
    Cp = torch.randn(*bc_shape, generator=gen)
    dt = F.softplus(torch.randn(B, L, H, generator=gen) * 0.5 - 3.0).clamp(1e-3, 0.1)
    A = -torch.exp(torch.rand(H, generator=gen) * math.log(16.0))
    ADT = A * dt
    trap = torch.sigmoid(torch.randn(B, L, H, generator=gen))
    Dw = torch.randn(H, generator=gen) * 0.5 + 1.0
    if rope:
        S = D // 4
        theta = 10000.0 ** (-2.0 * torch.arange(S, dtype=torch.float32) / D)
        ang = torch.cumsum(dt, dim=1).unsqueeze(-1) * theta  # (B,L,H,S)
        if R is not None:
            ang = ang.unsqueeze(2).expand(B, L, R, H, S)
        Bp = torch.cat([apply_rope(Bp[..., :2 * S], ang), Bp[..., 2 * S:]], dim=-1)
        Cp = torch.cat([apply_rope(Cp[..., :2 * S], ang), Cp[..., 2 * S:]], dim=-1)
    x = x.to(dtype)
    Bp = Bp.to(dtype)
    Cp = Cp.to(dtype)
    return x, Bp, Cp, ADT, dt, trap, Dw


def gen_siso_op(name, B, L, H, P, D, dtype, seed):
    import torch
    from mamba3_ssm.ops import ssm_scan_siso
    gen = torch.Generator().manual_seed(seed)
    x, Bp, Cp, ADT, DT, trap, Dw = scan_inputs(gen, B, L, H, P, D, dtype)
    dy = torch.randn(B, L, H, P, generator=gen).to(dtype)
    leaves = [t.clone().requires_grad_(True) for t in (x, Bp, Cp, ADT, DT, trap, Dw)]
    y = ssm_scan_siso(*leaves)
    y.backward(dy)
    out = dict(dtype=str(dtype).replace("torch.", ""), x=_np(x), B=_np(Bp), C=_np(Cp),
               ADT=_np(ADT), DT=_np(DT), trap=_np(trap), D=_np(Dw), dy=_np(dy), y=_np(y))
    for k, t in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), leaves):
        out[k] = _np(t.grad)
    np.savez_compressed(os.path.join(HERE, name), **out)


def gen_mimo_op(name, B, L, H, P, D, R, dtype, seed):
    import torch
    from mamba3_ssm.ops import ssm_scan_mimo
    gen = torch.Generator().manual_seed(seed)
    x, Bp, Cp, ADT, DT, trap, Dw = scan_inputs(gen, B, L, H, P, D, dtype, mimo_rank=R)
    mx = (torch.randn(H, R, P, generator=gen) * 0.3 + 1.0 / R).to(dtype)
    mo = (torch.randn(H, R, P, generator=gen) * 0.3 + 1.0 / R).to(dtype)
    dy = torch.randn(B, L, H, P, generator=gen).to(dtype)
    leaves = [t.clone().requires_grad_(True) for t in (x, Bp, Cp, ADT, DT, trap, Dw, mx, mo)]
    y = ssm_scan_mimo(*leaves)
    y.backward(dy)
    out = dict(dtype=str(dtype).replace("torch.", ""), x=_np(x), B=_np(Bp), C=_np(Cp),
               ADT=_np(ADT), DT=_np(DT), trap=_np(trap), D=_np(Dw), mimo_x=_np(mx),
               mimo_o=_np(mo), dy=_np(dy), y=_np(y))
    for k, t in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD", "dmimo_x", "dmimo_o"), leaves):
        out[k] = _np(t.grad)
    np.savez_compressed(os.path.join(HERE, name), **out)


def _sd(module):
    return {"w." + k: _np(v) for k, v in module.state_dict().items()}


def gen_layer(name, cfg, batch, L, dtype, seed_w, seed_x, grad, perturb=False):
    """Mamba3.forward (layer.py:168-266) at default init from torch.manual_seed(seed_w),
    optional backward with dy ~ N(0,1), and the token-by-token step() replay of the
    first few positions from a zero cache (layer.py:272-374, 380-412). With ``perturb``
    the parameters that init leaves constant (B_bias, C_bias and the B / C norm weights
    are all ones, D ones) get distinct seeded values, so that a fixture tells heads,
    ranks and state columns apart."""
    import torch
    from mamba3_ssm.layer import Mamba3
    torch.manual_seed(seed_w)
    m = Mamba3(**cfg)
    if perturb:
        pg = torch.Generator().manual_seed(seed_w + 1000)
        with torch.no_grad():
            for p in (m.B_bias, m.C_bias, m.B_norm.weight, m.C_norm.weight):
                p.copy_(1.0 + 0.5 * torch.randn(p.shape, generator=pg))
            m.D.copy_(torch.randn(m.D.shape, generator=pg))
    if dtype != torch.float32:
        m = m.to(dtype)
    gen = torch.Generator().manual_seed(seed_x)
    u = torch.randn(batch, L, cfg["d_model"], generator=gen).to(dtype)
    dy = torch.randn(batch, L, cfg["d_model"], generator=gen).to(dtype)
    out = dict(dtype=str(dtype).replace("torch.", ""), u=_np(u), dy=_np(dy))
    out.update(_sd(m))
    for k, v in cfg.items():
        out["cfg." + k] = np.asarray(v)
    if grad:
        ul = u.clone().requires_grad_(True)
        y = m(ul)
        y.backward(dy)
        out["y"] = _np(y)
        out["du"] = _np(ul.grad)
        for k, p in m.named_parameters():
            out["g." + k] = _np(p.grad)
    else:
        with torch.no_grad():
            out["y"] = _np(m(u))
    # step() replay over the first n_step positions
    n_step = min(L, 8)
    with torch.no_grad():
        a, s, bx = m.allocate_inference_cache(batch)
        ys = []
        for t in range(n_step):
            o, a, s, bx = m.step(u[:, t], a, s, bx)
            ys.append(o)
    out["step_y"] = _np(torch.stack(ys, dim=1))
    out["step_angle"] = _np(a)
    out["step_ssm"] = _np(s)
    out["step_bx"] = _np(bx)
    np.savez_compressed(os.path.join(HERE, name), **out)


def gen_lm(name, mcfg, batch, L, n_step, dtype, seed_w, seed_x):
    """MambaLMHeadModel.forward and step (block.py:93-139) at default init."""
    import torch
    from mamba3_ssm.block import MambaLMHeadModel
    from mamba3_ssm.config import MambaConfig
    torch.manual_seed(seed_w)
    m = MambaLMHeadModel(MambaConfig(**mcfg))
    if dtype != torch.float32:
        m = m.to(dtype)
    gen = torch.Generator().manual_seed(seed_x)
    ids = torch.randint(0, mcfg["vocab_size"], (batch, L), generator=gen)
    out = dict(dtype=str(dtype).replace("torch.", ""), ids=ids.numpy().copy())
    out.update(_sd(m))
    for k, v in mcfg.items():
        if k == "ssm_cfg":
            for kk, vv in v.items():
                out["ssm." + kk] = np.asarray(vv)
        else:
            out["cfg." + k] = np.asarray(v)
    with torch.no_grad():
        out["logits"] = _np(m(ids))
        cache = m.allocate_inference_cache(batch)
        lg = []
        for t in range(n_step):
            lo, cache = m.step(ids[:, t], cache)
            lg.append(lo)
    out["step_logits"] = _np(torch.stack(lg, dim=1))
    for i, (a, s, bx) in enumerate(cache):
        out[f"cache{i}.angle"] = _np(a)
        out[f"cache{i}.ssm"] = _np(s)
        out[f"cache{i}.bx"] = _np(bx)
    np.savez_compressed(os.path.join(HERE, name), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default="", help="comma-separated fixture names (without .npz) to write")
    args = ap.parse_args()
    only = set(filter(None, args.only.split(",")))

    def sel(fn):
        def run(name, *a, **k):
            if not only or name[:-4] in only:
                fn(name, *a, **k)
        return run

    g = globals()
    gen_siso_op, gen_mimo_op, gen_layer, gen_lm = (sel(g[n]) for n in ("gen_siso_op", "gen_mimo_op", "gen_layer",
                                                                        "gen_lm"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.ref)
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    import mamba3_ssm  # noqa: F401  (the reference package)
    assert os.path.abspath(mamba3_ssm.__file__).startswith(os.path.abspath(args.ref)), mamba3_ssm.__file__

    f32, bf16 = torch.float32, torch.bfloat16
    # scan ops (ops.py:126-177, 184-242), forward + autograd backward
    gen_siso_op("siso_op_f32.npz", 2, 64, 3, 16, 32, f32, 11)
    gen_siso_op("siso_op_f32_ragged.npz", 1, 37, 2, 32, 16, f32, 12)
    gen_siso_op("siso_op_f32_d128.npz", 1, 24, 2, 64, 128, f32, 13)
    gen_siso_op("siso_op_bf16.npz", 2, 80, 3, 64, 128, bf16, 14)
    gen_siso_op("siso_op_f32_l1.npz", 2, 1, 2, 16, 16, f32, 15)
    gen_mimo_op("mimo_op_f32.npz", 2, 48, 3, 16, 32, 4, f32, 21)
    gen_mimo_op("mimo_op_f32_r2.npz", 1, 33, 2, 32, 64, 2, f32, 22)
    gen_mimo_op("mimo_op_bf16.npz", 2, 64, 2, 32, 64, 4, bf16, 23)
    gen_mimo_op("mimo_op_f32_r1.npz", 1, 20, 2, 16, 16, 1, f32, 24)
    gen_mimo_op("mimo_op_f32_r8.npz", 1, 20, 2, 16, 32, 8, f32, 25)
    # layers
    c1 = dict(d_model=256, d_state=64, expand=2, headdim=32, ngroups=1, rope_fraction=0.5)
    gen_layer("layer_c1_siso_f32.npz", c1, 2, 128, f32, 0, 1234, grad=False)
    small = dict(d_model=128, d_state=32, expand=2, headdim=32)
    gen_layer("layer_siso_f32_grad.npz", small, 2, 16, f32, 7, 1235, grad=True)
    gen_layer("layer_siso_rope1_f32.npz", dict(small, rope_fraction=1.0), 1, 16, f32, 8, 1236, grad=True)
    gen_layer("layer_mimo_f32_grad.npz", dict(small, is_mimo=True, mimo_rank=2), 2, 16, f32, 9, 1237, grad=True)
    c2 = dict(d_model=256, d_state=64, expand=2, headdim=32, is_mimo=True, mimo_rank=4)
    gen_layer("layer_c2_mimo_bf16.npz", c2, 2, 32, bf16, 0, 1238, grad=True)
    gen_layer("layer_siso_bf16.npz", dict(d_model=128, d_state=64, expand=2, headdim=64), 2, 48, bf16, 3, 1239, grad=True)
    # distinct per-head / per-rank / per-column biases, norm weights and D
    gen_layer("layer_siso_f32_params.npz", small, 2, 40, f32, 10, 1243, grad=True, perturb=True)
    gen_layer("layer_mimo_f32_params.npz", dict(small, is_mimo=True, mimo_rank=2, rope_fraction=1.0), 2, 40, f32,
              11, 1244, grad=True, perturb=True)
    # language models
    lm_siso = dict(d_model=64, n_layer=2, vocab_size=300,
                   ssm_cfg=dict(d_state=32, expand=2, headdim=32, is_mimo=False))
    gen_lm("lm_siso_f32.npz", lm_siso, 2, 12, 6, f32, 5, 1240)
    lm_mimo = dict(d_model=64, n_layer=2, vocab_size=293,
                   ssm_cfg=dict(d_state=64, expand=2, headdim=32, is_mimo=True, mimo_rank=4))
    gen_lm("lm_mimo_f32.npz", lm_mimo, 3, 10, 6, f32, 6, 1241)
    gen_lm("lm_mimo_bf16.npz", lm_mimo, 2, 8, 4, bf16, 6, 1242)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
