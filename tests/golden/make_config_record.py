"""Record how close the reference's own outputs are to the float64 oracle at the real
shapes of the five workload configurations, and checksums of its seeded weights.

The GPU parity tests (tests/test_gpu_configs.py) check this build against the float64
oracle at those shapes. In bf16 the reference itself is not exact: its projections and
residual stream round to bf16 at every layer, so a 16- or 20-layer LM drifts from the
float64 result by more than the per-op bar. This script measures that drift on the
reference (CPU, the package imported from a read-only checkout) with the same seeds,
weights and inputs the GPU tests use, and writes ``config_record.json``:

* ``c2_layer``  Mamba3 MIMO layer, bf16, (8, 2048): forward + backward, the reference's
  rel error per tensor (y, du, every parameter gradient) against the oracle's
  ``mamba3_forward_backward``.
* ``c3_lm``     LM forward, SISO preset (d_model 1024, 16 layers, vocab 50000), bf16,
  2 x 512 tokens: rel error of the logits.
* ``c4_decode`` LM decode, MIMO preset (d_model 1536, 20 layers, R=4), bf16, batch 8,
  16-token prefill through ``step`` and 32 greedy steps: per-step rel error of the logits
  (the oracle fed the reference's own tokens) and the fraction of rows whose greedy token
  equals the oracle's argmax.
* ``c5_op``     the raw SISO op at L = 32768, bf16 inputs: forward on 2 (b, h) units and
  backward on 1 unit against the oracle (the reference computes in fp32).
* ``init``      (sum, sum of squares) per parameter of the seed-0 reference modules, so a
  CPU test can confirm that this build's modules draw the same weights.

Usage (build container only; nothing at test time imports the reference)::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_config_record.py [--ref /root/reference] [--only c4]
"""

import argparse
import json
import math
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "config_record.json")

# seeds shared with tests/test_gpu_configs.py
SEED_WEIGHTS = 0
SEED_INPUT = 1234
SEED_GRAD = 1235
C2 = dict(d_model=256, d_state=64, expand=2, headdim=32, is_mimo=True, mimo_rank=4)
C2_SHAPE = (8, 2048)
C3 = dict(d_model=1024, n_layer=16, vocab_size=50000, ssm_cfg=dict(d_state=64, expand=2, headdim=64))
C3_SHAPE = (2, 512)
C4 = dict(d_model=1536, n_layer=20, vocab_size=50000,
          ssm_cfg=dict(d_state=64, expand=2, headdim=64, is_mimo=True, mimo_rank=4))
C4_BATCH, C4_PREFILL, C4_STEPS = 8, 16, 32
C5_L, C5_H = 32768, 64


def rel(a, r):
    a = np.asarray(a, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.max(np.abs(a - r)) / max(float(np.max(np.abs(r))), 1e-300))


def f64(t):
    return t.detach().double().cpu().numpy()


def checksums(module):
    return {k: [float(v.double().sum()), float((v.double() ** 2).sum())] for k, v in module.state_dict().items()}


def c2(torch, ref, O):
    from mamba3_ssm import Mamba3
    torch.manual_seed(SEED_WEIGHTS)
    m = Mamba3(**C2)
    init = checksums(m)
    m = m.to(torch.bfloat16)
    Bn, L = C2_SHAPE
    u = torch.randn(Bn, L, C2["d_model"], generator=torch.Generator().manual_seed(SEED_INPUT)).to(torch.bfloat16)
    dy = torch.randn(Bn, L, C2["d_model"], generator=torch.Generator().manual_seed(SEED_GRAD)).to(torch.bfloat16)
    u.requires_grad_(True)
    t0 = time.time()
    y = m(u)
    y.backward(dy)
    t_ref = time.time() - t0
    w = {k: f64(v) for k, v in m.state_dict().items()}
    dims = O.LayerDims(**C2)
    out, grads = O.mamba3_forward_backward(w, dims, f64(u), f64(dy))
    errs = {"y": rel(f64(y), out), "du": rel(f64(u.grad), grads["u"])}
    for k, p in m.named_parameters():
        errs[k] = rel(f64(p.grad), grads[k])
    return {"shape": list(C2_SHAPE), "config": C2, "ref_vs_oracle": errs, "ref_seconds": t_ref}, init


def c3(torch, ref, O):
    from mamba3_ssm import MambaConfig, MambaLMHeadModel
    torch.manual_seed(SEED_WEIGHTS)
    m = MambaLMHeadModel(MambaConfig(**C3))
    init = checksums(m)
    m = m.to(torch.bfloat16).eval()
    Bn, L = C3_SHAPE
    ids = torch.randint(0, C3["vocab_size"], (Bn, L), generator=torch.Generator().manual_seed(SEED_INPUT))
    with torch.no_grad():
        lg = m(ids)
    w = {k: f64(v) for k, v in m.state_dict().items()}
    dims = O.LayerDims(d_model=C3["d_model"], **C3["ssm_cfg"])
    lo = O.lm_forward(w, dims, C3["n_layer"], ids.numpy())
    return {"shape": list(C3_SHAPE), "config": C3, "ref_vs_oracle": {"logits": rel(f64(lg), lo)}}, init


def c4(torch, ref, O):
    from mamba3_ssm import MambaConfig, MambaLMHeadModel
    torch.manual_seed(SEED_WEIGHTS)
    m = MambaLMHeadModel(MambaConfig(**C4))
    init = checksums(m)
    m = m.to(torch.bfloat16).eval()
    V = C4["vocab_size"]
    ids = torch.randint(0, V, (C4_BATCH, C4_PREFILL), generator=torch.Generator().manual_seed(SEED_INPUT))
    w = {k: f64(v) for k, v in m.state_dict().items()}
    dims = O.LayerDims(d_model=C4["d_model"], **C4["ssm_cfg"])
    n_layer = C4["n_layer"]
    cache = m.allocate_inference_cache(C4_BATCH)
    oc = [O.allocate_inference_cache(dims, C4_BATCH) for _ in range(n_layer)]
    errs, agree = [], []
    tok = None
    with torch.no_grad():
        for t in range(C4_PREFILL + C4_STEPS):
            inp = ids[:, t] if t < C4_PREFILL else tok
            lg, cache = m.step(inp, cache)
            lo, oc = O.lm_step(w, dims, n_layer, inp.numpy(), oc)
            lgf = f64(lg.float())
            errs.append(rel(lgf, lo))
            tok = lg.float().argmax(-1)
            agree.append(float((tok.numpy() == lo.argmax(-1)).mean()))
    return {"batch": C4_BATCH, "prefill": C4_PREFILL, "steps": C4_STEPS, "config": C4,
            "ref_vs_oracle": {"step_logits_max": max(errs), "per_step": errs},
            "greedy_agreement_min": min(agree), "greedy_agreement_mean": float(np.mean(agree))}, init


def c5(torch, ref, O):
    """The raw op at full length on a few (b, h) units: the reference's CPU loop with bf16
    inputs (it computes in fp32) against the fp64 oracle."""
    import torch.nn.functional as F
    from mamba3_ssm.ops import apply_rope, ssm_scan_siso
    g = torch.Generator().manual_seed(SEED_INPUT)
    L, H, P, D = C5_L, 2, 64, 128
    x = torch.randn(1, L, H, P, generator=g)
    Bm = torch.randn(1, L, H, D, generator=g)
    Cm = torch.randn(1, L, H, D, generator=g)
    dt = F.softplus(torch.randn(1, L, H, generator=g) * 0.5 - 3.0).clamp(1e-3, 0.1)
    A = -torch.exp(torch.rand(H, generator=g) * math.log(16.0))
    trap = torch.sigmoid(torch.randn(1, L, H, generator=g))
    Dw = torch.randn(H, generator=g) * 0.5 + 1.0
    S = D // 4
    theta = 10000.0 ** (-2.0 * torch.arange(S, dtype=torch.float32) / D)
    ang = torch.cumsum(dt, dim=1).unsqueeze(-1) * theta
    Bm = torch.cat([apply_rope(Bm[..., :2 * S], ang), Bm[..., 2 * S:]], -1)
    Cm = torch.cat([apply_rope(Cm[..., :2 * S], ang), Cm[..., 2 * S:]], -1)
    x, Bm, Cm = (t.to(torch.bfloat16) for t in (x, Bm, Cm))
    ADT = A * dt
    with torch.no_grad():
        y = ssm_scan_siso(x, Bm, Cm, ADT, dt, trap, Dw)
    args = [f64(t) for t in (x, Bm, Cm, ADT, dt, trap, Dw)]
    yo, _, _ = O.siso_scan_fwd(*args)
    fwd = rel(f64(y.float()), yo)
    # backward on the first unit
    sl = [t[:, :, :1] if t.dim() >= 3 else t[:1] for t in (x, Bm, Cm, ADT, dt, trap)] + [Dw[:1]]
    leaves = [t.detach().clone().requires_grad_(True) for t in sl]
    dy = torch.randn(1, L, 1, P, generator=g).to(torch.bfloat16)
    yb = ssm_scan_siso(*leaves)
    yb.backward(dy)
    go = O.siso_scan_bwd_segmented(*[f64(t) for t in leaves], f64(dy))
    bwd = {k: rel(f64(t.grad), go[k]) for k, t in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), leaves)}
    return {"L": L, "ref_vs_oracle": {"y": fwd, **bwd}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    sys.path.insert(0, ROOT)
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    import mamba3_ssm as ref
    from oracle import scan_oracle as O
    rec = {}
    if os.path.exists(OUT):
        with open(OUT) as f:
            rec = json.load(f)
    rec.setdefault("init", {})
    for name, fn in (("c2_layer", c2), ("c3_lm", c3), ("c4_decode", c4), ("c5_op", c5)):
        if a.only and a.only not in name:
            continue
        t0 = time.time()
        r = fn(torch, ref, O)
        if isinstance(r, tuple):
            r, init = r
            rec["init"][name] = init
        r["generator_seconds"] = round(time.time() - t0, 1)
        rec[name] = r
        print(name, json.dumps(r.get("ref_vs_oracle")), flush=True)
        with open(OUT, "w") as f:
            json.dump(rec, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
