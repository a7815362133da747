"""Pin the float64 oracle against fixtures recorded from the reference itself.

The fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py) hold the
reference's own CPU outputs: its scan loops (ops.py:160-177, 221-242), autograd through
them, Mamba3.forward/step (layer.py) and MambaLMHeadModel.forward/step (block.py).
fp32 fixtures must agree with the fp64 oracle to fp32 rounding (rel 1e-5); bf16
fixtures, which carry bf16 roundings of intermediates, to rel 2e-2.
"""

import numpy as np
import pytest

from conftest import load_golden, rel_err
from oracle import scan_oracle as O

SISO_OPS = ["siso_op_f32", "siso_op_f32_ragged", "siso_op_f32_d128", "siso_op_bf16", "siso_op_f32_l1"]
MIMO_OPS = ["mimo_op_f32", "mimo_op_f32_r2", "mimo_op_bf16", "mimo_op_f32_r1", "mimo_op_f32_r8"]


def _tol(g):
    return 2e-2 if str(g["dtype"]) == "bfloat16" else 1e-5


@pytest.mark.parametrize("name", SISO_OPS)
def test_siso_scan_oracle_matches_reference(name):
    g = load_golden(name)
    args = [g[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")]
    y, _, _ = O.siso_scan_fwd(*args)
    assert rel_err(y, g["y"]) < _tol(g)
    grads = O.siso_scan_bwd(*args, g["dy"])
    for k in ("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"):
        assert rel_err(grads[k], g[k]) < _tol(g), k


@pytest.mark.parametrize("name", MIMO_OPS)
def test_mimo_scan_oracle_matches_reference(name):
    g = load_golden(name)
    args = [g[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")]
    y, _, _ = O.mimo_scan_fwd(*args)
    assert rel_err(y, g["y"]) < _tol(g)
    grads = O.mimo_scan_bwd(*args, g["dy"])
    for k in ("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD", "dmimo_x", "dmimo_o"):
        assert rel_err(grads[k], g[k]) < _tol(g), k


def _weights(g):
    return {k[2:]: v for k, v in g.items() if k.startswith("w.")}


def _cfg(g, prefix):
    out = {}
    for k, v in g.items():
        if k.startswith(prefix):
            out[k[len(prefix):]] = v.item()
    return out


@pytest.mark.parametrize("name", ["layer_c1_siso_f32", "layer_siso_f32_grad", "layer_siso_rope1_f32",
                                  "layer_mimo_f32_grad", "layer_c2_mimo_bf16", "layer_siso_bf16",
                                  "layer_siso_f32_params", "layer_mimo_f32_params"])
def test_layer_oracle_matches_reference(name):
    g = load_golden(name)
    dims = O.LayerDims(**_cfg(g, "cfg."))
    w = _weights(g)
    y = O.mamba3_forward(w, dims, g["u"])
    tol = 2e-2 if str(g["dtype"]) == "bfloat16" else 1e-5
    assert rel_err(y, g["y"]) < tol
    n = g["step_y"].shape[1]
    a, s, b = O.allocate_inference_cache(dims, g["u"].shape[0])
    ys = []
    for t in range(n):
        o, a, s, b = O.mamba3_step(w, dims, g["u"][:, t], a, s, b)
        ys.append(o)
    assert rel_err(np.stack(ys, 1), g["step_y"]) < tol
    assert rel_err(s, g["step_ssm"]) < tol
    assert rel_err(b, g["step_bx"]) < tol
    assert rel_err(a, g["step_angle"]) < tol
    # the reference's own invariant (tests.py:67-108): step replay == forward
    assert rel_err(np.stack(ys, 1), y[:, :n]) < max(tol, 1e-6)


@pytest.mark.parametrize("name", ["lm_siso_f32", "lm_mimo_f32", "lm_mimo_bf16"])
def test_lm_oracle_matches_reference(name):
    g = load_golden(name)
    dims = O.LayerDims(d_model=int(g["cfg.d_model"]), **_cfg(g, "ssm."))
    n_layer = int(g["cfg.n_layer"])
    w = _weights(g)
    tol = 2e-2 if str(g["dtype"]) == "bfloat16" else 1e-5
    assert rel_err(O.lm_forward(w, dims, n_layer, g["ids"]), g["logits"]) < tol
    cache = [O.allocate_inference_cache(dims, g["ids"].shape[0]) for _ in range(n_layer)]
    lg = []
    for t in range(g["step_logits"].shape[1]):
        lo, cache = O.lm_step(w, dims, n_layer, g["ids"][:, t], cache)
        lg.append(lo)
    assert rel_err(np.stack(lg, 1), g["step_logits"]) < tol
    for i, (a, s, b) in enumerate(cache):
        assert rel_err(s, g[f"cache{i}.ssm"]) < tol


def test_a_floor_clamp_is_constant():
    """layer.py:207: -(softplus(v).clamp(max=-A_floor)) is +A_floor for every v."""
    v = np.linspace(-30, 30, 101)
    A = -np.minimum(O.softplus(v), -1e-4)
    assert np.all(A == 1e-4)


def test_oracle_bwd_matches_finite_difference():
    """Independent check of the hand adjoint on a tiny case (central differences)."""
    rng = np.random.default_rng(0)
    Bn, L, H, P, D = 1, 5, 2, 3, 4
    x = rng.standard_normal((Bn, L, H, P)); Bm = rng.standard_normal((Bn, L, H, D))
    C = rng.standard_normal((Bn, L, H, D)); ADT = -rng.uniform(0.01, 1, (Bn, L, H))
    DT = rng.uniform(0.01, 0.1, (Bn, L, H)); trap = rng.standard_normal((Bn, L, H))
    Dw = rng.standard_normal(H); dy = rng.standard_normal((Bn, L, H, P))
    args = dict(x=x, B=Bm, C=C, ADT=ADT, DT=DT, trap=trap, D=Dw)
    grads = O.siso_scan_bwd(*args.values(), dy)

    def loss(**kw):
        y, _, _ = O.siso_scan_fwd(**kw)
        return float(np.sum(y * dy))

    for k, gk in (("x", "dx"), ("B", "dB"), ("ADT", "dADT"), ("DT", "dDT"), ("trap", "dtrap")):
        base = args[k]
        fd = np.zeros_like(base)
        it = np.nditer(base, flags=["multi_index"])
        for _ in it:
            i = it.multi_index
            e = 1e-6
            p = base.copy(); p[i] += e
            m = base.copy(); m[i] -= e
            fd[i] = (loss(**{**args, k: p}) - loss(**{**args, k: m})) / (2 * e)
        assert rel_err(grads[gk], fd) < 1e-6, k


@pytest.mark.parametrize("name", ["siso_op_f32", "siso_op_f32_ragged", "siso_op_f32_d128", "siso_op_f32_l1",
                                  "siso_op_bf16"])
def test_c_restatement_matches_reference(name):
    """oracle/scan_ref.c (the CPU baseline) against the reference's own outputs."""
    from oracle import cpu_ref
    g = load_golden(name)
    y = cpu_ref.siso_fwd(*[g[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")])
    assert rel_err(y, g["y"]) < (2e-2 if str(g["dtype"]) == "bfloat16" else 1e-5)


@pytest.mark.parametrize("name", ["layer_siso_f32_grad", "layer_mimo_f32_grad", "layer_c2_mimo_bf16",
                                  "layer_siso_f32_params", "layer_mimo_f32_params"])
def test_layer_adjoint_matches_reference(name):
    """The oracle's layer adjoint (mamba3_forward_backward) against the gradients autograd
    returned through the reference's Mamba3.forward (fixtures recorded from the reference)."""
    g = load_golden(name)
    dims = O.LayerDims(**_cfg(g, "cfg."))
    w = _weights(g)
    out, grads = O.mamba3_forward_backward(w, dims, g["u"], g["dy"])
    bf = str(g["dtype"]) == "bfloat16"
    tol = 2e-2 if bf else 1e-5
    assert rel_err(out, g["y"]) < tol
    assert rel_err(grads["u"], g["du"]) < tol
    for k in w:
        if ("g." + k) in g:
            assert grads[k].shape == g["g." + k].shape, k
            assert rel_err(grads[k], g["g." + k]) < tol, k


def test_segmented_adjoint_equals_full_adjoint():
    """siso_scan_bwd_segmented (checkpointed, bounded memory) gives the adjoint of
    siso_scan_bwd on a ragged length with initial states."""
    rng = np.random.default_rng(3)
    Bn, L, H, P, D = 2, 37, 2, 4, 6
    x = rng.standard_normal((Bn, L, H, P)); Bm = rng.standard_normal((Bn, L, H, D))
    C = rng.standard_normal((Bn, L, H, D)); ADT = -rng.uniform(0.01, 1, (Bn, L, H))
    DT = rng.uniform(0.01, 0.1, (Bn, L, H)); trap = rng.standard_normal((Bn, L, H))
    Dw = rng.standard_normal(H); dy = rng.standard_normal((Bn, L, H, P))
    h0 = rng.standard_normal((Bn, H, P, D)); b0 = rng.standard_normal((Bn, H, P, D))
    full = O.siso_scan_bwd(x, Bm, C, ADT, DT, trap, Dw, dy, h0, b0)
    seg = O.siso_scan_bwd_segmented(x, Bm, C, ADT, DT, trap, Dw, dy, h0, b0, seg=8)
    for k in full:
        assert np.array_equal(full[k], seg[k]), k
