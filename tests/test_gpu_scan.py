"""Parity of the CUDA scan kernels (through the drop-in ops and the C ABI) with the
reference's own outputs (golden fixtures) and with the float64 oracle.

Tolerances (max|a - ref| / max|ref| per tensor): rel 1e-4 for fp32 I/O, rel 2e-2 for bf16
I/O, the bars of the parity target, for every output and every gradient.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import scan_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_kernel_timeouts():
    """Every bounded inter-warp wait of the warp-specialised kernels completed."""
    yield
    from mamba3_ssm import _lib as L
    assert L.device_timeouts(reset=True) == 0


def _t(g, k, dtype=None):
    a = torch.from_numpy(np.ascontiguousarray(g[k]))
    if dtype is None:
        dtype = torch.bfloat16 if k in g["bf16"] else torch.float32
    return a.to(dtype).to(DEV)


def _tol(dtype):
    return 2e-2 if dtype == torch.bfloat16 else 1e-4


SISO = ["siso_op_f32", "siso_op_f32_ragged", "siso_op_f32_d128", "siso_op_bf16", "siso_op_f32_l1"]
MIMO = ["mimo_op_f32", "mimo_op_f32_r2", "mimo_op_bf16", "mimo_op_f32_r1", "mimo_op_f32_r8"]


@pytest.mark.parametrize("name", SISO)
def test_siso_fwd_bwd_matches_reference(name):
    from mamba3_ssm import ssm_scan_siso
    g = load_golden(name)
    ins = [_t(g, k).requires_grad_(True) for k in ("x", "B", "C", "ADT", "DT", "trap", "D")]
    y = ssm_scan_siso(*ins)
    tol = _tol(ins[0].dtype)
    assert y.dtype == ins[0].dtype and y.shape == ins[0].shape
    assert rel_err(y.detach().float().cpu().numpy(), g["y"]) < tol
    y.backward(_t(g, "dy"))
    for k, t in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), ins):
        assert t.grad.dtype == t.dtype
        assert rel_err(t.grad.detach().float().cpu().numpy(), g[k]) < tol, k


@pytest.mark.parametrize("name", MIMO)
def test_mimo_fwd_bwd_matches_reference(name):
    from mamba3_ssm import ssm_scan_mimo
    g = load_golden(name)
    ins = [_t(g, k).requires_grad_(True) for k in ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")]
    y = ssm_scan_mimo(*ins)
    tol = _tol(ins[0].dtype)
    assert rel_err(y.detach().float().cpu().numpy(), g["y"]) < tol
    y.backward(_t(g, "dy"))
    for k, t in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD", "dmimo_x", "dmimo_o"), ins):
        assert rel_err(t.grad.detach().float().cpu().numpy(), g[k]) < tol, k


def _inputs(seed, Bn, L, H, P, D, R=None, dtype=torch.float32):
    rng = np.random.default_rng(seed)
    bc = (Bn, L, H, D) if R is None else (Bn, L, R, H, D)
    x = rng.standard_normal((Bn, L, H, P))
    Bm = rng.standard_normal(bc)
    C = rng.standard_normal(bc)
    dt = np.clip(np.log1p(np.exp(rng.normal(-3, 0.5, (Bn, L, H)))), 1e-3, 0.1)
    A = -np.exp(rng.uniform(0, np.log(16), H))
    ADT = A * dt
    trap = 1 / (1 + np.exp(-rng.standard_normal((Bn, L, H))))
    Dw = rng.standard_normal(H) * 0.5 + 1.0
    arrs = dict(x=x, B=Bm, C=C, ADT=ADT, DT=dt, trap=trap, D=Dw)
    if R is not None:
        arrs["mimo_x"] = rng.standard_normal((H, R, P)) * 0.3 + 1.0 / R
        arrs["mimo_o"] = rng.standard_normal((H, R, P)) * 0.3 + 1.0 / R
    tens = {}
    for k, v in arrs.items():
        dt_ = dtype if k in ("x", "B", "C") else torch.float32
        tens[k] = torch.tensor(v, dtype=torch.float32).to(dt_).to(DEV)
        arrs[k] = tens[k].detach().double().cpu().numpy()  # oracle sees the rounded values
    return arrs, tens


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("P,L", [(16, 33), (64, 70), (128, 40)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_siso_sweep_against_oracle(D, P, L, dtype):
    from mamba3_ssm import ssm_scan_siso
    arrs, t = _inputs(D * 1000 + P + L, 2, L, 3, P, D, dtype=dtype)
    ins = [t[k].requires_grad_(True) for k in ("x", "B", "C", "ADT", "DT", "trap", "D")]
    y = ssm_scan_siso(*ins)
    yo, _, _ = O.siso_scan_fwd(*[arrs[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")])
    tol = _tol(dtype)
    assert rel_err(y.detach().double().cpu().numpy(), yo) < tol
    dy = torch.randn_like(y)
    y.backward(dy)
    go = O.siso_scan_bwd(*[arrs[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")], dy.detach().double().cpu().numpy())
    for k, tt in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), ins):
        assert rel_err(tt.grad.detach().double().cpu().numpy(), go[k]) < tol, k


@pytest.mark.parametrize("R,D,P", [(1, 16, 16), (2, 32, 64), (4, 64, 32), (8, 128, 64), (4, 64, 64)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mimo_sweep_against_oracle(R, D, P, dtype):
    from mamba3_ssm import ssm_scan_mimo
    arrs, t = _inputs(R * 100 + D + P, 2, 77, 3, P, D, R=R, dtype=dtype)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")
    ins = [t[k].requires_grad_(True) for k in keys]
    y = ssm_scan_mimo(*ins)
    yo, _, _ = O.mimo_scan_fwd(*[arrs[k] for k in keys])
    tol = _tol(dtype)
    assert rel_err(y.detach().double().cpu().numpy(), yo) < tol
    dy = torch.randn_like(y)
    y.backward(dy)
    go = O.mimo_scan_bwd(*[arrs[k] for k in keys], dy.detach().double().cpu().numpy())
    for k, tt in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD", "dmimo_x", "dmimo_o"), ins):
        assert rel_err(tt.grad.detach().double().cpu().numpy(), go[k]) < tol, k


def test_siso_strided_views_and_state_continuation():
    """B/C as (B, L, R, H, D)[:, :, 0] views (layer.py:256-257) and a scan split in two
    halves with the carried (ssm_state, bx_prev) equal one full scan."""
    from mamba3_ssm import ssm_scan_siso
    from mamba3_ssm.ops import ssm_scan_siso_states
    arrs, t = _inputs(7, 2, 96, 4, 32, 64)
    B5 = torch.randn(2, 96, 2, 4, 64, device=DEV)
    C5 = torch.randn(2, 96, 2, 4, 64, device=DEV)
    y = ssm_scan_siso(t["x"], B5[:, :, 0], C5[:, :, 0], t["ADT"], t["DT"], t["trap"], t["D"])
    yo, ho, bo = O.siso_scan_fwd(arrs["x"], B5[:, :, 0].detach().double().cpu().numpy(), C5[:, :, 0].detach().double().cpu().numpy(),
                                 arrs["ADT"], arrs["DT"], arrs["trap"], arrs["D"])
    assert rel_err(y.detach().double().cpu().numpy(), yo) < 1e-4
    Bc, Cc = B5[:, :, 0].contiguous(), C5[:, :, 0].contiguous()
    a = slice(0, 41)
    b = slice(41, 96)
    y1, h1, b1 = ssm_scan_siso_states(t["x"][:, a], Bc[:, a], Cc[:, a], t["ADT"][:, a], t["DT"][:, a],
                                      t["trap"][:, a], t["D"])
    y2, h2, b2 = ssm_scan_siso_states(t["x"][:, b], Bc[:, b], Cc[:, b], t["ADT"][:, b], t["DT"][:, b],
                                      t["trap"][:, b], t["D"], h1, b1)
    assert rel_err(torch.cat([y1, y2], 1).detach().double().cpu().numpy(), yo) < 1e-4
    assert rel_err(h2.detach().double().cpu().numpy(), ho) < 1e-4
    assert rel_err(b2.detach().double().cpu().numpy(), bo) < 1e-4


def test_empty_and_single_token_inputs():
    from mamba3_ssm import ssm_scan_siso, ssm_scan_mimo
    for L in (0, 1):
        arrs, t = _inputs(3, 2, L, 2, 16, 32)
        y = ssm_scan_siso(*[t[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")])
        assert y.shape == (2, L, 2, 16)
        if L:
            yo, _, _ = O.siso_scan_fwd(*[arrs[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")])
            assert rel_err(y.detach().double().cpu().numpy(), yo) < 1e-4
        arrs, t = _inputs(4, 2, L, 2, 16, 32, R=2)
        y = ssm_scan_mimo(*[t[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")])
        assert y.shape == (2, L, 2, 16)
    x = torch.zeros(0, 5, 2, 16, device=DEV)
    B = torch.zeros(0, 5, 2, 32, device=DEV)
    s = torch.zeros(0, 5, 2, device=DEV)
    assert ssm_scan_siso(x, B, B, s, s, s, torch.ones(2, device=DEV)).shape == (0, 5, 2, 16)


def test_long_sequence_slices_against_oracle():
    """Long-context shape per (b, h) (H=2 of the 64 heads, full L = 32768, P=64, D=128,
    bf16 I/O) against the float64 oracle."""
    from mamba3_ssm import ssm_scan_siso
    arrs, t = _inputs(11, 1, 32768, 2, 64, 128, dtype=torch.bfloat16)
    y = ssm_scan_siso(*[t[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")])
    yo, _, _ = O.siso_scan_fwd(*[arrs[k] for k in ("x", "B", "C", "ADT", "DT", "trap", "D")])
    assert rel_err(y.detach().double().cpu().numpy(), yo) < 2e-2


@pytest.mark.parametrize("Ds", [128, 64])
@pytest.mark.parametrize("L", [1, 77, 128, 129, 300, 1000])
def test_siso_bf16_headdim64_dstate128_against_oracle(L, Ds):
    """The shape class of the chunked tensor-core kernel (bf16, P=64, d_state 128 or 64) on
    ragged lengths, with and without carried decode states."""
    from mamba3_ssm import ssm_scan_siso
    from mamba3_ssm.ops import ssm_scan_siso_states
    arrs, t = _inputs(100 + L + Ds, 2, L, 3, 64, Ds, dtype=torch.bfloat16)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    y = ssm_scan_siso(*[t[k] for k in keys])
    yo, ho, bo = O.siso_scan_fwd(*[arrs[k] for k in keys])
    assert rel_err(y.detach().double().cpu().numpy(), yo) < 2e-2
    rng = np.random.default_rng(L)
    h0 = torch.tensor(rng.standard_normal((2, 3, 64, Ds)), dtype=torch.float32, device=DEV)
    b0 = torch.tensor(rng.standard_normal((2, 3, 64, Ds)), dtype=torch.float32, device=DEV)
    y2, h2, b2 = ssm_scan_siso_states(*[t[k] for k in keys], h0, b0)
    yo2, ho2, bo2 = O.siso_scan_fwd(*[arrs[k] for k in keys], h0.double().cpu().numpy(), b0.double().cpu().numpy())
    assert rel_err(y2.detach().double().cpu().numpy(), yo2) < 2e-2
    assert rel_err(h2.detach().double().cpu().numpy(), ho2) < 2e-2
    assert rel_err(b2.detach().double().cpu().numpy(), bo2) < 2e-2


@pytest.mark.parametrize("L", [100, 128, 200])
def test_siso_bf16_chunked_final_states_many_units(L):
    """More (b, h) units than SMs with one or two chunks each, so that one CTA closes a unit
    on consecutive chunks: the final states h_last and bx_last = x_{L-1} B_{L-1}^T of every
    unit against the oracle (tensor-core path, bf16, P=64, d_state 128)."""
    from mamba3_ssm.ops import ssm_scan_siso_states
    arrs, t = _inputs(900 + L, 64, L, 4, 64, 128, dtype=torch.bfloat16)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    y, h, bx = ssm_scan_siso_states(*[t[k] for k in keys])
    yo, ho, bo = O.siso_scan_fwd(*[arrs[k] for k in keys])
    assert rel_err(y.double().cpu().numpy(), yo) < 2e-2
    assert rel_err(h.double().cpu().numpy(), ho) < 2e-2
    # bx_last is a product of two bf16 inputs, exact in fp32
    assert rel_err(bx.double().cpu().numpy(), bo) < 1e-6


@pytest.mark.parametrize("case", ["strong_decay", "mixed_sign"])
def test_siso_bf16_chunked_exact_mask_path(case):
    """Decays outside the split-exponent range of the chunked kernel: strong per-step decay
    (ADT down to -13, so 32-step column factors leave fp32) and isolated growth steps
    (ADT up to +0.7). Those mask blocks take the per-element path; results must still
    match the oracle."""
    from mamba3_ssm import ssm_scan_siso
    arrs, t = _inputs(7 if case == "strong_decay" else 8, 2, 700, 3, 64, 128, dtype=torch.bfloat16)
    rng = np.random.default_rng(99)
    if case == "strong_decay":
        adt = -rng.uniform(0.0, 13.0, arrs["ADT"].shape)
    else:
        adt = -rng.uniform(0.0, 3.0, arrs["ADT"].shape)
        grow = rng.random(adt.shape) < 0.05
        adt[grow] = rng.uniform(0.0, 0.7, grow.sum())
    t["ADT"] = torch.tensor(adt, dtype=torch.float32, device=DEV)
    arrs["ADT"] = t["ADT"].double().cpu().numpy()
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    y = ssm_scan_siso(*[t[k] for k in keys])
    yo, _, _ = O.siso_scan_fwd(*[arrs[k] for k in keys])
    assert np.isfinite(y.float().cpu().numpy()).all()
    assert rel_err(y.detach().double().cpu().numpy(), yo) < 2e-2


@pytest.mark.parametrize("L", [1, 15, 16, 17, 33, 63, 64, 65, 300, 2500])
@pytest.mark.parametrize("R,D,P", [(4, 64, 32), (8, 256, 16), (2, 16, 8)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mimo_chunked_forward_with_states(L, R, D, P, dtype):
    """The single-pass MIMO forward (16 / 32 / 64-step chunks by shared-memory size, carries
    found by looking back over earlier chunks) on chunk-boundary lengths and a long
    sequence of many chunks, with carried-in states h0 / bx0 and the returned h_last /
    bx_last, against the fp64 oracle; no bounded wait may give up."""
    from mamba3_ssm import _lib
    from mamba3_ssm.ops import _MimoScanFn
    arrs, t = _inputs(1000 + L + D, 2, L, 3, P, D, R=R, dtype=dtype)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")
    rng = np.random.default_rng(L + 7)
    h0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV)
    b0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV)
    _lib.device_timeouts(reset=True)
    y, hl, bl = _MimoScanFn.apply(*[t[k] for k in keys], h0, b0, True)
    yo, ho, bo = O.mimo_scan_fwd(*[arrs[k] for k in keys], h0.double().cpu().numpy(), b0.double().cpu().numpy())
    tol = _tol(dtype)
    assert rel_err(y.detach().double().cpu().numpy(), yo) < tol
    assert rel_err(hl.double().cpu().numpy(), ho) < 1e-4
    assert rel_err(bl.double().cpu().numpy(), bo) < 1e-4
    assert _lib.device_timeouts(reset=True) == 0


@pytest.mark.parametrize("L", [65, 300])
def test_mimo_forward_unaligned_rows_three_pass(L):
    """B / C whose rows do not start on 16-byte boundaries (a view of a wider d axis) take
    the three-pass forward (local states, carry pass, outputs); same results."""
    from mamba3_ssm.ops import _MimoScanFn
    R, D, P = 4, 64, 32
    arrs, t = _inputs(3000 + L, 2, L, 3, P, D, R=R, dtype=torch.float32)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")
    for k in ("B", "C"):
        wide = torch.zeros(*t[k].shape[:-1], D + 1, dtype=t[k].dtype, device=DEV)
        wide[..., :D] = t[k]
        t[k] = wide[..., :D]
        assert (t[k].stride(3) * 4) % 16 != 0
    rng = np.random.default_rng(L + 9)
    h0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV)
    b0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV)
    y, hl, bl = _MimoScanFn.apply(*[t[k] for k in keys], h0, b0, True)
    yo, ho, bo = O.mimo_scan_fwd(*[arrs[k] for k in keys], h0.double().cpu().numpy(), b0.double().cpu().numpy())
    assert rel_err(y.detach().double().cpu().numpy(), yo) < 1e-4
    assert rel_err(hl.double().cpu().numpy(), ho) < 1e-4
    assert rel_err(bl.double().cpu().numpy(), bo) < 1e-4


@pytest.mark.parametrize("L", [1, 15, 16, 17, 31, 32, 33, 200, 1500])
@pytest.mark.parametrize("R,D,P", [(4, 64, 32), (2, 128, 64), (2, 16, 8)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mimo_chunked_backward_with_states(L, R, D, P, dtype):
    """The single-pass MIMO backward (the forward's chunk-end states, adjoint carries found
    by looking ahead over later chunks, per-chunk gradients, cross-chunk dADT suffix sums)
    on chunk-boundary lengths and a long sequence, with initial states, against the fp64
    adjoint of the oracle (all gradients incl. dh0 / dbx0); no bounded wait may give up."""
    from mamba3_ssm import _lib
    from mamba3_ssm.ops import _MimoScanFn
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    arrs, t = _inputs(2000 + L + D, 2, L, 3, P, D, R=R, dtype=dtype)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")
    rng = np.random.default_rng(L + 11)
    h0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV).requires_grad_(True)
    b0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV).requires_grad_(True)
    ins = [t[k].requires_grad_(True) for k in keys]
    _lib.device_timeouts(reset=True)
    y, _, _ = _MimoScanFn.apply(*ins, h0, b0, False)
    dy = torch.randn_like(y)
    y.backward(dy)
    go = O.mimo_scan_bwd(*[arrs[k] for k in keys], dy.double().cpu().numpy(),
                         h0.detach().double().cpu().numpy(), b0.detach().double().cpu().numpy())
    for k, tt in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD", "dmimo_x", "dmimo_o"), ins):
        assert rel_err(tt.grad.double().cpu().numpy(), go[k]) < tol, k
    assert rel_err(h0.grad.double().cpu().numpy(), go["dh0"]) < tol
    assert rel_err(b0.grad.double().cpu().numpy(), go["dbx0"]) < tol
    assert _lib.device_timeouts(reset=True) == 0


@pytest.mark.parametrize("L", [33, 300])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mimo_backward_without_forward_workspace(L, dtype):
    """m3_mimo_scan_bwd (no forward workspace: the chunk-parallel kernels that recompute the
    forward) and m3_mimo_scan_bwd_ws (the single-pass backward) on the same inputs, both
    against the oracle's adjoint."""
    from mamba3_ssm.ops import _mimo_bwd_raw, _mimo_fwd_raw
    R, D, P = 4, 64, 32
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    arrs, t = _inputs(4000 + L, 2, L, 3, P, D, R=R, dtype=dtype)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D", "mimo_x", "mimo_o")
    rng = np.random.default_rng(L + 13)
    h0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV)
    b0 = torch.tensor(rng.standard_normal((2, 3, D)), dtype=torch.float32, device=DEV)
    ins = [t[k] for k in keys]
    _, _, _, fws = _mimo_fwd_raw(*ins, h0, b0, keep_ws=True)
    dy = torch.randn(2, L, 3, P, device=DEV).to(dtype)
    go = O.mimo_scan_bwd(*[arrs[k] for k in keys], dy.double().cpu().numpy(), h0.double().cpu().numpy(),
                         b0.double().cpu().numpy())
    names = ("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD", "dmimo_x", "dmimo_o", "dh0", "dbx0")
    for fw in (None, fws):
        g = _mimo_bwd_raw(*ins, h0, b0, dy, True, True, fwd_ws=fw)
        for k, v in zip(names, g):
            assert rel_err(v.double().cpu().numpy(), go[k]) < tol, (k, fw is None)


def _siso_grads(ins, h0=None, b0=None):
    from mamba3_ssm import ssm_scan_siso
    from mamba3_ssm.ops import ssm_scan_siso_states
    if h0 is None:
        y = ssm_scan_siso(*ins)
    else:
        y, _, _ = ssm_scan_siso_states(*ins, h0, b0)
    torch.manual_seed(1)
    dy = torch.randn_like(y)
    y.backward(dy)
    return y, dy


@pytest.mark.parametrize("Ds", [128, 64])
@pytest.mark.parametrize("L", [1, 77, 128, 129, 300, 700])
@pytest.mark.parametrize("states", [False, True])
def test_siso_bf16_chunked_backward_against_oracle(L, states, Ds):
    """The chunked tensor-core backward (bf16, headdim 64, d_state 128 or 64; the forward
    keeps its chunk-start states for it) on ragged lengths, with and without initial states,
    against the float64 adjoint of the loop."""
    Bn = 2 if L <= 300 else 1
    arrs, t = _inputs(500 + L + Ds, Bn, L, 2, 64, Ds, dtype=torch.bfloat16)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    ins = [t[k].requires_grad_(True) for k in keys]
    h0 = b0 = None
    if states:
        rng = np.random.default_rng(L)
        h0 = torch.tensor(rng.standard_normal((Bn, 2, 64, Ds)), dtype=torch.float32, device=DEV).requires_grad_(True)
        b0 = torch.tensor(rng.standard_normal((Bn, 2, 64, Ds)), dtype=torch.float32, device=DEV).requires_grad_(True)
    y, dy = _siso_grads(ins, h0, b0)
    npy = lambda v: None if v is None else v.detach().double().cpu().numpy()
    go = O.siso_scan_bwd(*[arrs[k] for k in keys], npy(dy), npy(h0), npy(b0))
    for k, tt in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), ins):
        assert rel_err(npy(tt.grad), go[k]) < 2e-2, k
    if states:
        assert rel_err(npy(h0.grad), go["dh0"]) < 2e-2
        assert rel_err(npy(b0.grad), go["dbx0"]) < 2e-2


@pytest.mark.parametrize("L,Ds", [(100, 128), (160, 64)])
def test_siso_bf16_chunked_backward_many_units(L, Ds):
    """The chunked backward with more (b, h) units than SMs (152 > 148) and one or two
    chunks per unit, so that a CTA moves from unit to unit on consecutive chunks, with
    initial states."""
    Bn, H = 38, 4
    arrs, t = _inputs(700 + L, Bn, L, H, 64, Ds, dtype=torch.bfloat16)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    ins = [t[k].requires_grad_(True) for k in keys]
    rng = np.random.default_rng(L + 1)
    h0 = torch.tensor(rng.standard_normal((Bn, H, 64, Ds)), dtype=torch.float32, device=DEV).requires_grad_(True)
    b0 = torch.tensor(rng.standard_normal((Bn, H, 64, Ds)), dtype=torch.float32, device=DEV).requires_grad_(True)
    y, dy = _siso_grads(ins, h0, b0)
    npy = lambda v: None if v is None else v.detach().double().cpu().numpy()
    go = O.siso_scan_bwd(*[arrs[k] for k in keys], npy(dy), npy(h0), npy(b0))
    for k, tt in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), ins):
        assert rel_err(npy(tt.grad), go[k]) < 2e-2, k
    assert rel_err(npy(h0.grad), go["dh0"]) < 2e-2
    assert rel_err(npy(b0.grad), go["dbx0"]) < 2e-2


@pytest.mark.parametrize("case", ["strong_decay", "mixed_sign"])
def test_siso_bf16_chunked_backward_extreme_decay(case):
    """Per-step decays whose in-chunk products leave the fp32 range (ADT down to -13) and
    isolated growth steps (ADT up to +0.7) through the chunked backward."""
    arrs, t = _inputs(11 if case == "strong_decay" else 12, 1, 300, 2, 64, 128, dtype=torch.bfloat16)
    rng = np.random.default_rng(5)
    if case == "strong_decay":
        adt = -rng.uniform(0.0, 13.0, arrs["ADT"].shape)
    else:
        adt = -rng.uniform(0.0, 3.0, arrs["ADT"].shape)
        grow = rng.random(adt.shape) < 0.05
        adt[grow] = rng.uniform(0.0, 0.7, grow.sum())
    t["ADT"] = torch.tensor(adt, dtype=torch.float32, device=DEV)
    arrs["ADT"] = t["ADT"].double().cpu().numpy()
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    ins = [t[k].requires_grad_(True) for k in keys]
    y, dy = _siso_grads(ins)
    go = O.siso_scan_bwd(*[arrs[k] for k in keys], dy.detach().double().cpu().numpy())
    for k, tt in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), ins):
        g = tt.grad.detach().double().cpu().numpy()
        assert np.isfinite(g).all(), k
        assert rel_err(g, go[k]) < 2e-2, k


def test_siso_bwd_entry_points_agree():
    """The three ways into the SISO backward on one bf16 problem: the state-carrying pair
    (autograd), m3_siso_scan_bwd with a full workspace (chunk states recomputed) and with
    the minimal workspace (CUDA-core path)."""
    from mamba3_ssm import _lib as L
    Bn, Ln, H = 2, 333, 3
    arrs, t = _inputs(77, Bn, Ln, H, 64, 128, dtype=torch.bfloat16)
    keys = ("x", "B", "C", "ADT", "DT", "trap", "D")
    ins = [t[k].requires_grad_(True) for k in keys]
    y, dy = _siso_grads(ins)
    ref = [tt.grad.detach().clone() for tt in ins]
    lib = L.load()
    for ws_bytes in (lib.m3_siso_scan_bwd_workspace_size(Bn, Ln, H, 64, 128), 4 * Bn * Ln * H):
        outs = [torch.empty_like(t["x"]), torch.empty_like(t["B"]), torch.empty_like(t["C"]),
                torch.empty_like(t["ADT"]), torch.empty_like(t["DT"]), torch.empty_like(t["trap"]),
                torch.empty(H, device=DEV)]
        ws = torch.empty(int(ws_bytes), dtype=torch.uint8, device=DEV)
        a = L.pack(*[t[k].detach() for k in keys], None, None, dy, *outs, None, None)
        rc = lib.m3_siso_scan_bwd(*a.ptrs, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        L.check(rc, "m3_siso_scan_bwd")
        torch.cuda.synchronize()
        for k, o, r in zip(("dx", "dB", "dC", "dADT", "dDT", "dtrap", "dD"), outs, ref):
            # same chunked kernels: equal up to the order of the dD atomics; the CUDA-core
            # path: within the bf16 bar
            tol = 1e-5 if ws_bytes > 4 * Bn * Ln * H else 2e-2
            assert rel_err(o.double().cpu().numpy(), r.double().cpu().numpy()) < tol, (k, ws_bytes)
