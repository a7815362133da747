"""The group-row formulation of the MIMO layer scan (m3_mimo_layer_scan_fwd, the group-row
form of csrc/mimo_chunked.cu), restated in float64 numpy and checked against the oracle's
layer forward, which materialises the per-head B / C of layer.py:214-244 and runs the scan of
ops.py:222-242 and the gate of layer.py:262-266. The restatement follows the kernel: per
chunk of Q steps the RMS factor of every group row of B and C, one rotation per (step, pair)
applied after the rank sum for Bx, a local scan from a zero state joined to the state
entering the chunk, the states rotated back for the readouts against the unrotated C rows,
and the gate applied to y. Small shapes, ragged chunks, both rope fractions. This pins the
algebra of the kernel on the CPU; the GPU tests check the kernel against the two-kernel path.
"""

import numpy as np
import pytest

from oracle import scan_oracle as O

EPS = 1e-5


def _weights(rng, dims):
    H, R, D, P = dims.H, dims.R, dims.d_state, dims.headdim
    return {
        "in_proj.weight": rng.standard_normal((dims.d_in_proj, dims.d_model)) * 0.4,
        "out_proj.weight": rng.standard_normal((dims.d_model, dims.d_inner)) * 0.2,
        "dt_bias": rng.uniform(-3.0, -1.0, H),
        "B_norm.weight": rng.uniform(0.5, 1.5, D),
        "C_norm.weight": rng.uniform(0.5, 1.5, D),
        "B_bias": rng.standard_normal((H, R, D)) * 0.5,
        "C_bias": rng.standard_normal((H, R, D)) * 0.5,
        "D": rng.standard_normal(H),
        "mimo_x": rng.standard_normal((H, R, P)) * 0.5,
        "mimo_o": rng.standard_normal((H, R, P)) * 0.5,
    }


def _rot(v, c, s, transpose=False):
    """Rotate pairs (2k, 2k+1), k < c.shape[-1], of the last axis by (c, s) (or by the
    transpose: the inverse rotation)."""
    out = v.copy()
    n = c.shape[-1]
    v0, v1 = v[..., 0:2 * n:2], v[..., 1:2 * n:2]
    if transpose:
        out[..., 0:2 * n:2], out[..., 1:2 * n:2] = v0 * c + v1 * s, v1 * c - v0 * s
    else:
        out[..., 0:2 * n:2], out[..., 1:2 * n:2] = v0 * c - v1 * s, v0 * s + v1 * c
    return out


def _group_row_forward(w, dims, u, Q):
    Bn, L, _ = u.shape
    H, P, R, D = dims.H, dims.headdim, dims.R, dims.d_state
    zx = u @ w["in_proj.weight"].T
    z, x, Braw, Craw, ddt, dA, trap, angr = dims.split_proj(zx)
    z = z.reshape(Bn, L, H, P)
    x = x.reshape(Bn, L, H, P)
    Braw = Braw.reshape(Bn, L, R, D)
    Craw = Craw.reshape(Bn, L, R, D)
    A = -np.minimum(O.softplus(dA), -dims.A_floor)
    DT = O.softplus(ddt + w["dt_bias"])
    ADT = A * DT
    ang = np.cumsum(angr[:, :, None, :] * DT[..., None], axis=1)  # (B, L, H, S)
    cs, sn = np.cos(ang), np.sin(ang)
    rsB = 1.0 / np.sqrt(np.mean(Braw * Braw, axis=-1) + EPS)  # (B, L, R): one per group row
    rsC = 1.0 / np.sqrt(np.mean(Craw * Craw, axis=-1) + EPS)
    a = np.exp(ADT)
    tr = O.sigmoid(trap)
    beta = DT * (1.0 - tr) + 0.5 * DT * tr
    gam = 0.5 * DT * tr
    wB, wC = w["B_norm.weight"], w["C_norm.weight"]
    y = np.empty((Bn, L, H, P))
    for h in range(H):
        xr = np.einsum("blp,rp->blr", x[:, :, h], w["mimo_x"][h])  # (B, L, R)
        # Bx = rot(w o sum_r xr rs raw_r + sum_r xr bias_r): the rotation after the rank sum
        ub = wB * np.einsum("blr,blrd->bld", xr * rsB, Braw) + xr @ w["B_bias"][h]
        bx = _rot(ub, cs[:, :, h], sn[:, :, h])  # (B, L, D)
        state = np.zeros((Bn, D))
        for t0 in range(0, L, Q):
            n = min(Q, L - t0)
            bxp = bx[:, t0 - 1] if t0 > 0 else np.zeros((Bn, D))
            hloc = np.zeros((Bn, D))
            cum = np.ones(Bn)
            hs = np.empty((Bn, n, D))
            for j in range(n):
                t = t0 + j
                hloc = a[:, t, h, None] * hloc + beta[:, t, h, None] * bx[:, t] + gam[:, t, h, None] * bxp
                cum = cum * a[:, t, h]
                hs[:, j] = hloc + cum[:, None] * state  # the carry joined to the local scan
                bxp = bx[:, t]
            state = hs[:, n - 1]
            hrot = _rot(hs, cs[:, t0:t0 + n, h], sn[:, t0:t0 + n, h], transpose=True)  # rot^T h
            # C_t[r] . h_t = rs (raw_r o w) . rot^T h + bias_r . rot^T h
            yr = (rsC[:, t0:t0 + n] * np.einsum("bjrd,bjd->bjr", Craw[:, t0:t0 + n] * wC, hrot)
                  + np.einsum("rd,bjd->bjr", w["C_bias"][h], hrot) + w["D"][h] * xr[:, t0:t0 + n])
            y[:, t0:t0 + n, h] = np.einsum("bjr,rp->bjp", yr, w["mimo_o"][h])
    g = y * (z * O.sigmoid(z))  # the gate fused into the store
    return g.reshape(Bn, L, dims.d_inner) @ w["out_proj.weight"].T


@pytest.mark.parametrize("rope_fraction", [0.5, 1.0])
@pytest.mark.parametrize("L,Q", [(13, 5), (16, 4), (1, 8)])
def test_group_row_formulation_matches_oracle_layer(rope_fraction, L, Q):
    dims = O.LayerDims(d_model=16, d_state=8, expand=2, headdim=4, is_mimo=True, mimo_rank=2,
                       rope_fraction=rope_fraction)
    rng = np.random.default_rng(L * 10 + Q)
    w = _weights(rng, dims)
    u = rng.standard_normal((2, L, dims.d_model))
    ref = O.mamba3_forward(w, dims, u)
    got = _group_row_forward(w, dims, u, Q)
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    assert err < 1e-12, err
