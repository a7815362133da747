"""The chunked (k-)formulation the tensor-core SISO kernels implement, restated in float64
numpy and checked against the oracle's sequential scan and its adjoint: forward chunk
states and outputs, and the backward's per-chunk matrix products, carried adjoint and the
per-step scalars feeding the dADT suffix sums. Small shapes, ragged lengths, initial states.
This pins the algebra of csrc/siso_chunk.cu and csrc/siso_chunk_bwd.cu on the CPU.
"""

import numpy as np
import pytest

from oracle import scan_oracle as O


def _inputs(seed, L, P, D):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, L, 1, P))
    Bm = rng.standard_normal((1, L, 1, D))
    C = rng.standard_normal((1, L, 1, D))
    dt = rng.uniform(0.01, 0.2, (1, L, 1))
    ADT = -rng.uniform(0.0, 1.0, (1, L, 1))
    trap = rng.standard_normal((1, L, 1))
    Dw = rng.standard_normal(1)
    h0 = rng.standard_normal((1, 1, P, D))
    bx0 = rng.standard_normal((1, 1, P, D))
    dy = rng.standard_normal((1, L, 1, P))
    return x, Bm, C, ADT, dt, trap, Dw, h0, bx0, dy


def _chunk_scalars(a, beta, gam, ADT, t0, Q, L):
    """lambda_0..Q (lambda_0 = 0), a_{i+1}, gamma_{i+1}, beta_i of the chunk at t0 (zero
    beyond the sequence)."""
    adt = np.zeros(Q + 1)
    adt[1:] = [ADT[t0 + i] if t0 + i < L else 0.0 for i in range(1, Q + 1)]
    lam = np.cumsum(adt)
    an = np.array([a[t0 + i + 1] if t0 + i + 1 < L else 0.0 for i in range(Q)])
    gn = np.array([gam[t0 + i + 1] if t0 + i + 1 < L else 0.0 for i in range(Q)])
    bb = np.array([beta[t0 + i] if t0 + i < L else 0.0 for i in range(Q)])
    return lam, an, gn, bb


def _pad(v, t0, Q):
    out = np.zeros((Q,) + v.shape[1:])
    n = min(Q, v.shape[0] - t0)
    out[:n] = v[t0:t0 + n]
    return out


@pytest.mark.parametrize("L,Q", [(37, 8), (64, 16), (5, 8), (16, 16)])
def test_chunked_forward_and_backward_match_the_sequential_scan(L, Q):
    P, D = 4, 6
    x, Bm, C, ADT, dt, trap, Dw, h0, bx0, dy = _inputs(L * 7 + Q, L, P, D)
    yo, ho, bo = O.siso_scan_fwd(x, Bm, C, ADT, dt, trap, Dw, h0, bx0)
    go = O.siso_scan_bwd(x, Bm, C, ADT, dt, trap, Dw, dy, h0, bx0)
    a = np.exp(ADT[0, :, 0])
    tr = 1 / (1 + np.exp(-trap[0, :, 0]))
    dtv = dt[0, :, 0]
    beta = dtv * (1 - tr) + 0.5 * dtv * tr
    gam = 0.5 * dtv * tr
    X, Bt, Ct, dY = x[0, :, 0], Bm[0, :, 0], C[0, :, 0], dy[0, :, 0]
    nch = (L + Q - 1) // Q
    low = np.tril(np.ones((Q, Q)), -1)

    # forward: k_c at every chunk start, y from the chunk formula
    k = a[0] * h0[0, 0] + gam[0] * bx0[0, 0]
    ks, y = [], np.zeros_like(X)
    for c in range(nch):
        t0 = c * Q
        n = min(Q, L - t0)
        lam, an, gn, bb = _chunk_scalars(a, beta, gam, ADT[0, :, 0], t0, Q, L)
        mu = an * bb + gn
        Xc, Bc, Cc = _pad(X, t0, Q), _pad(Bt, t0, Q), _pad(Ct, t0, Q)
        E = np.exp(lam[:Q, None] - lam[None, 1:Q + 1])
        M = E * mu[None, :] * low + np.diag(bb)
        Yc = np.exp(lam[:Q])[:, None] * (Cc @ k.T) + (M * (Cc @ Bc.T)) @ Xc + Dw[0] * Xc
        y[t0:t0 + n] = Yc[:n]
        ks.append(k.copy())
        w = np.exp(lam[Q] - lam[1:Q + 1]) * mu
        k = np.exp(lam[Q]) * k + Xc.T @ (w[:, None] * Bc)
    np.testing.assert_allclose(y, yo[0, :, 0], rtol=1e-10, atol=1e-10)

    # backward: per-chunk products with the carried adjoint, per-step q, dbeta, dgamma
    dx, dB, dC = np.zeros_like(X), np.zeros_like(Bt), np.zeros_like(Ct)
    sq, sb, sg = np.zeros(L), np.zeros(L), np.zeros(L)
    dkn = np.zeros((P, D))
    for c in reversed(range(nch)):
        t0 = c * Q
        n = min(Q, L - t0)
        lam, an, gn, bb = _chunk_scalars(a, beta, gam, ADT[0, :, 0], t0, Q, L)
        mu = an * bb + gn
        wdec = np.exp(lam[Q] - lam[1:Q + 1])
        w, el = wdec * mu, np.exp(lam[:Q])
        Xc, Bc, Cc, dYc = _pad(X, t0, Q), _pad(Bt, t0, Q), _pad(Ct, t0, Q), _pad(dY, t0, Q)
        kc = ks[c]
        G, S = Cc @ Bc.T, dYc @ Xc.T
        E = np.exp(lam[:Q, None] - lam[None, 1:Q + 1])
        Gh = G * E * low
        MS = S * E * mu[None, :] * low + np.diag(bb * np.diag(S))
        q = el * np.sum(dYc * (Cc @ kc.T), 1) + np.sum(G * MS, 1)
        V = Gh.T @ dYc + wdec[:, None] * (Bc @ dkn.T)
        dCc = (el[:, None] * dYc) @ kc + MS @ Bc
        dBc = MS.T @ Cc + (w[:, None] * Xc) @ dkn
        dXc = mu[:, None] * V + (bb * np.diag(G) + Dw[0])[:, None] * dYc
        dmu = np.sum(Xc * V, 1)
        dx[t0:t0 + n], dB[t0:t0 + n], dC[t0:t0 + n] = dXc[:n], dBc[:n], dCc[:n]
        sq[t0:t0 + n] = q[:n]
        sb[t0:t0 + n] = (np.diag(G) * np.diag(S) + an * dmu)[:n]
        for i in range(n):
            if t0 + i + 1 < L:
                sg[t0 + i + 1] = dmu[i]
        dkn = np.exp(lam[Q]) * dkn + (el[:, None] * dYc).T @ Cc
    sg[0] = np.sum(dkn * bx0[0, 0])
    dadt = np.cumsum((sq - beta * sb - gam * sg)[::-1])[::-1]
    ddt = sb * (1 - 0.5 * tr) + sg * 0.5 * tr
    dtrap = 0.5 * dtv * (sg - sb) * tr * (1 - tr)
    for name, got in (("dx", dx), ("dB", dB), ("dC", dC), ("dADT", dadt), ("dDT", ddt), ("dtrap", dtrap)):
        ref = go[name][0, :, 0]
        np.testing.assert_allclose(got, ref, rtol=1e-9, atol=1e-9 * np.abs(ref).max(), err_msg=name)
    np.testing.assert_allclose(a[0] * dkn, go["dh0"][0, 0], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(gam[0] * dkn, go["dbx0"][0, 0], rtol=1e-9, atol=1e-12)
