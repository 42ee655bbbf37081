"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): float64 restatement of the reference's symmetric contraction.

Reference = Yike-Ye/mace-mps-kernels v0.1.0, file src/mace_mps_kernels/symmetric.py.
"""
from __future__ import annotations

import itertools

import numpy as np


def poly_coeffs(ct):
    """{nu: {sorted index tuple: coefficient [e, M, c]}}, M, n_ell -- symmetric.py:20-39.

    T_nu[e, c, M, i1..i_nu] = sum_p U_nu[M, i1..i_nu, p] W_nu[e, p, c]; weights_max <-> nu = correlation,
    weights[j] <-> nu = correlation - 1 - j; coefficients of index tuples that sort to the same tuple are summed."""
    corr = int(ct.correlation)
    U = {nu: getattr(ct, f'U_matrix_{nu}').detach().cpu().double().numpy() for nu in range(1, corr + 1)}
    W = {corr: ct.weights_max.detach().cpu().double().numpy()}
    for j, w in enumerate(ct.weights):
        W[corr - 1 - j] = w.detach().cpu().double().numpy()
    lead = U[1].ndim - 2
    M = U[1].shape[0] if lead else 1
    n_ell = U[1].shape[-2]
    res = {}
    for nu in range(1, corr + 1):
        u = U[nu] if lead else U[nu][None]
        T = np.einsum('mip,epc->ecmi', u.reshape(M, -1, u.shape[-1]), W[nu])
        T = T.reshape(W[nu].shape[0], W[nu].shape[2], M, *([n_ell] * nu))
        acc = {}
        for idx in itertools.product(range(n_ell), repeat=nu):
            key = tuple(sorted(idx))
            acc[key] = acc.get(key, 0) + T[(slice(None),) * 3 + idx]
        res[nu] = {k: v.transpose(0, 2, 1) for k, v in acc.items()}          # [e, M, c]
    return res, M, n_ell


def sc_spec(sc, tol=1e-12):
    """Term list and packed coefficients -- symmetric.py:52-75.

    Returns dict(blocks=[dict(M, terms=[(idx, row0)], out_off)], T [e, rows, c] float64, C, n_ell, out_dim)."""
    blocks, rows, out_off, n_ell, C = [], [], 0, None, None
    for ct in sc.contractions:
        coeffs, M, n_ell = poly_coeffs(ct)
        terms = []
        for nu in sorted(coeffs, reverse=True):
            for idx, v in sorted(coeffs[nu].items()):
                if np.abs(v).max() <= tol:
                    continue
                terms.append((idx, len(rows)))
                rows += [v[:, m, :] for m in range(M)]
        C = next(iter(coeffs[1].values())).shape[2]
        blocks.append(dict(M=M, terms=terms, out_off=out_off))
        out_off += C * M
    return dict(blocks=blocks, T=np.stack(rows, axis=1), C=C, n_ell=n_ell, out_dim=out_off)


def sc_fwd(spec, x, elem):
    """out[b, off + c M + m] = sum_terms T[elem(b), row + m, c] prod_{i in idx} x[b, c, i] -- symmetric.py:82-105."""
    x = np.asarray(x, np.float64)
    N, C, _ = x.shape
    T = spec['T'][np.asarray(elem)]                                         # [N, rows, c]
    out = np.zeros((N, spec['out_dim']))
    for bl in spec['blocks']:
        M, off = bl['M'], bl['out_off']
        acc = np.zeros((N, C, M))
        for idx, r0 in bl['terms']:
            p = np.prod(x[:, :, list(idx)], axis=2)                          # [N, C]
            acc += T[:, r0:r0 + M, :].transpose(0, 2, 1) * p[:, :, None]
        out[:, off:off + C * M] = acc.reshape(N, C * M)
    return out


def sc_bwd(spec, x, elem, g):
    """gx[b, c, i] = sum_terms (sum_m T[elem(b), row+m, c] g[b, off + c M + m]) d(prod x)/dx_i -- symmetric.py:106-131."""
    x = np.asarray(x, np.float64)
    g = np.asarray(g, np.float64)
    N, C, n = x.shape
    T = spec['T'][np.asarray(elem)]
    gx = np.zeros_like(x)
    for bl in spec['blocks']:
        M, off = bl['M'], bl['out_off']
        G = g[:, off:off + C * M].reshape(N, C, M)
        for idx, r0 in bl['terms']:
            s = np.einsum('bmc,bcm->bc', T[:, r0:r0 + M, :], G)
            for i in sorted(set(idx)):
                rest = list(idx)
                rest.remove(i)
                k = idx.count(i)
                d = np.prod(x[:, :, rest], axis=2) if rest else np.ones((N, C))
                gx[:, :, i] += s * k * d
    return gx
