"""MACE-style ``SymmetricContraction`` (the product basis) with an in-repo equivariant basis.

For every output irrep L the layer evaluates, per node b and channel c,

    out[b, c, M] = sum_{nu=1..corr} sum_{i1..i_nu} U_nu[M, i1, .., i_nu, k] W_nu[elem(b), k, c] x[b,c,i1] .. x[b,c,i_nu]

in MACE's nested (Horner) order: ``out = U_corr W_max x``; then for nu = corr-1..1 ``out = (U_nu W_nu + out) x``, the
last ``ell`` axis being contracted first.  ``U_nu`` spans the O(3)-equivariant maps from the symmetric nu-th power of
the per-channel feature irreps (``0e+1o+2e+3o`` for l_max 3) to L: candidates come from chains of Clebsch-Gordan
couplings (l_1 x l_2 -> l_12, l_12 x l_3 -> ..., parities multiplied), are symmetrised over the nu input slots and
reduced to an orthonormal basis by SVD.  The basis differs from mace-torch's generalised-CG U matrices by an invertible
linear map per (nu, L); with random weights that choice does not matter for kernel-vs-oracle parity.

Attribute layout follows mace-torch 0.3.x (read by ``SCSpec`` in reference ``src/mace_mps_kernels/symmetric.py:20-39``):
``contractions[*].correlation``, buffers ``U_matrix_{nu}`` of shape ``[(2L+1,) n_ell x nu, k_nu]`` (no leading M axis
for L = 0), ``weights_max`` ``[n_elem, k_corr, C]`` and ``weights`` (nu = corr-1 down to 1) ``[n_elem, k_nu, C]``.
"""
from __future__ import annotations

import functools
import itertools

import numpy as np
import torch

from .o3 import Irrep, Irreps, clebsch_gordan


@functools.lru_cache(maxsize=None)
def symmetric_basis(in_ls: tuple, out_l: int, out_p: int, nu: int) -> np.ndarray:
    """Orthonormal basis [M, n_ell^nu, K] (float64) of symmetric equivariant nu-linear maps onto irrep (out_l, out_p).

    ``in_ls`` lists the per-channel input blocks as (l, p) pairs in layout order; n_ell = sum(2l+1)."""
    offs, n_ell = [], 0
    for l, _ in in_ls:
        offs.append(n_ell)
        n_ell += 2 * l + 1
    lmax_in = max(l for l, _ in in_ls)

    def embed(l, off):
        e = np.zeros((2 * l + 1, n_ell))
        e[np.arange(2 * l + 1), off + np.arange(2 * l + 1)] = 1.0
        return e

    states = [(embed(l, off), l, p) for (l, p), off in zip(in_ls, offs)]        # T[m, i1..ij]
    for step in range(1, nu):
        remaining = nu - 1 - step
        new = []
        for T, l, p in states:
            for (lb, pb), off in zip(in_ls, offs):
                for ln in range(abs(l - lb), l + lb + 1):
                    if remaining == 0 and (ln != out_l or p * pb != out_p):
                        continue
                    if ln - lmax_in * remaining > out_l:
                        continue
                    C = clebsch_gordan(l, lb, ln)                                  # [d_l, d_lb, d_ln]
                    E = embed(lb, off)                                             # [d_lb, n_ell]
                    Tn = np.einsum('abm,a...,bi->m...i', C, T, E)
                    new.append((Tn, ln, p * pb))
        states = new
    cands = [T for T, l, p in states if l == out_l and p == out_p]
    M = 2 * out_l + 1
    if not cands:
        return np.zeros((M, n_ell ** nu, 0))
    A = []
    for T in cands:
        S = np.zeros_like(T)
        perms = list(itertools.permutations(range(1, nu + 1)))
        for perm in perms:
            S += T.transpose((0,) + perm)
        A.append((S / len(perms)).reshape(-1))
    A = np.stack(A, 0)
    _, s, vt = np.linalg.svd(A, full_matrices=False)
    keep = s > 1e-9 * s[0]
    B = vt[keep]                                                                # [K, M * n^nu]
    for k in range(B.shape[0]):                                                 # deterministic sign
        j = np.argmax(np.abs(B[k]) > 1e-8)
        if B[k, j] < 0:
            B[k] = -B[k]
    B[np.abs(B) < 1e-14] = 0.0
    return B.reshape(B.shape[0], M, n_ell ** nu).transpose(1, 2, 0).copy()


class Contraction(torch.nn.Module):
    """One output irrep of the symmetric contraction (mace-torch ``Contraction``)."""

    def __init__(self, irreps_in, irrep_out, correlation, num_elements, num_features):
        super().__init__()
        self.correlation = correlation
        self.num_features = num_features
        in_ls = tuple((ir.l, ir.p) for _, ir in Irreps(irreps_in))
        self.n_ell = sum(2 * l + 1 for l, _ in in_ls)
        self.irrep_out = Irrep(irrep_out)
        M = self.irrep_out.dim
        self.has_m = self.irrep_out.l > 0
        for nu in range(1, correlation + 1):
            B = symmetric_basis(in_ls, self.irrep_out.l, self.irrep_out.p, nu)
            K = B.shape[-1]
            U = torch.from_numpy(B).float().reshape(M, *([self.n_ell] * nu), K)     # unit-norm paths, as CG products
            if not self.has_m:
                U = U[0]
            self.register_buffer(f'U_matrix_{nu}', U)
        k_max = getattr(self, f'U_matrix_{correlation}').shape[-1]
        self.weights_max = torch.nn.Parameter(torch.randn(num_elements, k_max, num_features) / max(k_max, 1))
        ws = []
        for nu in range(correlation - 1, 0, -1):
            k = getattr(self, f'U_matrix_{nu}').shape[-1]
            ws.append(torch.nn.Parameter(torch.randn(num_elements, k, num_features) / max(k, 1)))
        self.weights = torch.nn.ParameterList(ws)

    def U(self, nu):
        return getattr(self, f'U_matrix_{nu}')

    def forward(self, x, y):
        """x [N, C, n_ell], y [N, n_elem] -> [N, C * M] (channel-major, m fastest)."""
        N = x.shape[0]
        corr = self.correlation
        U = self.U(corr)
        K = U.shape[-1]
        lead = U.shape[:-2]                                     # (M?, ell^{corr-1})
        # sum_k U[..., i, k] W[e, k, c] y[b, e] x[b, c, i]
        wy = torch.einsum('ekc,be->bkc', self.weights_max, y)                  # [N, K, C]
        Uf = U.reshape(-1, U.shape[-2], K)                                     # [lead, i, k]
        t = torch.einsum('lik,bkc->bcli', Uf, wy)                              # [N, C, lead, i]
        out = torch.einsum('bcli,bci->bcl', t, x)                              # [N, C, lead]
        for j, w in enumerate(self.weights):
            nu = corr - 1 - j
            U = self.U(nu)
            K = U.shape[-1]
            wy = torch.einsum('ekc,be->bkc', w, y)
            c_t = torch.einsum('lk,bkc->bcl', U.reshape(-1, K), wy) + out     # [N, C, lead_nu * i]
            c_t = c_t.reshape(N, self.num_features, -1, self.n_ell)
            out = torch.einsum('bcli,bci->bcl', c_t, x)
        return out.reshape(N, -1)


class SymmetricContraction(torch.nn.Module):
    """mace-torch ``SymmetricContraction``: one ``Contraction`` per output irrep, outputs concatenated."""

    def __init__(self, irreps_in, irreps_out, correlation, num_elements):
        super().__init__()
        self.irreps_in, self.irreps_out = Irreps(irreps_in), Irreps(irreps_out)
        C = self.irreps_in[0].mul
        assert all(mul == C for mul, _ in self.irreps_in)
        per_channel = Irreps([(1, ir) for _, ir in self.irreps_in])
        self.contractions = torch.nn.ModuleList(
            [Contraction(per_channel, ir, correlation, num_elements, C) for mul, ir in self.irreps_out])

    def forward(self, x, y):
        return torch.cat([c(x, y) for c in self.contractions], dim=-1)
