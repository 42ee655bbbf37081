"""Generate the golden fixtures in this directory from the reference itself (run where the reference sources are
present: a sibling ``reference/src`` checkout, or the directory named by MMK_REFERENCE_SRC).

  python tests/golden/make_golden.py

For each case the reference's own code produces the expected values (reference = Yike-Ye/mace-mps-kernels v0.1.0):
  * ``ConvSpec`` (src/mace_mps_kernels/conv.py:57-88) probes a stand-in e3nn-style uvu TensorProduct -> the path
    coefficient table; ``csr_by`` (conv.py:229-235) -> receiver / sender CSRs;
  * the reference's generated conv kernels (conv.py:109-222), compiled as C++ by oracle/ref_build.py -> out, gx, gY, gW
    on seeded random inputs (a node with no edges included);
  * ``SCSpec`` (src/mace_mps_kernels/symmetric.py:52-75) on a duck-typed contraction built from seeded U / W arrays
    (stored in the fixture) -> packed coefficients T and the term list; its generated kernels (symmetric.py:82-131)
    -> out, gx.
The fixtures store inputs and these reference outputs; tests/test_oracle_golden.py (CPU) pins the oracle to them and
tests/test_gpu_golden.py checks the CUDA kernels against them.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import helpers  # noqa: E402
from oracle import ref_build  # noqa: E402

CONV_CASES = {               # tag: (hidden irreps of x, lmax of Y, N, E)
    'conv_x0e_l3': ('32x0e', 3, 9, 40),
    'conv_x0e1o_l3': ('32x0e+32x1o', 3, 12, 60),
    'conv_x0e1o2e_l3': ('32x0e+32x1o+32x2e', 3, 8, 30),
    'conv_x0e1o_l2': ('64x0e+64x1o', 2, 7, 25),
}

SC_CASES = {                 # tag: (lmax of the features, output irreps, correlation, C, n_elem, N)
    'sc_l2_c3_0e1o': (2, '0e+1o', 3, 6, 3, 9),
    'sc_l3_c2_0e1o2e': (3, '0e+1o+2e', 2, 5, 2, 7),
    'sc_l3_c3_0e': (3, '0e', 3, 4, 3, 6),
}


class _Contraction:
    """Duck-typed MACE Contraction (the attributes SCSpec reads)."""

    def __init__(self, corr, U, W):
        self.correlation = corr
        for nu, u in U.items():
            setattr(self, f'U_matrix_{nu}', torch.from_numpy(u))
        self.weights_max = torch.from_numpy(W[corr])
        self.weights = [torch.from_numpy(W[nu]) for nu in range(corr - 1, 0, -1)]


class _SC:
    def __init__(self, cts):
        self.contractions = cts


def sc_case(lmax, out_irreps, corr, C, n_elem, seed):
    """U from the stand-in's equivariant basis, seeded random weights; returns (duck-typed SC, arrays to store)."""
    from mace_mps_kernels_b200.standin import o3
    from mace_mps_kernels_b200.standin.symmetric_contraction import symmetric_basis
    rng = np.random.default_rng(seed)
    in_ls = tuple((l, (-1) ** l) for l in range(lmax + 1))
    n_ell = (lmax + 1) ** 2
    cts, arrays = [], {}
    for q, (_, ir) in enumerate(o3.Irreps(out_irreps)):
        U, W = {}, {}
        for nu in range(1, corr + 1):
            B = symmetric_basis(in_ls, ir.l, ir.p, nu).astype(np.float32)
            K = B.shape[-1]
            u = B.reshape(2 * ir.l + 1, *([n_ell] * nu), K)
            U[nu] = u if ir.l > 0 else u[0]
            W[nu] = (rng.normal(size=(n_elem, K, C)) / max(K, 1)).astype(np.float32)
            arrays[f'c{q}_U{nu}'] = U[nu]
            arrays[f'c{q}_W{nu}'] = W[nu]
        cts.append(_Contraction(corr, U, W))
    return _SC(cts), arrays


def main():
    rng = np.random.default_rng(2024)
    for tag, (hidden, lmax, N, E) in CONV_CASES.items():
        tp = helpers.conv_tp(hidden, lmax)
        rc = ref_build.RefConv(tp)
        ei = helpers.random_graph(N, E, seed=len(tag), isolated=[N - 1]).numpy()
        x = rng.normal(size=(N, rc.spec.x_dim)).astype(np.float32)
        Y = rng.normal(size=(E, rc.spec.y_dim)).astype(np.float32)
        W = rng.normal(size=(E, tp.weight_numel)).astype(np.float32)
        out = rc.fwd(x, Y, W, ei[0], ei[1], N)
        g = rng.normal(size=out.shape).astype(np.float32)
        gx, gY, gW = rc.bwd(x, Y, W, g, ei[0], ei[1], N)
        terms = [(c['k'], a, b, m, v) for c in rc.spec.coef for a, b, m, v in c['terms']]
        rr, re_ = rc.csr(ei[1], N)
        sr, se = rc.csr(ei[0], N)
        np.savez_compressed(
            os.path.join(HERE, tag + '.npz'), hidden=hidden, lmax=lmax, N=N, E=E, edge_index=ei, x=x, Y=Y, W=W, g=g,
            mul=rc.spec.mul, in1_l=[l for l, _, _ in rc.spec.in1], in2_l=[l for l, _, _ in rc.spec.in2],
            out_l=[l for l, _, _ in rc.spec.outb], ins=np.array(rc.spec.ins, np.int32),
            term_k=np.array([t[0] for t in terms], np.int32), term_a=np.array([t[1] for t in terms], np.int32),
            term_b=np.array([t[2] for t in terms], np.int32), term_m=np.array([t[3] for t in terms], np.int32),
            term_c=np.array([t[4] for t in terms], np.float64),
            ref_out=out, ref_gx=gx, ref_gY=gY, ref_gW=gW, recv_rowptr=rr, recv_eids=re_, send_rowptr=sr, send_eids=se)
        print(tag, 'nnz', len(terms), 'out', out.shape)
    for tag, (lmax, outs, corr, C, n_elem, N) in SC_CASES.items():
        sc, arrays = sc_case(lmax, outs, corr, C, n_elem, seed=len(tag))
        rs = ref_build.RefSC(sc)
        n_ell = (lmax + 1) ** 2
        x = rng.normal(size=(N, C, n_ell)).astype(np.float32)
        elem = rng.integers(0, n_elem, N).astype(np.int32)
        out = rs.fwd(x, elem)
        g = rng.normal(size=out.shape).astype(np.float32)
        gx = rs.bwd(x, elem, g)
        terms = [(q, idx, r0) for q, b in enumerate(rs.spec.blocks) for idx, r0 in b['terms']]
        D = max(len(t[1]) for t in terms)
        np.savez_compressed(
            os.path.join(HERE, tag + '.npz'), lmax=lmax, out_irreps=outs, corr=corr, C=C, n_elem=n_elem, N=N,
            n_contractions=len(sc.contractions), x=x, elem=elem, g=g, ref_T=rs.T,
            term_block=np.array([t[0] for t in terms], np.int32),
            term_idx=np.array([list(t[1]) + [-1] * (D - len(t[1])) for t in terms], np.int32),
            term_row=np.array([t[2] for t in terms], np.int32),
            block_M=np.array([b['M'] for b in rs.spec.blocks], np.int32), ref_out=out, ref_gx=gx, **arrays)
        print(tag, 'terms', len(terms), 'T', rs.T.shape)


if __name__ == '__main__':
    main()
