"""CPU: pin the oracle to the reference's own outputs (fixtures made by tests/golden/make_golden.py from the
reference's ConvSpec / SCSpec / csr_by and its generated kernels compiled as C++)."""
import glob
import os

import numpy as np
import pytest
import torch

import helpers
from oracle import conv_ref, sc_ref

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
CONV = sorted(glob.glob(os.path.join(GOLDEN, 'conv_*.npz')))
SC = sorted(glob.glob(os.path.join(GOLDEN, 'sc_*.npz')))


def rel(a, b):
    return np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30)


def conv_table(z):
    coef = []
    in1, _ = conv_ref.blocks([(int(z['mul']), _L(l)) for l in z['in1_l']])
    in2, _ = conv_ref.blocks([(1, _L(l)) for l in z['in2_l']])
    outb, out_dim = conv_ref.blocks([(int(z['mul']), _L(l)) for l in z['out_l']])
    for k, (i1, i2, io) in enumerate(z['ins']):
        coef.append(dict(k=k, l1=in1[i1][0], l2=in2[i2][0], l3=outb[io][0], o1=in1[i1][2], o2=in2[i2][2],
                         o3=outb[io][2], terms=[]))
    for k, a, b, m, c in zip(z['term_k'], z['term_a'], z['term_b'], z['term_m'], z['term_c']):
        coef[k]['terms'].append((int(a), int(b), int(m), float(c)))
    spec = dict(mul=int(z['mul']), x_dim=z['x'].shape[1], y_dim=z['Y'].shape[1], out_dim=out_dim)
    return spec, coef


class _L:
    def __init__(self, l):
        self.l = int(l)


def test_fixtures_present():
    assert len(CONV) >= 4 and len(SC) >= 3


@pytest.mark.parametrize('path', CONV, ids=os.path.basename)
def test_oracle_probe_matches_reference_conv_spec(path):
    z = np.load(path)
    tp = helpers.conv_tp(str(z['hidden']), int(z['lmax']))
    spec, coef = conv_ref.probe_coefficients(tp)
    terms = [(c['k'], a, b, m, v) for c in coef for a, b, m, v in c['terms']]
    assert [t[:4] for t in terms] == list(zip(z['term_k'], z['term_a'], z['term_b'], z['term_m']))
    assert np.allclose([t[4] for t in terms], z['term_c'], rtol=1e-7, atol=0)


@pytest.mark.parametrize('path', CONV, ids=os.path.basename)
def test_oracle_conv_matches_reference_kernels(path):
    z = np.load(path)
    spec, coef = conv_table(z)
    ei = z['edge_index']
    N = int(z['N'])
    out = conv_ref.conv_fwd(spec, coef, z['x'], z['Y'], z['W'], ei[0], ei[1], N)
    assert rel(z['ref_out'], out) < 1e-5
    gx, gY, gW = conv_ref.conv_bwd(spec, coef, z['x'], z['Y'], z['W'], z['g'], ei[0], ei[1])
    assert rel(z['ref_gx'], gx) < 1e-5
    assert rel(z['ref_gY'], gY) < 1e-5
    assert rel(z['ref_gW'], gW) < 1e-5
    assert np.abs(out[N - 1]).max() == 0.0          # the isolated node receives nothing


@pytest.mark.parametrize('path', CONV, ids=os.path.basename)
def test_oracle_csr_matches_reference_csr_by(path):
    z = np.load(path)
    ei, N = z['edge_index'], int(z['N'])
    r, e = conv_ref.csr_by(ei[1], N)
    assert np.array_equal(r, z['recv_rowptr']) and np.array_equal(e, z['recv_eids'])
    r, e = conv_ref.csr_by(ei[0], N)
    assert np.array_equal(r, z['send_rowptr']) and np.array_equal(e, z['send_eids'])


class _Ct:
    def __init__(self, z, q):
        corr = int(z['corr'])
        self.correlation = corr
        for nu in range(1, corr + 1):
            setattr(self, f'U_matrix_{nu}', torch.from_numpy(z[f'c{q}_U{nu}']))
        self.weights_max = torch.from_numpy(z[f'c{q}_W{corr}'])
        self.weights = [torch.from_numpy(z[f'c{q}_W{nu}']) for nu in range(corr - 1, 0, -1)]


class _SC:
    def __init__(self, z):
        self.contractions = [_Ct(z, q) for q in range(int(z['n_contractions']))]


@pytest.mark.parametrize('path', SC, ids=os.path.basename)
def test_oracle_sc_spec_matches_reference(path):
    z = np.load(path)
    spec = sc_ref.sc_spec(_SC(z))
    terms = [(q, tuple(idx), r0) for q, b in enumerate(spec['blocks']) for idx, r0 in b['terms']]
    ref_terms = [(int(q), tuple(int(i) for i in idx if i >= 0), int(r)) for q, idx, r in
                 zip(z['term_block'], z['term_idx'], z['term_row'])]
    assert terms == ref_terms
    assert rel(z['ref_T'], spec['T']) < 1e-6


@pytest.mark.parametrize('path', SC, ids=os.path.basename)
def test_oracle_sc_matches_reference_kernels(path):
    z = np.load(path)
    spec = sc_ref.sc_spec(_SC(z))
    assert rel(z['ref_out'], sc_ref.sc_fwd(spec, z['x'], z['elem'])) < 1e-5
    assert rel(z['ref_gx'], sc_ref.sc_bwd(spec, z['x'], z['elem'], z['g'])) < 1e-5


@pytest.mark.parametrize('path', SC, ids=os.path.basename)
def test_package_sc_spec_matches_reference(path):
    """The product's own coefficient builder (vectorised symmetrisation) gives the reference's table."""
    from mace_mps_kernels_b200.symmetric import SCSpec
    z = np.load(path)
    spec = SCSpec(_SC(z))
    terms = [(q, tuple(idx), r0) for q, b in enumerate(spec.blocks) for idx, r0 in b['terms']]
    ref_terms = [(int(q), tuple(int(i) for i in idx if i >= 0), int(r)) for q, idx, r in
                 zip(z['term_block'], z['term_idx'], z['term_row'])]
    assert terms == ref_terms
    assert rel(z['ref_T'], spec.T.double().numpy()) < 1e-6


@pytest.mark.parametrize('path', CONV, ids=os.path.basename)
def test_package_conv_spec_matches_reference(path):
    """The product's batched probe gives the reference's per-instruction probe table."""
    from mace_mps_kernels_b200.conv import ConvSpec
    z = np.load(path)
    spec = ConvSpec(helpers.conv_tp(str(z['hidden']), int(z['lmax'])))
    terms = [(c['k'], a, b, m, v) for c in spec.coef for a, b, m, v in c['terms']]
    assert [t[:4] for t in terms] == list(zip(z['term_k'], z['term_a'], z['term_b'], z['term_m']))
    assert np.allclose([t[4] for t in terms], z['term_c'], rtol=1e-7, atol=0)
