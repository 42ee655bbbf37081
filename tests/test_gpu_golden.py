"""GPU: the CUDA kernels (through the C ABI) reproduce the reference's own kernel outputs stored in tests/golden/."""
import glob
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
CONV = sorted(glob.glob(os.path.join(GOLDEN, 'conv_*.npz')))
SC = sorted(glob.glob(os.path.join(GOLDEN, 'sc_*.npz')))
REL = 2e-5


def rel(a, b):
    a = a.detach().double().cpu().numpy() if torch.is_tensor(a) else np.asarray(a, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


@pytest.mark.parametrize('path', CONV, ids=os.path.basename)
def test_conv_kernels_match_reference(cuda, path):
    from mace_mps_kernels_b200.conv import ConvSpec, CudaConvTP, graph_csr
    z = np.load(path)
    terms = list(zip(z['term_k'], z['term_a'], z['term_b'], z['term_m'], z['term_c']))
    spec = ConvSpec.from_table(int(z['mul']), z['in1_l'], z['in2_l'], z['out_l'], z['ins'], terms)
    op = CudaConvTP.from_spec(spec)
    t = lambda k: torch.from_numpy(z[k]).to(cuda)
    x, Y, W = (t(k).requires_grad_(True) for k in ('x', 'Y', 'W'))
    ei = t('edge_index').long()
    out = op(x, Y, W, ei)
    assert rel(out, z['ref_out']) < REL
    gx, gY, gW = torch.autograd.grad(out, (x, Y, W), t('g'))
    assert rel(gx, z['ref_gx']) < REL
    assert rel(gY, z['ref_gY']) < REL
    assert rel(gW, z['ref_gW']) < REL
    rr, re_, sr, se = graph_csr(ei, int(z['N']))
    for a, k in ((rr, 'recv_rowptr'), (re_, 'recv_eids'), (sr, 'send_rowptr'), (se, 'send_eids')):
        assert np.array_equal(a.cpu().numpy(), z[k]), k


@pytest.mark.parametrize('path', SC, ids=os.path.basename)
def test_sc_kernels_match_reference(cuda, path):
    from mace_mps_kernels_b200.symmetric import CudaSymmetricContraction, SCSpec
    z = np.load(path)
    nb = len(z['block_M'])
    block_terms = [[] for _ in range(nb)]
    for q, idx, r in zip(z['term_block'], z['term_idx'], z['term_row']):
        block_terms[q].append(([i for i in idx if i >= 0], r))
    spec = SCSpec.from_table(int(z['C']), z['x'].shape[2], z['block_M'], block_terms, z['ref_T'])
    op = CudaSymmetricContraction.from_spec(spec, device=cuda)
    x = torch.from_numpy(z['x']).to(cuda).requires_grad_(True)
    attrs = torch.nn.functional.one_hot(torch.from_numpy(z['elem']).long(), int(z['n_elem'])).float().to(cuda)
    out = op(x, attrs)
    assert rel(out, z['ref_out']) < REL
    (gx,) = torch.autograd.grad(out, (x,), torch.from_numpy(z['g']).to(cuda))
    assert rel(gx, z['ref_gx']) < REL
