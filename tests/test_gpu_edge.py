"""Edge-geometry kernels (spherical harmonics, radial embedding) on the GPU against the model's own modules, and the
whole model patched with ``edge_features=True`` against the unpatched model (the reference's tolerances)."""

import numpy as np
import pytest
import torch

import helpers
from helpers import E_ABS, E_TOL, F_ABS, F_TOL

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('lmax', [1, 2, 3])
def test_spherical_harmonics_match_module(cuda, lmax):
    from mace_mps_kernels_b200.edge import CudaSphericalHarmonics
    from mace_mps_kernels_b200.standin import o3
    mod = o3.SphericalHarmonics(o3.Irreps.spherical_harmonics(lmax), normalize=True, normalization='component')
    op = CudaSphericalHarmonics(mod)
    rng = np.random.default_rng(lmax)
    v = torch.tensor(rng.standard_normal((5001, 3)) * rng.uniform(0.5, 5, (5001, 1)), dtype=torch.float32)
    v[0] = torch.tensor([1e3, 0.0, 0.0])
    vd = v.to(cuda).requires_grad_(True)
    Y = op(vd)
    v64 = v.double().requires_grad_(True)
    Y64 = o3.spherical_harmonics(lmax, v64)
    assert Y.shape == Y64.shape
    scale = Y64.abs().max().item()
    assert (Y.double().cpu() - Y64.detach()).abs().max().item() < 2e-5 * scale
    g = torch.randn_like(Y)
    (gv,) = torch.autograd.grad(Y, vd, g)
    (gv64,) = torch.autograd.grad(Y64, v64, g.double().cpu())
    assert (gv.double().cpu() - gv64).abs().max().item() < 2e-5 * gv64.abs().max().item()


def test_radial_embedding_matches_module(cuda):
    from mace_mps_kernels_b200.edge import CudaRadialEmbedding
    from mace_mps_kernels_b200.standin.modules import RadialEmbeddingBlock
    blk = RadialEmbeddingBlock(5.0, 8, 5)
    op = CudaRadialEmbedding(blk)
    rng = np.random.default_rng(0)
    r = torch.tensor(np.concatenate([rng.uniform(0.5, 5.5, 3000), [5.0, 1e3]])[:, None], dtype=torch.float32)
    rd = r.to(cuda).requires_grad_(True)
    out = op(rd)
    r64 = r.double().requires_grad_(True)
    out64 = blk.double()(r64)
    assert (out.double().cpu() - out64.detach()).abs().max().item() < 2e-5 * out64.abs().max().item()
    g = torch.randn_like(out)
    (gr,) = torch.autograd.grad(out, rd, g)
    (gr64,) = torch.autograd.grad(out64, r64, g.double().cpu())
    assert (gr.double().cpu() - gr64).abs().max().item() < 2e-5 * gr64.abs().max().item()
    assert float(out[-1].abs().max()) == 0.0 and float(gr[-1].abs().max()) == 0.0


@pytest.mark.parametrize('config', ['l3_corr3', 'l2_corr2_scalar'])
def test_model_with_edge_features_matches_unpatched(cuda, config):
    if config not in helpers.CONFIGS:
        pytest.skip(f'no config {config}')
    ref, met, report = helpers.pair(config, cuda, edge_features=True)
    assert not report['skipped'], report['skipped']
    assert report['patched'][-3:] == ['spherical_harmonics', 'radial_embedding', 'get_edge_vectors_and_lengths'], report
    for s in (0, 1):
        st = helpers.make_structure(seed=s)
        E0, F0 = helpers.energy_forces(ref, st, cuda)
        E1, F1 = helpers.energy_forces(met, st, cuda)
        dE, dF = abs(E1 - E0), np.abs(F1 - F0).max()
        assert dE / len(st) < E_TOL and dF / max(np.abs(F0).max(), 1e-3) < F_TOL, (config, s, dE, dF)
        assert dE <= E_ABS and dF <= F_ABS


def test_edge_features_double_backward_raises(cuda):
    from mace_mps_kernels_b200.edge import CudaSphericalHarmonics
    from mace_mps_kernels_b200.standin import o3
    op = CudaSphericalHarmonics(o3.SphericalHarmonics(o3.Irreps.spherical_harmonics(3), normalize=True))
    v = torch.randn(10, 3, device=cuda, requires_grad=True)
    with pytest.raises(RuntimeError, match='double backward'):
        (g,) = torch.autograd.grad(op(v).square().sum(), v, create_graph=True)
        torch.autograd.grad(g.sum(), v)


@pytest.mark.parametrize('shift_grad', [False, True])
def test_edge_vectors_match_pytorch(cuda, shift_grad):
    """mmk_edge_vectors_fwd / _bwd against MACE's get_edge_vectors_and_lengths under autograd: vectors bit for bit,
    lengths to 1 ulp, the position gradient (per-node sums over the receiver and sender CSRs) and the shift gradient
    to float32 rounding.  Includes zero-length edges (the padding edges of a fixed-capacity graph: node to itself,
    zero shift), whose length gradient is 0 as in PyTorch's norm backward."""
    from mace_mps_kernels_b200.edge import edge_vectors_and_lengths
    from mace_mps_kernels_b200.standin.modules import get_edge_vectors_and_lengths
    rng = np.random.default_rng(7)
    N, E = 300, 9000
    pos = torch.tensor(rng.uniform(0, 12, (N, 3)), dtype=torch.float32, device=cuda)
    ei = torch.tensor(np.stack([rng.integers(0, N, E), rng.integers(0, N, E)]), device=cuda)
    ei[1, :50] = ei[0, :50]                                             # zero-length edges
    sh = torch.tensor(rng.choice([-3.6, 0.0, 3.6], (E, 3)), dtype=torch.float32, device=cuda)
    sh[:50] = 0.0
    gv = torch.randn(E, 3, device=cuda)
    gl = torch.randn(E, 1, device=cuda)
    outs = []
    for fn in (get_edge_vectors_and_lengths, None):
        p = pos.clone().requires_grad_(True)
        s = sh.clone().requires_grad_(shift_grad)
        if fn is None:
            v, ln = edge_vectors_and_lengths(p, ei.contiguous(), s)
        else:
            v, ln = fn(positions=p, edge_index=ei, shifts=s)
        grads = torch.autograd.grad((v, ln), (p, s) if shift_grad else (p,), (gv, gl))
        outs.append((v.detach(), ln.detach()) + tuple(g.detach() for g in grads))
    (v0, l0, *g0), (v1, l1, *g1) = outs
    assert torch.equal(v0, v1)
    assert (l0 - l1).abs().max().item() <= 1e-6 * l0.abs().max().item()
    assert float(l1[:50].abs().max()) == 0.0
    for a, b in zip(g0, g1):
        assert (a - b).abs().max().item() <= 2e-6 * a.abs().max().item()


def test_patched_model_routes_edge_vectors_to_cuda(cuda):
    """With edge_features=True the patched model's forward runs the fused edge-vector op (one launch each way) and
    matches the unpatched model; the unpatched model keeps calling PyTorch's version."""
    import copy
    from mace_mps_kernels_b200 import _lib, patch_model
    from mace_mps_kernels_b200 import standin as S
    ref = S.make_model('32x0e+32x1o', 3, 2, seed=0, elements=S.ELEMENTS_PTCOH).to(cuda).requires_grad_(False)
    met = copy.deepcopy(ref)
    rep = patch_model(met, verbose=False, edge_features=True)
    assert 'get_edge_vectors_and_lengths' in rep['patched']
    b = S.to_device(S.structure_batch([S.pt100_co_h(seed=0)], S.ELEMENTS_PTCOH, 5.0), cuda)
    res = []
    for m in (ref, met):
        n0 = _lib.LAUNCHES['mmk_edge_vectors_fwd']
        bb = dict(b)
        bb['positions'] = b['positions'].clone().requires_grad_(True)
        o = m(bb, compute_force=True)
        res.append((o['energy'].double().cpu(), o['forces'].double().cpu(), _lib.LAUNCHES['mmk_edge_vectors_fwd'] - n0))
    assert res[0][2] == 0 and res[1][2] == 1
    assert (res[0][0] - res[1][0]).abs().max().item() < E_ABS
    assert (res[0][1] - res[1][1]).abs().max().item() < F_ABS
