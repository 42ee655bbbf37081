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
    assert report['patched'][-2:] == ['spherical_harmonics', 'radial_embedding'], report
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
