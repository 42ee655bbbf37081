"""Block-linear kernels (equivariant linears and element-indexed skip connections) against the model's own modules on
the GPU, and the whole model with every extension patched (frozen weights) against the unpatched model."""
import copy

import numpy as np
import pytest
import torch

import helpers
from helpers import E_ABS, E_TOL, F_ABS, F_TOL

pytestmark = pytest.mark.gpu


def _frozen(m):
    for p in m.parameters():
        p.requires_grad_(False)
    return m


@pytest.mark.parametrize('irr_in,irr_out,N', [
    ('128x0e+128x1o', '128x0e+128x1o', 168),
    ('128x0e+128x1o+128x0e+128x2e+128x1o+128x3o', '128x0e+128x1o+128x2e+128x3o', 5003),
    ('16x0e', '1x0e', 70),
    ('40x0e+24x1o', '200x0e+24x1o+8x2e', 1000),
])
def test_linear_matches_module(cuda, irr_in, irr_out, N):
    from mace_mps_kernels_b200.dense import CudaLinear
    from mace_mps_kernels_b200.standin import o3
    torch.manual_seed(0)
    lin = _frozen(o3.Linear(o3.Irreps(irr_in), o3.Irreps(irr_out))).to(cuda)
    op = CudaLinear(lin)
    x = torch.randn(N, lin.irreps_in.dim, device=cuda, requires_grad=True)
    out = op(x)
    lin64 = copy.deepcopy(lin).double().cpu()
    x64 = x.detach().double().cpu().requires_grad_(True)
    ref = lin64(x64)
    assert (out.double().cpu() - ref.detach()).abs().max().item() < 2e-5 * ref.abs().max().item()
    g = torch.randn_like(out)
    (gx,) = torch.autograd.grad(out, x, g)
    (gx64,) = torch.autograd.grad(ref, x64, g.double().cpu())
    assert (gx.double().cpu() - gx64).abs().max().item() < 2e-5 * gx64.abs().max().item()
    assert torch.equal(op(x.detach()), out.detach())


@pytest.mark.parametrize('offset', [0, 1, 2])
def test_linear_odd_rows_and_unaligned_input(cuda, offset):
    """Rows of an odd length (23 floats) starting at any 4-byte boundary: the kernel's 16-byte copies apply only where
    the source is 16-byte aligned, the rest go as 4-byte copies."""
    from mace_mps_kernels_b200.dense import CudaLinear
    from mace_mps_kernels_b200.standin import o3
    torch.manual_seed(4)
    lin = _frozen(o3.Linear(o3.Irreps('3x0e+5x1o+1x2e'), o3.Irreps('7x0e+2x1o+3x2e'))).to(cuda)
    op = CudaLinear(lin)
    N, dim = 37, lin.irreps_in.dim
    buf = torch.randn(N * dim + offset, device=cuda)
    x = buf[offset:].view(N, dim)                    # storage offset: base pointer 4-byte but not 16-byte aligned
    out = op(x)
    ref = copy.deepcopy(lin).double().cpu()(x.double().cpu())
    assert (out.double().cpu() - ref).abs().max().item() < 2e-5 * ref.abs().max().item()


@pytest.mark.parametrize('N,n_elem', [(168, 4), (3001, 3), (5, 89)])
def test_skip_tp_matches_module(cuda, N, n_elem):
    from mace_mps_kernels_b200.dense import CudaSkipTP
    from mace_mps_kernels_b200.standin import o3
    torch.manual_seed(1)
    tp = _frozen(o3.FullyConnectedTensorProduct(o3.Irreps('128x0e+128x1o'), o3.Irreps(f'{n_elem}x0e'),
                                                o3.Irreps('128x0e+128x1o+128x2e'))).to(cuda)
    op = CudaSkipTP(tp)
    elem = torch.from_numpy(np.random.default_rng(N).integers(0, n_elem, N))
    attrs = torch.nn.functional.one_hot(elem, n_elem).float().to(cuda)
    x = torch.randn(N, tp.irreps_in1.dim, device=cuda, requires_grad=True)
    out = op(x, attrs)
    tp64 = copy.deepcopy(tp).double().cpu()
    x64 = x.detach().double().cpu().requires_grad_(True)
    ref = tp64(x64, attrs.double().cpu())
    assert (out.double().cpu() - ref.detach()).abs().max().item() < 2e-5 * ref.abs().max().item()
    g = torch.randn_like(out)
    (gx,) = torch.autograd.grad(out, x, g)
    (gx64,) = torch.autograd.grad(ref, x64, g.double().cpu())
    assert (gx.double().cpu() - gx64).abs().max().item() < 2e-5 * gx64.abs().max().item()


@pytest.mark.parametrize('E,hs', [(5218, [8, 64, 64, 64, 1280]), (37, [8, 64, 64, 64, 128]), (9001, [8, 16, 2176]),
                                  (20011, [8, 64, 64, 64, 256]), (301, [5, 30, 7, 128]), (77, [8, 96, 64, 128])])
def test_radial_mlp_matches_module(cuda, E, hs):
    from mace_mps_kernels_b200.dense import CudaFullyConnectedNet
    from mace_mps_kernels_b200.standin.modules import FullyConnectedNet
    torch.manual_seed(3)
    mlp = _frozen(FullyConnectedNet(hs)).to(cuda)
    op = CudaFullyConnectedNet(mlp)
    assert op.fused == (max(hs[:-1]) <= 64)          # one launch each way for MACE's 64-wide hidden layers
    x = torch.randn(E, hs[0], device=cuda, requires_grad=True)
    out = op(x)
    mlp64 = copy.deepcopy(mlp).double().cpu()
    x64 = x.detach().double().cpu().requires_grad_(True)
    ref = mlp64(x64)
    assert (out.double().cpu() - ref.detach()).abs().max().item() < 2e-5 * ref.abs().max().item()
    g = torch.randn_like(out)
    (gx,) = torch.autograd.grad(out, x, g)
    (gx64,) = torch.autograd.grad(ref, x64, g.double().cpu())
    assert (gx.double().cpu() - gx64).abs().max().item() < 2e-5 * gx64.abs().max().item()


@pytest.mark.parametrize('config', ['l3_corr3', 'l3_corr3_l2hidden'])
def test_model_all_extensions_matches_unpatched(cuda, config):
    from mace_mps_kernels_b200 import patch_model
    hidden, lmax, corr, seed = helpers.CONFIGS[config]
    ref = _frozen(helpers.make_model(hidden, lmax, corr, seed).to(cuda))
    met = copy.deepcopy(ref)
    report = patch_model(met, verbose=False, edge_features=True, linears=True)
    assert not report['skipped'], report['skipped']
    assert 'interactions.0.linear_up' in report['patched'] and 'interactions.1.skip_tp' in report['patched']
    assert 'interactions.1.conv_tp_weights' in report['patched']
    for s in (0, 1):
        st = helpers.make_structure(seed=s)
        E0, F0 = helpers.energy_forces(ref, st, cuda)
        E1, F1 = helpers.energy_forces(met, st, cuda)
        dE, dF = abs(E1 - E0), np.abs(F1 - F0).max()
        assert dE / len(st) < E_TOL and dF / max(np.abs(F0).max(), 1e-3) < F_TOL, (config, s, dE, dF)
        assert dE <= E_ABS and dF <= F_ABS


def test_linears_need_frozen_weights(cuda):
    from mace_mps_kernels_b200 import patch_model
    model = helpers.make_model().to(cuda)
    report = patch_model(model, verbose=False, linears=True)
    assert any('frozen weights only' in why for _, why in report['skipped'])


@pytest.mark.parametrize('irreps,N', [('128x0e+128x1o+128x2e+128x3o', 168), ('32x0e+32x1o', 1001), ('16x0e', 5)])
def test_reshape_irreps_matches_module(cuda, irreps, N):
    """CudaReshapeIrreps (one column gather each way) against MACE's reshape_irreps: forward and input gradient are
    pure data movement, so both are bit for bit."""
    from mace_mps_kernels_b200.dense import CudaReshapeIrreps
    from mace_mps_kernels_b200.standin import o3
    from mace_mps_kernels_b200.standin.modules import reshape_irreps
    m = reshape_irreps(o3.Irreps(irreps))
    op = CudaReshapeIrreps(m).to(cuda)
    x = torch.randn(N, m.irreps.dim, device=cuda)
    outs = []
    for mod in (m, op):
        xx = x.clone().requires_grad_(True)
        y = mod(xx)
        g = torch.arange(y.numel(), device=cuda, dtype=torch.float32).reshape(y.shape)
        (gx,) = torch.autograd.grad(y, xx, g)
        outs.append((y.detach(), gx))
    assert outs[0][0].shape == outs[1][0].shape
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
