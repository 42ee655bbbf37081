"""The reference's correctness tests (reference tests/test_kernels.py), restated on the stand-in MACE model on CUDA:

* every CONFIGS model: all convolutions and symmetric contractions patched, energies and forces of the patched model
  match the unpatched (e3nn-path) model within |dE|/atom < 1e-5 eV and max|dF| / max|F0| < 1e-5 on seeds 0, 1, 2,
  and within the absolute bounds max|dF| <= 1e-5 eV/A, |dE| <= 1 meV per structure;
* rotation equivariance of the patched model;
* double backward (training on forces) raises instead of silently returning wrong gradients;
* an unsupported block (multiplicity 48, not a multiple of 32) is skipped and keeps working on the torch path.
"""
import copy

import numpy as np
import pytest
import torch

import helpers
from helpers import E_ABS, E_TOL, F_ABS, F_TOL

pytestmark = pytest.mark.gpu


def _check_pair(config, cuda, seeds=(0, 1, 2)):
    ref, met, report = helpers.pair(config, cuda)
    assert not report['skipped'], report['skipped']
    assert len(report['patched']) == 4, report
    for s in seeds:
        st = helpers.make_structure(seed=s)
        E0, F0 = helpers.energy_forces(ref, st, cuda)
        E1, F1 = helpers.energy_forces(met, st, cuda)
        dE = abs(E1 - E0)
        dF = np.abs(F1 - F0).max()
        assert dE / len(st) < E_TOL, (config, s, dE)
        assert dF / max(np.abs(F0).max(), 1e-3) < F_TOL, (config, s, dF)
        assert dE <= E_ABS and dF <= F_ABS, (config, s, dE, dF)


@pytest.mark.parametrize('config', list(helpers.CONFIGS))
def test_matches_unpatched_all_configs(cuda, config):
    _check_pair(config, cuda)


def test_patch_is_idempotent_and_reports(cuda):
    from mace_mps_kernels_b200 import patch_model
    _, met, report = helpers.pair('l3_corr3', cuda)
    assert report['patched'] == ['interactions.0.conv_tp', 'interactions.1.conv_tp',
                                 'products.0.symmetric_contractions', 'products.1.symmetric_contractions']
    again = patch_model(met, verbose=False)
    assert again == {'patched': [], 'skipped': []}


def test_rotation_equivariance(cuda):
    _, met, _ = helpers.pair('l3_corr3', cuda)
    st = helpers.make_structure(seed=3)
    R = helpers.random_quaternion_rotation(0)
    E0, F0 = helpers.energy_forces(met, st, cuda)
    E1, F1 = helpers.energy_forces(met, st, cuda, R)
    assert abs(E1 - E0) / len(st) < E_TOL
    assert np.abs(F1 - F0 @ R.T).max() / np.abs(F0).max() < 1e-4


def test_double_backward_raises(cuda):
    _, met, _ = helpers.pair('l3_corr3', cuda)
    b = helpers.batch_for([helpers.make_structure(seed=4)], cuda)
    b['positions'].requires_grad_(True)
    out = met(b, compute_force=False, training=True)
    try:                                   # forces with create_graph=True (as in force training) must refuse
        (f,) = torch.autograd.grad(out['energy'].sum(), b['positions'], create_graph=True)
        torch.autograd.grad(f.sum(), b['positions'])
    except RuntimeError as e:
        assert 'double backward' in str(e), e
        return
    raise AssertionError('double backward did not raise')


def test_unsupported_block_is_skipped(cuda):
    from mace_mps_kernels_b200 import patch_model
    ref = helpers.make_model('48x0e+48x1o', 3, 3).to(cuda)
    met = copy.deepcopy(ref)
    report = patch_model(met, verbose=False)
    assert all('conv_tp' in n for n, _ in report['skipped']) and len(report['skipped']) == 2, report
    assert report['patched'] == ['products.0.symmetric_contractions', 'products.1.symmetric_contractions']
    st = helpers.make_structure(seed=5)
    E0, F0 = helpers.energy_forces(ref, st, cuda)
    E1, F1 = helpers.energy_forces(met, st, cuda)      # symmetric contractions patched, convolutions on torch
    assert abs(E1 - E0) / len(st) < E_TOL
    assert np.abs(F1 - F0).max() / np.abs(F0).max() < F_TOL


def test_batched_structures_match_single(cuda):
    """A batch of several structures (configuration 3's shape) gives each structure's own energy and forces."""
    _, met, _ = helpers.pair('l3_corr3', cuda)
    sts = [helpers.make_structure(seed=s) for s in (6, 7, 8)]
    b = helpers.batch_for(sts, cuda)
    out = met(b)
    off = 0
    for k, st in enumerate(sts):
        E, F = helpers.energy_forces(met, st, cuda)
        assert abs(float(out['energy'][k]) - E) < 1e-4
        assert np.abs(out['forces'][off:off + len(st)].detach().cpu().numpy() - F).max() < 1e-5
        off += len(st)


def test_patch_rejects_cpu_and_double(cuda):
    from mace_mps_kernels_b200 import patch_model
    m = helpers.make_model()
    with pytest.raises(RuntimeError, match='cuda'):
        patch_model(m)
    with pytest.raises(RuntimeError, match='float32'):
        patch_model(m.double().to(cuda))
