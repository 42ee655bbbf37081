"""Pins of the float64 oracle and the e3nn-path model that need no GPU: the oracle's backward equals finite
differences of its forward (conv_tp and symmetric contraction), the model's forces equal minus finite differences of
its energy, and energies / forces are rotation invariant / equivariant."""
import numpy as np
import torch

import helpers
from mace_mps_kernels_b200 import standin as S
from oracle import conv_ref, sc_ref


def _fd(f, x, eps=1e-6, idx=None):
    """Central differences of the scalar f at the flat indices idx of x (float64 numpy)."""
    x = np.array(x, np.float64)
    flat = x.reshape(-1)
    out = []
    for i in idx:
        v = flat[i]
        flat[i] = v + eps
        fp = f(x)
        flat[i] = v - eps
        fm = f(x)
        flat[i] = v
        out.append((fp - fm) / (2 * eps))
    return np.array(out)


def test_oracle_conv_backward_is_the_derivative_of_its_forward():
    tp = helpers.conv_tp('8x0e+8x1o', 2)
    spec, coef = conv_ref.probe_coefficients(tp)
    rng = np.random.default_rng(0)
    N, E = 5, 12
    send, recv = rng.integers(0, N, E), rng.integers(0, N, E)
    x = rng.standard_normal((N, spec['x_dim']))
    Y = rng.standard_normal((E, spec['y_dim']))
    W = rng.standard_normal((E, tp.weight_numel))
    g = rng.standard_normal((N, spec['out_dim']))
    gx, gY, gW = conv_ref.conv_bwd(spec, coef, x, Y, W, g, send, recv)
    L = lambda x_, Y_, W_: float((conv_ref.conv_fwd(spec, coef, x_, Y_, W_, send, recv, N) * g).sum())
    for arr, grad, f in ((x, gx, lambda a: L(a, Y, W)), (Y, gY, lambda a: L(x, a, W)), (W, gW, lambda a: L(x, Y, a))):
        idx = rng.choice(arr.size, 12, replace=False)
        num = _fd(f, arr, idx=idx)
        assert np.abs(num - np.asarray(grad).reshape(-1)[idx]).max() < 1e-6 * max(1.0, np.abs(num).max())


def test_oracle_sc_backward_is_the_derivative_of_its_forward():
    m = helpers.make_model('8x0e+8x1o', 3, 3)
    sc = m.products[0].symmetric_contractions
    spec = sc_ref.sc_spec(sc)
    rng = np.random.default_rng(1)
    N = 4
    x = rng.standard_normal((N, spec['C'], spec['n_ell']))
    elem = rng.integers(0, len(helpers.ELEMENTS), N)
    g = rng.standard_normal((N, spec['out_dim']))
    gx = sc_ref.sc_bwd(spec, x, elem, g)
    idx = rng.choice(x.size, 16, replace=False)
    num = _fd(lambda a: float((sc_ref.sc_fwd(spec, a, elem) * g).sum()), x, idx=idx)
    assert np.abs(num - gx.reshape(-1)[idx]).max() < 1e-6 * max(1.0, np.abs(num).max())


def _model64():
    return helpers.make_model('8x0e+8x1o', 3, 3).double().requires_grad_(False)


def _energy_forces(model, st):
    b = S.structure_batch([st], helpers.ELEMENTS, 5.0, dtype=torch.float64)
    out = model(b, compute_force=True)
    return float(out['energy'].detach().sum()), out['forces'].detach().numpy()


def test_model_forces_are_minus_the_energy_gradient():
    model = _model64()
    st = helpers.make_structure(seed=4, n_frag=3)
    E, F = _energy_forces(model, st)
    rng = np.random.default_rng(2)
    atoms = rng.choice(len(st), 4, replace=False)
    eps = 1e-5
    for a in atoms:
        for k in range(3):
            p = st.positions.copy()
            p[a, k] += eps
            Ep, _ = _energy_forces(model, type(st)(p, st.numbers, st.cell, st.pbc))
            p[a, k] -= 2 * eps
            Em, _ = _energy_forces(model, type(st)(p, st.numbers, st.cell, st.pbc))
            assert abs(-(Ep - Em) / (2 * eps) - F[a, k]) < 1e-6 * max(1.0, np.abs(F).max())


def test_model_is_rotation_equivariant():
    model = _model64()
    st = helpers.make_structure(seed=5, n_frag=3)
    R = helpers.random_quaternion_rotation(1)
    E0, F0 = _energy_forces(model, st)
    E1, F1 = _energy_forces(model, st.rotated(R))
    assert abs(E1 - E0) < 1e-9 * max(1.0, abs(E0))
    assert np.abs(F1 - F0 @ R.T).max() < 1e-9 * max(1.0, np.abs(F0).max())
