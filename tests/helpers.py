"""Shared fixtures for the tests: random stand-in MACE models and synthetic structures.

Mirrors reference tests/helpers.py: random models (r_max 5, 8 Bessel, p = 5, MLP 16x0e, avg_num_neighbors 20, zero
E0, 2 interactions, every parameter shifted by 0.05 randn) and Pt(100) slabs decorated with N/O/H fragments.
"""
from __future__ import annotations

import copy

import numpy as np
import torch

from mace_mps_kernels_b200 import standin as S
from mace_mps_kernels_b200.standin.structures import Structure, Z, fcc100_slab

ELEMENTS = S.ELEMENTS_TEST           # H, N, O, Pt

# name: (hidden_irreps, max_ell, correlation).  The reference's reduced / full CG variants of the first entry map to
# one basis here (the stand-in builds one orthonormal symmetric basis), so a second seed stands in for the full-CG one.
CONFIGS = {
    'l3_corr3': ('32x0e+32x1o', 3, 3, 0),
    'l3_corr3_seed1': ('32x0e+32x1o', 3, 3, 1),
    'l2_corr2_scalar': ('64x0e', 2, 2, 0),
    'l3_corr3_l2hidden': ('32x0e+32x1o+32x2e', 3, 3, 0),
}

E_TOL = 1e-5        # eV per atom (reference tests/test_kernels.py:19)
F_TOL = 1e-5        # relative to the largest force component (reference tests/test_kernels.py:20)
F_ABS = 1e-5        # eV/A, absolute bound from the build's north star
E_ABS = 1e-3        # eV per structure


def make_model(hidden='32x0e+32x1o', max_ell=3, correlation=3, seed=0):
    return S.make_model(hidden, max_ell, correlation, seed=seed, elements=ELEMENTS)


def make_structure(seed=0, n_frag=10):
    """4x4x3 Pt(100) slab (a = 3.92 A, 8 A vacuum both sides, fully periodic) with random NH3/NH2/NH/N/OH/O fragments
    1.2-2.2 A above the surface (min distance 1.6 A), as reference tests/helpers.py:56-78 builds with ASE."""
    rng = np.random.default_rng(seed)
    slab = fcc100_slab('Pt', 3.92, 4, 4, 3, 16.0)
    slab.positions[:, 2] += 8.0
    slab.pbc = np.array([True, True, True])
    ztop = slab.positions[:, 2].max()
    frags = [
        (['N', 'H', 'H', 'H'], [[0, 0, 0], [0.94, 0, 0.38], [-0.47, 0.81, 0.38], [-0.47, -0.81, 0.38]]),
        (['N', 'H', 'H'], [[0, 0, 0], [0.8, 0, 0.6], [-0.8, 0, 0.6]]),
        (['N', 'H'], [[0, 0, 0], [0, 0, 1.03]]),
        (['N'], [[0, 0, 0]]),
        (['O', 'H'], [[0, 0, 0], [0, 0, 0.98]]),
        (['O'], [[0, 0, 0]]),
    ]
    pos = list(slab.positions)
    nums = list(slab.numbers)
    n_slab = len(nums)
    tries = 0
    while len(nums) - n_slab < 3 * n_frag and tries < 2000:
        tries += 1
        sym, fp = frags[rng.integers(len(frags))]
        fp = np.array(fp, float)
        th = np.deg2rad(rng.uniform(0, 360))
        R = np.array([[np.cos(th), -np.sin(th), 0], [np.sin(th), np.cos(th), 0], [0, 0, 1]])
        fp = fp @ R.T
        xy = rng.uniform(0, 1, 2) @ slab.cell[:2, :2]
        fp = fp + np.array([xy[0], xy[1], ztop + rng.uniform(1.2, 2.2)]) - fp[0]
        cur = np.array(pos)
        d = fp[:, None, :] - cur[None]
        for ax in range(3):
            L = slab.cell[ax, ax]
            d[..., ax] -= L * np.round(d[..., ax] / L)
        if np.linalg.norm(d, axis=-1).min() > 1.6:
            pos += list(fp)
            nums += [Z[s] for s in sym]
    return Structure(np.array(pos), np.array(nums), slab.cell.copy(), np.array([True, True, True]))


def batch_for(structures, device, r_max=5.0):
    b = S.structure_batch(structures, ELEMENTS, r_max)
    return S.to_device(b, device)


def energy_forces(model, structure, device, R=None):
    st = structure if R is None else structure.rotated(R)
    b = batch_for([st], device)
    out = model(b, compute_force=True, training=False)
    return float(out['energy'].detach().sum()), out['forces'].detach().cpu().double().numpy()


def pair(config, device, **patch_kw):
    """(reference model, patched deep copy, report) for a CONFIGS entry."""
    from mace_mps_kernels_b200 import patch_model
    hidden, lmax, corr, seed = CONFIGS[config]
    ref = make_model(hidden, lmax, corr, seed).to(device)
    met = copy.deepcopy(ref)
    report = patch_model(met, verbose=False, **patch_kw)
    return ref, met, report


def random_quaternion_rotation(seed=0):
    rng = np.random.default_rng(seed)
    return S.o3.rotation_from_quaternion(rng.normal(size=4))


def conv_tp(hidden='32x0e+32x1o', lmax=3, C=None):
    """A stand-in conv_tp exactly as MACE builds it for node features ``hidden`` (second interaction)."""
    from mace_mps_kernels_b200.standin import o3
    hidden = o3.Irreps(hidden)
    C = hidden[0].mul if C is None else C
    sh = o3.Irreps.spherical_harmonics(lmax)
    target = (sh * C).sort()[0].simplify()
    irreps_mid, ins = o3.tp_out_irreps_with_instructions(hidden, sh, target)
    return o3.TensorProduct(hidden, sh, irreps_mid, ins, shared_weights=False, internal_weights=False)


def random_graph(n_nodes, n_edges, seed=0, isolated=()):
    """Random edge_index [2, E] (int64) with the given nodes never receiving nor sending."""
    rng = np.random.default_rng(seed)
    allowed = np.setdiff1d(np.arange(n_nodes), np.asarray(isolated, int))
    send = rng.choice(allowed, n_edges)
    recv = rng.choice(allowed, n_edges)
    return torch.from_numpy(np.stack([send, recv]).astype(np.int64))
