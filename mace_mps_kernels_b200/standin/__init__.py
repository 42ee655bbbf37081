"""In-repo stand-in for the parts of mace-torch 0.3.x and e3nn 0.4.x that a patched MACE model uses.

Neither package is installed here (and there is no network), so the model that ``patch_model`` patches, the
unpatched "e3nn path" the kernels are checked against, and the benchmark structures are built from this package.
``make_model`` mirrors the reference test helper (reference ``tests/helpers.py:25-39``): ScaleShiftMACE, r_max 5,
8 Bessel functions, polynomial cutoff p = 5, MLP 16x0e, avg_num_neighbors 20, zero E0, SiLU, 2 interactions (plain
first, residual after), seed-initialised, every parameter then shifted by 0.05 * randn so none stays zero.
"""
from __future__ import annotations

import numpy as np
import torch

from . import o3
from .graph import atoms_to_graph, collate, neighbor_list, pad_edges, to_device
from .modules import ScaleShiftMACE, interaction_classes
from .structures import Z, Structure, ceo2_au13, fcc_bulk, pt100_co_h, pt100_random

ELEMENTS_PTCOH = [1, 6, 8, 78]          # H, C, O, Pt  (benchmark configurations 1-3)
ELEMENTS_TEST = [1, 7, 8, 78]           # H, N, O, Pt  (reference tests/helpers.py:14)


def make_model(hidden='32x0e+32x1o', max_ell=3, correlation=3, seed=0, r_max=5.0, elements=ELEMENTS_PTCOH,
               num_interactions=2, avg_num_neighbors=20.0):
    torch.manual_seed(seed)
    n = len(elements)
    model = ScaleShiftMACE(
        atomic_inter_scale=1.0, atomic_inter_shift=0.0, r_max=r_max, num_bessel=8, num_polynomial_cutoff=5,
        max_ell=max_ell, interaction_cls=interaction_classes['RealAgnosticResidualInteractionBlock'],
        interaction_cls_first=interaction_classes['RealAgnosticInteractionBlock'],
        num_interactions=num_interactions, num_elements=n, hidden_irreps=o3.Irreps(hidden),
        MLP_irreps=o3.Irreps('16x0e'), atomic_energies=np.zeros(n), avg_num_neighbors=avg_num_neighbors,
        atomic_numbers=elements, correlation=correlation)
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.05 * torch.randn_like(p))
    return model.float()


def structure_batch(structures, z_table, r_max, pad_to=None, dtype=torch.float32):
    graphs = [atoms_to_graph(s, z_table, r_max, dtype) for s in structures]
    if pad_to is not None:
        graphs = [pad_edges(g, pad_to) for g in graphs]
    return collate(graphs)


__all__ = ['o3', 'make_model', 'structure_batch', 'ScaleShiftMACE', 'Structure', 'neighbor_list', 'atoms_to_graph',
           'collate', 'pad_edges', 'to_device', 'pt100_co_h', 'pt100_random', 'ceo2_au13', 'fcc_bulk', 'Z',
           'ELEMENTS_PTCOH', 'ELEMENTS_TEST']
