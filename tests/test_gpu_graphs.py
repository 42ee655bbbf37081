"""GPU: a CUDA-graphed E+F call (GraphedEnergyForces) equals the eager patched call, also after new positions and a
new (padded) neighbour list are copied into the captured inputs."""
import numpy as np
import pytest

import helpers
from mace_mps_kernels_b200 import standin as S

pytestmark = pytest.mark.gpu


def test_graphed_matches_eager(cuda):
    from mace_mps_kernels_b200.graphs import GraphedEnergyForces
    _, met, _ = helpers.pair('l3_corr3', cuda)
    sts = [helpers.make_structure(seed=s) for s in (10, 11)]
    pad = 3000
    batches = []
    for st in sts:
        b = S.structure_batch([st], helpers.ELEMENTS, 5.0, pad_to=pad)
        batches.append(S.to_device(b, cuda))
    b0 = batches[0]
    g = GraphedEnergyForces(met, b0)
    E, F = g(b0)
    E, F = E.clone(), F.clone()          # the graph's outputs are static buffers, overwritten by the next call
    out = met(dict(b0))
    assert abs(float(E.sum()) - float(out['energy'].detach().sum())) < 1e-4
    assert float((F - out['forces']).abs().max()) < 1e-5
    # same atoms, displaced positions and a rebuilt (padded) neighbour list
    st2 = sts[0].copy()
    st2.positions = st2.positions + np.random.default_rng(0).normal(0, 0.05, st2.positions.shape)
    b2 = S.to_device(S.structure_batch([st2], helpers.ELEMENTS, 5.0, pad_to=pad), cuda)
    E2, F2 = g(b2)
    E2, F2 = E2.clone(), F2.clone()
    out2 = met(dict(b2))
    assert abs(float(E2.sum()) - float(out2['energy'].detach().sum())) < 1e-4
    assert float((F2 - out2['forces']).abs().max()) < 1e-5
    assert float((F2 - F).abs().max()) > 1e-4            # it did recompute
    assert g.kernels_per_replay >= 17


def test_padding_edges_do_not_change_results(cuda):
    _, met, _ = helpers.pair('l3_corr3', cuda)
    st = helpers.make_structure(seed=12)
    b = S.to_device(S.structure_batch([st], helpers.ELEMENTS, 5.0), cuda)
    bp = S.to_device(S.structure_batch([st], helpers.ELEMENTS, 5.0, pad_to=b['edge_index'].shape[1] + 257), cuda)
    o, op = met(dict(b)), met(dict(bp))
    assert abs(float(o['energy'].detach().sum()) - float(op['energy'].detach().sum())) < 1e-5
    assert float((o['forces'] - op['forces']).abs().max()) < 1e-6


def test_graphed_all_extensions_matches_eager(cuda):
    """The bench's patch set (edge features, linears, fused radial MLP; frozen weights) captured in a graph replays
    to the eager result, and replays are bit-identical."""
    from mace_mps_kernels_b200 import patch_model
    from mace_mps_kernels_b200.graphs import GraphedEnergyForces
    hidden, lmax, corr, seed = helpers.CONFIGS['l3_corr3']
    met = helpers.make_model(hidden, lmax, corr, seed).to(cuda).requires_grad_(False)
    rep = patch_model(met, verbose=False, edge_features=True, linears=True)
    assert not rep['skipped'], rep['skipped']
    b0 = S.to_device(S.structure_batch([helpers.make_structure(seed=13)], helpers.ELEMENTS, 5.0, pad_to=3000), cuda)
    g = GraphedEnergyForces(met, b0)
    for _ in range(3):
        E, F = g(b0)
    E, F = E.clone(), F.clone()
    out = met(dict(b0))
    assert abs(float(E.sum()) - float(out['energy'].detach().sum())) < 1e-4
    assert float((F - out['forces']).abs().max()) < 1e-5
    assert float((g(b0)[1] - F).abs().max()) == 0.0        # replays are deterministic
