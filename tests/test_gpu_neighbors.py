"""GPU: the device neighbour list (DeviceNeighborList, C ABI mmk_neighbor_list) equals the host neighbour list edge for
edge (same order, same shifts), pads the unused capacity, reports overflow, replays inside a CUDA graph, and a model
evaluated on the device-built graph gives the host graph's energy and forces."""
import numpy as np
import pytest
import torch

import helpers
from mace_mps_kernels_b200 import standin as S
from mace_mps_kernels_b200.standin import structures as S_
from mace_mps_kernels_b200.standin.graph import neighbor_list
from mace_mps_kernels_b200.standin.structures import Structure

pytestmark = pytest.mark.gpu


def _skewed():
    rng = np.random.default_rng(5)
    cell = np.array([[7.1, 0.0, 0.0], [3.2, 6.4, 0.0], [-1.9, 2.2, 8.3]])
    return Structure(rng.uniform(-0.2, 1.2, (60, 3)) @ cell, np.full(60, 29), cell, np.array([True, True, True]))


def _slab_open_z():
    rng = np.random.default_rng(6)
    pos = rng.uniform(0, 1, (80, 3)) * [12.0, 11.0, 9.0] + [0, 0, 8.0]
    return Structure(pos, np.full(80, 8), np.diag([12.0, 11.0, 30.0]), np.array([True, True, False]))


CASES = {
    'slab_adsorbates': (lambda: helpers.make_structure(seed=3), 5.0, None),
    'bench_slab': (lambda: S_.pt100_random(seed=1), 5.0, None),
    'bulk_cu_4': (lambda: S_.fcc_bulk('Cu', n=4, seed=2), 5.0, None),
    'thin_cell': (lambda: S_.fcc_bulk('Cu', n=1, seed=3), 5.0, None),
    'skewed': (_skewed, 4.5, None),
    'open_z': (_slab_open_z, 5.0, ((0, 0, 0.3), (1, 1, 0.5))),
}


def _run(cuda, st, cutoff, cap, rng=None):
    from mace_mps_kernels_b200.neighbors import DeviceNeighborList
    lo, hi = rng if rng is not None else (None, None)
    nl = DeviceNeighborList(st.cell, st.pbc, cutoff, len(st), cap, cuda, lo=lo, hi=hi)
    return nl, nl(torch.tensor(st.positions, dtype=torch.float64, device=cuda))


@pytest.mark.parametrize('name', list(CASES))
def test_device_neighbor_list_matches_host(cuda, name):
    make, cutoff, rng = CASES[name]
    st = make()
    i, j, Sh = neighbor_list(st.positions, st.cell, st.pbc, cutoff)
    E = len(i)
    _, (ei, sh, ne) = _run(cuda, st, cutoff, E + 100, rng)
    assert int(ne.item()) == E
    assert np.array_equal(ei[0, :E].cpu().numpy(), i) and np.array_equal(ei[1, :E].cpu().numpy(), j)
    ref = (Sh.astype(np.float64) @ st.cell).astype(np.float32)
    assert np.abs(sh[:E].cpu().numpy() - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
    pad = torch.arange(ei.shape[1] - E, device=ei.device) % len(st)        # padding edge k: node k mod N
    assert bool((ei[0, E:] == pad).all()) and bool((ei[1, E:] == pad).all())
    assert bool((sh[E:, 0] == 1000.0).all()) and bool((sh[E:, 1:] == 0).all())


def test_overflow_is_reported(cuda):
    st = helpers.make_structure(seed=4)
    E = len(neighbor_list(st.positions, st.cell, st.pbc, 5.0)[0])
    _, (_, _, ne) = _run(cuda, st, 5.0, E // 2)
    assert int(ne.item()) == E                       # > capacity: the caller must rebuild with a larger one


def test_graph_capture_rebuilds_the_list(cuda):
    st = helpers.make_structure(seed=5)
    nl, _ = _run(cuda, st, 5.0, 4000)
    pos = torch.tensor(st.positions, dtype=torch.float64, device=cuda)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        nl(pos)
    moved = st.copy()
    moved.positions = moved.positions + np.random.default_rng(0).normal(0, 0.2, moved.positions.shape)
    pos.copy_(torch.tensor(moved.positions, dtype=torch.float64))
    g.replay()
    torch.cuda.synchronize()
    i, j, Sh = neighbor_list(moved.positions, moved.cell, moved.pbc, 5.0)
    E = len(i)
    assert int(nl.n_edges.item()) == E
    assert np.array_equal(nl.edge_index[0, :E].cpu().numpy(), i)
    assert np.array_equal(nl.edge_index[1, :E].cpu().numpy(), j)
    del g


def test_model_on_device_graph(cuda):
    from mace_mps_kernels_b200.neighbors import neighbor_list as device_neighbor_list
    _, met, _ = helpers.pair('l3_corr3', cuda)
    st = helpers.make_structure(seed=6)
    b = S.to_device(S.structure_batch([st], helpers.ELEMENTS, 5.0), cuda)
    ei, sh = device_neighbor_list(torch.tensor(st.positions, dtype=torch.float64, device=cuda), st.cell, st.pbc, 5.0)
    b2 = dict(b)
    b2['edge_index'], b2['shifts'] = ei, sh
    o1, o2 = met(dict(b)), met(b2)
    assert torch.equal(ei.cpu(), b['edge_index'].cpu())
    assert abs(float(o1['energy'].detach().sum()) - float(o2['energy'].detach().sum())) < 1e-6
    assert float((o1['forces'] - o2['forces']).abs().max()) < 1e-6
