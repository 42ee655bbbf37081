"""Periodic neighbour list on the GPU (C ABI ``mmk_neighbor_list``): every pair (i, j, S) with
0 < |r_j + S.cell - r_i| < cutoff, in the order and layout MACE's graph uses (``edge_index = [sender i, receiver j]``,
``shifts = S @ cell``, sorted by (i, j, S)), as ``mace_mps_kernels_b200.standin.graph.neighbor_list`` builds it on the
host.

A cell list over wrapped fractional coordinates (float64): atoms binned by a CSR build, one warp per atom walks the
neighbouring (bin, periodic image) pairs, a scan places every atom's edges and a per-atom rank sort orders them.  The
capacity is fixed per ``DeviceNeighborList``, rows past the pair count are padding edges (padding edge k: node k mod N
to itself, far away), and nothing synchronises with the host, so a step that rebuilds the graph can be captured in a
CUDA graph.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib


class DeviceNeighborList:
    """Neighbour list for a fixed cell, periodicity, cutoff, atom count and edge capacity.

    ``lo`` / ``hi``: fractional range binned along non-periodic axes (default: [0, 1]); atoms outside it are still
    found.  ``__call__(positions)`` (device float64 [n_atoms, 3]) returns the static outputs ``(edge_index [2, cap]
    int64, shifts [cap, 3] float32, n_edges [1] int64)``, overwritten by the next call; ``n_edges > capacity`` means
    the capacity was too small (outputs invalid)."""

    def __init__(self, cell, pbc, cutoff, n_atoms, capacity, device, lo=None, hi=None):
        cell = np.asarray(cell, np.float64).reshape(3, 3)
        self._cell = (ctypes.c_double * 9)(*cell.reshape(-1))
        self._pbc = (ctypes.c_int * 3)(*[int(bool(p)) for p in np.broadcast_to(np.asarray(pbc), (3,))])
        self._lo = (ctypes.c_double * 3)(*(np.zeros(3) if lo is None else np.asarray(lo, np.float64)))
        self._hi = (ctypes.c_double * 3)(*(np.ones(3) if hi is None else np.asarray(hi, np.float64)))
        self.cutoff, self.n_atoms, self.capacity = float(cutoff), int(n_atoms), int(capacity)
        nbytes = _lib.lib().mmk_nl_workspace_bytes(self._cell, self._pbc, self.cutoff, self._lo, self._hi,
                                                    self.n_atoms, self.capacity)
        if nbytes == 0:
            raise ValueError('invalid neighbour-list geometry: ' + _lib.lib().mmk_last_error().decode(errors='replace'))
        self.workspace = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
        self.edge_index = torch.empty(2, self.capacity, dtype=torch.long, device=device)
        self.shifts = torch.empty(self.capacity, 3, dtype=torch.float32, device=device)
        self.n_edges = torch.zeros(1, dtype=torch.long, device=device)

    def __call__(self, positions):
        if positions.dtype != torch.float64 or not positions.is_cuda or positions.shape != (self.n_atoms, 3):
            raise TypeError(f'positions must be a float64 CUDA tensor of shape ({self.n_atoms}, 3)')
        positions = positions.contiguous()
        _lib.call('mmk_neighbor_list', _lib.ptr(positions), self.n_atoms, self._cell, self._pbc, self.cutoff,
                  self._lo, self._hi, self.capacity, _lib.ptr(self.edge_index), _lib.ptr(self.shifts),
                  _lib.ptr(self.n_edges), _lib.ptr(self.workspace), self.workspace.numel(),
                  _lib.stream_of(positions))
        return self.edge_index, self.shifts, self.n_edges


def neighbor_list(positions, cell, pbc, cutoff, capacity=None):
    """Convenience form: ``(edge_index [2, E], shifts [E, 3])`` of the pairs, trimmed (reads the pair count back, and
    rebuilds with a larger capacity when the first guess was too small)."""
    n = positions.shape[0]
    cap = int(capacity) if capacity is not None else max(64, 64 * n)
    for _ in range(4):
        nl = DeviceNeighborList(cell, pbc, cutoff, n, cap, positions.device)
        ei, sh, ne = nl(positions)
        E = int(ne.item())
        if E <= cap:
            return ei[:, :E].clone(), sh[:E].clone()
        cap = E
    raise RuntimeError('neighbour list capacity did not converge')
