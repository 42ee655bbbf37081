"""Structure relaxation loop: limited-memory BFGS over energy + force calls at a fixed padded graph size.

This drives the patched model the way a geometry optimiser drives a MACE calculator (50 E+F calls
of an 89-element model on an Au13 cluster over CeO2(111)):

* the graph is rebuilt every step on the GPU by ``DeviceNeighborList`` (float64 positions, fixed edge capacity,
  padding edges carry zero messages), so the shapes never change;
* the E+F call is a replay of one CUDA graph (``GraphedEnergyForces``) when ``graphed`` is set, else the eager model;
* the optimiser runs on the host in float64, as atomistic optimisers do: one force read-back and one position upload
  per step.

The optimiser is the two-loop L-BFGS recursion (Nocedal and Wright, Numerical Optimization, algorithm 7.4) with a
constant initial inverse Hessian ``1 / alpha`` and a step scaled so that no atom moves further than ``maxstep``
(Angstrom), the variant common in atomistic codes.  Curvature pairs with s.y <= 0 are not stored.
"""
from __future__ import annotations

import numpy as np
import torch

from . import standin
from .graphs import GraphedEnergyForces
from .neighbors import DeviceNeighborList


class Relaxation:
    """L-BFGS relaxation of one structure with ``model`` (a float32 MACE model on ``device``).

    ``capacity``: fixed number of edges of the padded graph (must hold every step's pairs).  The loop runs a fixed
    number of calls (no convergence test), so that its cost is fixed."""

    def __init__(self, model, structure, z_table, r_max, device, capacity, graphed=True, maxstep=0.2, alpha=70.0,
                 memory=100):
        self.model, self.device = model, torch.device(device)
        self.maxstep, self.h0, self.memory = float(maxstep), 1.0 / float(alpha), int(memory)
        n = len(structure)
        self.n_atoms = n
        z_index = {z: k for k, z in enumerate(z_table)}
        idx = torch.tensor([z_index[int(z)] for z in structure.numbers])
        self.node_attrs = torch.nn.functional.one_hot(idx, len(z_table)).float().to(self.device)
        self.nl = DeviceNeighborList(structure.cell, structure.pbc, r_max, n, capacity, self.device)
        self.pos = np.array(structure.positions, dtype=np.float64)              # host, float64 (the optimiser's)
        self.pos_host = torch.zeros(n, 3, dtype=torch.float64).pin_memory()
        self.pos_dev = torch.zeros(n, 3, dtype=torch.float64, device=self.device)
        self.forces_host = torch.zeros(n, 3, dtype=torch.float32).pin_memory()
        self.batch_index = torch.zeros(n, dtype=torch.long, device=self.device)
        self.graphed = None
        if graphed:
            self.graphed = GraphedEnergyForces(model, self._batch())
        self.S, self.Y = [], []                            # curvature pairs, oldest first
        self.r0 = self.g0 = None

    def _batch(self):
        self.pos_host.numpy()[:] = self.pos
        self.pos_dev.copy_(self.pos_host, non_blocking=True)
        ei, sh, _ = self.nl(self.pos_dev)
        return {'positions': self.pos_dev.float(), 'node_attrs': self.node_attrs, 'edge_index': ei, 'shifts': sh,
                'batch': self.batch_index, 'num_graphs': 1}

    def energy_forces(self):
        """(energy [1] float32, forces [n, 3] float32) at the current positions, on the device."""
        b = self._batch()
        if self.graphed is not None:
            return self.graphed(b)
        b = dict(b)
        b['positions'] = b['positions'].detach().requires_grad_(True)
        out = self.model(b, compute_force=True, training=False)
        return out['energy'].detach(), out['forces'].detach()

    def _direction(self, g):
        """-H g by the two-loop recursion over the stored pairs (newest first, then oldest first)."""
        q = g.copy()
        alphas = []
        for s, y in zip(reversed(self.S), reversed(self.Y)):
            rho = 1.0 / float(y @ s)
            a = rho * float(s @ q)
            q -= a * y
            alphas.append((rho, a))
        z = self.h0 * q
        for (s, y), (rho, a) in zip(zip(self.S, self.Y), reversed(alphas)):
            z += s * (a - rho * float(y @ z))
        return -z

    def step(self):
        """One E+F call and one L-BFGS update of the positions; returns (energy, forces) of the call (device)."""
        E, F = self.energy_forces()
        self.forces_host.copy_(F)                          # the one read-back of the step (synchronises)
        g = -self.forces_host.numpy().astype(np.float64).reshape(-1)
        r = self.pos.reshape(-1)
        if self.r0 is not None:
            s, y = r - self.r0, g - self.g0
            if float(s @ y) > 0.0:                         # keep only pairs of positive curvature
                self.S.append(s)
                self.Y.append(y)
                if len(self.S) > self.memory:
                    del self.S[0], self.Y[0]
        dr = self._direction(g).reshape(-1, 3)
        longest = float(np.sqrt((dr * dr).sum(1)).max())
        if longest > self.maxstep:
            dr *= self.maxstep / longest
        self.r0, self.g0 = r.copy(), g
        self.pos = self.pos + dr
        return E, F

    def run(self, calls):
        """``calls`` E+F calls (each followed by an update); returns the energies [calls] (float64, on the device)
        and the forces of the last call."""
        energies = torch.empty(calls, dtype=torch.float64, device=self.device)
        F = None
        for t in range(calls):
            E, F = self.step()
            energies[t] = E.double().reshape(-1)[0]
        return energies, F.clone()


def ceo2_au13_workload(device, seed=0, r_max=6.0, capacity_margin=1.3):
    """89-element random MACE (128x0e+128x1o, l_max 3, correlation 3, r_max 6 A, elements Z = 1..89)
    and the CeO2(111) + Au13 structure; returns (model, structure, z_table, capacity)."""
    z_table = list(range(1, 90))
    model = standin.make_model('128x0e+128x1o', 3, 3, seed=seed, r_max=r_max, elements=z_table).to(device)
    model.requires_grad_(False)
    st = standin.ceo2_au13(seed=seed)
    i, _, _ = standin.neighbor_list(st.positions, st.cell, st.pbc, r_max)
    capacity = int(len(i) * capacity_margin) // 32 * 32 + 32
    return model, st, z_table, capacity
