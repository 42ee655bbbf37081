"""CUDA-graph capture of a whole energy + force call at a fixed (padded) graph size.

An E+F call of a patched MACE model is a few hundred short kernels (the patched conv / symmetric-contraction kernels
plus the PyTorch remainder: embeddings, radial MLP, linears, readouts, autograd), so at production sizes the host
launch path, not the GPU, sets the step time.  ``GraphedEnergyForces`` records one call into a ``torch.cuda.CUDAGraph``
on static input buffers; every call copies the new inputs in (positions, and for a changing neighbour list the
padded edge_index / shifts) and replays the graph.  The graph contains the device CSR builds, so a replay with a new
edge_index is correct.  Keep the number of nodes and edges fixed across calls (``standin.pad_edges`` pads with
zero-message edges), which is what the reference's README recommends for long runs as well.
"""
from __future__ import annotations

import torch

from . import _lib
from .conv import invalidate_graph_caches as _clear_caches


class GraphedEnergyForces:
    """Callable ``(batch) -> (energy [G], forces [N, 3])`` replaying a captured E+F call of ``model``.

    ``batch`` (dict of device tensors with MACE's keys) fixes the shapes; the returned tensors are static buffers
    overwritten by the next call (clone them to keep a result)."""

    INPUT_KEYS = ('positions', 'node_attrs', 'edge_index', 'shifts', 'batch')

    def __init__(self, model, batch, warmup=3):
        self.model = model
        self.num_graphs = int(batch['num_graphs'])
        self.static = {k: batch[k].detach().clone() for k in self.INPUT_KEYS}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._run()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        _clear_caches()                 # the CSR / element index must be rebuilt inside the graph on every replay
        self.graph = torch.cuda.CUDAGraph()
        before = sum(_lib.LAUNCHES.values())
        with torch.cuda.graph(self.graph):
            self.energy, self.forces = self._run()
        self.kernels_per_replay = sum(_lib.LAUNCHES.values()) - before     # this library's kernels in the graph
        _clear_caches()

    def _run(self):
        b = {k: v for k, v in self.static.items()}
        b['positions'] = self.static['positions'].detach().requires_grad_(True)
        b['num_graphs'] = self.num_graphs
        out = self.model(b, compute_force=True, training=False)
        return out['energy'].detach(), out['forces'].detach()

    def __call__(self, batch=None):
        if batch is not None:
            for k in self.INPUT_KEYS:
                v = batch[k]
                if v.shape != self.static[k].shape:
                    raise ValueError(f'{k}: shape {tuple(v.shape)} differs from the captured {tuple(self.static[k].shape)}'
                                     ' (pad to a fixed size)')
                self.static[k].copy_(v, non_blocking=True)
        self.graph.replay()
        return self.energy, self.forces
