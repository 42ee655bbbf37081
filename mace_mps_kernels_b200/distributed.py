"""Multi-GPU MACE energy + forces: one process per GPU, torch.distributed (NCCL over NVLink on GPUs, gloo on CPU).

Two decompositions:

* structure batches -- every rank evaluates its own structures (``structures[rank::world]``); the only collective is
  the per-step gather of the energies (``gather_energies``).  See ``bench.py --gpus N``.

* one large system partitioned by receiving atom -- ``partition_graph`` orders the atoms along a Z-order curve and
  gives rank r a contiguous block (its owned atoms, a compact spatial domain).  Rank r keeps every edge whose
  RECEIVER it owns, so the patched convolution (receiver-CSR forward, sender-CSR backward) runs on a local graph
  whose senders are its owned atoms plus a halo of atoms within r_max owned by other ranks.  Per interaction the halo
  rows of the node features are refreshed from their owners (``HaloExchange``: one ``all_to_all_single``); its
  backward sends the halo gradients back and adds them into the owners' rows (the reverse halo), which also carries
  the position gradients of halo atoms home.  The energy is the sum over ranks of owned-atom energies; forces on owned
  atoms are -dE/dx with every rank's contribution included.

``DistributedMACE`` evaluates a ScaleShiftMACE-structured model (this repository's stand-in, patched or not) on one
rank's partition.  Every rank must call it (and the backward) in the same order: the exchanges are collectives.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .standin.graph import neighbor_list
from .standin.modules import RealAgnosticInteractionBlock, scatter_sum
from .standin.structures import morton_order


@dataclass
class Partition:
    rank: int
    world: int
    owned: np.ndarray          # global ids of owned atoms, local order 0..n_own-1
    halo: np.ndarray           # global ids of halo atoms, local order n_own.., grouped by owner rank
    edge_index: np.ndarray     # [2, E_local] (sender local id, receiver local id < n_own)
    shifts: np.ndarray         # [E_local, 3] cartesian shifts (vector = pos[recv] - pos[send] + shift)
    numbers: np.ndarray        # [n_own + n_halo] atomic numbers of the local nodes
    send_idx: np.ndarray       # owned local ids to send, concatenated by destination rank
    send_counts: list          # [world]
    recv_counts: list          # [world] halo atoms received from each rank (the halo blocks, in rank order)

    @property
    def n_own(self):
        return len(self.owned)

    @property
    def n_local(self):
        return len(self.owned) + len(self.halo)


def partition_graph(structure, r_max, world):
    """Partitions of ``structure`` for ranks 0..world-1 (deterministic; every rank can compute all of them)."""
    order = morton_order(structure.positions, structure.cell)
    n = len(order)
    bounds = [(r * n) // world for r in range(world + 1)]
    owner = np.empty(n, np.int64)
    local_of = np.empty(n, np.int64)
    for r in range(world):
        ids = order[bounds[r]:bounds[r + 1]]
        owner[ids] = r
        local_of[ids] = np.arange(len(ids))
    i, j, S = neighbor_list(structure.positions, structure.cell, structure.pbc, r_max)
    shifts = S.astype(np.float64) @ structure.cell
    parts = []
    halos = []
    for r in range(world):
        owned = order[bounds[r]:bounds[r + 1]]
        m = owner[j] == r
        ei, ej, es = i[m], j[m], shifts[m]
        foreign = np.unique(ei[owner[ei] != r])
        # halo grouped by owner rank, then by the owner's local index (the order the owner sends them in)
        key = owner[foreign] * n + local_of[foreign]
        halo = foreign[np.argsort(key, kind='stable')]
        halos.append(halo)
        gl = np.full(n, -1, np.int64)
        gl[owned] = np.arange(len(owned))
        gl[halo] = len(owned) + np.arange(len(halo))
        edge_index = np.stack([gl[ei], gl[ej]])
        numbers = structure.numbers[np.concatenate([owned, halo])]
        recv_counts = [int((owner[halo] == q).sum()) for q in range(world)]
        parts.append(Partition(r, world, owned, halo, edge_index, es, numbers, None, None, recv_counts))
    for r in range(world):
        send, counts = [], []
        for q in range(world):
            blk = halos[q][owner[halos[q]] == r] if q != r else np.zeros(0, np.int64)
            send.append(local_of[blk])
            counts.append(len(blk))
        parts[r].send_idx = np.concatenate(send).astype(np.int64)
        parts[r].send_counts = counts
    return parts


class CommMeter:
    """Optional accounting of the halo exchanges: while ``enabled``, every exchange records CUDA events around its
    collective (on the current stream) and adds the bytes it sends and receives; ``summary()`` synchronises and
    returns (milliseconds inside the collectives, bytes sent, bytes received, exchanges) and resets the counters."""

    def __init__(self):
        self.enabled, self.events, self.sent, self.recv = False, [], 0, 0

    def summary(self):
        ms = 0.0
        if self.events:
            self.events[-1][1].synchronize()
            ms = sum(a.elapsed_time(b) for a, b in self.events)
        out = (ms, self.sent, self.recv, len(self.events))
        self.events, self.sent, self.recv = [], 0, 0
        return out


COMM = CommMeter()


def _all_to_all(out, inp, out_splits, in_splits, group):
    """``all_to_all_single`` into ``out``.  NCCL moves device memory directly; a gloo group (CPU ranks, or ranks
    without NCCL sharing a GPU) moves host memory only, so device tensors are staged through the host."""
    ev = None
    if COMM.enabled and inp.is_cuda:
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        COMM.sent += inp.numel() * inp.element_size()
        COMM.recv += out.numel() * out.element_size()
    _all_to_all_raw(out, inp, out_splits, in_splits, group)
    if ev is not None:
        ev[1].record()
        COMM.events.append(ev)


def _all_to_all_raw(out, inp, out_splits, in_splits, group):
    import torch.distributed as dist
    if inp.is_cuda and dist.get_backend(group) == 'gloo':
        host = torch.empty(out.shape, dtype=out.dtype)
        dist.all_to_all_single(host, inp.cpu(), output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=group)
        out.copy_(host)
    else:
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


class _HaloExchange(torch.autograd.Function):
    """x_owned [n_own, F] -> x_local [n_own + n_halo, F]; backward adds the halo gradients into their owners."""

    @staticmethod
    def forward(ctx, x_own, send_idx, send_counts, recv_counts, group):
        ctx.send_counts, ctx.recv_counts, ctx.group = send_counts, recv_counts, group
        ctx.save_for_backward(send_idx)
        send = x_own.index_select(0, send_idx).contiguous()
        recv = x_own.new_empty((sum(recv_counts),) + tuple(x_own.shape[1:]))
        _all_to_all(recv, send, recv_counts, send_counts, group)
        return torch.cat([x_own, recv], 0)

    @staticmethod
    def backward(ctx, g_local):
        (send_idx,) = ctx.saved_tensors
        n_halo = sum(ctx.recv_counts)
        n_own = g_local.shape[0] - n_halo
        g_halo = g_local[n_own:].contiguous()
        back = g_local.new_empty((sum(ctx.send_counts),) + tuple(g_local.shape[1:]))
        _all_to_all(back, g_halo, ctx.send_counts, ctx.recv_counts, ctx.group)
        g_own = g_local[:n_own].clone()
        g_own.index_add_(0, send_idx, back)
        return g_own, None, None, None, None


class DistributedMACE:
    """Energy + forces of a ScaleShiftMACE-structured model on one rank's ``Partition`` (see module docstring)."""

    def __init__(self, model, part, positions, z_table, device, group=None, dtype=torch.float32):
        self.model, self.part, self.group = model, part, group
        self.device = device
        z_index = {z: k for k, z in enumerate(z_table)}
        idx = torch.tensor([z_index[int(z)] for z in part.numbers])
        self.attrs = torch.nn.functional.one_hot(idx, len(z_table)).to(dtype).to(device)
        self.edge_index = torch.from_numpy(part.edge_index).to(device)
        self.shifts = torch.from_numpy(part.shifts).to(dtype).to(device)
        self.send_idx = torch.from_numpy(part.send_idx).to(device)
        self.positions_own = torch.as_tensor(positions[part.owned], dtype=dtype).to(device)

    def exchange(self, x_own):
        if self.part.world == 1:
            return x_own
        return _HaloExchange.apply(x_own, self.send_idx, self.part.send_counts, self.part.recv_counts, self.group)

    def _conv(self, inter, x, Y, W):
        if hasattr(inter, 'conv_fusion'):
            return inter.conv_tp(x, Y, W, self.edge_index)
        send, recv = self.edge_index[0], self.edge_index[1]
        return scatter_sum(inter.conv_tp(x[send], Y, W), recv, x.shape[0])

    def energy_forces(self, positions_own=None, compute_force=True):
        """(energy of the owned atoms, forces on the owned atoms); sum the energies over ranks for the total."""
        m, n_own = self.model, self.part.n_own
        pos_own = (self.positions_own if positions_own is None else positions_own).detach().requires_grad_(True)
        pos = self.exchange(pos_own)
        send, recv = self.edge_index[0], self.edge_index[1]
        vectors = pos[recv] - pos[send] + self.shifts
        lengths = vectors.norm(dim=-1, keepdim=True)
        Y = m.spherical_harmonics(vectors)
        feats = m.radial_embedding(lengths)
        attrs_own = self.attrs[:n_own]
        node_feats = m.node_embedding(self.attrs)
        node_es = 0.0
        for k, (inter, prod, readout) in enumerate(zip(m.interactions, m.products, m.readouts)):
            if k > 0:
                node_feats = self.exchange(node_feats_own)
            x = inter.linear_up(node_feats)
            W = inter.conv_tp_weights(feats)
            msg = self._conv(inter, x, Y, W)[:n_own]
            msg = inter.linear(msg) / inter.avg_num_neighbors
            if isinstance(inter, RealAgnosticInteractionBlock):
                msg = inter.skip_tp(msg, attrs_own)
                sc = None
            else:
                sc = inter.skip_tp(node_feats[:n_own], attrs_own)
            node_feats_own = prod(inter.reshape(msg), sc, attrs_own)
            node_es = node_es + readout(node_feats_own).squeeze(-1)
        node_energy = attrs_own @ m.atomic_energies.to(attrs_own.dtype) + m.scale * node_es + m.shift
        energy = node_energy.sum()
        forces = None
        if compute_force:
            (g,) = torch.autograd.grad(energy, pos_own)
            forces = -g
        return energy, forces


def gather_energies(energy, world, group=None):
    """all_gather of one scalar per rank (the only collective of the structure-batch decomposition)."""
    import torch.distributed as dist
    out = torch.zeros(world, dtype=energy.dtype, device=energy.device)
    dist.all_gather_into_tensor(out, energy.detach().reshape(1), group=group)
    return out
