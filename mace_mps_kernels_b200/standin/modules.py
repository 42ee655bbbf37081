"""A mace-torch 0.3.x-shaped ``ScaleShiftMACE`` built from the in-repo e3nn stand-in.

The module tree and attribute names follow mace-torch 0.3.x, because ``patch_model`` introspects them
(reference ``src/mace_mps_kernels/__init__.py:43-75``): ``interactions[i].conv_tp`` (a uvu ``TensorProduct`` with
external per-edge weights), a ``forward`` whose source takes the ``conv_fusion`` branch (
``conv_tp(node_feats, edge_attrs, tp_weights, edge_index)`` -> receiver-summed messages), and
``products[i].symmetric_contractions`` / ``products[i].cueq_config``.  The data flow per interaction is MACE's:
linear_up -> radial MLP weights -> conv (gather, uvu TP, scatter-sum over receivers) -> linear / avg_num_neighbors ->
element-dependent skip TP -> reshape [N, C, (l_max+1)^2] -> symmetric contraction -> linear (+ residual) -> readout.
Energy = per-graph sum of scale-shifted node energies plus E0; forces = -dE/dpositions by autograd.
"""
from __future__ import annotations

import math

import torch

from . import o3
from .symmetric_contraction import SymmetricContraction


def scatter_sum(src, index, dim_size):
    out = src.new_zeros((dim_size,) + src.shape[1:])
    return out.index_add_(0, index, src)


class BesselBasis(torch.nn.Module):
    def __init__(self, r_max, num_basis=8):
        super().__init__()
        self.register_buffer('bessel_weights', math.pi / r_max * torch.arange(1, num_basis + 1, dtype=torch.float32))
        self.register_buffer('prefactor', torch.tensor(math.sqrt(2.0 / r_max)))

    def forward(self, x):                                        # [E, 1] -> [E, num_basis]
        return self.prefactor * torch.sin(self.bessel_weights * x) / x


class PolynomialCutoff(torch.nn.Module):
    def __init__(self, r_max, p=5):
        super().__init__()
        self.register_buffer('r_max', torch.tensor(float(r_max)))
        self.register_buffer('p', torch.tensor(float(p)))

    def forward(self, x):
        p = self.p
        u = x / self.r_max
        env = (1.0 - (p + 1.0) * (p + 2.0) / 2.0 * u ** p + p * (p + 2.0) * u ** (p + 1.0)
               - p * (p + 1.0) / 2.0 * u ** (p + 2.0))
        return env * (x < self.r_max)


class RadialEmbeddingBlock(torch.nn.Module):
    def __init__(self, r_max, num_bessel, num_polynomial_cutoff):
        super().__init__()
        self.bessel_fn = BesselBasis(r_max, num_bessel)
        self.cutoff_fn = PolynomialCutoff(r_max, num_polynomial_cutoff)
        self.out_dim = num_bessel

    def forward(self, edge_lengths):
        return self.bessel_fn(edge_lengths) * self.cutoff_fn(edge_lengths)


class FullyConnectedNet(torch.nn.Module):
    """e3nn-style MLP without biases: h <- act(h @ W / sqrt(fan_in)), no activation after the last layer."""

    _SILU_2MOM = 1.6790177   # 1/sqrt(E[silu(z)^2]) for z ~ N(0,1): keeps the second moment at 1 (normalize2mom)

    def __init__(self, hs, act=torch.nn.functional.silu):
        super().__init__()
        self.hs = list(hs)
        self.act = act
        self.weights = torch.nn.ParameterList(
            [torch.nn.Parameter(torch.randn(a, b)) for a, b in zip(self.hs[:-1], self.hs[1:])])

    def forward(self, x):
        n = len(self.weights)
        for i, w in enumerate(self.weights):
            x = x @ (w / math.sqrt(w.shape[0]))
            if i < n - 1:
                x = self.act(x) * self._SILU_2MOM
        return x


class reshape_irreps(torch.nn.Module):
    """[N, sum mul*(2l+1)] in mul_ir layout -> [N, C, sum (2l+1)] (channel-major), equal multiplicities; mace-torch's
    ``reshape_irreps`` module (mace/modules/irreps_tools.py), held by every interaction block as ``reshape``."""

    def __init__(self, irreps):
        super().__init__()
        self.irreps = o3.Irreps(irreps)
        self.dims = [ir.dim for _, ir in self.irreps]
        self.muls = [mul for mul, _ in self.irreps]

    def forward(self, tensor):
        N = tensor.shape[0]
        parts, ix = [], 0
        for mul, d in zip(self.muls, self.dims):
            parts.append(tensor[:, ix:ix + mul * d].reshape(N, mul, d))
            ix += mul * d
        return torch.cat(parts, dim=-1)


def get_edge_vectors_and_lengths(positions, edge_index, shifts, normalize=False, eps=1e-9):
    """mace-torch's edge geometry (mace/modules/utils.py): vectors receiver - sender + shift and their lengths,
    called from the model's forward through this module's namespace."""
    sender, receiver = edge_index[0], edge_index[1]
    vectors = positions[receiver] - positions[sender] + shifts
    lengths = torch.linalg.norm(vectors, dim=-1, keepdim=True)
    if normalize:
        return vectors / (lengths + eps), lengths
    return vectors, lengths


class _InteractionBase(torch.nn.Module):
    def __init__(self, node_attrs_irreps, node_feats_irreps, edge_attrs_irreps, edge_feats_irreps, target_irreps,
                 hidden_irreps, avg_num_neighbors, radial_MLP=(64, 64, 64)):
        super().__init__()
        self.node_attrs_irreps = o3.Irreps(node_attrs_irreps)
        self.node_feats_irreps = o3.Irreps(node_feats_irreps)
        self.edge_attrs_irreps = o3.Irreps(edge_attrs_irreps)
        self.edge_feats_irreps = o3.Irreps(edge_feats_irreps)
        self.target_irreps = o3.Irreps(target_irreps)
        self.hidden_irreps = o3.Irreps(hidden_irreps)
        self.avg_num_neighbors = avg_num_neighbors
        self.linear_up = o3.Linear(self.node_feats_irreps, self.node_feats_irreps)
        irreps_mid, instructions = o3.tp_out_irreps_with_instructions(
            self.node_feats_irreps, self.edge_attrs_irreps, self.target_irreps)
        self.conv_tp = o3.TensorProduct(self.node_feats_irreps, self.edge_attrs_irreps, irreps_mid,
                                        instructions=instructions, shared_weights=False, internal_weights=False)
        self.conv_tp_weights = FullyConnectedNet([self.edge_feats_irreps.num_irreps] + list(radial_MLP)
                                                 + [self.conv_tp.weight_numel])
        self.irreps_out = self.target_irreps
        self.linear = o3.Linear(irreps_mid, self.irreps_out)
        self.reshape = reshape_irreps(self.irreps_out)

    def _conv(self, node_feats, edge_attrs, tp_weights, edge_index):
        raise NotImplementedError


class RealAgnosticInteractionBlock(_InteractionBase):
    """First interaction: message -> linear -> / avg_num_neighbors -> skip_tp(node_attrs) -> reshape."""

    def __init__(self, *args, **kw):
        super().__init__(*args, **kw)
        self.skip_tp = o3.FullyConnectedTensorProduct(self.irreps_out, self.node_attrs_irreps, self.irreps_out)

    def forward(self, node_attrs, node_feats, edge_attrs, edge_feats, edge_index):
        sender, receiver = edge_index[0], edge_index[1]
        num_nodes = node_feats.shape[0]
        node_feats = self.linear_up(node_feats)
        tp_weights = self.conv_tp_weights(edge_feats)
        if hasattr(self, 'conv_fusion'):
            message = self.conv_tp(node_feats, edge_attrs, tp_weights, edge_index)
        else:
            mji = self.conv_tp(node_feats[sender], edge_attrs, tp_weights)
            message = scatter_sum(mji, receiver, num_nodes)
        message = self.linear(message) / self.avg_num_neighbors
        message = self.skip_tp(message, node_attrs)
        return self.reshape(message), None


class RealAgnosticResidualInteractionBlock(_InteractionBase):
    """Later interactions: the skip TP acts on the incoming node features and is returned as the residual."""

    def __init__(self, *args, **kw):
        super().__init__(*args, **kw)
        self.skip_tp = o3.FullyConnectedTensorProduct(self.node_feats_irreps, self.node_attrs_irreps,
                                                      self.hidden_irreps)

    def forward(self, node_attrs, node_feats, edge_attrs, edge_feats, edge_index):
        sender, receiver = edge_index[0], edge_index[1]
        num_nodes = node_feats.shape[0]
        sc = self.skip_tp(node_feats, node_attrs)
        node_feats = self.linear_up(node_feats)
        tp_weights = self.conv_tp_weights(edge_feats)
        if hasattr(self, 'conv_fusion'):
            message = self.conv_tp(node_feats, edge_attrs, tp_weights, edge_index)
        else:
            mji = self.conv_tp(node_feats[sender], edge_attrs, tp_weights)
            message = scatter_sum(mji, receiver, num_nodes)
        message = self.linear(message) / self.avg_num_neighbors
        return self.reshape(message), sc


interaction_classes = {
    'RealAgnosticInteractionBlock': RealAgnosticInteractionBlock,
    'RealAgnosticResidualInteractionBlock': RealAgnosticResidualInteractionBlock,
}


class EquivariantProductBasisBlock(torch.nn.Module):
    def __init__(self, node_feats_irreps, target_irreps, correlation, use_sc, num_elements):
        super().__init__()
        self.use_sc = use_sc
        self.cueq_config = None
        self.symmetric_contractions = SymmetricContraction(node_feats_irreps, target_irreps, correlation, num_elements)
        self.linear = o3.Linear(target_irreps, target_irreps)

    def forward(self, node_feats, sc, node_attrs):
        node_feats = self.symmetric_contractions(node_feats, node_attrs)
        if self.use_sc and sc is not None:
            return self.linear(node_feats) + sc
        return self.linear(node_feats)


class LinearNodeEmbeddingBlock(torch.nn.Module):
    def __init__(self, irreps_in, irreps_out):
        super().__init__()
        self.linear = o3.Linear(irreps_in, irreps_out)

    def forward(self, node_attrs):
        return self.linear(node_attrs)


class LinearReadoutBlock(torch.nn.Module):
    def __init__(self, irreps_in):
        super().__init__()
        self.linear = o3.Linear(irreps_in, o3.Irreps('0e'))

    def forward(self, x):
        return self.linear(x)


class NonLinearReadoutBlock(torch.nn.Module):
    def __init__(self, irreps_in, MLP_irreps):
        super().__init__()
        self.linear_1 = o3.Linear(irreps_in, MLP_irreps)
        self.linear_2 = o3.Linear(MLP_irreps, o3.Irreps('0e'))

    def forward(self, x):
        return self.linear_2(torch.nn.functional.silu(self.linear_1(x)))


class ScaleShiftMACE(torch.nn.Module):
    def __init__(self, r_max, num_bessel, num_polynomial_cutoff, max_ell, interaction_cls, interaction_cls_first,
                 num_interactions, num_elements, hidden_irreps, MLP_irreps, atomic_energies, avg_num_neighbors,
                 atomic_numbers, correlation, gate=torch.nn.functional.silu, atomic_inter_scale=1.0,
                 atomic_inter_shift=0.0, radial_MLP=(64, 64, 64)):
        super().__init__()
        hidden_irreps = o3.Irreps(hidden_irreps)
        self.register_buffer('atomic_numbers', torch.tensor(list(atomic_numbers), dtype=torch.int64))
        self.register_buffer('r_max', torch.tensor(float(r_max)))
        self.register_buffer('num_interactions', torch.tensor(int(num_interactions)))
        self.register_buffer('atomic_energies', torch.tensor(list(atomic_energies), dtype=torch.float32))
        node_attr_irreps = o3.Irreps([(num_elements, '0e')])
        C = hidden_irreps.count('0e')
        node_feats_irreps = o3.Irreps([(C, '0e')])
        self.node_embedding = LinearNodeEmbeddingBlock(node_attr_irreps, node_feats_irreps)
        self.radial_embedding = RadialEmbeddingBlock(r_max, num_bessel, num_polynomial_cutoff)
        edge_feats_irreps = o3.Irreps(f'{num_bessel}x0e')
        sh_irreps = o3.Irreps.spherical_harmonics(max_ell)
        self.spherical_harmonics = o3.SphericalHarmonics(sh_irreps, normalize=True, normalization='component')
        interaction_irreps = (sh_irreps * C).sort()[0].simplify()
        self.interactions = torch.nn.ModuleList()
        self.products = torch.nn.ModuleList()
        self.readouts = torch.nn.ModuleList()
        for i in range(num_interactions):
            last = i == num_interactions - 1
            hid_out = o3.Irreps([hidden_irreps[0]]) if last else hidden_irreps
            cls = interaction_cls_first if i == 0 else interaction_cls
            inter = cls(node_attr_irreps, node_feats_irreps if i == 0 else hidden_irreps, sh_irreps,
                        edge_feats_irreps, interaction_irreps, hid_out, avg_num_neighbors, radial_MLP)
            self.interactions.append(inter)
            use_sc = i > 0 or 'Residual' in interaction_cls_first.__name__
            self.products.append(EquivariantProductBasisBlock(interaction_irreps, hid_out, correlation, use_sc,
                                                              num_elements))
            self.readouts.append(NonLinearReadoutBlock(hid_out, o3.Irreps(MLP_irreps)) if last
                                 else LinearReadoutBlock(hidden_irreps))
        self.scale = float(atomic_inter_scale)
        self.shift = float(atomic_inter_shift)

    def forward(self, data, compute_force=True, training=False):
        positions = data['positions']
        if compute_force and not positions.requires_grad:
            positions.requires_grad_(True)
        node_attrs, edge_index, shifts = data['node_attrs'], data['edge_index'], data['shifts']
        batch, num_graphs = data['batch'], int(data['num_graphs'])
        node_e0 = node_attrs @ self.atomic_energies
        e0 = scatter_sum(node_e0, batch, num_graphs)
        node_feats = self.node_embedding(node_attrs)
        vectors, lengths = get_edge_vectors_and_lengths(positions=positions, edge_index=edge_index, shifts=shifts)
        edge_attrs = self.spherical_harmonics(vectors)
        edge_feats = self.radial_embedding(lengths)
        node_es = 0.0
        for interaction, product, readout in zip(self.interactions, self.products, self.readouts):
            node_feats, sc = interaction(node_attrs, node_feats, edge_attrs, edge_feats, edge_index)
            node_feats = product(node_feats, sc, node_attrs)
            node_es = node_es + readout(node_feats).squeeze(-1)
        node_inter_es = self.scale * node_es + self.shift
        inter_e = scatter_sum(node_inter_es, batch, num_graphs)
        energy = e0 + inter_e
        out = {'energy': energy, 'node_energy': node_e0 + node_inter_es, 'forces': None}
        if compute_force:
            (g,) = torch.autograd.grad(energy.sum(), positions, create_graph=training, retain_graph=training)
            out['forces'] = -g
        return out
