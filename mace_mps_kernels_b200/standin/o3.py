"""Minimal e3nn-style O(3) toolkit: irreps, real spherical harmonics, Clebsch-Gordan tensors, and the three
equivariant layers MACE builds from them (``Linear``, uvu ``TensorProduct``, ``FullyConnectedTensorProduct``).

mace-torch and e3nn are not installed in this environment, so this module restates the pieces of them that a MACE
0.3.x model needs, written from the mathematics:

* real spherical harmonics, 'component' normalisation (sum_m Y_lm(r)^2 = 2l+1 for |r| = 1), m = -l..l, built from
  (x + i y)^m and the associated-Legendre recursion so the code is polynomial and differentiable everywhere;
* Wigner D matrices of that basis, fitted from the harmonics themselves (Y_l(R r) = D_l(R) Y_l(r));
* real Clebsch-Gordan tensors C[l1,l2,l3] = the unit-norm invariant of D_l1 (x) D_l2 (x) D_l3 (sign fixed so the first
  entry above 1e-6 in C-order is positive), the role e3nn's ``wigner_3j`` plays;
* a weighted 'uvu' tensor product with e3nn's 'component' irrep normalisation and 'element' path normalisation
  (path coefficient sqrt((2 l_out + 1) / fan_in)), which is the ``conv_tp`` the kernels replace.

Only the attributes that ``patch_model`` and the reference's ``ConvSpec`` read are part of the contract: ``instructions``
(``i_in1, i_in2, i_out, connection_mode, has_weight``), ``irreps_in1/in2/out`` (iterables of ``(mul, ir)`` with
``ir.l``), ``shared_weights``, ``internal_weights``, ``weight_numel``, ``buffers()`` and ``tp(x1, x2, w)``
(reference ``src/mace_mps_kernels/conv.py:31-88``).
"""
from __future__ import annotations

import functools
import math
import re
from collections import namedtuple
from typing import List, Sequence, Tuple

import numpy as np
import torch

# ----------------------------------------------------------------------------------------------------------------------
# irreps
# ----------------------------------------------------------------------------------------------------------------------


class Irrep(namedtuple('Irrep', ['l', 'p'])):
    """Irreducible representation of O(3): degree ``l`` and parity ``p`` (+1 even, -1 odd)."""

    def __new__(cls, l, p=None):
        if isinstance(l, Irrep):
            return l
        if isinstance(l, str):
            m = re.fullmatch(r'\s*(\d+)([eo])\s*', l)
            if not m:
                raise ValueError(f'bad irrep {l!r}')
            return super().__new__(cls, int(m.group(1)), 1 if m.group(2) == 'e' else -1)
        if isinstance(l, tuple):
            l, p = l
        return super().__new__(cls, int(l), int(p))

    @property
    def dim(self):
        return 2 * self.l + 1

    def __mul__(self, other):
        """Irreps appearing in the tensor product of two irreps."""
        other = Irrep(other)
        p = self.p * other.p
        return [Irrep(l, p) for l in range(abs(self.l - other.l), self.l + other.l + 1)]

    def __repr__(self):
        return f'{self.l}{"e" if self.p == 1 else "o"}'

    __str__ = __repr__


class MulIr(namedtuple('MulIr', ['mul', 'ir'])):
    @property
    def dim(self):
        return self.mul * self.ir.dim

    def __repr__(self):
        return f'{self.mul}x{self.ir}'


class Irreps(tuple):
    """Direct sum of irreps with multiplicities, e.g. ``Irreps('32x0e+32x1o')``; iterates as ``(mul, ir)`` pairs."""

    def __new__(cls, spec=()):
        if isinstance(spec, Irreps):
            return spec
        items = []
        if isinstance(spec, str):
            for part in spec.split('+'):
                part = part.strip()
                if not part:
                    continue
                if 'x' in part:
                    mul, ir = part.split('x')
                    items.append(MulIr(int(mul), Irrep(ir)))
                else:
                    items.append(MulIr(1, Irrep(part)))
        else:
            for x in spec:
                if isinstance(x, MulIr):
                    items.append(x)
                elif isinstance(x, Irrep):
                    items.append(MulIr(1, x))
                else:
                    mul, ir = x
                    items.append(MulIr(int(mul), Irrep(ir)))
        return super().__new__(cls, items)

    @property
    def dim(self):
        return sum(m.dim for m in self)

    @property
    def num_irreps(self):
        return sum(m.mul for m in self)

    @property
    def lmax(self):
        return max(ir.l for _, ir in self)

    def slices(self) -> List[slice]:
        out, off = [], 0
        for m in self:
            out.append(slice(off, off + m.dim))
            off += m.dim
        return out

    def sort(self):
        """(sorted irreps, p, inv) with p[i_old] = i_new; stable sort by (l, p)."""
        key = [(ir.l, ir.p, i) for i, (_, ir) in enumerate(self)]
        order = sorted(range(len(self)), key=lambda i: key[i])
        inv = order
        p = [0] * len(self)
        for new, old in enumerate(order):
            p[old] = new
        return Irreps([self[i] for i in order]), tuple(p), tuple(inv)

    def simplify(self):
        out = []
        for mul, ir in self:
            if out and out[-1][1] == ir:
                out[-1] = (out[-1][0] + mul, ir)
            elif mul > 0:
                out.append((mul, ir))
        return Irreps(out)

    def __add__(self, other):
        return Irreps(tuple(self) + tuple(Irreps(other)))

    def __mul__(self, k: int):
        """``Irreps * k`` multiplies every multiplicity (as e3nn does for ``sh_irreps * num_features``)."""
        return Irreps([(mul * k, ir) for mul, ir in self])

    def count(self, ir):
        ir = Irrep(ir)
        return sum(mul for mul, i in self if i == ir)

    def __contains__(self, ir):
        ir = Irrep(ir)
        return any(i == ir for _, i in self)

    def __repr__(self):
        return '+'.join(repr(m) for m in self)

    __str__ = __repr__

    @staticmethod
    def spherical_harmonics(lmax, p=-1):
        return Irreps([(1, Irrep(l, p ** l)) for l in range(lmax + 1)])


# ----------------------------------------------------------------------------------------------------------------------
# real spherical harmonics
# ----------------------------------------------------------------------------------------------------------------------


@functools.lru_cache(maxsize=None)
def _sh_norms(lmax):
    n = {}
    for l in range(lmax + 1):
        for m in range(l + 1):
            v = (2 * l + 1) * math.factorial(l - m) / math.factorial(l + m)
            n[l, m] = math.sqrt(v) * (math.sqrt(2.0) if m else 1.0)
    return n


def spherical_harmonics(lmax: int, vec: torch.Tensor, normalize: bool = True) -> torch.Tensor:
    """Real spherical harmonics Y_lm(vec) for l = 0..lmax, 'component' normalised, shape [..., (lmax+1)^2].

    Y_l,m>0 = N_lm P~_l^m(z) Re (x+iy)^m,  Y_l,m<0 = N_l|m| P~_l^|m|(z) Im (x+iy)^|m|,  Y_l0 = N_l0 P~_l^0(z), where
    P~_l^m = P_l^m / sin^m(theta) (no Condon-Shortley phase) follows the three-term Legendre recursion.
    """
    if normalize:
        vec = vec / vec.norm(dim=-1, keepdim=True)
    x, y, z = vec.unbind(-1)
    one = torch.ones_like(z)
    A, B = [one], [torch.zeros_like(z)]
    for m in range(1, lmax + 1):
        A.append(x * A[m - 1] - y * B[m - 1])
        B.append(x * B[m - 1] + y * A[m - 1])
    P = {}
    dfact = 1.0
    for m in range(lmax + 1):
        if m > 0:
            dfact *= (2 * m - 1)
        P[m, m] = one * dfact
        if m + 1 <= lmax:
            P[m + 1, m] = (2 * m + 1) * z * P[m, m]
        for l in range(m + 2, lmax + 1):
            P[l, m] = ((2 * l - 1) * z * P[l - 1, m] - (l + m - 1) * P[l - 2, m]) / (l - m)
    N = _sh_norms(lmax)
    out = []
    for l in range(lmax + 1):
        for m in range(-l, l + 1):
            if m < 0:
                out.append(N[l, -m] * P[l, -m] * B[-m])
            elif m == 0:
                out.append(N[l, 0] * P[l, 0])
            else:
                out.append(N[l, m] * P[l, m] * A[m])
    return torch.stack(out, dim=-1)


class SphericalHarmonics(torch.nn.Module):
    def __init__(self, irreps_out, normalize=True, normalization='component'):
        super().__init__()
        self.irreps_out = Irreps(irreps_out)
        self.lmax = self.irreps_out.lmax
        self.normalize = normalize
        assert normalization == 'component'
        assert [ir.l for _, ir in self.irreps_out] == list(range(self.lmax + 1))

    def forward(self, vec):
        return spherical_harmonics(self.lmax, vec, self.normalize)


# ----------------------------------------------------------------------------------------------------------------------
# rotations, Wigner D, Clebsch-Gordan
# ----------------------------------------------------------------------------------------------------------------------


def rotation_from_quaternion(q):
    q = np.asarray(q, dtype=np.float64)
    w, x, y, z = q / np.linalg.norm(q)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
                     [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
                     [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]])


_FIT_ROTATIONS = [rotation_from_quaternion(q) for q in
                  ([0.3, -0.2, 0.9, 0.25], [-0.7, 0.45, 0.1, 0.55], [0.15, 0.8, -0.35, -0.45])]


def wigner_D(l: int, R: np.ndarray) -> np.ndarray:
    """Real Wigner matrix of the harmonics above: Y_l(R r) = D_l(R) Y_l(r), fitted by least squares in float64."""
    rng = np.random.default_rng(1234 + l)
    pts = rng.normal(size=(8 * (2 * l + 1) + 16, 3))
    pts /= np.linalg.norm(pts, axis=1, keepdims=True)
    sl = slice(l * l, (l + 1) ** 2)
    Y0 = spherical_harmonics(l, torch.from_numpy(pts))[:, sl].numpy()
    Y1 = spherical_harmonics(l, torch.from_numpy(pts @ R.T))[:, sl].numpy()
    D, *_ = np.linalg.lstsq(Y0, Y1, rcond=None)       # Y1 = Y0 @ D^T
    return D.T


@functools.lru_cache(maxsize=None)
def _D_fit(l: int, k: int) -> np.ndarray:
    return wigner_D(l, _FIT_ROTATIONS[k])


@functools.lru_cache(maxsize=None)
def clebsch_gordan(l1: int, l2: int, l3: int) -> np.ndarray:
    """Real coupling tensor C[m1, m2, m3] (float64, unit Frobenius norm) invariant under D_l1 (x) D_l2 (x) D_l3."""
    if not abs(l1 - l2) <= l3 <= l1 + l2:
        raise ValueError(f'no coupling {l1} x {l2} -> {l3}')
    d = (2 * l1 + 1) * (2 * l2 + 1) * (2 * l3 + 1)
    rows = []
    for k in range(len(_FIT_ROTATIONS)):
        K = np.kron(np.kron(_D_fit(l1, k), _D_fit(l2, k)), _D_fit(l3, k))
        rows.append(K - np.eye(d))
    _, s, vt = np.linalg.svd(np.concatenate(rows, 0))
    assert s[-1] < 1e-9 and (d == 1 or s[-2] > 1e-3), (l1, l2, l3, s[-2:])
    c = vt[-1]
    c[np.abs(c) < 1e-13] = 0.0
    c /= np.linalg.norm(c)
    first = c[np.argmax(np.abs(c) > 1e-6)]
    if first < 0:
        c = -c
    return c.reshape(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1)


# ----------------------------------------------------------------------------------------------------------------------
# equivariant layers
# ----------------------------------------------------------------------------------------------------------------------

Instruction = namedtuple('Instruction', ['i_in1', 'i_in2', 'i_out', 'connection_mode', 'has_weight', 'path_weight',
                                         'path_shape'])


class TensorProduct(torch.nn.Module):
    """e3nn-style tensor product restricted to weighted 'uvu' paths (the only mode MACE's ``conv_tp`` uses).

    out[z, o3_k + u*d3 + m3] += sqrt(alpha_k) * w[z, k*mul + u] * sum_{a,b} C_k[a,b,m3] x1[z, o1 + u*d1 + a] x2[z, o2 + b]
    with alpha_k = (2 l3 + 1) / fan_in(i_out) ('component' irreps, 'element' paths; fan_in = number of uvu paths
    writing the same output block, each contributing mul_in2 = 1 element).
    """

    def __init__(self, irreps_in1, irreps_in2, irreps_out, instructions, shared_weights=False, internal_weights=False):
        super().__init__()
        self.irreps_in1, self.irreps_in2, self.irreps_out = Irreps(irreps_in1), Irreps(irreps_in2), Irreps(irreps_out)
        self.shared_weights, self.internal_weights = bool(shared_weights), bool(internal_weights)
        if self.shared_weights or self.internal_weights:
            raise NotImplementedError('this stand-in only builds per-sample (external) weights')
        ins = []
        for t in instructions:
            i1, i2, io, mode, train = t[:5]
            pw = t[5] if len(t) > 5 else 1.0
            assert mode == 'uvu' and train
            mul1, mul2, mulo = self.irreps_in1[i1].mul, self.irreps_in2[i2].mul, self.irreps_out[io].mul
            assert mul1 == mulo
            assert self.irreps_out[io].ir in self.irreps_in1[i1].ir * self.irreps_in2[i2].ir
            ins.append(Instruction(i1, i2, io, mode, True, pw, (mul1, mul2)))
        self.instructions = ins
        fan = {}
        for i in ins:
            fan[i.i_out] = fan.get(i.i_out, 0) + self.irreps_in2[i.i_in2].mul
        self._alpha = [math.sqrt(self.irreps_out[i.i_out].ir.dim / fan[i.i_out] * i.path_weight) for i in ins]
        self.weight_numel = sum(self.irreps_in1[i.i_in1].mul * self.irreps_in2[i.i_in2].mul for i in ins)
        self._s1, self._s2, self._so = self.irreps_in1.slices(), self.irreps_in2.slices(), self.irreps_out.slices()
        for k, i in enumerate(ins):
            l1, l2, l3 = self.irreps_in1[i.i_in1].ir.l, self.irreps_in2[i.i_in2].ir.l, self.irreps_out[i.i_out].ir.l
            self.register_buffer(f'cg{k}', torch.from_numpy(clebsch_gordan(l1, l2, l3)).float() * self._alpha[k],
                                 persistent=False)

    def forward(self, x1, x2, weight):
        Z = x1.shape[0]
        outs = [None] * len(self.irreps_out)
        woff = 0
        for k, ins in enumerate(self.instructions):
            mul, ir1 = self.irreps_in1[ins.i_in1]
            ir3 = self.irreps_out[ins.i_out].ir
            a = x1[:, self._s1[ins.i_in1]].reshape(Z, mul, ir1.dim)
            b = x2[:, self._s2[ins.i_in2]]
            w = weight[:, woff:woff + mul]
            woff += mul
            cg = getattr(self, f'cg{k}').to(x1.dtype)
            yc = torch.einsum('zb,abc->zac', b, cg)                  # edge-only part first
            o = torch.einsum('zua,zac->zuc', a, yc) * w.unsqueeze(-1)
            outs[ins.i_out] = o if outs[ins.i_out] is None else outs[ins.i_out] + o
        for i, (mul, ir) in enumerate(self.irreps_out):
            if outs[i] is None:
                outs[i] = x1.new_zeros(Z, mul, ir.dim)
        return torch.cat([o.reshape(Z, -1) for o in outs], dim=1)


def tp_out_irreps_with_instructions(irreps1, irreps2, target_irreps):
    """MACE's rule: one uvu path per (x block, Y block, allowed output irrep), output irreps then sorted."""
    irreps1, irreps2, target_irreps = Irreps(irreps1), Irreps(irreps2), Irreps(target_irreps)
    out_list, instructions = [], []
    for i, (mul, ir_in) in enumerate(irreps1):
        for j, (_, ir_edge) in enumerate(irreps2):
            for ir_out in ir_in * ir_edge:
                if ir_out in target_irreps:
                    k = len(out_list)
                    out_list.append((mul, ir_out))
                    instructions.append((i, j, k, 'uvu', True))
    irreps_out = Irreps(out_list)
    irreps_out, permut, _ = irreps_out.sort()
    instructions = [(i1, i2, permut[io], mode, train) for i1, i2, io, mode, train in instructions]
    instructions = sorted(instructions, key=lambda t: t[2])
    return irreps_out, instructions


class Linear(torch.nn.Module):
    """Equivariant linear map: each output block is sum over input blocks of the same irrep of x_block @ W / sqrt(fan)."""

    def __init__(self, irreps_in, irreps_out):
        super().__init__()
        self.irreps_in, self.irreps_out = Irreps(irreps_in), Irreps(irreps_out)
        self._si, self._so = self.irreps_in.slices(), self.irreps_out.slices()
        self.paths = []
        ws = []
        for io, (mo, iro) in enumerate(self.irreps_out):
            srcs = [ii for ii, (_, iri) in enumerate(self.irreps_in) if iri == iro]
            fan = sum(self.irreps_in[ii].mul for ii in srcs)
            for ii in srcs:
                self.paths.append((ii, io, 1.0 / math.sqrt(fan)))
                ws.append(torch.randn(self.irreps_in[ii].mul, mo))
        self.weight = torch.nn.ParameterList([torch.nn.Parameter(w) for w in ws])

    def forward(self, x):
        Z = x.shape[0]
        outs = [None] * len(self.irreps_out)
        for (ii, io, s), w in zip(self.paths, self.weight):
            mi, iri = self.irreps_in[ii]
            xb = x[:, self._si[ii]].reshape(Z, mi, iri.dim)
            o = torch.einsum('zui,uw->zwi', xb, w * s)
            outs[io] = o if outs[io] is None else outs[io] + o
        for i, (mul, ir) in enumerate(self.irreps_out):
            if outs[i] is None:
                outs[i] = x.new_zeros(Z, mul, ir.dim)
        return torch.cat([o.reshape(Z, -1) for o in outs], dim=1)


class FullyConnectedTensorProduct(torch.nn.Module):
    """'uvw' tensor product with a scalar second operand (MACE's ``skip_tp`` with one-hot element attributes):
    out[z, w, i] = sum_{u,v} W[u, v, w] x1[z, u, i] x2[z, v] / sqrt(fan_in) for every x1 block of the output's irrep."""

    def __init__(self, irreps_in1, irreps_in2, irreps_out):
        super().__init__()
        self.irreps_in1, self.irreps_in2, self.irreps_out = Irreps(irreps_in1), Irreps(irreps_in2), Irreps(irreps_out)
        assert all(ir.l == 0 and ir.p == 1 for _, ir in self.irreps_in2), 'second operand must be scalars'
        self.n2 = self.irreps_in2.dim
        self._s1, self._so = self.irreps_in1.slices(), self.irreps_out.slices()
        self.paths = []
        ws = []
        for io, (mo, iro) in enumerate(self.irreps_out):
            srcs = [ii for ii, (_, iri) in enumerate(self.irreps_in1) if iri == iro]
            fan = sum(self.irreps_in1[ii].mul for ii in srcs) * self.n2
            for ii in srcs:
                self.paths.append((ii, io, 1.0 / math.sqrt(fan)))
                ws.append(torch.randn(self.irreps_in1[ii].mul, self.n2, mo))
        self.weight = torch.nn.ParameterList([torch.nn.Parameter(w) for w in ws])

    def forward(self, x1, x2):
        Z = x1.shape[0]
        outs = [None] * len(self.irreps_out)
        for (ii, io, s), w in zip(self.paths, self.weight):
            mi, iri = self.irreps_in1[ii]
            mo = self.irreps_out[io].mul
            xb = x1[:, self._s1[ii]].reshape(Z, mi, iri.dim).transpose(1, 2)          # [Z, i, u]
            t = (xb @ (w * s).reshape(mi, self.n2 * mo)).reshape(Z, iri.dim, self.n2, mo)
            o = torch.einsum('zivw,zv->zwi', t, x2)
            outs[io] = o if outs[io] is None else outs[io] + o
        for i, (mul, ir) in enumerate(self.irreps_out):
            if outs[i] is None:
                outs[i] = x1.new_zeros(Z, mul, ir.dim)
        return torch.cat([o.reshape(Z, -1) for o in outs], dim=1)
