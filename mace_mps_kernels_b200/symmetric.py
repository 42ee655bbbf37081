"""MACE SymmetricContraction on B200 as a precomputed element-dependent polynomial.

At inference the product-basis weights and U matrices are constants, so for element e, channel c and output
component M the contraction is a polynomial in the channel's features x = x[b, c, :] (n_ell = (l_max+1)^2):
    out[b, c, M] = sum_{nu} sum_{i1 <= .. <= i_nu} T_nu[e, c, M, i] x_i1 .. x_i_nu
with T_nu = U_nu . W_nu symmetrised over index order (the reference's construction, symmetric.py:20-39; here the
symmetrisation is one matrix product with the 0/1 map "index tuple -> sorted tuple").  Terms whose coefficient
vanishes for every (e, M, c) are dropped (tolerance 1e-12, symmetric.py:66).  ``SCSpec.T`` is packed as the reference
does, T[e][row][c] (row = term's first row + M); terms are ordered by degree (descending) then index tuple, as in the
reference (symmetric.py:64-69).  The device copy the kernels read is channel-major, T[e][c][row] with the rows padded
to a multiple of 4 (``device_table``).

The CUDA kernels (monomial list baked into NVRTC-compiled code) evaluate the polynomial (forward) and its derivative
(first-order backward) node-major: a warp is 32 nodes of one element and one channel, the channel's coefficient column
is staged in shared memory by TMA and every coefficient load is a broadcast; double backward raises.
"""
from __future__ import annotations

import itertools

import numpy as np
import torch

from . import _lib
from .conv import DOUBLE_BACKWARD_MSG, _LayerHandle, _tensor_key


def _contraction_tensors(ct):
    """float64 numpy copies of one mace Contraction's constants: (correlation, {degree: U}, {degree: weights}, has an
    output-component axis, M = 2L+1, n_ell).  mace keeps the top-degree weights as ``weights_max`` and the lower
    degrees in ``weights`` ordered from degree correlation-1 down to 1."""
    corr = int(ct.correlation)
    as64 = lambda t: t.detach().cpu().double().numpy()
    U = {nu: as64(getattr(ct, f'U_matrix_{nu}')) for nu in range(1, corr + 1)}
    lower = [as64(w) for w in ct.weights]
    W = dict(zip(range(corr, 0, -1), [as64(ct.weights_max)] + lower))
    u1 = U[1]                                                # [M, n_ell, p] for L > 0, [n_ell, p] for L = 0
    has_m = u1.ndim == 3
    return corr, U, W, has_m, (u1.shape[0] if has_m else 1), u1.shape[-2]


def _sym_map(n_ell, nu):
    """(sorted index tuples in lexicographic order, 0/1 matrix [n_ell^nu, n_sym] mapping each tuple to its sort)."""
    tuples = list(itertools.combinations_with_replacement(range(n_ell), nu))
    pos = {t: i for i, t in enumerate(tuples)}
    P = np.zeros((n_ell ** nu, len(tuples)))
    for flat, idx in enumerate(itertools.product(range(n_ell), repeat=nu)):
        P[flat, pos[tuple(sorted(idx))]] = 1.0
    return tuples, P


def poly_coeffs(ct):
    """{nu: (tuples, coeffs[e, M, c, n_sym])} in float64, M = 2L+1 of this contraction's output."""
    corr, U, W, has_m, M, n_ell = _contraction_tensors(ct)
    res = {}
    for nu in range(1, corr + 1):
        u = U[nu] if has_m else U[nu][None]
        K = u.shape[-1]
        tuples, P = _sym_map(n_ell, nu)
        u_sym = np.einsum('mfk,fs->msk', u.reshape(M, -1, K), P)          # [M, n_sym, K]
        T = np.einsum('msk,ekc->emcs', u_sym, W[nu])                       # [e, M, c, n_sym]
        res[nu] = (tuples, T)
    return res, M, n_ell


def sc_supported(sc):
    try:
        cts = list(sc.contractions)
        for ct in cts:
            _ = ct.correlation, ct.weights_max, ct.U_matrix_1
    except AttributeError as e:
        return False, f'not a MACE SymmetricContraction ({e})'
    return True, ''


def term_table(ct, tol=1e-12):
    """The monomials of one contraction that survive ``tol``: ([(sorted index tuple, coefficients [n_elem, M, C])],
    M, n_ell), highest degree first and index tuples in lexicographic order within a degree (the order the
    reference's term list and generated kernels use, so rows agree one for one)."""
    coeffs, M, n_ell = poly_coeffs(ct)
    table = []
    for nu in sorted(coeffs, reverse=True):
        tuples, T = coeffs[nu]
        peak = np.abs(T).reshape(-1, T.shape[-1]).max(axis=0)              # largest |coefficient| per monomial
        table += [(tuples[s], T[..., s]) for s in np.flatnonzero(peak > tol)]
    return table, M, n_ell


class SCSpec:
    """Polynomial form of a mace SymmetricContraction: per output block (one per contraction) its M, its terms
    (index tuple, first row) and its output offset; ``T`` [n_elem, rows, C] float32 holds M consecutive rows per term
    (one per output component)."""

    def __init__(self, sc, tol=1e-12):
        ok, why = sc_supported(sc)
        if not ok:
            raise ValueError(why)
        tables = [term_table(ct, tol) for ct in sc.contractions]
        if len({n for _, _, n in tables}) != 1:
            raise ValueError('contractions disagree on the number of feature components')
        self.n_ell = tables[0][2]
        self.C = int(sc.contractions[0].weights_max.shape[-1])
        self.blocks, packed, row, out_off = [], [], 0, 0
        for table, M, _ in tables:
            terms = []
            for idx, v in table:
                terms.append((idx, row))
                packed.append(v)                                           # [n_elem, M, C]: rows row .. row+M-1
                row += M
            self.blocks.append(dict(M=M, terms=terms, out_off=out_off))
            out_off += self.C * M
        self.out_dim, self.nrows = out_off, row
        self.T = torch.from_numpy(np.concatenate(packed, axis=1)).float()  # [n_elem, rows, C]
        self.n_terms = sum(len(b['terms']) for b in self.blocks)
        self.max_degree = max(len(idx) for b in self.blocks for idx, _ in b['terms'])

    @classmethod
    def from_table(cls, C, n_ell, block_M, block_terms, T):
        """Spec from an explicit table: block_terms[q] = [(index tuple, first row)], T [n_elem, rows, C]."""
        self = cls.__new__(cls)
        self.C, self.n_ell = int(C), int(n_ell)
        self.blocks, out_off = [], 0
        for M, terms in zip(block_M, block_terms):
            self.blocks.append(dict(M=int(M), terms=[(tuple(int(i) for i in idx), int(r)) for idx, r in terms],
                                    out_off=out_off))
            out_off += self.C * int(M)
        self.out_dim = out_off
        self.T = torch.as_tensor(np.asarray(T), dtype=torch.float32)
        self.nrows = self.T.shape[1]
        self.n_terms = sum(len(b['terms']) for b in self.blocks)
        self.max_degree = max(len(idx) for b in self.blocks for idx, _ in b['terms'])
        return self

    def descriptor(self):
        keep = {}
        terms = [t for b in self.blocks for t in b['terms']]
        D = self.max_degree
        keep['M'] = _lib.int_array(b['M'] for b in self.blocks)
        keep['nt'] = _lib.int_array(len(b['terms']) for b in self.blocks)
        keep['deg'] = _lib.int_array(len(idx) for idx, _ in terms)
        keep['idx'] = _lib.int_array(v for idx, _ in terms for v in (list(idx) + [-1] * (D - len(idx))))
        keep['row'] = _lib.int_array(r for _, r in terms)
        d = _lib.SCDesc(self.C, self.n_ell, self.nrows, len(self.blocks), keep['M'], keep['nt'], D, keep['deg'],
                        keep['idx'], keep['row'])
        d._keep = keep
        return d

    def flops(self):
        """(forward, backward) fp32 operations per (node, channel), counted from the term list."""
        fwd = bwd = 0
        for b in self.blocks:
            M = b['M']
            for idx, _ in b['terms']:
                fwd += (len(idx) - 1) + 2 * M
                bwd += 2 * M + len(set(idx)) * (len(idx) + 1)
        return fwd, bwd


def executed_flops(spec):
    """(forward, backward) floating-point operations the generated term code executes per (node, channel): it is
    straight-line code, so every ``fmaf`` (2 flops) and every binary ``*`` or ``+`` of two floats (1 flop) in the
    bodies runs exactly once.  Fewer than ``flops()``, which counts the terms as the reference evaluates them."""
    import re
    src = source(spec)
    res = []
    for name in ('sc_fwd_body', 'sc_bwd_body'):
        i = src.index('void ' + name)
        body = src[i:src.index('\n}\n', i)]
        body = re.sub(r'\[[^\]]*\]', '[]', body)                 # index expressions are not float arithmetic
        res.append(2 * body.count('fmaf(') + len(re.findall(r'[\w\]\)] [*+] [\w(]', body)))
    return tuple(res)


_ELEM_CACHE = []


def source(spec):
    """Generated CUDA layer header for ``spec`` (sizes, launch plan and the Horner-scheme term code), the counterpart
    of the reference's ``source(spec)`` (symmetric.py:82)."""
    return _lib.generated_source('mmk_sc_source', spec.descriptor())


def element_groups(node_attrs: torch.Tensor):
    """(elem int32[N], erow int32[n_elem+1], perm int32[N]): the argmax element of every node (reference
    symmetric.py:169) and the nodes grouped by element, on the device.  Cached like the conv's CSRs: keyed on the
    tensor object, its storage address, shape, strides and version counter (``conv.invalidate_graph_caches``)."""
    import weakref
    key = _tensor_key(node_attrs)
    for ref, k, g in reversed(_ELEM_CACHE):
        if ref() is node_attrs and k == key:
            return g
    a = node_attrs.contiguous()
    if a.dtype != torch.float32 or not a.is_cuda:
        raise TypeError('node_attrs must be a float32 CUDA tensor')
    N, n_elem = a.shape
    st = _lib.stream_of(a)
    elem = torch.empty(N, dtype=torch.int32, device=a.device)
    erow = torch.empty(n_elem + 1, dtype=torch.int32, device=a.device)
    perm = torch.empty(N, dtype=torch.int32, device=a.device)
    _lib.call('mmk_elem_index', _lib.ptr(a), N, n_elem, _lib.ptr(elem), st)
    nb = _lib.lib().mmk_csr_workspace_bytes(n_elem, N)
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=a.device)
    _lib.call('mmk_elem_groups', _lib.ptr(elem), N, n_elem, _lib.ptr(erow), _lib.ptr(perm), _lib.ptr(ws), nb, st)
    g = (elem, erow, perm)
    _ELEM_CACHE.append((weakref.ref(node_attrs), key, g))
    del _ELEM_CACHE[:-4]
    return g


class _SCFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, erow, perm, op):
        if x.dtype != torch.float32 or not x.is_cuda:
            raise TypeError(f'x must be a float32 CUDA tensor (got {x.dtype} on {x.device})')
        x = _lib.aligned(x.contiguous())
        N = x.shape[0]
        if x.shape != (N, op.spec.C, op.spec.n_ell):
            raise ValueError(f'x must be [N, {op.spec.C}, {op.spec.n_ell}] (got {tuple(x.shape)})')
        n_elem = erow.shape[0] - 1
        if n_elem != op.T.shape[0]:
            raise ValueError(f'node_attrs has {n_elem} elements, the contraction {op.T.shape[0]}')
        out = torch.empty(N, op.spec.out_dim, device=x.device, dtype=torch.float32)
        _lib.call('mmk_sc_fwd', op.handle, _lib.ptr(x), _lib.ptr(perm), _lib.ptr(erow), n_elem, _lib.ptr(op.T),
                  _lib.ptr(out), N, _lib.stream_of(x))
        ctx.save_for_backward(x, erow, perm)
        ctx.op = op
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():          # only true under create_graph=True
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        x, erow, perm = ctx.saved_tensors
        op = ctx.op
        g = g.contiguous()
        gx = torch.empty_like(x)
        _lib.call('mmk_sc_bwd', op.handle, _lib.ptr(x), _lib.ptr(perm), _lib.ptr(erow), erow.shape[0] - 1,
                  _lib.ptr(op.T), _lib.ptr(g), _lib.ptr(gx), x.shape[0], _lib.stream_of(x))
        return gx, None, None, None


def device_table(T):
    """[n_elem, rows, C] (SCSpec.T) -> the kernels' layout [n_elem, C, RP], RP = rows rounded up to 4 (zero rows)."""
    T = torch.as_tensor(T, dtype=torch.float32).transpose(1, 2)
    rp = (T.shape[2] + 3) // 4 * 4
    if rp != T.shape[2]:
        T = torch.nn.functional.pad(T, (0, rp - T.shape[2]))
    return T.contiguous()


class CudaSymmetricContraction(torch.nn.Module):
    """Drop-in for mace ``SymmetricContraction`` at inference: forward(x[N, C, n_ell], node_attrs[N, n_elem])."""

    def __init__(self, sc, device='cuda', spec=None):
        super().__init__()
        self.spec = SCSpec(sc) if spec is None else spec
        self.register_buffer('T', device_table(self.spec.T).to(device))
        self._h = _LayerHandle('mmk_sc_layer_create', 'mmk_sc_layer_destroy', self.spec.descriptor())
        self.irreps_in = getattr(sc, 'irreps_in', None)
        self.irreps_out = getattr(sc, 'irreps_out', None)

    @classmethod
    def from_spec(cls, spec, device='cuda'):
        """Op for an explicit ``SCSpec`` (e.g. ``SCSpec.from_table``)."""
        return cls(None, device, spec)

    @property
    def handle(self):
        return self._h.value

    def status(self, reset=False):
        """Error status of this layer's kernels on the current device (0 = ok); synchronises with the device."""
        import ctypes
        v = ctypes.c_int(0)
        _lib.call('mmk_sc_layer_status', self.handle, ctypes.byref(v), int(reset))
        return v.value

    def __deepcopy__(self, memo):
        import copy
        new = self.__class__.__new__(self.__class__)
        torch.nn.Module.__init__(new)
        new.spec = self.spec
        new.register_buffer('T', copy.deepcopy(self.T, memo))
        new._h = self._h
        new.irreps_in, new.irreps_out = self.irreps_in, self.irreps_out
        return new

    def forward(self, x, y):
        _, erow, perm = element_groups(y)
        return _SCFn.apply(x, erow, perm, self)


MetalSymmetricContraction = CudaSymmetricContraction
