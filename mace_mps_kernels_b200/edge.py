"""MACE's per-edge geometry on B200: the edge vectors and lengths, the spherical harmonics of the vectors and the
radial embedding of the lengths, each one CUDA kernel forward and one backward (C ABI ``mmk_edge_vectors_*``,
``mmk_sh_*``, ``mmk_radial_*``).

In the reference these stay on e3nn / PyTorch, where they are a few dozen small elementwise kernels per call in each
direction; at the graph sizes of an MD step (thousands of edges) those launches, not the arithmetic, set their cost.
``patch_model(model, edge_features=True)`` swaps ``model.spherical_harmonics`` and ``model.radial_embedding`` for
the modules below and routes the model's ``get_edge_vectors_and_lengths`` calls to ``edge_vectors_and_lengths``
(``patch_edge_vectors``).  Same definitions and outputs as the modules they replace (see ``csrc/edge_geom.cuh``); first-order
backward only, double backward raises like the other patched ops.
"""
from __future__ import annotations

import ctypes
import inspect

import torch

from . import _lib
from .conv import DOUBLE_BACKWARD_MSG


def sh_supported(mod):
    """(ok, reason) for a spherical-harmonics module: normalised edge vectors, 'component' normalisation, every l from 0
    to l_max (at most 3) once, in order."""
    if mod is None:
        return False, 'no spherical_harmonics module'
    if not getattr(mod, 'normalize', False):
        return False, 'only normalize=True harmonics are supported'
    norm = getattr(mod, 'normalization', 'component')
    if norm != 'component':
        return False, f'only component normalisation is supported (got {norm})'
    irreps = getattr(mod, 'irreps_out', None)
    ls = [ir.l for _, ir in irreps] if irreps is not None else None
    muls = [mul for mul, _ in irreps] if irreps is not None else None
    if ls is None or ls != list(range(len(ls))) or any(m != 1 for m in muls):
        return False, 'spherical harmonics must be 1x0 + 1x1 + ... + 1xl_max'
    if len(ls) - 1 > 3:
        return False, 'l_max > 3 is not supported'
    return True, ''


def radial_supported(mod):
    """(ok, reason) for a radial-embedding block made of a Bessel basis and a polynomial cutoff."""
    b = getattr(mod, 'bessel_fn', None)
    c = getattr(mod, 'cutoff_fn', None)
    if b is None or c is None or not hasattr(b, 'bessel_weights') or not hasattr(c, 'p'):
        return False, 'radial embedding is not Bessel basis x polynomial cutoff'
    if b.bessel_weights.numel() > 16:
        return False, 'more than 16 Bessel functions'
    return True, ''


class _SHFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vec, lmax):
        v = vec.contiguous()
        if v.dtype != torch.float32 or not v.is_cuda:
            raise TypeError('edge vectors must be a float32 CUDA tensor')
        Y = torch.empty(v.shape[0], (lmax + 1) ** 2, device=v.device, dtype=torch.float32)
        _lib.call('mmk_sh_fwd', _lib.ptr(v), v.shape[0], lmax, _lib.ptr(Y), _lib.stream_of(v))
        ctx.save_for_backward(v)
        ctx.lmax = lmax
        return Y

    @staticmethod
    def backward(ctx, gY):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        (v,) = ctx.saved_tensors
        gY = gY.contiguous()
        gv = torch.empty_like(v)
        _lib.call('mmk_sh_bwd', _lib.ptr(v), _lib.ptr(gY), v.shape[0], ctx.lmax, _lib.ptr(gv), _lib.stream_of(v))
        return gv, None


class CudaSphericalHarmonics(torch.nn.Module):
    """Drop-in for MACE's ``o3.SphericalHarmonics(sh_irreps, normalize=True, normalization='component')``."""

    def __init__(self, sh):
        super().__init__()
        ok, why = sh_supported(sh)
        if not ok:
            raise ValueError(why)
        self.irreps_out = sh.irreps_out
        self.lmax = len(list(sh.irreps_out)) - 1
        self.normalize = True
        self.normalization = 'component'

    def forward(self, vec):
        return _SHFn.apply(vec, self.lmax)


class _RadialFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lengths, op):
        r = lengths.contiguous()
        if r.dtype != torch.float32 or not r.is_cuda:
            raise TypeError('edge lengths must be a float32 CUDA tensor')
        out = torch.empty(r.shape[0], op.n, device=r.device, dtype=torch.float32)
        _lib.call('mmk_radial_fwd', ctypes.byref(op.desc), _lib.ptr(r), r.shape[0], _lib.ptr(out), _lib.stream_of(r))
        ctx.save_for_backward(r)
        ctx.op = op
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        (r,) = ctx.saved_tensors
        g = g.contiguous()
        gr = torch.empty_like(r)
        _lib.call('mmk_radial_bwd', ctypes.byref(ctx.op.desc), _lib.ptr(r), _lib.ptr(g), r.shape[0], _lib.ptr(gr),
                  _lib.stream_of(r))
        return gr, None


class CudaRadialEmbedding(torch.nn.Module):
    """Drop-in for MACE's ``RadialEmbeddingBlock`` (Bessel basis x polynomial cutoff): forward(lengths[E, 1]) ->
    [E, num_bessel]; the constants are read from the block's buffers."""

    def __init__(self, block):
        super().__init__()
        ok, why = radial_supported(block)
        if not ok:
            raise ValueError(why)
        w = block.bessel_fn.bessel_weights.detach().float().cpu().reshape(-1)
        self.n = int(w.numel())
        self.out_dim = self.n
        self.consts = (w.tolist(), float(block.bessel_fn.prefactor), float(block.cutoff_fn.r_max),
                       float(block.cutoff_fn.p))
        self._cdesc = None

    @property
    def desc(self):
        """The C descriptor (built on first use; holds a pointer to its own frequency array)."""
        if self._cdesc is None:
            w, pref, r_max, p = self.consts
            arr = (ctypes.c_float * self.n)(*w)
            self._cdesc = (_lib.RadialDesc(self.n, arr, pref, r_max, p), arr)
        return self._cdesc[0]

    def __deepcopy__(self, memo):
        new = self.__class__.__new__(self.__class__)
        torch.nn.Module.__init__(new)
        new.n, new.out_dim, new.consts, new._cdesc = self.n, self.out_dim, self.consts, None
        return new

    def forward(self, edge_lengths):
        return _RadialFn.apply(edge_lengths, self)


class _EdgeVectorsFn(torch.autograd.Function):
    """(vectors [E, 3], lengths [E, 1]) of MACE's ``get_edge_vectors_and_lengths`` in one launch; the backward is
    one launch over the receiver and sender CSRs (built once per edge_index and shared with the convolution),
    deterministic, where PyTorch's indexing backward sorts the edge index every call."""

    @staticmethod
    def forward(ctx, positions, shifts, edge_index):
        from .conv import graph_csr
        pos, sh = positions.contiguous(), shifts.contiguous()
        for name, t in (('positions', pos), ('shifts', sh)):
            if t.dtype != torch.float32 or not t.is_cuda:
                raise TypeError(f'{name} must be a float32 CUDA tensor')
        E = edge_index.shape[1]
        vec = torch.empty(E, 3, device=pos.device, dtype=torch.float32)
        ln = torch.empty(E, 1, device=pos.device, dtype=torch.float32)
        _lib.call('mmk_edge_vectors_fwd', _lib.ptr(pos), _lib.ptr(edge_index), _lib.ptr(sh), E, _lib.ptr(vec),
                  _lib.ptr(ln), _lib.stream_of(pos))
        ctx.csr = graph_csr(edge_index, pos.shape[0]) if ctx.needs_input_grad[0] else None
        ctx.n_nodes = pos.shape[0]
        ctx.save_for_backward(vec, ln)
        return vec, ln

    @staticmethod
    def backward(ctx, gvec, glen):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        vec, ln = ctx.saved_tensors
        E, N = vec.shape[0], ctx.n_nodes
        if gvec is None and glen is None:
            return None, None, None
        if E == 0:                                     # no edges: nothing reaches the positions or the shifts
            gpos = torch.zeros(N, 3, device=vec.device) if ctx.needs_input_grad[0] else None
            gsh = torch.zeros(0, 3, device=vec.device) if ctx.needs_input_grad[1] else None
            return gpos, gsh, None
        gvec = gvec.contiguous() if gvec is not None else None
        glen = glen.contiguous() if glen is not None else None
        gpos = gsh = None
        if ctx.needs_input_grad[0]:
            gpos = torch.empty(N, 3, device=vec.device, dtype=torch.float32)
        if ctx.needs_input_grad[1]:
            gsh = torch.empty(E, 3, device=vec.device, dtype=torch.float32)
        rrp, reid, srp, seid = ctx.csr if ctx.csr is not None else (None,) * 4
        _lib.call('mmk_edge_vectors_bwd', _lib.ptr(gvec) if gvec is not None else None,
                  _lib.ptr(glen) if glen is not None else None, _lib.ptr(vec), _lib.ptr(ln),
                  _lib.ptr(rrp) if rrp is not None else None, _lib.ptr(reid) if reid is not None else None,
                  _lib.ptr(srp) if srp is not None else None, _lib.ptr(seid) if seid is not None else None,
                  N, E, _lib.ptr(gpos) if gpos is not None else None, _lib.ptr(gsh) if gsh is not None else None,
                  _lib.stream_of(vec))
        return gpos, gsh, None


def edge_vectors_and_lengths(positions, edge_index, shifts):
    """CUDA drop-in for MACE's ``get_edge_vectors_and_lengths(positions, edge_index, shifts)`` (normalize=False):
    float32 CUDA positions [N, 3] and shifts [E, 3], a contiguous int64 [2, E] edge_index on the same device."""
    if edge_index.dtype != torch.int64 or edge_index.dim() != 2 or edge_index.shape[0] != 2:
        raise ValueError(f'edge_index must be int64 [2, E] (got {edge_index.dtype} {tuple(edge_index.shape)})')
    if not edge_index.is_contiguous() or edge_index.device != positions.device:
        raise ValueError('edge_index must be contiguous and on the positions\' device')
    if positions.dim() != 2 or positions.shape[1] != 3 or shifts.shape != (edge_index.shape[1], 3):
        raise ValueError(f'positions must be [N, 3] and shifts [E, 3] (got {tuple(positions.shape)}, '
                         f'{tuple(shifts.shape)})')
    return _EdgeVectorsFn.apply(positions, shifts, edge_index)


_ACTIVE = [0]            # patched models whose forward is running (the wrapper is global to the model's module)


def _fused_get_edge_vectors_and_lengths(original):
    def get_edge_vectors_and_lengths(positions, edge_index, shifts, normalize=False, eps=1e-9):
        if (_ACTIVE[0] > 0 and not normalize and positions.is_cuda and positions.dtype == torch.float32
                and shifts.dtype == torch.float32 and edge_index.dtype == torch.int64 and edge_index.dim() == 2
                and edge_index.is_contiguous() and shifts.shape == (edge_index.shape[1], 3)):
            return edge_vectors_and_lengths(positions, edge_index, shifts)
        return original(positions=positions, edge_index=edge_index, shifts=shifts, normalize=normalize, eps=eps)

    get_edge_vectors_and_lengths._mmk_original = original
    return get_edge_vectors_and_lengths


def _enter(module, args, kwargs=None):
    _ACTIVE[0] += 1


def _leave(module, args, output):
    _ACTIVE[0] = max(0, _ACTIVE[0] - 1)


def patch_edge_vectors(model):
    """(ok, reason): route the model's ``get_edge_vectors_and_lengths`` calls to the fused CUDA op.

    MACE's forward calls the function through its module's namespace (mace.modules.models imports it from
    mace.modules.utils), so that name is replaced by a wrapper; the wrapper takes the CUDA path only while the
    forward of a model patched here is running (forward pre/post hooks on the model) and for the supported inputs,
    and calls the original function otherwise, so other models of the same class are unaffected."""
    import sys
    mod = sys.modules.get(type(model).__module__)
    fn = getattr(mod, 'get_edge_vectors_and_lengths', None) if mod is not None else None
    if not callable(fn):
        return False, 'the model forward does not call get_edge_vectors_and_lengths from its module'
    try:
        calls = 'get_edge_vectors_and_lengths' in inspect.getsource(type(model).forward)
    except (OSError, TypeError):
        calls = False
    if not calls:
        return False, 'the model forward does not call get_edge_vectors_and_lengths itself'
    if not hasattr(fn, '_mmk_original'):
        setattr(mod, 'get_edge_vectors_and_lengths', _fused_get_edge_vectors_and_lengths(fn))
    if not getattr(model, '_mmk_edge_vectors', False):
        model.register_forward_pre_hook(_enter)
        model.register_forward_hook(_leave, always_call=True)      # also when the forward raises
        model._mmk_edge_vectors = True
    return True, ''
