"""MACE's per-edge geometry on B200: spherical harmonics of the edge vectors and the radial embedding of the edge
lengths, each one CUDA kernel forward and one backward (C ABI ``mmk_sh_*`` / ``mmk_radial_*``).

In the reference these stay on e3nn / PyTorch, where they are a few dozen small elementwise kernels per call in each
direction; at the graph sizes of an MD step (thousands of edges) those launches, not the arithmetic, set their cost.
``patch_model(model, edge_features=True)`` swaps ``model.spherical_harmonics`` and ``model.radial_embedding`` for
the modules below.  Same definitions and outputs as the modules they replace (see ``csrc/edge_geom.cuh``); first-order
backward only, double backward raises like the other patched ops.
"""
from __future__ import annotations

import ctypes

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
