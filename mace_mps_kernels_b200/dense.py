"""MACE's equivariant linear layers on B200: ``o3.Linear`` and the element-indexed skip connection
(``FullyConnectedTensorProduct`` of the node features with the one-hot node attributes), one CUDA launch each way
(C ABI ``mmk_block_linear``) instead of a slice / scale / einsum / add chain per path.

A layer is a list of paths (input block ii -> output block io of the same irrep, weight W [mul_in, mul_out] scaled
by 1/sqrt(fan_in)); the forward applies them all at once, the backward (gradient w.r.t. the input only) applies the
transposed paths.  With one-hot node attributes the skip connection is a linear map whose weight is selected by the
node's element, W_e = W[:, e, :]; the kernel works on nodes grouped by element (the symmetric contraction's groups).

The hidden layers of an interaction's radial MLP (``FullyConnectedNet``: scalar layers without biases,
h <- c * silu(h @ W / sqrt(fan_in))) run in one launch each way (C ABI ``mmk_mlp_fwd`` / ``mmk_mlp_bwd``): a CTA keeps
every layer's weights and the activations of a block of edges in shared memory; the forward stores every
pre-activation, the backward applies c * silu'(z) to the gradient layer by layer.  Wider or deeper MLPs use the
block-linear kernel, one launch per layer with the activation fused.  The last layer (no activation, NINS x C wide)
is a float32 GEMM on the tensor cores (``gemm.TensorCoreLinear``: tcgen05 with the 3xTF32 split), both ways.

Inference only: the weights must be frozen (``requires_grad`` False, as MACE's calculators set them), the backward is
first order, double backward raises.  ``patch_model(model, linears=True)`` swaps every supported layer.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .conv import DOUBLE_BACKWARD_MSG


def _blocks(irreps):
    """[(offset, mul, dim)] of an Irreps (mul_ir layout)."""
    out, off = [], 0
    for mul, ir in irreps:
        out.append((off, mul, ir.dim))
        off += mul * ir.dim
    return out, off


def linear_supported(mod):
    """(ok, reason) for an equivariant linear with explicit per-path weights (the layout of this repository's MACE)."""
    if not hasattr(mod, 'paths') or not hasattr(mod, 'weight') or not (hasattr(mod, 'irreps_in') or
                                                                       hasattr(mod, 'irreps_in1')):
        return False, 'not a per-path equivariant linear'
    if any(p.requires_grad for p in mod.parameters()):
        return False, 'weights require grad (training): frozen weights only'
    return True, ''


def skip_supported(mod):
    ok, why = linear_supported(mod)
    if not ok:
        return ok, why
    if not hasattr(mod, 'irreps_in2') or any(ir.l != 0 for _, ir in mod.irreps_in2):
        return False, 'second operand must be scalar node attributes'
    return True, ''


class _Tables:
    """Device path tables of one direction: int32 blocks [n_out_blocks, 5], paths [n_paths, 3], packed weights."""

    def __init__(self, out_blocks, path_list, device):
        blocks, paths, w = [], [], []
        w_off = 0
        for b, (off, mul, d) in enumerate(out_blocks):
            mine = [p for p in path_list if p[1] == b]
            blocks.append([off, mul, d, len(paths), len(mine)])
            for src_off, _, W in mine:                 # W: [n_elem, mul_in, mul_out] float32
                paths.append([src_off, W.shape[1], w_off])
                w.append(W.reshape(-1))
                w_off += W.size
        self.n_blocks = len(blocks)
        self.max_d = max(d for _, _, d in out_blocks)
        self.max_mul = max(mul for _, mul, _ in out_blocks)
        self.blocks = torch.tensor(np.asarray(blocks, np.int32).reshape(-1, 5), device=device)
        self.paths = torch.tensor(np.asarray(paths, np.int32).reshape(-1, 3), device=device)
        wv = np.concatenate(w) if w else np.zeros(1, np.float32)
        self.w = torch.tensor(wv.astype(np.float32), device=device)
        if w_off >= 2 ** 31:
            raise ValueError('layer too large')


class _BlockLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, op, groups):
        x = x.contiguous()
        if x.dtype != torch.float32 or not x.is_cuda:
            raise TypeError('input must be a float32 CUDA tensor')
        N = x.shape[0]
        out = torch.empty(N, op.out_dim, device=x.device, dtype=torch.float32)
        op._launch(op.fwd, x, op.in_dim, out, op.out_dim, groups)
        ctx.op, ctx.groups = op, groups
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        op = ctx.op
        g = g.contiguous()
        gx = torch.empty(g.shape[0], op.in_dim, device=g.device, dtype=torch.float32)
        op._launch(op.bwd, g, op.out_dim, gx, op.in_dim, ctx.groups)
        return gx, None, None


class _BlockLinearBase(torch.nn.Module):
    def _build(self, in_irreps, out_irreps, path_list, device):
        """path_list: (ii, io, W [n_elem, mul_in, mul_out] float32 numpy, already scaled)."""
        ib, self.in_dim = _blocks(in_irreps)
        ob, self.out_dim = _blocks(out_irreps)
        self.fwd = _Tables(ob, [(ib[ii][0], io, W) for ii, io, W in path_list], device)
        self.bwd = _Tables(ib, [(ob[io][0], ii, np.ascontiguousarray(W.transpose(0, 2, 1)))
                                for ii, io, W in path_list], device)

    def _launch(self, t, x, ldx, out, ldo, groups):
        perm, erow, n_elem = groups if groups is not None else (None, None, 1)
        _lib.call('mmk_block_linear', _lib.ptr(x), ldx, _lib.ptr(out), ldo, _lib.ptr(t.blocks), t.n_blocks,
                  _lib.ptr(t.paths), _lib.ptr(t.w), t.max_d, t.max_mul, _lib.ptr(perm), _lib.ptr(erow), n_elem,
                  x.shape[0],
                  _lib.stream_of(x))


class CudaLinear(_BlockLinearBase):
    """Drop-in for the equivariant ``o3.Linear`` (frozen weights): forward(x[N, in_dim]) -> [N, out_dim]."""

    def __init__(self, lin):
        super().__init__()
        ok, why = linear_supported(lin)
        if not ok:
            raise ValueError(why)
        self.irreps_in, self.irreps_out = lin.irreps_in, lin.irreps_out
        dev = next(lin.parameters()).device
        path_list = [(ii, io, (w.detach() * s).float().cpu().numpy()[None]) for (ii, io, s), w in
                     zip(lin.paths, lin.weight)]
        self._build(lin.irreps_in, lin.irreps_out, path_list, dev)

    def forward(self, x):
        return _BlockLinearFn.apply(x, self, None)


class CudaSkipTP(_BlockLinearBase):
    """Drop-in for MACE's skip connection ``FullyConnectedTensorProduct(node_feats, node_attrs)`` with one-hot node
    attributes (frozen weights): forward(x1[N, in_dim], node_attrs[N, n_elem]) -> [N, out_dim]."""

    def __init__(self, tp):
        super().__init__()
        ok, why = skip_supported(tp)
        if not ok:
            raise ValueError(why)
        self.irreps_in1, self.irreps_in2, self.irreps_out = tp.irreps_in1, tp.irreps_in2, tp.irreps_out
        self.n_elem = tp.irreps_in2.dim
        dev = next(tp.parameters()).device
        path_list = [(ii, io, (w.detach() * s).float().cpu().numpy().transpose(1, 0, 2).copy()) for (ii, io, s), w
                     in zip(tp.paths, tp.weight)]                        # [mul_in, n_elem, mul_out] -> [e, u, w]
        self._build(tp.irreps_in1, tp.irreps_out, path_list, dev)

    def forward(self, x1, node_attrs):
        from .symmetric import element_groups
        _, erow, perm = element_groups(node_attrs)
        return _BlockLinearFn.apply(x1, self, (perm, erow, self.n_elem))


def mlp_supported(mod):
    """(ok, reason) for an e3nn-style scalar MLP without biases and with SiLU (MACE's radial MLP)."""
    ws = getattr(mod, 'weights', None)
    if ws is None or not hasattr(mod, 'hs') or not hasattr(mod, '_SILU_2MOM'):
        return False, 'not a bias-free scalar MLP'
    if getattr(mod, 'act', None) is not torch.nn.functional.silu:
        return False, 'activation is not SiLU'
    if any(p.requires_grad for p in mod.parameters()):
        return False, 'weights require grad (training): frozen weights only'
    return True, ''


class _MLPHiddenFn(torch.autograd.Function):
    """The hidden layers h_{i+1} = c * silu(h_i @ W_i) of the MLP (all but the last layer)."""

    @staticmethod
    def forward(ctx, x, op):
        h = x.contiguous()
        if h.dtype != torch.float32 or not h.is_cuda:
            raise TypeError('input must be a float32 CUDA tensor')
        N = h.shape[0]
        zs = []
        for fwd, dout in zip(op.fwd, op.dims[1:]):
            out = torch.empty(N, dout, device=h.device, dtype=torch.float32)
            z = torch.empty_like(out)
            op._launch(fwd, h, out, epilogue=z)
            zs.append(z)
            h = out
        ctx.save_for_backward(*zs)
        ctx.op = op
        return h

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        op, zs = ctx.op, ctx.saved_tensors
        g = g.contiguous()
        for i in range(len(op.bwd) - 1, -1, -1):
            gin = torch.empty(g.shape[0], op.dims[i], device=g.device, dtype=torch.float32)
            op._launch(op.bwd[i], g, gin, prologue=zs[i])            # through layer i's activation, then W_i^T
            g = gin
        return g, None


MLP_FUSED_MAX_WIDTH, MLP_FUSED_MAX_LAYERS = 64, 4      # limits of mmk_mlp_fwd / mmk_mlp_bwd


class _MLPFusedFn(torch.autograd.Function):
    """All hidden layers in one launch each way (mmk_mlp_fwd / mmk_mlp_bwd); the pre-activations are saved."""

    @staticmethod
    def forward(ctx, x, op):
        x = x.contiguous()
        if x.dtype != torch.float32 or not x.is_cuda:
            raise TypeError('input must be a float32 CUDA tensor')
        E, L = x.shape[0], len(op.hidden_widths) - 1
        h = torch.empty(E, op.hidden_widths[-1], device=x.device, dtype=torch.float32)
        z = torch.empty(E * sum(op.hidden_widths[1:]), device=x.device, dtype=torch.float32)
        _lib.call('mmk_mlp_fwd', _lib.ptr(x), E, L, op.widths_c(), _lib.ptr(op.w_hidden), op.scale, _lib.ptr(h),
                  _lib.ptr(z), _lib.stream_of(x))
        ctx.save_for_backward(z)
        ctx.op = op
        return h

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        op, (z,) = ctx.op, ctx.saved_tensors
        g = g.contiguous()
        E, L = g.shape[0], len(op.hidden_widths) - 1
        gx = torch.empty(E, op.hidden_widths[0], device=g.device, dtype=torch.float32)
        _lib.call('mmk_mlp_bwd', _lib.ptr(g), E, L, op.widths_c(), _lib.ptr(op.w_hidden_t), _lib.ptr(z), op.scale,
                  _lib.ptr(gx), _lib.stream_of(g))
        return gx, None


class CudaFullyConnectedNet(torch.nn.Module):
    """Drop-in for MACE's radial MLP (frozen weights): forward(x[E, h0]) -> [E, h_last].  The hidden layers run in one
    launch each way (``mmk_mlp_fwd`` / ``mmk_mlp_bwd``: every layer's weights and the activation tile of a block of
    edges stay in shared memory) when they have at most 4 layers of width <= 64 (MACE: 8 -> 64 -> 64 -> 64), else as
    one block-linear launch per layer with the activation fused.  The last layer (a plain product, large: h_last =
    NINS x C) is one tensor-core GEMM each way with the pre-scaled weight (``gemm.TensorCoreLinear``)."""

    def __init__(self, mlp):
        super().__init__()
        ok, why = mlp_supported(mlp)
        if not ok:
            raise ValueError(why)
        self.hs = list(mlp.hs)
        self.dims = self.hs
        self.scale = float(mlp._SILU_2MOM)
        dev = next(mlp.parameters()).device
        self.fwd, self.bwd = [], []
        ws = list(mlp.weights)
        scaled = [(w.detach() / np.sqrt(w.shape[0])).float() for w in ws]    # as the module scales them
        for W in (w.cpu().numpy() for w in scaled[:-1]):
            self.fwd.append(_Tables([(0, W.shape[1], 1)], [(0, 0, W[None])], dev))
            self.bwd.append(_Tables([(0, W.shape[0], 1)], [(0, 0, np.ascontiguousarray(W.T)[None])], dev))
        self.hidden_widths = tuple(int(h) for h in self.hs[:-1])
        self.fused = (1 <= len(self.hidden_widths) - 1 <= MLP_FUSED_MAX_LAYERS and
                      max(self.hidden_widths) <= MLP_FUSED_MAX_WIDTH)
        hidden = scaled[:-1] or [torch.zeros(1, 1)]
        self.register_buffer('w_hidden', torch.cat([w.reshape(-1) for w in hidden]).contiguous().to(dev))
        self.register_buffer('w_hidden_t', torch.cat([w.t().reshape(-1) for w in hidden]).contiguous().to(dev))
        self.register_buffer('w_last', scaled[-1].contiguous())
        from .gemm import TensorCoreLinear
        self.last = TensorCoreLinear(scaled[-1].to(dev))

    def widths_c(self):
        return (ctypes.c_int * len(self.hidden_widths))(*self.hidden_widths)

    def _launch(self, t, x, out, epilogue=None, prologue=None):
        _lib.call('mmk_block_linear_act', _lib.ptr(x), x.shape[1], _lib.ptr(out), out.shape[1], _lib.ptr(t.blocks),
                  t.n_blocks, _lib.ptr(t.paths), _lib.ptr(t.w), t.max_d, t.max_mul, None, None, 1, x.shape[0],
                  int(epilogue is not None), _lib.ptr(epilogue), int(prologue is not None), _lib.ptr(prologue),
                  self.scale, _lib.stream_of(x))

    def forward(self, x):
        if not self.fwd:
            h = x
        elif self.fused:
            h = _MLPFusedFn.apply(x, self)
        else:
            h = _MLPHiddenFn.apply(x, self)
        return self.last(h)


def reshape_supported(mod):
    """(ok, reason) for MACE's ``reshape_irreps`` module (irreps layout -> [N, mul, sum (2l+1)])."""
    irreps = getattr(mod, 'irreps', None)
    if irreps is None or not hasattr(mod, 'muls') or not hasattr(mod, 'dims'):
        return False, 'not a reshape_irreps module'
    if getattr(mod, 'cueq_config', None) is not None and getattr(mod.cueq_config, 'enabled', False):
        return False, 'cuequivariance layout'
    if len(set(int(m) for m in mod.muls)) != 1:
        return False, 'unequal multiplicities'
    return True, ''


class _GatherColumnsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fwd, bwd, shape):
        xc = x.contiguous()
        if xc.dtype != torch.float32 or not xc.is_cuda:
            raise TypeError('input must be a float32 CUDA tensor')
        N, D = xc.shape
        out = torch.empty((N,) + tuple(shape), device=xc.device, dtype=torch.float32)
        _lib.call('mmk_gather_columns', _lib.ptr(xc), D, _lib.ptr(out), D, _lib.ptr(fwd), N, D, _lib.stream_of(xc))
        ctx.bwd, ctx.D = bwd, D
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        gc = g.contiguous()
        N, D = gc.shape[0], ctx.D
        gx = torch.empty(N, D, device=gc.device, dtype=torch.float32)
        _lib.call('mmk_gather_columns', _lib.ptr(gc), D, _lib.ptr(gx), D, _lib.ptr(ctx.bwd), N, D, _lib.stream_of(gc))
        return gx, None, None, None


class CudaReshapeIrreps(torch.nn.Module):
    """Drop-in for MACE's ``reshape_irreps``: [N, sum mul (2l+1)] (mul_ir layout) -> [N, mul, sum (2l+1)], one
    column-gather launch each way (C ABI ``mmk_gather_columns``) instead of a slice + reshape + cat forward and a
    zero-fill + copy + add per block backward."""

    def __init__(self, mod, device=None):
        super().__init__()
        ok, why = reshape_supported(mod)
        if not ok:
            raise ValueError(why)
        self.irreps = mod.irreps
        self.muls, self.dims = list(mod.muls), list(mod.dims)
        mul, dsum = int(self.muls[0]), int(sum(self.dims))
        fwd = np.empty((mul, dsum), dtype=np.int32)          # out[n, u, off_b + m] = x[n, xoff_b + u d_b + m]
        xoff = off = 0
        for d in self.dims:
            fwd[:, off:off + d] = xoff + np.arange(mul)[:, None] * d + np.arange(d)[None, :]
            xoff += mul * d
            off += d
        fwd = fwd.reshape(-1)
        bwd = np.empty_like(fwd)
        bwd[fwd] = np.arange(fwd.size, dtype=np.int32)
        self.register_buffer('fwd_cols', torch.from_numpy(fwd).to(device), persistent=False)
        self.register_buffer('bwd_cols', torch.from_numpy(bwd).to(device), persistent=False)
        self.shape = (mul, dsum)

    def forward(self, tensor):
        return _GatherColumnsFn.apply(tensor, self.fwd_cols, self.bwd_cols, self.shape)
