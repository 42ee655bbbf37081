"""float32 matrix products on the B200 tensor cores (C ABI ``mmk_gemm_tf32x3``): tcgen05 ``kind::tf32`` MMAs with
the accumulator in tensor memory and the 3xTF32 split, a = tf32(a) + tf32(a - tf32(a)), so that the result keeps
float32 accuracy (the cross term of the two low parts, ~2^-22 relative, is the only one dropped).

``TensorCoreLinear`` holds a constant weight already split; its product with an activation matrix splits the
activation while the kernel stages it.  Used for the radial MLP's last layer (W[E, NINS*C] = h[E, 64] . Wr) and its
input gradient (gh = gW . Wr^T).
"""
from __future__ import annotations

import torch

from . import _lib
from .conv import DOUBLE_BACKWARD_MSG


def tf32_split(t: torch.Tensor):
    """(hi, lo) float32 tensors with hi = tf32(t) (round to nearest) and lo = tf32(t - hi), on t's device."""
    t = _lib.aligned(t.detach().float().contiguous())
    hi, lo = torch.empty_like(t), torch.empty_like(t)
    _lib.call('mmk_tf32_split', _lib.ptr(t), _lib.ptr(hi), _lib.ptr(lo), t.numel(), _lib.stream_of(t))
    return hi, lo


def tf32_split_host(t: torch.Tensor):
    """The same split computed on the host (for constant operands): round to nearest with ties away from zero to the
    10 explicit mantissa bits TF32 keeps (add half a TF32 unit to the magnitude bits, clear the 13 low bits)."""
    import numpy as np
    x = t.detach().cpu().float().contiguous().numpy()

    def rna(v):
        b = v.view(np.uint32)
        return ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)

    hi = rna(x)
    lo = rna((x - hi).astype(np.float32))
    return torch.from_numpy(hi.copy()), torch.from_numpy(lo.copy())


_WORKSPACE = {}          # device -> zero-initialised uint8 tensor (K-split partial tiles and tile counters)


def _workspace(M, N, K, device):
    """The per-device workspace of the K-split launches, grown on demand (zero-filled: the kernel leaves its tile
    counters at zero after every call, so a buffer is reused as is)."""
    need = int(_lib.lib().mmk_gemm_workspace_bytes(M, N, K))
    if need == 0:
        return None, 0
    ws = _WORKSPACE.get(device)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=device)
        _WORKSPACE[device] = ws
    return ws, ws.numel()


def matmul_nt(a: torch.Tensor, b_hi: torch.Tensor, b_lo: torch.Tensor, out: torch.Tensor | None = None):
    """a [M, K] . b^T with b = b_hi + b_lo [N, K] (split by ``tf32_split``) -> [M, N], float32."""
    if a.dtype != torch.float32 or not a.is_cuda:
        raise TypeError(f'expected a float32 CUDA tensor (got {a.dtype} on {a.device})')
    a = _lib.aligned(a.contiguous())
    M, K = a.shape
    N = b_hi.shape[0]
    if b_hi.shape != (N, K) or b_lo.shape != (N, K):
        raise ValueError(f'operand shapes {tuple(a.shape)} x {tuple(b_hi.shape)}^T do not match')
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=torch.float32)
    ws, nbytes = _workspace(M, N, K, a.device)
    _lib.call('mmk_gemm_tf32x3', _lib.ptr(a), a.stride(0), _lib.ptr(b_hi), _lib.ptr(b_lo), b_hi.stride(0),
              _lib.ptr(out), out.stride(0), M, N, K, _lib.ptr(ws), nbytes, _lib.stream_of(a))
    return out


def status(reset=False):
    """Nonzero if a tensor-core GEMM gave up on a pipeline wait (its output is invalid); synchronises the device."""
    import ctypes
    v = ctypes.c_int(0)
    _lib.call('mmk_gemm_status', ctypes.byref(v), int(reset))
    return v.value


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, op):
        ctx.op = op
        if op.k_pad:
            x = torch.nn.functional.pad(x, (0, op.k_pad))
        y = matmul_nt(x, op.wt_hi, op.wt_lo)                # x [M, K] . W  (W^T kept as the K-major operand)
        return y[:, :op.n] if op.n_pad else y

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        op = ctx.op
        if op.n_pad:
            g = torch.nn.functional.pad(g, (0, op.n_pad))
        gx = matmul_nt(g, op.w_hi, op.w_lo)                 # g [M, N] . W^T
        return (gx[:, :op.k] if op.k_pad else gx), None


class TensorCoreLinear(torch.nn.Module):
    """y = x . W for a constant W [K, N] (no bias), forward and input gradient on the tensor cores.  K and N are
    padded with zeros to multiples of 4 where needed (MACE's radial MLP never needs it: 64 x NINS*C)."""

    def __init__(self, weight: torch.Tensor):
        super().__init__()
        w = weight.detach().float()
        self.k, self.n = w.shape
        self.k_pad, self.n_pad = -self.k % 4, -self.n % 4
        w = torch.nn.functional.pad(w, (0, self.n_pad, 0, self.k_pad)).contiguous()
        dev = w.device
        wt_hi, wt_lo = tf32_split_host(w.t())               # [N, K]: forward operand
        w_hi, w_lo = tf32_split_host(w)                     # [K, N]: input-gradient operand
        self.register_buffer('wt_hi', wt_hi.to(dev))
        self.register_buffer('wt_lo', wt_lo.to(dev))
        self.register_buffer('w_hi', w_hi.to(dev))
        self.register_buffer('w_lo', w_lo.to(dev))

    def forward(self, x):
        return _LinearFn.apply(x, self)
