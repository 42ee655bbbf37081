"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): float64 restatement of the reference's convolution path.

Reference = Yike-Ye/mace-mps-kernels v0.1.0, file src/mace_mps_kernels/conv.py.
"""
from __future__ import annotations

import numpy as np
import torch


def blocks(irreps):
    """[(l, mul, offset)], total dim -- conv.py:23-28."""
    res, off = [], 0
    for mul, ir in irreps:
        res.append((ir.l, mul, off))
        off += mul * (2 * ir.l + 1)
    return res, off


def probe_coefficients(tp, tol=1e-7):
    """Per-instruction effective coefficients c_k[a, b, m] measured with unit inputs on channel 0 -- conv.py:57-88.

    Returns (spec dict, coef list); coef[k] = dict(k, l1, l2, l3, o1, o2, o3, terms=[(a, b, m, c)])."""
    in1, x_dim = blocks(tp.irreps_in1)
    in2, y_dim = blocks(tp.irreps_in2)
    outb, out_dim = blocks(tp.irreps_out)
    mul = in1[0][1]
    ins = [(i.i_in1, i.i_in2, i.i_out) for i in tp.instructions]
    dev = next(iter(tp.buffers()), torch.zeros(1)).device
    coef = []
    for k, (i1, i2, io) in enumerate(ins):
        l1, _, o1 = in1[i1]
        l2, _, o2 = in2[i2]
        l3, _, o3 = outb[io]
        d1, d2, d3 = 2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1
        x1 = torch.zeros(d1 * d2, x_dim, device=dev)
        x2 = torch.zeros(d1 * d2, y_dim, device=dev)
        w = torch.zeros(d1 * d2, tp.weight_numel, device=dev)
        for a in range(d1):
            for b in range(d2):
                x1[a * d2 + b, o1 + a] = 1.0
                x2[a * d2 + b, o2 + b] = 1.0
                w[a * d2 + b, k * mul] = 1.0
        with torch.no_grad():
            y = tp(x1, x2, w)[:, o3:o3 + d3].detach().cpu().double().reshape(d1, d2, d3).numpy()
        terms = [(a, b, m, float(y[a, b, m])) for a in range(d1) for b in range(d2) for m in range(d3)
                 if abs(float(y[a, b, m])) > tol]
        coef.append(dict(k=k, l1=l1, l2=l2, l3=l3, o1=o1, o2=o2, o3=o3, terms=terms))
    spec = dict(mul=mul, x_dim=x_dim, y_dim=y_dim, out_dim=out_dim, nins=len(ins), ins=ins)
    return spec, coef


def csr_by(index, n):
    """Stable sort of edges by index -> (rowptr int32[n+1], eids int32[E]) -- conv.py:229-235."""
    index = np.asarray(index, np.int64)
    order = np.argsort(index, kind='stable')
    counts = np.bincount(index, minlength=n)
    rowptr = np.zeros(n + 1, np.int64)
    rowptr[1:] = np.cumsum(counts)
    return rowptr.astype(np.int32), order.astype(np.int32)


def _dense(c):
    C = np.zeros((2 * c['l1'] + 1, 2 * c['l2'] + 1, 2 * c['l3'] + 1))
    for a, b, m, v in c['terms']:
        C[a, b, m] += v
    return C


def conv_fwd(spec, coef, x, Y, W, send, recv, n_nodes):
    """out[n, o3 + u d3 + m] = sum_{e: recv(e)=n} W[e, k mul + u] sum_{a,b} c_k[a,b,m] x[send(e), o1 + u d1 + a]
    Y[e, o2 + b] -- the semantics of the generated conv_fwd kernel, conv.py:109-141 (per-edge messages, then a
    scatter-sum as e3nn does)."""
    x, Y, W = (np.asarray(t, np.float64) for t in (x, Y, W))
    mul, E = spec['mul'], Y.shape[0]
    out = np.zeros((n_nodes, spec['out_dim']))
    for c in coef:
        d1, d2, d3 = 2 * c['l1'] + 1, 2 * c['l2'] + 1, 2 * c['l3'] + 1
        X1 = x[send, c['o1']:c['o1'] + mul * d1].reshape(E, mul, d1)
        Yb = Y[:, c['o2']:c['o2'] + d2]
        w = W[:, c['k'] * mul:(c['k'] + 1) * mul]
        msg = np.einsum('eua,eb,abm,eu->eum', X1, Yb, _dense(c), w).reshape(E, mul * d3)
        np.add.at(out[:, c['o3']:c['o3'] + mul * d3], recv, msg)
    return out


def conv_bwd(spec, coef, x, Y, W, g, send, recv):
    """(gx, gY, gW) of sum(out * g) -- conv.py:144-176 (conv_bwd_x) and conv.py:179-222 (conv_bwd_wy)."""
    x, Y, W, g = (np.asarray(t, np.float64) for t in (x, Y, W, g))
    mul, E = spec['mul'], Y.shape[0]
    gx = np.zeros_like(x)
    gY = np.zeros_like(Y)
    gW = np.zeros_like(W)
    for c in coef:
        d1, d2, d3 = 2 * c['l1'] + 1, 2 * c['l2'] + 1, 2 * c['l3'] + 1
        C = _dense(c)
        X1 = x[send, c['o1']:c['o1'] + mul * d1].reshape(E, mul, d1)
        Yb = Y[:, c['o2']:c['o2'] + d2]
        G = g[recv, c['o3']:c['o3'] + mul * d3].reshape(E, mul, d3)
        ks = slice(c['k'] * mul, (c['k'] + 1) * mul)
        w = W[:, ks]
        gW[:, ks] += np.einsum('eua,eb,abm,eum->eu', X1, Yb, C, G)
        gY[:, c['o2']:c['o2'] + d2] += np.einsum('eua,abm,eum,eu->eb', X1, C, G, w)
        gxe = np.einsum('eb,abm,eum,eu->eua', Yb, C, G, w).reshape(E, mul * d1)
        np.add.at(gx[:, c['o1']:c['o1'] + mul * d1], send, gxe)
    return gx, gY, gW
