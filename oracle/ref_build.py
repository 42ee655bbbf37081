"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): run the reference's own generated kernels on the CPU.

The reference (Yike-Ye/mace-mps-kernels, Python) generates its Metal kernels as source strings
(src/mace_mps_kernels/conv.py:225-226 ``source``, src/mace_mps_kernels/symmetric.py:82-131 ``source``).  Those kernels
use only scalar arithmetic plus, in ``conv_bwd_wy``, a ``simd_sum`` + threadgroup reduction for d/dY.  This recipe
takes the source the reference generates for a given spec, rewrites the Metal address-space words and attributes
into C++ (``kernel``/``device``/``constant``/``[[...]]``/``uint``), replaces the d/dY channel reduction by a store of
each thread's partial sums (summed afterwards in channel order), and compiles it with g++ into a shared library under
``oracle/_ref/`` (git-ignored), with one driver per kernel that loops over the Metal grid.

It needs a reference checkout: ``$MMK_REFERENCE_SRC`` (the checkout's ``src`` directory), else a ``reference/``
checkout next to this repository.  It only runs where one exists, to generate the committed golden fixtures
(tests/golden/make_golden.py); the GPU tests and the bench never need it.  No reference source is copied into the
repository.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import re
import subprocess
import sys

import numpy as np

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SRC = os.environ.get('MMK_REFERENCE_SRC', os.path.join(os.path.dirname(_REPO), 'reference', 'src'))
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), '_ref')


def reference_available():
    return os.path.isdir(os.path.join(REF_SRC, 'mace_mps_kernels'))


def import_reference():
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    import mace_mps_kernels.conv as rc
    import mace_mps_kernels.symmetric as rs
    return rc, rs


def metal_to_cpp(src: str) -> str:
    lines = []
    for ln in src.split('\n'):
        s = ln.strip()
        if s.startswith('#include <metal_stdlib>') or s == 'using namespace metal;':
            continue
        if s.startswith('threadgroup float part'):
            continue
        if s.startswith('threadgroup_barrier'):
            continue
        if 'simd_sum(' in s:                                   # per-thread partials instead of the simdgroup sum
            m = re.match(r'for \(int j = 0; j < (\d+); \+\+j\)', s)
            yd = m.group(1)
            lines.append(f'  for (int j = 0; j < {yd}; ++j) mmk_gy_partial[(size_t)gid * {yd} + j] = gy[j];')
            continue
        lines.append(ln)
    out = '\n'.join(lines)
    # drop the final threadgroup reduction block of conv_bwd_wy: "if (e < E && tid < Y) { ... gY[...] = v; }"
    out = re.sub(r'\n\s*if \(e < E && tid < \d+\) \{ float v = 0\.0f;\n\s*for \(int q = 0;[^\n]*\n\s*gY\[[^\n]*\}', '',
                 out)
    out = re.sub(r'\s*\[\[[^\]]*\]\]', '', out)
    out = out.replace('kernel void', 'static void').replace('device ', '').replace('constant ', 'const ')
    out = re.sub(r'\buint\b', 'unsigned', out)
    return out


CONV_DRIVER = r'''
#include <cstddef>
static float *mmk_gy_partial;
%(body)s
extern "C" void run_conv_fwd(const float *x, const float *Y, const float *W, const int *rowptr, const int *eids,
                             const int *senders, float *out, unsigned N, unsigned MUL) {
    for (unsigned gid = 0; gid < N * MUL; ++gid) conv_fwd(x, Y, W, rowptr, eids, senders, out, N, gid);
}
extern "C" void run_conv_bwd_x(const float *g, const float *Y, const float *W, const int *rowptr, const int *eids,
                               const int *receivers, float *gx, unsigned N, unsigned MUL) {
    for (unsigned gid = 0; gid < N * MUL; ++gid) conv_bwd_x(g, Y, W, rowptr, eids, receivers, gx, N, gid);
}
extern "C" void run_conv_bwd_wy(const float *x, const float *g, const float *Y, const float *W, const int *senders,
                                const int *receivers, float *gW, float *gy_partial, unsigned E, unsigned MUL) {
    mmk_gy_partial = gy_partial;
    for (unsigned gid = 0; gid < E * MUL; ++gid) {
        unsigned tid = gid %% MUL;
        conv_bwd_wy(x, g, Y, W, senders, receivers, gW, nullptr, E, gid, tid, tid / 32, tid %% 32);
    }
}
'''

SC_DRIVER = r'''
#include <cstddef>
%(body)s
extern "C" void run_sc_fwd(const float *X, const int *elem, const float *T, float *out, unsigned N, unsigned C) {
    for (unsigned gid = 0; gid < N * C; ++gid) sc_fwd(X, elem, T, out, N, gid);
}
extern "C" void run_sc_bwd(const float *X, const int *elem, const float *T, const float *G, float *GX, unsigned N,
                           unsigned C) {
    for (unsigned gid = 0; gid < N * C; ++gid) sc_bwd(X, elem, T, G, GX, N, gid);
}
'''


def _compile(cpp: str, tag: str):
    os.makedirs(OUT, exist_ok=True)
    h = hashlib.sha1(cpp.encode()).hexdigest()[:12]
    src = os.path.join(OUT, f'{tag}_{h}.cpp')
    so = os.path.join(OUT, f'{tag}_{h}.so')
    if not os.path.exists(so):
        with open(src, 'w') as f:
            f.write(cpp)
        subprocess.run(['g++', '-O1', '-std=c++17', '-fPIC', '-shared', '-ffp-contract=off', src, '-o', so],
                       check=True)
    return ctypes.CDLL(so)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class RefConv:
    """The reference's ConvSpec + its generated conv kernels, compiled for the CPU."""

    def __init__(self, tp):
        rc, _ = import_reference()
        self.spec = rc.ConvSpec(tp)
        self.lib = _compile(CONV_DRIVER % {'body': metal_to_cpp(rc.source(self.spec))}, 'conv')
        self.csr_by = rc.csr_by

    def csr(self, index, n):
        import torch
        rowptr, eids = self.csr_by(torch.as_tensor(np.asarray(index, np.int64)), n)
        return rowptr.numpy().astype(np.int32), eids.numpy().astype(np.int32)

    def fwd(self, x, Y, W, send, recv, N):
        x, Y, W = (np.ascontiguousarray(a, np.float32) for a in (x, Y, W))
        rowptr, eids = self.csr(recv, N)
        send32 = np.ascontiguousarray(send, np.int32)
        out = np.zeros((N, self.spec.out_dim), np.float32)
        self.lib.run_conv_fwd(_p(x), _p(Y), _p(W), _p(rowptr), _p(eids), _p(send32), _p(out), N, self.spec.mul)
        return out

    def bwd(self, x, Y, W, g, send, recv, N):
        x, Y, W, g = (np.ascontiguousarray(a, np.float32) for a in (x, Y, W, g))
        E = Y.shape[0]
        rowptr, eids = self.csr(send, N)
        s32, r32 = np.ascontiguousarray(send, np.int32), np.ascontiguousarray(recv, np.int32)
        gx = np.zeros_like(x)
        self.lib.run_conv_bwd_x(_p(g), _p(Y), _p(W), _p(rowptr), _p(eids), _p(r32), _p(gx), N, self.spec.mul)
        gW = np.zeros_like(W)
        part = np.zeros((E * self.spec.mul, Y.shape[1]), np.float32)
        self.lib.run_conv_bwd_wy(_p(x), _p(g), _p(Y), _p(W), _p(s32), _p(r32), _p(gW), _p(part), E, self.spec.mul)
        gY = part.reshape(E, self.spec.mul, Y.shape[1]).sum(1, dtype=np.float32)
        return gx, gY, gW


class RefSC:
    """The reference's SCSpec + its generated symmetric-contraction kernels, compiled for the CPU."""

    def __init__(self, sc):
        _, rs = import_reference()
        self.spec = rs.SCSpec(sc)
        self.lib = _compile(SC_DRIVER % {'body': metal_to_cpp(rs.source(self.spec))}, 'sc')
        self.T = np.ascontiguousarray(self.spec.T.numpy(), np.float32)

    def fwd(self, x, elem):
        x = np.ascontiguousarray(x, np.float32)
        N = x.shape[0]
        e32 = np.ascontiguousarray(elem, np.int32)
        out = np.zeros((N, self.spec.out_dim), np.float32)
        self.lib.run_sc_fwd(_p(x), _p(e32), _p(self.T), _p(out), N, self.spec.C)
        return out

    def bwd(self, x, elem, g):
        x, g = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(g, np.float32)
        N = x.shape[0]
        e32 = np.ascontiguousarray(elem, np.int32)
        gx = np.zeros_like(x)
        self.lib.run_sc_bwd(_p(x), _p(e32), _p(self.T), _p(g), _p(gx), N, self.spec.C)
        return gx
