"""The generated per-layer CUDA code, compiled for the host and checked against the float64 oracle (no GPU needed).

``conv.source`` / ``symmetric.source`` return the layer header the runtime compiles with NVRTC for sm_100a.  Its
arithmetic (the per-edge conv bodies of every instruction part, the Horner-scheme symmetric-contraction term code)
is plain C++; with a few host shims (``__device__`` -> nothing, ``float4``, ``__ldg``) g++ compiles it, and a small
driver evaluates it on random inputs.  This pins the code generator itself on the CPU, for the default plans and for
the plan overrides, before any kernel runs.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

import helpers
from oracle import conv_ref, sc_ref

SHIM = r'''
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#define __device__
#define __forceinline__ inline
#define __restrict__
struct alignas(16) float4 { float x, y, z, w; };
static inline float4 make_float4(float a, float b, float c, float d) { return float4{a, b, c, d}; }
template <class T> static inline T __ldg(const T *p) { return *p; }
'''

SC_DRIVER = SHIM + r'''
#include "layer.h"
// stdin: n, then per sample x[NELL] gv[OUTM] col[RP]; stdout: acc[OUTM] d[NELL]
int main() {
    int n;
    if (fread(&n, 4, 1, stdin) != 1) return 1;
    for (int s = 0; s < n; ++s) {
        float x[NELL], gv[OUTM];
        alignas(16) static float col[RP];
        if (fread(x, 4, NELL, stdin) != NELL || fread(gv, 4, OUTM, stdin) != OUTM || fread(col, 4, RP, stdin) != RP)
            return 2;
        float acc[OUTM] = {0}, d[NELL] = {0};
        sc_fwd_body(col, x, acc);
        sc_bwd_body(col, x, gv, d);
        fwrite(acc, 4, OUTM, stdout);
        fwrite(d, 4, NELL, stdout);
    }
    return 0;
}
'''

CONV_DRIVER = SHIM + r'''
#include "layer.h"
#define X_DIM (XR * MUL)
#define OUT_DIM (ORR * MUL)
#define W_DIM (NINS * MUL)
template <int H> void fwd_parts(const float *stage, const float *xrow, int u, const float (&y)[YD], float (&acc)[ORR]) {
    float xs[XR], w[NINS];
    load_x_s(xrow, u, xs);
    fwd_load_w<H>(stage, u, w);
    fwd_edge<H>(xs, y, w, acc);
    if constexpr (H + 1 < FWD_NP) fwd_parts<H + 1>(stage, xrow, u, y, acc);
}
template <int H> void bwd_parts(const float *stage, const float *grow, const float *xrow, int u, const float (&y)[YD],
                                float (&gx)[XR], float *gwrow, float (&gy)[16]) {
    float xs[XR], w[NINS], g[ORR], gw[NINS];
    load_x(xrow, u, xs);
    bwd_load_w<H>(stage, u, w);
    bwd_load_g<H>(grow, u, g);
    bwd_edge<H>(xs, y, w, g, gx, gw, gy);
    bwd_store_gw<H>(gwrow + u, gw);
    if constexpr (H + 1 < BWD_NP) bwd_parts<H + 1>(stage, grow, xrow, u, y, gx, gwrow, gy);
}
// stdin: n, then per edge x[X_DIM] y[YD] W[W_DIM] g[OUT_DIM]; stdout: out[OUT_DIM] gx[X_DIM] gW[W_DIM] gy[YD]
int main() {
    int n;
    if (fread(&n, 4, 1, stdin) != 1) return 1;
    static float x[X_DIM], y[YD], W[W_DIM], g[OUT_DIM], out[OUT_DIM], gx[X_DIM], gW[W_DIM];
    for (int s = 0; s < n; ++s) {
        if (fread(x, 4, X_DIM, stdin) != X_DIM || fread(y, 4, YD, stdin) != YD || fread(W, 4, W_DIM, stdin) != W_DIM ||
            fread(g, 4, OUT_DIM, stdin) != OUT_DIM)
            return 2;
        float gy[16] = {0};
        float yy[YD];
        memcpy(yy, y, sizeof yy);
        for (int u = 0; u < MUL; ++u) {
            float acc[ORR] = {0}, gxa[XR] = {0};
            fwd_parts<0>(W, x, u, yy, acc);
            store_out_all(out, u, acc);
            bwd_parts<0>(W, g, x, u, yy, gxa, gW, gy);
            store_x(gx, u, gxa);
        }
        fwrite(out, 4, OUT_DIM, stdout);
        fwrite(gx, 4, X_DIM, stdout);
        fwrite(gW, 4, W_DIM, stdout);
        fwrite(gy, 4, YD, stdout);
    }
    return 0;
}
'''


def _gxx():
    gxx = shutil.which('g++')
    if gxx is None:
        pytest.skip('g++ not available')
    return gxx


def _build(tmp_path, header, driver, extra=''):
    (tmp_path / 'layer.h').write_text(header + extra)
    (tmp_path / 'drv.cpp').write_text(driver)
    exe = tmp_path / 'drv'
    r = subprocess.run([_gxx(), '-O1', '-std=c++17', '-w', '-I', str(tmp_path), str(tmp_path / 'drv.cpp'), '-o',
                        str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


def _run(exe, payload):
    r = subprocess.run([str(exe)], input=payload, capture_output=True)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.frombuffer(r.stdout, dtype=np.float32)


def _rel(a, b):
    return np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30)


SC_CASES = [('32x0e+32x1o', 3, 3, 0), ('32x0e+32x1o', 3, 3, 1), ('32x0e+32x1o+32x2e', 3, 3, 0), ('32x0e', 2, 2, 0)]


@pytest.mark.parametrize('hidden,lmax,corr,which', SC_CASES)
def test_generated_sc_code_matches_oracle(tmp_path, hidden, lmax, corr, which):
    from mace_mps_kernels_b200 import symmetric
    from mace_mps_kernels_b200.standin import o3
    from mace_mps_kernels_b200.standin.symmetric_contraction import SymmetricContraction
    torch.manual_seed(3 + which)
    hid = o3.Irreps(hidden)
    C = hid[0].mul
    sh = o3.Irreps.spherical_harmonics(lmax)
    n_elem = 3
    target = hid if which == 0 else o3.Irreps(f'{C}x0e')
    sc = SymmetricContraction((sh * C).sort()[0].simplify(), target, corr, n_elem)
    spec = symmetric.SCSpec(sc)
    ref = sc_ref.sc_spec(sc)
    exe = _build(tmp_path, symmetric.source(spec), SC_DRIVER)
    Tdev = symmetric.device_table(spec.T).numpy()                  # [e, C, RP]
    n_ell, out_dim = (lmax + 1) ** 2, ref['out_dim']
    outm = sum(bl['M'] for bl in ref['blocks'])
    rng = np.random.default_rng(7)
    samples = [(int(rng.integers(n_elem)), int(rng.integers(C))) for _ in range(12)]
    xs = rng.standard_normal((len(samples), n_ell)).astype(np.float32)
    gvs = rng.standard_normal((len(samples), outm)).astype(np.float32)
    payload = np.int32(len(samples)).tobytes()
    for k, (e, c) in enumerate(samples):
        payload += xs[k].tobytes() + gvs[k].tobytes() + Tdev[e, c].astype(np.float32).tobytes()
    res = _run(exe, payload).reshape(len(samples), outm + n_ell)
    for k, (e, c) in enumerate(samples):
        xf = np.zeros((1, C, n_ell))
        xf[0, c] = xs[k]
        g = np.zeros((1, out_dim))
        moff = 0
        acc_ref = np.zeros(outm)
        out = sc_ref.sc_fwd(ref, xf, [e])
        for bl in ref['blocks']:
            M, off = bl['M'], bl['out_off']
            acc_ref[moff:moff + M] = out[0, off + c * M: off + (c + 1) * M]
            g[0, off + c * M: off + (c + 1) * M] = gvs[k, moff:moff + M]
            moff += M
        d_ref = sc_ref.sc_bwd(ref, xf, [e], g)[0, c]
        assert _rel(res[k, :outm], acc_ref) < 2e-5, (k, res[k, :outm], acc_ref)
        assert _rel(res[k, outm:], d_ref) < 2e-5, (k, res[k, outm:], d_ref)


CONV_PLANS = [{}, {'MMK_CONV_FWD_NP': '4', 'MMK_CONV_BWD_NP': '2'}, {'MMK_CONV_BWD_FORM': '0'}]


@pytest.mark.parametrize('env', CONV_PLANS, ids=['default', 'parts', 'per-term'])
@pytest.mark.parametrize('hidden', ['32x0e', '32x0e+32x1o', '32x0e+32x1o+32x2e'])
def test_generated_conv_code_matches_oracle(tmp_path, monkeypatch, env, hidden):
    from mace_mps_kernels_b200 import conv
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    tp = helpers.conv_tp(hidden, 3)
    spec = conv.ConvSpec(tp)
    header = conv.source(spec)
    # the driver stores every part's outputs of a channel at once
    extra = '\n'.join(['inline void store_out_all(float *row, int u, const float (&v)[ORR]) {'] +
                      [f'  fwd_store<{h}>(row, u, v);' for h in range(int(header.split('#define FWD_NP ')[1].split()[0]))] +
                      ['}'])
    exe = _build(tmp_path, header, CONV_DRIVER, '\n' + extra + '\n')
    rspec, coef = conv_ref.probe_coefficients(tp)
    rng = np.random.default_rng(11)
    E = 3
    x = rng.standard_normal((E, rspec['x_dim'])).astype(np.float32)
    Y = rng.standard_normal((E, rspec['y_dim'])).astype(np.float32)
    W = rng.standard_normal((E, tp.weight_numel)).astype(np.float32)
    g = rng.standard_normal((E, rspec['out_dim'])).astype(np.float32)
    payload = np.int32(E).tobytes() + b''.join(x[k].tobytes() + Y[k].tobytes() + W[k].tobytes() + g[k].tobytes()
                                                for k in range(E))
    sizes = [rspec['out_dim'], rspec['x_dim'], tp.weight_numel, rspec['y_dim']]
    res = _run(exe, payload).reshape(E, sum(sizes))
    for k in range(E):
        out, gx, gW, gy = np.split(res[k], np.cumsum(sizes)[:-1])
        # one edge 0 -> 0 (sender = receiver = node 0) with that edge's inputs
        ref = conv_ref.conv_fwd(rspec, coef, x[k:k + 1], Y[k:k + 1], W[k:k + 1], [0], [0], 1)[0]
        rgx, rgY, rgW = conv_ref.conv_bwd(rspec, coef, x[k:k + 1], Y[k:k + 1], W[k:k + 1], g[k:k + 1], [0], [0])
        assert _rel(out, ref) < 2e-5
        assert _rel(gx, rgx[0]) < 2e-5
        assert _rel(gW, rgW[0]) < 2e-5
        assert _rel(gy, rgY[0]) < 2e-5
