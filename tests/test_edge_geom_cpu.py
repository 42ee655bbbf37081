"""The per-edge geometry arithmetic of the CUDA kernels (csrc/edge_geom.cuh), compiled for the host, against the
model's own modules in float64 with autograd (no GPU needed): spherical harmonics and their gradient w.r.t. the edge
vector, radial embedding and its gradient w.r.t. the length, including lengths at and beyond the cutoff."""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from mace_mps_kernels_b200.standin import o3
from mace_mps_kernels_b200.standin.modules import RadialEmbeddingBlock

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'mace_mps_kernels_b200', 'csrc')

DRIVER = r'''
#include <cstdio>
#define MMK_HD
#include "edge_geom.cuh"
// stdin: n_sh, per sample v[3] gY[16]; n_rad, n_bessel, w[n_bessel], prefactor, r_max, p, per sample r g[n_bessel]
// stdout: per sh sample Y[16] gv[3]; per radial sample out[n_bessel] glen
int main() {
    int n;
    if (fread(&n, 4, 1, stdin) != 1) return 1;
    const MmkShNorm N = mmk_sh_norms(3);
    for (int s = 0; s < n; ++s) {
        float v[3], gY[16], Y[16], gv[3];
        if (fread(v, 4, 3, stdin) != 3 || fread(gY, 4, 16, stdin) != 16) return 2;
        sh_forward<3>(v, N, Y);
        sh_backward<3>(v, gY, N, gv);
        fwrite(Y, 4, 16, stdout);
        fwrite(gv, 4, 3, stdout);
    }
    MmkRadial R;
    if (fread(&n, 4, 1, stdin) != 1 || fread(&R.n, 4, 1, stdin) != 1) return 3;
    if (fread(R.w, 4, R.n, stdin) != (size_t)R.n || fread(&R.prefactor, 4, 1, stdin) != 1 ||
        fread(&R.r_max, 4, 1, stdin) != 1 || fread(&R.p, 4, 1, stdin) != 1)
        return 4;
    for (int s = 0; s < n; ++s) {
        float r, g[16], out[16];
        if (fread(&r, 4, 1, stdin) != 1 || fread(g, 4, R.n, stdin) != (size_t)R.n) return 5;
        radial_forward(r, R, out);
        const float gl = radial_backward(r, g, R);
        fwrite(out, 4, R.n, stdout);
        fwrite(&gl, 4, 1, stdout);
    }
    return 0;
}
'''


def test_edge_geometry_matches_model_modules(tmp_path):
    gxx = shutil.which('g++')
    if gxx is None:
        pytest.skip('g++ not available')
    (tmp_path / 'drv.cpp').write_text(DRIVER)
    exe = tmp_path / 'drv'
    r = subprocess.run([gxx, '-O1', '-std=c++17', '-I', CSRC, str(tmp_path / 'drv.cpp'), '-o', str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]

    rng = np.random.default_rng(5)
    n_sh = 64
    v = rng.standard_normal((n_sh, 3)).astype(np.float32) * rng.uniform(0.5, 5.0, (n_sh, 1)).astype(np.float32)
    v[0] = [0.0, 0.0, 2.0]                                   # on the z axis
    v[1] = [1e3, 0.0, 0.0]                                   # a padding edge (far along x)
    gY = rng.standard_normal((n_sh, 16)).astype(np.float32)
    block = RadialEmbeddingBlock(5.0, 8, 5)
    w = block.bessel_fn.bessel_weights.numpy().astype(np.float32)
    n_rad = 40
    lengths = np.concatenate([rng.uniform(0.3, 5.5, n_rad - 3), [5.0, 4.9999, 1e3]]).astype(np.float32)
    gR = rng.standard_normal((n_rad, 8)).astype(np.float32)
    payload = np.int32(n_sh).tobytes() + b''.join(v[k].tobytes() + gY[k].tobytes() for k in range(n_sh))
    payload += np.int32(n_rad).tobytes() + np.int32(8).tobytes() + w.tobytes()
    payload += np.float32(float(block.bessel_fn.prefactor)).tobytes() + np.float32(5.0).tobytes()
    payload += np.float32(5.0).tobytes()
    payload += b''.join(np.float32(lengths[k]).tobytes() + gR[k].tobytes() for k in range(n_rad))
    r = subprocess.run([str(exe)], input=payload, capture_output=True)
    assert r.returncode == 0, r.stderr
    res = np.frombuffer(r.stdout, dtype=np.float32)
    sh = res[:n_sh * 19].reshape(n_sh, 19)
    rad = res[n_sh * 19:].reshape(n_rad, 9)

    # float64 references through the model's own modules
    vt = torch.tensor(v, dtype=torch.float64, requires_grad=True)
    Y = o3.spherical_harmonics(3, vt, normalize=True)
    (gv,) = torch.autograd.grad(Y, vt, torch.tensor(gY, dtype=torch.float64))
    assert np.abs(sh[:, :16] - Y.detach().numpy()).max() < 2e-5 * np.abs(Y.detach().numpy()).max()
    gvn = gv.numpy()
    assert np.abs(sh[:, 16:] - gvn).max() < 2e-5 * np.abs(gvn).max()

    blk64 = RadialEmbeddingBlock(5.0, 8, 5).double()
    lt = torch.tensor(lengths[:, None], dtype=torch.float64, requires_grad=True)
    out = blk64(lt)
    (gl,) = torch.autograd.grad(out, lt, torch.tensor(gR, dtype=torch.float64))
    ref = out.detach().numpy()
    assert np.abs(rad[:, :8] - ref).max() < 2e-5 * np.abs(ref).max()
    assert np.abs(rad[:, 8] - gl.numpy()[:, 0]).max() < 2e-5 * np.abs(gl.numpy()).max()
    assert np.all(rad[-1] == 0.0)                            # beyond the cutoff: no feature, no gradient


def test_edge_vector_patch_is_scoped_to_patched_models():
    """patch_edge_vectors replaces the model module's get_edge_vectors_and_lengths by a wrapper that takes the CUDA
    path only inside a patched model's forward and for CUDA float32 inputs; everything else calls the original, so
    on the CPU a patched model and an unpatched one give the same energies and forces."""
    import copy
    import numpy as np
    import torch
    from mace_mps_kernels_b200 import standin
    from mace_mps_kernels_b200.edge import _ACTIVE, patch_edge_vectors
    from mace_mps_kernels_b200.standin import modules
    ref = standin.make_model('8x0e+8x1o', 2, 2, seed=0)
    met = copy.deepcopy(ref)
    before = modules.get_edge_vectors_and_lengths
    try:
        assert patch_edge_vectors(met) == (True, '')
        wrapped = modules.get_edge_vectors_and_lengths
        assert wrapped is not before and wrapped._mmk_original is before
        assert patch_edge_vectors(met) == (True, '')                  # idempotent: no second wrapper, no second hook
        assert modules.get_edge_vectors_and_lengths is wrapped
        st = standin.pt100_co_h(seed=0)
        b = standin.structure_batch([st], standin.ELEMENTS_PTCOH, 5.0)
        outs = []
        for m in (ref, met):
            bb = dict(b)
            bb['positions'] = b['positions'].clone().requires_grad_(True)
            o = m(bb, compute_force=True)
            outs.append((o['energy'].detach().numpy(), o['forces'].detach().numpy()))
        assert _ACTIVE[0] == 0                                        # the hooks balanced
        bad = dict(b)
        del bad['shifts']
        with pytest.raises(KeyError):
            met(bad, compute_force=False)
        assert _ACTIVE[0] == 0                                        # ... also when the forward raises
        # (the CPU's threaded reductions vary by ~1e-9 from run to run, so not bit for bit)
        np.testing.assert_allclose(outs[0][0], outs[1][0], rtol=1e-6, atol=0)
        np.testing.assert_allclose(outs[0][1], outs[1][1], rtol=0, atol=1e-8)
    finally:
        modules.get_edge_vectors_and_lengths = before


def test_edge_vectors_argument_errors():
    """The fused edge-vector op rejects what its kernel cannot read, before anything is launched (no GPU needed)."""
    import torch
    from mace_mps_kernels_b200.edge import edge_vectors_and_lengths
    pos, sh = torch.zeros(4, 3), torch.zeros(5, 3)
    with pytest.raises(ValueError, match='int64'):
        edge_vectors_and_lengths(pos, torch.zeros(2, 5, dtype=torch.int32), sh)
    with pytest.raises(ValueError, match='contiguous'):
        edge_vectors_and_lengths(pos, torch.zeros(5, 2, dtype=torch.int64).t(), sh)
    with pytest.raises(ValueError, match='shifts'):
        edge_vectors_and_lengths(pos, torch.zeros(2, 5, dtype=torch.int64), torch.zeros(4, 3))


def test_edge_vector_patch_skips_models_that_do_not_call_the_function():
    """A model whose forward does not call get_edge_vectors_and_lengths itself is reported as skipped, not patched."""
    import torch
    from mace_mps_kernels_b200.edge import patch_edge_vectors

    class Other(torch.nn.Module):
        def forward(self, x):
            return x

    ok, why = patch_edge_vectors(Other())
    assert not ok and 'get_edge_vectors_and_lengths' in why
