"""CPU: the C-ABI library loads without a GPU, exports every entry point include/mmk.h declares, validates
descriptors, and its generated sources compile with NVRTC for sm_100a (NVRTC needs no GPU)."""
import ctypes
import os
import re

import pytest

import helpers

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    hdrs = [os.path.join(ROOT, 'include', f) for f in os.listdir(os.path.join(ROOT, 'include')) if f.endswith('.h')]
    names = set()
    for h in hdrs:
        names |= set(re.findall(r'MMK_API\s+[\w\s\*]*?\b(mmk_\w+)\s*\(', open(h).read()))
    return names


def test_library_exports_every_declared_symbol():
    from mace_mps_kernels_b200 import _lib
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 17
    for n in names:
        assert hasattr(L, n), n
    assert set(_lib.SIGNATURES) == names, 'the ctypes binding and the header disagree'
    assert L.mmk_version().decode() == '0.1.0'


def test_descriptor_validation_errors():
    from mace_mps_kernels_b200 import _lib
    from mace_mps_kernels_b200.conv import ConvSpec
    spec = ConvSpec(helpers.conv_tp('32x0e+32x1o', 3))
    d = spec.descriptor()
    d.mul = 48
    assert _lib.lib().mmk_conv_compile_check(ctypes.byref(d)) == _lib.MMK_ERR_INVALID
    assert 'multiple of 32' in _lib.lib().mmk_last_error().decode()
    d = spec.descriptor()
    d._keep['ta'][0] = 7                      # x component beyond the block
    assert _lib.lib().mmk_conv_compile_check(ctypes.byref(d)) == _lib.MMK_ERR_INVALID
    h = ctypes.c_void_p()
    assert _lib.lib().mmk_conv_layer_create(None, ctypes.byref(h)) == _lib.MMK_ERR_INVALID


@pytest.mark.parametrize('hidden,lmax', [('32x0e', 3), ('32x0e+32x1o', 3), ('64x0e+64x1o', 2),
                                         ('128x0e+128x1o+128x2e', 3)])
def test_generated_conv_source_compiles(hidden, lmax):
    from mace_mps_kernels_b200 import _lib
    from mace_mps_kernels_b200.conv import ConvSpec
    d = ConvSpec(helpers.conv_tp(hidden, lmax)).descriptor()
    _lib.check(_lib.lib().mmk_conv_compile_check(ctypes.byref(d)))


@pytest.mark.parametrize('hidden', ['128x0e', '128x0e+128x1o', '128x0e+128x1o+128x2e'])
@pytest.mark.parametrize('groups', ['1', '4'])
def test_generated_tensor_core_forward_compiles(monkeypatch, hidden, groups):
    """The tcgen05 forward variant (MMK_CONV_FWD_TC=1, 128-channel layers) with one and with four column groups."""
    from mace_mps_kernels_b200 import _lib
    from mace_mps_kernels_b200.conv import ConvSpec
    monkeypatch.setenv('MMK_CONV_FWD_TC', '1')
    monkeypatch.setenv('MMK_CONV_TC_GROUPS', groups)
    d = ConvSpec(helpers.conv_tp(hidden, 3)).descriptor()
    _lib.check(_lib.lib().mmk_conv_compile_check(ctypes.byref(d)))


def test_generated_sc_source_compiles():
    from mace_mps_kernels_b200 import _lib
    from mace_mps_kernels_b200.symmetric import SCSpec
    m = helpers.make_model('32x0e+32x1o', 3, 3)
    for p in m.products:
        d = SCSpec(p.symmetric_contractions).descriptor()
        _lib.check(_lib.lib().mmk_sc_compile_check(ctypes.byref(d)))


def test_csr_workspace_size():
    from mace_mps_kernels_b200 import _lib
    assert _lib.lib().mmk_csr_workspace_bytes(100, 1000) >= 4 * 1100


def test_patch_model_host_checks():
    """Device / dtype checks and the support predicate work without a GPU."""
    from mace_mps_kernels_b200 import patch_model
    from mace_mps_kernels_b200.conv import conv_supported
    m = helpers.make_model('32x0e+32x1o', 3, 3)
    with pytest.raises(RuntimeError, match='cuda'):
        patch_model(m)
    ok, why = conv_supported(helpers.make_model('48x0e+48x1o', 3, 3).interactions[1].conv_tp)
    assert not ok and 'multiple of 32' in why
    assert conv_supported(m.interactions[1].conv_tp) == (True, '')
    assert conv_supported(object())[0] is False


def test_extension_entry_points_validate_arguments():
    """The edge-geometry and block-linear entry points reject bad arguments before any launch (no GPU needed)."""
    from mace_mps_kernels_b200 import _lib
    L = _lib.lib()
    dummy = ctypes.c_void_p(16)                      # never dereferenced: every call below fails validation first
    assert L.mmk_sh_fwd(dummy, 10, 4, dummy, None) == _lib.MMK_ERR_UNSUPPORTED            # l_max > 3
    assert L.mmk_sh_fwd(dummy, 0, 3, dummy, None) == _lib.MMK_OK                         # no edges: nothing to do
    assert L.mmk_sh_bwd(None, None, 5, 2, None, None) == _lib.MMK_ERR_INVALID              # null tensors
    w = (ctypes.c_float * 8)(*range(8))
    d = _lib.RadialDesc(0, w, 1.0, 5.0, 5.0)
    assert L.mmk_radial_fwd(ctypes.byref(d), dummy, 10, dummy, None) == _lib.MMK_ERR_UNSUPPORTED   # no Bessel fns
    d = _lib.RadialDesc(8, w, 1.0, -1.0, 5.0)
    assert L.mmk_radial_bwd(ctypes.byref(d), dummy, dummy, 10, dummy, None) == _lib.MMK_ERR_INVALID  # r_max <= 0
    args = [dummy, 4, dummy, 4, dummy, 1, dummy, dummy, 1, 4]
    # perm without erow
    assert L.mmk_block_linear(*args, dummy, None, 1, 10, None) == _lib.MMK_ERR_INVALID
    # element-indexed flag missing but several elements
    assert L.mmk_block_linear(*args, None, None, 3, 10, None) == _lib.MMK_ERR_INVALID
    # activation epilogue without a pre-activation buffer
    assert L.mmk_block_linear_act(*args, None, None, 1, 10, 1, None, 0, None, ctypes.c_float(1.0),
                                  None) == _lib.MMK_ERR_INVALID
    assert 'zout' in L.mmk_last_error().decode()
    # block dimension beyond the kernel's row tile
    args[8] = 65
    assert L.mmk_block_linear(*args, None, None, 1, 10, None) == _lib.MMK_ERR_INVALID


def test_mlp_and_neighbor_list_entry_points_validate_arguments():
    """The fused-MLP and neighbour-list entry points reject bad arguments before any launch (no GPU needed), and
    the neighbour-list workspace size follows the binning of the cell."""
    from mace_mps_kernels_b200 import _lib
    L = _lib.lib()
    dummy = ctypes.c_void_p(16)
    widths = lambda *w: (ctypes.c_int * len(w))(*w)
    f = ctypes.c_float(1.0)
    assert L.mmk_mlp_fwd(dummy, 10, 5, widths(8, 8, 8, 8, 8, 8), dummy, f, dummy, dummy, None) == _lib.MMK_ERR_UNSUPPORTED
    assert L.mmk_mlp_fwd(dummy, 10, 2, widths(8, 65, 8), dummy, f, dummy, dummy, None) == _lib.MMK_ERR_UNSUPPORTED
    assert '1..64' in L.mmk_last_error().decode()
    assert L.mmk_mlp_bwd(dummy, 10, 0, widths(8), dummy, dummy, f, dummy, None) == _lib.MMK_ERR_UNSUPPORTED
    assert L.mmk_mlp_bwd(None, 10, 1, widths(8, 8), dummy, dummy, f, dummy, None) == _lib.MMK_ERR_INVALID
    assert L.mmk_mlp_fwd(dummy, 0, 1, widths(8, 8), dummy, f, dummy, dummy, None) == _lib.MMK_OK   # no rows
    cell = (ctypes.c_double * 9)(10, 0, 0, 0, 11, 0, 0, 0, 12)
    pbc = (ctypes.c_int * 3)(1, 1, 1)
    n = L.mmk_nl_workspace_bytes(cell, pbc, 5.0, None, None, 100, 4000)
    # 2 x 2 x 2 bins: per atom 24 + 12 + 4 + 4 + 4 + 4 bytes, per edge 16, bins 4 + 4 per bin (+1), 256-byte aligned
    assert n >= 100 * 52 + 4000 * 16 + 8 * 8 and n < 100 * 52 + 4000 * 16 + 8 * 8 + 12 * 256
    assert L.mmk_nl_workspace_bytes(cell, pbc, 0.0, None, None, 100, 4000) == 0                  # cutoff <= 0
    flat = (ctypes.c_double * 9)(10, 0, 0, 0, 11, 0, 0, 0, 0)
    assert L.mmk_nl_workspace_bytes(flat, pbc, 5.0, None, None, 100, 4000) == 0                  # singular cell
    assert 'singular' in L.mmk_last_error().decode()
    assert L.mmk_neighbor_list(dummy, 100, cell, pbc, 5.0, None, None, 4000, dummy, dummy, dummy, dummy, 16,
                               None) == _lib.MMK_ERR_INVALID                                     # workspace too small
    assert L.mmk_neighbor_list(dummy, 100, cell, pbc, 5.0, None, None, 4000, None, dummy, dummy, dummy, n,
                               None) == _lib.MMK_ERR_INVALID                                     # no edge_index


def test_generated_sources_are_deterministic():
    """Same descriptor -> byte-identical generated source (the module cache and the NVRTC cubins depend on it)."""
    from mace_mps_kernels_b200 import conv, symmetric
    spec = conv.ConvSpec(helpers.conv_tp('32x0e+32x1o', 3))
    assert conv.source(spec) == conv.source(conv.ConvSpec(helpers.conv_tp('32x0e+32x1o', 3)))
    m = helpers.make_model('32x0e+32x1o', 3, 3)
    sc = m.products[1].symmetric_contractions
    assert symmetric.source(symmetric.SCSpec(sc)) == symmetric.source(symmetric.SCSpec(sc))
    assert 'sc_fwd_body' in symmetric.source(symmetric.SCSpec(sc))
    assert 'fwd_edge' in conv.source(spec) and 'bwd_edge' in conv.source(spec)


def test_gemm_entry_points_validate_arguments():
    """Argument errors are reported before anything is launched (no GPU needed)."""
    from mace_mps_kernels_b200 import _lib
    L = _lib.lib()
    p = ctypes.c_void_p(16)                                    # never dereferenced: validation fails first
    assert L.mmk_gemm_tf32x3(p, 64, p, p, 64, p, 64, -1, 8, 64, None, 0, None) == _lib.MMK_ERR_INVALID
    assert L.mmk_gemm_tf32x3(p, 64, p, p, 64, p, 64, 10, 8, 62, None, 0, None) == _lib.MMK_ERR_INVALID   # K % 4
    assert L.mmk_gemm_tf32x3(p, 32, p, p, 64, p, 64, 10, 8, 64, None, 0, None) == _lib.MMK_ERR_INVALID   # lda < K
    assert L.mmk_gemm_tf32x3(ctypes.c_void_p(20), 64, p, p, 64, p, 64, 10, 8, 64, None, 0, None) == _lib.MMK_ERR_INVALID
    assert L.mmk_gemm_tf32x3(None, 64, p, p, 64, p, 64, 10, 8, 64, None, 0, None) == _lib.MMK_ERR_INVALID
    assert L.mmk_gemm_tf32x3(p, 64, p, p, 64, p, 64, 0, 8, 64, None, 0, None) == _lib.MMK_OK              # empty
    assert L.mmk_gemm_workspace_bytes(5218, 64, 1280) > 0 and L.mmk_gemm_workspace_bytes(5218, 1280, 64) == 0
    # K splits stay within one wave of CTAs (148 SMs without a GPU, one CTA per SM): 41 row tiles x 3 splits, not 4;
    # the workspace is the 1 KB counter block plus the partial tiles (128 x 64 floats each)
    assert L.mmk_gemm_workspace_bytes(5218, 64, 1280) == 1024 + 3 * 41 * 128 * 64 * 4
    assert L.mmk_gemm_workspace_bytes(5218, 64, 512) == 1024 + 3 * 41 * 128 * 64 * 4
    assert L.mmk_gemm_workspace_bytes(200 * 128, 64, 1280) == 0        # more tiles than SMs: no split
    assert L.mmk_tf32_split(p, p, p, -1, None) == _lib.MMK_ERR_INVALID


def test_host_tf32_split():
    import numpy as np
    import torch
    from mace_mps_kernels_b200.gemm import tf32_split_host
    x = torch.randn(10000, dtype=torch.float32) * torch.logspace(-10, 10, 10000)
    hi, lo = tf32_split_host(x)
    assert (hi.numpy().view(np.uint32) & 0x1FFF == 0).all() and (lo.numpy().view(np.uint32) & 0x1FFF == 0).all()
    r = (x.double() - hi.double() - lo.double()).abs() / x.double().abs()
    assert float(r.max()) < 2 ** -21
    assert float(((hi.double() - x.double()).abs() / x.double().abs()).max()) <= 2 ** -11
