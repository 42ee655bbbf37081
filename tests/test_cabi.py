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
