"""ctypes binding of the C ABI (include/mmk.h) in ``_lib/libmmk.so``.

There is no fallback: if the library is missing, importing the patched ops raises, and every entry point's nonzero
status becomes an exception carrying ``mmk_last_error()``.
"""
from __future__ import annotations

import collections
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, '_lib', 'libmmk.so')

MMK_OK, MMK_ERR_INVALID, MMK_ERR_COMPILE, MMK_ERR_CUDA, MMK_ERR_UNSUPPORTED = 0, 1, 2, 3, 4

_i, _i64, _p, _sz, _d = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_double
_ip = ctypes.POINTER(ctypes.c_int)
_dp = ctypes.POINTER(ctypes.c_double)


class ConvDesc(ctypes.Structure):
    _fields_ = [('mul', _i), ('n_in1', _i), ('in1_l', _ip), ('n_in2', _i), ('in2_l', _ip), ('n_out', _i),
                ('out_l', _ip), ('nins', _i), ('ins_i1', _ip), ('ins_i2', _ip), ('ins_io', _ip), ('nterms', _i),
                ('term_ins', _ip), ('term_a', _ip), ('term_b', _ip), ('term_m', _ip), ('term_c', _dp)]


class RadialDesc(ctypes.Structure):
    _fields_ = [('n_bessel', _i), ('w', ctypes.POINTER(ctypes.c_float)), ('prefactor', ctypes.c_float),
                ('r_max', ctypes.c_float), ('p', ctypes.c_float)]


class SCDesc(ctypes.Structure):
    _fields_ = [('C', _i), ('n_ell', _i), ('n_rows', _i), ('n_blocks', _i), ('block_M', _ip), ('block_nterms', _ip),
                ('max_degree', _i), ('term_degree', _ip), ('term_idx', _ip), ('term_row', _ip)]


# name -> (restype, argtypes); kept in the same order as include/mmk.h
SIGNATURES = {
    'mmk_last_error': (ctypes.c_char_p, []),
    'mmk_version': (ctypes.c_char_p, []),
    'mmk_conv_layer_create': (_i, [ctypes.POINTER(ConvDesc), ctypes.POINTER(_p)]),
    'mmk_conv_layer_destroy': (_i, [_p]),
    'mmk_conv_layer_dims': (_i, [_p, _ip, _ip, _ip, _ip]),
    'mmk_conv_compile_check': (_i, [ctypes.POINTER(ConvDesc)]),
    'mmk_conv_source': (_i, [ctypes.POINTER(ConvDesc), ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    'mmk_conv_layer_status': (_i, [_p, _ip, _i]),
    'mmk_conv_fwd': (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p]),
    'mmk_conv_bwd': (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p]),
    'mmk_csr_workspace_bytes': (_sz, [_i64, _i64]),
    'mmk_csr_build': (_i, [_p, _i64, _i64, _p, _p, _p, _sz, _p, _p]),
    'mmk_csr_pair_workspace_bytes': (_sz, [_i64, _i64]),
    'mmk_csr_build_pair': (_i, [_p, _i64, _i64, _p, _p, _p, _sz, _p, _p]),
    'mmk_csr_build_noalloc': (_i, [_p, _i64, _i64, _p, _p, _p, _p]),
    'mmk_sc_layer_create': (_i, [ctypes.POINTER(SCDesc), ctypes.POINTER(_p)]),
    'mmk_sc_layer_destroy': (_i, [_p]),
    'mmk_sc_layer_dims': (_i, [_p, _ip, _ip, _ip, _ip]),
    'mmk_sc_compile_check': (_i, [ctypes.POINTER(SCDesc)]),
    'mmk_sh_fwd': (_i, [_p, _i64, _i, _p, _p]),
    'mmk_sh_bwd': (_i, [_p, _p, _i64, _i, _p, _p]),
    'mmk_radial_fwd': (_i, [ctypes.POINTER(RadialDesc), _p, _i64, _p, _p]),
    'mmk_radial_bwd': (_i, [ctypes.POINTER(RadialDesc), _p, _p, _i64, _p, _p]),
    'mmk_edge_vectors_fwd': (_i, [_p, _p, _p, _i64, _p, _p, _p]),
    'mmk_edge_vectors_bwd': (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p]),
    'mmk_gather_columns': (_i, [_p, _i64, _p, _i64, _p, _i64, _i, _p]),
    'mmk_block_linear': (_i, [_p, _i64, _p, _i64, _p, _i, _p, _p, _i, _i, _p, _p, _i, _i64, _p]),
    'mmk_block_linear_act': (_i, [_p, _i64, _p, _i64, _p, _i, _p, _p, _i, _i, _p, _p, _i, _i64, _i, _p, _i, _p,
                                  ctypes.c_float, _p]),
    'mmk_nl_workspace_bytes': (_sz, [_dp, _ip, _d, _dp, _dp, _i64, _i64]),
    'mmk_neighbor_list': (_i, [_p, _i64, _dp, _ip, _d, _dp, _dp, _i64, _p, _p, _p, _p, _sz, _p]),
    'mmk_mlp_fwd': (_i, [_p, _i64, _i, _ip, _p, ctypes.c_float, _p, _p, _p]),
    'mmk_mlp_bwd': (_i, [_p, _i64, _i, _ip, _p, _p, ctypes.c_float, _p, _p]),
    'mmk_sc_source': (_i, [ctypes.POINTER(SCDesc), ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    'mmk_sc_layer_status': (_i, [_p, _ip, _i]),
    'mmk_elem_index': (_i, [_p, _i64, _i, _p, _p]),
    'mmk_elem_groups': (_i, [_p, _i64, _i, _p, _p, _p, _sz, _p]),
    'mmk_sc_fwd': (_i, [_p, _p, _p, _p, _i, _p, _p, _i64, _p]),
    'mmk_sc_bwd': (_i, [_p, _p, _p, _p, _i, _p, _p, _p, _i64, _p]),
    'mmk_tf32_split': (_i, [_p, _p, _p, _i64, _p]),
    'mmk_gemm_workspace_bytes': (_sz, [_i64, _i64, _i64]),
    'mmk_gemm_tf32x3': (_i, [_p, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _p, _sz, _p]),
    'mmk_gemm_status': (_i, [_ip, _i]),
}

_lib = None


class MMKError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f'mace-b200-kernels: {msg} (status {code})')
        self.code = code


def lib():
    """The loaded library (raises if it has not been built: there is deliberately no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f'{LIB_PATH} is missing; build it with `python -m mace_mps_kernels_b200.csrc.build` '
                              '(or __graft_entry__.build())')
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def check(code):
    if code != MMK_OK:
        raise MMKError(code, lib().mmk_last_error().decode(errors='replace'))


# kernels each entry point launches (bench.py reports the count issued inside its timed region)
KERNELS_PER_CALL = {'mmk_conv_fwd': 1, 'mmk_conv_bwd': 1, 'mmk_sc_fwd': 1, 'mmk_sc_bwd': 1, 'mmk_csr_build': 4,
                    'mmk_csr_build_noalloc': 4, 'mmk_csr_build_pair': 4, 'mmk_elem_index': 1, 'mmk_elem_groups': 3,
                    'mmk_sh_fwd': 1, 'mmk_sh_bwd': 1, 'mmk_radial_fwd': 1, 'mmk_radial_bwd': 1,
                    'mmk_block_linear': 1, 'mmk_block_linear_act': 1, 'mmk_mlp_fwd': 1, 'mmk_mlp_bwd': 1,
                    'mmk_neighbor_list': 10, 'mmk_tf32_split': 1, 'mmk_gemm_tf32x3': 1,
                    'mmk_edge_vectors_fwd': 1, 'mmk_edge_vectors_bwd': 1, 'mmk_gather_columns': 1}
LAUNCHES = collections.Counter()


def call(name, *args):
    check(getattr(lib(), name)(*args))
    k = KERNELS_PER_CALL.get(name)
    if k:
        LAUNCHES[name] += k


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def aligned(t, nbytes=16):
    """``t`` if its data starts on an ``nbytes`` boundary (the TMA copies need 16), else a contiguous copy."""
    return t if t.data_ptr() % nbytes == 0 else t.clone(memory_format=torch.contiguous_format)


def int_array(vals):
    vals = list(vals)
    return (ctypes.c_int * max(1, len(vals)))(*vals)


def double_array(vals):
    vals = list(vals)
    return (ctypes.c_double * max(1, len(vals)))(*vals)


def generated_source(fn_name, desc):
    """The generated layer header for a descriptor (``mmk_conv_source`` / ``mmk_sc_source``)."""
    n = ctypes.c_size_t(0)
    check(getattr(lib(), fn_name)(ctypes.byref(desc), None, 0, ctypes.byref(n)))
    buf = ctypes.create_string_buffer(n.value + 1)
    check(getattr(lib(), fn_name)(ctypes.byref(desc), buf, n.value + 1, ctypes.byref(n)))
    return buf.value.decode()
