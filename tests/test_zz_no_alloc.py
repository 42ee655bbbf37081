"""GPU: the allocation-free CSR entry point (mmk_csr_build_noalloc) gives exactly what mmk_csr_build gives.

Some callers of this library cannot allocate device memory -- e.g. an MD engine or plugin host that owns all device
memory through its own pool and passes the library only inputs and outputs -- so they cannot supply the workspace
mmk_csr_build takes.  mmk_csr_build_noalloc keeps its scratch in a fixed-size array inside the library instead.
This file is collected last so that a run stopping at the first failure has already run every other test; it also
passes on its own in a fresh process (the first call on the device does the one-time address lookup).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _csr_alloc(idx, N, cuda):
    from mace_mps_kernels_b200 import _lib
    E = idx.numel()
    rowptr = torch.full((N + 1,), -7, dtype=torch.int32, device=cuda)
    eids = torch.full((E,), -7, dtype=torch.int32, device=cuda)
    nb = _lib.lib().mmk_csr_workspace_bytes(N, E)
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=cuda)
    _lib.call('mmk_csr_build', _lib.ptr(idx), E, N, _lib.ptr(rowptr), _lib.ptr(eids), _lib.ptr(ws), nb, None,
              _lib.stream_of(idx))
    return rowptr, eids


def _csr_noalloc(idx, N, cuda):
    from mace_mps_kernels_b200 import _lib
    E = idx.numel()
    rowptr = torch.full((N + 1,), -7, dtype=torch.int32, device=cuda)
    eids = torch.full((E,), -7, dtype=torch.int32, device=cuda)
    _lib.call('mmk_csr_build_noalloc', _lib.ptr(idx), E, N, _lib.ptr(rowptr), _lib.ptr(eids), None,
              _lib.stream_of(idx))
    return rowptr, eids


def test_noalloc_csr_matches_allocating_entry_point(cuda):
    rng = np.random.default_rng(7)
    # two calls in a row on different graphs: the second must not see the first one's scratch contents
    for N, E in ((5000, 200000), (777, 31000)):
        idx = torch.from_numpy(rng.integers(0, N, E)).to(cuda)
        r0, e0 = _csr_alloc(idx, N, cuda)
        r1, e1 = _csr_noalloc(idx, N, cuda)
        torch.cuda.synchronize()
        assert torch.equal(r0, r1)
        assert torch.equal(e0, e1)


def test_noalloc_csr_rejects_sizes_above_its_limit(cuda):
    from mace_mps_kernels_b200 import _lib
    L = _lib.lib()
    idx = torch.zeros(4, dtype=torch.int64, device=cuda)
    rowptr = torch.zeros(4, dtype=torch.int32, device=cuda)
    eids = torch.zeros(4, dtype=torch.int32, device=cuda)
    too_many_edges = (1 << 22) + 1
    rc = L.mmk_csr_build_noalloc(_lib.ptr(idx), too_many_edges, 3, _lib.ptr(rowptr), _lib.ptr(eids), None,
                                 _lib.stream_of(idx))
    assert rc == _lib.MMK_ERR_INVALID
    assert 'MMK_NOALLOC_MAX_EDGES' in L.mmk_last_error().decode()
    rc = L.mmk_csr_build_noalloc(_lib.ptr(idx), 4, (1 << 18) + 1, _lib.ptr(rowptr), _lib.ptr(eids), None,
                                 _lib.stream_of(idx))
    assert rc == _lib.MMK_ERR_INVALID
    assert 'MMK_NOALLOC_MAX_NODES' in L.mmk_last_error().decode()
