"""Failure path of the pipelined kernels on a GPU, without a fault: a wait that runs out ends in a status, not a hang.

Every mbarrier wait in the conv and symmetric-contraction kernels is bounded; when one gives up, the kernel records a
code in its module's status word and returns.  These tests build the layers in the test configuration
(``MMK_TEST_STALL=1``: the producer warps issue no copy at all, so nothing is in flight; ``MMK_WAIT_CYCLES``: a short
budget of about ten milliseconds) and check that the launch completes, the layer status is nonzero, resetting it
clears it, and that a normally built layer still runs correctly afterwards in the same context.
"""
import numpy as np
import pytest
import torch

from oracle import conv_ref, sc_ref

pytestmark = pytest.mark.gpu

STALL_ENV = {'MMK_TEST_STALL': '1', 'MMK_WAIT_CYCLES': '20000000'}     # ~10 ms at 1.9 GHz


def _graph(N, E, seed=0):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(np.stack([rng.integers(0, N, E), rng.integers(0, N, E)]))


def _conv_layer(monkeypatch, stalled):
    from mace_mps_kernels_b200 import standin
    from mace_mps_kernels_b200.conv import CudaConvTP
    m = standin.make_model('32x0e+32x1o', 3, 3, seed=0)
    for k, v in STALL_ENV.items():
        if stalled:
            monkeypatch.setenv(k, v)
        else:
            monkeypatch.delenv(k, raising=False)
    tp = m.interactions[1].conv_tp
    return tp, CudaConvTP(tp)


def test_conv_wait_timeout_sets_status_and_returns(cuda, monkeypatch):
    tp, op = _conv_layer(monkeypatch, stalled=True)
    N, E = 40, 600
    ei = _graph(N, E).to(cuda)
    x = torch.randn(N, op.spec.x_dim, device=cuda, requires_grad=True)
    Y = torch.randn(E, op.spec.y_dim, device=cuda, requires_grad=True)
    W = torch.randn(E, op.spec.w_dim, device=cuda, requires_grad=True)
    out = op(x, Y, W, ei)
    torch.cuda.synchronize()                       # the launch completes although no copy ever lands
    # 2: a forward consumer's ring wait ran out (9: a consumer group's hand-over wait, 10 / 11: the edge-balanced
    # split's waits for the pieces of a straddling node, if one of those gave up last)
    st = op.status()
    assert st in (2, 9, 10, 11), f'forward timeout status expected, got {st}'
    assert op.status(reset=True) == st
    assert op.status() == 0
    torch.autograd.grad(out, (x, Y, W), torch.ones_like(out))
    torch.cuda.synchronize()
    st = op.status(reset=True)
    assert st in (4, 9, 10, 11), f'backward timeout status expected, got {st}'

    # the context is still usable: a normally built layer gives the oracle's result
    tp, good = _conv_layer(monkeypatch, stalled=False)
    spec, coef = conv_ref.probe_coefficients(tp)
    with torch.no_grad():
        o = good(x, Y, W, ei)
    ref = conv_ref.conv_fwd(spec, coef, x.detach().cpu(), Y.detach().cpu(), W.detach().cpu(), ei[0].cpu().numpy(),
                            ei[1].cpu().numpy(), N)
    err = np.abs(o.double().cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 2e-5
    assert good.status() == 0


def test_sc_wait_timeout_sets_status_and_returns(cuda, monkeypatch):
    from mace_mps_kernels_b200 import standin
    from mace_mps_kernels_b200.symmetric import CudaSymmetricContraction
    sc = standin.make_model('32x0e+32x1o', 3, 3, seed=0).products[0].symmetric_contractions
    for k, v in STALL_ENV.items():
        monkeypatch.setenv(k, v)
    op = CudaSymmetricContraction(sc, device=cuda)
    N = 300
    rng = np.random.default_rng(1)
    elem = torch.from_numpy(rng.integers(0, 4, N))
    attrs = torch.nn.functional.one_hot(elem, 4).float().to(cuda)
    x = torch.randn(N, 32, 16, device=cuda, requires_grad=True)
    out = op(x, attrs)
    torch.cuda.synchronize()
    assert op.status(reset=True) == 6, 'symmetric-contraction consumer timeout expected (status 6)'
    torch.autograd.grad(out, (x,), torch.ones_like(out))
    torch.cuda.synchronize()
    assert op.status(reset=True) == 6
    for k in STALL_ENV:
        monkeypatch.delenv(k, raising=False)
    good = CudaSymmetricContraction(sc, device=cuda)
    spec = sc_ref.sc_spec(sc)
    with torch.no_grad():
        o = good(x, attrs)
    ref = sc_ref.sc_fwd(spec, x.detach().cpu(), elem.numpy())
    assert np.abs(o.double().cpu().numpy() - ref).max() / np.abs(ref).max() < 2e-5
    assert good.status() == 0
