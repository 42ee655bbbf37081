"""Per-op parity of the CUDA kernels (through the C ABI) against the float64 CPU oracle.

Tolerance: fp32 kernels vs fp64 oracle, max |gpu - oracle| <= REL * max |oracle| (+ a tiny absolute floor for
all-zero outputs); the CSR builder is checked bit-exactly against a stable argsort.
"""

import numpy as np
import pytest
import torch

import helpers
from oracle import conv_ref, sc_ref

pytestmark = pytest.mark.gpu

REL = 2e-5


def close(gpu, ref, rel=REL, what=''):
    gpu = gpu.detach().double().cpu().numpy() if torch.is_tensor(gpu) else np.asarray(gpu)
    ref = np.asarray(ref)
    assert gpu.shape == ref.shape, (what, gpu.shape, ref.shape)
    scale = max(np.abs(ref).max(initial=0.0), 1e-30)
    err = np.abs(gpu - ref).max(initial=0.0)
    assert err <= rel * scale + 1e-30, f'{what}: max err {err:.3e} vs scale {scale:.3e} (rel {err / scale:.2e})'
    return err / scale


CONV_CASES = [
    # hidden irreps of the node features, lmax, N, E
    ('32x0e', 3, 37, 300),
    ('32x0e+32x1o', 3, 50, 700),
    ('64x0e+64x1o', 2, 41, 333),
    ('128x0e+128x1o', 3, 160, 5000),
    ('128x0e+128x1o+128x2e', 3, 90, 2000),
    ('96x0e+96x1o', 3, 3, 17),
    ('64x0e+64x1o', 3, 3000, 90000),
    ('32x0e+32x1o', 3, 5, 900),
    # many nodes per CTA with small rings and two consumer groups (node boundaries inside a CTA's edge stream)
    ('128x0e+128x1o+128x2e', 3, 1500, 24000),
    ('128x0e', 3, 4000, 120000),
]


@pytest.mark.parametrize('hidden,lmax,N,E', CONV_CASES)
def test_conv_fwd_bwd_matches_oracle(cuda, hidden, lmax, N, E):
    _conv_case(cuda, hidden, lmax, N, E)


# Alternative launch plans (the layer-creation overrides used for tuning): channels per consumer thread, group
# counts, ring sizes and the per-term backward body.
PLAN_VARIANTS = [
    {'MMK_CONV_EDGE_SPLIT': '0'},              # node ranges per CTA on small graphs (no pieces)
    {'MMK_CONV_EDGE_SPLIT': '1'},              # edge-balanced ranges in both directions (default: backward only)
    {'MMK_CONV_FWD_TC': '1'},                  # forward on the tensor cores (layers with 128 channels)
    {'MMK_CONV_FWD_CPT': '2', 'MMK_CONV_BWD_CPT': '2'},
    {'MMK_CONV_FWD_CPT': '4', 'MMK_CONV_BWD_CPT': '4', 'MMK_CONV_FWD_CG': '8', 'MMK_CONV_BWD_CG': '8'},
    {'MMK_CONV_FWD_CPT': '2', 'MMK_CONV_BWD_CPT': '2', 'MMK_CONV_FWD_CG': '8', 'MMK_CONV_BWD_CG': '8'},
    {'MMK_CONV_BWD_FORM': '0', 'MMK_CONV_SMEM_KB': '200', 'MMK_CONV_FWD_CG': '1', 'MMK_CONV_BWD_CG': '1'},
    {'MMK_CONV_FWD_NP': '2', 'MMK_CONV_BWD_NP': '2'},
    {'MMK_CONV_FWD_NP': '4', 'MMK_CONV_BWD_NP': '4', 'MMK_CONV_BWD_CG': '1', 'MMK_CONV_BWD_MINB': '1'},
    {'MMK_CONV_FWD_NP': '2', 'MMK_CONV_BWD_NP': '2', 'MMK_CONV_FWD_CPT': '2', 'MMK_CONV_BWD_CPT': '2',
     'MMK_CONV_FWD_MINB': '2'},
    {'MMK_CONV_FWD_NB': '3', 'MMK_CONV_BWD_NB': '5'},
]


@pytest.mark.parametrize('env', PLAN_VARIANTS, ids=lambda e: ','.join(f'{k[9:]}={v}' for k, v in e.items()))
@pytest.mark.parametrize('hidden,N,E', [('128x0e', 1500, 30000), ('128x0e+128x1o', 300, 6000),
                                         ('128x0e+128x1o+128x2e', 120, 2500)])
def test_conv_plan_variants_match_oracle(cuda, monkeypatch, env, hidden, N, E):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    _conv_case(cuda, hidden, 3, N, E)


def _conv_case(cuda, hidden, lmax, N, E):
    from mace_mps_kernels_b200.conv import CudaConvTP
    torch.manual_seed(0)
    tp = helpers.conv_tp(hidden, lmax).to(cuda)
    op = CudaConvTP(tp)
    spec, coef = conv_ref.probe_coefficients(tp)
    ei = helpers.random_graph(N, E, seed=N, isolated=[1] if N > 3 else ())
    x = torch.randn(N, spec['x_dim'], device=cuda)
    Y = torch.randn(E, spec['y_dim'], device=cuda)
    W = torch.randn(E, tp.weight_numel, device=cuda)
    x.requires_grad_(True); Y.requires_grad_(True); W.requires_grad_(True)
    out = op(x, Y, W, ei.to(cuda))
    send, recv = ei[0].numpy(), ei[1].numpy()
    ref = conv_ref.conv_fwd(spec, coef, x.detach().cpu(), Y.detach().cpu(), W.detach().cpu(), send, recv, N)
    close(out, ref, what='out')
    g = torch.randn_like(out)
    gx, gY, gW = torch.autograd.grad(out, (x, Y, W), g)
    rgx, rgY, rgW = conv_ref.conv_bwd(spec, coef, x.detach().cpu(), Y.detach().cpu(), W.detach().cpu(), g.cpu(),
                                      send, recv)
    close(gx, rgx, what='gx')
    close(gY, rgY, what='gY')
    close(gW, rgW, what='gW')
    assert op.status() == 0
    # the unpatched e3nn-style path on the GPU (fp32) agrees too
    with torch.no_grad():
        mji = tp(x.detach()[ei[0].to(cuda)], Y.detach(), W.detach())
        msg = torch.zeros_like(out).index_add_(0, ei[1].to(cuda), mji)
    close(out, msg.double().cpu().numpy(), rel=1e-4, what='vs torch path')


def test_conv_no_edges_and_isolated_nodes(cuda):
    from mace_mps_kernels_b200.conv import CudaConvTP
    tp = helpers.conv_tp('32x0e+32x1o', 3).to(cuda)
    op = CudaConvTP(tp)
    N = 5
    x = torch.randn(N, 128, device=cuda, requires_grad=True)
    Y = torch.randn(0, 16, device=cuda, requires_grad=True)
    W = torch.randn(0, tp.weight_numel, device=cuda, requires_grad=True)
    ei = torch.zeros(2, 0, dtype=torch.long, device=cuda)
    out = op(x, Y, W, ei)
    assert out.shape == (N, 32 * 40) and float(out.abs().max()) == 0.0
    gx, = torch.autograd.grad(out, (x,), torch.randn_like(out))
    assert float(gx.abs().max()) == 0.0


@pytest.mark.parametrize('N,E,seed', [(1, 0, 0), (7, 50, 1), (1000, 40000, 2), (300, 2, 3)])
def test_csr_matches_stable_argsort(cuda, N, E, seed):
    from mace_mps_kernels_b200.conv import csr_build
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, N, E) if seed != 2 else np.repeat(np.arange(N), E // N)[rng.permutation(E)]
    rowptr, eids = csr_build(torch.from_numpy(idx).to(cuda), N)
    r0, e0 = conv_ref.csr_by(idx, N)
    assert np.array_equal(rowptr.cpu().numpy(), r0)
    assert np.array_equal(eids.cpu().numpy(), e0)


@pytest.mark.parametrize('N,E,seed', [(1, 0, 0), (7, 50, 1), (1000, 40000, 2), (300, 2, 3), (5000, 150000, 4)])
def test_csr_pair_matches_stable_argsort_of_each_row(cuda, N, E, seed):
    """mmk_csr_build_pair (both CSRs of an edge_index in one launch sequence) equals the oracle's csr_by of the
    receiver row and of the sender row, bit for bit (including empty graphs, empty nodes and very long segments)."""
    from mace_mps_kernels_b200.conv import csr_build_pair
    rng = np.random.default_rng(seed)
    ei = rng.integers(0, N, (2, E))
    if seed == 2:
        ei[1] = np.repeat(np.arange(N), E // N)[rng.permutation(E)]
    if seed == 4:
        ei[0, : E // 30] = 0                                     # one sender with 5 000 edges
    rr, re, sr, se = csr_build_pair(torch.from_numpy(ei).to(cuda).contiguous(), N)
    for (rowptr, eids), row in (((rr, re), ei[1]), ((sr, se), ei[0])):
        r0, e0 = conv_ref.csr_by(row, N)
        assert np.array_equal(rowptr.cpu().numpy(), r0)
        assert np.array_equal(eids.cpu().numpy(), e0)


@pytest.mark.parametrize('N,n_elem,seed', [(5, 4, 0), (1000, 1, 1), (70000, 3, 2), (257, 89, 3)])
def test_elem_groups_match_stable_argsort(cuda, N, n_elem, seed):
    """Nodes grouped by element = a stable argsort of the element index (long segments: one element can hold every
    node)."""
    from mace_mps_kernels_b200.symmetric import element_groups
    rng = np.random.default_rng(seed)
    e = rng.integers(0, n_elem, N) if seed != 2 else np.where(rng.random(N) < 0.97, 0, rng.integers(0, n_elem, N))
    attrs = torch.nn.functional.one_hot(torch.from_numpy(e), n_elem).float().to(cuda)
    elem, erow, perm = element_groups(attrs)
    assert np.array_equal(elem.cpu().numpy(), e)
    assert np.array_equal(erow.cpu().numpy(), np.concatenate([[0], np.cumsum(np.bincount(e, minlength=n_elem))]))
    assert np.array_equal(perm.cpu().numpy(), np.argsort(e, kind='stable'))


def test_csr_flags_out_of_range(cuda):
    from mace_mps_kernels_b200 import _lib
    idx = torch.tensor([0, 5, 1, -1, 2], device=cuda)
    N = 3
    rowptr = torch.empty(N + 1, dtype=torch.int32, device=cuda)
    eids = torch.empty(5, dtype=torch.int32, device=cuda)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    nb = _lib.lib().mmk_csr_workspace_bytes(N, 5)
    ws = torch.empty(nb, dtype=torch.uint8, device=cuda)
    _lib.call('mmk_csr_build', _lib.ptr(idx), 5, N, _lib.ptr(rowptr), _lib.ptr(eids), _lib.ptr(ws), nb, _lib.ptr(flag),
              _lib.stream_of(idx))
    assert int(flag.item()) == 1
    assert rowptr.cpu().tolist() == [0, 1, 2, 3]
    assert eids[:3].cpu().tolist() == [0, 2, 4]


SC_CASES = [
    ('32x0e+32x1o', 3, 3, 40),
    ('128x0e+128x1o', 3, 3, 160),
    ('128x0e', 3, 3, 33),
    ('64x0e', 2, 2, 20),
    ('32x0e+32x1o+32x2e', 3, 3, 25),
    ('128x0e+128x1o', 3, 3, 1001),
    ('32x0e', 2, 3, 3),
    # few-node variant (term list split over four groups) with several tiles per CTA, and the many-node variant
    ('128x0e+128x1o+128x2e', 3, 3, 900),
    ('128x0e+128x1o', 3, 3, 3000),
]


@pytest.mark.parametrize('hidden,lmax,corr,N', SC_CASES)
def test_sc_fwd_bwd_matches_oracle(cuda, hidden, lmax, corr, N):
    from mace_mps_kernels_b200.standin import o3
    from mace_mps_kernels_b200.standin.symmetric_contraction import SymmetricContraction
    from mace_mps_kernels_b200.symmetric import CudaSymmetricContraction
    torch.manual_seed(1)
    hid = o3.Irreps(hidden)
    C = hid[0].mul
    sh = o3.Irreps.spherical_harmonics(lmax)
    n_elem = 4
    sc = SymmetricContraction((sh * C).sort()[0].simplify(), hid, corr, n_elem).to(cuda)
    op = CudaSymmetricContraction(sc, device=cuda)
    spec = sc_ref.sc_spec(sc)
    x = torch.randn(N, C, (lmax + 1) ** 2, device=cuda, requires_grad=True)
    elem = torch.randint(0, n_elem, (N,))
    attrs = torch.nn.functional.one_hot(elem, n_elem).float().to(cuda)
    out = op(x, attrs)
    ref = sc_ref.sc_fwd(spec, x.detach().cpu(), elem.numpy())
    close(out, ref, what='sc out')
    for _ in range(2):                  # repeated launches (ring stages reused many times per CTA) give the same bits
        assert torch.equal(op(x.detach(), attrs), out.detach())
    with torch.no_grad():
        close(out, sc(x.detach(), attrs).double().cpu().numpy(), rel=1e-4, what='sc vs torch path')
    g = torch.randn_like(out)
    gx, = torch.autograd.grad(out, (x,), g)
    close(gx, sc_ref.sc_bwd(spec, x.detach().cpu(), elem.numpy(), g.cpu()), what='sc gx')
    assert op.status() == 0


def test_double_backward_raises_on_ops(cuda):
    from mace_mps_kernels_b200.conv import CudaConvTP
    tp = helpers.conv_tp('32x0e+32x1o', 3).to(cuda)
    op = CudaConvTP(tp)
    ei = helpers.random_graph(6, 20).to(cuda)
    x = torch.randn(6, 128, device=cuda, requires_grad=True)
    Y = torch.randn(20, 16, device=cuda)
    W = torch.randn(20, tp.weight_numel, device=cuda)
    out = op(x, Y, W, ei)
    with pytest.raises(RuntimeError, match='double backward'):
        (g,) = torch.autograd.grad(out.square().sum(), x, create_graph=True)
        torch.autograd.grad(g.sum(), x)


@pytest.mark.parametrize('hidden,N,E', [('128x0e+128x1o', 5, 2000), ('128x0e+128x1o+128x2e', 168, 5218),
                                        ('128x0e', 40, 6000)])
def test_conv_edge_split_repeatable_and_equal_to_node_ranges(cuda, monkeypatch, hidden, N, E):
    """Small graphs run the edge-balanced split (pieces of straddling nodes summed in CTA order): launches repeat
    bit for bit (the per-CTA flags are back at zero after every launch), and the result equals the node-range split
    within float32 rounding."""
    from mace_mps_kernels_b200.conv import CudaConvTP
    torch.manual_seed(1)
    tp = helpers.conv_tp(hidden, 3).to(cuda)
    ei = helpers.random_graph(N, E, seed=7).to(cuda)
    x = torch.randn(N, tp.irreps_in1.dim, device=cuda, requires_grad=True)
    Y = torch.randn(E, tp.irreps_in2.dim, device=cuda, requires_grad=True)
    W = torch.randn(E, tp.weight_numel, device=cuda, requires_grad=True)

    def run(op):
        out = op(x, Y, W, ei)
        g = torch.ones_like(out)
        return (out.detach(),) + torch.autograd.grad(out, (x, Y, W), g)

    monkeypatch.setenv('MMK_CONV_EDGE_SPLIT', '1')
    op = CudaConvTP(tp)
    first = run(op)
    for _ in range(3):
        again = run(op)
        assert all(torch.equal(a, b) for a, b in zip(first, again))
    assert op.status() == 0
    monkeypatch.setenv('MMK_CONV_EDGE_SPLIT', '0')
    nodes = run(CudaConvTP(tp))
    for a, b, name in zip(first, nodes, ('out', 'gx', 'gY', 'gW')):
        close(a, b.double().cpu().numpy(), what=name)


@pytest.mark.parametrize('hidden,lmax,N,E', [c for c in CONV_CASES if c[0].startswith('128x')])
def test_conv_tensor_core_forward_matches_oracle(cuda, monkeypatch, hidden, lmax, N, E):
    """The tcgen05 forward (per-edge x . M_e with the 3xTF32 split, W weighting and receiver sums on the CUDA cores)
    against the float64 oracle, on every 128-channel case; the backward is the CUDA-core kernel."""
    monkeypatch.setenv('MMK_CONV_FWD_TC', '1')
    _conv_case(cuda, hidden, lmax, N, E)
