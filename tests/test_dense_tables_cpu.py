"""Path tables of the block-linear layers (dense.py), evaluated with numpy exactly as the CUDA kernel reads them, against
the model's own equivariant linear / skip-connection modules and their input gradients (CPU, no GPU needed)."""
import numpy as np
import torch

from mace_mps_kernels_b200.dense import CudaLinear, CudaSkipTP
from mace_mps_kernels_b200.standin import o3


def _apply(t, x, elem=None):
    """out = what mmk_block_linear computes from the tables t (blocks, paths, packed weights)."""
    blocks, paths, w = t.blocks.numpy(), t.paths.numpy(), t.w.numpy()
    N = x.shape[0]
    e = np.zeros(N, int) if elem is None else elem
    dim = max(b[0] + b[1] * b[2] for b in blocks)
    out = np.full((N, dim), np.nan)
    for dst_off, mul_out, d, p0, n_p in blocks:
        acc = np.zeros((N, mul_out, d))
        for src_off, mul_in, w_off in paths[p0:p0 + n_p]:
            W = w[w_off:w_off + (e.max() + 1) * mul_in * mul_out].reshape(-1, mul_in, mul_out)[e]   # [N, u, v]
            xb = x[:, src_off:src_off + mul_in * d].reshape(N, mul_in, d)
            acc += np.einsum('nud,nuv->nvd', xb, W)
        out[:, dst_off:dst_off + mul_out * d] = acc.reshape(N, -1)
    return out


def _frozen(m):
    for p in m.parameters():
        p.requires_grad_(False)
    return m


def test_linear_tables_match_module():
    torch.manual_seed(0)
    lin = _frozen(o3.Linear(o3.Irreps('8x0e+4x1o+8x0e+3x2e+2x1o'), o3.Irreps('5x0e+6x1o+2x2e+3x3o')))
    op = CudaLinear(lin)
    x = torch.randn(7, lin.irreps_in.dim, dtype=torch.float32)
    ref = lin(x).numpy()
    out = _apply(op.fwd, x.numpy())
    assert np.abs(out - ref).max() < 1e-5 * np.abs(ref).max()          # 3x3o has no source: zeros
    xr = x.clone().requires_grad_(True)
    g = torch.randn(7, lin.irreps_out.dim)
    (gx,) = torch.autograd.grad(lin(xr), xr, g)
    gout = _apply(op.bwd, g.numpy())
    assert np.abs(gout - gx.numpy()).max() < 1e-5 * np.abs(gx.numpy()).max()


def test_skip_tables_match_module():
    torch.manual_seed(1)
    n_elem = 4
    tp = _frozen(o3.FullyConnectedTensorProduct(o3.Irreps('16x0e+8x1o'), o3.Irreps(f'{n_elem}x0e'),
                                                o3.Irreps('16x0e+8x1o+4x2e')))
    op = CudaSkipTP(tp)
    N = 9
    x1 = torch.randn(N, tp.irreps_in1.dim)
    elem = np.arange(N) % n_elem
    attrs = torch.nn.functional.one_hot(torch.from_numpy(elem), n_elem).float()
    ref = tp(x1, attrs).numpy()
    out = _apply(op.fwd, x1.numpy(), elem)
    assert np.abs(out - ref).max() < 1e-5 * np.abs(ref).max()
    xr = x1.clone().requires_grad_(True)
    g = torch.randn(N, tp.irreps_out.dim)
    (gx,) = torch.autograd.grad(tp(xr, attrs), xr, g)
    gout = _apply(op.bwd, g.numpy(), elem)
    assert np.abs(gout - gx.numpy()).max() < 1e-5 * np.abs(gx.numpy()).max()


def test_mlp_tables_match_module():
    from mace_mps_kernels_b200.dense import CudaFullyConnectedNet
    from mace_mps_kernels_b200.standin.modules import FullyConnectedNet
    torch.manual_seed(2)
    mlp = _frozen(FullyConnectedNet([8, 64, 64, 64, 320]))
    op = CudaFullyConnectedNet(mlp)
    x = torch.randn(11, 8)
    c = op.scale
    silu = lambda z: z / (1 + np.exp(-z))
    dsilu = lambda z: (1 / (1 + np.exp(-z))) * (1 + z * (1 - 1 / (1 + np.exp(-z))))
    h, zs = x.double().numpy(), []
    for t in op.fwd:                                  # hidden layers (kernel), then the last layer (GEMM)
        z = _apply(t, h)
        zs.append(z)
        h = c * silu(z)
    h = h @ op.w_last.double().numpy()
    x64 = x.double().requires_grad_(True)
    ref = copy_double(mlp)(x64)
    assert np.abs(h - ref.detach().numpy()).max() < 1e-5 * np.abs(ref.detach().numpy()).max()
    g = torch.randn(11, 320, dtype=torch.float64)
    (gx,) = torch.autograd.grad(ref, x64, g)
    gg = g.numpy() @ op.w_last.double().numpy().T
    for i in range(len(op.bwd) - 1, -1, -1):
        gg = _apply(op.bwd[i], gg * c * dsilu(zs[i]))
    assert np.abs(gg - gx.numpy()).max() < 1e-5 * np.abs(gx.numpy()).max()


def copy_double(m):
    import copy
    return copy.deepcopy(m).double()


def test_mlp_packed_hidden_weights():
    """The packed buffer mmk_mlp_fwd / mmk_mlp_bwd read (W_1 .. W_L row-major, one after the other), evaluated as the
    kernels evaluate it, against the module, forward and input gradient."""
    from mace_mps_kernels_b200.dense import CudaFullyConnectedNet
    from mace_mps_kernels_b200.standin.modules import FullyConnectedNet
    torch.manual_seed(5)
    mlp = _frozen(FullyConnectedNet([5, 30, 7, 96]))
    op = CudaFullyConnectedNet(mlp)
    assert op.fused and op.hidden_widths == (5, 30, 7)
    w = op.w_hidden.double().numpy()
    widths, c = op.hidden_widths, op.scale
    silu = lambda z: z / (1 + np.exp(-z))
    dsilu = lambda z: (1 / (1 + np.exp(-z))) * (1 + z * (1 - 1 / (1 + np.exp(-z))))
    x = torch.randn(13, 5, dtype=torch.float64)
    h, zs, off, Ws = x.numpy(), [], 0, []
    for win, wout in zip(widths[:-1], widths[1:]):
        W = w[off:off + win * wout].reshape(win, wout)
        off += win * wout
        Ws.append(W)
        z = h @ W
        zs.append(z)
        h = c * silu(z)
    assert off == w.size
    wt, off = op.w_hidden_t.double().numpy(), 0                  # mmk_mlp_bwd's operand: W_l^T, packed alike
    for W in Ws:
        assert np.array_equal(wt[off:off + W.size].reshape(W.shape[1], W.shape[0]), W.T)
        off += W.size
    out = h @ op.w_last.double().numpy()
    x64 = x.clone().requires_grad_(True)
    ref = copy_double(mlp)(x64)
    assert np.abs(out - ref.detach().numpy()).max() < 1e-5 * np.abs(ref.detach().numpy()).max()
    g = torch.randn(13, 96, dtype=torch.float64)
    (gx,) = torch.autograd.grad(ref, x64, g)
    gg = g.numpy() @ op.w_last.double().numpy().T
    for W, z in zip(reversed(Ws), reversed(zs)):
        gg = (gg * c * dsilu(z)) @ W.T
    assert np.abs(gg - gx.numpy()).max() < 1e-5 * np.abs(gx.numpy()).max()


def test_reshape_irreps_column_tables_match_the_module():
    """CudaReshapeIrreps' gather tables applied on the host equal MACE's reshape_irreps, and the backward table is
    the inverse permutation."""
    import torch
    from mace_mps_kernels_b200.dense import CudaReshapeIrreps, reshape_supported
    from mace_mps_kernels_b200.standin import o3
    from mace_mps_kernels_b200.standin.modules import reshape_irreps
    for irreps in ('16x0e', '8x0e+8x1o+8x2e+8x3o', '4x1o+4x0e+4x2e'):
        m = reshape_irreps(o3.Irreps(irreps))
        assert reshape_supported(m) == (True, '')
        op = CudaReshapeIrreps(m)
        x = torch.randn(7, m.irreps.dim)
        got = x[:, op.fwd_cols.long()].reshape(7, *op.shape)
        assert torch.equal(got, m(x))
        assert torch.equal(got.reshape(7, -1)[:, op.bwd_cols.long()], x)
    assert not reshape_supported(reshape_irreps(o3.Irreps('8x0e+4x1o')))[0]
