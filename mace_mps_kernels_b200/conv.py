"""Fused MACE interaction convolution on B200: gather -> channel-wise weighted uvu tensor product -> scatter-sum.

Drop-in for an interaction block's ``conv_tp`` under MACE's ``conv_fusion`` path, as in reference
``src/mace_mps_kernels/conv.py``: ``forward(node_feats, edge_attrs, tp_weights, edge_index) -> [N, OUT_DIM]`` summed
over receivers (unnormalised; MACE divides by avg_num_neighbors afterwards).

* ``conv_supported`` keeps the reference's support rules (reference conv.py:31-51).
* ``ConvSpec`` measures the effective coefficient of every path (CG x normalisation x path weight, as the
  TensorProduct applies it) by probing the TensorProduct with unit inputs on channel 0, keeping |c| > 1e-7 -- the
  reference's method (conv.py:57-88); here all instructions are probed in one batch.
* The kernels are generated per layer by the C library (coefficients baked in as constants, NVRTC, sm_100a):
  persistent, warp-specialised, with the per-edge rows streamed into shared memory by TMA; forward over the receiver
  CSR (deterministic, no atomics); backward in one fused pass over the sender CSR giving gx per sender and gW, gY per
  edge.
* The receiver and sender CSRs are built on the GPU once per edge_index tensor (both interaction layers and the
  backward reuse them); the reference re-sorts on every forward and backward (conv.py:245, 262).
"""
from __future__ import annotations

import weakref

import torch

from . import _lib

DOUBLE_BACKWARD_MSG = ('mace-b200-kernels: double backward (create_graph=True, e.g. training on forces/stress or an '
                       'autograd Hessian) is not supported by the CUDA kernels; use the unpatched e3nn model for that')


class _Ir:
    def __init__(self, l):
        self.l = int(l)


def _blocks(irreps):
    res, off = [], 0
    for mul, ir in irreps:
        res.append((ir.l, mul, off))
        off += mul * (2 * ir.l + 1)
    return res, off


def conv_supported(tp):
    """(ok, reason) -- whether an e3nn-style TensorProduct can be replaced by the fused CUDA convolution."""
    try:
        ins = tp.instructions
        if any(i.connection_mode != 'uvu' or not i.has_weight for i in ins):
            return False, 'only weighted uvu instructions are supported'
        if getattr(tp, 'shared_weights', True) or getattr(tp, 'internal_weights', True):
            return False, 'per-edge (external, unshared) weights required'
        muls = {m for m, _ in tp.irreps_in1} | {m for m, _ in tp.irreps_out}
        if len(muls) != 1:
            return False, 'all node/out blocks must have the same multiplicity'
        mul = muls.pop()
        if mul % 32:
            return False, f'multiplicity {mul} is not a multiple of 32'
        if mul > 512:
            return False, f'multiplicity {mul} is above 512'
        if any(m != 1 for m, _ in tp.irreps_in2):
            return False, 'edge attributes must have multiplicity 1 per l'
        if sum(2 * ir.l + 1 for _, ir in tp.irreps_in2) > 16:
            return False, 'edge attributes wider than 16 components (l_max > 3)'
        if tp.weight_numel != len(ins) * mul:
            return False, 'unexpected weight layout'
    except AttributeError as e:
        return False, f'not an e3nn TensorProduct ({e})'
    return True, ''


class ConvSpec:
    """Instruction table and probed path coefficients of one uvu TensorProduct."""

    def __init__(self, tp, tol=1e-7):
        ok, why = conv_supported(tp)
        if not ok:
            raise ValueError(why)
        self.in1, self.x_dim = _blocks(tp.irreps_in1)
        self.in2, self.y_dim = _blocks(tp.irreps_in2)
        self.outb, self.out_dim = _blocks(tp.irreps_out)
        self.mul = self.in1[0][1]
        self.ins = [(i.i_in1, i.i_in2, i.i_out) for i in tp.instructions]
        self.nins = len(self.ins)
        self.w_dim = self.nins * self.mul
        dev = next(iter(tp.buffers()), torch.zeros(1)).device
        # one probe row per (instruction k, x component a, Y component b): unit x on channel 0, unit Y, unit w_k
        rows = []
        for k, (i1, i2, io) in enumerate(self.ins):
            d1, d2 = 2 * self.in1[i1][0] + 1, 2 * self.in2[i2][0] + 1
            rows += [(k, a, b) for a in range(d1) for b in range(d2)]
        R = len(rows)
        x1 = torch.zeros(R, self.x_dim, device=dev)
        x2 = torch.zeros(R, self.y_dim, device=dev)
        w = torch.zeros(R, tp.weight_numel, device=dev)
        rk = torch.tensor([r[0] for r in rows], device=dev)
        ra = torch.tensor([self.in1[self.ins[r[0]][0]][2] + r[1] for r in rows], device=dev)
        rb = torch.tensor([self.in2[self.ins[r[0]][1]][2] + r[2] for r in rows], device=dev)
        ar = torch.arange(R, device=dev)
        x1[ar, ra] = 1.0
        x2[ar, rb] = 1.0
        w[ar, rk * self.mul] = 1.0
        with torch.no_grad():
            y = tp(x1, x2, w).detach().cpu().double()
        self.coef = []
        for k, (i1, i2, io) in enumerate(self.ins):
            l1, _, o1 = self.in1[i1]
            l2, _, o2 = self.in2[i2]
            l3, _, o3 = self.outb[io]
            self.coef.append(dict(k=k, l1=l1, l2=l2, l3=l3, o1=o1, o2=o2, o3=o3, terms=[]))
        for r, (k, a, b) in enumerate(rows):
            c = self.coef[k]
            for m in range(2 * c['l3'] + 1):
                v = float(y[r, c['o3'] + m])
                if abs(v) > tol:
                    c['terms'].append((a, b, m, v))
        self.nnz = sum(len(c['terms']) for c in self.coef)

    @classmethod
    def from_table(cls, mul, in1_l, in2_l, out_l, ins, terms):
        """Spec from an explicit coefficient table: ``ins`` = [(i_in1, i_in2, i_out)], ``terms`` = [(k, a, b, m, c)]."""
        self = cls.__new__(cls)
        mk = lambda ls, mult: _blocks([(mult, _Ir(l)) for l in ls])
        self.in1, self.x_dim = mk(in1_l, mul)
        self.in2, self.y_dim = mk(in2_l, 1)
        self.outb, self.out_dim = mk(out_l, mul)
        self.mul = mul
        self.ins = [tuple(int(v) for v in t) for t in ins]
        self.nins = len(self.ins)
        self.w_dim = self.nins * mul
        self.coef = []
        for k, (i1, i2, io) in enumerate(self.ins):
            self.coef.append(dict(k=k, l1=self.in1[i1][0], l2=self.in2[i2][0], l3=self.outb[io][0], o1=self.in1[i1][2],
                                  o2=self.in2[i2][2], o3=self.outb[io][2], terms=[]))
        for k, a, b, m, c in terms:
            self.coef[int(k)]['terms'].append((int(a), int(b), int(m), float(c)))
        self.nnz = len(terms)
        return self

    def descriptor(self):
        """ctypes ``mmk_conv_desc`` (arrays kept alive on the returned object)."""
        keep = {}
        keep['in1'] = _lib.int_array(l for l, _, _ in self.in1)
        keep['in2'] = _lib.int_array(l for l, _, _ in self.in2)
        keep['out'] = _lib.int_array(l for l, _, _ in self.outb)
        keep['i1'] = _lib.int_array(i for i, _, _ in self.ins)
        keep['i2'] = _lib.int_array(i for _, i, _ in self.ins)
        keep['io'] = _lib.int_array(i for _, _, i in self.ins)
        terms = [(c['k'], a, b, m, v) for c in self.coef for a, b, m, v in c['terms']]
        keep['tk'] = _lib.int_array(t[0] for t in terms)
        keep['ta'] = _lib.int_array(t[1] for t in terms)
        keep['tb'] = _lib.int_array(t[2] for t in terms)
        keep['tm'] = _lib.int_array(t[3] for t in terms)
        keep['tc'] = _lib.double_array(t[4] for t in terms)
        d = _lib.ConvDesc(self.mul, len(self.in1), keep['in1'], len(self.in2), keep['in2'], len(self.outb),
                          keep['out'], self.nins, keep['i1'], keep['i2'], keep['io'], len(terms), keep['tk'],
                          keep['ta'], keep['tb'], keep['tm'], keep['tc'])
        d._keep = keep
        return d


# ----------------------------------------------------------------------------------------------------------------------
# CSR of the graph, built on the device once per edge_index tensor
# ----------------------------------------------------------------------------------------------------------------------
_CSR_CACHE = []          # [(weakref(edge_index), key, csr)], most recent last
_CSR_CACHE_SIZE = 4


def _tensor_key(t: torch.Tensor, *extra):
    """What a cached per-tensor result depends on: the storage address, shape, strides, device and autograd version
    counter.  In-place writes through PyTorch bump the version; writes that bypass it (DLPack, C extensions,
    ``.data``, a CUDA-graph replay) are not seen -- call ``invalidate_graph_caches()`` after those."""
    return (t.data_ptr(), tuple(t.shape), tuple(t.stride()), str(t.device), t._version) + extra


def invalidate_graph_caches():
    """Forget every cached receiver/sender CSR and element grouping.  Needed only when an ``edge_index`` or
    ``node_attrs`` tensor's contents were changed in a way PyTorch's version counter does not see."""
    _CSR_CACHE.clear()
    from . import symmetric
    symmetric._ELEM_CACHE.clear()


def source(spec):
    """Generated CUDA layer header for ``spec`` (sizes, launch plan and the straight-line per-edge bodies with the
    probed coefficients), the counterpart of the reference's ``source(spec)`` (conv.py:225)."""
    return _lib.generated_source('mmk_conv_source', spec.descriptor())


def csr_build(index: torch.Tensor, n_nodes: int):
    """(rowptr int32[n+1], eids int32[E]) with eids grouped by ``index`` in increasing edge id, on index's device
    (the reference's ``csr_by``, conv.py:229-235)."""
    E = index.numel()
    rowptr = torch.empty(n_nodes + 1, dtype=torch.int32, device=index.device)
    eids = torch.empty(E, dtype=torch.int32, device=index.device)
    ws_bytes = _lib.lib().mmk_csr_workspace_bytes(n_nodes, E)
    ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=index.device)
    _lib.call('mmk_csr_build', _lib.ptr(index), E, n_nodes, _lib.ptr(rowptr), _lib.ptr(eids), _lib.ptr(ws), ws_bytes,
              None, _lib.stream_of(index))
    return rowptr, eids


def csr_build_pair(edge_index: torch.Tensor, n_nodes: int):
    """(recv_rowptr, recv_eids, send_rowptr, send_eids) of a contiguous int64 [2, E] edge_index in one sequence of
    launches (C ABI ``mmk_csr_build_pair``); each equals ``csr_build`` of that row."""
    E = edge_index.shape[1]
    rowptr = torch.empty(2, n_nodes + 1, dtype=torch.int32, device=edge_index.device)
    eids = torch.empty(2, E, dtype=torch.int32, device=edge_index.device)
    ws_bytes = _lib.lib().mmk_csr_pair_workspace_bytes(n_nodes, E)
    ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=edge_index.device)
    _lib.call('mmk_csr_build_pair', _lib.ptr(edge_index), E, n_nodes, _lib.ptr(rowptr), _lib.ptr(eids), _lib.ptr(ws),
              ws_bytes, None, _lib.stream_of(edge_index))
    return rowptr[1], eids[1], rowptr[0], eids[0]


def graph_csr(edge_index: torch.Tensor, n_nodes: int):
    """Receiver and sender CSRs of a contiguous int64 [2, E] edge_index.  Both interaction layers and the backward of
    one evaluation see the same edge_index tensor, so the CSRs are built once and cached, keyed on the tensor object,
    its storage address, shape, strides and version counter, and n_nodes (see ``invalidate_graph_caches``)."""
    key = _tensor_key(edge_index, int(n_nodes))
    for ref, k, csr in reversed(_CSR_CACHE):
        if ref() is edge_index and k == key:
            return csr
    csr = csr_build_pair(edge_index, n_nodes)
    _CSR_CACHE.append((weakref.ref(edge_index), key, csr))
    del _CSR_CACHE[:-_CSR_CACHE_SIZE]
    return csr


def _check_inputs(x, Y, W, edge_index, spec):
    for name, t in (('node_feats', x), ('edge_attrs', Y), ('tp_weights', W)):
        if t.dtype != torch.float32 or not t.is_cuda:
            raise TypeError(f'{name} must be a float32 CUDA tensor (got {t.dtype} on {t.device})')
    N, E = x.shape[0], Y.shape[0]
    if x.shape != (N, spec.x_dim) or Y.shape != (E, spec.y_dim) or W.shape != (E, spec.w_dim):
        raise ValueError(f'shape mismatch: x {tuple(x.shape)}, Y {tuple(Y.shape)}, W {tuple(W.shape)} for layer '
                         f'x_dim={spec.x_dim} y_dim={spec.y_dim} w_dim={spec.w_dim}')
    if edge_index.shape != (2, E):
        raise ValueError(f'edge_index must be [2, {E}] (got {tuple(edge_index.shape)})')


class _ConvFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, Y, W, edge_index, op):
        _check_inputs(x, Y, W, edge_index, op.spec)
        x, Y, W = (_lib.aligned(t.contiguous()) for t in (x, Y, W))
        ei = edge_index.to(device=x.device, dtype=torch.int64).contiguous()
        n, E = x.shape[0], Y.shape[0]
        rrow, reid, srow, seid = graph_csr(ei, n)
        out = torch.empty(n, op.spec.out_dim, device=x.device, dtype=torch.float32)
        _lib.call('mmk_conv_fwd', op.handle, _lib.ptr(x), _lib.ptr(Y), _lib.ptr(W), _lib.ptr(rrow), _lib.ptr(reid),
                  _lib.ptr(ei), _lib.ptr(out), n, E, _lib.stream_of(x))
        ctx.save_for_backward(x, Y, W, ei, srow, seid)
        ctx.op = op
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():          # only true under create_graph=True
            raise RuntimeError(DOUBLE_BACKWARD_MSG)
        x, Y, W, ei, srow, seid = ctx.saved_tensors
        op = ctx.op
        g = _lib.aligned(g.contiguous())
        n, E = x.shape[0], Y.shape[0]
        gx = torch.empty_like(x) if ctx.needs_input_grad[0] else None
        gY = gW = None
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            gY, gW = torch.empty_like(Y), torch.empty_like(W)
        if gx is None and gY is None:
            return None, None, None, None, None
        recv_ptr = ei.data_ptr() + E * ei.element_size()
        _lib.call('mmk_conv_bwd', op.handle, _lib.ptr(x), _lib.ptr(Y), _lib.ptr(W), _lib.ptr(g), _lib.ptr(srow),
                  _lib.ptr(seid), recv_ptr, _lib.ptr(gx), _lib.ptr(gY), _lib.ptr(gW), n, E, _lib.stream_of(x))
        return gx, gY, gW, None, None


class _LayerHandle:
    """Owns one mmk_conv_layer / mmk_sc_layer handle."""

    def __init__(self, create, destroy, desc):
        import ctypes
        h = ctypes.c_void_p()
        _lib.call(create, ctypes.byref(desc), ctypes.byref(h))
        self.value = h
        self._destroy = getattr(_lib.lib(), destroy)

    def __del__(self):
        try:
            if self.value:
                self._destroy(self.value)
        except Exception:       # interpreter shutdown
            pass


class CudaConvTP(torch.nn.Module):
    """Replacement for an interaction block's ``conv_tp`` under MACE's ``conv_fusion`` path:
    forward(node_feats, edge_attrs, tp_weights, edge_index) -> summed messages [N, OUT_DIM]."""

    def __init__(self, tp, spec=None):
        super().__init__()
        self.spec = ConvSpec(tp) if spec is None else spec
        self._h = _LayerHandle('mmk_conv_layer_create', 'mmk_conv_layer_destroy', self.spec.descriptor())
        if tp is not None:
            self.irreps_in1, self.irreps_in2, self.irreps_out = tp.irreps_in1, tp.irreps_in2, tp.irreps_out
            self.weight_numel = tp.weight_numel
        else:
            self.irreps_in1 = self.irreps_in2 = self.irreps_out = None
            self.weight_numel = self.spec.w_dim

    @classmethod
    def from_spec(cls, spec):
        """Op for an explicit ``ConvSpec`` (e.g. ``ConvSpec.from_table``) without a TensorProduct object."""
        return cls(None, spec)

    @property
    def handle(self):
        return self._h.value

    def status(self, reset=False):
        """Error status of this layer's kernels on the current device (0 = ok); synchronises with the device."""
        import ctypes
        v = ctypes.c_int(0)
        _lib.call('mmk_conv_layer_status', self.handle, ctypes.byref(v), int(reset))
        return v.value

    def __deepcopy__(self, memo):
        new = self.__class__.__new__(self.__class__)
        torch.nn.Module.__init__(new)
        new.spec = self.spec
        new._h = self._h
        new.irreps_in1, new.irreps_in2, new.irreps_out = self.irreps_in1, self.irreps_in2, self.irreps_out
        new.weight_numel = self.weight_numel
        return new

    def forward(self, node_feats, edge_attrs, tp_weights, edge_index):
        return _ConvFn.apply(node_feats, edge_attrs, tp_weights, edge_index, self)


MetalConvTP = CudaConvTP        # the reference's class name, for drop-in imports
