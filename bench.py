"""Energy + force throughput of a patched MACE model on B200 (and the CPU e3nn-path baseline).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the configuration the headline metric is quoted on): random 128-channel MACE,
hidden 128x0e+128x1o, l_max 3, correlation 3, 4 elements (H, C, O, Pt), r_max 5 A, 2 interactions; one Pt(100) 6x6x4
slab with seeded CO/O/H adsorbates (~160 atoms, ~5 000 edges).  With N GPUs (torchrun, one process per GPU) every
rank runs its own structure (seed = rank): weak scaling, the only collective is the per-step energy all_gather.

One step = one energy + force call (model forward + autograd backward through the patched kernels).  The model is
patched with patch_model(model, edge_features=True, linears=True) on frozen weights: the reference's two ops (conv,
symmetric contraction) plus this repository's edge-geometry (edge vectors and lengths, spherical harmonics, radial
basis), equivariant-linear, reshape and radial-MLP kernels.  Inputs are
much smaller than L2, so L2 is flushed (256 MB write) before every timed step, outside the CUDA-event interval.

The timed step is a replay of the whole E+F call captured in a CUDA graph (GraphedEnergyForces); the eager time is
reported beside it.

Printed JSON (rank 0): value = atoms x ranks / step time (max over ranks, CUDA events); e2e = the same through the
public API with host inputs (pinned H2D copies of the graph and a D2H copy of the forces inside the timed interval);
ops = every patched op's forward and backward kernel on the step's own inputs, launched through the C ABI ('cold':
1 GiB L2 flush before each launch; 'hot': back to back); roofline = the dominant one's algorithmic bytes / its
CUDA-event duration against the measured HBM copy bandwidth; ops_large / roofline_large = the same ops of the
configs[4] architecture on a bulk Cu supercell far larger than L2 (symmetric contraction against a measured FP32 GEMM
peak); cpu_baseline = the unpatched e3nn-path model on the host cores (rank 0, N = 1 only).

Extra keys, the other BASELINE configurations (skipped with --no-extras):
  batch16      configs[2]: 16 configs[0]-style structures, padded to 6 000 edges each, sharded by structure over the
               ranks (weak in structures per rank: N ranks share the fixed 16), graphed, energy gather per step;
  partitioned  configs[4]: one bulk Cu system (--part-cells^3 cells, 128x0e+128x1o+128x2e) partitioned by receiving
               atom over the ranks, halo all_to_all per interaction (strong scaling; time and bytes of the halo
               collectives reported);
  relax89      configs[3] (N = 1 only): 89-element model on CeO2(111) + Au13, 50-call L-BFGS loop at a fixed padded
               graph, with the energy match against the same loop on the unpatched model.

Profiling entry points (ncu --profile-from-start off ...): --profile step (three graph replays of the E+F step),
--profile ops [--large-cells K] (one launch of every large-system op), --profile gemm (the radial MLP's last-layer
GEMM at the configs[1] layer-2 shapes).
"""
from __future__ import annotations

import argparse
import copy
import json
import os
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from mace_mps_kernels_b200 import _lib, patch_model, standin  # noqa: E402
from mace_mps_kernels_b200.conv import CudaConvTP  # noqa: E402
from mace_mps_kernels_b200.graphs import GraphedEnergyForces  # noqa: E402
from mace_mps_kernels_b200.symmetric import CudaSymmetricContraction  # noqa: E402

METRIC = 'E+F atom-steps/s'
UNIT = 'atom-steps/s'
HIDDEN, LMAX, CORR, RMAX = '128x0e+128x1o', 3, 3, 5.0
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d['hbm_gbs']), 'measured'
    return FALLBACK_HBM_GBS, 'fallback'


def workload(rank):
    st = standin.pt100_random(seed=rank)
    batch = standin.structure_batch([st], standin.ELEMENTS_PTCOH, RMAX)
    return st, batch


def config_dict(atoms_total, edges_total, world):
    """atoms_total / edges_total: summed over the ranks (each rank evaluates its own seeded structure)."""
    per = '' if world == 1 else f' in total over {world} structures (one per rank)'
    return {'workload': f'configs[1]: MACE 128ch {HIDDEN} l_max {LMAX} corr {CORR} 4 elements r_max {RMAX}; '
                        f'Pt(100) 6x6x4 + CO/O/H, {atoms_total} atoms, {edges_total} edges{per}',
            'model': 'ScaleShiftMACE (in-repo mace-torch 0.3.x stand-in, random weights seed 0, frozen)',
            'patched': 'conv_tp, symmetric contraction, edge features, equivariant linears, radial MLP',
            'global_batch': world, 'atoms_total': atoms_total, 'edges_total': edges_total,
            'parallelism': f'dp{world} (structure batch, one structure per rank)',
            'l2': 'flushed (256 MB write) before every timed step'}


class ClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU, sampled every 20 ms by a thread through NVML (read
    only) during a timed region (no samples, and None in the summary, where NVML is unavailable)."""

    REASONS = [('hw_slowdown', 'nvmlClocksEventReasonHwSlowdown'),
               ('hw_thermal_slowdown', 'nvmlClocksEventReasonHwThermalSlowdown'),
               ('sw_thermal_slowdown', 'nvmlClocksEventReasonSwThermalSlowdown'),
               ('sw_power_cap', 'nvmlClocksEventReasonSwPowerCap')]

    def __init__(self, index):
        self.index = index
        self.sm, self.mx, self.power, self.reasons = [], None, [], set()
        self._stop = threading.Event()
        self._thread = None

    def _handle(self, nv):
        try:
            pr = torch.cuda.get_device_properties(self.index)
            return nv.nvmlDeviceGetHandleByPciBusId(f'{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0')
        except Exception:                                        # noqa: BLE001
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def _loop(self, nv, h):
        bits = [(name, getattr(nv, const)) for name, const in self.REASONS]
        while not self._stop.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                self.power.append(nv.nvmlDeviceGetPowerUsage(h) / 1000.0)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in bits:
                    if r & bit:
                        self.reasons.add(name)
            except Exception:                                    # noqa: BLE001
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._loop, args=(nv, h), daemon=True)
            self._thread.start()
        except Exception:                                        # noqa: BLE001
            self._thread = None
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        return {'sm_mhz': float(np.median(self.sm)) if self.sm else None, 'sm_max_mhz': self.mx,
                'reasons': sorted(self.reasons), 'samples': len(self.sm),
                'power_w_max': round(max(self.power), 1) if self.power else None}


def flush_l2(buf):
    buf.zero_()


def e_and_f(model, batch):
    b = dict(batch)
    b['positions'] = b['positions'].detach().requires_grad_(True)
    out = model(b, compute_force=True, training=False)
    return out['energy'], out['forces']


def capture_op_inputs(model, batch):
    """Arguments every patched op sees in one E+F call (for per-op timing)."""
    calls = []

    def hook(mod, args, kwargs, out):
        calls.append((mod, [a.detach() if torch.is_tensor(a) else a for a in args], out.detach()))

    hs = [m.register_forward_hook(hook, with_kwargs=True) for m in model.modules()
          if isinstance(m, (CudaConvTP, CudaSymmetricContraction))]
    e_and_f(model, batch)
    for h in hs:
        h.remove()
    return calls


def conv_bytes(spec, N, E):
    """Algorithmic bytes of one conv launch: unique tensors once (fp32) + CSR (int32) + edge index (int64)."""
    fwd = 4 * (N * spec.x_dim + E * spec.y_dim + E * spec.w_dim + N * spec.out_dim) + 4 * (N + 1 + E) + 8 * E
    bwd = 4 * (N * spec.out_dim + N * spec.x_dim + E * spec.y_dim + E * spec.w_dim + E * spec.w_dim
               + E * spec.y_dim + N * spec.x_dim) + 4 * (N + 1 + E) + 8 * E
    return fwd, bwd


def layer_dims(spec):
    return [spec.x_dim, spec.y_dim, spec.w_dim, spec.out_dim]


def conv_case(mod, x, Y, W, ei, name):
    """(fwd, bwd) closures launching one conv layer's kernels through the C ABI on preallocated buffers."""
    from mace_mps_kernels_b200.conv import graph_csr
    P = _lib.ptr
    st = _lib.stream_of(x)
    N, E = x.shape[0], Y.shape[0]
    rr, re_, sr, se = graph_csr(ei, N)
    o = torch.empty(N, mod.spec.out_dim, device=x.device)
    g = torch.randn_like(o)
    gx, gY, gW = torch.empty_like(x), torch.empty_like(Y), torch.empty_like(W)
    recv = ei.data_ptr() + E * 8
    fwd = lambda: _lib.call('mmk_conv_fwd', mod.handle, P(x), P(Y), P(W), P(rr), P(re_), P(ei), P(o), N, E, st)
    bwd = lambda: _lib.call('mmk_conv_bwd', mod.handle, P(x), P(Y), P(W), P(g), P(sr), P(se), recv, P(gx), P(gY),
                            P(gW), N, E, st)
    bf, bb = conv_bytes(mod.spec, N, E)
    return dict(op=name, kind='conv', N=N, E=E, nnz=mod.spec.nnz, fwd=fwd, bwd=bwd, fwd_bytes=bf, bwd_bytes=bb,
                dims=layer_dims(mod.spec), keep=(mod, o, g, gx, gY, gW, rr, re_, sr, se))


def sc_case(mod, x, attrs, name):
    from mace_mps_kernels_b200.symmetric import element_groups
    P = _lib.ptr
    st = _lib.stream_of(x)
    N = x.shape[0]
    _, erow, perm = element_groups(attrs)
    ne = erow.shape[0] - 1
    o = torch.empty(N, mod.spec.out_dim, device=x.device)
    g = torch.randn_like(o)
    gx = torch.empty_like(x)
    fwd = lambda: _lib.call('mmk_sc_fwd', mod.handle, P(x), P(perm), P(erow), ne, P(mod.T), P(o), N, st)
    bwd = lambda: _lib.call('mmk_sc_bwd', mod.handle, P(x), P(perm), P(erow), ne, P(mod.T), P(g), P(gx), N, st)
    from mace_mps_kernels_b200.symmetric import executed_flops
    ff, fb = mod.spec.flops()
    ef, eb = executed_flops(mod.spec)
    C = mod.spec.C
    return dict(op=name, kind='sc', N=N, terms=mod.spec.n_terms, fwd=fwd, bwd=bwd, fwd_flops=ff * N * C,
                bwd_flops=fb * N * C, fwd_exec_flops=ef * N * C, bwd_exec_flops=eb * N * C,
                keep=(mod, o, g, gx, erow, perm))


def time_cases(cases, reps, flush):
    """Per launch, CUDA events: 'cold' = L2 flushed (1 GiB write) before each launch, which also lets the host enqueue
    the launch before the GPU reaches the start event; 'hot' = reps launches back to back between two events."""
    res = []
    for c in cases:
        print(f'[bench] timing {c["op"]}', file=sys.stderr, flush=True)
        out = {k: v for k, v in c.items() if k not in ('fwd', 'bwd', 'keep', 'dims')}
        out['_dims'] = c.get('dims')
        for tag in ('fwd', 'bwd'):
            fn = c[tag]
            ts = []
            for r in range(reps + 2):
                flush()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                e1.synchronize()
                if r >= 2:
                    ts.append(e0.elapsed_time(e1) * 1e3)
            out[f'{tag}_us'] = float(np.median(ts))
            flush()
            fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            e1.synchronize()
            out[f'{tag}_hot_us'] = e0.elapsed_time(e1) * 1e3 / reps
            if c['kind'] == 'conv':
                out[f'{tag}_gbs'] = c[f'{tag}_bytes'] / out[f'{tag}_us'] * 1e-3
            elif f'{tag}_flops' in c:
                out[f'{tag}_tflops'] = c[f'{tag}_flops'] / out[f'{tag}_us'] * 1e-6
                if f'{tag}_exec_flops' in c:        # what the generated code executes (fewer than the term count)
                    out[f'{tag}_exec_tflops'] = c[f'{tag}_exec_flops'] / out[f'{tag}_us'] * 1e-6
        res.append(out)
    return res


def other_cases(model, batch):
    """The other library ops of one E+F call (equivariant linears and skip connections, the radial MLP's hidden
    layers and its tensor-core last layer), each with the inputs it saw, as (fwd, bwd) launch closures."""
    from mace_mps_kernels_b200 import gemm as G
    from mace_mps_kernels_b200.dense import CudaFullyConnectedNet, CudaLinear, CudaSkipTP
    from mace_mps_kernels_b200.symmetric import element_groups
    calls = []

    def hook(mod, args, kwargs, out):
        calls.append((mod, [a.detach() if torch.is_tensor(a) else a for a in args]))

    hs = [m.register_forward_hook(hook, with_kwargs=True) for m in model.modules()
          if isinstance(m, (CudaLinear, CudaSkipTP, CudaFullyConnectedNet))]
    e_and_f(model, batch)
    for h in hs:
        h.remove()
    cases = []
    for k, (mod, args) in enumerate(calls):
        x = args[0].contiguous()
        if isinstance(mod, CudaFullyConnectedNet):
            if not mod.fused:
                continue
            E, L = x.shape[0], len(mod.hidden_widths) - 1
            h = torch.empty(E, mod.hidden_widths[-1], device=x.device)
            z = torch.empty(E * sum(mod.hidden_widths[1:]), device=x.device)
            gh = torch.randn_like(h)
            gx = torch.empty_like(x)
            P = _lib.ptr
            st = _lib.stream_of(x)
            fwd = lambda x=x, h=h, z=z, mod=mod, E=E, L=L, st=st: _lib.call(
                'mmk_mlp_fwd', P(x), E, L, mod.widths_c(), P(mod.w_hidden), mod.scale, P(h), P(z), st)
            bwd = lambda gh=gh, z=z, gx=gx, mod=mod, E=E, L=L, st=st: _lib.call(
                'mmk_mlp_bwd', P(gh), E, L, mod.widths_c(), P(mod.w_hidden_t), P(z), mod.scale, P(gx), st)
            flops = sum(2 * E * a * b for a, b in zip(mod.hidden_widths[:-1], mod.hidden_widths[1:]))
            cases.append(dict(op=f'mlp_hidden[{k}]', kind='mlp', N=E, fwd=fwd, bwd=bwd, fwd_flops=flops,
                              bwd_flops=flops, keep=(x, h, z, gh, gx)))
            lin = mod.last
            W = torch.empty(E, lin.n + lin.n_pad, device=x.device)
            gW = torch.randn_like(W)
            gh2 = torch.empty(E, lin.k + lin.k_pad, device=x.device)
            hp = torch.randn(E, lin.k + lin.k_pad, device=x.device)
            fwd = lambda hp=hp, lin=lin, W=W: G.matmul_nt(hp, lin.wt_hi, lin.wt_lo, out=W)
            bwd = lambda gW=gW, lin=lin, gh2=gh2: G.matmul_nt(gW, lin.w_hi, lin.w_lo, out=gh2)
            f = 2 * E * lin.k * lin.n
            cases.append(dict(op=f'mlp_last_gemm[{k}]', kind='gemm', N=E, fwd=fwd, bwd=bwd, fwd_flops=f,
                              bwd_flops=f, keep=(hp, W, gW, gh2)))
            continue
        groups = None
        if isinstance(mod, CudaSkipTP):
            _, erow, perm = element_groups(args[1].contiguous())
            groups = (perm, erow, mod.n_elem)
        N = x.shape[0]
        out = torch.empty(N, mod.out_dim, device=x.device)
        g = torch.randn_like(out)
        gx = torch.empty_like(x)
        fwd = lambda mod=mod, x=x, out=out, groups=groups: mod._launch(mod.fwd, x, mod.in_dim, out, mod.out_dim, groups)
        bwd = lambda mod=mod, g=g, gx=gx, groups=groups: mod._launch(mod.bwd, g, mod.out_dim, gx, mod.in_dim, groups)
        cases.append(dict(op=f'{type(mod).__name__}[{k}]', kind='block_linear', N=N, fwd=fwd, bwd=bwd,
                          keep=(x, out, g, gx, groups)))
    return cases


def step_breakdown(conv_sc_ops, other_ops):
    """Measured time per library-op family in one E+F step (sum over its launches of the cold per-launch times) and
    the family with the largest share."""
    fam = {}
    for o in conv_sc_ops + other_ops:
        name = {'conv': 'conv_tp (mmk_conv_fwd/bwd_kernel)', 'sc': 'symmetric contraction (mmk_sc_fwd/bwd_kernel)',
                'block_linear': 'equivariant linears + skip (k_block_linear)',
                'mlp': 'radial MLP hidden layers (k_mlp_fwd/bwd)',
                'gemm': 'radial MLP last layer (k_gemm_tf32x3)'}[o['kind']]
        f = fam.setdefault(name, {'us': 0.0, 'launches': 0})
        f['us'] += o['fwd_us'] + o['bwd_us']
        f['launches'] += 2
    total = sum(f['us'] for f in fam.values())
    for f in fam.values():
        f['share'] = round(f['us'] / total, 4)
        f['us'] = round(f['us'], 1)
    top = max(fam, key=lambda k: fam[k]['us'])
    return {'families': fam, 'top': top, 'library_us_sum': round(total, 1),
            'timing': "each op's forward and backward launch on the step's own inputs, cold (1 GiB L2 flush before "
                      "each launch), summed per family; launch gaps and PyTorch glue kernels not included"}


def step_cases(model, batch):
    """The patched ops of one E+F call of ``model`` on ``batch``, with the inputs they saw."""
    calls = capture_op_inputs(model, batch)
    cases, nc, ns = [], 0, 0
    for mod, args, out in calls:
        if isinstance(mod, CudaConvTP):
            x, Y, W, ei = (a.contiguous() for a in args)
            cases.append(conv_case(mod, x, Y, W, ei, f'conv_tp[{nc}]'))
            nc += 1
        else:
            x, attrs = (a.contiguous() for a in args)
            cases.append(sc_case(mod, x, attrs, f'symcon[{ns}]'))
            ns += 1
    return cases


LARGE_CELLS = 10
TRAFFIC_FILE = os.path.join(ROOT, 'profiles', 'conv_dram_traffic.json')


def profile_gemm(dev, M=5218):
    """--profile gemm: the radial MLP's last layer at the configs[1] layer-2 shapes, forward W = h . Wr
    (M x 1280 x 64) and the input gradient gh = gW . Wr^T (M x 64 x 1280), one launch each between
    cudaProfilerStart/Stop after three warm launches."""
    from mace_mps_kernels_b200 import gemm
    torch.manual_seed(0)
    cases = []
    for m, n, k in ((M, 1280, 64), (M, 64, 1280)):
        A, B = torch.randn(m, k, device=dev), torch.randn(n, k, device=dev)
        hi, lo = gemm.tf32_split(B)
        cases.append((A, hi, lo, torch.empty(m, n, device=dev)))
    for _ in range(3):
        for A, hi, lo, C in cases:
            gemm.matmul_nt(A, hi, lo, out=C)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for A, hi, lo, C in cases:
        gemm.matmul_nt(A, hi, lo, out=C)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({'profile': 'gemm', 'launch_order': [f'{m}x{n}x{k}' for m, n, k in ((M, 1280, 64), (M, 64, 1280))]}))


def measured_traffic(kernel_pair, N, E, spec_key):
    """DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum, forward + backward launch) of this conv layer at
    exactly this graph size, from the committed ncu capture (None when no capture of this exact launch exists)."""
    if not os.path.exists(TRAFFIC_FILE):
        return None
    rec = json.load(open(TRAFFIC_FILE))
    import hashlib
    src = os.path.join(ROOT, 'mace_mps_kernels_b200', 'csrc', 'conv_tp.cuh')
    if hashlib.sha1(open(src, 'rb').read()).hexdigest()[:16] != rec.get('conv_tp_cuh_sha1_16'):
        return None                                 # captured from another version of the kernels
    for r in rec.get('launches', []):
        if (r.get('layer_dims') == spec_key and r.get('N') == N and r.get('E') == E
                and set(r.get('dram_bytes', {})) >= set(kernel_pair)):
            tot = sum(r['dram_bytes'][k] for k in kernel_pair)
            return tot, f"ncu capture: {rec.get('command', '?')}"
    return None


def large_cases(dev, cells=LARGE_CELLS):
    """configs[4]'s architecture (128x0e+128x1o+128x2e, l_max 3, correlation 3) on a bulk fcc Cu supercell of
    LARGE_CELLS^3 conventional cells (Morton-ordered atoms, r_max 5 A): per-op inputs far larger than L2."""
    torch.manual_seed(1)
    model = standin.make_model('128x0e+128x1o+128x2e', 3, 3, seed=0, elements=[29, 30, 31, 32]).to(dev)
    patch_model(model, verbose=False)
    st = standin.fcc_bulk('Cu', 3.61, cells, seed=0, jitter=0.1)
    st = st.permuted(standin.structures.morton_order(st.positions, st.cell))
    i, j, _ = standin.neighbor_list(st.positions, st.cell, st.pbc, 5.0)
    ei = torch.from_numpy(np.stack([i, j])).to(dev)
    N, E = len(st), ei.shape[1]
    cases = []
    for k, blk in enumerate(model.interactions):
        sp = blk.conv_tp.spec
        x = torch.randn(N, sp.x_dim, device=dev)
        Y = torch.randn(E, sp.y_dim, device=dev)
        W = torch.randn(E, sp.w_dim, device=dev)
        cases.append(conv_case(blk.conv_tp, x, Y, W, ei, f'conv_tp[{k}] Cu{cells}^3'))
    attrs = torch.zeros(N, 4, device=dev)
    attrs[:, 0] = 1.0
    for k, prod in enumerate(model.products):
        sc = prod.symmetric_contractions
        x = torch.randn(N, sc.spec.C, sc.spec.n_ell, device=dev)
        cases.append(sc_case(sc, x, attrs, f'symcon[{k}] Cu{cells}^3'))
    return cases, dict(atoms=N, edges=E, model='128x0e+128x1o+128x2e l_max 3 corr 3')


def fp32_peak(dev):
    """Measured FP32 (no TF32) GEMM throughput, TFLOP/s: the FP32-issue roof for the symmetric contraction."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(8192, 8192, device=dev)
    b = torch.randn(8192, 8192, device=dev)
    for _ in range(2):
        a @ b
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        a @ b
    e1.record()
    e1.synchronize()
    torch.backends.cuda.matmul.allow_tf32 = prev
    return 2 * 8192 ** 3 * 5 / (e0.elapsed_time(e1) * 1e-3) / 1e12


def cpu_baseline(n_steps_cap=5, budget_s=20.0):
    """Unpatched (e3nn-path) stand-in model on the host cores: E+F atom-steps/s on this rank's structure."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    model = standin.make_model(HIDDEN, LMAX, CORR, seed=0, elements=standin.ELEMENTS_PTCOH).requires_grad_(False)
    st, batch = workload(0)
    e_and_f(model, batch)                       # warm-up (allocations, caches)
    times = []
    t_start = time.perf_counter()
    while len(times) < n_steps_cap and time.perf_counter() - t_start < budget_s:
        t0 = time.perf_counter()
        e_and_f(model, batch)
        times.append(time.perf_counter() - t0)
    sec = float(np.mean(times))
    return {'value': len(st) / sec, 'unit': UNIT, 'cores': cores, 'kind': 'port',
            'sample': f'{len(times)} E+F calls of the unpatched model (e3nn-style materialise-then-index_add conv, '
                      f'einsum symmetric contraction), fp32, {len(st)} atoms, {sec * 1e3:.0f} ms each'}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=300)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--op-reps', type=int, default=20)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-large', action='store_true', help='skip the large-system per-op measurement')
    ap.add_argument('--large-cells', type=int, default=LARGE_CELLS, help='fcc Cu supercell edge of the large case')
    ap.add_argument('--profile', choices=['step', 'ops', 'gemm'], default=None,
                    help='run only the region to profile between cudaProfilerStart/Stop (for ncu '
                         '--profile-from-start off): three replays of the graphed E+F step, one launch of every '
                         'large-system op, or the radial MLP last-layer GEMM at the configs[1] layer-2 shapes')
    ap.add_argument('--partitioned', action='store_true',
                    help='only the configs[4] run: one bulk Cu system (--part-cells) partitioned by receiving atom over '
                         'the ranks (halo exchange per interaction), strong scaling')
    ap.add_argument('--part-cells', type=int, default=PART_CELLS, help='fcc Cu supercell edge of the partitioned run')
    ap.add_argument('--no-extras', action='store_true',
                    help='skip the configs[2] batch, configs[3] relaxation and configs[4] partitioned measurements')
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))

    if a.impl == 'reference':
        return reference_arm(a, rank, world)
    if a.partitioned:
        return partitioned_arm(a, rank, world, local)

    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)

    torch.manual_seed(0)
    model = standin.make_model(HIDDEN, LMAX, CORR, seed=0, elements=standin.ELEMENTS_PTCOH).to(dev)
    model.requires_grad_(False)                 # inference: frozen weights, as MACE's calculators run the model
    rep = patch_model(model, verbose=False, edge_features=True, linears=True)
    assert not rep['skipped'] and len(rep['patched']) >= 6, rep
    st, host_batch = workload(rank)
    n_atoms, n_edges = len(st), int(host_batch['edge_index'].shape[1])
    tot = torch.tensor([n_atoms, n_edges], dtype=torch.float64, device=dev)
    if dist is not None:                            # every rank has its own structure: the job total is the sum
        dist.all_reduce(tot)
    atoms_total, edges_total = int(tot[0].item()), int(tot[1].item())
    batch = standin.to_device(host_batch, dev)
    flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)   # 2x L2, between steps
    e_all = torch.zeros(world, device=dev)

    # eager E+F (for reference in the JSON line), then the CUDA-graphed E+F that is timed
    for _ in range(a.warmup):
        e_and_f(model, batch)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        e_and_f(model, batch)
    torch.cuda.synchronize()
    eager_ms = (time.perf_counter() - t0) / 5 * 1e3
    graphed = GraphedEnergyForces(model, batch)
    if a.profile == 'step':
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for _ in range(3):
            graphed()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        convs = [{'layer': f'conv_tp[{k}]', 'N': n_atoms, 'E': n_edges, 'layer_dims': layer_dims(blk.conv_tp.spec)}
                 for k, blk in enumerate(model.interactions)]
        print(json.dumps({'profile': 'step', 'conv_launch_order': 'per replay: conv_tp[0] fwd, conv_tp[1] fwd, '
                          'conv_tp[1] bwd, conv_tp[0] bwd', 'convs': convs}))
        return
    if a.profile == 'gemm':
        return profile_gemm(dev)
    if a.profile == 'ops':
        cases, info = large_cases(dev, a.large_cells)
        for c in cases:                              # warm (module load, CSR) outside the profiled region
            c['fwd']()
            c['bwd']()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for c in cases:
            c['fwd']()
            c['bwd']()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        info['launch_order'] = [f"{c['op']} {t}" for c in cases for t in ('fwd', 'bwd')]
        info['convs'] = [{'layer': c['op'].split()[0], 'N': c['N'], 'E': c['E'], 'layer_dims': c['dims']}
                         for c in cases if c['kind'] == 'conv']
        print(json.dumps(info))
        return

    def step(b=None):
        E, F = graphed(b)
        if dist is not None:
            dist.all_gather_into_tensor(e_all, E.reshape(1))
        return E, F

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()

    # ---- device-resident inputs -------------------------------------------------------------------------------
    _lib.LAUNCHES.clear()
    evs = []
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        for _ in range(a.steps):
            flush_l2(flush_buf)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    launches = graphed.kernels_per_replay * a.steps
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / a.steps
    ms_t = torch.tensor([ms], device=dev)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())

    # ---- end to end through the public API with host buffers ----------------------------------------------------
    pinned = {k: (v.pin_memory() if torch.is_tensor(v) else v) for k, v in host_batch.items()}
    h2d = sum(v.numel() * v.element_size() for v in pinned.values() if torch.is_tensor(v))
    forces_host = torch.empty(n_atoms, 3).pin_memory()
    d2h = forces_host.numel() * 4 + 4
    evs = []
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    for _ in range(a.steps):
        flush_l2(flush_buf)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        E, F = step(pinned)                  # H2D copies of the pinned inputs into the graph's static inputs, replay
        forces_host.copy_(F, non_blocking=True)
        e_host = E.detach().to('cpu', non_blocking=True)
        e1.record()
        evs.append((e0, e1))
        e1.synchronize()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms_e2e = sum(e0.elapsed_time(e1) for e0, e1 in evs) / a.steps
    t = torch.tensor([ms_e2e], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_e2e = float(t.item())

    # ---- per-op kernel timing (dominant kernel -> roofline) -----------------------------------------------------
    big_flush = torch.empty(1024 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush = lambda: flush_l2(big_flush)
    ops = time_cases(step_cases(model, batch), a.op_reps, flush)
    other_ops = time_cases(other_cases(model, batch), max(3, a.op_reps // 2), flush)
    breakdown = step_breakdown(ops, other_ops)
    hbm, hbm_kind = peaks()

    def conv_roof(o, note, traffic=None):
        b = o['fwd_bytes'] + o['bwd_bytes']
        us = o['fwd_us'] + o['bwd_us']
        ach = b / (us * 1e-6) / 1e9
        r = {'kernel': f"{o['op']} fwd+bwd (mmk_conv_fwd_kernel + mmk_conv_bwd_kernel), N={o['N']} E={o['E']}",
             'bound': 'hbm', 'achieved': round(ach, 1), 'peak': hbm, 'peak_kind': hbm_kind, 'unit': 'GB/s',
             'frac': round(ach / hbm, 4), 'traffic': None, 'algorithmic_bytes_per_launch': b,
             'us_per_launch': round(us, 2), 'note': note}
        if traffic is not None:
            r.update(traffic=int(traffic[0]), traffic_source=traffic[1],
                     traffic_over_algorithmic=round(traffic[0] / b, 3))
        return r

    pair = ('mmk_conv_fwd_kernel', 'mmk_conv_bwd_kernel')
    dom = max((o for o in ops if o['kind'] == 'conv'), key=lambda o: o['fwd_us'] + o['bwd_us'])
    roofline = conv_roof(dom, 'the hot path\'s dominant kernel in the timed E+F step (the conv layer with the '
                              'longest forward + backward); its data fits in L2, so it is latency-bound (cold: L2 '
                              'flushed before the launch).  The largest library share of the step is named in '
                              'step_breakdown.top',
                         traffic=measured_traffic(pair, dom['N'], dom['E'], dom['_dims']))
    large, roof_large, fp32 = None, None, None
    if not a.no_large and rank == 0:
        cases, info = large_cases(dev, a.large_cells)
        with ClockSampler(local) as clk_large:
            large_ops = time_cases(cases, max(3, a.op_reps // 4), flush)
        large = dict(info, ops=large_ops, clocks=clk_large.summary())
        del cases
        big = max((o for o in large['ops'] if o['kind'] == 'conv'), key=lambda o: o['fwd_us'] + o['bwd_us'])
        roof_large = conv_roof(big, 'inputs far larger than L2 (bulk Cu, configs[4] architecture)',
                               traffic=measured_traffic(pair, big['N'], big['E'], big['_dims']))
        fp32 = fp32_peak(dev)
        for o in large['ops'] + ops:
            if o['kind'] == 'sc':
                o['fp32_peak_tflops'] = round(fp32, 1)
                for tag in ('fwd', 'bwd'):          # executed work against the measured FP32 peak
                    o[f'{tag}_exec_frac_of_fp32_peak'] = round(o[f'{tag}_exec_tflops'] / fp32, 4)

    extras = {}
    if not a.no_extras:
        del graphed
        torch.cuda.empty_cache()
        extras['batch16'] = measure_batch16(dev, rank, world, dist, local)
        extras['partitioned'] = measure_partitioned(dev, rank, world, dist, local, a.part_cells)
        if world == 1:                              # one structure: not sharded, measured on a single GPU
            extras['relax89'] = measure_relax89(dev, local)

    if rank == 0:
        cpu = None
        if world == 1 and not a.no_cpu_baseline:
            cpu = cpu_baseline()
        res = {
            'metric': METRIC, 'value': round(atoms_total / (ms * 1e-3), 1), 'unit': UNIT, 'n_gpus': world,
            'steps': a.steps, 'warmup': a.warmup, 'ms_per_step': round(ms, 4), 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic (seeded structures, '
            'random-init weights of the configs[1] architecture)',
            'config': config_dict(atoms_total, edges_total, world),
            'e2e': {'value': round(atoms_total / (ms_e2e * 1e-3), 1), 'unit': UNIT, 'h2d_bytes_per_step': h2d,
                    'd2h_bytes_per_step': d2h, 'ms_per_step': round(ms_e2e, 4)},
            'roofline': roofline, 'cpu_baseline': cpu, 'gpu_launches': launches, 'clocks': clk.summary(),
            'eager_ms_per_step': round(eager_ms, 3),
            'ops': [rounded(o) for o in ops],
            'step_breakdown': breakdown,
            'ops_other': [rounded(o) for o in other_ops],
            'roofline_large': roof_large,
            'ops_large': None if large is None else dict(large, ops=[rounded(o) for o in large['ops']]),
        }
        res.update(extras)
        print(json.dumps(res))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def timed_steps(step, steps, warmup, dev, dist, local):
    """``warmup`` untimed calls, then ``steps`` calls each bracketed by CUDA events, with a barrier and a device
    synchronisation on both sides; returns (mean ms per step, max over ranks; clock summary)."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = []
    with ClockSampler(local) as clk:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    return max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps, dev, dist), clk.summary()


def max_over_ranks(v, dev, dist):
    t = torch.tensor([float(v)], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v, dev, dist):
    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t)
    return float(t.item())


PART_CELLS = 16
PART_ELEMENTS = [29, 30, 31, 32]


def measure_partitioned(dev, rank, world, dist, local, cells=PART_CELLS, steps=10, warmup=3):
    """configs[4]-style strong scaling: one bulk fcc Cu system of cells^3 conventional cells (128x0e+128x1o+128x2e,
    l_max 3, correlation 3, r_max 5 A, every patch option, frozen weights) partitioned over the ranks by receiving
    atom (mace_mps_kernels_b200.distributed); per interaction one halo all_to_all forward and one reverse in the
    backward.  Eager steps (the collectives sit inside autograd), CUDA events, max over ranks; value = all atoms /
    step time.  Also the time spent inside the halo collectives and the bytes they move."""
    from mace_mps_kernels_b200.distributed import COMM, DistributedMACE, partition_graph
    torch.manual_seed(0)
    model = standin.make_model('128x0e+128x1o+128x2e', 3, 3, seed=0, elements=PART_ELEMENTS).to(dev)
    model.requires_grad_(False)
    rep = patch_model(model, verbose=False, edge_features=True, linears=True)
    assert not rep['skipped'], rep
    st = standin.fcc_bulk('Cu', 3.61, cells, seed=0, jitter=0.1)
    t0 = time.perf_counter()
    parts = partition_graph(st, RMAX, world)
    part_s = time.perf_counter() - t0
    part = parts[rank]
    dm = DistributedMACE(model, part, st.positions, PART_ELEMENTS, dev)
    e_tot = torch.zeros(1, device=dev)

    def step():
        E, F = dm.energy_forces()
        e_tot.copy_(E.detach().reshape(1))
        if dist is not None:
            dist.all_reduce(e_tot)
        return F

    ms, clocks = timed_steps(step, steps, warmup, dev, dist, local)
    COMM.enabled = True                             # one more step, metered (not part of the timed steps)
    step()
    torch.cuda.synchronize()
    COMM.enabled = False
    comm_ms, sent, recv, n_x = COMM.summary()
    comm_ms = max_over_ranks(comm_ms, dev, dist)
    halo = max_over_ranks(len(part.halo), dev, dist)
    sent = max_over_ranks(sent, dev, dist)
    n_edges = sum(p.edge_index.shape[1] for p in parts)
    res = {'metric': 'E+F atom-steps/s (partitioned large system)', 'value': round(len(st) / (ms * 1e-3), 1),
           'unit': UNIT, 'n_gpus': world, 'ms_per_step': round(ms, 3), 'scaling': 'strong', 'steps': steps,
           'warmup': warmup,
           'config': {'workload': f'configs[4]: MACE 128x0e+128x1o+128x2e l_max 3 corr 3, fcc Cu {cells}^3 cells, '
                                  f'{len(st)} atoms, {n_edges} edges, partitioned by receiving atom over {world} '
                                  f'rank(s)',
                      'owned_atoms_per_rank': len(part.owned), 'max_halo_atoms': int(halo),
                      'patched': ', '.join(rep['patched'][:4]) + ', ... (every patch option)',
                      'parallelism': f'domain decomposition, {world} rank(s), NCCL all_to_all_single halo exchange',
                      'timing': 'eager E+F steps (no CUDA graph), CUDA events, max over ranks'},
           'halo_exchange': {'collective': 'all_to_all_single (NCCL), 2 forward + 2 reverse per step',
                             'exchanges_per_step': n_x, 'ms_per_step_max_rank': round(comm_ms, 3),
                             'bytes_sent_per_step_max_rank': int(sent),
                             'share_of_step': round(comm_ms / ms, 4) if world > 1 else 0.0},
           'partition_build_s': round(part_s, 2), 'clocks': clocks}
    del dm, model
    torch.cuda.empty_cache()
    return res


def measure_batch16(dev, rank, world, dist, local, steps=20, warmup=3):
    """16 structures of the configs[0] slab generator (Pt(100) 4x4x4 + 5 CO + 5 H, seeds 0..15) with the
    32-channel model, each padded to 6 000 edges; rank r evaluates structures r, r+N, ... as one batched, CUDA-graphed
    E+F call; the only collective is the energy gather.  value = all atoms / step time (max over ranks)."""
    from mace_mps_kernels_b200.distributed import gather_energies
    model = standin.make_model('32x0e+32x1o', 3, 3, seed=0, elements=standin.ELEMENTS_PTCOH).to(dev)
    model.requires_grad_(False)
    patch_model(model, verbose=False, edge_features=True, linears=True)
    mine = list(range(rank, 16, world))
    sts = [standin.pt100_co_h(seed=s) for s in mine]
    batch = standin.to_device(standin.structure_batch(sts, standin.ELEMENTS_PTCOH, RMAX, pad_to=6000), dev)
    graphed = GraphedEnergyForces(model, batch)

    def step():
        E, _ = graphed()
        if dist is not None:
            gather_energies(E.sum(), world)
        return E

    ms, clocks = timed_steps(step, steps, warmup, dev, dist, local)
    atoms = sum_over_ranks(sum(len(s) for s in sts), dev, dist)
    res = {'metric': 'E+F atom-steps/s (batch of 16 structures)', 'value': round(atoms / (ms * 1e-3), 1),
           'unit': UNIT, 'ms_per_step': round(ms, 3), 'ms_per_structure_per_gpu': round(ms / max(1, len(mine)), 4),
           'structures_per_rank_max': len(mine), 'steps': steps, 'warmup': warmup,
           'config': {'workload': 'configs[2]: 16 x (Pt(100) 4x4x4 + 5 CO + 5 H, 79 atoms), padded to 6000 edges each; '
                                  'MACE 32x0e+32x1o l_max 3 corr 3, every patch option, CUDA-graphed',
                      'atoms_total': int(atoms), 'parallelism': f'structure batch over {world} rank(s)'},
           'clocks': clocks}
    del graphed, model
    torch.cuda.empty_cache()
    return res


def measure_relax89(dev, local, calls=50):
    """the 89-element model (128x0e+128x1o, r_max 6 A) on CeO2(111) + Au13, an L-BFGS loop of ``calls``
    E+F calls at a fixed padded graph (device neighbour list, CUDA-graphed E+F, optimiser on the device), against the
    same loop on the unpatched model (eager) for the energies."""
    from mace_mps_kernels_b200.relax import Relaxation, ceo2_au13_workload
    model, st, z_table, cap = ceo2_au13_workload(dev)
    met = copy.deepcopy(model)
    patch_model(met, verbose=False, edge_features=True, linears=True)
    Relaxation(met, st, z_table, 6.0, dev, cap).run(3)                      # warm-up (compilation, allocations)
    relax = Relaxation(met, st, z_table, 6.0, dev, cap)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        energies, _ = relax.run(calls)
        e1.record()
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    ref_e, _ = Relaxation(model, st, z_table, 6.0, dev, cap, graphed=False).run(calls)
    dE = (energies - ref_e).abs()
    res = {'metric': 'E+F atom-steps/s (L-BFGS loop, 89-element model)', 'value': round(len(st) * calls / (ms * 1e-3), 1),
           'unit': UNIT, 'ms_per_call': round(ms / calls, 4), 'calls': calls,
           'energy_first_last_eV': [round(float(energies[0]), 6), round(float(energies[-1]), 6)],
           'max_abs_dE_vs_unpatched_loop_eV': float(dE.max()),
           'config': {'workload': f'configs[3]: MACE 128x0e+128x1o l_max 3 corr 3, 89 elements (Z 1-89), r_max 6 A; '
                                  f'CeO2(111) 4x4 x 3 trilayers + Au13, {len(st)} atoms, padded to {cap} edges',
                      'loop': 'L-BFGS (memory 100, maxstep 0.2 A), device neighbour list, CUDA-graphed E+F',
                      'timing': 'CUDA events around the whole loop (includes the optimiser and neighbour list)'},
           'clocks': clk.summary()}
    del relax, met, model
    torch.cuda.empty_cache()
    return res


def partitioned_arm(a, rank, world, local):
    """--partitioned: only the configs[4] partitioned measurement, printed as its own line."""
    import datetime
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=dev)
    res = measure_partitioned(dev, rank, world, dist, local, a.part_cells, a.steps, a.warmup)
    if rank == 0:
        res.update(higher_is_better=True, dtype='f32', data='synthetic (seeded bulk Cu)')
        print(json.dumps(res))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def rounded(o):
    return {k: (round(v, 2) if isinstance(v, float) else v) for k, v in o.items() if not k.startswith('_')}


def reference_arm(a, rank, world):
    """The reference's path on the host cores: the unpatched e3nn-path model, E+F on the same workload (rank 0)."""
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    model = standin.make_model(HIDDEN, LMAX, CORR, seed=0, elements=standin.ELEMENTS_PTCOH).requires_grad_(False)
    st, batch = workload(0)
    for _ in range(a.warmup):
        e_and_f(model, batch)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        e_and_f(model, batch)
    sec = (time.perf_counter() - t0) / a.steps
    v = round(len(st) / sec, 2)
    res = {'impl': 'reference', 'metric': METRIC, 'value': v, 'unit': UNIT, 'n_gpus': world, 'steps': a.steps,
           'warmup': a.warmup, 'ms_per_step': round(sec * 1e3, 3), 'higher_is_better': True, 'scaling': 'weak',
           'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
           'config': config_dict(len(st), int(batch['edge_index'].shape[1]), 1),
           'cpu_baseline': {'value': v, 'unit': UNIT, 'cores': cores, 'kind': 'port',
                            'sample': f'one E+F call of the unpatched e3nn-path model per step, {len(st)} atoms'},
           'e2e': {'value': v, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(res))


if __name__ == '__main__':
    main()
