"""Multi-GPU checks (skipped with fewer than two CUDA devices): one process per GPU over NCCL.

* the partitioned large-system evaluation (receiver-owned edges, halo exchange before every interaction, reverse halo
  in the backward) running the patched kernels on each rank's local graph reproduces the single-GPU energy and forces,
  with the reference's model-level tolerances (|dE|/atom < 1e-5 eV, max|dF| / max|F| < 1e-5);
* the structure-batch energy gather returns every rank's energy.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mace_mps_kernels_b200 import patch_model
from mace_mps_kernels_b200 import standin as S

pytestmark = pytest.mark.gpu

HIDDEN, LMAX, CORR = '64x0e+64x1o', 3, 3
ELEMENTS = [29, 30, 31, 32]


def _need_gpus(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f'needs {n} CUDA devices')


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _structure():
    st = S.fcc_bulk('Cu', 3.61, 4, seed=3, jitter=0.1)          # 256 atoms, periodic
    st.numbers = np.where(np.arange(len(st)) % 5 == 0, 30, 29)   # two elements, so the SC element groups matter
    return st


def _worker(rank, world, port, out_dir, model):
    import torch.distributed as dist
    from mace_mps_kernels_b200.distributed import DistributedMACE, gather_energies, partition_graph
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dev = torch.device('cuda', rank)
    torch.cuda.set_device(dev)
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        model = model.to(dev)
        rep = patch_model(model, verbose=False)
        st = _structure()
        parts = partition_graph(st, 5.0, world)
        dm = DistributedMACE(model, parts[rank], st.positions, ELEMENTS, dev)
        E, F = dm.energy_forces()
        Ein = E.detach().clone()
        es = gather_energies(Ein, world)
        Etot = Ein.clone()
        dist.all_reduce(Etot)
        torch.cuda.synchronize()
        torch.save({'owned': parts[rank].owned, 'F': F.detach().cpu(), 'E': float(Etot), 'E_rank': float(Ein),
                    'gathered': es.cpu(), 'patched': len(rep['patched'])}, os.path.join(out_dir, f'{rank}.pt'))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2])
def test_partitioned_patched_energy_forces_match_single_gpu(tmp_path, world):
    _need_gpus(world)
    torch.manual_seed(0)
    model = S.make_model(HIDDEN, LMAX, CORR, seed=0, elements=ELEMENTS)
    ref = S.make_model(HIDDEN, LMAX, CORR, seed=0, elements=ELEMENTS).to('cuda:0')
    patch_model(ref, verbose=False)
    st = _structure()
    b = S.to_device(S.structure_batch([st], ELEMENTS, 5.0), torch.device('cuda', 0))
    b['positions'] = b['positions'].detach().requires_grad_(True)
    out = ref(b, compute_force=True, training=False)
    E0, F0 = float(out['energy'].sum()), out['forces'].detach().cpu().numpy()
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), model), nprocs=world, join=True)
    seen = np.zeros(len(st), bool)
    e_ranks = []
    for r in range(world):
        res = torch.load(os.path.join(tmp_path, f'{r}.pt'), weights_only=False)
        assert res['patched'] == 4
        assert abs(res['E'] - E0) / len(st) < 1e-5, (res['E'], E0)
        owned = np.asarray(res['owned'])
        dF = np.abs(res['F'].numpy() - F0[owned]).max()
        assert dF / np.abs(F0).max() < 1e-5, dF
        seen[owned] = True
        e_ranks.append(res['E_rank'])
    assert seen.all()
    g = torch.load(os.path.join(tmp_path, '0.pt'), weights_only=False)['gathered'].numpy()
    assert np.allclose(g, np.asarray(e_ranks), rtol=0, atol=0)
