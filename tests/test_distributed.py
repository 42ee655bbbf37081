"""Multi-process tests of the distributed decompositions on CPU (gloo ranks, world size 2 and 3; no GPU needed):

* a system partitioned by receiving atom with halo exchange gives exactly the single-process energy and forces;
* the partition bookkeeping (owned / halo / send lists) is consistent;
* a rank that fails before a collective makes the others fail with an error (short process-group timeout), not hang.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mace_mps_kernels_b200 import standin as S
from mace_mps_kernels_b200.distributed import DistributedMACE, partition_graph


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    return S.make_model('32x0e+32x1o', 3, 3, seed=0, elements=S.ELEMENTS_PTCOH).double()


def _structure():
    return S.pt100_co_h(seed=1)


def _worker(rank, world, port, out_dir, model):
    import datetime
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    st = _structure()
    parts = partition_graph(st, 5.0, world)
    dm = DistributedMACE(model, parts[rank], st.positions, S.ELEMENTS_PTCOH, 'cpu', dtype=torch.float64)
    E, F = dm.energy_forces()
    Etot = E.detach().clone()
    dist.all_reduce(Etot)
    torch.save({'owned': parts[rank].owned, 'F': F.detach(), 'E': float(Etot), 'n_halo': len(parts[rank].halo)},
               os.path.join(out_dir, f'{rank}.pt'))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 3])
def test_partitioned_energy_forces_match_single_process(tmp_path, world):
    st = _structure()
    model = _model()
    b = S.structure_batch([st], S.ELEMENTS_PTCOH, 5.0, dtype=torch.float64)
    out = model(b)
    E0, F0 = float(out['energy'].sum()), out['forces'].detach().numpy()
    # the model is built here and pickled to the ranks: building it in every rank at once oversubscribes the BLAS threads
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), model), nprocs=world, join=True)
    seen = np.zeros(len(st), bool)
    for r in range(world):
        res = torch.load(os.path.join(tmp_path, f'{r}.pt'), weights_only=False)
        assert abs(res['E'] - E0) < 1e-9 * max(1.0, abs(E0))
        owned = np.asarray(res['owned'])
        assert np.abs(res['F'].numpy() - F0[owned]).max() < 1e-9
        assert res['n_halo'] > 0
        seen[owned] = True
    assert seen.all()


def test_partition_bookkeeping():
    st = S.fcc_bulk('Cu', 3.61, 4, seed=0, jitter=0.1)
    world = 4
    parts = partition_graph(st, 5.0, world)
    owners = np.concatenate([p.owned for p in parts])
    assert np.array_equal(np.sort(owners), np.arange(len(st)))
    owner = np.empty(len(st), int)
    for p in parts:
        owner[p.owned] = p.rank
    i, j, _ = S.neighbor_list(st.positions, st.cell, st.pbc, 5.0)
    assert sum(p.edge_index.shape[1] for p in parts) == len(i)
    for p in parts:
        assert (p.edge_index[1] < p.n_own).all()                 # receivers are owned
        assert (p.edge_index[0] < p.n_local).all()
        assert sum(p.recv_counts) == len(p.halo) and p.recv_counts[p.rank] == 0
        for q in parts:                                           # what q receives from p is what p sends to q
            assert q.recv_counts[p.rank] == p.send_counts[q.rank]
        off = np.cumsum([0] + p.send_counts)
        for q in range(world):
            sent = p.owned[p.send_idx[off[q]:off[q + 1]]]
            blk = parts[q].halo[owner[parts[q].halo] == p.rank]
            assert np.array_equal(sent, blk)


def _failing_worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise SystemExit(0)                      # leaves between steps, before the collective
    try:
        x = torch.ones(4)
        dist.all_reduce(x)
        ok = 'no error'
    except Exception as e:                       # noqa: BLE001
        ok = f'error: {type(e).__name__}'
    with open(os.path.join(out_dir, 'rank0.txt'), 'w') as f:
        f.write(ok)


def test_lost_rank_surfaces_as_error(tmp_path):
    ctx = mp.get_context('spawn')
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError('a rank did not finish')
    assert open(os.path.join(tmp_path, 'rank0.txt')).read().startswith('error')
