"""Periodic neighbour lists and MACE-style graph batches (what mace's ``AtomicData`` / ``Batch`` carry).

Edges follow matscipy/ASE ``neighbour_list('ijS')`` semantics as MACE uses them: ``edge_index = [sender i,
receiver j]``, ``shifts = S @ cell`` and the edge vector is ``positions[j] - positions[i] + shifts``; every pair
(i, j, S) with 0 < |vector| < r_max is listed, so the graph holds both directions.  Edges are sorted by (i, j, S).
"""
from __future__ import annotations

import itertools

import numpy as np
import torch


def neighbor_list(positions, cell, pbc, cutoff, chunk=1 << 16):
    """(i, j, S) arrays of all pairs with |r_j + S.cell - r_i| < cutoff (cell-list search, float64)."""
    pos = np.asarray(positions, np.float64)
    cell = np.asarray(cell, np.float64)
    pbc = np.asarray(pbc, bool)
    N = len(pos)
    inv = np.linalg.inv(cell)
    frac = pos @ inv
    shift0 = np.where(pbc, np.floor(frac), 0.0)
    fw = frac - shift0
    posw = fw @ cell
    vol = abs(np.linalg.det(cell))
    heights = np.array([vol / np.linalg.norm(np.cross(cell[(a + 1) % 3], cell[(a + 2) % 3])) for a in range(3)])
    nrep = np.where(pbc, np.ceil(cutoff / heights).astype(int), 0)
    margin = cutoff / heights
    img_pos, img_j, img_S = [], [], []
    for S in itertools.product(*[range(-n, n + 1) for n in nrep]):
        S = np.array(S, float)
        f = fw + S
        keep = np.all((f > -margin - 1e-9) & (f < 1 + margin + 1e-9) | ~pbc, axis=1)
        idx = np.nonzero(keep)[0]
        img_pos.append(posw[idx] + S @ cell)
        img_j.append(idx)
        img_S.append(np.repeat(S[None], len(idx), 0))
    img_pos = np.concatenate(img_pos)
    img_j = np.concatenate(img_j)
    img_S = np.concatenate(img_S)
    lo = img_pos.min(0) - 1e-6
    nb = np.maximum(1, np.floor((img_pos.max(0) - lo) / cutoff).astype(int))
    binsz = (img_pos.max(0) - lo) / nb + 1e-9

    def bin3(p):
        return np.clip(np.floor((p - lo) / binsz).astype(int), 0, nb - 1)

    ib = bin3(img_pos)
    lin = (ib[:, 0] * nb[1] + ib[:, 1]) * nb[2] + ib[:, 2]
    order = np.argsort(lin, kind='stable')
    lin_sorted = lin[order]
    cb = bin3(posw)
    out_i, out_j, out_S = [], [], []
    for c0 in range(0, N, chunk):
        ci = np.arange(c0, min(N, c0 + chunk))
        for off in itertools.product((-1, 0, 1), repeat=3):
            b = cb[ci] + off
            ok = np.all((b >= 0) & (b < nb), axis=1)
            li = (b[:, 0] * nb[1] + b[:, 1]) * nb[2] + b[:, 2]
            st = np.searchsorted(lin_sorted, li, 'left')
            en = np.searchsorted(lin_sorted, li, 'right')
            cnt = np.where(ok, en - st, 0)
            tot = int(cnt.sum())
            if tot == 0:
                continue
            ii = np.repeat(ci, cnt)
            first = np.repeat(np.cumsum(cnt) - cnt, cnt)
            kk = order[np.repeat(st, cnt) + (np.arange(tot) - first)]
            d = img_pos[kk] - posw[ii]
            r2 = (d * d).sum(1)
            m = (r2 < cutoff * cutoff) & ~((img_j[kk] == ii) & np.all(img_S[kk] == 0, axis=1))
            out_i.append(ii[m])
            out_j.append(img_j[kk[m]])
            out_S.append(img_S[kk[m]])
    if not out_i:
        return np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros((0, 3), np.int64)
    i = np.concatenate(out_i)
    j = np.concatenate(out_j)
    S = np.concatenate(out_S) - shift0[j] + shift0[i]
    S = np.rint(S).astype(np.int64)
    o = np.lexsort((S[:, 2], S[:, 1], S[:, 0], j, i))
    return i[o], j[o], S[o]


def atoms_to_graph(st, z_table, r_max, dtype=torch.float32):
    """One structure -> dict of tensors with MACE's keys (CPU)."""
    i, j, S = neighbor_list(st.positions, st.cell, st.pbc, r_max)
    z_index = {z: k for k, z in enumerate(z_table)}
    idx = torch.tensor([z_index[int(z)] for z in st.numbers])
    return {
        'positions': torch.tensor(st.positions, dtype=dtype),
        'node_attrs': torch.nn.functional.one_hot(idx, len(z_table)).to(dtype),
        'edge_index': torch.from_numpy(np.stack([i, j])).long(),
        'shifts': torch.from_numpy(S.astype(np.float64) @ st.cell).to(dtype),
        'cell': torch.tensor(st.cell, dtype=dtype),
        'num_nodes': len(st),
    }


def pad_edges(g, n_edges, far=1.0e3):
    """Pad a graph to exactly ``n_edges`` with self-edges shifted by ``far`` A (beyond any cutoff), padding edge k on
    node k mod N (spread over the nodes, so that no node's CSR segment grows with the padding).

    A padding edge has a finite direction (harmonics are defined) and a length past r_max, so the polynomial cutoff
    makes its radial features, its per-edge weights and hence its message and every gradient through it exactly 0."""
    E = g['edge_index'].shape[1]
    if E > n_edges:
        raise ValueError(f'graph has {E} edges > pad size {n_edges}')
    if E == n_edges:
        return g
    k = n_edges - E
    g = dict(g)
    v = torch.arange(k, dtype=torch.long) % max(int(g['num_nodes']), 1)
    g['edge_index'] = torch.cat([g['edge_index'], torch.stack([v, v])], 1)
    pad = torch.zeros(k, 3, dtype=g['shifts'].dtype)
    pad[:, 0] = far
    g['shifts'] = torch.cat([g['shifts'], pad], 0)
    return g


def collate(graphs):
    """Concatenate graphs into one batch (node offsets applied to edge_index), as torch_geometric's Batch does."""
    pos, attrs, ei, sh, batch, ptr = [], [], [], [], [], [0]
    off = 0
    for k, g in enumerate(graphs):
        n = g['num_nodes']
        pos.append(g['positions'])
        attrs.append(g['node_attrs'])
        ei.append(g['edge_index'] + off)
        sh.append(g['shifts'])
        batch.append(torch.full((n,), k, dtype=torch.long))
        off += n
        ptr.append(off)
    return {
        'positions': torch.cat(pos), 'node_attrs': torch.cat(attrs), 'edge_index': torch.cat(ei, 1),
        'shifts': torch.cat(sh), 'batch': torch.cat(batch), 'ptr': torch.tensor(ptr), 'num_graphs': len(graphs),
    }


def to_device(batch, device):
    return {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in batch.items()}
