"""Synthetic structures for the benchmark configurations (ASE is not installed; these are built with numpy).

* ``pt100_co_h``      Pt(100) slab 4x4 cells x 4 layers (a = 3.92 A, 64 Pt) + 5 atop CO (C 1.85 A above Pt, O 1.15 A
                      above C) + 5 hollow H, 15 A vacuum, periodic in x/y, jitter N(0, 0.05 A)       (79 atoms)
* ``pt100_random``    Pt(100) 6x6 cells x 4 layers (144 Pt) + seeded CO/O/H on atop/bridge/hollow sites (140-181 atoms)
* ``ceo2_au13``       CeO2(111) 3 O-Ce-O trilayers, 4x4 surface cells (a = 5.41 A) + Au13 cuboctahedron (157 atoms)
* ``fcc_bulk``        bulk fcc supercell (Cu 30^3 conventional cells = 108 000 atoms, a = 3.61 A), jitter N(0, 0.1 A)
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SYMBOLS = ['X', 'H', 'He', 'Li', 'Be', 'B', 'C', 'N', 'O', 'F', 'Ne', 'Na', 'Mg', 'Al', 'Si', 'P', 'S', 'Cl', 'Ar', 'K',
           'Ca', 'Sc', 'Ti', 'V', 'Cr', 'Mn', 'Fe', 'Co', 'Ni', 'Cu', 'Zn', 'Ga', 'Ge', 'As', 'Se', 'Br', 'Kr', 'Rb',
           'Sr', 'Y', 'Zr', 'Nb', 'Mo', 'Tc', 'Ru', 'Rh', 'Pd', 'Ag', 'Cd', 'In', 'Sn', 'Sb', 'Te', 'I', 'Xe', 'Cs',
           'Ba', 'La', 'Ce', 'Pr', 'Nd', 'Pm', 'Sm', 'Eu', 'Gd', 'Tb', 'Dy', 'Ho', 'Er', 'Tm', 'Yb', 'Lu', 'Hf', 'Ta',
           'W', 'Re', 'Os', 'Ir', 'Pt', 'Au', 'Hg', 'Tl', 'Pb', 'Bi', 'Po', 'At', 'Rn', 'Fr', 'Ra', 'Ac']
Z = {s: i for i, s in enumerate(SYMBOLS)}


@dataclass
class Structure:
    positions: np.ndarray                  # [N, 3] float64, Angstrom
    numbers: np.ndarray                    # [N] int atomic numbers
    cell: np.ndarray                       # [3, 3] rows are lattice vectors
    pbc: np.ndarray = field(default_factory=lambda: np.array([True, True, True]))

    def __len__(self):
        return len(self.numbers)

    def copy(self):
        return Structure(self.positions.copy(), self.numbers.copy(), self.cell.copy(), self.pbc.copy())

    def rotated(self, R):
        return Structure(self.positions @ R.T, self.numbers.copy(), self.cell @ R.T, self.pbc.copy())

    def permuted(self, perm):
        perm = np.asarray(perm)
        return Structure(self.positions[perm].copy(), self.numbers[perm].copy(), self.cell.copy(), self.pbc.copy())


def morton_order(positions, cell, bits=10):
    """Permutation sorting atoms along a Z-order (Morton) curve of their fractional coordinates.

    Atoms close in space get close indices, so the rows a block of receivers gathers from its neighbours overlap
    and stay in L2 while the convolution streams the per-edge weights."""
    f = np.asarray(positions, np.float64) @ np.linalg.inv(np.asarray(cell, np.float64))
    f = f - np.floor(f.min(0))
    f = f / max(f.max(), 1e-12)
    q = np.minimum((f * (1 << bits)).astype(np.int64), (1 << bits) - 1)
    code = np.zeros(len(q), np.int64)
    for b in range(bits):
        for ax in range(3):
            code |= ((q[:, ax] >> b) & 1) << (3 * b + ax)
    return np.argsort(code, kind='stable')


def fcc100_slab(symbol, a, nx, ny, nlayers, vacuum):
    """Square (100) surface cells of side a/sqrt2; layer k at z = k a/2, odd layers shifted by half a cell."""
    s = a / np.sqrt(2.0)
    pos = []
    for k in range(nlayers):
        off = 0.5 * s if k % 2 else 0.0
        for i in range(nx):
            for j in range(ny):
                pos.append([i * s + off, j * s + off, k * a / 2.0])
    pos = np.array(pos)
    cell = np.diag([nx * s, ny * s, (nlayers - 1) * a / 2.0 + vacuum])
    return Structure(pos, np.full(len(pos), Z[symbol]), cell, np.array([True, True, False]))


def _top_layer(slab):
    z = slab.positions[:, 2]
    return np.where(z > z.max() - 0.1)[0]


def _sites_100(slab, a):
    """atop / bridge / hollow sites (xy) of an fcc(100) top layer, with the top z."""
    s = a / np.sqrt(2.0)
    top = slab.positions[_top_layer(slab)]
    ztop = top[:, 2].max()
    atop = top[:, :2]
    bridge = np.concatenate([atop + [0.5 * s, 0.0], atop + [0.0, 0.5 * s]])
    hollow = atop + [0.5 * s, 0.5 * s]
    return {'atop': atop, 'bridge': bridge, 'hollow': hollow}, ztop


_ADS_HEIGHT = {('CO', 'atop'): 1.85, ('CO', 'bridge'): 1.45, ('CO', 'hollow'): 1.25,
               ('O', 'atop'): 1.75, ('O', 'bridge'): 1.35, ('O', 'hollow'): 1.05,
               ('H', 'atop'): 1.55, ('H', 'bridge'): 1.1, ('H', 'hollow'): 0.95}


def _add(st, pos, nums):
    return Structure(np.concatenate([st.positions, np.asarray(pos, float).reshape(-1, 3)]),
                     np.concatenate([st.numbers, np.asarray(nums, int)]), st.cell.copy(), st.pbc.copy())


def _min_image_dist_xy(p, q, cell):
    d = p - q
    for ax in range(2):
        L = cell[ax, ax]
        d[..., ax] -= L * np.round(d[..., ax] / L)
    return np.linalg.norm(d, axis=-1)


def pt100_co_h(seed=0, jitter=0.05):
    """Configuration 1: 64 Pt + 5 atop CO + 5 hollow H (79 atoms)."""
    a = 3.92
    rng = np.random.default_rng(seed)
    slab = fcc100_slab('Pt', a, 4, 4, 4, 15.0)
    sites, ztop = _sites_100(slab, a)
    atop = rng.choice(len(sites['atop']), 5, replace=False)
    st = slab
    for i in atop:
        x, y = sites['atop'][i]
        st = _add(st, [[x, y, ztop + 1.85], [x, y, ztop + 1.85 + 1.15]], [Z['C'], Z['O']])
    hol = sites['hollow']
    chosen = []
    for i in rng.permutation(len(hol)):
        if len(chosen) == 5:
            break
        d = _min_image_dist_xy(hol[i][None], sites['atop'][atop], slab.cell).min()
        if d > 1.9 and all(_min_image_dist_xy(hol[i], hol[j], slab.cell) > 2.0 for j in chosen):
            chosen.append(i)
    for i in chosen:
        st = _add(st, [[hol[i][0], hol[i][1], ztop + _ADS_HEIGHT['H', 'hollow']]], [Z['H']])
    st.positions = st.positions + rng.normal(0, jitter, st.positions.shape)
    return st


def pt100_random(seed=0, jitter=0.05, nx=6, ny=6, nlayers=4):
    """Configuration 2: Pt(100) 6x6x4 (144 Pt) + seeded CO/O/H on random atop/bridge/hollow sites (140-181 atoms)."""
    a = 3.92
    rng = np.random.default_rng(seed)
    slab = fcc100_slab('Pt', a, nx, ny, nlayers, 15.0)
    sites, ztop = _sites_100(slab, a)
    n_ads = int(rng.integers(10, 19))
    st, placed = slab, []
    tries = 0
    while len(placed) < n_ads and tries < 5000:
        tries += 1
        kind = ['atop', 'bridge', 'hollow'][rng.integers(3)]
        mol = ['CO', 'O', 'H'][rng.integers(3)]
        xy = sites[kind][rng.integers(len(sites[kind]))]
        if any(_min_image_dist_xy(xy, q, slab.cell) < 2.6 for q in placed):
            continue
        placed.append(xy)
        h = ztop + _ADS_HEIGHT[mol, kind]
        if mol == 'CO':
            st = _add(st, [[xy[0], xy[1], h], [xy[0], xy[1], h + 1.15]], [Z['C'], Z['O']])
        else:
            st = _add(st, [[xy[0], xy[1], h]], [Z[mol]])
    st.positions = st.positions + rng.normal(0, jitter, st.positions.shape)
    return st


def ceo2_au13(seed=0, jitter=0.05, a=5.41, n=4, trilayers=3):
    """Configuration 4: CeO2(111), 3 O-Ce-O trilayers of n x n hexagonal cells, plus an Au13 cuboctahedron 2.4 A above.

    Fluorite along [111]: Ce planes every h = a/sqrt3 in ABC stacking; the O of trilayer k sit at z = kh -/+ h/4 on the
    neighbouring stacking positions (tetrahedral holes), which gives the Ce-O distance a sqrt3/4."""
    rng = np.random.default_rng(seed)
    ahex = a / np.sqrt(2.0)
    h = a / np.sqrt(3.0)
    a1 = np.array([ahex, 0.0, 0.0])
    a2 = np.array([0.5 * ahex, np.sqrt(3.0) / 2 * ahex, 0.0])
    P = [np.zeros(3), (a1 + a2) / 3.0, 2.0 * (a1 + a2) / 3.0]
    pos, nums = [], []
    for k in range(trilayers):
        for i in range(n):
            for j in range(n):
                base = i * a1 + j * a2
                pos.append(base + P[(k - 1) % 3] + [0, 0, k * h - h / 4]); nums.append(Z['O'])
                pos.append(base + P[k % 3] + [0, 0, k * h]); nums.append(Z['Ce'])
                pos.append(base + P[(k + 1) % 3] + [0, 0, k * h + h / 4]); nums.append(Z['O'])
    pos = np.array(pos)
    pos[:, 2] += 8.0
    ztop = pos[:, 2].max()
    cell = np.array([n * a1, n * a2, [0.0, 0.0, ztop + 8.0 + 10.0]])
    d = 2.88 / np.sqrt(2.0)                                            # Au-Au 2.88 A
    cub = [[0, 0, 0]] + [[sx * d, sy * d, 0] for sx in (-1, 1) for sy in (-1, 1)] \
        + [[sx * d, 0, sz * d] for sx in (-1, 1) for sz in (-1, 1)] + [[0, sy * d, sz * d] for sy in (-1, 1) for sz in (-1, 1)]
    cub = np.array(cub, float)
    centre = (cell[0] + cell[1]) / 2.0
    cub += np.array([centre[0], centre[1], ztop + 2.4 - cub[:, 2].min()])
    pos = np.concatenate([pos, cub])
    nums = np.concatenate([nums, np.full(13, Z['Au'])])
    pos = pos + rng.normal(0, jitter, pos.shape)
    return Structure(pos, np.asarray(nums), cell, np.array([True, True, False]))


def fcc_bulk(symbol='Cu', a=3.61, n=30, seed=0, jitter=0.1):
    """Configuration 5: n^3 conventional fcc cells (4 atoms each), periodic, positions jittered N(0, jitter)."""
    rng = np.random.default_rng(seed)
    basis = np.array([[0, 0, 0], [0.5, 0.5, 0], [0.5, 0, 0.5], [0, 0.5, 0.5]])
    g = np.stack(np.meshgrid(np.arange(n), np.arange(n), np.arange(n), indexing='ij'), -1).reshape(-1, 1, 3)
    pos = ((g + basis[None]) * a).reshape(-1, 3)
    pos = pos + rng.normal(0, jitter, pos.shape)
    return Structure(pos, np.full(len(pos), Z[symbol]), np.eye(3) * n * a, np.array([True, True, True]))
