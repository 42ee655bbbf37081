"""The neighbour-list arithmetic of the CUDA kernels (csrc/neighbors.cuh), compiled for the host and run in the order
the kernels use (wrap and bin every atom, walk the neighbouring (bin, image) pairs of each atom, order each atom's
pairs by (j, S)), against the stand-in's host neighbour list (matscipy / ASE 'ijS' semantics) -- no GPU needed.
Cases: slabs and bulk, a cell thinner than the cutoff (several images per axis), a skewed cell, non-periodic axes
with atoms outside the binned range."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import helpers
from mace_mps_kernels_b200.standin import structures as S_
from mace_mps_kernels_b200.standin.graph import neighbor_list
from mace_mps_kernels_b200.standin.structures import Structure

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'mace_mps_kernels_b200', 'csrc')

DRIVER = r'''
#include <algorithm>
#include <cstdio>
#include <vector>
#define MMK_HD
#include "neighbors.cuh"
// stdin: n, positions[n*3], cell[9], pbc[3] (int), cutoff, lo[3], hi[3] (doubles)
// stdout: m, then per pair i, j, S0, S1, S2 (int) and the float shift vector[3]
int main() {
    int n;
    if (fread(&n, 4, 1, stdin) != 1) return 1;
    std::vector<double> pos(3 * (size_t)n);
    double cell[9], cutoff, lo[3], hi[3];
    int pbc[3];
    if (fread(pos.data(), 8, pos.size(), stdin) != pos.size() || fread(cell, 8, 9, stdin) != 9 ||
        fread(pbc, 4, 3, stdin) != 3 || fread(&cutoff, 8, 1, stdin) != 1 || fread(lo, 8, 3, stdin) != 3 ||
        fread(hi, 8, 3, stdin) != 3)
        return 2;
    MmkNlGeom G;
    if (!mmk_nl_geometry(cell, pbc, cutoff, lo, hi, 1024, G)) return 3;
    const int nbins = G.nb[0] * G.nb[1] * G.nb[2];
    std::vector<double> rw(3 * (size_t)n);
    std::vector<int> s0(3 * (size_t)n), bin(n);
    std::vector<std::vector<int>> members(nbins);
    for (int i = 0; i < n; ++i) {
        int b[3];
        nl_wrap(&pos[3 * i], G, &rw[3 * i], &s0[3 * i], b);
        bin[i] = nl_bin_id(b, G);
        members[bin[i]].push_back(i);                 // atoms of a bin in index order (the stable CSR)
    }
    struct P { int i, j, S[3]; };
    std::vector<P> out;
    const int w1 = 2 * G.reach[1] + 1, w2 = 2 * G.reach[2] + 1, n_off = (2 * G.reach[0] + 1) * w1 * w2;
    for (int i = 0; i < n; ++i) {
        const int id = bin[i];
        const int b[3] = {id / (G.nb[1] * G.nb[2]), (id / G.nb[2]) % G.nb[1], id % G.nb[2]};
        std::vector<P> mine;
        for (int o = 0; o < n_off; ++o) {
            const int off[3] = {o / (w1 * w2) - G.reach[0], (o / w2) % w1 - G.reach[1], o % w2 - G.reach[2]};
            int nbb[3], img[3];
            bool ok = true;
            for (int a = 0; a < 3; ++a) ok = ok && nl_step(b[a], off[a], a, G, nbb[a], img[a]);
            if (!ok) continue;
            for (int j : members[nl_bin_id(nbb, G)]) {
                if (!nl_pair(&rw[3 * i], &rw[3 * j], img, j == i, G)) continue;
                P p{i, j, {0, 0, 0}};
                nl_shift(img, &s0[3 * i], &s0[3 * j], p.S);
                mine.push_back(p);
            }
        }
        std::sort(mine.begin(), mine.end(), [](const P &x, const P &y) { return nl_less(x.j, x.S, y.j, y.S); });
        out.insert(out.end(), mine.begin(), mine.end());
    }
    const int m = (int)out.size();
    fwrite(&m, 4, 1, stdout);
    for (const P &p : out) {
        const int rec[5] = {p.i, p.j, p.S[0], p.S[1], p.S[2]};
        float v[3];
        nl_shift_vector(p.S, G, v);
        fwrite(rec, 4, 5, stdout);
        fwrite(v, 4, 3, stdout);
    }
    return 0;
}
'''


@pytest.fixture(scope='module')
def driver(tmp_path_factory):
    gxx = shutil.which('g++')
    if gxx is None:
        pytest.skip('g++ not available')
    d = tmp_path_factory.mktemp('nl')
    (d / 'drv.cpp').write_text(DRIVER)
    exe = d / 'drv'
    r = subprocess.run([gxx, '-O1', '-std=c++17', '-I', CSRC, str(d / 'drv.cpp'), '-o', str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return str(exe)


def _run(exe, st, cutoff, lo=(0, 0, 0), hi=(1, 1, 1)):
    buf = (np.int32(len(st)).tobytes() + np.ascontiguousarray(st.positions, np.float64).tobytes() +
           np.ascontiguousarray(st.cell, np.float64).tobytes() + np.asarray(st.pbc, np.int32).tobytes() +
           np.float64(cutoff).tobytes() + np.asarray(lo, np.float64).tobytes() + np.asarray(hi, np.float64).tobytes())
    r = subprocess.run([exe], input=buf, capture_output=True)
    assert r.returncode == 0, r.returncode
    m = int(np.frombuffer(r.stdout[:4], np.int32)[0])
    rec = np.frombuffer(r.stdout[4:], np.uint8).reshape(m, 32)
    ints = rec[:, :20].copy().view(np.int32).reshape(m, 5)
    vec = rec[:, 20:].copy().view(np.float32).reshape(m, 3)
    return ints, vec


def _check(exe, st, cutoff, **kw):
    ints, vec = _run(exe, st, cutoff, **kw)
    i, j, S = neighbor_list(st.positions, st.cell, st.pbc, cutoff)
    assert len(i) > 0 and ints.shape[0] == len(i), (ints.shape, len(i))
    assert np.array_equal(ints[:, 0], i) and np.array_equal(ints[:, 1], j) and np.array_equal(ints[:, 2:], S)
    ref = (S.astype(np.float64) @ st.cell).astype(np.float32)
    assert np.abs(vec - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_slab_with_adsorbates(driver):
    _check(driver, helpers.make_structure(seed=3), 5.0)


def test_bench_slab_and_bulk(driver):
    _check(driver, S_.pt100_random(seed=1), 5.0)
    _check(driver, S_.fcc_bulk('Cu', n=4, seed=2), 5.0)


def test_cell_thinner_than_cutoff(driver):
    _check(driver, S_.fcc_bulk('Cu', n=1, seed=3), 5.0)           # 3.61 A cell: two images each way per axis
    _check(driver, S_.fcc_bulk('Cu', n=2, seed=4), 6.0)


def test_skewed_cell(driver):
    rng = np.random.default_rng(5)
    cell = np.array([[7.1, 0.0, 0.0], [3.2, 6.4, 0.0], [-1.9, 2.2, 8.3]])
    frac = rng.uniform(-0.2, 1.2, (60, 3))                          # also atoms outside the cell
    st = Structure(frac @ cell, np.full(60, 29), cell, np.array([True, True, True]))
    _check(driver, st, 4.5)


def test_non_periodic_axes(driver):
    rng = np.random.default_rng(6)
    cell = np.diag([12.0, 11.0, 30.0])
    pos = rng.uniform(0, 1, (80, 3)) * [12.0, 11.0, 9.0] + [0, 0, 8.0]
    st = Structure(pos, np.full(80, 8), cell, np.array([True, True, False]))
    _check(driver, st, 5.0, lo=(0, 0, 0.3), hi=(1, 1, 0.5))      # some atoms outside the binned z range
    st = Structure(pos, np.full(80, 8), cell, np.array([False, False, False]))
    _check(driver, st, 5.0)
