// neighbors.cuh -- periodic neighbour list on B200: every pair (i, j, S) with 0 < |r_j + S.cell - r_i| < cutoff
// (matscipy / ASE neighbour_list('ijS') semantics as MACE uses them: sender i, receiver j, shift S in cells), by a
// cell list over the wrapped fractional coordinates.
//
// Per-atom arithmetic shared by the CUDA kernels (mmk_runtime.cu) and, compiled for the host, by the tests (MMK_HD
// expands to nothing there).  Float64 throughout; products and sums are written out with fma / plain operations in a
// fixed order so that host and device give identical bits.
//
// Binning: along a periodic axis the wrapped fractional coordinate f in [0, 1) falls in nb = floor(height / cutoff)
// bins (at least 1; height = distance between the lattice planes of that axis), and the search visits the bins
// t = b - reach .. b + reach, reach = ceil(cutoff * nb / height), each t standing for bin t mod nb of image
// floor(t / nb): since |floor(x) - floor(y)| <= ceil(|x - y|), every image within the cutoff is visited, and each
// (bin, image) once.  Along a non-periodic axis the caller gives a fractional range [lo, hi]; nb bins of at least one
// cutoff each cover it, coordinates outside are clamped into the end bins (clamping never separates two points by
// more bins than before, so reach 1 still finds every pair), and there are no images.
#pragma once

#include <cmath>

#ifndef MMK_HD
#define MMK_HD __host__ __device__
#endif

struct MmkNlGeom {
    double cell[3][3];    // lattice vectors as rows: r = f . cell
    double inv[3][3];     // cell^-1: f = r . inv
    int pbc[3];
    int nb[3];            // bins per axis
    int reach[3];         // bins searched on either side
    double lo[3];         // binned fractional range start (0 on periodic axes)
    double scale[3];      // bins per unit of fractional coordinate
    double cutoff2;
};

// r . M for a row vector r and a 3 x 3 matrix M, in a fixed order
MMK_HD inline void nl_rowmul(const double r[3], const double M[3][3], double out[3]) {
    for (int c = 0; c < 3; ++c) out[c] = fma(r[2], M[2][c], fma(r[1], M[1][c], r[0] * M[0][c]));
}

// wrapped coordinates of one atom: f = r . inv, s0 = floor(f) on periodic axes (0 elsewhere), fw = f - s0,
// rw = fw . cell; bin b[3] of fw
MMK_HD inline void nl_wrap(const double r[3], const MmkNlGeom &G, double rw[3], int s0[3], int b[3]) {
    double f[3], fw[3];
    nl_rowmul(r, G.inv, f);
    for (int a = 0; a < 3; ++a) {
        const double s = G.pbc[a] ? floor(f[a]) : 0.0;
        s0[a] = (int)s;
        fw[a] = f[a] - s;
        int k = (int)floor((fw[a] - G.lo[a]) * G.scale[a]);
        k = k < 0 ? 0 : (k >= G.nb[a] ? G.nb[a] - 1 : k);
        b[a] = k;
    }
    nl_rowmul(fw, G.cell, rw);
}

MMK_HD inline int nl_bin_id(const int b[3], const MmkNlGeom &G) { return (b[0] * G.nb[1] + b[1]) * G.nb[2] + b[2]; }

// the (bin, image) visited for offset o from bin b along axis a: false when it lies outside a non-periodic range
MMK_HD inline bool nl_step(int b, int o, int a, const MmkNlGeom &G, int &bin, int &img) {
    const int t = b + o;
    if (!G.pbc[a]) {
        if (t < 0 || t >= G.nb[a]) return false;
        bin = t;
        img = 0;
        return true;
    }
    img = t >= 0 ? t / G.nb[a] : -((-t + G.nb[a] - 1) / G.nb[a]);      // floor(t / nb)
    bin = t - img * G.nb[a];
    return true;
}

// squared distance from atom i (wrapped ri) to the image img of atom j (wrapped rj), and whether the pair counts
MMK_HD inline bool nl_pair(const double ri[3], const double rj[3], const int img[3], bool same_atom,
                           const MmkNlGeom &G) {
    if (same_atom && img[0] == 0 && img[1] == 0 && img[2] == 0) return false;
    const double s[3] = {(double)img[0], (double)img[1], (double)img[2]};
    double sc[3];
    nl_rowmul(s, G.cell, sc);
    double r2 = 0.0;
    for (int c = 0; c < 3; ++c) {
        const double d = (rj[c] + sc[c]) - ri[c];
        r2 = fma(d, d, r2);
    }
    return r2 < G.cutoff2;
}

// the reported shift of a pair: S = img - s0[j] + s0[i] (the image in unwrapped coordinates)
MMK_HD inline void nl_shift(const int img[3], const int s0i[3], const int s0j[3], int S[3]) {
    for (int a = 0; a < 3; ++a) S[a] = img[a] - s0j[a] + s0i[a];
}

// (j, S) order of the edges of one sender: j, then S0, S1, S2 (the order of lexsort((S2, S1, S0, j, i)))
MMK_HD inline bool nl_less(int j1, const int S1[3], int j2, const int S2[3]) {
    if (j1 != j2) return j1 < j2;
    for (int a = 0; a < 3; ++a)
        if (S1[a] != S2[a]) return S1[a] < S2[a];
    return false;
}

// shift vector S . cell as the float32 the graph stores (double product and sum in a fixed order, then rounded)
MMK_HD inline void nl_shift_vector(const int S[3], const MmkNlGeom &G, float out[3]) {
    const double s[3] = {(double)S[0], (double)S[1], (double)S[2]};
    double v[3];
    nl_rowmul(s, G.cell, v);
    for (int c = 0; c < 3; ++c) out[c] = (float)v[c];
}

// Binning geometry from the cell (host).  lo / hi: fractional range of non-periodic axes (ignored on periodic ones).
// Returns false when the cell is singular or the cutoff is not positive.
inline bool mmk_nl_geometry(const double cell[9], const int pbc[3], double cutoff, const double lo[3],
                            const double hi[3], int max_bins_axis, MmkNlGeom &G) {
    if (!(cutoff > 0.0)) return false;
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) G.cell[r][c] = cell[3 * r + c];
    const double(*m)[3] = G.cell;
    const double det = m[0][0] * (m[1][1] * m[2][2] - m[1][2] * m[2][1]) - m[0][1] * (m[1][0] * m[2][2] - m[1][2] * m[2][0]) +
                       m[0][2] * (m[1][0] * m[2][1] - m[1][1] * m[2][0]);
    if (!(std::fabs(det) > 0.0)) return false;
    // inverse by cofactors: inv[r][c] = cof[c][r] / det
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c) {
            const int r1 = (c + 1) % 3, r2 = (c + 2) % 3, c1 = (r + 1) % 3, c2 = (r + 2) % 3;
            G.inv[r][c] = (m[r1][c1] * m[r2][c2] - m[r1][c2] * m[r2][c1]) / det;
        }
    for (int a = 0; a < 3; ++a) {
        // height of axis a: |det| / |cell[a+1] x cell[a+2]|
        const double *u = m[(a + 1) % 3], *v = m[(a + 2) % 3];
        const double x = u[1] * v[2] - u[2] * v[1], y = u[2] * v[0] - u[0] * v[2], z = u[0] * v[1] - u[1] * v[0];
        const double height = std::fabs(det) / std::sqrt(x * x + y * y + z * z);
        G.pbc[a] = pbc[a] ? 1 : 0;
        if (pbc[a]) {
            int nb = (int)std::floor(height / cutoff);
            nb = nb < 1 ? 1 : (nb > max_bins_axis ? max_bins_axis : nb);
            G.nb[a] = nb;
            G.reach[a] = (int)std::ceil(cutoff * nb / height);
            G.lo[a] = 0.0;
            G.scale[a] = nb;
        } else {
            const double l = lo[a], h = hi[a] > lo[a] ? hi[a] : lo[a];
            int nb = (int)std::floor((h - l) * height / cutoff);
            nb = nb < 1 ? 1 : (nb > max_bins_axis ? max_bins_axis : nb);
            G.nb[a] = nb;
            G.reach[a] = 1;
            G.lo[a] = l;
            G.scale[a] = h > l ? nb / (h - l) : 0.0;
        }
    }
    G.cutoff2 = cutoff * cutoff;
    return true;
}
