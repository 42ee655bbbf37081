// edge_geom.cuh -- per-edge geometry of MACE on B200: real spherical harmonics of the edge vectors and the radial
// embedding (Bessel basis times polynomial cutoff) of the edge lengths, forward and first-order backward.
//
// One thread per edge; plain arithmetic shared by the CUDA kernels (mmk_runtime.cu) and, compiled for the host, by the
// tests (MMK_HD expands to nothing there).  The definitions are those of the model's own modules:
//   Y_l,m>0 = N_lm P~_l^m(z) Re (x+iy)^m,  Y_l,m<0 = N_l|m| P~_l^|m|(z) Im (x+iy)^|m|,  Y_l0 = N_l0 P~_l^0(z)
// on the unit vector (x, y, z) = v / |v| ('component' normalisation, N_lm = sqrt((2l+1)(l-m)!/(l+m)!) * (sqrt 2 for
// m > 0), P~_l^m = P_l^m / sin^m(theta) by the three-term Legendre recursion without the Condon-Shortley phase), and
//   radial_n(r) = prefactor * sin(w_n r) / r * env(r),
//   env(r) = 1 - (p+1)(p+2)/2 u^p + p(p+2) u^(p+1) - p(p+1)/2 u^(p+2) for u = r / r_max < 1, else 0.
// The backward of the harmonics differentiates the recursions alongside them (d/dx, d/dy of Re/Im (x+iy)^m, d/dz of
// P~) and projects the gradient on the tangent plane of the normalisation: g_v = (g_u - u (u . g_u)) / |v|.
#pragma once

#include <cmath>

#ifndef MMK_HD
#define MMK_HD __host__ __device__
#endif

#define MMK_SH_MAX_L 3

struct MmkShNorm {
    float n[(MMK_SH_MAX_L + 1) * (MMK_SH_MAX_L + 1)];      // N_lm at index l*l + l + m for m >= 0 (m < 0 unused)
};

// N_lm for l <= lmax (host; double, rounded to float as the model's float32 products use them)
inline MmkShNorm mmk_sh_norms(int lmax) {
    MmkShNorm N{};
    for (int l = 0; l <= lmax; ++l)
        for (int m = 0; m <= l; ++m) {
            double f = 1.0;                                      // (l-m)! / (l+m)!
            for (int i = l - m + 1; i <= l + m; ++i) f /= i;
            N.n[l * l + l + m] = (float)(std::sqrt((2 * l + 1) * f) * (m ? std::sqrt(2.0) : 1.0));
        }
    return N;
}

// Y[(l+1)^2 components, l = 0..L] of the unit vector (x, y, z)
template <int L>
MMK_HD inline void sh_values(float x, float y, float z, const MmkShNorm &N, float *Y) {
    float A[L + 1], B[L + 1], P[L + 1][L + 1];
    A[0] = 1.0f;
    B[0] = 0.0f;
    for (int m = 1; m <= L; ++m) {
        A[m] = x * A[m - 1] - y * B[m - 1];
        B[m] = x * B[m - 1] + y * A[m - 1];
    }
    float dfact = 1.0f;
    for (int m = 0; m <= L; ++m) {
        if (m > 0) dfact *= (float)(2 * m - 1);
        P[m][m] = dfact;
        if (m + 1 <= L) P[m + 1][m] = (float)(2 * m + 1) * z * P[m][m];
        for (int l = m + 2; l <= L; ++l)
            P[l][m] = ((float)(2 * l - 1) * z * P[l - 1][m] - (float)(l + m - 1) * P[l - 2][m]) / (float)(l - m);
    }
    for (int l = 0; l <= L; ++l)
        for (int m = -l; m <= l; ++m) {
            const int am = m < 0 ? -m : m;
            const float c = N.n[l * l + l + am] * P[l][am];
            Y[l * l + l + m] = m < 0 ? c * B[am] : (m == 0 ? c : c * A[am]);
        }
}

// forward: Y of the edge vector v (normalised here)
template <int L>
MMK_HD inline void sh_forward(const float *v, const MmkShNorm &N, float *Y) {
    const float r = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    sh_values<L>(v[0] / r, v[1] / r, v[2] / r, N, Y);
}

// backward: g_v from g_Y
template <int L>
MMK_HD inline void sh_backward(const float *v, const float *gY, const MmkShNorm &N, float *gv) {
    const float r = sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
    const float x = v[0] / r, y = v[1] / r, z = v[2] / r;
    float A[L + 1], B[L + 1], Ax[L + 1], Ay[L + 1], Bx[L + 1], By[L + 1];
    A[0] = 1.0f; B[0] = 0.0f; Ax[0] = Ay[0] = Bx[0] = By[0] = 0.0f;
    for (int m = 1; m <= L; ++m) {
        A[m] = x * A[m - 1] - y * B[m - 1];
        B[m] = x * B[m - 1] + y * A[m - 1];
        Ax[m] = A[m - 1] + x * Ax[m - 1] - y * Bx[m - 1];
        Ay[m] = x * Ay[m - 1] - B[m - 1] - y * By[m - 1];
        Bx[m] = B[m - 1] + x * Bx[m - 1] + y * Ax[m - 1];
        By[m] = x * By[m - 1] + A[m - 1] + y * Ay[m - 1];
    }
    float P[L + 1][L + 1], Pz[L + 1][L + 1];
    float dfact = 1.0f;
    for (int m = 0; m <= L; ++m) {
        if (m > 0) dfact *= (float)(2 * m - 1);
        P[m][m] = dfact;
        Pz[m][m] = 0.0f;
        if (m + 1 <= L) {
            P[m + 1][m] = (float)(2 * m + 1) * z * P[m][m];
            Pz[m + 1][m] = (float)(2 * m + 1) * P[m][m];
        }
        for (int l = m + 2; l <= L; ++l) {
            P[l][m] = ((float)(2 * l - 1) * z * P[l - 1][m] - (float)(l + m - 1) * P[l - 2][m]) / (float)(l - m);
            Pz[l][m] = ((float)(2 * l - 1) * (P[l - 1][m] + z * Pz[l - 1][m]) - (float)(l + m - 1) * Pz[l - 2][m]) /
                       (float)(l - m);
        }
    }
    float gx = 0.0f, gy = 0.0f, gz = 0.0f;
    for (int l = 0; l <= L; ++l)
        for (int m = -l; m <= l; ++m) {
            const int am = m < 0 ? -m : m;
            const float g = gY[l * l + l + m] * N.n[l * l + l + am];
            if (m < 0) {
                gx += g * P[l][am] * Bx[am];
                gy += g * P[l][am] * By[am];
                gz += g * Pz[l][am] * B[am];
            } else if (m == 0) {
                gz += g * Pz[l][0];
            } else {
                gx += g * P[l][am] * Ax[am];
                gy += g * P[l][am] * Ay[am];
                gz += g * Pz[l][am] * A[am];
            }
        }
    const float d = x * gx + y * gy + z * gz;
    gv[0] = (gx - x * d) / r;
    gv[1] = (gy - y * d) / r;
    gv[2] = (gz - z * d) / r;
}

// radial embedding constants (the model's buffers)
struct MmkRadial {
    float w[16];          // Bessel frequencies w_n
    float prefactor;      // sqrt(2 / r_max)
    float r_max, p;       // cutoff radius and polynomial order
    int n;                // number of Bessel functions (<= 16)
};

MMK_HD inline float radial_env(float r, const MmkRadial &R, float *denv) {
    const float p = R.p, u = r / R.r_max;
    const float c1 = (p + 1.0f) * (p + 2.0f) / 2.0f, c2 = p * (p + 2.0f), c3 = p * (p + 1.0f) / 2.0f;
    const float up = powf(u, p), up1 = powf(u, p + 1.0f), up2 = powf(u, p + 2.0f);
    const float inside = r < R.r_max ? 1.0f : 0.0f;
    if (denv) {
        const float um1 = powf(u, p - 1.0f);
        *denv = inside * (-c1 * p * um1 + c2 * (p + 1.0f) * up - c3 * (p + 2.0f) * up1) / R.r_max;
    }
    return (1.0f - c1 * up + c2 * up1 - c3 * up2) * inside;
}

MMK_HD inline void radial_forward(float r, const MmkRadial &R, float *out) {
    const float env = radial_env(r, R, nullptr);
    for (int k = 0; k < R.n; ++k) out[k] = R.prefactor * sinf(R.w[k] * r) / r * env;
}

MMK_HD inline float radial_backward(float r, const float *g, const MmkRadial &R) {
    float denv;
    const float env = radial_env(r, R, &denv);
    float s = 0.0f;
    for (int k = 0; k < R.n; ++k) {
        float sn, cs;
        sn = sinf(R.w[k] * r);
        cs = cosf(R.w[k] * r);
        const float b = R.prefactor * sn / r;
        const float db = R.prefactor * (R.w[k] * cs * r - sn) / (r * r);
        s += g[k] * (db * env + b * denv);
    }
    return s;
}
