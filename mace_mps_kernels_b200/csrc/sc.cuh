// sc.cuh -- sm_100a kernels of MACE's symmetric contraction evaluated as a precomputed polynomial.
//
// Compiled by NVRTC with a generated "mmk_layer.h" that bakes in one SymmetricContraction's monomial list
// (reference src/mace_mps_kernels/symmetric.py:52-75 builds the same list): sizes CH (channels), NELL, NROWS, OUTD and the
// straight-line bodies sc_fwd_node / sc_bwd_node.  The coefficients T[elem][row][c] stay in global memory (they are
// weights, read coalesced across the channel lanes of a node and shared by all nodes of an element through L1/L2).
//
// Thread (c, node) evaluates, for every output block, out[b, off + c*M + m] = sum_t T[elem, row_t + m, c] x^idx_t
// (forward) or gx[b, c, i] = sum_t (sum_m T[elem, row_t + m, c] g[b, off + c*M + m]) d(x^idx_t)/dx_i (backward).
// CTA = CH (channels) threads x NPB nodes.
#include "mmk_layer.h"

template <int NPB>
__global__ void __launch_bounds__(CH * NPB)
mmk_sc_fwd_kernel(const float *__restrict__ x, const int *__restrict__ elem, const float *__restrict__ T,
                  float *__restrict__ out, long long n_nodes) {
    const long long b = (long long)blockIdx.x * NPB + threadIdx.y;
    if (b >= n_nodes) return;
    const int c = threadIdx.x;
    float xs[NELL];
    load_feat(x + (b * CH + c) * NELL, xs);
    const float *t = T + (long long)elem[b] * (NROWS * CH) + c;
    sc_fwd_node(xs, t, out + b * OUTD, c);
}

template <int NPB>
__global__ void __launch_bounds__(CH * NPB)
mmk_sc_bwd_kernel(const float *__restrict__ x, const int *__restrict__ elem, const float *__restrict__ T,
                  const float *__restrict__ g, float *__restrict__ gx, long long n_nodes) {
    const long long b = (long long)blockIdx.x * NPB + threadIdx.y;
    if (b >= n_nodes) return;
    const int c = threadIdx.x;
    float xs[NELL], d[NELL];
    load_feat(x + (b * CH + c) * NELL, xs);
#pragma unroll
    for (int i = 0; i < NELL; ++i) d[i] = 0.0f;
    const float *t = T + (long long)elem[b] * (NROWS * CH) + c;
    sc_bwd_node(xs, t, g + b * OUTD, c, d);
    store_feat(gx + (b * CH + c) * NELL, d);
}
