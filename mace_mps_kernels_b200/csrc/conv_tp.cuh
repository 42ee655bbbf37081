// conv_tp.cuh -- sm_100a kernels of the MACE interaction convolution (channel-wise weighted uvu tensor product).
//
// Compiled at layer-creation time by NVRTC together with a generated header "mmk_layer.h" that bakes in one
// TensorProduct: the sizes (MUL, XR, YD, ORR, NINS) and the straight-line per-edge bodies fwd_edge / bwd_edge whose
// constants are the probed path coefficients (reference src/mace_mps_kernels/conv.py:57-88 measures the same numbers).
//
// Work decomposition (one CTA per node, MUL threads per edge slice, SLICES slices; SLICES is a template parameter
// so the host can pick the instantiation whose static shared memory fits):
//   forward   CTA = receiver n, thread (u, slice) = channel u over edges p = rowptr[n] + slice + k*SLICES of the
//             receiver CSR; slices are summed in shared memory in a fixed order -> deterministic, no atomics.
//   backward  CTA = sender s over the sender CSR; each edge of s is owned by one slice, which writes gW[e, :, u]
//             per thread and gY[e, :] after a channel reduction (register transpose-reduce in the warp, then the
//             slice's warps through shared memory behind a named barrier); gx[s] is summed over slices like out.
// Reads per edge: W[e] (NINS*MUL floats, coalesced across channels), Y[e] (YD floats, broadcast), x[sender] (XR
// floats per channel).  64-bit offsets everywhere: E * NINS * MUL exceeds 2^31 on large systems.
#include "mmk_layer.h"

#define X_DIM (XR * MUL)
#define OUT_DIM (ORR * MUL)
#define W_DIM (NINS * MUL)
#define NWARP_SLICE (MUL / 32)

// Reduce v[0..15] over the 32 lanes of a warp; afterwards lanes 2j and 2j+1 both hold the full sum of v[j].
__device__ __forceinline__ float warp_transpose_reduce16(float (&v)[16]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const bool hi = lane & 16;
        float keep = hi ? v[8 + i] : v[i];
        float send = hi ? v[i] : v[8 + i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool hi = lane & 8;
        float keep = hi ? v[4 + i] : v[i];
        float send = hi ? v[i] : v[4 + i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool hi = lane & 4;
        float keep = hi ? v[2 + i] : v[i];
        float send = hi ? v[i] : v[2 + i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
        const bool hi = lane & 2;
        float keep = hi ? v[1] : v[0];
        float send = hi ? v[0] : v[1];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    return v[0];
}

template <int SLICES>
__global__ void __launch_bounds__(MUL * SLICES)
mmk_conv_fwd_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                    const int *__restrict__ rowptr, const int *__restrict__ eids,
                    const long long *__restrict__ senders, float *__restrict__ out, long long n_nodes) {
    const long long n = blockIdx.x;
    if (n >= n_nodes) return;
    const int u = threadIdx.x;
    const int slice = threadIdx.y;
    float acc[ORR];
#pragma unroll
    for (int i = 0; i < ORR; ++i) acc[i] = 0.0f;
    const int p1 = rowptr[n + 1];
    for (int p = rowptr[n] + slice; p < p1; p += SLICES) {
        const long long e = eids[p];
        const long long s = senders[e];
        float xs[XR], y[YD], w[NINS];
        load_x(x + s * X_DIM, u, xs);
        const float *ye = Y + e * YD;
#pragma unroll
        for (int j = 0; j < YD; ++j) y[j] = __ldg(ye + j);
        const float *we = W + e * W_DIM + u;
#pragma unroll
        for (int k = 0; k < NINS; ++k) w[k] = __ldg(we + k * MUL);
        fwd_edge(xs, y, w, acc);
    }
    if constexpr (SLICES > 1) {
    __shared__ float red[SLICES - 1][ORR][MUL];
    if (slice > 0) {
#pragma unroll
        for (int i = 0; i < ORR; ++i) red[slice - 1][i][u] = acc[i];
    }
    __syncthreads();
    if (slice > 0) return;
#pragma unroll
    for (int q = 0; q < SLICES - 1; ++q) {
#pragma unroll
        for (int i = 0; i < ORR; ++i) acc[i] += red[q][i][u];
    }
    }
    store_out(out + n * OUT_DIM, u, acc);
}

template <int SLICES>
__global__ void __launch_bounds__(MUL * SLICES)
mmk_conv_bwd_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                    const float *__restrict__ g, const int *__restrict__ rowptr, const int *__restrict__ eids,
                    const long long *__restrict__ receivers, float *__restrict__ gx, float *__restrict__ gY,
                    float *__restrict__ gW, long long n_nodes) {
    const long long s = blockIdx.x;
    if (s >= n_nodes) return;
    const int u = threadIdx.x;
    const int slice = threadIdx.y;
    const int warp = u >> 5, lane = u & 31;
    __shared__ float part[SLICES][2][NWARP_SLICE][16];
    float xs[XR], gxa[XR];
    load_x(x + s * X_DIM, u, xs);
#pragma unroll
    for (int i = 0; i < XR; ++i) gxa[i] = 0.0f;
    const int p1 = rowptr[s + 1];
    int parity = 0;
    for (int p = rowptr[s] + slice; p < p1; p += SLICES, parity ^= 1) {
        const long long e = eids[p];
        const long long r = receivers[e];
        float y[YD], w[NINS], go[ORR], gw[NINS], gy[16];
        const float *ye = Y + e * YD;
#pragma unroll
        for (int j = 0; j < YD; ++j) y[j] = __ldg(ye + j);
        const float *we = W + e * W_DIM + u;
#pragma unroll
        for (int k = 0; k < NINS; ++k) w[k] = __ldg(we + k * MUL);
        load_out(g + r * OUT_DIM, u, go);
#pragma unroll
        for (int j = 0; j < 16; ++j) gy[j] = 0.0f;
        bwd_edge(xs, y, w, go, gxa, gw, gy);
        if (gW != nullptr) {
            float *gwe = gW + e * W_DIM + u;
#pragma unroll
            for (int k = 0; k < NINS; ++k) gwe[k * MUL] = gw[k];
        }
        if (gY != nullptr) {
            const float v = warp_transpose_reduce16(gy);
            if ((lane & 1) == 0) part[slice][parity][warp][lane >> 1] = v;
            if constexpr (NWARP_SLICE > 1) {
                asm volatile("bar.sync %0, %1;" ::"r"(slice + 1), "r"(MUL) : "memory");
            } else {
                __syncwarp();
            }
            if (u < YD) {
                float t = 0.0f;
#pragma unroll
                for (int q = 0; q < NWARP_SLICE; ++q) t += part[slice][parity][q][u];
                gY[e * YD + u] = t;
            }
            // the next edge of this slice writes the other parity buffer; the barrier of the edge after that
            // orders this read before that overwrite.
        }
    }
    if (gx == nullptr) return;
    if constexpr (SLICES > 1) {
    __shared__ float red[SLICES - 1][XR][MUL];
    if (slice > 0) {
#pragma unroll
        for (int i = 0; i < XR; ++i) red[slice - 1][i][u] = gxa[i];
    }
    __syncthreads();
    if (slice > 0) return;
#pragma unroll
    for (int q = 0; q < SLICES - 1; ++q) {
#pragma unroll
        for (int i = 0; i < XR; ++i) gxa[i] += red[q][i][u];
    }
    }
    store_x(gx + s * X_DIM, u, gxa);
}
