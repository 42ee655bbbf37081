// conv_tp.cuh -- sm_100a kernels of the MACE interaction convolution (channel-wise weighted uvu tensor product).
//
// Compiled at layer-creation time by NVRTC together with a generated header "mmk_layer.h" that bakes in one
// TensorProduct: the sizes (MUL, XR, YD, ORR, NINS), the row accessors, and the straight-line per-edge bodies
// fwd_edge / bwd_edge whose constants are the probed path coefficients (reference src/mace_mps_kernels/conv.py:57-88
// measures the same numbers).
//
// Both kernels are persistent and warp-specialised:
//   * one producer warp streams, edge by edge in CSR order, the rows an edge needs into a STAGES-deep ring of shared
//     memory with TMA bulk copies (cp.async.bulk, completion counted on a per-stage mbarrier): W[e] (NINS*MUL floats)
//     plus x[sender] (forward) or grad_out[receiver] (backward), plus Y[e] when its row is 16-byte sized;
//   * MUL consumer threads (one per channel u) wait for a stage, run the generated per-edge body on their channel's
//     values, and release the stage back to the producer.
// Nodes are dealt to CTAs round-robin (node = blockIdx.x + k * gridDim.x) so that the CTAs work on a contiguous window
// of nodes at any time and the gathered rows of their shared neighbours are reused from L2.
//   forward   node = receiver; out[n] accumulated in registers over the receiver CSR segment, written once:
//             deterministic, no atomics.
//   backward  node = sender; x[s] in registers; per edge gW[e, :, u] (coalesced over u) and gY[e, :] (channel sum:
//             register transpose-reduce in each warp, then across the consumer warps through shared memory, handed
//             over with an mbarrier); gx[s] accumulated in registers, written once.  Fuses the reference's
//             conv_bwd_x and conv_bwd_wy (conv.py:144-222), which gather x and grad_out twice.
// Every wait is bounded (about a second of clock64); on expiry the CTA records an error code in mmk_status, the
// producer waits (bounded) for the copies it issued, and the CTA returns -- no trap, no hang.
#include "mmk_layer.h"

#define X_DIM (XR * MUL)
#define OUT_DIM (ORR * MUL)
#define W_DIM (NINS * MUL)
#define NCW (MUL / 32)                      // consumer warps
#define Y_TMA ((YD * 4) % 16 == 0)         // Y rows are copied with TMA when 16-byte sized
#define MMK_WAIT_BUDGET (2000000000LL)      // clock64 cycles, ~1 s

// Error status of this module's kernels on this device (0 = ok); read and reset by mmk_conv_layer_status().
__device__ int mmk_status;

typedef unsigned long long u64;
typedef unsigned int u32;

__device__ __forceinline__ u32 smem_addr(const void *p) { return (u32)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(u64 *bar, u32 count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(u64 *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(u64 *bar, u32 bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(u64 *bar, u32 parity) {
    u32 ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait: false after about MMK_WAIT_BUDGET cycles
__device__ __forceinline__ bool mbar_wait(u64 *bar, u32 parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > MMK_WAIT_BUDGET) return false;
    }
    return true;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, u32 bytes, u64 *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

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

// Producer: issue the TMA copies of every edge of the CTA's nodes, in the consumers' order.  All 32 lanes walk the
// loop (they fetch edge ids 32 at a time); lane 0 waits for free stages and issues.  Returns false on a timeout.
template <int STAGES, class Issue>
__device__ __forceinline__ bool produce(const int *__restrict__ rowptr, const int *__restrict__ eids,
                                        const long long *__restrict__ other, long long n_nodes, u64 *full, u64 *empty,
                                        u32 &it, Issue issue) {
    const int lane = threadIdx.x & 31;
    for (long long n = blockIdx.x; n < n_nodes; n += gridDim.x) {
        const int p0 = rowptr[n], p1 = rowptr[n + 1];
        for (int q = p0; q < p1; q += 32) {
            long long e = 0, o = 0;
            if (q + lane < p1) {
                e = eids[q + lane];
                o = other[e];
            }
            const int cnt = min(32, p1 - q);
            for (int j = 0; j < cnt; ++j, ++it) {
                const long long ej = __shfl_sync(0xffffffffu, e, j);
                const long long oj = __shfl_sync(0xffffffffu, o, j);
                const u32 st = it % STAGES, ph = (it / STAGES) & 1;
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&empty[st], ph ^ 1);
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return false;
                if (lane == 0) issue(st, ej, oj, &full[st]);
                __syncwarp();
            }
        }
    }
    return true;
}

// After a timeout: wait (bounded) until the copies already issued into the ring have landed, so that no TMA write
// targets the shared memory of an exited CTA.
template <int STAGES>
__device__ __forceinline__ void drain(u64 *full, u32 issued) {
    if ((threadIdx.x & 31) != 0) return;
    const u32 first = issued > STAGES ? issued - STAGES : 0;
    for (u32 i = first; i < issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
}

// ------------------------------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------------------------------
template <int STAGES>
__global__ void __launch_bounds__(MUL + 32)
mmk_conv_fwd_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                    const int *__restrict__ rowptr, const int *__restrict__ eids,
                    const long long *__restrict__ senders, float *__restrict__ out, long long n_nodes) {
    constexpr u32 STAGE_F = W_DIM + X_DIM + 16;     // floats per stage: W row | x row | Y row (padded to 16)
    extern __shared__ __align__(128) float smem[];
    u64 *full = reinterpret_cast<u64 *>(smem + STAGES * STAGE_F);
    u64 *empty = full + STAGES;
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (tid >= MUL) {                               // producer warp
        u32 it = 0;
        auto issue = [&](u32 st, long long e, long long s, u64 *bar) {
            float *stage = smem + st * STAGE_F;
            mbar_arrive_expect_tx(bar, (W_DIM + X_DIM) * 4 + (Y_TMA ? YD * 4 : 0));
            bulk_g2s(stage, W + e * W_DIM, W_DIM * 4, bar);
            bulk_g2s(stage + W_DIM, x + s * X_DIM, X_DIM * 4, bar);
            if constexpr (Y_TMA) bulk_g2s(stage + W_DIM + X_DIM, Y + e * YD, YD * 4, bar);
        };
        if (!produce<STAGES>(rowptr, eids, senders, n_nodes, full, empty, it, issue)) {
            if ((tid & 31) == 0) atomicExch(&mmk_status, 1);
            drain<STAGES>(full, it);
        }
        return;
    }

    const int u = tid;
    u32 it = 0;
    for (long long n = blockIdx.x; n < n_nodes; n += gridDim.x) {
        float acc[ORR];
#pragma unroll
        for (int i = 0; i < ORR; ++i) acc[i] = 0.0f;
        const int p0 = rowptr[n], p1 = rowptr[n + 1];
        for (int p = p0; p < p1; ++p, ++it) {
            const u32 st = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[st], ph)) {
                if ((tid & 31) == 0) atomicExch(&mmk_status, 2);
                return;
            }
            const float *stage = smem + st * STAGE_F;
            float xs[XR], y[YD], w[NINS];
#pragma unroll
            for (int k = 0; k < NINS; ++k) w[k] = stage[k * MUL + u];
            load_x_s(stage + W_DIM, u, xs);
            if constexpr (Y_TMA) {
#pragma unroll
                for (int j = 0; j < YD; ++j) y[j] = stage[W_DIM + X_DIM + j];
            } else {
                const long long e = eids[p];
#pragma unroll
                for (int j = 0; j < YD; ++j) y[j] = __ldg(Y + e * YD + j);
            }
            __syncwarp();
            if ((tid & 31) == 0) mbar_arrive(&empty[st]);
            fwd_edge(xs, y, w, acc);
        }
        store_out(out + n * OUT_DIM, u, acc);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------------------------------
template <int STAGES>
__global__ void __launch_bounds__(MUL + 32)
mmk_conv_bwd_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                    const float *__restrict__ g, const int *__restrict__ rowptr, const int *__restrict__ eids,
                    const long long *__restrict__ receivers, float *__restrict__ gx, float *__restrict__ gY,
                    float *__restrict__ gW, long long n_nodes) {
    constexpr u32 STAGE_F = W_DIM + OUT_DIM + 16;   // W row | grad_out row | Y row (padded to 16)
    extern __shared__ __align__(128) float smem[];
    u64 *full = reinterpret_cast<u64 *>(smem + STAGES * STAGE_F);
    u64 *empty = full + STAGES;
    u64 *red = empty + STAGES;                                    // [2] consumer warps' gY partials are in
    float *part = reinterpret_cast<float *>(red + 2);             // [2][NCW][16] channel-sum partials of gY
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_init(&red[0], NCW);
        mbar_init(&red[1], NCW);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (tid >= MUL) {
        u32 it = 0;
        auto issue = [&](u32 st, long long e, long long r, u64 *bar) {
            float *stage = smem + st * STAGE_F;
            mbar_arrive_expect_tx(bar, (W_DIM + OUT_DIM) * 4 + (Y_TMA ? YD * 4 : 0));
            bulk_g2s(stage, W + e * W_DIM, W_DIM * 4, bar);
            bulk_g2s(stage + W_DIM, g + r * OUT_DIM, OUT_DIM * 4, bar);
            if constexpr (Y_TMA) bulk_g2s(stage + W_DIM + OUT_DIM, Y + e * YD, YD * 4, bar);
        };
        if (!produce<STAGES>(rowptr, eids, receivers, n_nodes, full, empty, it, issue)) {
            if ((tid & 31) == 0) atomicExch(&mmk_status, 3);
            drain<STAGES>(full, it);
        }
        return;
    }

    const int u = tid, warp = tid >> 5, lane = tid & 31;
    u32 it = 0;
    for (long long s = blockIdx.x; s < n_nodes; s += gridDim.x) {
        float xs[XR], gxa[XR];
        load_x(x + s * X_DIM, u, xs);
#pragma unroll
        for (int i = 0; i < XR; ++i) gxa[i] = 0.0f;
        const int p0 = rowptr[s], p1 = rowptr[s + 1];
        for (int p = p0; p < p1; ++p, ++it) {
            const u32 st = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[st], ph)) {
                if (lane == 0) atomicExch(&mmk_status, 4);
                return;
            }
            const long long e = eids[p];
            const float *stage = smem + st * STAGE_F;
            float y[YD], w[NINS], go[ORR], gw[NINS], gy[16];
#pragma unroll
            for (int k = 0; k < NINS; ++k) w[k] = stage[k * MUL + u];
            load_out_s(stage + W_DIM, u, go);
            if constexpr (Y_TMA) {
#pragma unroll
                for (int j = 0; j < YD; ++j) y[j] = stage[W_DIM + OUT_DIM + j];
            } else {
#pragma unroll
                for (int j = 0; j < YD; ++j) y[j] = __ldg(Y + e * YD + j);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
            for (int j = 0; j < 16; ++j) gy[j] = 0.0f;
            bwd_edge(xs, y, w, go, gxa, gw, gy);
            if (gW != nullptr) {
                float *gwe = gW + e * W_DIM + u;
#pragma unroll
                for (int k = 0; k < NINS; ++k) gwe[k * MUL] = gw[k];
            }
            if (gY != nullptr) {
                const u32 b = it & 1;
                float *pb = part + b * (NCW * 16);
                const float v = warp_transpose_reduce16(gy);
                if ((lane & 1) == 0) pb[warp * 16 + (lane >> 1)] = v;
                __syncwarp();
                if (lane == 0) mbar_arrive(&red[b]);
                if (!mbar_wait(&red[b], (it >> 1) & 1)) {
                    if (lane == 0) atomicExch(&mmk_status, 5);
                    return;
                }
                if (u < YD) {
                    float t = 0.0f;
#pragma unroll
                    for (int q = 0; q < NCW; ++q) t += pb[q * 16 + u];
                    gY[e * YD + u] = t;
                }
                // edge it+1 uses the other half; the writes of edge it+2 into this half come after every warp passed
                // red[b ^ 1] at edge it+1, i.e. after these reads
            }
        }
        if (gx != nullptr) store_x(gx + s * X_DIM, u, gxa);
    }
}
