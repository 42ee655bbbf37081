// sc.cuh -- sm_100a kernels of MACE's symmetric contraction evaluated as a precomputed polynomial.
//
// Compiled by NVRTC with a generated "mmk_layer.h" that bakes in one SymmetricContraction's monomial list
// (reference src/mace_mps_kernels/symmetric.py:52-75 builds the same list): sizes CH (channels), NELL, NROWS, OUTD,
// the row chunking of the coefficient table (NCHUNK chunks of at most RCH rows, cut at term boundaries: CHUNK_ROW0[])
// and the straight-line bodies sc_fwd_body / sc_bwd_body, which take the next chunk from the ring (ring.begin()) before
// its first term and hand it back (ring.end()) after its last.
//
// Work: nodes are grouped by element (perm / erow: the node CSR of the element index).  A tile is NG*G nodes of one
// element; consumer thread (c, sub) evaluates channel c of G nodes, so every coefficient T[e, row, c] read from shared
// memory feeds G nodes.  One producer warp streams T[e] chunk by chunk (TMA bulk copies of RCH*CH contiguous floats)
// through a STAGES-deep ring; T[e] is re-streamed for every tile (it stays in L2).  Tiles are dealt round-robin to
// persistent CTAs.  Forward: out[b, off + c*M + m] = sum_t T[e, row_t + m, c] x^idx_t.  Backward: gx[b, c, i] =
// sum_t (sum_m T[e, row_t + m, c] g[b, off + c*M + m]) d(x^idx_t)/dx_i.  Waits are bounded as in conv_tp.cuh.
#include "mmk_layer.h"

#define MMK_WAIT_BUDGET (2000000000LL)
#define NCONS (CH * NG)

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

// tile t -> (element, first position in perm, node count) for tiles of TN nodes; tiles of one element are consecutive
template <int TN>
__device__ __forceinline__ bool tile_of(long long t, const int *__restrict__ erow, int n_elem, int &e, int &p0, int &cnt) {
    long long before = 0;
    for (int k = 0; k < n_elem; ++k) {
        const int a = erow[k], b = erow[k + 1];
        const long long nt = (b - a + TN - 1) / TN;
        if (t < before + nt) {
            e = k;
            p0 = a + (int)(t - before) * TN;
            cnt = min(TN, b - p0);
            return true;
        }
        before += nt;
    }
    return false;
}

// Consumer-side pipeline state: ring position of the next chunk and the CTA's failure flag.
struct Ring {
    const float *smem;
    u64 *full, *empty;
    u32 it;
    bool ok;
    __device__ __forceinline__ const float *begin() {
        const u32 st = it % STAGES, ph = (it / STAGES) & 1;
        if (ok && !mbar_wait(&full[st], ph)) {
            ok = false;
            if ((threadIdx.x & 31) == 0) atomicExch(&mmk_status, 6);
        }
        return smem + (size_t)st * RCH * CH;
    }
    __device__ __forceinline__ void end() {
        const u32 st = it % STAGES;
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[st]);
        ++it;
    }
};

template <int TN>
__device__ __forceinline__ void sc_produce(const float *__restrict__ T, const int *__restrict__ erow, int n_elem,
                                           long long n_tiles, const float *smem, u64 *full, u64 *empty) {
    const int lane = threadIdx.x & 31;
    u32 it = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        int e, p0, cnt;
        if (!tile_of<TN>(t, erow, n_elem, e, p0, cnt)) break;
        const float *Te = T + (size_t)e * NROWS * CH;
        for (int k = 0; k < NCHUNK && ok; ++k, ++it) {
            const u32 st = it % STAGES, ph = (it / STAGES) & 1;
            if (lane == 0) {
                if (!mbar_wait(&empty[st], ph ^ 1)) {
                    ok = false;
                    atomicExch(&mmk_status, 7);
                } else {
                    const u32 bytes = (u32)(CHUNK_ROW0[k + 1] - CHUNK_ROW0[k]) * CH * 4;
                    mbar_arrive_expect_tx(&full[st], bytes);
                    bulk_g2s((void *)(smem + (size_t)st * RCH * CH), Te + (size_t)CHUNK_ROW0[k] * CH, bytes, &full[st]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
    }
    if (!ok && lane == 0) {                       // let the copies already issued land before the CTA exits
        const u32 first = it > STAGES ? it - STAGES : 0;
        for (u32 i = first; i < it; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    }
}

__device__ __forceinline__ void sc_setup(u64 *full, u64 *empty) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCONS / 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
}

extern "C" __global__ void __launch_bounds__(NCONS + 32)
mmk_sc_fwd_kernel(const float *__restrict__ x, const int *__restrict__ perm, const int *__restrict__ erow, int n_elem,
                  const float *__restrict__ T, float *__restrict__ out, long long n_tiles) {
    extern __shared__ __align__(128) float smem[];
    u64 *full = reinterpret_cast<u64 *>(smem + (size_t)STAGES * RCH * CH);
    u64 *empty = full + STAGES;
    sc_setup(full, empty);
    const int tid = threadIdx.x;
    if (tid >= NCONS) {
        sc_produce<NG * G>(T, erow, n_elem, n_tiles, smem, full, empty);
        return;
    }
    const int c = tid % CH, sub = tid / CH;
    Ring ring{smem, full, empty, 0u, true};
    for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        int e, p0, cnt;
        if (!tile_of<NG * G>(t, erow, n_elem, e, p0, cnt)) break;
        long long nodes[G];
        float xv[G][NELL];
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int q = sub * G + j;
            nodes[j] = q < cnt ? (long long)perm[p0 + q] : -1;
            if (nodes[j] >= 0) {
                load_feat(x + (nodes[j] * CH + c) * NELL, xv[j]);
            } else {
#pragma unroll
                for (int i = 0; i < NELL; ++i) xv[j][i] = 0.0f;
            }
        }
        sc_fwd_body(ring, xv, nodes, out, c);
        if (!ring.ok) return;
    }
}

extern "C" __global__ void __launch_bounds__(NCONS + 32)
mmk_sc_bwd_kernel(const float *__restrict__ x, const int *__restrict__ perm, const int *__restrict__ erow, int n_elem,
                  const float *__restrict__ T, const float *__restrict__ g, float *__restrict__ gx, long long n_tiles) {
    extern __shared__ __align__(128) float smem[];
    u64 *full = reinterpret_cast<u64 *>(smem + (size_t)STAGES * RCH * CH);
    u64 *empty = full + STAGES;
    sc_setup(full, empty);
    const int tid = threadIdx.x;
    if (tid >= NCONS) {
        sc_produce<NG * GB>(T, erow, n_elem, n_tiles, smem, full, empty);
        return;
    }
    const int c = tid % CH, sub = tid / CH;
    Ring ring{smem, full, empty, 0u, true};
    for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        int e, p0, cnt;
        if (!tile_of<NG * GB>(t, erow, n_elem, e, p0, cnt)) break;
        long long nodes[GB];
        float xv[GB][NELL], d[GB][NELL];
#pragma unroll
        for (int j = 0; j < GB; ++j) {
            const int q = sub * GB + j;
            nodes[j] = q < cnt ? (long long)perm[p0 + q] : -1;
            if (nodes[j] >= 0) {
                load_feat(x + (nodes[j] * CH + c) * NELL, xv[j]);
            } else {
#pragma unroll
                for (int i = 0; i < NELL; ++i) xv[j][i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < NELL; ++i) d[j][i] = 0.0f;
        }
        sc_bwd_body(ring, xv, nodes, g, c, d);
        if (!ring.ok) return;
#pragma unroll
        for (int j = 0; j < GB; ++j)
            if (nodes[j] >= 0) store_feat(gx + (nodes[j] * CH + c) * NELL, d[j]);
    }
}
