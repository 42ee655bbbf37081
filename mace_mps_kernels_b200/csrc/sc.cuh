// sc.cuh -- sm_100a kernels of MACE's symmetric contraction evaluated as a precomputed polynomial.
//
// Compiled by NVRTC with a generated "mmk_layer.h" that bakes in one SymmetricContraction's monomial list
// (reference src/mace_mps_kernels/symmetric.py:52-75 builds the same list): sizes CH (channels), CP (channel stride of
// the coefficient table, CH rounded up to 4), NELL, NROWS, OUTD (output row), OUTM (outputs per channel), the row
// chunking of the table (NCHUNK chunks of at most RCH rows cut at term boundaries, CHUNK_ROW0[]), and per chunk the
// straight-line term code sc_fwd_body<GG, TG> / sc_bwd_body<GG, TG> (chunk k run by the group that owns its ring
// position, taken from and handed back to the ring around its terms), sc_fwd_store<GG>, sc_load_grad<GG>.
//
// Work: nodes are grouped by element (perm / erow: the node CSR of the element index).  A tile is NG*GG nodes of one
// element.  The CTA has TG consumer groups of CPG threads (CPG = CH*NG rounded up to whole warps, NG and GG template
// parameters) and one producer warp.  Thread (group, sub, c) evaluates channel c of the GG nodes of sub-tile `sub` for the chunks whose ring
// position is group modulo TG; every coefficient T[e, row, c] read from shared memory feeds GG nodes.  The producer streams T[e]
// chunk by chunk (TMA bulk copies of rows*CP contiguous floats) through a STAGES-deep ring of shared memory, each stage
// released by the warps of the group that owns it.  With TG > 1 the groups' partial sums are added in shared memory
// in group order (deterministic), handed over with a pair of mbarriers per tile parity.
// Two instantiations (GG, NG, TG): many nodes -> one node per thread, NG = 512/CH sub-tiles sharing every staged
// coefficient row, one group; few nodes -> NG = 128/CH, the term list split over TG = 4 groups.
// Forward: out[b, off + c*M + m] = sum_t T[e, row_t + m, c] x^idx_t.  Backward: gx[b, c, i] = sum_t (sum_m
// T[e, row_t + m, c] g[b, off + c*M + m]) d(x^idx_t)/dx_i.  Waits are bounded as in conv_tp.cuh.
#include "mmk_layer.h"

#define MMK_WAIT_BUDGET (2000000000LL)

// consumer threads per group: CH channels x NG node sub-tiles, rounded up to whole warps
template <int NG>
struct Cpg {
    static constexpr int value = ((CH * NG) + 31) / 32 * 32;
};

__device__ int mmk_status;

// With MMK_CHECKS defined (environment MMK_CHECKS=1 at layer creation) node and element indices are range-checked: a
// bad one is recorded in mmk_status (100 + where) and the node is skipped.
#ifdef MMK_CHECKS
#define MMK_BAD_INDEX(v, n, where) (((v) < 0 || (v) >= (n)) ? (atomicExch(&mmk_status, 100 + (where)), true) : false)
#else
#define MMK_BAD_INDEX(v, n, where) false
#endif

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

// shared-memory layout: [STAGES][RCH*CP] coefficient ring | full[STAGES] | empty[STAGES] | red_full[2] | red_free[2]
//                       | reduction buffer [2][TG-1][GG*K][CPG]
struct Smem {
    float *ring;
    u64 *full, *empty, *red_full, *red_free;
    float *red;
};

__device__ __forceinline__ Smem smem_layout(float *base) {
    Smem s;
    s.ring = base;
    s.full = reinterpret_cast<u64 *>(base + STAGES * RCH * CP);
    s.empty = s.full + STAGES;
    s.red_full = s.empty + STAGES;
    s.red_free = s.red_full + 2;
    s.red = reinterpret_cast<float *>(s.red_free + 2);
    return s;
}

template <int NG, int TG>
__device__ __forceinline__ void sc_setup(const Smem &s) {
    constexpr int CPG = Cpg<NG>::value;
    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], CPG / 32);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.red_full[i], TG > 1 ? (TG - 1) * (CPG / 32) : 1);
            mbar_init(&s.red_free[i], CPG / 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
}

// Consumer view of the ring for one tile: chunk k of the tile lives in stage (it + k) % STAGES.
struct Ring {
    const Smem &s;
    u32 it;
    int c;
    __device__ __forceinline__ const float *wait(int k) {
        const u32 i = it + k, st = i % STAGES;
        if (!mbar_wait(&s.full[st], (i / STAGES) & 1)) {
            if ((threadIdx.x & 31) == 0) atomicExch(&mmk_status, 6);
            return nullptr;
        }
        return s.ring + (size_t)st * RCH * CP + c;
    }
    __device__ __forceinline__ void release(int k) {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&s.empty[(it + k) % STAGES]);
    }
    __device__ __forceinline__ void advance(int n) { it += n; }
    // group that consumes chunk k of this tile: by ring position, so that (STAGES a multiple of TG) every slot always
    // belongs to one group and a group never waits on a phase of a slot another group still holds
    __device__ __forceinline__ int owner(int k, int tg) const { return (int)((it + k) % (u32)tg); }
};

template <int TN>
__device__ __forceinline__ void sc_produce(const float *__restrict__ T, const int *__restrict__ erow, int n_elem,
                                           long long n_tiles, const Smem &s) {
    const int lane = threadIdx.x & 31;
    u32 it = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        int e, p0, cnt;
        if (!tile_of<TN>(t, erow, n_elem, e, p0, cnt)) break;
        const float *Te = T + (size_t)e * NROWS * CP;
        for (int k = 0; k < NCHUNK && ok; ++k, ++it) {
            const u32 st = it % STAGES, ph = (it / STAGES) & 1;
            if (lane == 0) {
                if (!mbar_wait(&s.empty[st], ph ^ 1)) {
                    ok = false;
                    atomicExch(&mmk_status, 7);
                } else {
                    const u32 bytes = (u32)(CHUNK_ROW0[k + 1] - CHUNK_ROW0[k]) * CP * 4;
                    mbar_arrive_expect_tx(&s.full[st], bytes);
                    bulk_g2s(s.ring + (size_t)st * RCH * CP, Te + (size_t)CHUNK_ROW0[k] * CP, bytes, &s.full[st]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
    }
    if (!ok && lane == 0) {                       // let the copies already issued land before the CTA exits
        const u32 first = it > STAGES ? it - STAGES : 0;
        for (u32 i = first; i < it; ++i) mbar_wait(&s.full[i % STAGES], (i / STAGES) & 1);
    }
}

// Add the groups' partial sums v[GG][K] of one tile into group 0 (fixed group order).  The buffer half used by
// tile_it is refilled two tiles later only after group 0 has released it (red_free).  False on a timeout.
template <int GG, int NG, int TG, int K>
__device__ __forceinline__ bool reduce_groups(const Smem &s, int grp, int r, u32 tile_it, float (&v)[GG][K]) {
    constexpr int CPG = Cpg<NG>::value;
    if constexpr (TG == 1) {
        return true;
    } else {
        const u32 par = tile_it & 1, ph = (tile_it >> 1) & 1;
        float *buf = s.red + (size_t)par * (TG - 1) * GG * K * CPG;
        const int lane = threadIdx.x & 31;
        if (grp > 0) {
            if (!mbar_wait(&s.red_free[par], ph ^ 1)) return false;
            float *dst = buf + (size_t)(grp - 1) * GG * K * CPG + r;
#pragma unroll
            for (int j = 0; j < GG; ++j)
#pragma unroll
                for (int i = 0; i < K; ++i) dst[(j * K + i) * CPG] = v[j][i];
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.red_full[par]);
        } else {
            if (!mbar_wait(&s.red_full[par], ph)) return false;
#pragma unroll
            for (int q = 0; q < TG - 1; ++q) {
                const float *src = buf + (size_t)q * GG * K * CPG + r;
#pragma unroll
                for (int j = 0; j < GG; ++j)
#pragma unroll
                    for (int i = 0; i < K; ++i) v[j][i] += src[(j * K + i) * CPG];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.red_free[par]);
        }
        return true;
    }
}

template <int GG, int NG, int TG>
__global__ void __launch_bounds__(TG * Cpg<NG>::value + 32)
mmk_sc_fwd_kernel(const float *__restrict__ x, const int *__restrict__ perm, const int *__restrict__ erow, int n_elem,
                  const float *__restrict__ T, float *__restrict__ out, long long n_tiles, long long n_nodes) {
    extern __shared__ __align__(128) float smem[];
    constexpr int CPG = Cpg<NG>::value;
    const Smem s = smem_layout(smem);
    sc_setup<NG, TG>(s);
    const int tid = threadIdx.x;
    if (tid >= TG * CPG) {
        sc_produce<NG * GG>(T, erow, n_elem, n_tiles, s);
        return;
    }
    const int grp = tid / CPG, r = tid % CPG, c = r % CH, sub = r / CH;
    const int lane = tid & 31;
    Ring ring{s, 0u, c};
    u32 tile_it = 0;
    for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++tile_it) {
        int e, p0, cnt;
        if (!tile_of<NG * GG>(t, erow, n_elem, e, p0, cnt)) break;
        long long nodes[GG];
        float xv[GG][NELL], acc[GG][OUTM];
#pragma unroll
        for (int j = 0; j < GG; ++j) {
            const int q = sub * GG + j;
            nodes[j] = (sub < NG && q < cnt) ? (long long)perm[p0 + q] : -1;
            if (nodes[j] >= 0 && MMK_BAD_INDEX(nodes[j], n_nodes, 11)) nodes[j] = -1;
            if (nodes[j] >= 0) {
                load_feat(x + (nodes[j] * CH + c) * NELL, xv[j]);
            } else {
#pragma unroll
                for (int i = 0; i < NELL; ++i) xv[j][i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < OUTM; ++i) acc[j][i] = 0.0f;
        }
        if (!sc_fwd_body<GG, TG>(ring, grp, xv, acc)) return;
        if (!reduce_groups<GG, NG, TG, OUTM>(s, grp, r, tile_it, acc)) {
            if (lane == 0) atomicExch(&mmk_status, 8);
            return;
        }
        if (grp == 0) sc_fwd_store<GG>(acc, nodes, out, c);
    }
}

template <int GG, int NG, int TG>
__global__ void __launch_bounds__(TG * Cpg<NG>::value + 32)
mmk_sc_bwd_kernel(const float *__restrict__ x, const int *__restrict__ perm, const int *__restrict__ erow, int n_elem,
                  const float *__restrict__ T, const float *__restrict__ g, float *__restrict__ gx, long long n_tiles,
                  long long n_nodes) {
    extern __shared__ __align__(128) float smem[];
    constexpr int CPG = Cpg<NG>::value;
    const Smem s = smem_layout(smem);
    sc_setup<NG, TG>(s);
    const int tid = threadIdx.x;
    if (tid >= TG * CPG) {
        sc_produce<NG * GG>(T, erow, n_elem, n_tiles, s);
        return;
    }
    const int grp = tid / CPG, r = tid % CPG, c = r % CH, sub = r / CH;
    const int lane = tid & 31;
    Ring ring{s, 0u, c};
    u32 tile_it = 0;
    for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++tile_it) {
        int e, p0, cnt;
        if (!tile_of<NG * GG>(t, erow, n_elem, e, p0, cnt)) break;
        long long nodes[GG];
        float xv[GG][NELL], gv[GG][OUTM], d[GG][NELL];
#pragma unroll
        for (int j = 0; j < GG; ++j) {
            const int q = sub * GG + j;
            nodes[j] = (sub < NG && q < cnt) ? (long long)perm[p0 + q] : -1;
            if (nodes[j] >= 0 && MMK_BAD_INDEX(nodes[j], n_nodes, 11)) nodes[j] = -1;
            if (nodes[j] >= 0) {
                load_feat(x + (nodes[j] * CH + c) * NELL, xv[j]);
            } else {
#pragma unroll
                for (int i = 0; i < NELL; ++i) xv[j][i] = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < NELL; ++i) d[j][i] = 0.0f;
        }
        sc_load_grad<GG>(g, nodes, c, gv);
        if (!sc_bwd_body<GG, TG>(ring, grp, xv, gv, d)) return;
        if (!reduce_groups<GG, NG, TG, NELL>(s, grp, r, tile_it, d)) {
            if (lane == 0) atomicExch(&mmk_status, 8);
            return;
        }
        if (grp == 0) {
#pragma unroll
            for (int j = 0; j < GG; ++j)
                if (nodes[j] >= 0) store_feat(gx + (nodes[j] * CH + c) * NELL, d[j]);
        }
    }
}
