// sc.cuh -- sm_100a kernels of MACE's symmetric contraction evaluated as a precomputed polynomial.
//
// Compiled by NVRTC with a generated "mmk_layer.h" that bakes in one SymmetricContraction's monomial list
// (reference src/mace_mps_kernels/symmetric.py:52-75 builds the same list): sizes CH (channels), NELL, NROWS, RP (rows
// rounded up to 4), OUTD (output row), OUTM (outputs per channel), the launch shape SC_NT / SC_CC / STAGES, and the
// straight-line term code sc_fwd_body / sc_bwd_body (one (node, channel) each, coefficients read as float4 from the
// channel's column), sc_fwd_store, sc_load_grad.
//
// Coefficient table T[e][c][RP]: one contiguous column of rows per (element, channel).  Row of term t, output m:
// row_t + m.
//
// Work is node-major.  Nodes are grouped by element (perm / erow: the node CSR of the element index).  A unit is
// (node group of SC_NT*32 nodes of one element, chunk of SC_CC channels).  The CTA has SC_NT*SC_CC consumer warps and
// one producer warp: warp (t, j) evaluates channel c = chunk*SC_CC + j of the 32 nodes t*32 .. t*32+31 of the group,
// lane = node.  The producer copies the chunk's SC_CC coefficient columns of element e (SC_CC*RP contiguous floats,
// one TMA bulk copy) into a STAGES-deep ring; within a warp every coefficient load is a broadcast (all lanes read the
// same address), so shared-memory bandwidth is not the limit and each 16-byte load feeds four rows of FMAs.
// Forward: out[b, off + c*M + m] = sum_t T[e, c, row_t + m] x^idx_t.  Backward: gx[b, c, i] = sum_t (sum_m
// T[e, c, row_t + m] g[b, off + c*M + m]) d(x^idx_t)/dx_i.  Waits are bounded as in conv_tp.cuh.
#include "mmk_layer.h"

#ifndef MMK_WAIT_HINT_NS
#define MMK_WAIT_HINT_NS 1000000    // ns a thread may sleep in one mbarrier.try_wait (it wakes when the phase completes)
#endif
#ifndef MMK_WAIT_BUDGET
#define MMK_WAIT_BUDGET (2000000000LL)              // clock64 cycles, ~1 s (MMK_WAIT_CYCLES overrides it)
#endif
#define SC_NWARP (SC_NT * SC_CC)                      // consumer warps
#define SC_NCH ((CH + SC_CC - 1) / SC_CC)             // channel chunks
#define SC_UNIT_NODES (SC_NT * 32)

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
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"((unsigned)MMK_WAIT_HINT_NS)
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

// node group g -> (element, first position in perm, node count) for groups of TN nodes; groups of one element are
// consecutive
template <int TN>
__device__ __forceinline__ bool group_of(long long g, const int *__restrict__ erow, int n_elem, int &e, int &p0,
                                         int &cnt) {
    long long before = 0;
    for (int k = 0; k < n_elem; ++k) {
        const int a = erow[k], b = erow[k + 1];
        const long long ng = (b - a + TN - 1) / TN;
        if (g < before + ng) {
            e = k;
            p0 = a + (int)(g - before) * TN;
            cnt = min(TN, b - p0);
            return true;
        }
        before += ng;
    }
    return false;
}

// Before a consumer warp hands a stage back to the producer: the producer's next TMA copy writes the stage through
// the async proxy, and without a proxy fence those writes are not ordered after this warp's generic-proxy reads of
// the stage (observed on B200: a warp still reading late rows of a column saw the next unit's coefficients).
__device__ __forceinline__ void release_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// shared memory: ring [STAGES][SC_CC][RP] floats | full[STAGES] | empty[STAGES]
struct Smem {
    float *ring;
    u64 *full, *empty;
};

__device__ __forceinline__ Smem smem_setup(float *base) {
    Smem s;
    s.ring = base;
    s.full = reinterpret_cast<u64 *>(base + (size_t)STAGES * SC_CC * RP);
    s.empty = s.full + STAGES;
    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], SC_NWARP);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    return s;
}

// Producer (lane 0 of the last warp): unit u = (node group u / SC_NCH, channel chunk u % SC_NCH); copy the chunk's
// coefficient columns of the group's element into ring position it.
__device__ __forceinline__ void sc_produce(const float *__restrict__ T, const int *__restrict__ erow, int n_elem,
                                           long long n_units, const Smem &s) {
    if ((threadIdx.x & 31) != 0) return;
#ifdef MMK_TEST_STALL
    return;                                       // test build: nothing issued, the consumers' waits run out
#endif
    u32 it = 0;
    bool ok = true;
    for (long long u = blockIdx.x; u < n_units; u += gridDim.x, ++it) {
        int e, p0, cnt;
        if (!group_of<SC_UNIT_NODES>(u / SC_NCH, erow, n_elem, e, p0, cnt)) break;
        const int c0 = (int)(u % SC_NCH) * SC_CC;
        const int cols = min(SC_CC, CH - c0);
        const u32 st = it % STAGES, ph = (it / STAGES) & 1;
        if (!mbar_wait(&s.empty[st], ph ^ 1)) {
            ok = false;
            atomicExch(&mmk_status, 7);
            break;
        }
        const u32 bytes = (u32)cols * RP * 4;
        mbar_arrive_expect_tx(&s.full[st], bytes);
        bulk_g2s(s.ring + (size_t)st * SC_CC * RP, T + ((size_t)e * CH + c0) * RP, bytes, &s.full[st]);
    }
    if (!ok) {                                    // let the copies already issued land before the CTA exits
        const u32 first = it > STAGES ? it - STAGES : 0;
        for (u32 i = first; i < it; ++i) mbar_wait(&s.full[i % STAGES], (i / STAGES) & 1);
    }
}

// Consumer view of one unit: the node of this lane (-1 if none) and the channel of this warp (>= CH if none).
struct Unit {
    long long node;
    int c;
    bool ok;
};

__device__ __forceinline__ Unit unit_of(long long u, const int *__restrict__ perm, const int *__restrict__ erow,
                                        int n_elem, long long n_nodes) {
    Unit r{-1, CH, false};
    int e, p0, cnt;
    if (!group_of<SC_UNIT_NODES>(u / SC_NCH, erow, n_elem, e, p0, cnt)) return r;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = warp / SC_CC, j = warp % SC_CC;
    const int q = t * 32 + lane;
    r.ok = true;
    r.c = (int)(u % SC_NCH) * SC_CC + j;
    if (q < cnt) {
        r.node = perm[p0 + q];
        if (MMK_BAD_INDEX(r.node, n_nodes, 11)) r.node = -1;
    }
    return r;
}

template <int NT, int CC>
__global__ void __launch_bounds__(NT * CC * 32 + 32, SC_MINB)
mmk_sc_fwd_kernel(const float *__restrict__ x, const int *__restrict__ perm, const int *__restrict__ erow, int n_elem,
                  const float *__restrict__ T, float *__restrict__ out, long long n_units, long long n_nodes) {
    static_assert(NT == SC_NT && CC == SC_CC, "launch shape of the generated header");
    extern __shared__ __align__(128) float smem[];
    const Smem s = smem_setup(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == SC_NWARP) {
        sc_produce(T, erow, n_elem, n_units, s);
        return;
    }
    const int j = warp % SC_CC;
    u32 it = 0;
    // the node features of the next unit are loaded while the current unit's terms are evaluated
    Unit nx = unit_of(blockIdx.x, perm, erow, n_elem, n_nodes);
    float xn[NELL];
    if (nx.ok && nx.node >= 0 && nx.c < CH) load_feat(x + (nx.node * CH + nx.c) * NELL, xn);
    for (long long u = blockIdx.x; u < n_units; u += gridDim.x, ++it) {
        const Unit un = nx;
        if (!un.ok) break;
        const bool active = un.node >= 0 && un.c < CH;
        float xv[NELL], acc[OUTM];
#pragma unroll
        for (int i = 0; i < NELL; ++i) xv[i] = active ? xn[i] : 0.0f;
        if (u + gridDim.x < n_units) {
            nx = unit_of(u + gridDim.x, perm, erow, n_elem, n_nodes);
            if (nx.ok && nx.node >= 0 && nx.c < CH) load_feat(x + (nx.node * CH + nx.c) * NELL, xn);
        } else {
            nx.ok = false;
        }
#pragma unroll
        for (int i = 0; i < OUTM; ++i) acc[i] = 0.0f;
        const u32 st = it % STAGES;
        if (!mbar_wait(&s.full[st], (it / STAGES) & 1)) {
            if (lane == 0) atomicExch(&mmk_status, 6);
            return;
        }
        if (un.c < CH) sc_fwd_body(s.ring + ((size_t)st * SC_CC + j) * RP, xv, acc);   // warp-uniform
        release_fence();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[st]);
        if (active) sc_fwd_store(acc, un.node, out, un.c);
    }
}

template <int NT, int CC>
__global__ void __launch_bounds__(NT * CC * 32 + 32, SC_MINB)
mmk_sc_bwd_kernel(const float *__restrict__ x, const int *__restrict__ perm, const int *__restrict__ erow, int n_elem,
                  const float *__restrict__ T, const float *__restrict__ g, float *__restrict__ gx, long long n_units,
                  long long n_nodes) {
    static_assert(NT == SC_NT && CC == SC_CC, "launch shape of the generated header");
    extern __shared__ __align__(128) float smem[];
    const Smem s = smem_setup(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == SC_NWARP) {
        sc_produce(T, erow, n_elem, n_units, s);
        return;
    }
    const int j = warp % SC_CC;
    u32 it = 0;
    // the node features and output gradients of the next unit are loaded while the current unit is evaluated
    Unit nx = unit_of(blockIdx.x, perm, erow, n_elem, n_nodes);
    float xn[NELL], gn[OUTM];
    if (nx.ok && nx.node >= 0 && nx.c < CH) {
        load_feat(x + (nx.node * CH + nx.c) * NELL, xn);
        sc_load_grad(g, nx.node, nx.c, gn);
    }
    for (long long u = blockIdx.x; u < n_units; u += gridDim.x, ++it) {
        const Unit un = nx;
        if (!un.ok) break;
        const bool active = un.node >= 0 && un.c < CH;
        float xv[NELL], gv[OUTM], d[NELL];
#pragma unroll
        for (int i = 0; i < NELL; ++i) xv[i] = active ? xn[i] : 0.0f;
#pragma unroll
        for (int i = 0; i < OUTM; ++i) gv[i] = active ? gn[i] : 0.0f;
        if (u + gridDim.x < n_units) {
            nx = unit_of(u + gridDim.x, perm, erow, n_elem, n_nodes);
            if (nx.ok && nx.node >= 0 && nx.c < CH) {
                load_feat(x + (nx.node * CH + nx.c) * NELL, xn);
                sc_load_grad(g, nx.node, nx.c, gn);
            }
        } else {
            nx.ok = false;
        }
#pragma unroll
        for (int i = 0; i < NELL; ++i) d[i] = 0.0f;
        const u32 st = it % STAGES;
        if (!mbar_wait(&s.full[st], (it / STAGES) & 1)) {
            if (lane == 0) atomicExch(&mmk_status, 6);
            return;
        }
        if (un.c < CH) sc_bwd_body(s.ring + ((size_t)st * SC_CC + j) * RP, xv, gv, d);   // warp-uniform
        release_fence();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[st]);
        if (active) store_feat(gx + (un.node * CH + un.c) * NELL, d);
    }
}
