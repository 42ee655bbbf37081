// conv_tp.cuh -- sm_100a kernels of the MACE interaction convolution (channel-wise weighted uvu tensor product).
//
// Compiled at layer-creation time by NVRTC together with a generated header "mmk_layer.h" that bakes in one
// TensorProduct: the sizes (MUL, XR, YD, ORR, NINS), the row accessors, and the straight-line per-edge bodies
// fwd_edge<H> / bwd_edge<H> of every instruction part H, whose constants are the probed path coefficients (reference
// src/mace_mps_kernels/conv.py:57-88 measures the same numbers).
//
// Both kernels are persistent and warp-specialised:
//   * one producer warp streams, edge by edge in CSR order, the rows an edge needs into a STAGES-deep ring of shared
//     memory with TMA bulk copies (cp.async.bulk, completion counted on a per-stage mbarrier): W[e] (NINS*MUL floats)
//     plus x[sender] (forward) or grad_out[receiver] (backward), plus Y[e] when its row is 16-byte sized;
//   * CG consumer groups take the edges round-robin (ring position it -> group it % CG).  A group is NP parts x
//     MUL/CPT threads: thread (part h, u0) handles channels u0 + q*MUL/CPT (CPT channels per thread) and the
//     instructions of part h (NP threads per channel); every part of a group reads each stage the group owns, then
//     releases it to the producer (after a proxy fence: the next TMA copy into the stage is an async-proxy write).
//     Partial sums of a node over groups and parts are added in shared memory in a fixed order.
// Nodes are cut into chunks dealt round-robin to the CTAs (one contiguous range per CTA, or chunks of a few nodes on
// large graphs so that all CTAs work in one compact window and gathered rows stay in L2); with atoms ordered along a
// space-filling curve a chunk is a compact domain and one stretch of the CSR.
//   forward   node = receiver; out[n] accumulated in registers over the receiver CSR segment, written once:
//             deterministic, no atomics.
//   backward  node = sender; x[s] in registers; per edge gW[e, :, u] (coalesced over u) and gY[e, :] (channel sum:
//             register transpose-reduce in each warp, then the last warp of the group adds the warps' partials in warp
//             order); gx[s] accumulated in registers, written once.  Fuses the reference's conv_bwd_x and conv_bwd_wy
//             (conv.py:144-222), which gather x and grad_out twice.
// Every wait is bounded (about a second of clock64); on expiry the CTA records an error code in mmk_status, the
// producer waits (bounded) for the copies it issued, and the CTA returns -- no trap, no hang.  A test build
// (MMK_TEST_STALL, environment MMK_TEST_STALL=1 at layer creation) has a producer that issues nothing, so the
// consumers' waits run out with no copy in flight and the status path can be checked on a GPU.
#include "mmk_layer.h"

#define X_DIM (XR * MUL)
#define OUT_DIM (ORR * MUL)
#define W_DIM (NINS * MUL)
#define Y_TMA ((YD * 4) % 16 == 0)         // Y rows are copied with TMA when 16-byte sized
// launch bounds: the block size, plus a minimum of resident CTAs per SM when the plan asks for one (MMK_*_MINB > 0;
// it caps the registers per thread), else the register count is left to the compiler
#if MMK_FWD_MINB > 0
#define MMK_FWD_BOUNDS(T) __launch_bounds__(T, MMK_FWD_MINB)
#else
#define MMK_FWD_BOUNDS(T) __launch_bounds__(T)
#endif
#if MMK_BWD_MINB > 0
#define MMK_BWD_BOUNDS(T) __launch_bounds__(T, MMK_BWD_MINB)
#else
#define MMK_BWD_BOUNDS(T) __launch_bounds__(T)
#endif
#ifndef MMK_WAIT_HINT_NS
#define MMK_WAIT_HINT_NS 1000000    // ns a thread may sleep in one mbarrier.try_wait (it wakes when the phase completes)
#endif
#ifndef MMK_WAIT_BUDGET
#define MMK_WAIT_BUDGET (2000000000LL)      // clock64 cycles, ~1 s (MMK_WAIT_CYCLES at layer creation overrides it)
#endif

// Error status of this module's kernels on this device (0 = ok); read and reset by mmk_conv_layer_status().
__device__ int mmk_status;

// With MMK_CHECKS defined (environment MMK_CHECKS=1 at layer creation) every gathered index is range-checked: a bad
// one is recorded in mmk_status (100 + where) and replaced by 0, so the access stays in bounds.
#ifdef MMK_CHECKS
#define MMK_CHECK_INDEX(v, n, where)                          \
    do {                                                      \
        if ((v) < 0 || (v) >= (n)) {                          \
            atomicExch(&mmk_status, 100 + (where));           \
            (v) = 0;                                          \
        }                                                     \
    } while (0)
#else
#define MMK_CHECK_INDEX(v, n, where) \
    do {                             \
    } while (0)
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
// bounded wait: false after about MMK_WAIT_BUDGET cycles
__device__ __forceinline__ bool mbar_wait(u64 *bar, u32 parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > MMK_WAIT_BUDGET) return false;
    }
    return true;
}
// Before a consumer warp releases a ring stage: the producer's next TMA copy writes the stage through the async proxy,
// and only a proxy fence orders those writes after this warp's generic-proxy reads of the stage.
__device__ __forceinline__ void release_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, u32 bytes, u64 *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// The same copy with an L2 eviction-priority hint (the per-edge rows W[e] and Y[e] are read exactly once: streamed
// with evict_first so that they do not push the gathered node rows, which other edges read again, out of L2).
__device__ __forceinline__ u64 l2_evict_first() {
    u64 p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, u32 bytes, u64 *bar, u64 pol) {
#if MMK_L2_HINT
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
#else
    bulk_g2s(dst, src, bytes, bar);
#endif
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

// Work split: the nodes are cut into chunks of nb consecutive nodes and CTA b takes chunks b, b + G, b + 2G, ...
// (G = gridDim.x).  The host picks nb: either N / G (one contiguous range per CTA: a compact domain when atoms are
// ordered along a space-filling curve, its edges one stretch of the CSR) or a few nodes (all CTAs then work inside one
// compact window of G*nb atoms at a time, so the rows they gather stay in L2).  Every chunk is a contiguous stretch of
// the CSR.
// Edge-balanced split (small graphs: nb < 0): CTA c of G takes the CSR positions [q0, q1) = [E c / G, E (c+1) / G),
// so every CTA has the same number of edges whatever the node degrees; its nodes are those with an edge in the range
// plus the edgeless nodes whose row starts in it.  A node whose edges straddle a boundary is computed in pieces:
// every CTA but the one holding the node's last edge writes its piece of the node's row to part[2c] and raises
// flags[c]; the CTA holding the last edge keeps its own piece in part[2c + 1] and, after its range, waits (bounded) for
// the flags of the earlier pieces and writes the row as the sum of the pieces in CTA order (deterministic).  A CTA
// raises its flag before it waits, and waits only on lower CTAs, so the chain resolves; the grid is never larger than
// the CTAs resident at once.  Node-chunk mode (nb > 0) has q0 = 0, q1 = E: no clipping, no pieces.
struct ERange {
    long long q0, q1, n_first, n_end;
};

__device__ __forceinline__ long long rowptr_lower_bound(const int *__restrict__ rowptr, long long n_nodes,
                                                        long long q) {
    long long lo = 0, hi = n_nodes;                          // rowptr[n_nodes] = E >= q
    while (lo < hi) {
        const long long mid = (lo + hi) >> 1;
        if (rowptr[mid] >= q) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

__device__ __forceinline__ ERange edge_range(const int *__restrict__ rowptr, long long n_nodes, long long n_edges,
                                             long long nb) {
    ERange r{0, n_edges, 0, n_nodes};
    if (nb >= 0) return r;
    const long long c = blockIdx.x, G = gridDim.x;
    r.q0 = n_edges * c / G;
    r.q1 = n_edges * (c + 1) / G;
    const long long lo = rowptr_lower_bound(rowptr, n_nodes, r.q0);
    r.n_first = (lo > 0 && rowptr[lo] > r.q0) ? lo - 1 : lo;          // lo - 1: a node continued from CTA c - 1
    r.n_end = c == G - 1 ? n_nodes : rowptr_lower_bound(rowptr, n_nodes, r.q1);
    return r;
}

// CTA c' whose range holds CSR position q
__device__ __forceinline__ long long cta_of_edge(long long q, long long n_edges) {
    const long long G = gridDim.x;
    long long c = q * G / (n_edges > 0 ? n_edges : 1);
    while (c + 1 < G && n_edges * (c + 1) / G <= q) ++c;
    while (c > 0 && n_edges * c / G > q) --c;
    return c;
}

__device__ __forceinline__ bool next_chunk(long long &c, long long nb, long long n_nodes, const ERange &er,
                                           long long &n0, long long &n1) {
    if (nb < 0) {                                            // edge-balanced: one range per CTA
        if (c != blockIdx.x) return false;
        n0 = er.n_first;
        n1 = er.n_end;
        c += gridDim.x;
        return true;
    }
    if (c * nb >= n_nodes) return false;
    n0 = c * nb;
    n1 = min(n_nodes, n0 + nb);
    c += gridDim.x;
    return true;
}

// Where the finished row of node n goes: the output row when the CTA holds all of n's edges, else its piece's slot
// (part[2c] when later CTAs hold more of n's edges, part[2c + 1] when this CTA holds the last ones).
__device__ __forceinline__ float *row_of_node(float *out, float *part, long long n, int row, const int *rowptr,
                                              const ERange &er) {
    const bool head = rowptr[n] < er.q0, tail = rowptr[n + 1] > er.q1;
    if (!head && !tail) return out + n * (long long)row;
    return part + (2LL * blockIdx.x + (tail ? 0 : 1)) * row;
}

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(int *p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// End of an edge-balanced range, run by every consumer thread (ct = consumer thread index, NC = consumer threads):
// publish this CTA's piece of its last node, then finish its first node if the CTA holds that node's last edges.
// Every warp arrives on `done` once its stores are fenced; thread 0 waits for all of them, raises the flag, waits
// for the flags of the earlier pieces and releases the others through `go`.  All waits are bounded.
template <int NC>
__device__ __forceinline__ void finish_pieces(float *out, float *part, int *flags, int row, const int *rowptr,
                                              const ERange &er, long long n_edges, u64 *done, u64 *go, int ct,
                                              int lane) {
    const long long c = blockIdx.x;
    const bool any = er.n_end > er.n_first;
    const bool publish = any && rowptr[er.n_end] > er.q1;
    const bool finalize = any && rowptr[er.n_first] < er.q0 && rowptr[er.n_first + 1] <= er.q1;
    __threadfence();                                         // this thread's rows, visible GPU-wide
    __syncwarp();
    if (lane == 0) mbar_arrive(done);
    long long c_first = c;
    if (finalize) c_first = cta_of_edge(rowptr[er.n_first], n_edges);
    __shared__ int pieces_ok;
    if (ct == 0) {
        bool ok = mbar_wait(done, 0);
        if (ok && publish) st_release(&flags[c], 1);
        if (ok && finalize) {
            for (long long k = c_first; k < c && ok; ++k) {
                const long long t0 = clock64();
                while (ld_acquire(&flags[k]) == 0)
                    if (clock64() - t0 > MMK_WAIT_BUDGET) {
                        ok = false;
                        break;
                    }
            }
            for (long long k = c_first; k < c; ++k) flags[k] = 0;   // read once: ready for the next launch
        }
        if (!ok) atomicExch(&mmk_status, 10);
        pieces_ok = ok ? 1 : 0;
        mbar_arrive(go);
        if (!ok) return;
    }
    if (!finalize) return;
    if (!mbar_wait(go, 0)) {
        if (lane == 0) atomicExch(&mmk_status, 11);
        return;
    }
    if (!pieces_ok) return;                                  // thread 0 gave up on the flags: leave the row
    // the row = earlier pieces in CTA order, then this CTA's own; rows are whole float4 (MUL is a multiple of 32) and
    // each thread sums 8 float4 at a time so that the loads of a piece are in flight together
    float4 *dst = reinterpret_cast<float4 *>(out + er.n_first * (long long)row);
    const float4 *p4 = reinterpret_cast<const float4 *>(part);
    const int row4 = row / 4;
#pragma unroll 1
    for (int b0 = ct; b0 < row4; b0 += 8 * NC) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
        for (long long k = c_first; k <= c; ++k) {
            const long long slot = k < c ? 2 * k : 2 * c + 1;
            float4 t[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = b0 + u * NC;
                t[u] = i < row4 ? __ldcg(p4 + slot * row4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u].x += t[u].x; v[u].y += t[u].y; v[u].z += t[u].z; v[u].w += t[u].w;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (b0 + u * NC < row4) dst[b0 + u * NC] = v[u];
    }
}

// Producer: stream the TMA copies of the CTA's edges [rowptr[n0], rowptr[n1]) in CSR order.  The warp fetches the
// edge ids (and the gathered node of each edge) 32 at a time, one batch ahead, so the index loads overlap the issue of
// the current batch; each lane then waits for its own ring slot and issues its edge's copies, so up to
// min(32, STAGES) edges are issued at once.  False on a timeout.
template <int STAGES, class Issue>
__device__ __forceinline__ bool produce(const int *__restrict__ rowptr, const int *__restrict__ eids,
                                        const long long *__restrict__ other, long long n0, long long n1,
                                        const ERange &er, long long n_nodes, long long n_edges, u64 *full, u64 *empty,
                                        u32 &it, Issue issue) {
    const int lane = threadIdx.x & 31;
    if (n0 >= n1) return true;
    const int q0 = (int)max((long long)rowptr[n0], er.q0), q1 = (int)min((long long)rowptr[n1], er.q1);
    long long e_next = 0, o_next = 0;
    if (q0 + lane < q1) {
        e_next = eids[q0 + lane];
        MMK_CHECK_INDEX(e_next, n_edges, 1);
        o_next = other[e_next];
        MMK_CHECK_INDEX(o_next, n_nodes, 2);
    }
    for (int q = q0; q < q1; q += 32) {
        const long long e = e_next, o = o_next;
        if (q + 32 + lane < q1) {                  // next batch: in flight while this one is issued
            e_next = eids[q + 32 + lane];
            MMK_CHECK_INDEX(e_next, n_edges, 1);
            o_next = other[e_next];
            MMK_CHECK_INDEX(o_next, n_nodes, 2);
        }
        // lanes issue in parallel, in rounds of ROUND edges (one ring slot each; lane j of the batch owns ring position
        // it + j).  A round waits for the slowest of its slots, so ROUND is a fraction of the ring (STAGES / 2 by
        // default): the slots of the next round are being refilled while the current round is consumed.
        constexpr int ROUND = STAGES / MMK_ROUND_DIV < 1 ? 1 : (STAGES / MMK_ROUND_DIV > 32 ? 32 : STAGES / MMK_ROUND_DIV);
        const int cnt = min(32, q1 - q);
        for (int j0 = 0; j0 < cnt; j0 += ROUND) {
            const int j = j0 + lane;
            const long long ej = __shfl_sync(0xffffffffu, e, j & 31);
            const long long oj = __shfl_sync(0xffffffffu, o, j & 31);
            const bool mine = lane < ROUND && j < cnt;
            const u32 i = it + j, st = i % STAGES;
            bool ok = true;
            if (mine) {
                ok = mbar_wait(&empty[st], ((i / STAGES) & 1) ^ 1);
                if (ok) issue(st, ej, oj, &full[st]);
            }
            if (!__all_sync(0xffffffffu, ok)) {
                // a slot never came free: let every copy already issued land before the CTA exits
                if (mine && ok) mbar_wait(&full[st], (i / STAGES) & 1);
                if (lane == 0) {
                    const u32 last = it + j0, first = last > STAGES ? last - STAGES : 0;
                    for (u32 k = first; k < last; ++k) mbar_wait(&full[k % STAGES], (k / STAGES) & 1);
                }
                return false;
            }
        }
        it += cnt;
    }
    return true;
}


// Consumer groups: the CG groups of MUL threads of a CTA take the CTA's edge stream round-robin (ring position it ->
// group it % CG), so one node's edges are worked on by CG*MUL/32 warps at once; their partial sums of a node are added
// in shared memory in group order (deterministic).  STAGES is a multiple of CG, so every ring slot always belongs to
// the same group: a group only ever waits for the next phase of its own slots, never for a phase of a slot another
// group has not released yet (an mbarrier parity wait cannot tell phases two apart).  The hand-over buffer has two halves (node parity); red_full[h] completes
// when groups 1.. have written half h, red_free[h] when group 0 has read it.
template <int CG, int CPT, int K>
__device__ __forceinline__ bool reduce_groups(u64 *red_full, u64 *red_free, float *red, int grp, int u0, u32 node_it,
                                              float (&v)[CPT][K]) {
    if constexpr (CG == 1) {
        return true;
    } else {
        constexpr int GT = MUL / CPT;
        const u32 h = node_it & 1, ph = (node_it >> 1) & 1;
        float *buf = red + (size_t)h * (CG - 1) * K * MUL;
        const int lane = threadIdx.x & 31;
        if (grp > 0) {
            if (!mbar_wait(&red_free[h], ph ^ 1)) return false;
            float *dst = buf + (size_t)(grp - 1) * K * MUL + u0;
#pragma unroll
            for (int q = 0; q < CPT; ++q)
#pragma unroll
                for (int i = 0; i < K; ++i) dst[i * MUL + q * GT] = v[q][i];
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_full[h]);
        } else {
            if (!mbar_wait(&red_full[h], ph)) return false;
#pragma unroll
            for (int g = 0; g < CG - 1; ++g) {
                const float *src = buf + (size_t)g * K * MUL + u0;
#pragma unroll
                for (int q = 0; q < CPT; ++q)
#pragma unroll
                    for (int i = 0; i < K; ++i) v[q][i] += src[i * MUL + q * GT];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_free[h]);
        }
        return true;
    }
}

// Y[e] of a stage: four 16-byte shared-memory loads (the same address in every lane: broadcast) when the row was
// copied with TMA, else read from global memory.
__device__ __forceinline__ void load_y(const float *ys, const float *__restrict__ Y, long long e, float (&y)[YD]) {
    if constexpr (Y_TMA) {
#pragma unroll
        for (int j = 0; j < YD / 4; ++j) {
            const float4 q = reinterpret_cast<const float4 *>(ys)[j];
            y[4 * j] = q.x; y[4 * j + 1] = q.y; y[4 * j + 2] = q.z; y[4 * j + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < YD; ++j) y[j] = __ldg(Y + e * YD + j);
    }
}

__device__ __forceinline__ void init_barriers(u64 *full, u64 *empty, int stages, u32 ncw, u64 *extra, int n_extra,
                                              u32 extra_count, u64 *extra2, int n_extra2, u32 extra2_count,
                                              u64 *edone, u32 n_cons_warps) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ncw);
        }
        for (int i = 0; i < n_extra; ++i) mbar_init(&extra[i], extra_count);
        for (int i = 0; i < n_extra2; ++i) mbar_init(&extra2[i], extra2_count);
        mbar_init(&edone[0], n_cons_warps);                  // edge-balanced split: consumer warps done
        mbar_init(&edone[1], 1);                             // ... and the pieces of the first node are ready
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
}

// ------------------------------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------------------------------
// Consumer code of part H of a group (the forward's per-thread work; see mmk_conv_fwd_kernel).
template <int STAGES, int CG, int CPT, int NP, int H>
__device__ __forceinline__ void fwd_consume(const float *smem, u64 *full, u64 *empty, u64 *red_full, u64 *red_free,
                                            float *red, const float *__restrict__ Y, const int *__restrict__ rowptr,
                                            float *__restrict__ out, long long n_nodes, long long n_edges,
                                            long long nb, const ERange &er, float *part, int *flags, u64 *edone,
                                            int grp, int u0, int lane) {
    constexpr int GT = MUL / CPT;
    constexpr u32 STAGE_F = W_DIM + X_DIM + 20;
    u32 it = 0, node_it = 0;
    long long chunk = blockIdx.x, n0, n1;
    while (next_chunk(chunk, nb, n_nodes, er, n0, n1))
    for (long long n = n0; n < n1; ++n, ++node_it) {
        float acc[CPT][ORR];
#pragma unroll
        for (int q = 0; q < CPT; ++q)
#pragma unroll
            for (int i = 0; i < ORR; ++i) acc[q][i] = 0.0f;
        const int p0 = (int)max((long long)rowptr[n], er.q0), p1 = (int)min((long long)rowptr[n + 1], er.q1);
        for (int p = p0; p < p1; ++p, ++it) {
            if (it % CG != (u32)grp) continue;  // ring position it is always group it % CG's (STAGES % CG == 0)
            const u32 st = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[st], ph)) {
                if (lane == 0) atomicExch(&mmk_status, 2);
                return;
            }
            const float *stage = smem + st * STAGE_F;
            float xs[CPT][XR], y[YD], w[CPT][NINS];
            load_y(stage + W_DIM + X_DIM, Y, *reinterpret_cast<const long long *>(stage + W_DIM + X_DIM + 16), y);
#pragma unroll
            for (int q = 0; q < CPT; ++q) {
                const int u = u0 + q * GT;
                fwd_load_w<H>(stage, u, w[q]);
                load_x_s(stage + W_DIM, u, xs[q]);
            }
            release_fence();
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
            for (int q = 0; q < CPT; ++q) fwd_edge<H>(xs[q], y, w[q], acc[q]);
        }
        if (!reduce_groups<CG, CPT, ORR>(red_full, red_free, red, grp, u0, node_it, acc)) {
            if (lane == 0) atomicExch(&mmk_status, 9);
            return;
        }
        if (grp == 0) {
            float *row = row_of_node(out, part, n, OUT_DIM, rowptr, er);
#pragma unroll
            for (int q = 0; q < CPT; ++q) fwd_store<H>(row, u0 + q * GT, acc[q]);
        }
    }
    if (nb < 0)
        finish_pieces<CG * NP * GT>(out, part, flags, OUT_DIM, rowptr, er, n_edges, &edone[0], &edone[1],
                                    (int)threadIdx.x, lane);
}

// CTA = CG consumer groups x NP parts x GT = MUL / CPT threads (+ the producer warp).  Thread (grp, part, u0) computes,
// for channels u0 + q*GT (q < CPT), the outputs of part `part` of the instructions; every part of a group reads every
// stage the group owns.  With NP > 1 the plan runs one group (no cross-group sum of the outputs).
template <int STAGES, int CG, int CPT, int NP>
__global__ void MMK_FWD_BOUNDS(CG * NP * (MUL / CPT) + 32)
mmk_conv_fwd_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                    const int *__restrict__ rowptr, const int *__restrict__ eids,
                    const long long *__restrict__ senders, float *__restrict__ out, long long n_nodes,
                    long long n_edges, long long nb, float *pieces, int *piece_flags) {
    static_assert(NP == 1 || CG == 1, "a forward split over parts runs one consumer group");
    constexpr int GT = MUL / CPT;                   // threads of one part of a group
    constexpr u32 NCW = GT / 32;                    // warps of one part
    constexpr int GTH = NP * GT;                    // threads of one group
    constexpr u32 STAGE_F = W_DIM + X_DIM + 20;     // floats per stage: W row | x row | Y row (16) | edge id (4)
    extern __shared__ __align__(128) float smem[];
    u64 *full = reinterpret_cast<u64 *>(smem + STAGES * STAGE_F);
    u64 *empty = full + STAGES;
    u64 *red_full = empty + STAGES;                 // [2]
    u64 *red_free = red_full + 2;                   // [2]
    u64 *edone = red_free + 2;                      // [2] edge-balanced split
    float *red = reinterpret_cast<float *>(edone + 2);      // [2][CG-1][ORR][MUL]
    const int tid = threadIdx.x;
    init_barriers(full, empty, STAGES, NP * NCW, red_full, 2, CG > 1 ? (CG - 1) * NCW : 1, red_free, 2, NCW, edone,
                  CG * NP * NCW);
    const ERange er = edge_range(rowptr, n_nodes, n_edges, nb);

    if (tid >= CG * GTH) {                          // producer warp
#ifdef MMK_TEST_STALL
        return;
#endif
        u32 it = 0;
        const u64 pol = l2_evict_first();
        auto issue = [&](u32 st, long long e, long long s, u64 *bar) {
            float *stage = smem + st * STAGE_F;
            *reinterpret_cast<long long *>(stage + W_DIM + X_DIM + 16) = e;       // released by the arrive below
            mbar_arrive_expect_tx(bar, (W_DIM + X_DIM) * 4 + (Y_TMA ? YD * 4 : 0));
            bulk_g2s_stream(stage, W + e * W_DIM, W_DIM * 4, bar, pol);
            bulk_g2s(stage + W_DIM, x + s * X_DIM, X_DIM * 4, bar);
            if constexpr (Y_TMA) bulk_g2s_stream(stage + W_DIM + X_DIM, Y + e * YD, YD * 4, bar, pol);
        };
        long long chunk = blockIdx.x, n0, n1;
        while (next_chunk(chunk, nb, n_nodes, er, n0, n1)) {
            if (!produce<STAGES>(rowptr, eids, senders, n0, n1, er, n_nodes, n_edges, full, empty, it, issue)) {
                if ((tid & 31) == 0) atomicExch(&mmk_status, 1);
                break;
            }
        }
        return;
    }

    const int grp = tid / GTH, part = (tid % GTH) / GT, u0 = tid % GT, lane = tid & 31;
    if (part == 0) fwd_consume<STAGES, CG, CPT, NP, 0>(smem, full, empty, red_full, red_free, red, Y, rowptr, out, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, u0, lane);
    if constexpr (NP > 1) {
        if (part == 1) fwd_consume<STAGES, CG, CPT, NP, 1>(smem, full, empty, red_full, red_free, red, Y, rowptr, out, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, u0, lane);
    }
    if constexpr (NP > 2) {
        if (part == 2) fwd_consume<STAGES, CG, CPT, NP, 2>(smem, full, empty, red_full, red_free, red, Y, rowptr, out, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, u0, lane);
        if (part == 3) fwd_consume<STAGES, CG, CPT, NP, 3>(smem, full, empty, red_full, red_free, red, Y, rowptr, out, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, u0, lane);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------------------------------
// Consumer code of part H of a group (the backward's per-thread work; see mmk_conv_bwd_kernel).
template <int STAGES, int CG, int CPT, int NP, int H>
__device__ __forceinline__ void bwd_consume(const float *smem, u64 *full, u64 *empty, u64 *red_full, u64 *red_free,
                                            float *red, float *part_buf, int *arrived, const float *__restrict__ x,
                                            const float *__restrict__ Y, const int *__restrict__ rowptr,
                                            float *__restrict__ gx, float *__restrict__ gY, float *__restrict__ gW,
                                            long long n_nodes, long long n_edges, long long nb, const ERange &er,
                                            float *part, int *flags, u64 *edone, int grp, int lg, int u0, int gwarp,
                                            int lane) {
    constexpr int GT = MUL / CPT;
    constexpr u32 GW = NP * (GT / 32);
    constexpr u32 STAGE_F = W_DIM + OUT_DIM + 20;
    u32 it = 0, node_it = 0;
    long long chunk = blockIdx.x, n0, n1;
    while (next_chunk(chunk, nb, n_nodes, er, n0, n1))
    for (long long s = n0; s < n1; ++s, ++node_it) {
        float xs[CPT][XR], gxa[CPT][XR];
#pragma unroll
        for (int q = 0; q < CPT; ++q) {
            load_x(x + s * X_DIM, u0 + q * GT, xs[q]);
#pragma unroll
            for (int i = 0; i < XR; ++i) gxa[q][i] = 0.0f;
        }
        const int p0 = (int)max((long long)rowptr[s], er.q0), p1 = (int)min((long long)rowptr[s + 1], er.q1);
        for (int p = p0; p < p1; ++p, ++it) {
            if (it % CG != (u32)grp) continue;  // ring position it is always group it % CG's (STAGES % CG == 0)
            const u32 st = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[st], ph)) {
                if (lane == 0) atomicExch(&mmk_status, 4);
                return;
            }
            const float *stage = smem + st * STAGE_F;
            long long e = *reinterpret_cast<const long long *>(stage + W_DIM + OUT_DIM + 16);
            MMK_CHECK_INDEX(e, n_edges, 3);
            float y[YD], gy[16];
            load_y(stage + W_DIM + OUT_DIM, Y, e, y);
#pragma unroll
            for (int j = 0; j < 16; ++j) gy[j] = 0.0f;
#pragma unroll
            for (int q = 0; q < CPT; ++q) {
                const int u = u0 + q * GT;
                float w[NINS], go[ORR], gw[NINS];
                bwd_load_w<H>(stage, u, w);
                bwd_load_g<H>(stage + W_DIM, u, go);
                bwd_edge<H>(xs[q], y, w, go, gxa[q], gw, gy);
                if (gW != nullptr) bwd_store_gw<H>(gW + e * W_DIM + u, gw);
            }
            if (gY != nullptr) {
                // channel sum of gY[e]: each warp reduces its channels in registers and leaves 16 partials in the
                // stage's slot; the warp that finishes last adds the GW partials in warp order (deterministic),
                // writes gY[e] and clears the counter.  The stage is released only afterwards, so the slot is
                // free.
                float *pb = part_buf + (size_t)st * GW * 16;
                const float v = warp_transpose_reduce16(gy);
                if ((lane & 1) == 0) pb[gwarp * 16 + (lane >> 1)] = v;
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd(&arrived[st], 1) == (int)GW - 1;
                    if (last) __threadfence_block();
                }
                if (__shfl_sync(0xffffffffu, last, 0)) {
                    if (lane < YD) {
                        float t = 0.0f;
#pragma unroll
                        for (int w8 = 0; w8 < (int)GW; ++w8) t += pb[w8 * 16 + lane];
                        gY[e * YD + lane] = t;
                    }
                    if (lane == 0) arrived[st] = 0;
                }
            }
            release_fence();
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        if (!reduce_groups<CG * NP, CPT, XR>(red_full, red_free, red, lg, u0, node_it, gxa)) {
            if (lane == 0) atomicExch(&mmk_status, 9);
            return;
        }
        if (gx != nullptr && lg == 0) {
            float *row = row_of_node(gx, part, s, X_DIM, rowptr, er);
#pragma unroll
            for (int q = 0; q < CPT; ++q) store_x(row, u0 + q * GT, gxa[q]);
        }
    }
    if (nb < 0 && gx != nullptr)
        finish_pieces<CG * NP * GT>(gx, part, flags, X_DIM, rowptr, er, n_edges, &edone[0], &edone[1],
                                    (int)threadIdx.x, lane);
}

// Same CTA shape.  The CG*NP (group, part) pairs are the "logical groups" of the gx sum at the end of a sender: each
// holds a partial gx[s] (its edges, its instructions), added in shared memory in logical-group order.
template <int STAGES, int CG, int CPT, int NP>
__global__ void MMK_BWD_BOUNDS(CG * NP * (MUL / CPT) + 32)
mmk_conv_bwd_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                    const float *__restrict__ g, const int *__restrict__ rowptr, const int *__restrict__ eids,
                    const long long *__restrict__ receivers, float *__restrict__ gx, float *__restrict__ gY,
                    float *__restrict__ gW, long long n_nodes, long long n_edges, long long nb, float *pieces,
                    int *piece_flags) {
    constexpr int GT = MUL / CPT;                   // threads of one part of a group
    constexpr u32 NCW = GT / 32;                    // warps of one part
    constexpr int GTH = NP * GT;                    // threads of one group
    constexpr u32 GW = NP * NCW;                    // warps of one group
    constexpr u32 STAGE_F = W_DIM + OUT_DIM + 20;   // W row | grad_out row | Y row (16) | edge id (4)
    extern __shared__ __align__(128) float smem[];
    u64 *full = reinterpret_cast<u64 *>(smem + STAGES * STAGE_F);
    u64 *empty = full + STAGES;
    u64 *red_full = empty + STAGES;                 // [2]   gx hand-over between logical groups
    u64 *red_free = red_full + 2;                   // [2]
    u64 *edone = red_free + 2;                      // [2] edge-balanced split
    float *part_buf = reinterpret_cast<float *>(edone + 2);         // [STAGES][GW][16] gY partials of each warp
    int *arrived = reinterpret_cast<int *>(part_buf + STAGES * GW * 16);   // [STAGES] warps done with the stage's gY
    float *red = reinterpret_cast<float *>(arrived + STAGES);       // [2][CG*NP-1][XR][MUL]
    const int tid = threadIdx.x;
    for (int i = tid; i < STAGES; i += blockDim.x) arrived[i] = 0;
    init_barriers(full, empty, STAGES, GW, red_full, 2, CG * NP > 1 ? (CG * NP - 1) * NCW : 1, red_free, 2, NCW, edone,
                  CG * NP * NCW);
    const ERange er = edge_range(rowptr, n_nodes, n_edges, nb);

    if (tid >= CG * GTH) {
#ifdef MMK_TEST_STALL
        return;
#endif
        u32 it = 0;
        const u64 pol = l2_evict_first();
        auto issue = [&](u32 st, long long e, long long r, u64 *bar) {
            float *stage = smem + st * STAGE_F;
            *reinterpret_cast<long long *>(stage + W_DIM + OUT_DIM + 16) = e;     // released by the arrive below
            mbar_arrive_expect_tx(bar, (W_DIM + OUT_DIM) * 4 + (Y_TMA ? YD * 4 : 0));
            bulk_g2s_stream(stage, W + e * W_DIM, W_DIM * 4, bar, pol);
            bulk_g2s(stage + W_DIM, g + r * OUT_DIM, OUT_DIM * 4, bar);
            if constexpr (Y_TMA) bulk_g2s_stream(stage + W_DIM + OUT_DIM, Y + e * YD, YD * 4, bar, pol);
        };
        long long chunk = blockIdx.x, n0, n1;
        while (next_chunk(chunk, nb, n_nodes, er, n0, n1)) {
            if (!produce<STAGES>(rowptr, eids, receivers, n0, n1, er, n_nodes, n_edges, full, empty, it, issue)) {
                if ((tid & 31) == 0) atomicExch(&mmk_status, 3);
                break;
            }
        }
        return;
    }

    const int grp = tid / GTH, part = (tid % GTH) / GT, u0 = tid % GT;
    const int gwarp = (tid % GTH) >> 5, lane = tid & 31;   // warp index within the group (all parts)
    const int lg = grp * NP + part;                        // logical group of the gx sum
    if (part == 0) bwd_consume<STAGES, CG, CPT, NP, 0>(smem, full, empty, red_full, red_free, red, part_buf, arrived, x, Y, rowptr, gx, gY, gW, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, lg, u0, gwarp, lane);
    if constexpr (NP > 1) {
        if (part == 1) bwd_consume<STAGES, CG, CPT, NP, 1>(smem, full, empty, red_full, red_free, red, part_buf, arrived, x, Y, rowptr, gx, gY, gW, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, lg, u0, gwarp, lane);
    }
    if constexpr (NP > 2) {
        if (part == 2) bwd_consume<STAGES, CG, CPT, NP, 2>(smem, full, empty, red_full, red_free, red, part_buf, arrived, x, Y, rowptr, gx, gY, gW, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, lg, u0, gwarp, lane);
        if (part == 3) bwd_consume<STAGES, CG, CPT, NP, 3>(smem, full, empty, red_full, red_free, red, part_buf, arrived, x, Y, rowptr, gx, gY, gW, n_nodes, n_edges, nb, er, pieces, piece_flags, edone, grp, lg, u0, gwarp, lane);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// forward on the tensor cores (layers with MUL = 128; the generated header defines MMK_FWD_TC 1 and its helpers)
// ------------------------------------------------------------------------------------------------------------------
// Per edge e (sender s) and x block b: t[u, n] = sum_a x[s, u, a] M_b,e[a, n] with M_b,e[a, n] = sum_j c Y[e, j]
// (the columns n of block b are its instructions' output components), then out[r, k, u, m] += W[e, k, u] t[u, n(k,m)].
// The product runs on tcgen05 (kind::tf32, M = 128 channels in the TMEM lanes, K = 8 per block, N = the block's
// columns padded to 16) with the 3xTF32 split (x = hi + lo and M = hi + lo; lo.hi + hi.lo + hi.hi into one fresh
// accumulator per edge, so at most 3 MMAs add into it), the rest on the CUDA cores.  Warps of a CTA
// (32 (4 TC_NG + 2) threads):
//   0 .. 4 TC_NG - 1  compute: warp w serves channels u = 32 (w % 4) + lane (the TMEM lane quadrant w % 4 it may
//        read) and column group w / 4: the 16-column TMEM groups of the layer are dealt over the TC_NG groups, and
//        so are the output accumulators (every output component belongs to one column).  For the edge LAG ahead
//        of its epilogue a warp stages its share of A (x[s] row of the TMA ring -> TF32 parts) and of B (entries of
//        M_e from Y[e], spread over all compute threads); then the epilogue of the edge: its columns from tensor
//        memory (all loads issued before one wait), W from the ring, out accumulated in registers over the
//        receiver's edges, written once;
//   4 TC_NG       producer: the TMA ring of (W[e], x[s], Y[e], e), as in the CUDA-core forward;
//   4 TC_NG + 1   MMA: lane 0 issues the edge's MMAs into its TMEM slot once A and B are staged and the slot's
//        previous epilogue is done, and commits them to t_full.
// Edge slots (A, B, 128 TMEM columns) form a ring of NS.  A compute warp restages slot (q mod NS) only after its own
// wait for the MMAs of edge q - NS (its epilogue of that edge), so the operands are free when it writes them.  Every
// wait is bounded and every role reaches the teardown (tensor memory freed) also on the error path.
#if MMK_FWD_TC
__device__ __forceinline__ float tc_rna(float v) {
    u32 r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}
__device__ __forceinline__ void tc_st4(u32 addr, float a, float b, float c, float d) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
// 16-byte piece c (K = 4c .. 4c+3) of A row u, split into the high and low TF32 tiles (128-byte swizzle)
__device__ __forceinline__ void tc_put_a(u32 a_hi, u32 a_lo, int u, int c, const float (&v)[4]) {
    const u32 off = (u32)u * 128u + ((u32)(c ^ (u & 7)) << 4);
    float h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[i] = tc_rna(v[i]);
        l[i] = tc_rna(v[i] - h[i]);
    }
    tc_st4(a_hi + off, h[0], h[1], h[2], h[3]);
    tc_st4(a_lo + off, l[0], l[1], l[2], l[3]);
}
// 16 consecutive TMEM columns of this thread's lane; the values are valid after tc_wait_ld()
__device__ __forceinline__ void tc_ld16(u32 taddr, u32 (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ unsigned long long tc_desc(u32 saddr) {      // K-major, 128-byte swizzle, 8-row groups 1 KB apart
    return (unsigned long long)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((unsigned long long)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void tc_mma(u32 d, unsigned long long a, unsigned long long b, u32 idesc, u32 acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(u64 *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// the CTA's edges in order: node chunks dealt round-robin (nb nodes each), nodes in order, CSR edges in order
struct TcCursor {
    long long chunk, n, n1;
    int p, p1;
    bool live;
};
__device__ __forceinline__ void tc_open(TcCursor &c, const int *rowptr, long long nb, long long n_nodes) {
    c.chunk = blockIdx.x;
    c.live = false;
    for (; c.chunk * nb < n_nodes; c.chunk += gridDim.x) {
        for (c.n = c.chunk * nb, c.n1 = min(n_nodes, c.chunk * nb + nb); c.n < c.n1; ++c.n) {
            c.p = rowptr[c.n];
            c.p1 = rowptr[c.n + 1];
            if (c.p < c.p1) {
                c.live = true;
                return;
            }
        }
    }
}
__device__ __forceinline__ void tc_next(TcCursor &c, const int *rowptr, long long nb, long long n_nodes) {
    if (++c.p < c.p1) return;
    for (++c.n;; ++c.n) {
        if (c.n >= c.n1) {
            c.chunk += gridDim.x;
            if (c.chunk * nb >= n_nodes) {
                c.live = false;
                return;
            }
            c.n = c.chunk * nb;
            c.n1 = min(n_nodes, c.n + nb);
        }
        c.p = rowptr[c.n];
        c.p1 = rowptr[c.n + 1];
        if (c.p < c.p1) return;
    }
}

template <int STAGES, int NS>
__global__ void __launch_bounds__(32 * (4 * TC_NG + 2), 1)
mmk_conv_fwd_tc_kernel(const float *__restrict__ x, const float *__restrict__ Y, const float *__restrict__ W,
                       const int *__restrict__ rowptr, const int *__restrict__ eids,
                       const long long *__restrict__ senders, float *__restrict__ out, long long n_nodes,
                       long long n_edges, long long nb) {
    constexpr int NCW = 4 * TC_NG;                    // compute warps
    constexpr int LAG = NS - 1;                       // edges staged ahead of the epilogue
    constexpr u32 STAGE_F = W_DIM + X_DIM + 20;       // W row | x row | Y row (16) | edge id (4)
    constexpr u32 A_BYTES = 128 * 128, B_BYTES = TC_BROWS * 128, SLOT = 2 * A_BYTES + 2 * B_BYTES;
    static_assert(MUL == 128 && YD == 16, "tensor-core forward: 128 channels, Y rows of 16");
    static_assert(STAGES > LAG, "the ring must hold the staged edges");
    extern __shared__ __align__(1024) float smem_tc[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<unsigned long long>(smem_tc) + 1023) & ~1023ull);
    const u32 slots = smem_addr(base);
    float *ring = reinterpret_cast<float *>(base + NS * SLOT);
    u64 *full = reinterpret_cast<u64 *>(ring + STAGES * STAGE_F);
    u64 *empty = full + STAGES;
    u64 *ab_full = empty + STAGES;                    // [NS] the compute warps staged A and B
    u64 *t_full = ab_full + NS;                       // [NS] the edge's MMAs completed
    u64 *t_free = t_full + NS;                        // [NS] the edge's epilogue read its TMEM slot
    u32 *tmem_box = reinterpret_cast<u32 *>(t_free + NS);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        for (int s = 0; s < NS; ++s) {
            mbar_init(&ab_full[s], NCW);
            mbar_init(&t_full[s], 1);
            mbar_init(&t_free[s], NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the B tiles are written only at their structurally nonzero entries: everything else must read as zero
    for (u32 i = tid; i < NS * 2 * B_BYTES / 16; i += blockDim.x) {
        const u32 sl = i / (2 * B_BYTES / 16), o = (i % (2 * B_BYTES / 16)) * 16;
        tc_st4(slots + sl * SLOT + 2 * A_BYTES + o, 0.f, 0.f, 0.f, 0.f);
    }
    release_fence();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tmem_box))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const u32 tmem = *tmem_box;
    const ERange er{0, n_edges, 0, n_nodes};

    if (warp == NCW) {                                 // producer
#ifndef MMK_TEST_STALL
        u32 it = 0;
        auto issue = [&](u32 st, long long e, long long s, u64 *bar) {
            float *stage = ring + st * STAGE_F;
            *reinterpret_cast<long long *>(stage + W_DIM + X_DIM + 16) = e;
            mbar_arrive_expect_tx(bar, (W_DIM + X_DIM + YD) * 4);
            bulk_g2s(stage, W + e * W_DIM, W_DIM * 4, bar);
            bulk_g2s(stage + W_DIM, x + s * X_DIM, X_DIM * 4, bar);
            bulk_g2s(stage + W_DIM + X_DIM, Y + e * YD, YD * 4, bar);
        };
        long long chunk = blockIdx.x, n0, n1;
        while (next_chunk(chunk, nb, n_nodes, er, n0, n1)) {
            if (!produce<STAGES>(rowptr, eids, senders, n0, n1, er, n_nodes, n_edges, full, empty, it, issue)) {
                if (lane == 0) atomicExch(&mmk_status, 1);
                break;
            }
        }
#endif
    } else if (warp == NCW + 1) {                      // MMA issue
        TcCursor c;
        tc_open(c, rowptr, nb, n_nodes);
        bool ok = true;
        long long issued = -1;                         // last edge whose MMAs were committed
        for (u32 q = 0; c.live && ok; ++q, tc_next(c, rowptr, nb, n_nodes)) {
            const u32 sl = q % NS;
            ok = __all_sync(0xffffffffu,
                            mbar_wait(&ab_full[sl], (q / NS) & 1) && mbar_wait(&t_free[sl], ((q / NS) & 1) ^ 1));
            if (!ok) break;
            if (lane == 0) {
                tc_fence_after();
                const u32 a_hi = slots + sl * SLOT, a_lo = a_hi + A_BYTES, b_hi = a_hi + 2 * A_BYTES, b_lo = b_hi + B_BYTES;
#pragma unroll
                for (int b = 0; b < TC_NB; ++b) {
                    const u32 d = tmem + sl * 128 + tc_col0(b);
                    const u32 idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((u32)(tc_ncol(b) >> 3) << 17) | ((128u >> 4) << 24);
                    const u32 ko = 32u * b;
                    tc_mma(d, tc_desc(a_lo + ko), tc_desc(b_hi + ko), idesc, 0u);
                    tc_mma(d, tc_desc(a_hi + ko), tc_desc(b_lo + ko), idesc, 1u);
                    tc_mma(d, tc_desc(a_hi + ko), tc_desc(b_hi + ko), idesc, 1u);
                }
                tc_commit(&t_full[sl]);
            }
            issued = q;
            __syncwarp();
        }
        if (!ok && lane == 0) atomicExch(&mmk_status, 12);
        // the tensor memory is freed at the end: wait (bounded) for the last committed MMAs
        if (issued >= 0) mbar_wait(&t_full[issued % NS], (u32)(issued / NS) & 1);
    } else if (warp < NCW) {                           // compute: channel u, column group g
        const int g = warp >> 2, u = ((warp & 3) << 5) | lane;
        const u32 tlane = (u32)((warp & 3) * 32) << 16;
        TcCursor cs;                                   // staging cursor, LAG edges ahead of the epilogue
        tc_open(cs, rowptr, nb, n_nodes);
        bool ok = true;
        u32 qs = 0, qe = 0;
        float acc[TC_ACC];
#pragma unroll
        for (int i = 0; i < TC_ACC; ++i) acc[i] = 0.0f;
        // nodes in order; edgeless nodes are written as zeros
        long long chunk = blockIdx.x, n0, n1;
        while (ok && next_chunk(chunk, nb, n_nodes, er, n0, n1))
            for (long long n = n0; n < n1 && ok; ++n) {
                for (int p = rowptr[n]; p < rowptr[n + 1] && ok; ++p, ++qe) {
                    while (cs.live && qs <= qe + LAG) {  // stage A and B of edge qs
                        const u32 st = qs % STAGES, sl = qs % NS;
                        if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (qs / STAGES) & 1))) {
                            ok = false;
                            break;
                        }
                        const float *stage = ring + st * STAGE_F;
                        const u32 a_hi = slots + sl * SLOT, a_lo = a_hi + A_BYTES;
                        const u32 b_hi = a_hi + 2 * A_BYTES, b_lo = b_hi + B_BYTES;
                        tc_stage_a(g, stage + W_DIM, u, a_hi, a_lo);
                        const float *ys = stage + W_DIM + X_DIM;
                        for (int i = tid; i < TC_NE; i += 32 * NCW) {
                            float v = 0.0f;
#pragma unroll
                            for (int j = 0; j < TC_EMAX; ++j) v = fmaf(tc_e_c[i * TC_EMAX + j], ys[tc_e_y[i * TC_EMAX + j]], v);
                            const float hv = tc_rna(v), lv = tc_rna(v - hv);
                            const u32 o = tc_e_off[i];
                            asm volatile("st.shared.f32 [%0], %1;" ::"r"(b_hi + o), "f"(hv) : "memory");
                            asm volatile("st.shared.f32 [%0], %1;" ::"r"(b_lo + o), "f"(lv) : "memory");
                        }
                        release_fence();               // A and B written (generic) -> read by the MMA (async proxy)
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&ab_full[sl]);
                        ++qs;
                        tc_next(cs, rowptr, nb, n_nodes);
                    }
                    if (!ok) break;
                    const u32 st = qe % STAGES, sl = qe % NS;
                    if (!__all_sync(0xffffffffu, mbar_wait(&t_full[sl], (qe / NS) & 1))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    tc_epilogue(g, ring + st * STAGE_F, u, tmem + tlane + sl * 128, acc);
                    tc_fence_before();
                    release_fence();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&t_free[sl]);
                        mbar_arrive(&empty[st]);
                    }
                }
                if (!ok) break;
                tc_store(g, out + n * OUT_DIM, u, acc);
#pragma unroll
                for (int i = 0; i < TC_ACC; ++i) acc[i] = 0.0f;
            }
        if (!ok && lane == 0) atomicExch(&mmk_status, 13);
    }
    // teardown: wait (bounded) until the last MMAs completed, then free the tensor memory
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}
#endif
