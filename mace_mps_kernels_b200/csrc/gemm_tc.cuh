// gemm_tc.cuh -- float32 GEMM on the 5th-generation tensor cores of sm_100a (tcgen05.mma kind::tf32, accumulator in
// tensor memory), with the 3xTF32 split for float32 accuracy:
//
//     C[M, N] = A[M, K] . B[N, K]^T          (A, B row-major with K contiguous: "K-major" operands)
//
// a = a_hi + a_lo with a_hi = tf32(a) (round to nearest) and a_lo = tf32(a - a_hi); the product is accumulated in
// float32 as a_lo.b_hi + a_hi.b_lo + a_hi.b_hi (the a_lo.b_lo term, ~2^-22 relative, is dropped), which keeps the
// error at the float32 level (~1e-6 relative for these K) instead of TF32's ~1e-3.  B is a constant operand here (the
// weights of a layer), so the caller passes it already split (mmk_tf32_split); A is split while it is staged.
//
// Accumulation: the tensor cores add into the float32 accumulator without round-to-nearest, so its error grows with
// the number of MMAs that add into it (measured: ~7x a float32 SIMT product at K = 1280 with one accumulator).  The
// kernel therefore keeps 2 x KS accumulators in tensor memory: the hi.hi products and the two small cross products
// in separate ones, and the K chunks dealt round-robin over KS such pairs; the epilogue adds them on the CUDA cores.
//
// One CTA of 8 warps computes a 128 x BN tile of C (BN = 64 / 128 / 256 columns of tensor memory, lane = row):
//   * every K chunk of 32 (one 128-byte row of each operand) is staged by all 256 threads into a ring of STAGES
//     shared-memory stages in the 128B-swizzled K-major layout the MMA descriptors describe (16-byte piece c of row r
//     stored at r*128 + ((c ^ (r % 8)) * 16); 4 rows per warp instruction, coalesced 128-byte row reads);
//   * thread 0 issues, per chunk, 4 K-steps x 3 products of tcgen05.mma (M = 128, N = BN, K = 8) and commits them to
//     the stage's mbarrier; the threads stage the next chunk meanwhile and wait on that barrier only before they
//     overwrite the stage;
//   * the epilogue reads the accumulator back with tcgen05.ld (warps w and w + 4: lanes 32w..32w+31, each half of
//     the columns, 16 at a time),
//     stages the tile in shared memory and stores whole rows (coalesced);
//   * the next chunk is in flight while a chunk is split and multiplied: its A in registers, its (already split) B
//     by cp.async straight into the swizzled tiles;
//   * outputs with fewer tiles than SMs split K over a third grid dimension; partial tiles go to a caller-provided
//     workspace and the last CTA of a tile adds them in split order (deterministic).
// Every wait is bounded; on expiry the kernel records a status (mmk_gemm_status), still waits (bounded) for its MMAs,
// frees its tensor memory and returns.

namespace mmk_gemm {

__device__ int g_status;

constexpr int BM = 128;                 // tile rows = MMA M = tensor-memory lanes
constexpr int NW = 8;                   // warps per CTA (two per tensor-memory lane quadrant)
constexpr int NT = 32 * NW;             // threads per CTA
constexpr int BK = 32;                  // K chunk: 32 floats = one 128-byte swizzle row
constexpr long long WAIT_BUDGET = 2000000000LL;   // clock64 cycles (~1 s)
// a waiting thread sleeps in mbarrier.try_wait until the phase completes or this many ns pass, instead of spinning
constexpr unsigned WAIT_HINT_NS = 1000000;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"((unsigned)WAIT_HINT_NS)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > WAIT_BUDGET) return false;
    return true;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte swizzled layout: rows of 128 bytes,
// groups of 8 rows 1024 bytes apart (stride byte offset), descriptor version 1 (sm_100), swizzle mode 2 (128 B).
// The leading byte offset is not used by swizzled K-major layouts.  Tiles start on 1024-byte boundaries; the K-step
// j of a chunk starts 32*j bytes into the row (the hardware applies the swizzle to the full address).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::tf32: D float32, A and B tf32, both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <int M, int N>
__host__ __device__ constexpr uint32_t idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// A chunk (ROWS rows x 32 floats of K) of a K-major matrix: warp w, instruction i loads rows 4*NW*i + 4*w + lane/8,
// 16-byte piece lane % 8 (coalesced: 8 lanes read one 128-byte row).  Rows or columns out of range are zero.
template <int ROWS>
struct Chunk {
    float4 v[ROWS / (4 * NW)];
};

template <int ROWS>
__device__ __forceinline__ void load_chunk(Chunk<ROWS> &ch, const float *__restrict__ src, long long ld,
                                           long long rows, int K, int k0) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int k = k0 + 4 * (lane & 7);
#pragma unroll
    for (int i = 0; i < ROWS / (4 * NW); ++i) {
        const int r = 4 * NW * i + 4 * warp + (lane >> 3);
        ch.v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows && k < K) ch.v[i] = __ldg(reinterpret_cast<const float4 *>(src + (long long)r * ld + k));
    }
}

// Byte offset of 16-byte piece c of row r in a 128B-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4); }

// Split a staged chunk into its TF32 high and low parts, stored in the swizzled tiles at hi / lo.
template <int ROWS>
__device__ __forceinline__ void store_split(const Chunk<ROWS> &ch, uint32_t hi, uint32_t lo) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c = lane & 7;
#pragma unroll
    for (int i = 0; i < ROWS / (4 * NW); ++i) {
        const int r = 4 * NW * i + 4 * warp + (lane >> 3);
        const float4 v = ch.v[i];
        const float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
        const float4 l = make_float4(tf32_rna(v.x - h.x), tf32_rna(v.y - h.y), tf32_rna(v.z - h.z), tf32_rna(v.w - h.w));
        st_shared_v4(hi + sw128_off(r, c), h);
        st_shared_v4(lo + sw128_off(r, c), l);
    }
}

// Copy a chunk of an already split operand straight into its swizzled tile with cp.async (16 bytes per thread and
// instruction, no registers); out-of-range pieces are zero-filled (src-size 0).
template <int ROWS>
__device__ __forceinline__ void async_chunk(uint32_t dst, const float *__restrict__ src, long long ld, long long rows,
                                            int K, int k0) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c = lane & 7;
    const int k = k0 + 4 * c;
#pragma unroll
    for (int i = 0; i < ROWS / (4 * NW); ++i) {
        const int r = 4 * NW * i + 4 * warp + (lane >> 3);
        const bool in = r < rows && k < K;
        const float *g = in ? src + (long long)r * ld + k : src;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst + sw128_off(r, c)), "l"(g),
                     "r"(in ? 16 : 0)
                     : "memory");
    }
}

// C tile: thread (warp w, lane l) holds row 32 (w % 4) + l of the accumulator; the tile goes through shared memory
// (row stride BN + 4 floats: the 16-byte stores of a warp fall on distinct banks) so that global stores are whole
// rows.
template <int BN>
__device__ __forceinline__ void tile_to_smem(float *tile, const float (&v)[16], int j) {
    const int row = 32 * ((threadIdx.x >> 5) & 3) + (threadIdx.x & 31);
#pragma unroll
    for (int q = 0; q < 16; q += 4)
        *reinterpret_cast<float4 *>(tile + row * (BN + 4) + j + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
}

// Rows [0, 128) x columns [0, ncols) of the smem tile -> dst (row stride ld), warp w writing rows w, w + NW, ...
template <int BN>
__device__ __forceinline__ void smem_to_rows(float *__restrict__ dst, long long ld, const float *tile, long long rows,
                                             int ncols) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = warp; r < BM && r < rows; r += NW) {
        const float *src = tile + r * (BN + 4);
        float *d = dst + (long long)r * ld;
        for (int c = 4 * lane; c < ncols; c += 128) {
            if (c + 4 <= ncols) {
                *reinterpret_cast<float4 *>(d + c) = *reinterpret_cast<const float4 *>(src + c);
            } else {
                for (int q = c; q < ncols; ++q) d[q] = src[q];
            }
        }
    }
}

// grid (M tiles, N tiles, K splits).  With K splits > 1 every CTA writes its partial tile to ws (tile-major,
// [split][tile][128][BN]) and the CTA that arrives last for a tile (counter per tile, back to zero afterwards) adds
// the partials in split order -- deterministic whichever CTA is last.
template <int BN, int STAGES, int KS>
__global__ void __launch_bounds__(NT, 1)
k_gemm_tf32x3(const float *__restrict__ A, long long lda, const float *__restrict__ Bhi,
              const float *__restrict__ Blo, long long ldb, float *__restrict__ C, long long ldc, long long M, int N,
              int K, float *__restrict__ ws, int *__restrict__ counters) {
    static_assert(BN == 64 || BN == 128 || BN == 256, "tensor-memory columns: a power of two, M = 128 needs N % 16");
    static_assert(2 * KS * BN <= 512, "2 x KS accumulators of BN columns in the 512 columns of tensor memory");
    constexpr uint32_t TCOLS = 2 * KS * BN;
    constexpr uint32_t A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4;
    constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static_assert(STAGES * STAGE_BYTES >= BM * (BN + 4) * 4, "the C tile reuses the operand stages");
    constexpr uint32_t IDESC = idesc_tf32<BM, BN>();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + STAGES);
    int *last_flag = reinterpret_cast<int *>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long m0 = (long long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const int nk_all = (K + BK - 1) / BK, splits = gridDim.z;
    const int kz0 = (int)((long long)nk_all * blockIdx.z / splits), kz1 = (int)((long long)nk_all * (blockIdx.z + 1) / splits);
    const int nk = kz1 - kz0;                                 // chunks of this CTA

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const float *Ab = A + m0 * lda;
    const float *Bh = Bhi + (long long)n0 * ldb, *Bl = Blo + (long long)n0 * ldb;
    const long long rows_a = M - m0, rows_b = (long long)N - n0;
    bool ok = true;
    int committed = -1;                                       // last chunk whose MMAs thread 0 committed
    Chunk<BM> a_next;
    if (nk > 0) {                                             // prologue: chunk 0 in flight
        const uint32_t base = smem_u32(smem);
        async_chunk<BN>(base + 2 * A_BYTES, Bh, ldb, rows_b, K, kz0 * BK);
        async_chunk<BN>(base + 2 * A_BYTES + B_BYTES, Bl, ldb, rows_b, K, kz0 * BK);
        asm volatile("cp.async.commit_group;" ::: "memory");
        load_chunk<BM>(a_next, Ab, lda, rows_a, K, kz0 * BK);
    }
    for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
        store_split<BM>(a_next, base, base + A_BYTES);        // this chunk's A (its stage was freed before its B)
        bool free_ = true;
        if (i + 1 < nk) {                                     // next chunk: B by cp.async, A into registers
            const int s1 = (i + 1) % STAGES;
            const uint32_t b1 = smem_u32(smem + s1 * STAGE_BYTES);
            // stage s1 is free once the MMAs of its previous use (chunk i + 1 - STAGES) have completed
            free_ = i + 1 < STAGES || mbar_wait(&bars[s1], (uint32_t)(((i + 1) / STAGES) - 1) & 1u);
            if (free_) {
                async_chunk<BN>(b1 + 2 * A_BYTES, Bh, ldb, rows_b, K, (kz0 + i + 1) * BK);
                async_chunk<BN>(b1 + 2 * A_BYTES + B_BYTES, Bl, ldb, rows_b, K, (kz0 + i + 1) * BK);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            load_chunk<BM>(a_next, Ab, lda, rows_a, K, (kz0 + i + 1) * BK);
            asm volatile("cp.async.wait_group 1;" ::: "memory");   // this chunk's B has landed
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");    // generic writes -> tensor-core reads
        tc_fence_before();
        if (!__syncthreads_and(free_)) {                      // block-uniform: stop if any thread gave up
            ok = false;
            break;
        }
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a_hi = base, a_lo = base + A_BYTES, b_hi = base + 2 * A_BYTES, b_lo = b_hi + B_BYTES;
            const uint32_t big = tmem + (uint32_t)(2 * (i % KS) * BN), small = big + BN;   // this chunk's pair
            const bool first = i < KS;
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
                const uint32_t o = 32u * j, acc = (first && j == 0) ? 0u : 1u;
                mma_tf32(small, sw128_desc(a_lo + o), sw128_desc(b_hi + o), IDESC, acc);
                mma_tf32(small, sw128_desc(a_hi + o), sw128_desc(b_lo + o), IDESC, 1u);
                mma_tf32(big, sw128_desc(a_hi + o), sw128_desc(b_hi + o), IDESC, acc);
            }
            mma_commit(&bars[s]);
        }
        committed = i;
        __syncwarp();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // the barrier of the last committed chunk tracks every MMA issued before it
    bool done = committed < 0 ||
                mbar_wait(&bars[committed % STAGES], (uint32_t)(committed / STAGES) & 1u);
    done = __syncthreads_and(done) != 0;
    tc_fence_after();
    float *tile = reinterpret_cast<float *>(smem);            // the operand stages are free now
    if (ok && done) {
        // warps w and w + 4 read the lane quadrant w % 4, each half of the columns
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const int npairs = nk < KS ? nk : KS;               // accumulator pairs that received MMAs
        const int j0 = (warp >> 2) * (BN / 2);
#pragma unroll 1
        for (int j = j0; j < j0 + BN / 2; j += 16) {
            float v[16], w[16], t[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] = w[q] = 0.0f;
#pragma unroll 1
            for (int q = 0; q < npairs; ++q) {
                tmem_ld16(lane_base + (uint32_t)(2 * q * BN + BN + j), t);   // small cross products
#pragma unroll
                for (int r = 0; r < 16; ++r) w[r] += t[r];
                tmem_ld16(lane_base + (uint32_t)(2 * q * BN + j), t);        // hi.hi products
#pragma unroll
                for (int r = 0; r < 16; ++r) v[r] += t[r];
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) v[r] += w[r];
            tile_to_smem<BN>(tile, v, j);
        }
    } else if (tid == 0) {
        atomicExch(&g_status, done ? 1 : 2);
    }
    tc_fence_before();
    const bool good = __syncthreads_and(ok && done) != 0;     // the tile is complete in shared memory
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
    if (!good) return;
    const int ncols = min(BN, N - n0);
    if (splits == 1) {
        smem_to_rows<BN>(C + m0 * ldc + n0, ldc, tile, rows_a, ncols);
        return;
    }
    const long long n_tiles = (long long)gridDim.x * gridDim.y;
    const long long tile_id = (long long)blockIdx.y * gridDim.x + blockIdx.x;
    smem_to_rows<BN>(ws + ((long long)blockIdx.z * n_tiles + tile_id) * BM * BN, BN, tile, BM, BN);
    __threadfence();
    __syncthreads();
    if (tid == 0) *last_flag = atomicAdd(&counters[tile_id], 1) == splits - 1;
    __syncthreads();
    if (!*last_flag) return;
    __threadfence();
    // partials added in split order; each thread sums 8 float4 of the tile at a time (independent loads in flight)
    constexpr int PER = BM * BN / 4 / NT;                     // float4 of the tile per thread
    const float4 *part4 = reinterpret_cast<const float4 *>(ws + tile_id * BM * BN);
    const long long split_stride4 = n_tiles * BM * BN / 4;
#pragma unroll 1
    for (int b0 = 0; b0 < PER; b0 += 8) {
        float4 acc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
        for (int z = 0; z < splits; ++z) {
            float4 t[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) t[u] = __ldcg(part4 + z * split_stride4 + tid + (b0 + u) * NT);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                acc[u].x += t[u].x; acc[u].y += t[u].y; acc[u].z += t[u].z; acc[u].w += t[u].w;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int q = (tid + (b0 + u) * NT) * 4, r = q / BN, c = q % BN;
            if (r >= rows_a || c >= ncols) continue;
            float *d = C + (m0 + r) * ldc + n0 + c;
            if (c + 4 <= ncols) {
                *reinterpret_cast<float4 *>(d) = acc[u];
            } else {
                const float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
                for (int k = 0; k < ncols - c; ++k) d[k] = a4[k];
            }
        }
    }
    if (tid == 0) counters[tile_id] = 0;                      // ready for the next launch
}

__global__ void k_tf32_split(const float *__restrict__ x, float *__restrict__ hi, float *__restrict__ lo,
                             long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float h = tf32_rna(x[i]);
        hi[i] = h;
        lo[i] = tf32_rna(x[i] - h);
    }
}

template <int BN, int STAGES>
constexpr int smem_bytes() {
    return STAGES * (2 * BM * BK * 4 + 2 * BN * BK * 4) + STAGES * 8 + 16 + 1024;
}

// K splits of a launch when the output has few tiles: as many as keep tiles x splits within one wave (one CTA per SM:
// a second, partial wave would double the launch), at least 4 chunks per split.
inline int gemm_splits(long long tiles, int nk, int sms) {
    if (tiles >= sms || nk < 8) return 1;
    long long s = sms / tiles;
    s = s < nk / 4 ? s : nk / 4;
    return (int)(s < 1 ? 1 : (s > 16 ? 16 : s));
}

}  // namespace mmk_gemm
