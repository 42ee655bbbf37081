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
// One CTA of 4 warps computes a 128 x BN tile of C (BN = 64 / 128 / 256 columns of tensor memory, lane = row):
//   * every K chunk of 32 (one 128-byte row of each operand) is staged by all 128 threads into a ring of STAGES
//     shared-memory stages in the 128B-swizzled K-major layout the MMA descriptors describe (16-byte piece c of row r
//     stored at r*128 + ((c ^ (r % 8)) * 16); 4 rows per warp instruction, coalesced 128-byte row reads);
//   * thread 0 issues, per chunk, 4 K-steps x 3 products of tcgen05.mma (M = 128, N = BN, K = 8) and commits them to
//     the stage's mbarrier; the threads stage the next chunk meanwhile and wait on that barrier only before they
//     overwrite the stage;
//   * the epilogue reads the accumulator back with tcgen05.ld (warp w: lanes 32w..32w+31, 32 columns at a time) and
//     stores the rows.
// Every wait is bounded; on expiry the kernel records a status (mmk_gemm_status), still waits (bounded) for its MMAs,
// frees its tensor memory and returns.

namespace mmk_gemm {

__device__ int g_status;

constexpr int BM = 128;                 // tile rows = MMA M = tensor-memory lanes
constexpr int BK = 32;                  // K chunk: 32 floats = one 128-byte swizzle row
constexpr long long WAIT_BUDGET = 2000000000LL;   // clock64 cycles (~1 s)

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
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
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

// Stage rows [0, ROWS) x floats [k0, k0 + 32) of a K-major matrix (row stride ld floats, `rows` valid rows, K valid
// columns) into the swizzled tile at `hi` (and its TF32 split at hi / lo when SPLIT).  Warp w, instruction i: rows
// 16*i + 4*w + lane/8, 16-byte piece lane % 8.  Rows or columns out of range are zero.
template <int ROWS, bool SPLIT>
__device__ __forceinline__ void stage_rows(const float *__restrict__ src, long long ld, long long rows, int K, int k0,
                                           uint32_t hi, uint32_t lo) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c = lane & 7;
    const int k = k0 + 4 * c;
    constexpr int IT = ROWS / 16;
    float4 v[IT];
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const int r = 16 * i + 4 * warp + (lane >> 3);
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rows && k < K) v[i] = __ldg(reinterpret_cast<const float4 *>(src + (long long)r * ld + k));
    }
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const int r = 16 * i + 4 * warp + (lane >> 3);
        const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
        if constexpr (SPLIT) {
            const float4 h = make_float4(tf32_rna(v[i].x), tf32_rna(v[i].y), tf32_rna(v[i].z), tf32_rna(v[i].w));
            const float4 l = make_float4(tf32_rna(v[i].x - h.x), tf32_rna(v[i].y - h.y), tf32_rna(v[i].z - h.z),
                                         tf32_rna(v[i].w - h.w));
            st_shared_v4(hi + off, h);
            st_shared_v4(lo + off, l);
        } else {
            st_shared_v4(hi + off, v[i]);
        }
    }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(128, 1)
k_gemm_tf32x3(const float *__restrict__ A, long long lda, const float *__restrict__ Bhi,
              const float *__restrict__ Blo, long long ldb, float *__restrict__ C, long long ldc, long long M, int N,
              int K) {
    static_assert(BN == 64 || BN == 128 || BN == 256, "tensor-memory columns: a power of two, M = 128 needs N % 16");
    constexpr uint32_t A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4;
    constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    constexpr uint32_t IDESC = idesc_tf32<BM, BN>();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + STAGES);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long m0 = (long long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN)
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
    const int nk = (K + BK - 1) / BK;
    bool ok = true;
    int committed = -1;                                       // last chunk whose MMAs thread 0 committed
    for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % STAGES;
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
        // the stage is free once the MMAs of chunk kc - STAGES (its previous use) have completed
        const bool free_ = kc < STAGES || mbar_wait(&bars[s], (uint32_t)((kc / STAGES) - 1) & 1u);
        if (free_) {
            stage_rows<BM, true>(Ab, lda, rows_a, K, kc * BK, base, base + A_BYTES);
            stage_rows<BN, false>(Bh, ldb, rows_b, K, kc * BK, base + 2 * A_BYTES, 0);
            stage_rows<BN, false>(Bl, ldb, rows_b, K, kc * BK, base + 2 * A_BYTES + B_BYTES, 0);
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
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
                const uint32_t o = 32u * j;
                mma_tf32(tmem, sw128_desc(a_lo + o), sw128_desc(b_hi + o), IDESC, (kc > 0 || j > 0) ? 1u : 0u);
                mma_tf32(tmem, sw128_desc(a_hi + o), sw128_desc(b_lo + o), IDESC, 1u);
                mma_tf32(tmem, sw128_desc(a_hi + o), sw128_desc(b_hi + o), IDESC, 1u);
            }
            mma_commit(&bars[s]);
        }
        committed = kc;
        __syncwarp();
    }
    // the barrier of the last committed chunk tracks every MMA issued before it
    bool done = committed < 0 ||
                mbar_wait(&bars[committed % STAGES], (uint32_t)(committed / STAGES) & 1u);
    done = __syncthreads_and(done) != 0;
    tc_fence_after();
    if (ok && done) {
        const long long row = m0 + warp * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int j = 0; j < BN; j += 16) {
            float v[16];
            tmem_ld16(lane_base + (uint32_t)j, v);
            const int col = n0 + j;
            if (row < M && col < N) {
                float *dst = C + row * ldc + col;
                if (col + 16 <= N) {
#pragma unroll
                    for (int q = 0; q < 16; q += 4)
                        *reinterpret_cast<float4 *>(dst + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
                } else {
                    for (int q = 0; q < N - col; ++q) dst[q] = v[q];
                }
            }
        }
    } else if (tid == 0) {
        atomicExch(&g_status, done ? 1 : 2);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
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

}  // namespace mmk_gemm
