/*
 * mmk.h -- C ABI of the B200 (sm_100a) MACE kernels: the interaction convolution ``conv_tp`` (gather -> channel-wise
 * weighted uvu tensor product -> scatter-sum over receivers) and the symmetric contraction (product basis), each
 * with forward and first-order backward, plus the receiver/sender CSR builder they run on.
 *
 * Conventions for every entry point:
 *   - all tensor arguments are DEVICE pointers to contiguous row-major arrays owned by the caller; the library never
 *     allocates tensor memory on these paths (per-layer constant tables are owned by the layer handles);
 *   - ``stream`` is a cudaStream_t (NULL = legacy default stream); work is only enqueued, nothing synchronises;
 *   - return value 0 (MMK_OK) on success, otherwise an MMK_ERR_* code; ``mmk_last_error()`` gives a message
 *     (thread-local, valid until the next call from the same thread);
 *   - fp32 data, int32 CSR arrays, int64 edge indices (PyTorch's edge_index dtype).
 *
 * Layouts (e3nn "mul_ir", per node / edge), MUL = channels per irrep block:
 *   x   [N, X_DIM]        x block i (degree l_i): x_off[i] + u*(2 l_i + 1) + m
 *   Y   [E, Y_DIM]        Y block j (multiplicity 1): y_off[j] + m
 *   W   [E, NINS*MUL]     instruction k, channel u at k*MUL + u
 *   out [N, OUT_DIM]      output block o: o_off[o] + u*(2 l_o + 1) + m
 *   out[n] = sum_{e : receiver(e) = n} TP(x[sender(e)], Y[e], W[e])
 */
#ifndef MMK_H
#define MMK_H

#include <stddef.h>
#include <stdint.h>

#if defined(MMK_BUILD)
#define MMK_API __attribute__((visibility("default")))
#else
#define MMK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MMK_OK 0
#define MMK_ERR_INVALID 1       /* bad descriptor or argument (message says which)      */
#define MMK_ERR_COMPILE 2       /* NVRTC failed on the generated layer source             */
#define MMK_ERR_CUDA 3          /* a CUDA runtime call failed                             */
#define MMK_ERR_UNSUPPORTED 4   /* valid request this build does not implement            */

MMK_API const char *mmk_last_error(void);
/* library version, e.g. "0.1.0" */
MMK_API const char *mmk_version(void);

/* ------------------------------------------------------------------------------------------------------------------
 * conv_tp layer
 * ---------------------------------------------------------------------------------------------------------------- */

/* Description of one uvu TensorProduct (what reference src/mace_mps_kernels/conv.py:57-88 ``ConvSpec`` holds).
 * terms: the effective coefficient c of path (instruction k, x component a, Y component b, output component m),
 * i.e. CG x normalisation x path weight exactly as the probed TensorProduct applies it. */
typedef struct mmk_conv_desc {
    int mul;                 /* channels per block, a multiple of 32 (reference conv.py:43-44)          */
    int n_in1;               /* number of x blocks                                                      */
    const int *in1_l;        /* [n_in1] degree of each x block, layout order                            */
    int n_in2;               /* number of Y blocks (multiplicity 1 each)                                */
    const int *in2_l;        /* [n_in2]                                                                 */
    int n_out;               /* number of output blocks                                                 */
    const int *out_l;        /* [n_out]                                                                 */
    int nins;                /* number of instructions                                                  */
    const int *ins_i1;       /* [nins] x block of instruction k                                         */
    const int *ins_i2;       /* [nins] Y block                                                          */
    const int *ins_io;       /* [nins] output block (several instructions may share one: they sum)      */
    int nterms;              /* number of nonzero coefficients                                          */
    const int *term_ins;     /* [nterms] instruction k                                                  */
    const int *term_a;       /* [nterms] component of the x block, 0..2 l1                              */
    const int *term_b;       /* [nterms] component of the Y block, 0..2 l2                              */
    const int *term_m;       /* [nterms] component of the output block, 0..2 l3                         */
    const double *term_c;    /* [nterms] coefficient                                                    */
} mmk_conv_desc;

typedef struct mmk_conv_layer mmk_conv_layer;

/* Generates the layer's specialised sm_100a kernels (coefficients baked in as constants), compiles them with NVRTC
 * and loads them.  Replaces ``MetalConvTP.__init__`` -> ``ConvSpec`` + ``torch.mps.compile_shader(source(spec))``
 * (reference src/mace_mps_kernels/conv.py:277-282).  Identical descriptors share one compiled module.  The handle also
 * owns, on the device current at creation, the scratch of the edge-balanced work split that small graphs use (two
 * rows per CTA for the pieces of nodes whose edges straddle CTA ranges, and one flag per CTA): forward and backward
 * launches of one handle must therefore be ordered (one stream, or explicit events); on another device the handle
 * falls back to node ranges. */
MMK_API int mmk_conv_layer_create(const mmk_conv_desc *desc, mmk_conv_layer **layer);
MMK_API int mmk_conv_layer_destroy(mmk_conv_layer *layer);
/* dims of a created layer: x_dim, y_dim, out_dim, w_dim (= nins*mul) */
MMK_API int mmk_conv_layer_dims(const mmk_conv_layer *layer, int *x_dim, int *y_dim, int *out_dim, int *w_dim);
/* NVRTC-compile the generated source without loading it (needs no GPU); for build checks and tests. */
MMK_API int mmk_conv_compile_check(const mmk_conv_desc *desc);
/* The generated layer header (sizes, launch plan and the straight-line per-edge bodies with the baked coefficients)
 * for this descriptor, as the reference's ``source(spec)`` returns its generated Metal source (conv.py:225-226).
 * Copies at most cap bytes (NUL-terminated when it fits) and sets *len to the full length; buf may be NULL. */
MMK_API int mmk_conv_source(const mmk_conv_desc *desc, char *buf, size_t cap, size_t *len);
/* Error status of the layer's kernels on the current device (0 = ok; nonzero = a pipeline wait gave up and the kernel
 * returned early, its outputs are invalid).  Synchronises with the device; reset != 0 clears it. */
MMK_API int mmk_conv_layer_status(const mmk_conv_layer *layer, int32_t *status, int reset);

/* Forward: out[n] = sum over the receiver-CSR segment of n.  Deterministic (fixed edge order), no atomics.
 * Replaces reference conv.py:109-141 (``conv_fwd`` kernel) as launched by conv.py:245-247.
 *   recv_rowptr [N+1], recv_eids [E] : receiver CSR (mmk_csr_build on edge_index[1])
 *   senders [E] int64                : edge_index[0]                                                          */
MMK_API int mmk_conv_fwd(const mmk_conv_layer *layer, const float *x, const float *Y, const float *W,
                 const int32_t *recv_rowptr, const int32_t *recv_eids, const int64_t *senders,
                 float *out, int64_t n_nodes, int64_t n_edges, void *stream);

/* Backward (first order), fused: one pass over the sender CSR computes
 *   gx[s]  = sum_{e: sender(e)=s} dTP/dx   (per sender, atomic-free),
 *   gW[e], gY[e]                           (per edge; the channel sum of gY is a warp-shuffle + shared reduction).
 * Replaces reference conv.py:144-176 (``conv_bwd_x``) and conv.py:179-222 (``conv_bwd_wy``) as launched by
 * conv.py:262-269.  Any of gx / gY / gW may be NULL to skip that output (gY and gW are computed together). */
MMK_API int mmk_conv_bwd(const mmk_conv_layer *layer, const float *x, const float *Y, const float *W, const float *grad_out,
                 const int32_t *send_rowptr, const int32_t *send_eids, const int64_t *receivers,
                 float *gx, float *gY, float *gW, int64_t n_nodes, int64_t n_edges, void *stream);

/* ------------------------------------------------------------------------------------------------------------------
 * CSR of an edge index (reference src/mace_mps_kernels/conv.py:229-235 ``csr_by``)
 * ---------------------------------------------------------------------------------------------------------------- */

/* Bytes of device workspace mmk_csr_build needs for (n_nodes, n_edges). */
MMK_API size_t mmk_csr_workspace_bytes(int64_t n_nodes, int64_t n_edges);
/* rowptr[n+1] and eids[E] such that eids[rowptr[v]:rowptr[v+1]] lists the edges with index[e] == v in increasing e
 * -- exactly torch.argsort(index, stable=True) grouped by bincount/cumsum.  Out-of-range indices set *error_flag
 * (device int, may be NULL) to 1 and are dropped.  workspace: mmk_csr_workspace_bytes() bytes, 16-byte aligned. */
MMK_API int mmk_csr_build(const int64_t *index, int64_t n_edges, int64_t n_nodes, int32_t *rowptr, int32_t *eids,
                  void *workspace, size_t workspace_bytes, int32_t *error_flag, void *stream);

/* Both CSRs of an edge index in one sequence of launches (4 kernels and a memset instead of 2 x (4 kernels, a memset
 * and a copy)): rowptr [2][n+1] and eids [2][E], row 0 the CSR of edge_index[0] (senders), row 1 of edge_index[1]
 * (receivers), each row equal to mmk_csr_build of that index row.  edge_index: device int64 [2][E]; workspace:
 * mmk_csr_pair_workspace_bytes() bytes, 16-byte aligned.  Sizes below 2^30. */
MMK_API size_t mmk_csr_pair_workspace_bytes(int64_t n_nodes, int64_t n_edges);
MMK_API int mmk_csr_build_pair(const int64_t *edge_index, int64_t n_edges, int64_t n_nodes, int32_t *rowptr,
                               int32_t *eids, void *workspace, size_t workspace_bytes, int32_t *error_flag,
                               void *stream);

/* Same result as mmk_csr_build, for callers that cannot allocate device memory: an MD engine or plugin host that
 * owns every device allocation through its own pool and hands this library only its inputs and outputs, or code
 * that must not call cudaMalloc where it runs.  This entry point has no counterpart in the reference (which always
 * lets PyTorch allocate); it allocates nothing.  Its scratch is one array of fixed size inside this library's
 * device image, so every GPU that loads the library holds it until the process exits:
 *   n_nodes <= MMK_NOALLOC_MAX_NODES and n_edges <= MMK_NOALLOC_MAX_EDGES (17 MiB per GPU); larger inputs return
 *   MMK_ERR_INVALID without launching anything.
 * The first call on a device looks up that device's copy of the array (cudaGetSymbolAddress); make it before any
 * stream capture.  The address is remembered together with the device's current context and looked up again when
 * that context changes (after cudaDeviceReset, for instance); that call is then again a first call.  All calls share
 * the one array: calls that overlap on the GPU (different streams, or threads) race and must be serialised by the
 * caller.  The array keeps the last call's contents; everything a call reads
 * from it is written first by the same call. */
#define MMK_NOALLOC_MAX_NODES (1 << 18)
#define MMK_NOALLOC_MAX_EDGES (1 << 22)
MMK_API int mmk_csr_build_noalloc(const int64_t *index, int64_t n_edges, int64_t n_nodes, int32_t *rowptr,
                                  int32_t *eids, int32_t *error_flag, void *stream);

/* ------------------------------------------------------------------------------------------------------------------
 * symmetric contraction layer
 * ---------------------------------------------------------------------------------------------------------------- */

/* Polynomial form of one MACE SymmetricContraction (reference src/mace_mps_kernels/symmetric.py:52-75 ``SCSpec``):
 * for output block q (M_q components, output offset out_off_q = C * sum_{q'<q} M_q'), term t with monomial
 * prod_{i in idx_t} x_i (degree deg_t, indices into the n_ell per-channel components) and first row row_t:
 *   out[b, out_off_q + c*M_q + m] = sum_t T[elem(b), c, row_t + m] * prod_{i in idx_t} x[b, c, i]
 * T is [n_elem, C, RP] fp32 on the device (caller-owned): one column of rows per (element, channel), RP = n_rows
 * rounded up to a multiple of 4 (zero padded), so every column the kernels copy with TMA starts on a 16-byte
 * boundary.  (The reference packs T[e][row][c], symmetric.py:69, 74; the B200 kernels work node-major and read one
 * channel's column at a time.) */
typedef struct mmk_sc_desc {
    int C;                   /* channels                                                             */
    int n_ell;               /* per-channel feature components, (l_max+1)^2                          */
    int n_rows;              /* rows of T                                                            */
    int n_blocks;            /* output blocks (one per output irrep)                                 */
    const int *block_M;      /* [n_blocks] components per block (2L+1)                               */
    const int *block_nterms; /* [n_blocks] terms of each block (terms are stored block after block)  */
    int max_degree;          /* largest monomial degree (= correlation order)                        */
    const int *term_degree;  /* [nterms] degree of term t, 1..max_degree                             */
    const int *term_idx;     /* [nterms * max_degree] sorted component indices, padded with -1      */
    const int *term_row;     /* [nterms] first row of T for term t                                   */
} mmk_sc_desc;

typedef struct mmk_sc_layer mmk_sc_layer;

/* Compiles the specialised kernels (monomial list baked in).  Replaces ``MetalSymmetricContraction.__init__``
 * (reference symmetric.py:161-166). */
MMK_API int mmk_sc_layer_create(const mmk_sc_desc *desc, mmk_sc_layer **layer);
MMK_API int mmk_sc_layer_destroy(mmk_sc_layer *layer);
MMK_API int mmk_sc_layer_dims(const mmk_sc_layer *layer, int *C, int *n_ell, int *out_dim, int *n_rows);
MMK_API int mmk_sc_compile_check(const mmk_sc_desc *desc);
/* The generated layer header (sizes, launch plan, the Horner-scheme term code), as the reference's ``source(spec)``
 * (symmetric.py:82-131); same buffer contract as mmk_conv_source. */
MMK_API int mmk_sc_source(const mmk_sc_desc *desc, char *buf, size_t cap, size_t *len);

MMK_API int mmk_sc_layer_status(const mmk_sc_layer *layer, int32_t *status, int reset);

/* elem[b] = argmax_e node_attrs[b, e] (first maximum), as torch.argmax (reference symmetric.py:169). */
MMK_API int mmk_elem_index(const float *node_attrs, int64_t n_nodes, int n_elem, int32_t *elem, void *stream);
/* Nodes grouped by element: perm[erow[e]:erow[e+1]] = the nodes of element e in increasing order (the CSR of elem;
 * workspace: mmk_csr_workspace_bytes(n_elem, n_nodes) bytes).  The symmetric-contraction kernels work on these
 * groups so that one coefficient column feeds 32 nodes at a time. */
MMK_API int mmk_elem_groups(const int32_t *elem, int64_t n_nodes, int n_elem, int32_t *erow, int32_t *perm,
                            void *workspace, size_t workspace_bytes, void *stream);

/* out[N, out_dim] from x[N, C, n_ell]; replaces reference symmetric.py:82-105 (``sc_fwd``, launched at :140).
 * perm / erow: mmk_elem_groups of the element index. */
MMK_API int mmk_sc_fwd(const mmk_sc_layer *layer, const float *x, const int32_t *perm, const int32_t *erow, int n_elem,
                       const float *T, float *out, int64_t n_nodes, void *stream);
/* gx[N, C, n_ell] = d(sum out*grad_out)/dx; replaces reference symmetric.py:106-131 (``sc_bwd``, launched at :154). */
MMK_API int mmk_sc_bwd(const mmk_sc_layer *layer, const float *x, const int32_t *perm, const int32_t *erow, int n_elem,
                       const float *T, const float *grad_out, float *gx, int64_t n_nodes, void *stream);

/* ------------------------------------------------------------------------------------------------------------------
 * edge geometry (no counterpart in the reference, which leaves MACE's spherical harmonics and radial embedding to
 * e3nn / PyTorch): the per-edge inputs of the convolution, one thread per edge
 * ---------------------------------------------------------------------------------------------------------------- */

/* Y[E, (lmax+1)^2] = real spherical harmonics of vectors[E, 3] normalised to unit length ('component' normalisation,
 * l = 0..lmax <= 3, e3nn's component order m = -l..l), as MACE's o3.SphericalHarmonics(normalize=True). */
MMK_API int mmk_sh_fwd(const float *vectors, int64_t n_edges, int lmax, float *Y, void *stream);
/* grad_vectors[E, 3] = d(sum Y * grad_Y)/d vectors. */
MMK_API int mmk_sh_bwd(const float *vectors, const float *grad_Y, int64_t n_edges, int lmax, float *grad_vectors,
                       void *stream);

/* MACE's radial embedding: out[e, n] = prefactor * sin(w[n] r) / r * env(r), env = the polynomial cutoff of order p
 * (1 - (p+1)(p+2)/2 u^p + p(p+2) u^(p+1) - p(p+1)/2 u^(p+2), u = r / r_max, 0 beyond r_max); w, prefactor, r_max, p
 * are the model's BesselBasis / PolynomialCutoff constants (w: host array of n_bessel floats). */
typedef struct mmk_radial_desc {
    int n_bessel;            /* 1..16 */
    const float *w;          /* [n_bessel] Bessel frequencies (host memory) */
    float prefactor;         /* sqrt(2 / r_max) */
    float r_max;
    float p;
} mmk_radial_desc;
MMK_API int mmk_radial_fwd(const mmk_radial_desc *desc, const float *lengths, int64_t n_edges, float *out, void *stream);
/* grad_lengths[E] = d(sum out * grad_out)/d lengths */
MMK_API int mmk_radial_bwd(const mmk_radial_desc *desc, const float *lengths, const float *grad_out, int64_t n_edges,
                           float *grad_lengths, void *stream);

/* MACE's get_edge_vectors_and_lengths (mace/modules/utils.py): vectors[e] = positions[edge_index[1, e]] -
 * positions[edge_index[0, e]] + shifts[e] (float32, PyTorch's order of operations) and lengths[e] = |vectors[e]|.
 *   positions [n_nodes, 3], shifts [E, 3], vectors [E, 3], lengths [E] (device float32); edge_index device int64
 *   [2, E] (row 0 senders, row 1 receivers). */
MMK_API int mmk_edge_vectors_fwd(const float *positions, const int64_t *edge_index, const float *shifts,
                                 int64_t n_edges, float *vectors, float *lengths, void *stream);
/* Backward: g[e] = grad_vectors[e] + vectors[e] * (grad_lengths[e] / lengths[e]) (the length term is 0 where the
 * length is 0, as PyTorch's norm backward; either incoming gradient may be NULL, not both);
 * grad_positions[n] = sum of g over n's receiver CSR row - sum of g over n's sender CSR row (CSRs as mmk_csr_build
 * makes them; one warp per node, fixed summation order: deterministic); grad_shifts[e] = g[e].  grad_positions or
 * grad_shifts may be NULL (not computed). */
MMK_API int mmk_edge_vectors_bwd(const float *grad_vectors, const float *grad_lengths, const float *vectors,
                                 const float *lengths, const int32_t *recv_rowptr, const int32_t *recv_eids,
                                 const int32_t *send_rowptr, const int32_t *send_eids, int64_t n_nodes,
                                 int64_t n_edges, float *grad_positions, float *grad_shifts, void *stream);

/* out[r, j] = x[r, cols[j]] for r < n_rows, j < n_cols (device float32, row-major with leading dimensions ldx, ldo;
 * cols device int32).  With cols a permutation it is MACE's reshape_irreps ([N, sum mul (2l+1)] in irreps layout ->
 * [N, mul, sum (2l+1)]) and, with the inverse permutation, its backward. */
MMK_API int mmk_gather_columns(const float *x, int64_t ldx, float *out, int64_t ldo, const int32_t *cols,
                               int64_t n_rows, int n_cols, void *stream);

/* ------------------------------------------------------------------------------------------------------------------
 * neighbour list (no counterpart in the reference, which takes the graph MACE builds on the host): the periodic pairs
 * within the cutoff, built on the device
 * ---------------------------------------------------------------------------------------------------------------- */

/* Every pair (i, j, S) with 0 < |positions[j] + S . cell - positions[i]| < cutoff, S an integer cell shift along the
 * periodic axes (matscipy / ASE neighbour_list('ijS') semantics as MACE builds its graph): edge_index[0, e] = i
 * (sender), edge_index[1, e] = j (receiver), shifts[e] = S . cell (float32), sorted by (i, j, S); rows
 * [n_edges, capacity) are padding edges (padding edge k: node k mod n_atoms to itself, shift (1000, 0, 0), beyond
 * any cutoff).
 *   positions: device float64 [n_atoms, 3]; cell (3 row vectors, 9 doubles), pbc (3), lo / hi (3 each): host.  lo / hi
 *   give the fractional range binned along non-periodic axes (atoms outside it are still found, only slower; NULL =
 *   [0, 1]); they are ignored on periodic axes.
 *   edge_index: device int64 [2, capacity]; shifts: device float32 [capacity, 3]; n_edges: device int64 = the number
 *   of pairs; above capacity the outputs are invalid and a larger capacity is needed.
 *   workspace: device, at least mmk_nl_workspace_bytes(...) bytes (0 = invalid arguments).
 * Nothing synchronises with the host, so the call can be captured in a CUDA graph at a fixed capacity. */
MMK_API size_t mmk_nl_workspace_bytes(const double *cell, const int32_t *pbc, double cutoff, const double *lo,
                                      const double *hi, int64_t n_atoms, int64_t capacity);
MMK_API int mmk_neighbor_list(const double *positions, int64_t n_atoms, const double *cell, const int32_t *pbc,
                              double cutoff, const double *lo, const double *hi, int64_t capacity, int64_t *edge_index,
                              float *shifts, int64_t *n_edges, void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------------------------------------
 * block linear (no counterpart in the reference, which leaves MACE's equivariant linears to e3nn): every path of one
 * equivariant linear layer in one launch
 * ---------------------------------------------------------------------------------------------------------------- */

/* out[n, dst_off_b + v*d_b + i] = sum over the paths p of block b of
 *                                  sum_u x[n, src_off_p + u*d_b + i] * weights[w_off_p + e(n)*mul_in_p*mul_out_b + u*mul_out_b + v]
 * blocks: device int32 [n_blocks][5] = (dst_off, mul_out, d, first path, number of paths); every output block is
 * written (zero when it has no path); paths: device int32 [*][3] = (src_off, mul_in, w_off); rows x[n] / out[n] at
 * n*ldx / n*ldo floats; max_d / max_mul_out = the largest d / mul_out of any block.  Element-indexed weights (MACE's
 * skip connection with
 * one-hot node attributes): perm / erow = mmk_elem_groups of the element index, e(n) = the node's element; otherwise
 * perm = erow = NULL, n_elem = 1, e = 0. */
MMK_API int mmk_block_linear(const float *x, int64_t ldx, float *out, int64_t ldo, const int32_t *blocks, int n_blocks,
                             const int32_t *paths, const float *weights, int max_d, int max_mul_out,
                             const int32_t *perm, const int32_t *erow, int n_elem, int64_t n_nodes, void *stream);

/* mmk_block_linear with the activation of an MLP layer (MACE's radial MLP: SiLU times a constant):
 *   epilogue != 0: zout = the product (pre-activation), out = act_scale * silu(zout)           (forward of a layer)
 *   prologue != 0: every input element x is multiplied by act_scale * silu'(zin) first          (input-gradient pass)
 * zout / zin have the layout of out / x.  Not both. */
MMK_API int mmk_block_linear_act(const float *x, int64_t ldx, float *out, int64_t ldo, const int32_t *blocks,
                                 int n_blocks, const int32_t *paths, const float *weights, int max_d, int max_mul_out,
                                 const int32_t *perm, const int32_t *erow, int n_elem, int64_t n_nodes, int epilogue,
                                 float *zout, int prologue, const float *zin, float act_scale, void *stream);

/* The hidden layers of MACE's radial MLP (e3nn FullyConnectedNet without biases, SiLU), all in one launch:
 *   h_0 = x [n_rows, widths[0]],  z_l = h_{l-1} @ W_l,  h_l = act_scale * silu(z_l),  l = 1 .. n_layers.
 * widths: host int32 [n_layers + 1], each 1..64; 1 <= n_layers <= 4.  weights: device, W_1 .. W_L packed one after
 * the other, W_l [widths[l-1]][widths[l]] row-major, already scaled by 1/sqrt(fan_in).  Writes h_out = h_L
 * [n_rows, widths[L]] and z_out = z_1 .. z_L packed ([n_rows, widths[l]] each, one after the other). */
MMK_API int mmk_mlp_fwd(const float *x, int64_t n_rows, int n_layers, const int32_t *widths, const float *weights,
                        float act_scale, float *h_out, float *z_out, void *stream);
/* grad_x [n_rows, widths[0]] = d(sum h_L * grad_h)/dx through the same layers, from the z_out of the forward.
 * weights_t: the transposed matrices, W_l^T [widths[l]][widths[l-1]] row-major, packed in the same order. */
MMK_API int mmk_mlp_bwd(const float *grad_h, int64_t n_rows, int n_layers, const int32_t *widths,
                        const float *weights_t, const float *z, float act_scale, float *grad_x, void *stream);

/* ------------------------------------------------------------------------------------------------------------------
 * float32 GEMM on the tensor cores (no counterpart in the reference, which leaves MACE's radial MLP to PyTorch):
 * the last layer of the radial MLP, W[E, NINS*C] = h[E, 64] . Wr, and its input gradient, on tcgen05 (kind::tf32)
 * with the 3xTF32 split (a = tf32(a) + tf32(a - tf32(a)); the three cross products that matter are accumulated in
 * float32), so the result has float32 accuracy.
 * ---------------------------------------------------------------------------------------------------------------- */

/* hi[i] = tf32(x[i]) (round to nearest), lo[i] = tf32(x[i] - hi[i]): the split of a constant operand. */
MMK_API int mmk_tf32_split(const float *x, float *hi, float *lo, int64_t n, void *stream);
/* C[M, N] = A[M, K] . B[N, K]^T, all float32 row-major (A row i at A + i*lda, B row j at B + j*ldb, C row i at
 * C + i*ldc); B given split (mmk_tf32_split).  K, lda, ldb, ldc multiples of 4; A, B_hi, B_lo, C 16-byte aligned.
 * Tiles of 128 rows x 64/128/256 columns, accumulator in tensor memory.  Outputs with fewer tiles than SMs split K
 * over several CTAs when a workspace of mmk_gemm_workspace_bytes(M, N, K) bytes (16-byte aligned, zero-filled before
 * its first use; its first 1 KB holds tile counters that every call leaves at zero, so one workspace of the largest
 * size serves calls of every shape) is given; with workspace NULL (or too small) they do not.
 * Deterministic either way.  Calls that share a workspace must be ordered on the GPU. */
MMK_API size_t mmk_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
MMK_API int mmk_gemm_tf32x3(const float *A, int64_t lda, const float *B_hi, const float *B_lo, int64_t ldb, float *C,
                            int64_t ldc, int64_t M, int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                            void *stream);
/* Nonzero when a GEMM's pipeline wait gave up (its output is invalid).  Synchronises the device; reset clears it. */
MMK_API int mmk_gemm_status(int32_t *status, int reset);

#ifdef __cplusplus
}
#endif

#endif /* MMK_H */
