/*
 * flasheq_b200.h -- C ABI of libflasheq_b200.so, the B200 (sm_100a) kernels behind
 * the drop-in ``flash_eq`` Python package.
 *
 * Conventions (all entry points):
 *   - Plain device pointers and sizes; no framework types.  The caller owns every
 *     buffer, including the workspace (size from the matching *_workspace_bytes).
 *   - Work is enqueued on ``stream`` (a cudaStream_t passed as void*); nothing
 *     synchronises the host, nothing allocates device memory.
 *   - Return FEQ_OK or an FEQ_ERR_* code; never abort or trap.  feq_status_string
 *     turns a code into text.  Problems only a kernel can see (an index out of
 *     range) are written to the caller's int32 ``status`` word, which the caller
 *     may read after the stream completes (0 == fine).
 *   - Tensors are row-major and contiguous, float32 unless stated.
 *   - Layouts follow hmblair/flash-eq: features (E, C, dim) in the standard
 *     (l, m = -l..l) order; "m-first" order as built by
 *     flash_eq/representations/wigner.py:243-272; radial table
 *     (num_bins + 1, C_out, C_in, W) with W = ProductRepr(in, out).nreps().
 *
 * Each entry point names the reference interface it replaces.
 */
#ifndef FLASHEQ_B200_H
#define FLASHEQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *feq_stream_t; /* cudaStream_t */

enum feq_status_code {
    FEQ_OK = 0,
    FEQ_ERR_INVALID_ARGUMENT = 1,   /* bad pointer / size / layout */
    FEQ_ERR_UNSUPPORTED = 2,        /* valid request outside this build's limits */
    FEQ_ERR_WORKSPACE = 3,          /* workspace missing or too small */
    FEQ_ERR_CUDA = 4,               /* a CUDA runtime call or launch failed */
    FEQ_ERR_NO_DEVICE = 5           /* no usable CUDA device */
};

/* Limits.  FEQ_MAX_L matches the reference's MAX_LVALS = 17 (l <= 16,
 * flash_eq/cuda/csrc/block_diagonal.cu:172, :1298-1300). */
#define FEQ_MAX_L 16
#define FEQ_MAX_IRREPS 64
#define FEQ_MAX_DIM 512

/* Basis output layouts for feq_wigner_basis. */
#define FEQ_BASIS_MFIRST 0     /* WignerDBasis.forward: rot_to_ez(d).mT[..., perm] */
#define FEQ_BASIS_ROT_TO_EZ 1  /* WignerD.rot_to_ez: rot(axis, angle).mT, standard order */

/* Pooling / reduction modes (flash_eq/layers/pooling.py:21-57). */
#define FEQ_REDUCE_SUM 0
#define FEQ_REDUCE_MEAN 1
#define FEQ_REDUCE_MAX 2

/* ---------------------------------------------------------------------------
 * Library
 * ------------------------------------------------------------------------ */
const char *feq_status_string(int status);
/* 2: FeqAttnArgs gained k / num_src_nodes (partitioned graphs).
 * 3: attention / pooling backward entry points, node-level operators.
 * 4: feq_set_wait_limit_ns; the separable (low-rank) edgewise entry point. */
int feq_abi_version(void);
/* Limit, in nanoseconds, of every pipeline wait of the tensor-core kernels launched
 * after this call (no counterpart in the reference).  A wait that runs past it ends
 * its kernel early with status 2 ("a tensor-core wait timed out", result invalid)
 * instead of waiting on; the kernel first waits for its own copies and MMAs in flight
 * and releases its tensor memory, so the context stays usable.  0 restores the
 * default (4 s).  Returns the previous limit.  Process-wide; meant for tests of the
 * time-out path and for callers that want a tighter bound. */
uint64_t feq_set_wait_limit_ns(uint64_t limit_ns);
/* Human-readable last CUDA error seen by this thread (empty when none). */
const char *feq_last_error(void);
/* Kernels this library has enqueued since load (its own kernels; each CUB radix
 * sort call is counted once per kernel it launches: 3).  No counterpart in the
 * reference; used by benchmarks to report how many native kernels ran. */
int64_t feq_launch_count(void);
/* Stage timing (no counterpart in the reference).  While enabled, each kernel stage
 * of the Wigner basis and of the edgewise path is bracketed by two CUDA events
 * recorded on the stream the stage is launched on.  feq_profile_enable(1) starts a
 * new record set (0 stops recording).  feq_profile_read synchronises the events and
 * returns the number of distinct stages; for 0 <= index < that number it also fills
 * the stage name, the summed event time in milliseconds and the number of launches.
 * Returns a negative status on error. */
int feq_profile_enable(int32_t on);
int feq_profile_read(int32_t index, char *name, int32_t name_capacity, double *total_ms, int64_t *launches);

/* ---------------------------------------------------------------------------
 * Wigner-D basis.
 * Replaces WignerDBasis.forward / WignerD.rot_to_ez
 * (flash_eq/representations/wigner.py:198-240, :341-370), which build the
 * matrices with a batched torch.linalg.matrix_exp.  Here each (edge, l) block is
 * a closed form in (theta, phi) evaluated per edge.
 *   directions (E, 3) need not be normalised; out (E, dim, dim).
 * ------------------------------------------------------------------------ */
int feq_wigner_basis(const float *directions, int64_t num_edges, const int32_t *lvals,
                     int32_t num_lvals, int32_t layout, float *out, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Distance binning (block_diagonal.cu:82-115 compute_binning): per edge the bin
 * index lo (int32, bit-exact) and interpolation weight t (unclamped in linear mode).
 * ------------------------------------------------------------------------ */
int feq_edge_binning(const float *distances, int64_t num_edges, float bin_param1,
                     float bin_param2, int32_t num_bins, int32_t log_bins, int32_t *bin_lo,
                     float *t, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Stable sort of edges by an int32 key in [0, num_keys): perm[i] = id of the i-th
 * edge in (key, id) order, offsets[k] = first position of key k (num_keys + 1
 * entries).  Keys outside the range set *status and are treated as num_keys - 1.
 * Used for the bin grouping of the radial mix and for dst-sorted (CSR) segments.
 * The reference sorts with torch.argsort (flash_eq/cuda/block_diagonal.py:102-103)
 * and pools with scatter_add_ (flash_eq/layers/pooling.py:21-30).
 * ------------------------------------------------------------------------ */
size_t feq_edge_sort_workspace_bytes(int64_t num_edges, int32_t num_keys);
int feq_edge_sort(const int32_t *keys, int64_t num_edges, int32_t num_keys, int64_t *perm,
                  int64_t *offsets, int32_t *status, void *workspace, size_t workspace_bytes,
                  feq_stream_t stream);
/* Same, reading int64 keys (e.g. Graph.dst). */
int feq_edge_sort_i64(const int64_t *keys, int64_t num_edges, int32_t num_keys, int64_t *perm,
                      int64_t *offsets, int32_t *status, void *workspace, size_t workspace_bytes,
                      feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Block-diagonal radial mix in the m-first basis.
 * Replaces _block_diagonal_cuda.forward (flash_eq/cuda/csrc/block_diagonal.cu:
 * 1268-1540) called through block_diagonal_cuda (flash_eq/cuda/block_diagonal.py:
 * 206-274): features (E, Cin, Din) m-first, radial_table (num_bins+1, Cout, Cin, W),
 * distances (E,) -> output (E, Cout, Dout) m-first.  No host sync, no sort/unsort
 * copies: edges are grouped by bin internally and results land in input order.
 * ------------------------------------------------------------------------ */
size_t feq_block_diagonal_workspace_bytes(int64_t num_edges, int32_t c_in, int32_t c_out,
                                          const int32_t *lvals_in, int32_t n_lvals_in,
                                          const int32_t *lvals_out, int32_t n_lvals_out,
                                          int32_t num_bins);
int feq_block_diagonal_fwd(const float *features, const float *radial_table,
                           const float *distances, int64_t num_edges, int32_t c_in,
                           int32_t c_out, const int32_t *lvals_in, int32_t n_lvals_in,
                           const int32_t *lvals_out, int32_t n_lvals_out, float sh_scale,
                           float bin_param1, float bin_param2, int32_t num_bins,
                           int32_t log_bins, float *output, void *workspace,
                           size_t workspace_bytes, feq_stream_t stream);

/* feq_block_diagonal_fwd with a selectable mix arithmetic (no counterpart in the reference):
 * FEQ_MIX_FP32 is feq_block_diagonal_fwd itself; FEQ_MIX_BF16X3 / FEQ_MIX_BF16 run the
 * tensor-core (tcgen05) mix on the m-first rows (sort by bin, rows to the mix layout, mix,
 * rows back), the forward used by training. */
size_t feq_block_diagonal_fwd_mix_workspace_bytes(int64_t num_edges, int32_t c_in, int32_t c_out,
                                                  const int32_t *lvals_in, int32_t n_lvals_in,
                                                  const int32_t *lvals_out, int32_t n_lvals_out,
                                                  int32_t num_bins, int32_t mix_mode);
int feq_block_diagonal_fwd_mix(const float *features, const float *radial_table, const float *distances,
                               int64_t num_edges, int32_t c_in, int32_t c_out, const int32_t *lvals_in,
                               int32_t n_lvals_in, const int32_t *lvals_out, int32_t n_lvals_out,
                               float sh_scale, float bin_param1, float bin_param2, int32_t num_bins,
                               int32_t log_bins, int32_t mix_mode, float *output, void *workspace,
                               size_t workspace_bytes, feq_stream_t stream);

/* Backward of feq_block_diagonal_fwd.
 * Replaces _block_diagonal_cuda.backward (flash_eq/cuda/csrc/block_diagonal.cu:1543-1758,
 * kernels :747-1161; wrapper _BlockDiagonalFunction.backward, block_diagonal.py:140-174):
 * grad_output (E, c_out, d_out) and features (E, c_in, d_in) m-first, radial_table as in the
 * forward; writes grad_features (E, c_in, d_in), grad_table (num_bins+1, c_out, c_in, W) and
 * grad_distances (E,).  Deterministic: no atomics; grad_table is reduced per distance bin
 * in sorted-edge order.  mix_mode FEQ_MIX_BF16X3 (float32-level accuracy) or FEQ_MIX_BF16
 * selects the tensor-core arithmetic of the two mixes it runs (W_t A and G W_t^T).
 * grad_distances follows the reference's expression, NaN at distance 0 when some
 * l_in + l_out > 0 (as the reference). */
size_t feq_block_diagonal_bwd_workspace_bytes(int64_t num_edges, int32_t c_in, int32_t c_out,
                                              const int32_t *lvals_in, int32_t n_lvals_in,
                                              const int32_t *lvals_out, int32_t n_lvals_out,
                                              int32_t num_bins, int32_t mix_mode);
int feq_block_diagonal_bwd(const float *grad_output, const float *features, const float *radial_table,
                           const float *distances, int64_t num_edges, int32_t c_in, int32_t c_out,
                           const int32_t *lvals_in, int32_t n_lvals_in, const int32_t *lvals_out,
                           int32_t n_lvals_out, float sh_scale, float bin_param1, float bin_param2,
                           int32_t num_bins, int32_t log_bins, int32_t mix_mode, float *grad_features,
                           float *grad_table, float *grad_distances, void *workspace,
                           size_t workspace_bytes, feq_stream_t stream);

/* Same operation as feq_block_diagonal_fwd for callers that cannot allocate device
 * memory: code running where cudaMalloc is unavailable or not allowed (a host
 * framework that owns every allocation, a plugin without an allocator handle), or
 * that must not allocate while it runs.  No counterpart in the reference.
 *   - The scratch is a fixed array of FEQ_NOALLOC_SCRATCH_BYTES in the library's
 *     device memory (every GPU that loads the library holds it until exit); inputs
 *     and the output are still the caller's.  A problem whose scratch would exceed
 *     it returns FEQ_ERR_WORKSPACE and feq_last_error() gives the sizes.
 *   - Every call looks up the array's device address on the current device
 *     (cudaGetSymbolAddress, which allocates nothing), so the address stays right
 *     after a device reset.  The first call on a device also loads the library's
 *     module there; make that first call before any stream capture.
 *   - All calls share the one array and it keeps the previous call's contents (no
 *     part needs to start at zero: each call writes every region before reading it).
 *     Calls whose GPU work overlaps in time race on it: serialise them (one stream,
 *     or events between streams).
 *   - Allocates nothing: no cudaMalloc / cudaFree and no allocating library call. */
#define FEQ_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
int feq_block_diagonal_fwd_noalloc(const float *features, const float *radial_table,
                                   const float *distances, int64_t num_edges, int32_t c_in,
                                   int32_t c_out, const int32_t *lvals_in, int32_t n_lvals_in,
                                   const int32_t *lvals_out, int32_t n_lvals_out,
                                   float sh_scale, float bin_param1, float bin_param2,
                                   int32_t num_bins, int32_t log_bins, float *output,
                                   feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused edgewise linear: out = Q . Lambda(r) . P^T . f.
 * Replaces EquivariantEdgewiseLinear.forward (flash_eq/layers/linear.py:100-160):
 * bmm(f, P) -> block_diagonal_cuda -> bmm(out, Q^T).
 *
 * Input rows: f[e] = x[src[e]] (+ edge_add[e]) when src != NULL (the gather of
 * EquivariantAttention, flash_eq/layers/attention.py:307-310), else x[e].
 * Basis: when directions != NULL, P and Q blocks are built per edge from the edge
 * direction (never materialised); otherwise the dense (E, d, d) matrices P_in and
 * Q_out are read as given, exactly like the reference's bmm.
 * ------------------------------------------------------------------------ */
typedef struct FeqEdgewiseArgs {
    const float *x;            /* (E or N, c_in, d_in) */
    const int64_t *src;        /* optional (E,) gather index into x */
    int64_t num_src_rows;      /* rows of x when src != NULL (bounds check) */
    const float *edge_add;     /* optional (E, c_in, d_in) added after the gather */
    const float *directions;   /* optional (E, 3): fused basis */
    const float *P_in;         /* (E, d_in, d_in) when directions == NULL */
    const float *Q_out;        /* (E, d_out, d_out) when directions == NULL */
    const float *distances;    /* (E,) */
    const float *radial_table; /* (num_bins + 1, c_out, c_in, W) */
    int64_t num_edges;
    int32_t c_in, c_out;
    const int32_t *lvals_in;   /* host array */
    int32_t n_lvals_in;
    const int32_t *lvals_out;  /* host array */
    int32_t n_lvals_out;
    float sh_scale, bin_param1, bin_param2;
    int32_t num_bins, log_bins;
    float *out;                /* (E, c_out, d_out) standard order */
    int32_t *status;           /* optional device int32: 1 = a src index was out of range,
                                  2 = a tensor-core wait timed out (result invalid) */
    int32_t mix_mode;          /* FEQ_MIX_* below */
} FeqEdgewiseArgs;

/* Radial-mix arithmetic for feq_edgewise_fwd.
 *   FEQ_MIX_FP32       float32 FMA on CUDA cores (the reference's arithmetic)
 *   FEQ_MIX_BF16       tcgen05 tensor cores, bf16 operands, fp32 accumulation
 *                      (the "bf16-mix" mode: ~1e-3 relative error)
 *   FEQ_MIX_BF16X3     tcgen05 tensor cores with every operand split into two bf16
 *                      terms (hi.hi + hi.lo + lo.hi): float32-level accuracy */
#define FEQ_MIX_FP32 0
#define FEQ_MIX_BF16 1
#define FEQ_MIX_BF16X3 2

size_t feq_edgewise_workspace_bytes(const FeqEdgewiseArgs *args);
int feq_edgewise_fwd(const FeqEdgewiseArgs *args, void *workspace, size_t workspace_bytes,
                     feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Separable edgewise linear: the same result as feq_edgewise_fwd for the radial tables
 * EquivariantEdgewiseLinear builds, in ONE kernel (gather, rotation in, mix, rotation
 * back), without a workspace.
 * Replaces EquivariantEdgewiseLinear.forward (flash_eq/layers/linear.py:100-160) together
 * with the table its SeparableRadialNet materialises (flash_eq/layers/radial.py:259-275):
 *   table[b, o, i, w] = sum_k channel_patterns[k, o, i] * radial_features[b, k, w]
 * is never formed; the kernel interpolates radial_features per edge and applies
 * channel_patterns on the tensor cores (tcgen05) with a weight shared by every edge.
 *   radial_features: (num_bins + 1, rank, W) = the radial net's head output viewed as
 *   (B, K, W) (radial.py:266-267); channel_patterns: (rank, c_out, c_in).
 * Input rows f[e] = x[src[e]] (+ edge_add[e]) or x[e]; the basis comes from directions.
 * feq_edgewise_separable_supported() says whether this build runs a request (lvals
 * [0..L] in and out with L <= 4, c_in = c_out = 64, rank 4, mix FEQ_MIX_BF16X3 or
 * FEQ_MIX_BF16, directions given); otherwise use feq_edgewise_fwd with the table.
 * status (optional): 1 = a src index was out of range (that row reads as zero),
 * 2 = a tensor-core wait timed out (result invalid).
 * ------------------------------------------------------------------------ */
typedef struct FeqSeparableArgs {
    const float *x;                 /* (E or N, c_in, d_in) standard order, 16-byte aligned */
    const int64_t *src;             /* optional (E,) gather index into x */
    int64_t num_src_rows;           /* rows of x when src != NULL */
    const float *edge_add;          /* optional (E, c_in, d_in), 16-byte aligned */
    const float *directions;        /* (E, 3) */
    const float *distances;         /* (E,) */
    const float *channel_patterns;  /* (rank, c_out, c_in) */
    const float *radial_features;   /* (num_bins + 1, rank, W), 16-byte aligned */
    int64_t num_edges;
    int32_t c_in, c_out, rank;
    const int32_t *lvals_in;        /* host array */
    int32_t n_lvals_in;
    const int32_t *lvals_out;       /* host array */
    int32_t n_lvals_out;
    float sh_scale, bin_param1, bin_param2;
    int32_t num_bins, log_bins;
    float *out;                     /* (E, c_out, d_out) standard order, 16-byte aligned */
    int32_t *status;
    int32_t mix_mode;               /* FEQ_MIX_BF16X3 or FEQ_MIX_BF16 */
} FeqSeparableArgs;

int feq_edgewise_separable_supported(const FeqSeparableArgs *args);
int feq_edgewise_separable_fwd(const FeqSeparableArgs *args, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Segment softmax over edges that share a destination
 * (EquivariantEdgeAttention._neighbor_softmax, flash_eq/layers/attention.py:108-141):
 *   w[e, h] = exp(l[e,h] - max_seg) / (sum_seg exp(. - max_seg) + 1e-8)
 * with perm/offsets from feq_edge_sort on dst.  Deterministic (no atomics).
 * ------------------------------------------------------------------------ */
int feq_segment_softmax(const float *logits, int64_t num_edges, int32_t num_heads,
                        const int64_t *perm, const int64_t *offsets, int64_t num_nodes,
                        float *weights, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Edge attention logits and weights for edge-level Q, K
 * (EquivariantEdgeAttention.forward, attention.py:92-103):
 *   logits[e,h] = scale * sum_i Q[e,h,i] K[e,h,i] - (decay > 0 ? dist[e]/decay : 0)
 *   weights = segment softmax of logits.
 * ------------------------------------------------------------------------ */
int feq_edge_attention_weights(const float *Q, const float *K, int64_t num_edges,
                               int32_t num_heads, int32_t qk_dim, float scale,
                               const float *distances, float decay_scale, const int64_t *perm,
                               const int64_t *offsets, int64_t num_nodes, float *weights,
                               feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Segmented pooling of edge rows onto destination nodes
 * (GraphPooling, flash_eq/layers/pooling.py:21-57; scatter_add_ / scatter_reduce_):
 *   out[n, :] = reduce_{e : dst[e] = n} (w[e, head(j)] *) X[e, :]
 * row_len = C * dim.  When weights != NULL each row is first multiplied per head:
 * element j of a row belongs to head j / (row_len / num_heads)
 * (EquivariantEdgeAttention._apply_attention, attention.py:143-167).
 * Nodes without edges get 0 (sum, mean, max).  Deterministic.
 * ------------------------------------------------------------------------ */
int feq_segment_pool(const float *edge_rows, int64_t row_len, const float *weights,
                     int32_t num_heads, const int64_t *perm, const int64_t *offsets,
                     int64_t num_nodes, int32_t reduce, float *out, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused attention + pooling for EquivariantAttention (attention.py:271-314):
 *   Q = QK[dst, :C], K = QK[src, C:], logits per head as above (online softmax
 *   over the dst segment), out[n] = reduce_e w[e, head] * V[e]   (sum or mean).
 * QK (N, 2C, d) node rows; V (E, Cv, dv) edge rows.
 * ------------------------------------------------------------------------ */
typedef struct FeqAttnArgs {
    const float *qk;          /* (N, 2*c_qk, d_qk) */
    const float *v;           /* (E, c_v, d_v) */
    const int64_t *src;       /* (E,) */
    const float *distances;   /* (E,), may be NULL when decay_scale <= 0 */
    const int64_t *perm;      /* dst-sorted edge ids (E,) */
    const int64_t *offsets;   /* (N + 1,) */
    int64_t num_nodes, num_edges;
    int32_t c_qk, d_qk, c_v, d_v, num_heads;
    float scale, decay_scale;
    int32_t reduce;           /* FEQ_REDUCE_SUM or FEQ_REDUCE_MEAN */
    float *out;               /* (N, c_v, d_v) */
    int32_t *status;          /* optional: 1 = a src index was out of range */
    /* Partitioned graphs (no counterpart in the reference): when k is not NULL, qk holds
     * only the destinations' Q rows (num_nodes, c_qk, d_qk), k holds the K rows of every
     * source node (num_src_nodes, c_qk, d_qk) and src indexes k. */
    const float *k;
    int64_t num_src_nodes;
} FeqAttnArgs;

int feq_attn_pool_fwd(const FeqAttnArgs *args, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Backward of the attention and pooling operators.  The reference has no native
 * backward for these: PyTorch autograd differentiates its scatter / gather ops
 * (attention.py:92-167, pooling.py:21-57).  Softmax gradient
 *   dl = w (dw - sum_seg w dw),   w = exp(l - max) / (sum_seg exp(. - max) + 1e-8),
 * with the segment max held constant (its derivative is below 1e-8 relative).
 * All reductions run over sorted segments in a fixed order: deterministic.
 * ------------------------------------------------------------------------ */

/* Backward of feq_attn_pool_fwd.  fwd holds the forward's arguments (fwd.out and
 * fwd.status are not read / may be set).  Writes
 *   grad_q (num_nodes rows, row stride ldq floats): dL/dQ of every destination row,
 *   grad_k (num_src rows, stride ldk): dL/dK of every source row (num_src = num_nodes,
 *          or fwd.num_src_nodes when fwd.k is set); for the unsplit QK layout pass
 *          grad_q = grad_qk, grad_k = grad_qk + c_qk*d_qk, ldq = ldk = 2*c_qk*d_qk,
 *   grad_v (E, c_v, d_v), grad_distances (E,) (the distance-decay term only; NULL to
 *   skip), grad_scale_partial (num_nodes,): per destination node, the share of
 *   dL/dlog(scale) (sum them for the scalar).
 * src_perm / src_offsets: feq_edge_sort of src over num_src keys.  edge_scratch:
 * 2 * E * num_heads floats. */
typedef struct FeqAttnBwdArgs {
    FeqAttnArgs fwd;
    const float *grad_out;        /* (N, c_v, d_v) */
    const int64_t *dst;           /* (E,) */
    const int64_t *src_perm;      /* (E,) */
    const int64_t *src_offsets;   /* (num_src + 1,) */
    float *grad_q;
    int64_t ldq;
    float *grad_k;
    int64_t ldk;
    float *grad_v;
    float *grad_distances;
    float *grad_scale_partial;
    float *edge_scratch;
} FeqAttnBwdArgs;

int feq_attn_pool_bwd(const FeqAttnBwdArgs *args, feq_stream_t stream);

/* Backward of feq_segment_softmax: grad_logits = w * (grad_w - sum_seg w grad_w).
 * grad_logits may alias grad_weights. */
int feq_segment_softmax_bwd(const float *weights, const float *grad_weights, int64_t num_edges,
                            int32_t num_heads, const int64_t *perm, const int64_t *offsets,
                            int64_t num_nodes, float *grad_logits, feq_stream_t stream);

/* Backward of feq_edge_attention_weights (weights = its output).  grad_logits (E, H)
 * is written (scratch or result); grad_Q, grad_K (E, H, qk_dim), grad_distances (E,)
 * (-sum_h dl / decay; 0 when decay_scale <= 0) and grad_scale_partial (E,) (per edge
 * share of dL/dlog(scale)) may each be NULL. */
int feq_edge_attention_weights_bwd(const float *Q, const float *K, int64_t num_edges, int32_t num_heads,
                                   int32_t qk_dim, float scale, float decay_scale, const int64_t *perm,
                                   const int64_t *offsets, int64_t num_nodes, const float *weights,
                                   const float *grad_weights, float *grad_logits, float *grad_Q,
                                   float *grad_K, float *grad_distances, float *grad_scale_partial,
                                   feq_stream_t stream);

/* Backward of feq_segment_pool.  dst (E,) is each edge's destination; perm / offsets
 * the dst-sorted segments; out the forward's output and tie_scratch (N, row_len)
 * floats, both needed for max only (the gradient of an output element is split
 * evenly between the edges equal to it, like torch's scatter_reduce amax).
 * grad_rows (E, row_len); grad_weights (E, H) when weights != NULL (may be NULL). */
int feq_segment_pool_bwd(const float *edge_rows, int64_t row_len, const float *weights, int32_t num_heads,
                         const int64_t *dst, const int64_t *perm, const int64_t *offsets, int64_t num_nodes,
                         int64_t num_edges, int32_t reduce, const float *out, const float *grad_out,
                         float *tie_scratch, float *grad_rows, float *grad_weights, int32_t *status,
                         feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Node-level operators of the transformer block (forward; no counterpart kernels in
 * the reference, which composes them from PyTorch ops).  x, out: (N, C, d) float32
 * with d = sum(2 l + 1) over lvals.
 * ------------------------------------------------------------------------ */
/* SeparableEquivariantLayerNorm (flash_eq/layers/norm.py:177-249): every l = 0 position
 * p_s gets a LayerNorm over channels, (x - mean) / (std + eps) * w_scalar[c, s] +
 * b_scalar[c, s] (std biased; w/b (C, n_scalar)); all other positions share one RMS,
 * x * w_higher[c] / sqrt(mean(x^2) + eps). */
int feq_node_sep_layernorm(const float *x, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                           const float *w_scalar, const float *b_scalar, const float *w_higher, float eps,
                           float *out, feq_stream_t stream);
/* EquivariantLayerNorm (norm.py:111-174): norms[c, r] = sqrt(sum over irrep r of x^2 +
 * rep_eps); when ln_weight != NULL a LayerNorm of the norms over channels per irrep
 * (ln_eps, affine (C,)); out = x * ln / (norms + eps) (1 / (norms + eps) without it). */
int feq_node_layernorm(const float *x, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                       const float *ln_weight, const float *ln_bias, float ln_eps, float rep_eps, float eps,
                       float *out, feq_stream_t stream);
/* RepNorm (norm.py:19-64): norms (N, C, n_lvals) = sqrt(sum over each irrep of x^2 + eps). */
int feq_node_rep_norm(const float *x, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                      float eps, float *norms, feq_stream_t stream);
/* EquivariantLinear (linear.py:172-268) in three steps: feq_node_to_posmajor
 * (xt[p][n][c] = x[n][c][p], xt (d, N, C)); one plain GEMM per irrep on the contiguous
 * rows p = off .. off + 2l of xt (the caller's BLAS: y_r = x_r W_r^T); feq_node_from_posmajor
 * (y[n][c][p] = yt[p][n][c] + bias[c, scalar_index[p]] where scalar_index[p] >= 0; bias
 * (C, n_scalar) and scalar_index (d,) int8 device arrays, both NULL for no bias).  C a
 * multiple of 4 and xt / yt 16-byte aligned (FEQ_ERR_UNSUPPORTED otherwise). */
int feq_node_to_posmajor(const float *x, int64_t num_nodes, int32_t C, int32_t d, float *xt, feq_stream_t stream);
int feq_node_from_posmajor(const float *yt, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                           const float *bias, const int8_t *scalar_index, float *y, feq_stream_t stream);
/* EquivariantLinear (linear.py:172-268) as one tensor-core (tcgen05) kernel: y (N, c_out, d)
 * = per irrep r, W_r x over the positions of r, plus bias[co] at the l = 0 position; x
 * (N, c_in, d) node rows, weight (n_lvals, c_out, c_in) float32 (the module's weight viewed per
 * irrep), bias (c_out,) or NULL.  mix_mode FEQ_MIX_BF16X3 (float32-level accuracy) or
 * FEQ_MIX_BF16.  Shapes served: lvals [0..L] with L <= 2 and (c_in, c_out) in {(64, 64),
 * (64, 128), (128, 64)} (FEQ_ERR_UNSUPPORTED otherwise: use the three-step path above).  The
 * workspace (feq_node_linear_tc_workspace_bytes, 16-byte aligned) receives the weights re-laid
 * as tensor-core tiles; x and y 16-byte aligned; status (may be NULL) is set to 2 when a
 * pipeline wait ran out (feq_set_wait_limit_ns). */
size_t feq_node_linear_tc_workspace_bytes(int32_t c_in, int32_t c_out, const int32_t *lvals, int32_t n_lvals,
                                          int32_t mix_mode);
int feq_node_linear_tc(const float *x, int64_t num_nodes, int32_t c_in, int32_t c_out, const int32_t *lvals,
                       int32_t n_lvals, const float *weight, const float *bias, int32_t mix_mode, float *y,
                       void *workspace, size_t workspace_bytes, int32_t *status, feq_stream_t stream);
/* The dense nn.Linear of EquivariantGating (gating.py:17-76: z = Linear(irrep norms), the
 * (C * n_lvals)^2 mix before the sigmoid) on the tensor cores: y (n, m) = x (n, k) w^T + bias,
 * w (m, k) float32 as nn.Linear holds it, bias (m,) or NULL, all row-major; m a multiple of
 * 128 up to 512, k a multiple of 64 up to 512 (FEQ_ERR_UNSUPPORTED otherwise: use a library
 * GEMM).  mix_mode FEQ_MIX_BF16X3 (float32-level accuracy) or FEQ_MIX_BF16.  The workspace
 * (feq_dense_linear_tc_workspace_bytes, 16-byte aligned) receives w re-laid as tensor-core
 * tiles; x 16-byte aligned; status (may be NULL) is set to 2 when a pipeline wait ran out. */
size_t feq_dense_linear_tc_workspace_bytes(int32_t m, int32_t k, int32_t mix_mode);
int feq_dense_linear_tc(const float *x, int64_t n, int32_t m, int32_t k, const float *weight, const float *bias,
                        int32_t mix_mode, float *y, void *workspace, size_t workspace_bytes, int32_t *status,
                        feq_stream_t stream);
/* SeparableRadialNet.radial_features (radial.py:226-267): at every bin edge r_b
 * (num_edges of them) the sinusoid x envelope basis of x = clamp((r_b - min_val) /
 * (max_val - min_val), 0, 1) with the given frequencies (num_freqs <= 64), then
 * SiLU(w1 . + b1), SiLU(w2 . + b2), w3 . + b3, the weights as nn.Linear holds them (w1
 * (hidden, 2 num_freqs), w2 (hidden, hidden), w3 (out_dim, hidden), hidden <= 256); out
 * (num_edges, out_dim) float32.  One launch for what PyTorch runs as about twenty. */
int feq_radial_features(const float *bin_edges, int32_t num_edges, float min_val, float max_val,
                        const float *frequencies, int32_t num_freqs, const float *w1, const float *b1,
                        int32_t hidden, const float *w2, const float *b2, const float *w3, const float *b3,
                        int32_t out_dim, float *out, feq_stream_t stream);
/* EquivariantGating's gate (gating.py:17-76): out = x * sigmoid(z)[c, irrep of the
 * position], z (N, C * n_lvals) the pre-activation. */
int feq_node_gate(const float *x, const float *z, int64_t num_nodes, int32_t C, const int32_t *lvals,
                  int32_t n_lvals, float *out, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * k-nearest-neighbour graph construction (no counterpart in the reference, which leaves
 * graph building to the user; its examples use torch.cdist + topk).  xyz (N, 3) float32;
 * nbr (N, k) int64: the k nearest other points of every point by Euclidean distance,
 * ascending (ties by index), -1 when fewer than k exist.  Points are binned into cubic
 * cells of side `cell` with corner (x0, y0, z0) (any cell > 0 gives the exact result;
 * about the k-th neighbour distance is fastest); status (may be NULL) is set to 1 when a
 * point's search stopped before it was exact (cell far smaller than the point spacing).
 * 1 <= k <= 64, N < 2^31.
 * ------------------------------------------------------------------------ */
size_t feq_knn_workspace_bytes(int64_t num_points);
int feq_knn_graph(const float *xyz, int64_t num_points, int32_t k, float cell, float x0, float y0, float z0,
                  int64_t *nbr, int32_t *status, void *workspace, size_t workspace_bytes, feq_stream_t stream);

/* ---------------------------------------------------------------------------
 * Radius graph construction (no counterpart in the reference, which leaves graph building
 * to the user, README.md:49-52; its benchmark graphs are "all pairs within r"): every
 * ordered pair (i, j) of points with batch[i] == batch[j] (batch may be NULL: one graph),
 * j != i unless loop != 0, and |x_j - x_i| < r, with the squared distance rounded as the
 * float32 expression (dx*dx + dy*dy) + dz*dz (no fused multiply-add), so the edge set equals
 * a brute-force evaluation bit for bit.  Edges come out as src = i, dst = j in (src, dst)
 * order.  Two calls:
 *   1. feq_radius_count fills offsets (N + 1 int64): point i has offsets[i + 1] - offsets[i]
 *      neighbours, offsets[N] = the edge count (read it, then allocate src / dst).
 *   2. feq_radius_fill writes src / dst (num_edges each) from the same inputs and the SAME
 *      workspace, untouched since the count (it holds the sorted cell lists), plus a pair
 *      workspace of feq_radius_pairs_workspace_bytes(num_edges).
 * Cells are cubes of side `cell` >= r with corner (x0, y0, z0); at most 16384 cells per axis
 * and batch ids below 2^21.  status (may be NULL) is set to 1 when a point falls outside
 * that grid, has a non-finite coordinate or a batch id out of range (result invalid).
 * N < 2^31.
 * ------------------------------------------------------------------------ */
size_t feq_radius_workspace_bytes(int64_t num_points);
size_t feq_radius_pairs_workspace_bytes(int64_t num_edges);
int feq_radius_count(const float *xyz, const int64_t *batch, int64_t num_points, float r, int32_t loop, float cell,
                     float x0, float y0, float z0, int64_t *offsets, int32_t *status, void *workspace,
                     size_t workspace_bytes, feq_stream_t stream);
int feq_radius_fill(const float *xyz, const int64_t *batch, int64_t num_points, float r, int32_t loop, float cell,
                    float x0, float y0, float z0, const int64_t *offsets, int64_t num_edges, int64_t *src,
                    int64_t *dst, const void *workspace, size_t workspace_bytes, void *pair_workspace,
                    size_t pair_workspace_bytes, feq_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASHEQ_B200_H */
