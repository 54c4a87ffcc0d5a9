// feq_node.cu -- node-level operators of the transformer block (inference path).
//
// Reference behaviour replaced (PyTorch in the reference, one launch per elementary op):
//   SeparableEquivariantLayerNorm   flash_eq/layers/norm.py:177-249
//       scalars (l = 0 positions): LayerNorm over channels, (x - mu) / (sd + eps) * w + b
//       higher degrees: one RMS over channels and positions, x * w[c] / sqrt(mean x^2 + eps)
//   EquivariantLayerNorm            flash_eq/layers/norm.py:111-174
//       norms[c, r] = sqrt(sum_{pos in irrep r} x^2 + eps); LayerNorm of norms over channels
//       per irrep (weight / bias over channels, eps 1e-5); x * ln / (norms + eps)
//   RepNorm                         flash_eq/layers/norm.py:19-64
//   EquivariantGating (the gate)    flash_eq/layers/gating.py:17-76: x * sigmoid(z)[c, irrep]
//
// One warp per node: the node's row (C x d floats) is staged in shared memory once, the
// per-node statistics are warp reductions, and the output row is written coalesced.
// All four are memory-bound: one read and one write of the row (plus z / norms).
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <algorithm>

#include "feq_internal.cuh"

namespace feq {
namespace {

constexpr int kNodeWarps = 4;
constexpr int kNodeMaxIrreps = 32;
constexpr int kNodeMaxScalars = 16;

__device__ __forceinline__ float nwsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

struct NodeRepr {
    int C, d, n_irreps;
    int8_t irr_l[kNodeMaxIrreps];
    int16_t irr_off[kNodeMaxIrreps];
    int8_t pos_irr[kMaxDim];          // position -> irrep
};

struct SepLnArgs {
    NodeRepr R;
    int nscalar, n_higher;            // scalar positions, higher positions
    int16_t scalar_pos[kNodeMaxScalars];
    int8_t scalar_idx[kMaxDim];       // position -> scalar index, -1 for higher positions
    const float *x, *w_s, *b_s, *w_h;  // w_s, b_s: (C, nscalar); w_h: (C)
    float eps;
    float *out;
    int64_t N;
};

// Walk the row elements j = lane, lane + 32, ... with their (channel, position) pair
// updated incrementally (no integer division per element).
struct RowWalk {
    int c, p, dc, dp, d;
    __device__ __forceinline__ RowWalk(int lane, int d_) : d(d_) {
        c = lane / d_;
        p = lane - c * d_;
        dc = 32 / d_;
        dp = 32 - dc * d_;
    }
    __device__ __forceinline__ void next() {
        c += dc;
        p += dp;
        if (p >= d) {
            p -= d;
            c++;
        }
    }
};

// Copy one node row into shared memory, all of a lane's loads issued before its stores
// (a load -> store pair per iteration would serialise on the load latency).
__device__ __forceinline__ void stage_row(float *row, const float *src, int n, int lane) {
    constexpr int kB = 8;
    if ((n & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(row)) & 15) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *r4 = reinterpret_cast<float4 *>(row);
        const int n4 = n / 4;
        for (int i0 = lane; i0 < n4; i0 += 32 * kB) {
            float4 v[kB];
#pragma unroll
            for (int u = 0; u < kB; u++)
                if (i0 + 32 * u < n4) v[u] = __ldg(s4 + i0 + 32 * u);
#pragma unroll
            for (int u = 0; u < kB; u++)
                if (i0 + 32 * u < n4) r4[i0 + 32 * u] = v[u];
        }
    } else {
        for (int i0 = lane; i0 < n; i0 += 32 * kB) {
            float v[kB];
#pragma unroll
            for (int u = 0; u < kB; u++)
                if (i0 + 32 * u < n) v[u] = __ldg(src + i0 + 32 * u);
#pragma unroll
            for (int u = 0; u < kB; u++)
                if (i0 + 32 * u < n) row[i0 + 32 * u] = v[u];
        }
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kNodeWarps * 32) sep_layernorm_kernel(const __grid_constant__ SepLnArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *row = nsm + (size_t)warp * n;
    __shared__ float mu_s[kNodeWarps][kNodeMaxScalars], inv_s[kNodeWarps][kNodeMaxScalars], rms_s[kNodeWarps];
    __shared__ int8_t sidx_s[kMaxDim];     // per-lane lookups from shared memory, not the parameter bank
    for (int i = threadIdx.x; i < d; i += blockDim.x) sidx_s[i] = a.scalar_idx[i];
    __syncthreads();
    for (int64_t node = (int64_t)blockIdx.x * kNodeWarps + warp; node < a.N; node += (int64_t)gridDim.x * kNodeWarps) {
        stage_row(row, a.x + node * n, n, lane);
        for (int s = 0; s < a.nscalar; s++) {
            const int p = a.scalar_pos[s];
            float sum = 0.0f;
            for (int c = lane; c < C; c += 32) sum += row[c * d + p];
            const float mu = nwsum(sum) / (float)C;
            float sq = 0.0f;
            for (int c = lane; c < C; c += 32) {
                const float t = row[c * d + p] - mu;
                sq = fmaf(t, t, sq);
            }
            const float sd = sqrtf(nwsum(sq) / (float)C);
            if (lane == 0) {
                mu_s[warp][s] = mu;
                inv_s[warp][s] = sd + a.eps;
            }
        }
        if (a.n_higher > 0) {
            float sq = 0.0f;
            RowWalk w(lane, d);
            for (int j = lane; j < n; j += 32, w.next())
                if (sidx_s[w.p] < 0) sq = fmaf(row[j], row[j], sq);
            sq = nwsum(sq);
            if (lane == 0) rms_s[warp] = sqrtf(sq / (float)(C * a.n_higher) + a.eps);
        }
        __syncwarp();
        float *orow = a.out + node * n;
        const float rms = a.n_higher > 0 ? rms_s[warp] : 1.0f;
        RowWalk w(lane, d);
        for (int j = lane; j < n; j += 32, w.next()) {
            float v = row[j];
            const int s = sidx_s[w.p];
            if (s >= 0) {
                v = (v - mu_s[warp][s]) / inv_s[warp][s] * a.w_s[w.c * a.nscalar + s] + a.b_s[w.c * a.nscalar + s];
            } else {
                v = v * (a.w_h[w.c] / rms);
            }
            orow[j] = v;
        }
        __syncwarp();
    }
}

struct EqLnArgs {
    NodeRepr R;
    const float *x, *ln_w, *ln_b;   // ln_w / ln_b: (C) or NULL (mult 1: no LayerNorm)
    float ln_eps, rn_eps, eps;
    float *out;
    int64_t N;
};

// norms of this warp's node row into nrm[c * n_irreps + r] (irrep offsets / sizes from shared memory)
__device__ __forceinline__ void row_norms(const NodeRepr &R, const int16_t *ioff, const int16_t *ik, const float *row,
                                          float rn_eps, float *nrm, int lane) {
    const int C = R.C, d = R.d;
    for (int i = lane; i < C * R.n_irreps; i += 32) {
        const int c = i / R.n_irreps, r = i - c * R.n_irreps;
        const int off = ioff[r], k = ik[r];
        float s = 0.0f;
        for (int m = 0; m < k; m++) {
            const float v = row[c * d + off + m];
            s = fmaf(v, v, s);
        }
        nrm[i] = sqrtf(s + rn_eps);
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kNodeWarps * 32) equi_layernorm_kernel(const __grid_constant__ EqLnArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d, nr = a.R.n_irreps;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *row = nsm + (size_t)warp * (n + C * nr);
    float *nrm = row + n;               // norms, then the rescaling factors
    __shared__ int8_t pirr_s[kMaxDim];
    __shared__ int16_t ioff_s[kNodeMaxIrreps], ik_s[kNodeMaxIrreps];
    for (int i = threadIdx.x; i < d; i += blockDim.x) pirr_s[i] = a.R.pos_irr[i];
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        ioff_s[i] = a.R.irr_off[i];
        ik_s[i] = 2 * a.R.irr_l[i] + 1;
    }
    __syncthreads();
    for (int64_t node = (int64_t)blockIdx.x * kNodeWarps + warp; node < a.N; node += (int64_t)gridDim.x * kNodeWarps) {
        stage_row(row, a.x + node * n, n, lane);
        row_norms(a.R, ioff_s, ik_s, row, a.rn_eps, nrm, lane);
        for (int r = 0; r < nr; r++) {
            if (a.ln_w) {
                float s = 0.0f;
                for (int c = lane; c < C; c += 32) s += nrm[c * nr + r];
                const float mu = nwsum(s) / (float)C;
                float q = 0.0f;
                for (int c = lane; c < C; c += 32) {
                    const float t = nrm[c * nr + r] - mu;
                    q = fmaf(t, t, q);
                }
                const float rstd = rsqrtf(nwsum(q) / (float)C + a.ln_eps);
                for (int c = lane; c < C; c += 32) {
                    const float v = nrm[c * nr + r];
                    const float ln = (v - mu) * rstd * a.ln_w[c] + a.ln_b[c];
                    nrm[c * nr + r] = ln / (v + a.eps);
                }
            } else {
                for (int c = lane; c < C; c += 32) nrm[c * nr + r] = 1.0f / (nrm[c * nr + r] + a.eps);
            }
        }
        __syncwarp();
        float *orow = a.out + node * n;
        RowWalk w(lane, d);
        for (int j = lane; j < n; j += 32, w.next()) orow[j] = row[j] * nrm[w.c * nr + pirr_s[w.p]];
        __syncwarp();
    }
}

struct RepNormArgs {
    NodeRepr R;
    const float *x;
    float eps;
    float *norms;    // (N, C, n_irreps)
    const float *z;  // gate: (N, C * n_irreps) pre-activation
    float *out;      // gate: (N, C, d)
    int64_t N;
};

__global__ void __launch_bounds__(kNodeWarps * 32) rep_norm_kernel(const __grid_constant__ RepNormArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d, nr = a.R.n_irreps;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *row = nsm + (size_t)warp * n;
    __shared__ int16_t ioff_s[kNodeMaxIrreps], ik_s[kNodeMaxIrreps];
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        ioff_s[i] = a.R.irr_off[i];
        ik_s[i] = 2 * a.R.irr_l[i] + 1;
    }
    __syncthreads();
    for (int64_t node = (int64_t)blockIdx.x * kNodeWarps + warp; node < a.N; node += (int64_t)gridDim.x * kNodeWarps) {
        stage_row(row, a.x + node * n, n, lane);
        float *o = a.norms + node * (int64_t)C * nr;
        for (int i = lane; i < C * nr; i += 32) {
            const int c = i / nr, r = i - c * nr;
            const int off = ioff_s[r], k = ik_s[r];
            float s = 0.0f;
            for (int m = 0; m < k; m++) {
                const float v = row[c * d + off + m];
                s = fmaf(v, v, s);
            }
            o[i] = sqrtf(s + a.eps);
        }
        __syncwarp();
    }
}

// out[n, c, p] = x[n, c, p] * sigmoid(z[n, c * n_irreps + irrep(p)]); one warp per node,
// the node's gates computed once into shared memory.
__global__ void __launch_bounds__(kNodeWarps * 32) gate_kernel(const __grid_constant__ RepNormArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d, nr = a.R.n_irreps;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *gs = nsm + (size_t)warp * C * nr;
    __shared__ int8_t pirr_s[kMaxDim];
    for (int i = threadIdx.x; i < d; i += blockDim.x) pirr_s[i] = a.R.pos_irr[i];
    __syncthreads();
    for (int64_t node = (int64_t)blockIdx.x * kNodeWarps + warp; node < a.N; node += (int64_t)gridDim.x * kNodeWarps) {
        const float *zr = a.z + node * (int64_t)C * nr;
        for (int i = lane; i < C * nr; i += 32) gs[i] = 1.0f / (1.0f + expf(-__ldg(zr + i)));
        __syncwarp();
        const float *xr = a.x + node * n;
        float *orow = a.out + node * n;
        RowWalk w(lane, d);
        for (int j = lane; j < n; j += 32, w.next()) orow[j] = __ldg(xr + j) * gs[w.c * nr + pirr_s[w.p]];
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Position-major layout for EquivariantLinear (flash_eq/layers/linear.py:172-268):
// xt[p][n][c] = x[n][c][p].  Each irrep's positions p = off .. off + 2l are then one
// contiguous ((2l+1) N x C) matrix and its channel mix y = W_r x a single plain GEMM
// (a library SGEMM, 1 / nreps of the reference's FLOPs: the reference multiplies every
// irrep's weight block with every position and gathers).  CTA = up to 16 nodes: the node rows
// are read contiguously into shared memory and each position's (8 x C) slab written
// contiguously (and the reverse on the way back, with the bias added).
// ---------------------------------------------------------------------------
constexpr int kPmNodes = 16;

// nodes per CTA: up to 16, as many as fit 96 KB of shared memory
inline int pm_nodes(int C, int d) {
    return (int)std::min<int64_t>(kPmNodes, (int64_t)(96 * 1024) / ((int64_t)C * d * 4));
}

// the (nodes x C x d) tile of this CTA into shared memory, float4 when aligned
__device__ __forceinline__ void pm_load_tile(float *tsm, const float *src, int tile) {
    if ((tile & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *t4 = reinterpret_cast<float4 *>(tsm);
        for (int i = threadIdx.x; i < tile / 4; i += blockDim.x) t4[i] = __ldg(s4 + i);
    } else {
        for (int i = threadIdx.x; i < tile; i += blockDim.x) tsm[i] = __ldg(src + i);
    }
}

__global__ void __launch_bounds__(256) to_posmajor_kernel(const float *__restrict__ x, int64_t N, int C, int d,
                                                          int tn, float *__restrict__ xt) {
    extern __shared__ float tsm[];
    const int64_t n0 = (int64_t)blockIdx.x * tn;
    const int nn = (int)min64(tn, N - n0);
    pm_load_tile(tsm, x + n0 * C * d, nn * C * d);
    __syncthreads();
    const int slab = nn * C;                 // (nodes x channels) of one position, a multiple of 4
    for (int p = 0; p < d; p++) {
        float4 *dst = reinterpret_cast<float4 *>(xt + (int64_t)p * N * C + n0 * C);
        for (int r = 4 * threadIdx.x; r < slab; r += 4 * blockDim.x)     // r = node * C + c
            dst[r / 4] = make_float4(tsm[r * d + p], tsm[(r + 1) * d + p], tsm[(r + 2) * d + p], tsm[(r + 3) * d + p]);
    }
}

// y[n][c][p] = yt[p][n][c] (+ bias[c, s] at the s-th scalar position)
__global__ void __launch_bounds__(256) from_posmajor_kernel(const float *__restrict__ yt, int64_t N, int C, int d,
                                                            const float *__restrict__ bias, int nscalar,
                                                            const int8_t *__restrict__ scalar_idx_d, int tn,
                                                            float *__restrict__ y) {
    extern __shared__ float tsm[];
    const int64_t n0 = (int64_t)blockIdx.x * tn;
    const int nn = (int)min64(tn, N - n0);
    const int slab = nn * C;
    for (int p = 0; p < d; p++) {
        const float4 *src = reinterpret_cast<const float4 *>(yt + (int64_t)p * N * C + n0 * C);
        const int sb = (bias && scalar_idx_d) ? scalar_idx_d[p] : -1;
        for (int r = 4 * threadIdx.x; r < slab; r += 4 * blockDim.x) {
            float4 v = __ldg(src + r / 4);
            if (sb >= 0) {
                const int c = r % C;             // C % 4 == 0: r .. r + 3 share the node
                v.x += __ldg(bias + c * nscalar + sb);
                v.y += __ldg(bias + (c + 1) * nscalar + sb);
                v.z += __ldg(bias + (c + 2) * nscalar + sb);
                v.w += __ldg(bias + (c + 3) * nscalar + sb);
            }
            tsm[r * d + p] = v.x;
            tsm[(r + 1) * d + p] = v.y;
            tsm[(r + 2) * d + p] = v.z;
            tsm[(r + 3) * d + p] = v.w;
        }
    }
    __syncthreads();
    const int tile = slab * d;
    float *dst = y + n0 * C * d;
    if ((tile & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        for (int i = threadIdx.x; i < tile / 4; i += blockDim.x)
            reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(tsm)[i];
    } else {
        for (int i = threadIdx.x; i < tile; i += blockDim.x) dst[i] = tsm[i];
    }
}

int fill_node_repr(const int32_t *lvals, int32_t n, int32_t C, NodeRepr *R) {
    if (!lvals || n < 1 || n > kNodeMaxIrreps || C < 1) return FEQ_ERR_INVALID_ARGUMENT;
    memset(R, 0, sizeof(*R));
    int off = 0;
    for (int r = 0; r < n; r++) {
        if (lvals[r] < 0 || lvals[r] > kMaxL) return FEQ_ERR_INVALID_ARGUMENT;
        R->irr_l[r] = (int8_t)lvals[r];
        R->irr_off[r] = (int16_t)off;
        for (int m = 0; m < 2 * lvals[r] + 1; m++) {
            if (off + m >= kMaxDim) return FEQ_ERR_UNSUPPORTED;
            R->pos_irr[off + m] = (int8_t)r;
        }
        off += 2 * lvals[r] + 1;
    }
    R->C = C;
    R->d = off;
    R->n_irreps = n;
    return FEQ_OK;
}

int node_grid(int64_t N) { return (int)min64((N + kNodeWarps - 1) / kNodeWarps, 148 * 16); }

int set_smem(const void *fn, size_t smem) {
    if (smem > 200 * 1024) return FEQ_ERR_UNSUPPORTED;
    if (smem > 48 * 1024)
        FEQ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    return FEQ_OK;
}

}  // namespace
}  // namespace feq

using namespace feq;

extern "C" {

int feq_node_sep_layernorm(const float *x, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                           const float *w_scalar, const float *b_scalar, const float *w_higher, float eps, float *out,
                           feq_stream_t stream) {
    SepLnArgs a;
    memset(&a, 0, sizeof(a));
    int rc = fill_node_repr(lvals, n_lvals, C, &a.R);
    if (rc != FEQ_OK) return rc;
    if (num_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    memset(a.scalar_idx, -1, sizeof(a.scalar_idx));
    for (int r = 0; r < n_lvals; r++) {
        if (lvals[r] == 0) {
            if (a.nscalar >= kNodeMaxScalars) return FEQ_ERR_UNSUPPORTED;
            a.scalar_idx[a.R.irr_off[r]] = (int8_t)a.nscalar;
            a.scalar_pos[a.nscalar++] = a.R.irr_off[r];
        }
    }
    a.n_higher = a.R.d - a.nscalar;
    if (!x || !out || (a.nscalar > 0 && (!w_scalar || !b_scalar)) || (a.n_higher > 0 && !w_higher))
        return FEQ_ERR_INVALID_ARGUMENT;
    a.x = x;
    a.w_s = w_scalar;
    a.b_s = b_scalar;
    a.w_h = w_higher;
    a.eps = eps;
    a.out = out;
    a.N = num_nodes;
    const size_t smem = sizeof(float) * kNodeWarps * (size_t)C * a.R.d;
    if ((rc = set_smem((const void *)sep_layernorm_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_norm", (cudaStream_t)stream);
    sep_layernorm_kernel<<<node_grid(num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_node_layernorm(const float *x, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                       const float *ln_weight, const float *ln_bias, float ln_eps, float rep_eps, float eps, float *out,
                       feq_stream_t stream) {
    EqLnArgs a;
    memset(&a, 0, sizeof(a));
    int rc = fill_node_repr(lvals, n_lvals, C, &a.R);
    if (rc != FEQ_OK) return rc;
    if (num_nodes < 0 || (ln_weight == nullptr) != (ln_bias == nullptr)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !out) return FEQ_ERR_INVALID_ARGUMENT;
    a.x = x;
    a.ln_w = ln_weight;
    a.ln_b = ln_bias;
    a.ln_eps = ln_eps;
    a.rn_eps = rep_eps;
    a.eps = eps;
    a.out = out;
    a.N = num_nodes;
    const size_t smem = sizeof(float) * kNodeWarps * ((size_t)C * a.R.d + (size_t)C * n_lvals);
    if ((rc = set_smem((const void *)equi_layernorm_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_norm", (cudaStream_t)stream);
    equi_layernorm_kernel<<<node_grid(num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_node_rep_norm(const float *x, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals, float eps,
                      float *norms, feq_stream_t stream) {
    RepNormArgs a;
    memset(&a, 0, sizeof(a));
    int rc = fill_node_repr(lvals, n_lvals, C, &a.R);
    if (rc != FEQ_OK) return rc;
    if (num_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !norms) return FEQ_ERR_INVALID_ARGUMENT;
    a.x = x;
    a.eps = eps;
    a.norms = norms;
    a.N = num_nodes;
    const size_t smem = sizeof(float) * kNodeWarps * (size_t)C * a.R.d;
    if ((rc = set_smem((const void *)rep_norm_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_norm", (cudaStream_t)stream);
    rep_norm_kernel<<<node_grid(num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_node_to_posmajor(const float *x, int64_t num_nodes, int32_t C, int32_t d, float *xt, feq_stream_t stream) {
    if (num_nodes < 0 || C < 1 || d < 1 || d > kMaxDim) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !xt) return FEQ_ERR_INVALID_ARGUMENT;
    if (C % 4 || (reinterpret_cast<uintptr_t>(xt) & 15)) return FEQ_ERR_UNSUPPORTED;
    const int tn = pm_nodes(C, d);
    if (tn < 1) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = sizeof(float) * tn * (size_t)C * d;
    int rc;
    if ((rc = set_smem((const void *)to_posmajor_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_layout", (cudaStream_t)stream);
    to_posmajor_kernel<<<(unsigned)((num_nodes + tn - 1) / tn), 256, smem, (cudaStream_t)stream>>>(
        x, num_nodes, C, d, tn, xt);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_node_from_posmajor(const float *yt, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                           const float *bias, const int8_t *scalar_index, float *y, feq_stream_t stream) {
    NodeRepr R;
    int rc = fill_node_repr(lvals, n_lvals, C, &R);
    if (rc != FEQ_OK) return rc;
    if (num_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!yt || !y || (bias && !scalar_index)) return FEQ_ERR_INVALID_ARGUMENT;
    if (C % 4 || (reinterpret_cast<uintptr_t>(yt) & 15)) return FEQ_ERR_UNSUPPORTED;
    int nscalar = 0;
    for (int r = 0; r < n_lvals; r++) nscalar += lvals[r] == 0;
    const int tn = pm_nodes(C, R.d);
    if (tn < 1) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = sizeof(float) * tn * (size_t)C * R.d;
    if ((rc = set_smem((const void *)from_posmajor_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_layout", (cudaStream_t)stream);
    from_posmajor_kernel<<<(unsigned)((num_nodes + tn - 1) / tn), 256, smem, (cudaStream_t)stream>>>(
        yt, num_nodes, C, R.d, bias, nscalar, scalar_index, tn, y);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_node_gate(const float *x, const float *z, int64_t num_nodes, int32_t C, const int32_t *lvals, int32_t n_lvals,
                  float *out, feq_stream_t stream) {
    RepNormArgs a;
    memset(&a, 0, sizeof(a));
    int rc = fill_node_repr(lvals, n_lvals, C, &a.R);
    if (rc != FEQ_OK) return rc;
    if (num_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !z || !out) return FEQ_ERR_INVALID_ARGUMENT;
    a.x = x;
    a.z = z;
    a.out = out;
    a.N = num_nodes;
    const size_t smem = sizeof(float) * kNodeWarps * (size_t)C * n_lvals;
    if ((rc = set_smem((const void *)gate_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_gate", (cudaStream_t)stream);
    gate_kernel<<<node_grid(num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // extern "C"
