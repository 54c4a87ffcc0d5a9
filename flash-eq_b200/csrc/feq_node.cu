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
// EquivariantLinear (flash_eq/layers/linear.py:172-268):
//   y[n, co, p] = sum_ci W[irrep(p) * Cout + co, ci] x[n, ci, p]  (+ bias[co, s] at the
//   s-th l = 0 position).  The reference multiplies every irrep's weight block with every
//   position and gathers; here each position only meets its own irrep's block.
// CTA = 4096 / Cout nodes.  Per irrep r the x tile is re-laid in shared memory as a
// (Cin x nodes * K_r) matrix whose columns are the (node, position) pairs of the irrep,
// and the weight block
// W_r^T as (Cin x Cout): the irrep's product is one small GEMM.  Thread = 4 consecutive
// output channels x K_r quads of 4 consecutive columns; per input channel one float4
// weight load and K_r float4 x loads feed 16 K_r FMAs.  Float32 CUDA-core FMAs, results
// stored straight to y.
// ---------------------------------------------------------------------------
constexpr int kLinThreads = 256;

struct LinArgs {
    NodeRepr R;                    // input and output share the degrees
    int Cin, Cout;
    int8_t scalar_idx[kNodeMaxIrreps];   // irrep -> bias column (-1: not a scalar irrep)
    int nscalar;
    const float *x, *w, *bias;
    float *y;
    int64_t N;
};

// QPT column quads per thread, starting at quad q0 + g (the thread's group g), K = 2l+1.
template <int K, int QPT>
__device__ __forceinline__ void lin_gemm(const LinArgs &a, const float *xs, const float *wt, int wld, int tn,
                                         int64_t n0, int n_nodes, int r, int q0) {
    const int Cin = a.Cin, Cout = a.Cout, d = a.R.d, off = a.R.irr_off[r];
    const int ncol = tn * K;                       // columns: (node, position) pairs, node-major
    const int nq4 = Cout / 4, groups = kLinThreads / nq4;
    const int t = threadIdx.x, cq = t % nq4, g = t / nq4;
    const int sb = a.scalar_idx[r];
    float acc[QPT][4][4];
#pragma unroll
    for (int u = 0; u < QPT; u++)
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[u][c][j] = 0.0f;
    const float *wp = wt + 4 * cq;
    const float *xp = xs + 4 * (q0 + g);
#pragma unroll 2
    for (int ci = 0; ci < Cin; ci++, wp += wld, xp += ncol) {
        const float4 w = *reinterpret_cast<const float4 *>(wp);
#pragma unroll
        for (int u = 0; u < QPT; u++) {
            const float4 xv = *reinterpret_cast<const float4 *>(xp + 4 * u * groups);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                acc[u][0][j] = fmaf(w.x, xa[j], acc[u][0][j]);
                acc[u][1][j] = fmaf(w.y, xa[j], acc[u][1][j]);
                acc[u][2][j] = fmaf(w.z, xa[j], acc[u][2][j]);
                acc[u][3][j] = fmaf(w.w, xa[j], acc[u][3][j]);
            }
        }
    }
    float b[4];
#pragma unroll
    for (int c = 0; c < 4; c++) b[c] = sb >= 0 ? a.bias[(4 * cq + c) * a.nscalar + sb] : 0.0f;
    float *yb = a.y + (n0 * Cout + 4 * cq) * d + off;
#pragma unroll
    for (int u = 0; u < QPT; u++) {
        const int col0 = 4 * (q0 + g + u * groups);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int col = col0 + j, node = col / K, m = col - node * K;   // K constant: no division
            if (node >= n_nodes) continue;
            float *yr = yb + (int64_t)node * Cout * d + m;
#pragma unroll
            for (int c = 0; c < 4; c++) yr[c * d] = acc[u][c][j] + b[c];
        }
    }
}

// One irrep of 2l+1 = K positions: re-lay its x columns, then the GEMM in passes of <= 5 quads.
template <int K>
__device__ __forceinline__ void lin_irrep(const LinArgs &a, float *xs, const float *wt, int wld, int tn,
                                          const float *xg, int64_t n0, int n_nodes, int r) {
    const int Cin = a.Cin, d = a.R.d, off = a.R.irr_off[r], ncol = tn * K;
    // xs[ci][node * K + m] = x[n0 + node, ci, off + m], a batch of loads per thread before the stores
    constexpr int kB = 8;
    for (int i0 = threadIdx.x; i0 < Cin * ncol; i0 += kLinThreads * kB) {
        float v[kB];
#pragma unroll
        for (int u = 0; u < kB; u++) {
            const int i = i0 + u * kLinThreads;
            const int ci = i / ncol, col = i - ci * ncol, node = col / K, m = col - node * K;
            v[u] = (i < Cin * ncol && node < n_nodes) ? __ldg(xg + ((int64_t)node * Cin + ci) * d + off + m) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kB; u++) {
            const int i = i0 + u * kLinThreads;
            if (i < Cin * ncol) xs[i] = v[u];
        }
    }
    __syncthreads();
    const int groups = kLinThreads / (a.Cout / 4);
    // K * groups column quads: each group takes K of them
    if constexpr (K <= 5) {
        lin_gemm<K, K>(a, xs, wt, wld, tn, n0, n_nodes, r, 0);
    } else {
        lin_gemm<K, 5>(a, xs, wt, wld, tn, n0, n_nodes, r, 0);
        lin_gemm<K, K - 5>(a, xs, wt, wld, tn, n0, n_nodes, r, 5 * groups);
    }
}

__global__ void __launch_bounds__(kLinThreads, 1) node_linear_kernel(const __grid_constant__ LinArgs a) {
    extern __shared__ float lsm[];
    const int Cin = a.Cin, Cout = a.Cout, d = a.R.d;
    const int wld = Cout + 4;
    const int nq4 = Cout / 4, groups = kLinThreads / nq4, tn = 4 * groups;   // nodes of this CTA
    float *wt = lsm;                                   // Cin x (Cout + 4)
    float *xs = wt + (size_t)Cin * wld;                // Cin x (tn K_r) for the current irrep
    const int64_t n0 = (int64_t)blockIdx.x * tn;
    const int n_nodes = (int)min64(tn, a.N - n0);
    const float *xg = a.x + n0 * Cin * d;
    for (int r = 0; r < a.R.n_irreps; r++) {
        __syncthreads();   // the previous irrep's tiles are no longer read
        const float *wr = a.w + (int64_t)r * Cout * Cin;
        constexpr int kV = 8;
        for (int i0 = threadIdx.x * 4; i0 < Cout * Cin; i0 += kLinThreads * 4 * kV) {
            float4 v[kV];
#pragma unroll
            for (int u = 0; u < kV; u++) {
                const int i = i0 + u * kLinThreads * 4;
                v[u] = i < Cout * Cin ? __ldg(reinterpret_cast<const float4 *>(wr + i)) : make_float4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < kV; u++) {
                const int i = i0 + u * kLinThreads * 4;
                if (i >= Cout * Cin) break;
                const int co = i / Cin, ci = i - co * Cin;     // Cin % 4 == 0: the 4 share co
                wt[ci * wld + co] = v[u].x;
                wt[(ci + 1) * wld + co] = v[u].y;
                wt[(ci + 2) * wld + co] = v[u].z;
                wt[(ci + 3) * wld + co] = v[u].w;
            }
        }
        switch (a.R.irr_l[r]) {
            case 0: lin_irrep<1>(a, xs, wt, wld, tn, xg, n0, n_nodes, r); break;
            case 1: lin_irrep<3>(a, xs, wt, wld, tn, xg, n0, n_nodes, r); break;
            case 2: lin_irrep<5>(a, xs, wt, wld, tn, xg, n0, n_nodes, r); break;
            case 3: lin_irrep<7>(a, xs, wt, wld, tn, xg, n0, n_nodes, r); break;
            default: lin_irrep<9>(a, xs, wt, wld, tn, xg, n0, n_nodes, r); break;
        }
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

int feq_node_linear(const float *x, int64_t num_nodes, int32_t c_in, int32_t c_out, const int32_t *lvals,
                    int32_t n_lvals, const float *weight, const float *bias, float *y, feq_stream_t stream) {
    LinArgs a;
    memset(&a, 0, sizeof(a));
    int rc = fill_node_repr(lvals, n_lvals, c_in, &a.R);
    if (rc != FEQ_OK) return rc;
    if (num_nodes < 0 || c_out < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !weight || !y) return FEQ_ERR_INVALID_ARGUMENT;
    // channel quads must tile the threads (Cout in 4 .. 1024, a power-of-two multiple of 4)
    if (c_in % 4 || c_out % 4 || c_out > 1024 || kLinThreads % (c_out / 4) || (reinterpret_cast<uintptr_t>(weight) & 15))
        return FEQ_ERR_UNSUPPORTED;
    int kmax = 1;
    for (int r = 0; r < n_lvals; r++) {
        if (lvals[r] > 4) return FEQ_ERR_UNSUPPORTED;
        a.scalar_idx[r] = -1;
        if (lvals[r] == 0 && bias) a.scalar_idx[r] = (int8_t)a.nscalar++;
        kmax = std::max(kmax, 2 * lvals[r] + 1);
    }
    a.Cin = c_in;
    a.Cout = c_out;
    a.x = x;
    a.w = weight;
    a.bias = bias;
    a.y = y;
    a.N = num_nodes;
    const int tn = 4 * (kLinThreads / (c_out / 4));
    const size_t smem = sizeof(float) * ((size_t)c_in * (c_out + 4) + (size_t)c_in * tn * kmax);
    if ((rc = set_smem((const void *)node_linear_kernel, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_linear", (cudaStream_t)stream);
    node_linear_kernel<<<(unsigned)((num_nodes + tn - 1) / tn), kLinThreads, smem, (cudaStream_t)stream>>>(a);
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
