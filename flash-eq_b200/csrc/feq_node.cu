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
// per-node statistics are warp reductions, the transform runs in place with lane = channel,
// and the output row is written coalesced.
// All four are memory-bound: one read and one write of the row (plus z / norms).
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "feq_internal.cuh"

namespace feq {
namespace {

constexpr int kNodeWarps = 4;
constexpr int kNodeBlocksPerSm = 6;      // 24 warps per SM: <= 85 registers per thread
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

// Row layout in shared memory: element (c, p) at c * ds + p, with the channel stride ds = d
// for odd d and d + 1 for even d.  The per-node transforms then run with lane = channel over
// the positions p: the 32 lanes read 32 rows ds apart (distinct banks, as ds is odd), the
// branch on the position's kind is uniform across the warp and no (c, p) pair is decoded
// from a flat index.
__host__ __device__ __forceinline__ int odd_stride(int d) { return d | 1; }

// Float4 i of a row with d % 4 == 0 holds positions 4q .. 4q + 3 of one channel c; walk
// (c, q) for i = lane, lane + 32, ... without a division per step.
struct QuadWalk {
    int c, q, dc, dq, d4;
    __device__ __forceinline__ QuadWalk(int lane, int d4_) : d4(d4_) {
        c = lane / d4_;
        q = lane - c * d4_;
        dc = 32 / d4_;
        dq = 32 - dc * d4_;
    }
    __device__ __forceinline__ void next() {
        c += dc;
        q += dq;
        if (q >= d4) {
            q -= d4;
            c++;
        }
    }
};

// Node row -> row[c * ds + p]: a straight float4 copy when ds == d; for d % 4 == 0 float4
// loads (four positions of one channel each) scattered to the padded rows; else scalar loads.
// All of a batch's loads are issued before its stores.
__device__ __forceinline__ void stage_row_ds(float *row, const float *src, int C, int d, int ds, int lane) {
    const int n = C * d;
    if (ds == d) {
        stage_row(row, src, n, lane);
        return;
    }
    constexpr int kB = 8;
    if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        constexpr int kB4 = 4;                // float4s per lane in flight (registers are short)
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        const int n4 = n / 4;
        QuadWalk w(lane, d / 4);
        for (int i0 = lane; i0 < n4; i0 += 32 * kB4) {
            float4 v[kB4];
#pragma unroll
            for (int u = 0; u < kB4; u++)
                if (i0 + 32 * u < n4) v[u] = __ldg(s4 + i0 + 32 * u);
#pragma unroll
            for (int u = 0; u < kB4; u++)
                if (i0 + 32 * u < n4) {
                    float *r = row + w.c * ds + 4 * w.q;
                    r[0] = v[u].x;
                    r[1] = v[u].y;
                    r[2] = v[u].z;
                    r[3] = v[u].w;
                    w.next();
                }
        }
        __syncwarp();
        return;
    }
    RowWalk w(lane, d);
    for (int i0 = lane; i0 < n; i0 += 32 * kB) {
        float v[kB];
#pragma unroll
        for (int u = 0; u < kB; u++)
            if (i0 + 32 * u < n) v[u] = __ldg(src + i0 + 32 * u);
#pragma unroll
        for (int u = 0; u < kB; u++)
            if (i0 + 32 * u < n) {
                row[w.c * ds + w.p] = v[u];
                w.next();
            }
    }
    __syncwarp();
}

// row[c * ds + p] -> node row in global memory, coalesced (float4 when ds == d and aligned)
__device__ __forceinline__ void write_row_ds(float *dst, const float *row, int C, int d, int ds, int lane) {
    const int n = C * d;
    __syncwarp();
    if (ds == d && (n & 3) == 0 && ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(row)) & 15) == 0) {
        const float4 *r4 = reinterpret_cast<const float4 *>(row);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = lane; i < n / 4; i += 32) d4[i] = r4[i];
    } else if (ds == d) {
        for (int i = lane; i < n; i += 32) dst[i] = row[i];
    } else if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        QuadWalk w(lane, d / 4);
        for (int i = lane; i < n / 4; i += 32, w.next()) {
            const float *r = row + w.c * ds + 4 * w.q;
            d4[i] = make_float4(r[0], r[1], r[2], r[3]);
        }
    } else {
        RowWalk w(lane, d);
        for (int i = lane; i < n; i += 32, w.next()) dst[i] = row[w.c * ds + w.p];
    }
    __syncwarp();
}

// ---- node loop: the next node's row is copied into shared memory (cp.async, 16 bytes a
// lane) while the current one is transformed.  kAsync needs ds == d, C * d % 4 == 0 and
// 16-byte aligned rows; otherwise each row is staged through registers (stage_row_ds).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// body(node, row) reads the staged row (C * ds floats) and writes the node's outputs.
template <bool kAsync, typename Body>
__device__ __forceinline__ void node_loop(const float *__restrict__ x, int64_t N, int C, int d, int ds, float *buf,
                                          int lane, int64_t first, int64_t stride, Body body) {
    const int n = C * d;
    if constexpr (!kAsync) {
        for (int64_t node = first; node < N; node += stride) {
            stage_row_ds(buf, x + node * n, C, d, ds, lane);
            body(node, buf);
            __syncwarp();
        }
    } else {
        const int slot_floats = C * ds;
        auto issue = [&](float *dst, int64_t node) {
            const float4 *s4 = reinterpret_cast<const float4 *>(x + node * n);
            float4 *d4 = reinterpret_cast<float4 *>(dst);
            for (int i = lane; i < n / 4; i += 32) cp_async16(d4 + i, s4 + i);
        };
        if (first < N) issue(buf, first);
        cp_async_commit();
        int slot = 0;
        for (int64_t node = first; node < N; node += stride, slot ^= 1) {
            if (node + stride < N) issue(buf + (slot ^ 1) * slot_floats, node + stride);
            cp_async_commit();
            cp_async_wait1();                // this lane's copies of the current row have landed
            __syncwarp();                    // ... and every other lane's
            body(node, buf + slot * slot_floats);
            __syncwarp();                    // this slot is refilled by the next iteration's copies
        }
    }
}

// Shared memory: per warp the node row (C * ds floats); per block the weights w_s, b_s
// (C x nscalar) and w_h (C).
template <bool kAsync>
__global__ void __launch_bounds__(kNodeWarps * 32, kNodeBlocksPerSm) sep_layernorm_kernel(const __grid_constant__ SepLnArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d, ds = odd_stride(d), ns = a.nscalar;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kSlots = kAsync ? 2 : 1;      // row buffers per warp (the next row in flight)
    float *buf = nsm + (size_t)warp * kSlots * C * ds;
    float *ws = nsm + (size_t)kNodeWarps * kSlots * C * ds, *bs = ws + C * ns, *wh = bs + C * ns;
    __shared__ float mu_s[kNodeWarps][kNodeMaxScalars], inv_s[kNodeWarps][kNodeMaxScalars];
    __shared__ int8_t sidx_s[kMaxDim];
    for (int i = threadIdx.x; i < d; i += blockDim.x) sidx_s[i] = a.scalar_idx[i];
    for (int i = threadIdx.x; i < C * ns; i += blockDim.x) {
        ws[i] = a.w_s[i];
        bs[i] = a.b_s[i];
    }
    if (a.n_higher > 0)
        for (int i = threadIdx.x; i < C; i += blockDim.x) wh[i] = a.w_h[i];
    __syncthreads();
    node_loop<kAsync>(a.x, a.N, C, d, ds, buf, lane, (int64_t)blockIdx.x * kNodeWarps + warp,
                      (int64_t)gridDim.x * kNodeWarps, [&](int64_t node, float *row) {
        // scalar positions: LayerNorm over the channels (mean, then the biased variance)
        for (int s = 0; s < ns; s++) {
            const int p = a.scalar_pos[s];
            float sum = 0.0f;
            for (int c = lane; c < C; c += 32) sum += row[c * ds + p];
            const float mu = nwsum(sum) / (float)C;
            float sq = 0.0f;
            for (int c = lane; c < C; c += 32) {
                const float t = row[c * ds + p] - mu;
                sq = fmaf(t, t, sq);
            }
            const float sd = sqrtf(nwsum(sq) / (float)C);
            if (lane == 0) {
                mu_s[warp][s] = mu;
                inv_s[warp][s] = 1.0f / (sd + a.eps);
            }
        }
        // higher positions: one RMS over every channel and higher position
        float inv_rms = 1.0f;
        if (a.n_higher > 0) {
            float sq = 0.0f;
            for (int c = lane; c < C; c += 32)
#pragma unroll 4
                for (int p = 0; p < d; p++)
                    if (sidx_s[p] < 0) {
                        const float v = row[c * ds + p];
                        sq = fmaf(v, v, sq);
                    }
            inv_rms = 1.0f / sqrtf(nwsum(sq) / (float)(C * a.n_higher) + a.eps);
        }
        __syncwarp();
        for (int c = lane; c < C; c += 32) {
            const float hs = a.n_higher > 0 ? wh[c] * inv_rms : 0.0f;
#pragma unroll 4
            for (int p = 0; p < d; p++) {
                const int s = sidx_s[p];
                float v = row[c * ds + p];
                if (s >= 0) v = fmaf(v - mu_s[warp][s], ws[c * ns + s] * inv_s[warp][s], bs[c * ns + s]);
                else v *= hs;
                row[c * ds + p] = v;
            }
        }
        write_row_ds(a.out + node * n, row, C, d, ds, lane);
    });
}

struct EqLnArgs {
    NodeRepr R;
    const float *x, *ln_w, *ln_b;   // ln_w / ln_b: (C) or NULL (mult 1: no LayerNorm)
    float ln_eps, rn_eps, eps;
    float *out;
    int64_t N;
};

// norms of this warp's node row: nrm[c * nrs + r] = sqrt(sum over irrep r's positions of
// x^2 + rn_eps), lane = channel (nrs: odd stride >= n_irreps)
__device__ __forceinline__ void row_norms(const NodeRepr &R, const int16_t *ioff, const int16_t *ik, const float *row,
                                          int ds, float rn_eps, float *nrm, int nrs, int lane) {
    for (int c = lane; c < R.C; c += 32)
        for (int r = 0; r < R.n_irreps; r++) {
            const float *v = row + c * ds + ioff[r];
            float s = 0.0f;
            for (int m = 0; m < ik[r]; m++) s = fmaf(v[m], v[m], s);
            nrm[c * nrs + r] = sqrtf(s + rn_eps);
        }
    __syncwarp();
}

template <bool kAsync>
__global__ void __launch_bounds__(kNodeWarps * 32, kNodeBlocksPerSm) equi_layernorm_kernel(const __grid_constant__ EqLnArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d, nr = a.R.n_irreps, ds = odd_stride(d), nrs = odd_stride(nr);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kSlots = kAsync ? 2 : 1;
    float *buf = nsm + (size_t)warp * (kSlots * C * ds + C * nrs);
    float *nrm = buf + kSlots * C * ds;      // norms, then the rescaling factors
    __shared__ int8_t pirr_s[kMaxDim];
    __shared__ int16_t ioff_s[kNodeMaxIrreps], ik_s[kNodeMaxIrreps];
    for (int i = threadIdx.x; i < d; i += blockDim.x) pirr_s[i] = a.R.pos_irr[i];
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        ioff_s[i] = a.R.irr_off[i];
        ik_s[i] = 2 * a.R.irr_l[i] + 1;
    }
    __syncthreads();
    node_loop<kAsync>(a.x, a.N, C, d, ds, buf, lane, (int64_t)blockIdx.x * kNodeWarps + warp,
                      (int64_t)gridDim.x * kNodeWarps, [&](int64_t node, float *row) {
        row_norms(a.R, ioff_s, ik_s, row, ds, a.rn_eps, nrm, nrs, lane);
        for (int r = 0; r < nr; r++) {
            if (a.ln_w) {
                float s = 0.0f;
                for (int c = lane; c < C; c += 32) s += nrm[c * nrs + r];
                const float mu = nwsum(s) / (float)C;
                float q = 0.0f;
                for (int c = lane; c < C; c += 32) {
                    const float t = nrm[c * nrs + r] - mu;
                    q = fmaf(t, t, q);
                }
                const float rstd = rsqrtf(nwsum(q) / (float)C + a.ln_eps);
                for (int c = lane; c < C; c += 32) {
                    const float v = nrm[c * nrs + r];
                    const float ln = (v - mu) * rstd * a.ln_w[c] + a.ln_b[c];
                    nrm[c * nrs + r] = ln / (v + a.eps);
                }
            } else {
                for (int c = lane; c < C; c += 32) nrm[c * nrs + r] = 1.0f / (nrm[c * nrs + r] + a.eps);
            }
        }
        __syncwarp();
        for (int c = lane; c < C; c += 32)
#pragma unroll 4
            for (int p = 0; p < d; p++) row[c * ds + p] *= nrm[c * nrs + pirr_s[p]];
        write_row_ds(a.out + node * n, row, C, d, ds, lane);
    });
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

template <bool kAsync>
__global__ void __launch_bounds__(kNodeWarps * 32, kNodeBlocksPerSm) rep_norm_kernel(const __grid_constant__ RepNormArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, nr = a.R.n_irreps, ds = odd_stride(d);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kSlots = kAsync ? 2 : 1;
    float *buf = nsm + (size_t)warp * kSlots * C * ds;
    __shared__ int16_t ioff_s[kNodeMaxIrreps], ik_s[kNodeMaxIrreps];
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        ioff_s[i] = a.R.irr_off[i];
        ik_s[i] = 2 * a.R.irr_l[i] + 1;
    }
    __syncthreads();
    node_loop<kAsync>(a.x, a.N, C, d, ds, buf, lane, (int64_t)blockIdx.x * kNodeWarps + warp,
                      (int64_t)gridDim.x * kNodeWarps, [&](int64_t node, float *row) {
        float *o = a.norms + node * (int64_t)C * nr;
        for (int c = lane; c < C; c += 32)
            for (int r = 0; r < nr; r++) {
                const float *v = row + c * ds + ioff_s[r];
                float s = 0.0f;
                for (int m = 0; m < ik_s[r]; m++) s = fmaf(v[m], v[m], s);
                o[c * nr + r] = sqrtf(s + a.eps);
            }
    });
}

// out[n, c, p] = x[n, c, p] * sigmoid(z[n, c * n_irreps + irrep(p)]); one warp per node:
// the node's gates into shared memory (coalesced z reads), the row staged, scaled with
// lane = channel and written back coalesced.
template <bool kAsync>
__global__ void __launch_bounds__(kNodeWarps * 32, kNodeBlocksPerSm) gate_kernel(const __grid_constant__ RepNormArgs a) {
    extern __shared__ float nsm[];
    const int C = a.R.C, d = a.R.d, n = C * d, nr = a.R.n_irreps, ds = odd_stride(d);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kSlots = kAsync ? 2 : 1;
    float *buf = nsm + (size_t)warp * (kSlots * C * ds + C * nr);
    float *gs = buf + kSlots * C * ds;
    __shared__ int8_t pirr_s[kMaxDim];
    for (int i = threadIdx.x; i < d; i += blockDim.x) pirr_s[i] = a.R.pos_irr[i];
    __syncthreads();
    node_loop<kAsync>(a.x, a.N, C, d, ds, buf, lane, (int64_t)blockIdx.x * kNodeWarps + warp,
                      (int64_t)gridDim.x * kNodeWarps, [&](int64_t node, float *row) {
        const float *zr = a.z + node * (int64_t)C * nr;
        {
            constexpr int kB = 8;            // all of a batch's loads in flight before the stores
            for (int i0 = lane; i0 < C * nr; i0 += 32 * kB) {
                float z[kB];
#pragma unroll
                for (int u = 0; u < kB; u++)
                    if (i0 + 32 * u < C * nr) z[u] = __ldg(zr + i0 + 32 * u);
#pragma unroll
                for (int u = 0; u < kB; u++)
                    if (i0 + 32 * u < C * nr) gs[i0 + 32 * u] = 1.0f / (1.0f + expf(-z[u]));
            }
        }
        __syncwarp();
        for (int c = lane; c < C; c += 32)
#pragma unroll 4
            for (int p = 0; p < d; p++) row[c * ds + p] *= gs[c * nr + pirr_s[p]];
        write_row_ds(a.out + node * n, row, C, d, ds, lane);
    });
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

// Walk (a, b) = (i / period, i % period) for i = start, start + step, ... without a division
// per step.
struct StepWalk {
    int a, b, da, db, period;
    __device__ __forceinline__ StepWalk(int start, int period_, int step) : period(period_) {
        a = start / period_;
        b = start - a * period_;
        da = step / period_;
        db = step - da * period_;
    }
    __device__ __forceinline__ void next() {
        a += da;
        b += db;
        if (b >= period) {
            b -= period;
            a++;
        }
    }
};

// Rows of d floats (global, contiguous) <-> shared memory rows at the odd stride dsp > d, so
// that reading one position of consecutive rows does not fall on one bank (at d = 16 a
// stride of d put all 32 lanes on two banks).  Float4 on the global side when d % 4 == 0.
__device__ __forceinline__ void pm_load_tile_padded(float *tsm, const float *src, int rows, int d, int dsp) {
    if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        StepWalk w(threadIdx.x, d / 4, blockDim.x);
        for (int i = threadIdx.x; i < rows * d / 4; i += blockDim.x, w.next()) {
            const float4 v = __ldg(s4 + i);
            float *t = tsm + w.a * dsp + 4 * w.b;
            t[0] = v.x;
            t[1] = v.y;
            t[2] = v.z;
            t[3] = v.w;
        }
    } else {
        StepWalk w(threadIdx.x, d, blockDim.x);
        for (int i = threadIdx.x; i < rows * d; i += blockDim.x, w.next()) tsm[w.a * dsp + w.b] = __ldg(src + i);
    }
}

__device__ __forceinline__ void pm_store_tile_padded(float *dst, const float *tsm, int rows, int d, int dsp) {
    if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        StepWalk w(threadIdx.x, d / 4, blockDim.x);
        for (int i = threadIdx.x; i < rows * d / 4; i += blockDim.x, w.next()) {
            const float *t = tsm + w.a * dsp + 4 * w.b;
            d4[i] = make_float4(t[0], t[1], t[2], t[3]);
        }
    } else {
        StepWalk w(threadIdx.x, d, blockDim.x);
        for (int i = threadIdx.x; i < rows * d; i += blockDim.x, w.next()) dst[i] = tsm[w.a * dsp + w.b];
    }
}

__global__ void __launch_bounds__(256) to_posmajor_kernel(const float *__restrict__ x, int64_t N, int C, int d,
                                                          int tn, float *__restrict__ xt) {
    extern __shared__ float tsm[];
    const int64_t n0 = (int64_t)blockIdx.x * tn;
    const int nn = (int)min64(tn, N - n0);
    const int dsp = odd_stride(d);           // shared-memory row stride (== d for odd d)
    if (dsp == d)
        pm_load_tile(tsm, x + n0 * C * d, nn * C * d);
    else
        pm_load_tile_padded(tsm, x + n0 * C * d, nn * C, d, dsp);
    __syncthreads();
    const int slab = nn * C;                 // (nodes x channels) of one position, a multiple of 4
    for (int p = 0; p < d; p++) {
        float4 *dst = reinterpret_cast<float4 *>(xt + (int64_t)p * N * C + n0 * C);
        for (int r = 4 * threadIdx.x; r < slab; r += 4 * blockDim.x)     // r = node * C + c
            dst[r / 4] = make_float4(tsm[r * dsp + p], tsm[(r + 1) * dsp + p], tsm[(r + 2) * dsp + p],
                                     tsm[(r + 3) * dsp + p]);
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
    const int dsp = odd_stride(d);
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
            tsm[r * dsp + p] = v.x;
            tsm[(r + 1) * dsp + p] = v.y;
            tsm[(r + 2) * dsp + p] = v.z;
            tsm[(r + 3) * dsp + p] = v.w;
        }
    }
    __syncthreads();
    const int tile = slab * d;
    float *dst = y + n0 * C * d;
    if (dsp != d) {
        pm_store_tile_padded(dst, tsm, slab, d, dsp);
    } else if ((tile & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
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

// the cp.async row pipeline applies: odd d (no row padding), whole float4 rows, aligned input
bool node_async(const float *x, int C, int d) {
    return (d & 1) && ((int64_t)C * d) % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

// row buffers per warp: two on the cp.async pipeline (the next row lands while the current
// one is transformed), one when rows are staged through registers
int node_slots(bool async) { return async ? 2 : 1; }

// One wave of blocks: as many as are resident on the device at once for this kernel and
// shared memory (occupancy, cached per kernel and size), each warp then walking its nodes
// with the next row in flight.  More blocks than that only add waves, each reloading the
// block's weights; at a few thousand nodes (config 3) the tail of a second wave was most of
// the launch.
int node_grid(const void *fn, size_t smem, int64_t N) {
    const int64_t want = (N + kNodeWarps - 1) / kNodeWarps;
    struct Entry {
        const void *fn;
        size_t smem;
        int dev, blocks;
    };
    static Entry cache[16];
    static int used = 0;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    {
        std::lock_guard<std::mutex> g(mu);
        for (int i = 0; i < used; i++)
            if (cache[i].fn == fn && cache[i].smem == smem && cache[i].dev == dev) return (int)min64(want, cache[i].blocks);
    }
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kNodeWarps * 32, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int blocks = sms * per_sm;
    {
        std::lock_guard<std::mutex> g(mu);
        if (used < 16) cache[used++] = Entry{fn, smem, dev, blocks};
    }
    return (int)min64(want, blocks);
}

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
    const bool async = node_async(x, C, a.R.d);
    const size_t smem = sizeof(float) * ((size_t)kNodeWarps * node_slots(async) * C * odd_stride(a.R.d) +
                                         (size_t)C * (2 * a.nscalar + 1));
    const auto k = async ? sep_layernorm_kernel<true> : sep_layernorm_kernel<false>;
    if ((rc = set_smem((const void *)k, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_norm", (cudaStream_t)stream);
    k<<<node_grid((const void *)k, smem, num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
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
    const bool async = node_async(x, C, a.R.d);
    const size_t smem = sizeof(float) * kNodeWarps *
                        ((size_t)node_slots(async) * C * odd_stride(a.R.d) + (size_t)C * odd_stride(n_lvals));
    const auto k = async ? equi_layernorm_kernel<true> : equi_layernorm_kernel<false>;
    if ((rc = set_smem((const void *)k, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_norm", (cudaStream_t)stream);
    k<<<node_grid((const void *)k, smem, num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
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
    const bool async = node_async(x, C, a.R.d);
    const size_t smem = sizeof(float) * kNodeWarps * (size_t)node_slots(async) * C * odd_stride(a.R.d);
    const auto k = async ? rep_norm_kernel<true> : rep_norm_kernel<false>;
    if ((rc = set_smem((const void *)k, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_norm", (cudaStream_t)stream);
    k<<<node_grid((const void *)k, smem, num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_node_to_posmajor(const float *x, int64_t num_nodes, int32_t C, int32_t d, float *xt, feq_stream_t stream) {
    if (num_nodes < 0 || C < 1 || d < 1 || d > kMaxDim) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !xt) return FEQ_ERR_INVALID_ARGUMENT;
    if (C % 4 || (reinterpret_cast<uintptr_t>(xt) & 15)) return FEQ_ERR_UNSUPPORTED;
    const int tn = pm_nodes(C, odd_stride(d));
    if (tn < 1) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = sizeof(float) * tn * (size_t)C * odd_stride(d);
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
    const int tn = pm_nodes(C, odd_stride(R.d));
    if (tn < 1) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = sizeof(float) * tn * (size_t)C * odd_stride(R.d);
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
    const bool async = node_async(x, C, a.R.d);
    const size_t smem =
        sizeof(float) * kNodeWarps * ((size_t)node_slots(async) * C * odd_stride(a.R.d) + (size_t)C * n_lvals);
    const auto k = async ? gate_kernel<true> : gate_kernel<false>;
    if ((rc = set_smem((const void *)k, smem)) != FEQ_OK) return rc;
    ProfScope ps("node_gate", (cudaStream_t)stream);
    k<<<node_grid((const void *)k, smem, num_nodes), kNodeWarps * 32, smem, (cudaStream_t)stream>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // extern "C"
