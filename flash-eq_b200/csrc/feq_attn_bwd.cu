// feq_attn_bwd.cu -- backward of the attention and pooling operators.
//
// Forward behaviour being differentiated (the reference obtains these gradients
// from PyTorch autograd through its scatter / gather ops):
//   logits (Q*K).sum(-1) * exp(log_scale) - d / decay   flash_eq/layers/attention.py:92-99
//   _neighbor_softmax (amax, exp, scatter_add, divide)   flash_eq/layers/attention.py:108-141
//   _apply_attention (per-head weighting of V)          flash_eq/layers/attention.py:143-167
//   GraphPooling sum / mean / max                       flash_eq/layers/pooling.py:21-57
//
// Softmax: with u = exp(l - max), w = u / (S + 1e-8), S = sum_seg u, the gradient is
//   dl = w * (dw - sum_seg w dw).
// The segment max is treated as a constant.  Its exact derivative (the one autograd
// takes through scatter_reduce amax) adds -1e-8 / (S + 1e-8) * sum_seg w dw to the
// arg-max logit; S >= 1, so that term is below 1e-8 of the others.
// Max pooling follows torch's scatter_reduce amax backward: the gradient of an
// output element is split evenly between the edges whose value equals it, and an
// empty node (output -inf, replaced by 0) passes no gradient.
//
// Every reduction runs over a dst- or src-sorted segment in a fixed order, with
// no atomics: results are bitwise reproducible run to run.
#include <cuda_runtime.h>
#include <math.h>

#include "feq_internal.cuh"

namespace feq {
namespace {

constexpr int kThreads = 128;
constexpr int kChunk = 32;
constexpr int kMaxHeads = 64;

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// Fused attention pooling (EquivariantAttention), one CTA per destination node.
//
// Pass 1 over the node's in-edges (chunks of kChunk): logits l (recomputed from Q
// and K exactly as the forward does), dw = <g_n, V_e> per head, and the online
// max / sum / sum(u dw).  Pass 2: w, dl = w (dw - <w, dw>), dV_e = w g_n,
// dQ_n = scale sum_e dl K_e, the decay term of dd, and this node's share of
// dL/dlog_scale = sum dl * scale <q, k>.  dl is left in edge_scratch for the
// src-segment kernel that forms dK.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) attn_pool_bwd_dst_kernel(const __grid_constant__ FeqAttnBwdArgs b) {
    const FeqAttnArgs &a = b.fwd;
    extern __shared__ float smem[];
    const int64_t n = blockIdx.x;
    const int64_t E = a.num_edges;
    const int H = a.num_heads;
    const int qrow = a.c_qk * a.d_qk, vrow = a.c_v * a.d_v;
    const int hd = qrow / H, vhd = vrow / H;
    float *q_s = smem;            // Q row of this node
    float *g_s = q_s + qrow;      // upstream gradient of this node's output (divided by the count for mean)
    float *gq_s = g_s + vrow;     // dQ accumulator
    __shared__ float x_s[kChunk][kMaxHeads], y_s[kChunk][kMaxHeads];
    __shared__ float m_s[kMaxHeads], inv_s[kMaxHeads], dot_s[kMaxHeads];
    __shared__ int64_t eid_s[kChunk], sid_s[kChunk];
    __shared__ float red_s[kThreads / 32];

    const bool split_k = a.k != nullptr;
    const int64_t nsrc = split_k ? a.num_src_nodes : a.num_nodes;
    const int64_t qk_ld = split_k ? qrow : 2 * (int64_t)qrow;
    const float *kbase = split_k ? a.k : a.qk + qrow;
    const bool decay = a.decay_scale > 0.0f && a.distances != nullptr;
    const int64_t s0 = a.offsets[n], s1 = a.offsets[n + 1];
    const float cnt = (float)max64(s1 - s0, 1);
    // per-thread dot products need float4-aligned rows and head slices
    const bool per_thread = hd <= 128 && vhd <= 128 && ((hd | vhd | qrow | vrow) & 3) == 0 &&
                            ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(a.v)) & 15) == 0;
    for (int j = threadIdx.x; j < qrow; j += kThreads) {
        q_s[j] = __ldg(a.qk + n * qk_ld + j);
        gq_s[j] = 0.0f;
    }
    for (int j = threadIdx.x; j < vrow; j += kThreads) {
        const float g = __ldg(b.grad_out + n * (int64_t)vrow + j);
        g_s[j] = a.reduce == FEQ_REDUCE_MEAN ? g / cnt : g;
    }
    if (threadIdx.x < H) {
        m_s[threadIdx.x] = -INFINITY;
        inv_s[threadIdx.x] = 0.0f;
        dot_s[threadIdx.x] = 0.0f;
    }
    float *lg_e = b.edge_scratch;             // (E, H) logits
    float *gl_e = b.edge_scratch + E * H;     // (E, H) dL/dw, then dL/dl
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = kThreads / 32;

    // ---- pass 1 ----
    for (int64_t c0 = s0; c0 < s1; c0 += kChunk) {
        const int cn = (int)min64(kChunk, s1 - c0);
        __syncthreads();
        if (threadIdx.x < cn) {
            const int64_t e = a.perm[c0 + threadIdx.x];
            int64_t sidx = a.src[e];
            if (sidx < 0 || sidx >= nsrc) {
                set_status(a.status, 1);
                sidx = -1;
            }
            eid_s[threadIdx.x] = e;
            sid_s[threadIdx.x] = sidx;
        }
        __syncthreads();
        if (per_thread) {
            // short heads: one thread per (edge, head) pair, float4 rows of K and V
            for (int pr = threadIdx.x; pr < cn * H; pr += kThreads) {
                const int k = pr / H, h = pr - k * H;
                const int64_t e = eid_s[k], sidx = sid_s[k];
                float acc = 0.0f, accg = 0.0f;
                if (sidx >= 0) {
                    const float4 *kr = reinterpret_cast<const float4 *>(kbase + sidx * qk_ld + h * hd);
                    const float4 *qr = reinterpret_cast<const float4 *>(q_s + h * hd);
#pragma unroll 6
                    for (int i = 0; i < hd / 4; i++) {
                        const float4 kv = __ldg(kr + i), qv = qr[i];
                        acc = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, acc))));
                    }
                }
                const float4 *vr = reinterpret_cast<const float4 *>(a.v + e * (int64_t)vrow + h * vhd);
                const float4 *gr = reinterpret_cast<const float4 *>(g_s + h * vhd);
#pragma unroll 6
                for (int i = 0; i < vhd / 4; i++) {
                    const float4 vv = __ldg(vr + i), gv = gr[i];
                    accg = fmaf(gv.x, vv.x, fmaf(gv.y, vv.y, fmaf(gv.z, vv.z, fmaf(gv.w, vv.w, accg))));
                }
                float v = acc * a.scale;
                if (decay) v -= a.distances[e] / a.decay_scale;
                x_s[k][h] = v;
                y_s[k][h] = accg;
                lg_e[e * H + h] = v;
                gl_e[e * H + h] = accg;
            }
        } else {
            for (int pr = warp; pr < cn * H; pr += nwarps) {
                const int k = pr / H, h = pr - k * H;
                const int64_t e = eid_s[k], sidx = sid_s[k];
                float acc = 0.0f, accg = 0.0f;
                if (sidx >= 0) {
                    const float *kr = kbase + sidx * qk_ld + h * hd;
                    const float *qr = q_s + h * hd;
                    for (int i = lane; i < hd; i += 32) acc = fmaf(qr[i], __ldg(kr + i), acc);
                }
                const float *vr = a.v + e * (int64_t)vrow + h * vhd;
                const float *gr = g_s + h * vhd;
                for (int i = lane; i < vhd; i += 32) accg = fmaf(gr[i], __ldg(vr + i), accg);
                acc = wsum(acc);
                accg = wsum(accg);
                if (lane == 0) {
                    float v = acc * a.scale;
                    if (decay) v -= a.distances[e] / a.decay_scale;
                    x_s[k][h] = v;
                    y_s[k][h] = accg;
                    lg_e[e * H + h] = v;
                    gl_e[e * H + h] = accg;
                }
            }
        }
        __syncthreads();
        if (threadIdx.x < H) {
            const int h = threadIdx.x;
            float mc = -INFINITY;
            for (int k = 0; k < cn; k++) mc = fmaxf(mc, x_s[k][h]);
            const float mold = m_s[h], mnew = fmaxf(mold, mc);
            const float corr = (mold == -INFINITY) ? 0.0f : expf(mold - mnew);
            float sm = inv_s[h] * corr, dt = dot_s[h] * corr;
            for (int k = 0; k < cn; k++) {
                const float p = expf(x_s[k][h] - mnew);
                sm += p;
                dt = fmaf(p, y_s[k][h], dt);
            }
            inv_s[h] = sm;
            dot_s[h] = dt;
            m_s[h] = mnew;
        }
    }
    __syncthreads();
    if (threadIdx.x < H) {
        const float inv = 1.0f / (inv_s[threadIdx.x] + 1e-8f);
        inv_s[threadIdx.x] = inv;
        dot_s[threadIdx.x] *= inv;      // <w, dw>
    }

    // ---- pass 2 ----
    float ls_acc = 0.0f;
    for (int64_t c0 = s0; c0 < s1; c0 += kChunk) {
        const int cn = (int)min64(kChunk, s1 - c0);
        __syncthreads();
        if (threadIdx.x < cn) {
            const int64_t e = a.perm[c0 + threadIdx.x];
            int64_t sidx = a.src[e];
            if (sidx < 0 || sidx >= nsrc) sidx = -1;
            eid_s[threadIdx.x] = e;
            sid_s[threadIdx.x] = sidx;
        }
        __syncthreads();
        for (int pr = threadIdx.x; pr < cn * H; pr += kThreads) {
            const int k = pr / H, h = pr - k * H;
            const int64_t e = eid_s[k];
            const float l = lg_e[e * H + h], gw = gl_e[e * H + h];
            const float w = expf(l - m_s[h]) * inv_s[h];
            const float gl = w * (gw - dot_s[h]);
            x_s[k][h] = w;
            y_s[k][h] = gl;
            gl_e[e * H + h] = gl;
            const float sqk = decay ? l + a.distances[e] / a.decay_scale : l;   // scale * <q, k>
            ls_acc = fmaf(gl, sqk, ls_acc);
        }
        __syncthreads();
        if (b.grad_distances && decay && threadIdx.x < cn) {
            float s = 0.0f;
            for (int h = 0; h < H; h++) s += y_s[threadIdx.x][h];
            b.grad_distances[eid_s[threadIdx.x]] = -s / a.decay_scale;
        }
        if (b.grad_v) {
            for (int k = 0; k < cn; k++) {
                float *gv = b.grad_v + eid_s[k] * (int64_t)vrow;
                for (int j = threadIdx.x; j < vrow; j += kThreads) gv[j] = x_s[k][j / vhd] * g_s[j];
            }
        }
        for (int j = threadIdx.x; j < qrow; j += kThreads) {
            const int h = j / hd;
            float acc = gq_s[j];
            for (int k0 = 0; k0 < cn; k0 += 8) {      // 8 K loads in flight per batch
                float kv[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int64_t sidx = k0 + u < cn ? sid_s[k0 + u] : -1;
                    kv[u] = sidx >= 0 ? __ldg(kbase + sidx * qk_ld + j) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if (k0 + u < cn) acc = fmaf(y_s[k0 + u][h] * a.scale, kv[u], acc);
            }
            gq_s[j] = acc;
        }
    }
    __syncthreads();
    if (b.grad_q)
        for (int j = threadIdx.x; j < qrow; j += kThreads) b.grad_q[n * b.ldq + j] = gq_s[j];
    ls_acc = wsum(ls_acc);
    if (lane == 0) red_s[warp] = ls_acc;
    __syncthreads();
    if (threadIdx.x == 0 && b.grad_scale_partial) {
        float s = 0.0f;
        for (int w = 0; w < nwarps; w++) s += red_s[w];
        b.grad_scale_partial[n] = s;
    }
}

// dK of every source row: dK_m = scale sum_{e : src[e] = m} dl_e Q[dst_e], over the
// src-sorted segment of m, one CTA per source row.
__global__ void __launch_bounds__(kThreads) attn_pool_bwd_src_kernel(const __grid_constant__ FeqAttnBwdArgs b) {
    const FeqAttnArgs &a = b.fwd;
    extern __shared__ float gk_s[];
    const int64_t m = blockIdx.x;
    const int64_t E = a.num_edges;
    const int H = a.num_heads;
    const int qrow = a.c_qk * a.d_qk, hd = qrow / H;
    const bool split_k = a.k != nullptr;
    const int64_t qk_ld = split_k ? qrow : 2 * (int64_t)qrow;
    __shared__ float gl_s[kChunk][kMaxHeads];
    __shared__ int64_t did_s[kChunk];
    const float *gl_e = b.edge_scratch + E * H;
    for (int j = threadIdx.x; j < qrow; j += kThreads) gk_s[j] = 0.0f;
    const int64_t s0 = b.src_offsets[m], s1 = b.src_offsets[m + 1];
    for (int64_t c0 = s0; c0 < s1; c0 += kChunk) {
        const int cn = (int)min64(kChunk, s1 - c0);
        __syncthreads();
        if (threadIdx.x < cn) {
            const int64_t e = b.src_perm[c0 + threadIdx.x];
            int64_t dd = b.dst[e];
            if (dd < 0 || dd >= a.num_nodes) {
                set_status(a.status, 1);
                dd = -1;
            }
            did_s[threadIdx.x] = dd;
        }
        for (int pr = threadIdx.x; pr < cn * H; pr += kThreads) {
            const int k = pr / H, h = pr - k * H;
            gl_s[k][h] = gl_e[b.src_perm[c0 + k] * H + h] * a.scale;
        }
        __syncthreads();
        for (int j = threadIdx.x; j < qrow; j += kThreads) {
            const int h = j / hd;
            float acc = gk_s[j];
            for (int k0 = 0; k0 < cn; k0 += 8) {      // 8 Q loads in flight per batch
                float qv[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int64_t dd = k0 + u < cn ? did_s[k0 + u] : -1;
                    qv[u] = dd >= 0 ? __ldg(a.qk + dd * qk_ld + j) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if (k0 + u < cn) acc = fmaf(gl_s[k0 + u][h], qv[u], acc);
            }
            gk_s[j] = acc;
        }
    }
    for (int j = threadIdx.x; j < qrow; j += kThreads) b.grad_k[m * b.ldk + j] = gk_s[j];
}

// ---------------------------------------------------------------------------
// Materialised attention weights (EquivariantEdgeAttention, attention dropout,
// max pooling).
// ---------------------------------------------------------------------------
// dl = w (dw - sum_seg w dw), one warp per destination node, heads looped.
// In place (grad_logits == grad_weights) is fine.
__global__ void segment_softmax_bwd_kernel(const float *w, const float *gw, int64_t N, int H,
                                           const int64_t *__restrict__ perm, const int64_t *__restrict__ offsets,
                                           float *gl) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t n = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
        const int64_t s0 = offsets[n], s1 = offsets[n + 1];
        for (int h = 0; h < H; h++) {
            float dot = 0.0f;
            for (int64_t p = s0 + lane; p < s1; p += 32) {
                const int64_t e = perm[p];
                dot = fmaf(w[e * H + h], gw[e * H + h], dot);
            }
            dot = wsum(dot);
            for (int64_t p = s0 + lane; p < s1; p += 32) {
                const int64_t e = perm[p];
                const float ww = w[e * H + h];
                gl[e * H + h] = ww * (gw[e * H + h] - dot);
            }
        }
    }
}

// Backward of logits[e,h] = scale <Q[e,h], K[e,h]> - d[e] / decay, one warp per edge:
// dQ = scale dl K, dK = scale dl Q, dd = -sum_h dl / decay, and the per-edge share of
// dL/dlog_scale = sum_h dl * scale <Q, K>.
__global__ void edge_logits_bwd_kernel(const float *__restrict__ Q, const float *__restrict__ K, int64_t E, int H,
                                       int D, float scale, float decay, const float *__restrict__ gl,
                                       float *__restrict__ gQ, float *__restrict__ gK, float *__restrict__ gd,
                                       float *__restrict__ gpart) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t e = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); e < E; e += warps) {
        float sum_gl = 0.0f, part = 0.0f;
        for (int h = 0; h < H; h++) {
            const int64_t r = (e * H + h) * (int64_t)D;
            const float g = gl[e * H + h];
            const float gs = g * scale;
            float dot = 0.0f;
            for (int i = lane; i < D; i += 32) {
                const float qv = __ldg(Q + r + i), kv = __ldg(K + r + i);
                dot = fmaf(qv, kv, dot);
                if (gQ) gQ[r + i] = gs * kv;
                if (gK) gK[r + i] = gs * qv;
            }
            dot = wsum(dot);
            sum_gl += g;
            part = fmaf(g, dot * scale, part);
        }
        if (lane == 0) {
            if (gd) gd[e] = decay > 0.0f ? -sum_gl / decay : 0.0f;
            if (gpart) gpart[e] = part;
        }
    }
}

// ---------------------------------------------------------------------------
// Pooling backward.
// ---------------------------------------------------------------------------
// Max only: gs[n, j] = g[n, j] / (number of edges of n whose value equals out[n, j]).
__global__ void segment_pool_max_ties_kernel(const float *__restrict__ rows, int64_t L, const float *__restrict__ w,
                                             int H, const int64_t *__restrict__ perm,
                                             const int64_t *__restrict__ offsets, const float *__restrict__ out,
                                             const float *__restrict__ gout, float *__restrict__ gs) {
    const int64_t n = blockIdx.x;
    const int64_t s0 = offsets[n], s1 = offsets[n + 1];
    const int64_t hd = H > 0 ? L / H : L;
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
        const int h = (w && H > 0) ? (int)(j / hd) : 0;
        const float o = out[n * L + j];
        int c = 0;
        for (int64_t p = s0; p < s1; p++) {
            const int64_t e = perm[p];
            float v = __ldg(rows + e * L + j);
            if (w) v *= __ldg(w + e * H + h);
            c += (v == o);
        }
        gs[n * L + j] = c > 0 ? gout[n * L + j] / (float)c : 0.0f;
    }
}

// One warp per (edge, head group): d rows = (w *) g[dst], d w[e,h] = sum_j g[dst, j] rows[e, j]
// over the head's elements; g is the upstream gradient (/ count for mean; the tie-split
// gradient, masked to the edges equal to the output, for max).
__global__ void segment_pool_bwd_edges_kernel(const float *__restrict__ rows, int64_t L, const float *__restrict__ w,
                                              int H, const int64_t *__restrict__ dst, const int64_t *__restrict__ offsets,
                                              int64_t N, int64_t E, int reduce, const float *__restrict__ out,
                                              const float *__restrict__ gsrc, float *__restrict__ grows,
                                              float *__restrict__ gw, int32_t *status) {
    const int lane = threadIdx.x & 31;
    const int groups = w ? H : 1;
    const int64_t glen = L / groups;
    const int64_t items = E * groups;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
        const int64_t e = it / groups;
        const int h = (int)(it - e * groups);
        const int64_t n = dst[e];
        const bool ok = n >= 0 && n < N;
        if (!ok && lane == 0) set_status(status, 1);
        const float ww = w ? __ldg(w + e * H + h) : 1.0f;
        const float cnt = ok ? (float)max64(offsets[n + 1] - offsets[n], 1) : 1.0f;
        float acc = 0.0f;
        for (int64_t i = lane; i < glen; i += 32) {
            const int64_t j = h * glen + i;
            const float x = __ldg(rows + e * L + j);
            float g = 0.0f;
            if (ok) {
                g = __ldg(gsrc + n * L + j);
                if (reduce == FEQ_REDUCE_MEAN) {
                    g = g / cnt;
                } else if (reduce == FEQ_REDUCE_MAX) {
                    const float v = w ? x * ww : x;
                    if (!(v == __ldg(out + n * L + j))) g = 0.0f;
                }
            }
            grows[e * L + j] = w ? g * ww : g;
            acc = fmaf(g, x, acc);
        }
        if (w && gw) {
            acc = wsum(acc);
            if (lane == 0) gw[e * H + h] = acc;
        }
    }
}

int check_attn_bwd(const FeqAttnBwdArgs *b) {
    if (!b) return FEQ_ERR_INVALID_ARGUMENT;
    const FeqAttnArgs &a = b->fwd;
    if (a.num_nodes < 0 || a.num_edges < 0 || a.num_heads < 1 || a.c_qk < 1 || a.d_qk < 1 || a.c_v < 1 ||
        a.d_v < 1)
        return FEQ_ERR_INVALID_ARGUMENT;
    if (a.c_qk % a.num_heads || a.c_v % a.num_heads) return FEQ_ERR_INVALID_ARGUMENT;
    if (a.num_heads > kMaxHeads) return FEQ_ERR_UNSUPPORTED;
    if (a.reduce != FEQ_REDUCE_SUM && a.reduce != FEQ_REDUCE_MEAN) return FEQ_ERR_UNSUPPORTED;
    if (a.k && a.num_src_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (a.decay_scale > 0.0f && !a.distances) return FEQ_ERR_INVALID_ARGUMENT;
    const int64_t nsrc = a.k ? a.num_src_nodes : a.num_nodes;
    const int64_t qrow = (int64_t)a.c_qk * a.d_qk;
    if (a.num_nodes > 0x7fffffffll || nsrc > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    if (a.num_nodes > 0 && (!a.qk || !a.offsets || !b->grad_out)) return FEQ_ERR_INVALID_ARGUMENT;
    if (a.num_edges > 0 && (!a.v || !a.src || !a.perm || !b->dst || !b->src_perm || !b->src_offsets ||
                            !b->edge_scratch))
        return FEQ_ERR_INVALID_ARGUMENT;
    if ((b->grad_q && b->ldq < qrow) || (b->grad_k && b->ldk < qrow)) return FEQ_ERR_INVALID_ARGUMENT;
    if (b->grad_k && nsrc > 0 && !b->src_offsets) return FEQ_ERR_INVALID_ARGUMENT;
    return FEQ_OK;
}

}  // namespace
}  // namespace feq

using namespace feq;

extern "C" {

int feq_attn_pool_bwd(const FeqAttnBwdArgs *b, feq_stream_t stream) {
    int rc = check_attn_bwd(b);
    if (rc != FEQ_OK) return rc;
    const FeqAttnArgs &a = b->fwd;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t nsrc = a.k ? a.num_src_nodes : a.num_nodes;
    const size_t qrow = (size_t)a.c_qk * a.d_qk, vrow = (size_t)a.c_v * a.d_v;
    if (a.num_nodes > 0) {
        const size_t smem = sizeof(float) * (2 * qrow + vrow);
        if (smem > 160 * 1024) return FEQ_ERR_UNSUPPORTED;
        ProfScope ps("attn_bwd_dst", s);
        FEQ_CUDA_TRY(cudaFuncSetAttribute(attn_pool_bwd_dst_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        attn_pool_bwd_dst_kernel<<<(unsigned)a.num_nodes, kThreads, smem, s>>>(*b);
        FEQ_LAUNCH_CHECK();
    }
    if (b->grad_k && nsrc > 0) {
        const size_t smem = sizeof(float) * qrow;
        if (smem > 160 * 1024) return FEQ_ERR_UNSUPPORTED;
        ProfScope ps("attn_bwd_src", s);
        FEQ_CUDA_TRY(cudaFuncSetAttribute(attn_pool_bwd_src_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
        attn_pool_bwd_src_kernel<<<(unsigned)nsrc, kThreads, smem, s>>>(*b);
        FEQ_LAUNCH_CHECK();
    }
    return FEQ_OK;
}

int feq_segment_softmax_bwd(const float *weights, const float *grad_weights, int64_t num_edges, int32_t num_heads,
                            const int64_t *perm, const int64_t *offsets, int64_t num_nodes, float *grad_logits,
                            feq_stream_t stream) {
    if (num_edges < 0 || num_nodes < 0 || num_heads < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0 || num_nodes == 0) return FEQ_OK;
    if (!weights || !grad_weights || !perm || !offsets || !grad_logits) return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t grid = min64((num_nodes + 7) / 8, 148 * 64);
    segment_softmax_bwd_kernel<<<(unsigned)grid, 256, 0, s>>>(weights, grad_weights, num_nodes, num_heads, perm,
                                                               offsets, grad_logits);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_edge_attention_weights_bwd(const float *Q, const float *K, int64_t num_edges, int32_t num_heads,
                                   int32_t qk_dim, float scale, float decay_scale, const int64_t *perm,
                                   const int64_t *offsets, int64_t num_nodes, const float *weights,
                                   const float *grad_weights, float *grad_logits, float *grad_Q, float *grad_K,
                                   float *grad_distances, float *grad_scale_partial, feq_stream_t stream) {
    if (num_edges < 0 || num_nodes < 0 || num_heads < 1 || qk_dim < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0) return FEQ_OK;
    if (!Q || !K || !perm || !offsets || !weights || !grad_weights || !grad_logits) return FEQ_ERR_INVALID_ARGUMENT;
    int rc = feq_segment_softmax_bwd(weights, grad_weights, num_edges, num_heads, perm, offsets, num_nodes,
                                     grad_logits, stream);
    if (rc != FEQ_OK) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t grid = min64((num_edges + 7) / 8, 148 * 32);
    edge_logits_bwd_kernel<<<(unsigned)grid, 256, 0, s>>>(Q, K, num_edges, num_heads, qk_dim, scale, decay_scale,
                                                           grad_logits, grad_Q, grad_K, grad_distances,
                                                           grad_scale_partial);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int feq_segment_pool_bwd(const float *edge_rows, int64_t row_len, const float *weights, int32_t num_heads,
                         const int64_t *dst, const int64_t *perm, const int64_t *offsets, int64_t num_nodes,
                         int64_t num_edges, int32_t reduce, const float *out, const float *grad_out,
                         float *tie_scratch, float *grad_rows, float *grad_weights, int32_t *status,
                         feq_stream_t stream) {
    if (row_len < 0 || num_nodes < 0 || num_edges < 0 || reduce < FEQ_REDUCE_SUM || reduce > FEQ_REDUCE_MAX)
        return FEQ_ERR_INVALID_ARGUMENT;
    if (weights && (num_heads < 1 || row_len % num_heads)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0 || row_len == 0) return FEQ_OK;
    if (!edge_rows || !dst || !offsets || !grad_out || !grad_rows) return FEQ_ERR_INVALID_ARGUMENT;
    if (reduce == FEQ_REDUCE_MAX && (!perm || !out || !tie_scratch)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    const int H = weights ? num_heads : 0;
    const float *gsrc = grad_out;
    if (reduce == FEQ_REDUCE_MAX && num_nodes > 0) {
        const int threads = (int)min64(256, ((row_len + 31) / 32) * 32);
        segment_pool_max_ties_kernel<<<(unsigned)num_nodes, threads, 0, s>>>(edge_rows, row_len, weights, H, perm,
                                                                             offsets, out, grad_out, tie_scratch);
        FEQ_LAUNCH_CHECK();
        gsrc = tie_scratch;
    }
    const int64_t items = num_edges * (weights ? num_heads : 1);
    const int64_t grid = min64((items + 7) / 8, 148 * 32);
    segment_pool_bwd_edges_kernel<<<(unsigned)grid, 256, 0, s>>>(edge_rows, row_len, weights, H, dst, offsets,
                                                                  num_nodes, num_edges, reduce, out, gsrc, grad_rows,
                                                                  grad_weights, status);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // extern "C"
