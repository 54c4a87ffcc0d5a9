// feq_graph.cu -- edge bookkeeping and the dst-segment operators.
//
// Reference behaviour replaced:
//   compute_binning                    flash_eq/cuda/csrc/block_diagonal.cu:82-115
//   torch.argsort(distances)           flash_eq/cuda/block_diagonal.py:102-103
//   _neighbor_softmax (scatter amax / exp / scatter_add / divide)
//                                      flash_eq/layers/attention.py:108-141
//   logits (Q*K).sum(-1)*scale - d/decay
//                                      flash_eq/layers/attention.py:92-99
//   _apply_attention + GraphPooling    flash_eq/layers/attention.py:143-167,
//                                      flash_eq/layers/pooling.py:21-57
//
// Everything that reduces over a destination works on dst-sorted segments
// (perm/offsets from a stable radix sort), one CTA or warp per segment, in a
// fixed order: results are deterministic run to run, unlike scatter_add_.
#include <cub/device/device_radix_sort.cuh>
#include <cuda_runtime.h>
#include <math.h>

#include "feq_internal.cuh"
#include "feq_rot_common.cuh"
#include "feq_sm100.cuh"

namespace feq {

// ---------------------------------------------------------------------------
// Binning
// ---------------------------------------------------------------------------
__global__ void binning_kernel(const float *__restrict__ dist, int64_t E, Binning b,
                               int32_t *__restrict__ lo_out, float *__restrict__ t_out) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E;
         e += (int64_t)gridDim.x * blockDim.x) {
        int lo;
        float t;
        bin_of(dist[e], b, lo, t);
        if (lo_out) lo_out[e] = lo;
        if (t_out) t_out[e] = t;
    }
}

int launch_binning(const float *dist, int64_t E, Binning b, int32_t *lo, float *t, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const int64_t grid = min64((E + 255) / 256, 148 * 32);
    binning_kernel<<<(unsigned)grid, 256, 0, s>>>(dist, E, b, lo, t);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// ---------------------------------------------------------------------------
// Stable sort by key with segment offsets
// ---------------------------------------------------------------------------
template <typename K>
__global__ void prep_keys_kernel(const K *__restrict__ keys, int64_t E, int32_t nk,
                                 int32_t *__restrict__ kout, int64_t *__restrict__ ids,
                                 int32_t *status) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E;
         e += (int64_t)gridDim.x * blockDim.x) {
        K k = keys[e];
        if (k < 0 || k >= (K)nk) {
            set_status(status, 1);
            k = (K)(nk - 1);
        }
        kout[e] = (int32_t)k;
        ids[e] = e;
    }
}

// offsets[k] = first sorted position whose key is >= k; offsets[nk] = E.
__global__ void offsets_kernel(const int32_t *__restrict__ sk, int64_t E, int32_t nk,
                               int64_t *__restrict__ offsets) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= E;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t prev = i > 0 ? sk[i - 1] : -1;
        const int32_t cur = i < E ? sk[i] : nk;
        for (int32_t k = prev + 1; k <= cur; k++) offsets[k] = i;
    }
}

static int key_bits(int32_t nk) {
    int bits = 1;
    while (bits < 31 && (1ll << bits) < (long long)nk) bits++;
    return bits;
}

static size_t cub_sort_bytes(int64_t E, int32_t nk) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const int32_t *)nullptr, (int32_t *)nullptr,
                                    (const int64_t *)nullptr, (int64_t *)nullptr, E, 0, key_bits(nk),
                                    (cudaStream_t)0);
    return bytes;
}

size_t edge_sort_workspace(int64_t E, int32_t nk) {
    WsCarver w{nullptr, 0, 0};
    w.take(sizeof(int32_t) * max64(E, 1));   // keys in
    w.take(sizeof(int32_t) * max64(E, 1));   // keys out
    w.take(sizeof(int64_t) * max64(E, 1));   // ids in
    w.take(std::max<size_t>(cub_sort_bytes(E, nk), 16));
    return w.used + 256;
}

template <typename K>
int launch_edge_sort(const K *keys, int64_t E, int32_t nk, int64_t *perm, int64_t *offsets,
                     int32_t *status, void *ws, size_t ws_bytes, cudaStream_t s) {
    if (nk <= 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (E == 0) {
        FEQ_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int64_t) * (nk + 1), s));
        return FEQ_OK;
    }
    if (ws_bytes < edge_sort_workspace(E, nk) || ws == nullptr) return FEQ_ERR_WORKSPACE;
    WsCarver w{(char *)ws, 0, ws_bytes};
    int32_t *kin = (int32_t *)w.take(sizeof(int32_t) * E);
    int32_t *kout = (int32_t *)w.take(sizeof(int32_t) * E);
    int64_t *ids = (int64_t *)w.take(sizeof(int64_t) * E);
    size_t tmp_bytes = std::max<size_t>(cub_sort_bytes(E, nk), 16);
    void *tmp = w.take(tmp_bytes);
    const int64_t grid = min64((E + 255) / 256, 148 * 32);
    prep_keys_kernel<K><<<(unsigned)grid, 256, 0, s>>>(keys, E, nk, kin, ids, status);
    FEQ_LAUNCH_CHECK();
    FEQ_CUDA_TRY(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, kin, kout, ids, perm, E, 0,
                                                 key_bits(nk), s));
    count_launches(3);
    const int64_t grid2 = min64((E + 256) / 256, 148 * 32);
    offsets_kernel<<<(unsigned)grid2, 256, 0, s>>>(kout, E, nk, offsets);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

template int launch_edge_sort<int32_t>(const int32_t *, int64_t, int32_t, int64_t *, int64_t *,
                                       int32_t *, void *, size_t, cudaStream_t);
template int launch_edge_sort<int64_t>(const int64_t *, int64_t, int32_t, int64_t *, int64_t *,
                                       int32_t *, void *, size_t, cudaStream_t);

// ---------------------------------------------------------------------------
// Edge logits (edge-level Q, K) and segment softmax
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One warp per (edge, head): logits[e, h] = scale * <Q[e,h,:], K[e,h,:]> - dist/decay.
__global__ void edge_logits_kernel(const float *__restrict__ Q, const float *__restrict__ K, int64_t E,
                                   int H, int D, float scale, const float *__restrict__ dist,
                                   float decay, float *__restrict__ logits) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < E * H; w += warps) {
        const float *q = Q + w * D, *k = K + w * D;
        float acc = 0.0f;
        for (int i = lane; i < D; i += 32) acc = fmaf(__ldg(q + i), __ldg(k + i), acc);
        acc = warp_sum(acc);
        if (lane == 0) {
            float v = acc * scale;
            if (decay > 0.0f && dist) v -= dist[w / H] / decay;
            logits[w] = v;
        }
    }
}

// One warp per destination node; heads looped.  In place (logits == weights) is fine.
__global__ void segment_softmax_kernel(const float *logits, int64_t N, int H,
                                       const int64_t *__restrict__ perm,
                                       const int64_t *__restrict__ offsets, float *weights) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t n = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
        const int64_t s0 = offsets[n], s1 = offsets[n + 1];
        for (int h = 0; h < H; h++) {
            float mx = -INFINITY;
            for (int64_t p = s0 + lane; p < s1; p += 32) mx = fmaxf(mx, logits[perm[p] * H + h]);
            mx = warp_max(mx);
            float sm = 0.0f;
            for (int64_t p = s0 + lane; p < s1; p += 32) sm += expf(logits[perm[p] * H + h] - mx);
            sm = warp_sum(sm);
            const float inv = 1.0f / (sm + 1e-8f);
            for (int64_t p = s0 + lane; p < s1; p += 32) {
                const int64_t e = perm[p];
                weights[e * H + h] = expf(logits[e * H + h] - mx) * inv;
            }
        }
    }
}

int launch_edge_logits(const float *Q, const float *K, int64_t E, int H, int D, float scale,
                       const float *dist, float decay, float *logits, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const int64_t grid = min64((E * H + 7) / 8, 148 * 32);
    edge_logits_kernel<<<(unsigned)grid, 256, 0, s>>>(Q, K, E, H, D, scale, dist, decay, logits);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_segment_softmax(const float *logits, int64_t N, int H, const int64_t *perm,
                           const int64_t *offsets, float *weights, cudaStream_t s) {
    if (N == 0) return FEQ_OK;
    const int64_t grid = min64((N + 7) / 8, 148 * 64);
    segment_softmax_kernel<<<(unsigned)grid, 256, 0, s>>>(logits, N, H, perm, offsets, weights);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// ---------------------------------------------------------------------------
// Segmented pooling: one CTA per node, threads over row elements.
// ---------------------------------------------------------------------------
__global__ void segment_pool_kernel(const float *__restrict__ rows, int64_t L,
                                    const float *__restrict__ w, int H,
                                    const int64_t *__restrict__ perm,
                                    const int64_t *__restrict__ offsets, int reduce,
                                    float *__restrict__ out) {
    const int64_t n = blockIdx.x;
    const int64_t s0 = offsets[n], s1 = offsets[n + 1];
    const int64_t hd = H > 0 ? L / H : L;
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
        const int h = (w && H > 0) ? (int)(j / hd) : 0;
        float acc = reduce == FEQ_REDUCE_MAX ? -INFINITY : 0.0f;
        for (int64_t p = s0; p < s1; p++) {
            const int64_t e = perm[p];
            float v = __ldg(rows + e * L + j);
            if (w) v *= __ldg(w + e * H + h);
            acc = reduce == FEQ_REDUCE_MAX ? fmaxf(acc, v) : acc + v;
        }
        if (reduce == FEQ_REDUCE_MAX) {
            if (s1 == s0) acc = 0.0f;   // empty segment: -inf -> 0 (pooling.py:57)
        } else if (reduce == FEQ_REDUCE_MEAN) {
            acc = acc / (float)max64(s1 - s0, 1);
        }
        out[n * L + j] = acc;
    }
}

int launch_segment_pool(const float *rows, int64_t L, const float *w, int H, const int64_t *perm,
                        const int64_t *offsets, int64_t N, int reduce, float *out, cudaStream_t s) {
    if (N == 0 || L == 0) return FEQ_OK;
    if (N > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    const int threads = (int)min64(256, ((L + 31) / 32) * 32);
    segment_pool_kernel<<<(unsigned)N, threads, 0, s>>>(rows, L, w, H, perm, offsets, reduce, out);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// ---------------------------------------------------------------------------
// Fused attention + pooling (EquivariantAttention without the V projection).
// One CTA per destination node, online softmax over chunks of the segment.
// ---------------------------------------------------------------------------
constexpr int kAttnThreads = 128;
constexpr int kAttnChunk = 32;
constexpr int kAttnMaxHeads = 64;

__global__ void __launch_bounds__(kAttnThreads)
attn_pool_kernel(const __grid_constant__ FeqAttnArgs a) {
    extern __shared__ float smem[];
    const int64_t n = blockIdx.x;
    const int C = a.c_qk, d = a.d_qk, H = a.num_heads;
    const int qrow = C * d;                 // one of Q / K
    const int vrow = a.c_v * a.d_v;
    const int hd = qrow / H;                // Q/K floats per head
    const int vhd = vrow / H;               // V floats per head
    float *q_s = smem;                      // qrow
    float *acc_s = q_s + qrow;              // vrow
    __shared__ float lg_s[kAttnChunk][kAttnMaxHeads];
    __shared__ float corr_s[kAttnMaxHeads], m_s[kAttnMaxHeads], sum_s[kAttnMaxHeads];
    __shared__ int64_t eid_s[kAttnChunk], sid_s[kAttnChunk];

    const bool split_k = a.k != nullptr;   // Q rows in qk, K rows in k (partitioned graphs)
    const int64_t nsrc = split_k ? a.num_src_nodes : a.num_nodes;
    const float *kbase = split_k ? a.k : a.qk + qrow;
    const int64_t k_ld = split_k ? qrow : 2 * (int64_t)qrow;
    // float4 V rows: whole float4 per head slice, aligned rows and accumulators
    const bool v_vec = (vhd & 3) == 0 && (vrow & 3) == 0 && (qrow & 3) == 0 &&
                       (reinterpret_cast<uintptr_t>(a.v) & 15) == 0;
    // per-thread dot products need 16-byte aligned K rows and head segments
    const bool per_thread = hd <= 128 && (hd & 3) == 0 && (qrow & 3) == 0 &&
                            ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(a.qk)) & 15) == 0;
    const float *qn = a.qk + n * (int64_t)(split_k ? qrow : 2 * qrow);
    for (int j = threadIdx.x; j < qrow; j += kAttnThreads) q_s[j] = __ldg(qn + j);
    for (int j = threadIdx.x; j < vrow; j += kAttnThreads) acc_s[j] = 0.0f;
    if (threadIdx.x < H) {
        m_s[threadIdx.x] = -INFINITY;
        sum_s[threadIdx.x] = 0.0f;
    }
    const int64_t s0 = a.offsets[n], s1 = a.offsets[n + 1];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = kAttnThreads / 32;
    for (int64_t c0 = s0; c0 < s1; c0 += kAttnChunk) {
        const int cn = (int)min64(kAttnChunk, s1 - c0);
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
            // logits, short heads: one thread per (edge, head) pair, float4 loads of the K row
            for (int pr = threadIdx.x; pr < cn * H; pr += kAttnThreads) {
                const int k = pr / H, h = pr - k * H;
                const int64_t sidx = sid_s[k];
                float acc0 = 0.0f, acc1 = 0.0f;
                if (sidx >= 0) {
                    const float4 *kr = reinterpret_cast<const float4 *>(kbase + sidx * k_ld + h * hd);
                    const float4 *qr = reinterpret_cast<const float4 *>(q_s + h * hd);
#pragma unroll 6
                    for (int i = 0; i < hd / 4; i++) {
                        const float4 kv = __ldg(kr + i), qv = qr[i];
                        acc0 = fmaf(qv.x, kv.x, acc0);
                        acc1 = fmaf(qv.y, kv.y, acc1);
                        acc0 = fmaf(qv.z, kv.z, acc0);
                        acc1 = fmaf(qv.w, kv.w, acc1);
                    }
                }
                float v = (acc0 + acc1) * a.scale;
                if (a.decay_scale > 0.0f && a.distances) v -= a.distances[eid_s[k]] / a.decay_scale;
                lg_s[k][h] = v;
            }
        } else {
            // logits, long heads: one warp per (edge, head) pair
            for (int pr = warp; pr < cn * H; pr += nwarps) {
                const int k = pr / H, h = pr - k * H;
                const int64_t sidx = sid_s[k];
                float acc = 0.0f;
                if (sidx >= 0) {
                    const float *kr = kbase + sidx * k_ld + h * hd;
                    const float *qr = q_s + h * hd;
                    for (int i = lane; i < hd; i += 32) acc = fmaf(qr[i], __ldg(kr + i), acc);
                }
                acc = warp_sum(acc);
                if (lane == 0) {
                    float v = acc * a.scale;
                    if (a.decay_scale > 0.0f && a.distances) v -= a.distances[eid_s[k]] / a.decay_scale;
                    lg_s[k][h] = v;
                }
            }
        }
        __syncthreads();
        // online softmax update per head
        if (threadIdx.x < H) {
            const int h = threadIdx.x;
            float mc = -INFINITY;
            for (int k = 0; k < cn; k++) mc = fmaxf(mc, lg_s[k][h]);
            const float mold = m_s[h], mnew = fmaxf(mold, mc);
            const float corr = (mold == -INFINITY) ? 0.0f : expf(mold - mnew);
            float sm = sum_s[h] * corr;
            for (int k = 0; k < cn; k++) {
                const float p = expf(lg_s[k][h] - mnew);
                lg_s[k][h] = p;
                sm += p;
            }
            sum_s[h] = sm;
            m_s[h] = mnew;
            corr_s[h] = corr;
        }
        __syncthreads();
        // weighted V accumulation (float4 rows when a head's slice is a whole number of float4)
        if (v_vec) {
            const float4 *v4 = reinterpret_cast<const float4 *>(a.v);
            float4 *acc4 = reinterpret_cast<float4 *>(acc_s);
            const int vrow4 = vrow / 4;
            for (int j = threadIdx.x; j < vrow4; j += kAttnThreads) {
                const int h = (4 * j) / vhd;
                const float c = corr_s[h];
                float4 acc = acc4[j];
                acc.x *= c;
                acc.y *= c;
                acc.z *= c;
                acc.w *= c;
                // batches of 8 edges (the last one predicated): 8 row loads in flight together
                for (int k = 0; k < cn; k += 8) {
                    float4 v[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        v[u] = k + u < cn ? __ldg(v4 + eid_s[k + u] * (int64_t)vrow4 + j) : make_float4(0, 0, 0, 0);
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        const float p = k + u < cn ? lg_s[k + u][h] : 0.0f;
                        acc.x = fmaf(p, v[u].x, acc.x);
                        acc.y = fmaf(p, v[u].y, acc.y);
                        acc.z = fmaf(p, v[u].z, acc.z);
                        acc.w = fmaf(p, v[u].w, acc.w);
                    }
                }
                acc4[j] = acc;
            }
        } else {
            for (int j = threadIdx.x; j < vrow; j += kAttnThreads) {
                const int h = j / vhd;
                float acc = acc_s[j] * corr_s[h];
                int k = 0;
                for (; k + 8 <= cn; k += 8) {
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) v[u] = __ldg(a.v + eid_s[k + u] * (int64_t)vrow + j);
#pragma unroll
                    for (int u = 0; u < 8; u++) acc = fmaf(lg_s[k + u][h], v[u], acc);
                }
                for (; k < cn; k++) acc = fmaf(lg_s[k][h], __ldg(a.v + eid_s[k] * (int64_t)vrow + j), acc);
                acc_s[j] = acc;
            }
        }
    }
    __syncthreads();
    const float cnt = (float)max64(s1 - s0, 1);
    for (int j = threadIdx.x; j < vrow; j += kAttnThreads) {
        const int h = j / vhd;
        float v = acc_s[j] / (sum_s[h] + 1e-8f);
        if (a.reduce == FEQ_REDUCE_MEAN) v /= cnt;
        a.out[n * (int64_t)vrow + j] = v;
    }
}

// Warp-per-destination variant for rows that split evenly over the lanes: lane l owns the
// S contiguous floats [l S, (l + 1) S) of the Q, K and V rows; with 32 % H == 0 each head is a
// group of 32 / H lanes, so a head's logit is a shuffle reduction within the group and the
// online softmax (max, rescale, sum) runs per lane on values the group agrees on.  The next
// edge's K and V slices are loaded while the current edge is folded in; no block barriers.
// Same arithmetic as attn_pool_kernel: logit = scale <q, k> (- d / decay), running max m,
// p = exp(logit - m_new), acc = acc exp(m_old - m_new) + p v, out = acc / (sum + 1e-8).
template <int S>
__global__ void __launch_bounds__(128)
attn_pool_warp_kernel(const __grid_constant__ FeqAttnArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (n >= a.num_nodes) return;
    const int qrow = a.c_qk * a.d_qk;
    const int H = a.num_heads, gl = 32 / H;      // lanes per head
    const bool split_k = a.k != nullptr;
    const int64_t nsrc = split_k ? a.num_src_nodes : a.num_nodes;
    const float *kbase = split_k ? a.k : a.qk + qrow;
    const int64_t k_ld = split_k ? qrow : 2 * (int64_t)qrow;
    const float *qn = a.qk + n * (int64_t)(split_k ? qrow : 2 * qrow) + lane * S;
    float q[S], acc[S];
#pragma unroll
    for (int i = 0; i < S; i++) {
        q[i] = __ldg(qn + i);
        acc[i] = 0.0f;
    }
    float m = -INFINITY, ssum = 0.0f;
    const int64_t s0 = a.offsets[n], s1 = a.offsets[n + 1];
    float kn[S], vn[S];
    int64_t en = 0;
    auto fetch = [&](int64_t pos) {
        en = a.perm[pos];
        int64_t sidx = a.src[en];
        if (sidx < 0 || sidx >= nsrc) {
            if (lane == 0) set_status(a.status, 1);
            sidx = -1;
        }
        const float *kr = kbase + (sidx >= 0 ? sidx : 0) * k_ld + lane * S;
        const float *vr = a.v + en * (int64_t)(32 * S) + lane * S;
        if constexpr ((S & 1) == 0) {      // 8-byte aligned slices: float2 loads
#pragma unroll
            for (int i = 0; i < S; i += 2) {
                const float2 kk = __ldg(reinterpret_cast<const float2 *>(kr + i));
                const float2 vv = __ldg(reinterpret_cast<const float2 *>(vr + i));
                kn[i] = sidx >= 0 ? kk.x : 0.0f;
                kn[i + 1] = sidx >= 0 ? kk.y : 0.0f;
                vn[i] = vv.x;
                vn[i + 1] = vv.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < S; i++) {
                kn[i] = sidx >= 0 ? __ldg(kr + i) : 0.0f;
                vn[i] = __ldg(vr + i);
            }
        }
    };
    if (s0 < s1) fetch(s0);
    for (int64_t pos = s0; pos < s1; pos++) {
        float kc[S], vc[S];
#pragma unroll
        for (int i = 0; i < S; i++) {
            kc[i] = kn[i];
            vc[i] = vn[i];
        }
        const int64_t ec = en;
        if (pos + 1 < s1) fetch(pos + 1);
        float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
        for (int i = 0; i + 1 < S; i += 2) {
            d0 = fmaf(q[i], kc[i], d0);
            d1 = fmaf(q[i + 1], kc[i + 1], d1);
        }
        if (S & 1) d0 = fmaf(q[S - 1], kc[S - 1], d0);
        float dot = d0 + d1;
        for (int o = 1; o < gl; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        float lg = dot * a.scale;
        if (a.decay_scale > 0.0f && a.distances) lg -= a.distances[ec] / a.decay_scale;
        const float mnew = fmaxf(m, lg);
        const float corr = (m == -INFINITY) ? 0.0f : expf(m - mnew);
        const float p = expf(lg - mnew);
        ssum = ssum * corr + p;
#pragma unroll
        for (int i = 0; i < S; i++) acc[i] = fmaf(p, vc[i], acc[i] * corr);
        m = mnew;
    }
    const float inv = 1.0f / (ssum + 1e-8f);
    const float cnt = (float)max64(s1 - s0, 1);
    float *on = a.out + n * (int64_t)(32 * S) + lane * S;
#pragma unroll
    for (int i = 0; i < S; i++) {
        float v = acc[i] * inv;
        if (a.reduce == FEQ_REDUCE_MEAN) v /= cnt;
        on[i] = v;
    }
}

// The same pooling with the K and V rows of each destination's edges brought into a
// per-warp ring of kAttnRing shared-memory slots by bulk copies, kAttnRing edges ahead.  The
// warp-per-edge chain of the kernel above -- perm[pos], then src[e], then the K / V rows,
// three round trips to L2 or HBM per edge -- is what bounds it; here the lanes load a whole
// batch of 32 edge ids and src ids with one coalesced load each, and lane 0 keeps the rows of
// the next kAttnRing edges in flight while the current one is folded in.  Arithmetic, and so
// the result, is that of attn_pool_warp_kernel.  Every wait is bounded: on time-out the kernel
// sets status 2, waits for its copies and leaves.
constexpr int kAttnRing = 4;

template <int S>
__global__ void __launch_bounds__(128)
attn_pool_ring_kernel(const __grid_constant__ FeqAttnArgs a, uint64_t wait_ns) {
    constexpr int ROW = 32 * S;                 // floats of one K or V row
    constexpr uint32_t RB = ROW * 4;            // bytes of one row
    extern __shared__ __align__(128) float attn_ring_sm[];
    __shared__ uint64_t bars[4][kAttnRing];
    __shared__ int abort_s[4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *ring = attn_ring_sm + (size_t)warp * kAttnRing * 2 * ROW;
    if (lane == 0) {
        for (int r = 0; r < kAttnRing; r++) sm100::mbar_init(&bars[warp][r], 1);
        abort_s[warp] = 0;
        sm100::fence_mbar_init();
    }
    __syncwarp();
    const int64_t n = (int64_t)blockIdx.x * 4 + warp;
    if (n >= a.num_nodes) return;
    volatile int *abort_flag = &abort_s[warp];
    const int qrow = a.c_qk * a.d_qk;
    const int H = a.num_heads, gl = 32 / H;
    const bool split_k = a.k != nullptr;
    const int64_t nsrc = split_k ? a.num_src_nodes : a.num_nodes;
    const float *kbase = split_k ? a.k : a.qk + qrow;
    const int64_t k_ld = split_k ? qrow : 2 * (int64_t)qrow;
    const float *qn = a.qk + n * (int64_t)(split_k ? qrow : 2 * qrow) + lane * S;
    const bool decay = a.decay_scale > 0.0f && a.distances;
    float q[S], acc[S];
#pragma unroll
    for (int i = 0; i < S; i++) {
        q[i] = __ldg(qn + i);
        acc[i] = 0.0f;
    }
    float m = -INFINITY, ssum = 0.0f;
    const int64_t s0 = a.offsets[n], s1 = a.offsets[n + 1];
    uint32_t issued = 0, used = 0;              // copies issued / consumed by this warp
    bool ok = true;
    for (int64_t base = s0; base < s1 && ok; base += 32) {
        const int cnt = (int)((s1 - base) < 32 ? (s1 - base) : 32);
        int64_t my_e = 0, my_s = -1;
        float my_d = 0.0f;
        if (lane < cnt) {
            my_e = a.perm[base + lane];
            my_s = a.src[my_e];
            if (my_s < 0 || my_s >= nsrc) {
                set_status(a.status, 1);
                my_s = -1;
            }
            if (decay) my_d = a.distances[my_e];
        }
        auto issue = [&](int k) {                // edge k of the batch into the next slot
            const int64_t e = __shfl_sync(0xffffffffu, my_e, k);
            const int64_t sidx = __shfl_sync(0xffffffffu, my_s, k);
            if (lane == 0) {
                const int slot = (int)(issued % kAttnRing);
                float *dst = ring + (size_t)slot * 2 * ROW;
                sm100::mbar_arrive_expect_tx(&bars[warp][slot], sidx >= 0 ? 2 * RB : RB);
                if (sidx >= 0) rot::bulk_load(dst, kbase + sidx * k_ld, RB, &bars[warp][slot]);
                rot::bulk_load(dst + ROW, a.v + e * (int64_t)ROW, RB, &bars[warp][slot]);
            }
            issued++;
        };
        const int pre = cnt < kAttnRing ? cnt : kAttnRing;
        for (int k = 0; k < pre; k++) issue(k);
        for (int k = 0; k < cnt; k++) {
            const int slot = (int)(used % kAttnRing);
            if (!sm100::mbar_wait(&bars[warp][slot], (used / kAttnRing) & 1u, abort_flag, wait_ns)) {
                set_status(a.status, 2);
                ok = false;
                break;
            }
            used++;
            const float *row = ring + (size_t)slot * 2 * ROW + lane * S;
            const bool has_k = __shfl_sync(0xffffffffu, my_s, k) >= 0;
            const float dd = __shfl_sync(0xffffffffu, my_d, k);
            float kc[S], vc[S];
#pragma unroll
            for (int i = 0; i < S; i++) {
                kc[i] = has_k ? row[i] : 0.0f;
                vc[i] = row[ROW + i];
            }
            // every lane has read the slot: it may be refilled (generic reads before the
            // async-proxy writes of the next copy)
            rot::fence_async_smem();
            __syncwarp();
            if (k + kAttnRing < cnt) issue(k + kAttnRing);
            float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
            for (int i = 0; i + 1 < S; i += 2) {
                d0 = fmaf(q[i], kc[i], d0);
                d1 = fmaf(q[i + 1], kc[i + 1], d1);
            }
            if (S & 1) d0 = fmaf(q[S - 1], kc[S - 1], d0);
            float dot = d0 + d1;
            for (int o = 1; o < gl; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            float lg = dot * a.scale;
            if (decay) lg -= dd / a.decay_scale;
            const float mnew = fmaxf(m, lg);
            const float corr = (m == -INFINITY) ? 0.0f : expf(m - mnew);
            const float p = expf(lg - mnew);
            ssum = ssum * corr + p;
#pragma unroll
            for (int i = 0; i < S; i++) acc[i] = fmaf(p, vc[i], acc[i] * corr);
            m = mnew;
        }
    }
    if (!ok) {                                   // copies still in flight land before the exit
        if (lane == 0)
            for (; used < issued; used++)
                sm100::mbar_wait_drain(&bars[warp][used % kAttnRing], (used / kAttnRing) & 1u);
        __syncwarp();
        return;
    }
    const float inv = 1.0f / (ssum + 1e-8f);
    const float cnt_all = (float)max64(s1 - s0, 1);
    float *on = a.out + n * (int64_t)ROW + lane * S;
#pragma unroll
    for (int i = 0; i < S; i++) {
        float v = acc[i] * inv;
        if (a.reduce == FEQ_REDUCE_MEAN) v /= cnt_all;
        on[i] = v;
    }
}

template <int S>
static int launch_attn_pool_ring(const FeqAttnArgs &a, cudaStream_t s) {
    const size_t smem = (size_t)4 * kAttnRing * 2 * 32 * S * sizeof(float);
    FEQ_CUDA_TRY(cudaFuncSetAttribute(attn_pool_ring_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_pool_ring_kernel<S><<<(unsigned)((a.num_nodes + 3) / 4), 128, smem, s>>>(a, wait_limit_ns());
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

template <int S>
static int launch_attn_pool_warp(const FeqAttnArgs &a, cudaStream_t s) {
    attn_pool_warp_kernel<S><<<(unsigned)((a.num_nodes + 3) / 4), 128, 0, s>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_attn_pool(const FeqAttnArgs &a, cudaStream_t s) {
    if (a.num_nodes == 0) return FEQ_OK;
    {
        // warp-per-destination path: Q / K and V rows of equal length split over 32 lanes,
        // whole heads per lane group
        const int qrow = a.c_qk * a.d_qk, vrow = a.c_v * a.d_v, H = a.num_heads;
        const bool aligned = ((reinterpret_cast<uintptr_t>(a.qk) | reinterpret_cast<uintptr_t>(a.v) |
                               reinterpret_cast<uintptr_t>(a.k)) & 7) == 0;
        if (qrow == vrow && qrow % 32 == 0 && H >= 1 && H <= 32 && 32 % H == 0 && aligned &&
            a.num_nodes <= 0x1ffffffffll) {
            const int S = qrow / 32;
            // rows by bulk copy: 16-byte aligned rows (32 S floats are a multiple of 16 bytes)
            const bool aligned16 = ((reinterpret_cast<uintptr_t>(a.qk) | reinterpret_cast<uintptr_t>(a.v) |
                                     reinterpret_cast<uintptr_t>(a.k)) & 15) == 0;
            if (aligned16) {
                if (S == 18) return launch_attn_pool_ring<18>(a, s);
                if (S == 9) return launch_attn_pool_ring<9>(a, s);
                if (S == 16) return launch_attn_pool_ring<16>(a, s);
                if (S == 8) return launch_attn_pool_ring<8>(a, s);
            }
            if (S == 18) return launch_attn_pool_warp<18>(a, s);    // Repr([0,1,2], 64)
            if (S == 9) return launch_attn_pool_warp<9>(a, s);      // Repr([0,1,2], 32)
            if (S == 16) return launch_attn_pool_warp<16>(a, s);    // Repr([0..3], 32)
            if (S == 8) return launch_attn_pool_warp<8>(a, s);      // Repr([0,1], 64)
        }
    }
    if (a.num_heads < 1 || a.num_heads > kAttnMaxHeads) return FEQ_ERR_UNSUPPORTED;
    if (a.num_nodes > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = sizeof(float) * ((size_t)a.c_qk * a.d_qk + (size_t)a.c_v * a.d_v);
    if (smem > 160 * 1024) return FEQ_ERR_UNSUPPORTED;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(attn_pool_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_pool_kernel<<<(unsigned)a.num_nodes, kAttnThreads, smem, s>>>(a);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
