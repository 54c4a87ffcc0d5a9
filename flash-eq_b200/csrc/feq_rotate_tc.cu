// feq_rotate_tc.cu -- the rotations into and out of the edge frame that feed and
// drain the tensor-core radial mix, for bases given by edge directions.
//
// Reference behaviour replaced:
//   torch.bmm(edge_features, P) and the solid-harmonic factor   flash_eq/layers/linear.py:135-140
//   torch.bmm(out_diag, Q.mT)                                    flash_eq/layers/linear.py:160
//
// One warp streams edges in sorted-bin order.  Every input row moves as a single
// bulk copy (cp.async.bulk, completion on an mbarrier, no multicast): the next
// edge's row is in flight while the current one is rotated.  rotate_in writes its
// bf16 columns straight to HBM (lanes hold consecutive channel pairs, so each store
// covers 128 contiguous bytes); rotate_out stages the output row in shared memory
// and writes it back with one bulk store.  Every lane rotates two channels of each
// irrep in registers through the factored block D_l = R(phi) M_l R(phi)^T: two
// z-rotations by the edge azimuth around the sparse M_l, whose entries are generated
// code (gen_wigner_tables.py) with s^l folded in.  Degrees above 6 fall back to
// per-edge blocks built in shared memory (rows padded to 4 floats, float4 reads).
//
//   rotate_in : A[p][base(j) + c] = s^l (f[e][c] . D)[j]          (bf16, or bf16 hi + lo)
//   rotate_out: out[e][c][k]      = sum_q D[k][q] s^l h[p][base(q) + c]
//
// The closed form of the blocks and the direction reduction are those of the basis
// kernel (feq_rotate.cu), so the fused path and a materialised basis agree.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <numeric>

#include "feq_internal.cuh"
#include "feq_sm100.cuh"
#include "_build/feq_wigner_tables.inc"
#include "feq_rot_common.cuh"

namespace feq {
namespace {

using namespace rot;

constexpr int kRotWarps = 4;     // warps per block
constexpr int kGroup = 32;       // edges whose per-edge scalars are computed together
constexpr int kWtcKUpTo4[5] = FEQ_WTC_K_UPTO4;   // terms per M entry, degrees 0..4


// Float offset of degree-slot u's padded block (N rows of pad4(N) floats).
__host__ __device__ inline int rblock_floats(const ReprLayout &L) {
    int t = 0;
    for (int u = 0; u < L.n_unique; u++) {
        const int n = 2 * L.unique_l[u] + 1;
        t += n * pad4(n);
    }
    return t;
}

// M_l(theta') = sum_q T_l[:, :, q] tv[q] for one degree, then the padded rotation block
//   kIn : R[q][o] = s^l D[q][o]      (input side: y[o] = sum_q f[q] R[q][o])
//   !kIn: R[q][o] = s^l D[o][q]      (output side: y[o] = sum_q h[q] R[q][o])
// D = R(phi) M R(phi)^T as in the basis kernel.  Whole warp; ends with __syncwarp.
template <int N, bool kIn>
__device__ __forceinline__ void build_rblock(const float *__restrict__ tr, int lmax, float sl, float *__restrict__ m_s,
                                             float *__restrict__ r_s, int lane) {
    constexpr int l = (N - 1) / 2, P = pad4(N), K = l / 2 + 1, kRounds = (N * N + 31) / 32;
    static_assert(kWtcKUpTo4[l] == K, "compressed Wigner table layout");
    const float *tv = tr, *cp = tr + 2 * lmax + 1, *sp = cp + lmax + 1;
    const float *coef = feq_wtc_coef + feq_wtc_offset[l];
    const unsigned char *term = feq_wtc_term + feq_wtc_offset[l];
#pragma unroll
    for (int rd = 0; rd < kRounds; rd++) {
        const int idx = lane + 32 * rd;
        if (idx < N * N) {
            float acc = 0.0f;
#pragma unroll
            for (int k = 0; k < K; k++) acc = fmaf(__ldg(coef + idx * K + k), tv[__ldg(term + idx * K + k)], acc);
            m_s[idx] = acc;
        }
    }
    __syncwarp();
#pragma unroll
    for (int rd = 0; rd < kRounds; rd++) {
        const int idx = lane + 32 * rd;
        if (idx >= N * N) break;
        const int a = idx / N, b = idx - a * N;
        const int ma = a < l ? l - a : a - l, mb = b < l ? l - b : b - l;
        const float ca = cp[ma], cb = cp[mb];
        const float sa = a < l ? sp[ma] : -sp[ma];
        const float sb = b < l ? sp[mb] : -sp[mb];
        float v = ca * cb * m_s[a * N + b];
        if (mb) v = fmaf(ca * sb, m_s[a * N + (2 * l - b)], v);
        if (ma) v = fmaf(sa * cb, m_s[(2 * l - a) * N + b], v);
        if (ma && mb) v = fmaf(sa * sb, m_s[(2 * l - a) * N + (2 * l - b)], v);
        if (kIn) r_s[a * P + b] = v * sl;
        else r_s[b * P + a] = v * sl;
    }
    __syncwarp();
}

// Runtime-degree variant of build_rblock (degrees above 4).
template <bool kIn>
__device__ void build_rblock_any(int l, const float *__restrict__ tr, int lmax, float sl, float *__restrict__ m_s,
                                 float *__restrict__ r_s, int lane) {
    const int N = 2 * l + 1, P = pad4(N), K = feq_wtc_k[l];
    const float *tv = tr, *cp = tr + 2 * lmax + 1, *sp = cp + lmax + 1;
    const float *coef = feq_wtc_coef + feq_wtc_offset[l];
    const unsigned char *term = feq_wtc_term + feq_wtc_offset[l];
    for (int idx = lane; idx < N * N; idx += 32) {
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc = fmaf(__ldg(coef + idx * K + k), tv[__ldg(term + idx * K + k)], acc);
        m_s[idx] = acc;
    }
    __syncwarp();
    for (int idx = lane; idx < N * N; idx += 32) {
        const int a = idx / N, b = idx - a * N;
        const int ma = a < l ? l - a : a - l, mb = b < l ? l - b : b - l;
        const float ca = cp[ma], cb = cp[mb];
        const float sa = a < l ? sp[ma] : -sp[ma];
        const float sb = b < l ? sp[mb] : -sp[mb];
        float v = ca * cb * m_s[a * N + b];
        if (mb) v = fmaf(ca * sb, m_s[a * N + (2 * l - b)], v);
        if (ma) v = fmaf(sa * cb, m_s[(2 * l - a) * N + b], v);
        if (ma && mb) v = fmaf(sa * sb, m_s[(2 * l - a) * N + (2 * l - b)], v);
        if (kIn) r_s[a * P + b] = v * sl;
        else r_s[b * P + a] = v * sl;
    }
    __syncwarp();
}

// All degree blocks of one edge.  rdoff[u] = float offset of slot u's padded block.
template <bool kIn>
__device__ __forceinline__ void build_all_rblocks(const ReprLayout &L, const int16_t *rdoff, const float *tr, float s,
                                                  float *m_s, float *r_s, int lane) {
    for (int u = 0; u < L.n_unique; u++) {
        const int l = L.unique_l[u];
        const float sl = ipowf(s, l);
        float *R = r_s + rdoff[u];
        switch (l) {
            case 0: build_rblock<1, kIn>(tr, L.lmax, sl, m_s, R, lane); break;
            case 1: build_rblock<3, kIn>(tr, L.lmax, sl, m_s, R, lane); break;
            case 2: build_rblock<5, kIn>(tr, L.lmax, sl, m_s, R, lane); break;
            case 3: build_rblock<7, kIn>(tr, L.lmax, sl, m_s, R, lane); break;
            case 4: build_rblock<9, kIn>(tr, L.lmax, sl, m_s, R, lane); break;
            default: build_rblock_any<kIn>(l, tr, L.lmax, sl, m_s, R, lane);
        }
    }
}

// y[o] = sum_q x[q] R[q][o] for two channels at once; x from get(q) -> float2, rows of R
// read as float4 broadcasts, every output emitted as emit(o, y_ch0, y_ch1).
template <int N, typename Get, typename Emit>
__device__ __forceinline__ void rotate_pair(const float *__restrict__ R, Get get, Emit emit) {
    constexpr int P = pad4(N);
    float2 x[N];
#pragma unroll
    for (int q = 0; q < N; q++) x[q] = get(q);
    float a0[P], a1[P];
#pragma unroll
    for (int o = 0; o < P; o++) a0[o] = a1[o] = 0.0f;
#pragma unroll
    for (int q = 0; q < N; q++) {
        const float4 *row = reinterpret_cast<const float4 *>(R + q * P);
#pragma unroll
        for (int o4 = 0; o4 < P / 4; o4++) {
            const float4 r = row[o4];
            const float rv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (4 * o4 + i < N) {   // padding columns are never read back
                    a0[4 * o4 + i] = fmaf(x[q].x, rv[i], a0[4 * o4 + i]);
                    a1[4 * o4 + i] = fmaf(x[q].y, rv[i], a1[4 * o4 + i]);
                }
            }
        }
    }
#pragma unroll
    for (int o = 0; o < N; o++) emit(o, a0[o], a1[o]);
}

template <typename Get, typename Emit>
__device__ __forceinline__ void rotate_pair_any(int l, const float *__restrict__ R, Get get, Emit emit) {
    switch (l) {
        case 0: rotate_pair<1>(R, get, emit); break;
        case 1: rotate_pair<3>(R, get, emit); break;
        case 2: rotate_pair<5>(R, get, emit); break;
        case 3: rotate_pair<7>(R, get, emit); break;
        case 4: rotate_pair<9>(R, get, emit); break;
        default: {
            const int N = 2 * l + 1, P = pad4(N);
            for (int o = 0; o < N; o++) {
                float y0 = 0.0f, y1 = 0.0f;
                for (int q = 0; q < N; q++) {
                    const float2 v = get(q);
                    const float r = R[q * P + o];
                    y0 = fmaf(v.x, r, y0);
                    y1 = fmaf(v.y, r, y1);
                }
                emit(o, y0, y1);
            }
        }
    }
}

// Shared per-warp scratch, in floats: the group's trig, one M block, the rotation blocks.
struct RotScratch {
    int trig, mblk, rblk;      // float counts
    __host__ __device__ int total() const { return trig + mblk + rblk; }
};
__host__ __device__ inline RotScratch rot_scratch(const ReprLayout &L) {
    RotScratch s;
    s.trig = pad4(kGroup * trig_floats(L.lmax));
    s.mblk = pad4((2 * L.lmax + 1) * (2 * L.lmax + 1));
    s.rblk = pad4(rblock_floats(L));
    return s;
}

__device__ __forceinline__ void rblock_offsets(const ReprLayout &L, int16_t *rdoff) {
    int t = 0;
    for (int u = 0; u < L.n_unique; u++) {
        rdoff[u] = (int16_t)t;
        const int n = 2 * L.unique_l[u] + 1;
        t += n * pad4(n);
    }
}

__device__ __forceinline__ void copy_layout(const ReprLayout &src, ReprLayout &dst) {
    const int *s = reinterpret_cast<const int *>(&src);
    int *d = reinterpret_cast<int *>(&dst);
    for (int i = threadIdx.x; i < (int)(sizeof(ReprLayout) / 4); i += blockDim.x) d[i] = s[i];
}

// Per-block shared state in front of the per-warp areas.
struct RotShared {
    ReprLayout L;
    int16_t rdoff[kMaxL + 1];
    uint64_t bar[kRotWarps][2];
    int abort_flag;
};

// Per-warp dynamic shared memory (floats): in[2] rows, the out row, scratch.
struct RotWarpLayout {
    int in_row, out_row, scratch;   // floats, each a multiple of 4
    uint64_t wait_ns;               // limit of each row wait (wait_limit_ns())
    __host__ __device__ int total() const { return 2 * in_row + out_row + scratch; }
};

// Bounded wait for row buffer `b`; false on time-out (status 2, the CTA aborts).
__device__ __forceinline__ bool wait_row(RotShared &S, int w, int b, uint32_t &phase_bits, int32_t *status,
                                         uint64_t limit_ns) {
    const bool ok = sm100::mbar_wait(&S.bar[w][b], (phase_bits >> b) & 1u, &S.abort_flag, limit_ns);
    if (ok) phase_bits ^= 1u << b;
    else set_status(status, 2);
    return ok;
}

// A[p][base_std(k) + c] = s_e^l(k) (f[e][c] . D_e)[k] as bf16 (hi, and lo = f - hi when kSplit);
// f[e] = x[src[e]] (kGather) or x[e], plus edge_add[e] when given; tval[p] = t_e.
template <bool kGather, bool kSplit, bool kFactored>
__global__ void __launch_bounds__(kRotWarps * 32)
rot_in_kernel(const float *__restrict__ x, const int64_t *__restrict__ src, int64_t nsrc,
              const float *__restrict__ edge_add, const float *__restrict__ dirs, const float *__restrict__ dist,
              const int64_t *__restrict__ perm, int64_t E, int C, const __grid_constant__ ReprLayout Lp,
              const __grid_constant__ TcPosMap Mp, int k_total, Binning bins, float sh_scale, RotWarpLayout WL,
              __nv_bfloat16 *__restrict__ A_hi, __nv_bfloat16 *__restrict__ A_lo, float *__restrict__ tval,
              int32_t *status) {
    extern __shared__ __align__(128) float dsm[];
    __shared__ RotShared S;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    copy_layout(Lp, S.L);
    if (threadIdx.x == 0) {
        S.abort_flag = 0;
        for (int i = 0; i < kRotWarps; i++) {
            sm100::mbar_init(&S.bar[i][0], 1);
            sm100::mbar_init(&S.bar[i][1], 1);
        }
        sm100::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) rblock_offsets(S.L, S.rdoff);
    const ReprLayout &L = S.L;
    const int d = L.dim, row = C * d;
    int32_t *bstd = reinterpret_cast<int32_t *>(dsm);
    for (int i = threadIdx.x; i < d; i += blockDim.x) bstd[i] = Mp.base_std[i];
    __syncthreads();

    float *ws = dsm + pad4(d) + (size_t)w * WL.total();
    const RotScratch SC = rot_scratch(L);
    float *trig = ws + 2 * WL.in_row + WL.out_row;
    float *m_s = trig + SC.trig, *r_s = m_s + SC.mblk;
    const int TF = trig_floats(L.lmax);
    const uint32_t row_bytes = (uint32_t)row * 4u;
    uint32_t phase_bits = 0;
    int pending = 0;   // bit b: a bulk load into buffer b is in flight
    bool alive = true;

    for (int64_t g0 = ((int64_t)blockIdx.x * kRotWarps + w) * kGroup; alive && g0 < E;
         g0 += (int64_t)gridDim.x * kRotWarps * kGroup) {
        const int ng = (int)min64(kGroup, E - g0);
        int64_t e_l = 0, xr_l = -1;
        float s_l = 0.0f;
        if (lane < ng) {
            const int64_t p = g0 + lane;
            e_l = perm[p];
            const float dd = dist[e_l];
            s_l = dd / (dd + sh_scale);
            int lo;
            float t;
            bin_of(dd, bins, lo, t);
            tval[p] = t;
            edge_trig_compact(dirs[e_l * 3], dirs[e_l * 3 + 1], dirs[e_l * 3 + 2], L.lmax, trig + lane * TF);
            xr_l = e_l;
            if (kGather) {
                xr_l = src[e_l];
                if (xr_l < 0 || xr_l >= nsrc) {
                    set_status(status, 1);
                    xr_l = -1;
                }
            }
        }
        __syncwarp();
        auto issue = [&](int j) {
            const int64_t xr = __shfl_sync(0xffffffffu, xr_l, j);
            const int b = j & 1;
            if (xr >= 0 && lane == 0) {
                fence_async_smem();
                sm100::mbar_arrive_expect_tx(&S.bar[w][b], row_bytes);
                bulk_load(ws + b * WL.in_row, x + xr * (int64_t)row, row_bytes, &S.bar[w][b]);
            }
            if (xr >= 0) pending |= 1 << b;
        };
        issue(0);
        for (int j = 0; j < ng; j++) {
            const int64_t e = __shfl_sync(0xffffffffu, e_l, j);
            const int64_t xr = __shfl_sync(0xffffffffu, xr_l, j);
            const float s = __shfl_sync(0xffffffffu, s_l, j);
            const int64_t p = g0 + j;
            const int b = j & 1;
            if (j + 1 < ng) issue(j + 1);
            if constexpr (!kFactored) build_all_rblocks<true>(L, S.rdoff, trig + j * TF, s, m_s, r_s, lane);
            const float *trj = trig + j * TF;
            float *fb = ws + b * WL.in_row;
            if (xr >= 0) {
                if (!wait_row(S, w, b, phase_bits, status, WL.wait_ns)) {
                    alive = false;
                    break;
                }
                pending &= ~(1 << b);
            } else {
                for (int i = lane; i < row; i += 32) fb[i] = 0.0f;
            }
            if (edge_add) {
                const float4 *ea = reinterpret_cast<const float4 *>(edge_add + e * (int64_t)row);
                float4 *f4 = reinterpret_cast<float4 *>(fb);
                for (int i = lane; i < row / 4; i += 32) {
                    const float4 a = __ldg(ea + i);
                    float4 v = f4[i];
                    v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
                    f4[i] = v;
                }
            }
            __syncwarp();
            __nv_bfloat16 *ah = A_hi + p * (int64_t)k_total;
            __nv_bfloat16 *al = kSplit ? A_lo + p * (int64_t)k_total : nullptr;
            for (int r = 0; r < Mp.n_pad; r++)      // K padding of the m-blocks (zero columns)
                for (int i = Mp.pad_lo[r] + 2 * lane; i < Mp.pad_hi[r]; i += 64) {
                    *reinterpret_cast<uint32_t *>(ah + i) = 0u;
                    if (kSplit) *reinterpret_cast<uint32_t *>(al + i) = 0u;
                }
            // lanes hold consecutive channel pairs: every column store is 128 contiguous bytes
            for (int c = 2 * lane; c < C; c += 64) {
                const float *f0 = fb + c * d, *f1 = f0 + d;
                for (int r = 0; r < L.n_irreps; r++) {
                    const int l = L.irrep_l[r], off = L.irrep_off[r];
                    const int32_t *bo = bstd + off;
                    auto get = [&](int q) { return make_float2(f0[off + q], f1[off + q]); };
                    auto emit = [&](int o, float y0, float y1) {
                        const int bcol = bo[o];
                        if (bcol < 0) return;
                        const __nv_bfloat162 hi = __floats2bfloat162_rn(y0, y1);
                        *reinterpret_cast<__nv_bfloat162 *>(ah + bcol + c) = hi;
                        if (kSplit) {
                            const float2 hf = __bfloat1622float2(hi);
                            *reinterpret_cast<__nv_bfloat162 *>(al + bcol + c) =
                                __floats2bfloat162_rn(y0 - hf.x, y1 - hf.y);
                        }
                    };
                    if constexpr (kFactored)
                        rot_irrep2_any<false>(l, trj, L.lmax, ipowf(s, l), get, emit);
                    else
                        rotate_pair_any(l, r_s + S.rdoff[L.irrep_slot[r]], get, emit);
                }
            }
            __syncwarp();
        }
    }
    // drain: loads still in flight (only after an abort) and the last stores
    for (int b = 0; b < 2; b++)
        if (pending & (1 << b)) sm100::mbar_wait_drain(&S.bar[w][b], (phase_bits >> b) & 1u);
    if (lane == 0) bulk_wait0();
}

// out[e][c][k] = sum_q D_e[k][q] s_e^l h[q][c], h[q][c] = H[p][base_std(q) + c] (0 where
// base_std < 0: output blocks that receive no input).
template <bool kFactored>
__global__ void __launch_bounds__(kRotWarps * 32)
rot_out_kernel(const float *__restrict__ H, int h_ld, const float *__restrict__ dirs, const float *__restrict__ dist,
               const int64_t *__restrict__ perm, int64_t E, int C, const __grid_constant__ ReprLayout Lp,
               const __grid_constant__ TcPosMap Mp, float sh_scale, RotWarpLayout WL, float *__restrict__ out,
               int32_t *status) {
    extern __shared__ __align__(128) float dsm[];
    __shared__ RotShared S;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    copy_layout(Lp, S.L);
    if (threadIdx.x == 0) {
        S.abort_flag = 0;
        for (int i = 0; i < kRotWarps; i++) {
            sm100::mbar_init(&S.bar[i][0], 1);
            sm100::mbar_init(&S.bar[i][1], 1);
        }
        sm100::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) rblock_offsets(S.L, S.rdoff);
    const ReprLayout &L = S.L;
    const int d = L.dim, row = C * d;
    int32_t *bstd = reinterpret_cast<int32_t *>(dsm);
    for (int i = threadIdx.x; i < d; i += blockDim.x) bstd[i] = Mp.base_std[i];
    __syncthreads();

    float *ws = dsm + pad4(d) + (size_t)w * WL.total();
    float *ob = ws + 2 * WL.in_row;
    const RotScratch SC = rot_scratch(L);
    float *trig = ob + WL.out_row;
    float *m_s = trig + SC.trig, *r_s = m_s + SC.mblk;
    const int TF = trig_floats(L.lmax);
    const uint32_t h_bytes = (uint32_t)h_ld * 4u, o_bytes = (uint32_t)row * 4u;
    uint32_t phase_bits = 0;
    int pending = 0;
    bool alive = true;

    for (int64_t g0 = ((int64_t)blockIdx.x * kRotWarps + w) * kGroup; alive && g0 < E;
         g0 += (int64_t)gridDim.x * kRotWarps * kGroup) {
        const int ng = (int)min64(kGroup, E - g0);
        int64_t e_l = 0;
        float s_l = 0.0f;
        if (lane < ng) {
            e_l = perm[g0 + lane];
            const float dd = dist[e_l];
            s_l = dd / (dd + sh_scale);
            edge_trig_compact(dirs[e_l * 3], dirs[e_l * 3 + 1], dirs[e_l * 3 + 2], L.lmax, trig + lane * TF);
        }
        __syncwarp();
        auto issue = [&](int j) {
            const int b = j & 1;
            if (lane == 0) {
                fence_async_smem();
                sm100::mbar_arrive_expect_tx(&S.bar[w][b], h_bytes);
                bulk_load(ws + b * WL.in_row, H + (g0 + j) * (int64_t)h_ld, h_bytes, &S.bar[w][b]);
            }
            pending |= 1 << b;
        };
        issue(0);
        for (int j = 0; j < ng; j++) {
            const int64_t e = __shfl_sync(0xffffffffu, e_l, j);
            const float s = __shfl_sync(0xffffffffu, s_l, j);
            const int b = j & 1;
            if (j + 1 < ng) issue(j + 1);
            if constexpr (!kFactored) build_all_rblocks<false>(L, S.rdoff, trig + j * TF, s, m_s, r_s, lane);
            const float *trj = trig + j * TF;
            if (!wait_row(S, w, b, phase_bits, status, WL.wait_ns)) {
                alive = false;
                break;
            }
            pending &= ~(1 << b);
            const float *hb = ws + b * WL.in_row;
            if (lane == 0) bulk_wait_read0();   // the previous output row has left shared memory
            __syncwarp();
            for (int c = 2 * lane; c < C; c += 64) {
                float *o0 = ob + c * d, *o1 = o0 + d;
                for (int r = 0; r < L.n_irreps; r++) {
                    const int l = L.irrep_l[r], off = L.irrep_off[r];
                    const int32_t *bi = bstd + off;
                    auto get = [&](int q) {
                        const int bcol = bi[q];
                        return bcol < 0 ? make_float2(0.0f, 0.0f) : *reinterpret_cast<const float2 *>(hb + bcol + c);
                    };
                    auto emit = [&](int o, float y0, float y1) {
                        o0[off + o] = y0;
                        o1[off + o] = y1;
                    };
                    if constexpr (kFactored)
                        rot_irrep2_any<true>(l, trj, L.lmax, ipowf(s, l), get, emit);
                    else
                        rotate_pair_any(l, r_s + S.rdoff[L.irrep_slot[r]], get, emit);
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                bulk_store(out + e * (int64_t)row, ob, o_bytes);
                bulk_commit();
            }
        }
    }
    for (int b = 0; b < 2; b++)
        if (pending & (1 << b)) sm100::mbar_wait_drain(&S.bar[w][b], (phase_bits >> b) & 1u);
    if (lane == 0) bulk_wait0();
}

// Dense per-edge basis: MFIRST  out[e][k][j] = D_e[k][perm[j]]  (same irrep, else 0)
//                      ROT_TO_EZ out[e][k][j] = D_e[j][k]       (std order, D^T)
// One warp per edge; lanes own columns, so every row is written with contiguous stores.
__global__ void __launch_bounds__(kRotWarps * 32)
basis_warp_kernel(const float *__restrict__ dirs, int64_t E, const __grid_constant__ ReprLayout Lp, int mfirst,
                  int scratch_floats, float *__restrict__ out) {
    extern __shared__ __align__(128) float dsm[];
    __shared__ RotShared S;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    copy_layout(Lp, S.L);
    __syncthreads();
    if (threadIdx.x == 0) rblock_offsets(S.L, S.rdoff);
    __syncthreads();
    const ReprLayout &L = S.L;
    const int d = L.dim;
    const int64_t dd = (int64_t)d * d;
    const RotScratch SC = rot_scratch(L);
    float *trig = dsm + (size_t)w * scratch_floats;
    float *m_s = trig + SC.trig, *r_s = m_s + SC.mblk;
    const int TF = trig_floats(L.lmax);
    for (int64_t g0 = ((int64_t)blockIdx.x * kRotWarps + w) * kGroup; g0 < E;
         g0 += (int64_t)gridDim.x * kRotWarps * kGroup) {
        const int ng = (int)min64(kGroup, E - g0);
        if (lane < ng) {
            const float *v = dirs + (g0 + lane) * 3;
            edge_trig_compact(v[0], v[1], v[2], L.lmax, trig + lane * TF);
        }
        __syncwarp();
        for (int j0 = 0; j0 < ng; j0++) {
            build_all_rblocks<true>(L, S.rdoff, trig + j0 * TF, 1.0f, m_s, r_s, lane);
            float *o = out + (g0 + j0) * dd;
            for (int jc = lane; jc < d; jc += 32) {
                const int a = mfirst ? L.perm[jc] : jc;           // std index carried by this column
                const int ir = L.std_irrep[a], off = L.irrep_off[ir], n = 2 * L.irrep_l[ir] + 1;
                const float *R = r_s + S.rdoff[L.irrep_slot[ir]];
                const int P = pad4(n);
                for (int k = 0; k < d; k++) {
                    const int rel = k - off;
                    float v = 0.0f;
                    if (rel >= 0 && rel < n) v = mfirst ? R[rel * P + (a - off)] : R[(a - off) * P + rel];
                    o[(int64_t)k * d + jc] = v;
                }
            }
            __syncwarp();
        }
    }
}

// Dense basis, one lane per edge, in two phases per group of 32 edges.
//  1. Every lane builds its edge's block of each DISTINCT degree (irreps of equal degree
//     share it) in registers and writes it, compact, to its row of the warp's stage:
//       row a of D   (kT = false):  u = R[a] M,    v = R u
//       row a of D^T (kT = true):   u = M R[a]^T,  v = R u
//     (R = R(phi): R[x][x] = cos m phi, R[l-m][l+m] = sin m phi, R[l+m][l-m] = -sin m phi),
//     which equals D = R M R^T entry by entry.  The stage row stride is odd, so the lanes'
//     writes fall in distinct banks, and slot `zero` of every row holds 0.
//  2. The warp streams the group's output -- 32 * d * d contiguous floats -- as float4
//     stores.  Output float f of a period of P edges (P * d * d a multiple of 4) comes
//     from stage float pos[f] (computed once per block: the edge within the period times
//     the row stride, plus the compact entry or the zero slot).
constexpr int kBasisMaxStage = 200 * 1024;

struct BasisCompact {
    int stride;        // floats per stage row (odd)
    int zero;          // slot holding 0
    int period;        // edges after which the float4 pattern repeats (1, 2 or 4)
    int entries;       // float4 entries of one period
    int nwarps;        // warps per block
    int per_warp;      // floats of shared memory per warp (trig + stage)
    size_t smem;       // dynamic shared memory bytes
};

template <int Lg, bool kT>
__device__ __forceinline__ void basis_block(const float *__restrict__ tr, int lmax, float *__restrict__ mine) {
    constexpr int N = 2 * Lg + 1;
    const float *tv = tr, *cp = tr + 2 * lmax + 1, *sp = cp + lmax + 1;
    float M[N * N];
    WA<Lg>::wmd(tv, M);
    float c[Lg + 1], sn[Lg + 1];
#pragma unroll
    for (int m = 0; m <= Lg; m++) {
        c[m] = cp[m];
        sn[m] = sp[m];
    }
    auto rdiag = [&](int x) { return x == Lg ? 1.0f : c[x < Lg ? Lg - x : x - Lg]; };
    auto roff = [&](int x) { return x < Lg ? sn[Lg - x] : (x > Lg ? -sn[x - Lg] : 0.0f); };
#pragma unroll
    for (int a = 0; a < N; a++) {
        const int pa = 2 * Lg - a;
        float u[N];
#pragma unroll
        for (int q = 0; q < N; q++) {
            const float mq = kT ? M[q * N + a] : M[a * N + q];
            const float mp = kT ? M[q * N + pa] : M[pa * N + q];
            u[q] = a == Lg ? mq : rdiag(a) * mq + roff(a) * mp;
        }
#pragma unroll
        for (int b = 0; b < N; b++) {
            const int pb = 2 * Lg - b;
            mine[a * N + b] = b == Lg ? u[b] : rdiag(b) * u[b] + roff(b) * u[pb];
        }
    }
}

__global__ void basis_compact_kernel(const float *__restrict__ dirs, int64_t E, const __grid_constant__ ReprLayout Lp,
                                     int mfirst, BasisCompact B, float *__restrict__ out) {
    extern __shared__ __align__(128) float dsm[];
    __shared__ ReprLayout L;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    copy_layout(Lp, L);
    __syncthreads();
    const int d = L.dim, dd = d * d, TF = trig_floats(L.lmax);
    short4 *pos = reinterpret_cast<short4 *>(dsm);
    // output float f of a period -> stage float (one-time table; divisions are fine here)
    for (int t = threadIdx.x; t < B.entries; t += blockDim.x) {
        short v[4];
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int f = 4 * t + s, er = f / dd, p = f - er * dd, k = p / d, j = p - k * d;
            const int sj = mfirst ? L.perm[j] : j;       // std column carried by output column j
            const int r = L.std_irrep[k];
            int c = B.zero;
            if (L.std_irrep[sj] == r) {
                const int off = L.irrep_off[r], n = 2 * L.irrep_l[r] + 1;
                c = L.unique_doff[L.irrep_slot[r]] + (k - off) * n + (sj - off);
            }
            v[s] = (short)(er * B.stride + c);
        }
        pos[t] = make_short4(v[0], v[1], v[2], v[3]);
    }
    float *trig = dsm + 2 * pad4(B.entries) + (size_t)w * B.per_warp;
    float *stage = trig + pad4(kGroup * TF);
    stage[lane * B.stride + B.zero] = 0.0f;
    __syncthreads();
    const float *tr = trig + lane * TF;
    float *mine = stage + lane * B.stride;
    const int pstride = B.period * B.stride;
    for (int64_t g0 = ((int64_t)blockIdx.x * B.nwarps + w) * kGroup; g0 < E;
         g0 += (int64_t)gridDim.x * B.nwarps * kGroup) {
        const int ng = (int)min64(kGroup, E - g0);
        {
            const int64_t e = g0 + min(lane, ng - 1);
            edge_trig_compact(dirs[e * 3], dirs[e * 3 + 1], dirs[e * 3 + 2], L.lmax, trig + lane * TF);
        }
        __syncwarp();
        for (int u = 0; u < L.n_unique; u++) {
            float *blk = mine + L.unique_doff[u];
#define FEQ_BASIS_CASE(LL)                                                  \
    case LL:                                                                \
        if (mfirst) basis_block<LL, false>(tr, L.lmax, blk);                \
        else basis_block<LL, true>(tr, L.lmax, blk);                        \
        break;
            switch (L.unique_l[u]) {
                case 0: blk[0] = 1.0f; break;
                FEQ_BASIS_CASE(1)
                FEQ_BASIS_CASE(2)
                FEQ_BASIS_CASE(3)
                FEQ_BASIS_CASE(4)
                FEQ_BASIS_CASE(5)
                FEQ_BASIS_CASE(6)
            }
#undef FEQ_BASIS_CASE
        }
        __syncwarp();
        // the group's output is contiguous and starts 16-byte aligned (g0 is a multiple of 32)
        const int nf = ng * dd, nq = nf >> 2;
        float4 *o4 = reinterpret_cast<float4 *>(out + g0 * (int64_t)dd);
        int t = lane, pb = 0;
        while (t >= B.entries) {
            t -= B.entries;
            pb += pstride;
        }
#pragma unroll 4
        for (int q = lane; q < nq; q += 32) {
            const short4 ix = pos[t];
            float4 v;
            v.x = stage[pb + ix.x];
            v.y = stage[pb + ix.y];
            v.z = stage[pb + ix.z];
            v.w = stage[pb + ix.w];
            o4[q] = v;
            t += 32;
            while (t >= B.entries) {
                t -= B.entries;
                pb += pstride;
            }
        }
        if (lane == 0 && (nf & 3)) {               // ragged last group: the trailing floats
            const int tt = nq % B.entries, pp = (nq / B.entries) * pstride;
            const short4 ix = pos[tt];
            const short iv[4] = {ix.x, ix.y, ix.z, ix.w};
            float *o = out + g0 * (int64_t)dd + 4 * (int64_t)nq;
            for (int s = 0; s < (nf & 3); s++) o[s] = stage[pp + iv[s]];
        }
        __syncwarp();
    }
}

}  // namespace

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int rot_grid(const void *kernel, size_t smem, int64_t E) {
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kRotWarps * 32, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    const int64_t want = (E + kRotWarps * kGroup - 1) / (kRotWarps * kGroup);
    return (int)std::max<int64_t>(1, min64(want, (int64_t)sms * per_sm));
}

// Streaming rotation into the A matrix of the tensor-core mix.  Returns
// FEQ_ERR_UNSUPPORTED (nothing launched) when the shapes or alignments do not allow
// whole-row bulk copies; the caller then uses the general kernels.
int launch_rot_in_stream(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add, const float *dirs,
                         const float *dist, const int64_t *perm, int64_t E, int C, const ReprLayout &L,
                         const TcPosMap &M, int k_total, Binning bins, float sh_scale, bool split,
                         __nv_bfloat16 *A_hi, __nv_bfloat16 *A_lo, float *tval, int32_t *status, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    if (!dirs || (C & 1) || ((int64_t)C * L.dim) % 4 || k_total % 8 || !aligned16(x) ||
        (edge_add && !aligned16(edge_add)) || !aligned16(A_hi) || (split && !aligned16(A_lo)))
        return FEQ_ERR_UNSUPPORTED;
    RotWarpLayout WL;
    WL.in_row = pad4(C * L.dim);
    WL.out_row = 0;
    WL.wait_ns = wait_limit_ns();
    const bool factored = L.lmax <= kFactoredLmax;
    WL.scratch = factored ? rot_scratch(L).trig : rot_scratch(L).total();
    const size_t smem = ((size_t)pad4(L.dim) + (size_t)kRotWarps * WL.total()) * 4;
    if (smem + sizeof(RotShared) > 200 * 1024) return FEQ_ERR_UNSUPPORTED;
#define FEQ_ROT_IN(G, S)                                                                                        \
    do {                                                                                                        \
        auto k = factored ? rot_in_kernel<G, S, true> : rot_in_kernel<G, S, false>;                                                                         \
        FEQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));          \
        const int grid = rot_grid((const void *)k, smem, E);                                                    \
        k<<<grid, kRotWarps * 32, smem, s>>>(x, src, nsrc, edge_add, dirs, dist, perm, E, C, L, M, k_total, bins, \
                                             sh_scale, WL, A_hi, A_lo, tval, status);                           \
    } while (0)
    if (src) {
        if (split) FEQ_ROT_IN(true, true); else FEQ_ROT_IN(true, false);
    } else {
        if (split) FEQ_ROT_IN(false, true); else FEQ_ROT_IN(false, false);
    }
#undef FEQ_ROT_IN
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// Streaming rotation of the mix result back out of the edge frame.
int launch_rot_out_stream(const float *H, int h_ld, const float *dirs, const float *dist, const int64_t *perm,
                          int64_t E, int C, const ReprLayout &L, const TcPosMap &M, float sh_scale, float *out,
                          int32_t *status, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    if (!dirs || (C & 1) || ((int64_t)C * L.dim) % 4 || h_ld % 4 || !aligned16(H) || !aligned16(out))
        return FEQ_ERR_UNSUPPORTED;
    RotWarpLayout WL;
    WL.in_row = pad4(h_ld);
    WL.out_row = pad4(C * L.dim);
    WL.wait_ns = wait_limit_ns();
    const bool factored = L.lmax <= kFactoredLmax;
    WL.scratch = factored ? rot_scratch(L).trig : rot_scratch(L).total();
    const size_t smem = ((size_t)pad4(L.dim) + (size_t)kRotWarps * WL.total()) * 4;
    if (smem + sizeof(RotShared) > 200 * 1024) return FEQ_ERR_UNSUPPORTED;
    auto k = factored ? rot_out_kernel<true> : rot_out_kernel<false>;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int grid = rot_grid((const void *)k, smem, E);
    k<<<grid, kRotWarps * 32, smem, s>>>(H, h_ld, dirs, dist, perm, E, C, L, M, sh_scale, WL, out, status);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// Dense basis matrices: the compact lane-per-edge kernel where its tables fit in shared
// memory, else warp per edge.  FEQ_ERR_UNSUPPORTED when neither layout fits.
static bool basis_compact_plan(const ReprLayout &L, BasisCompact &B) {
    if (L.lmax > kFactoredLmax) return false;
    const int64_t dd = (int64_t)L.dim * L.dim;
    B.stride = (L.dblock_floats + 1) | 1;
    B.zero = L.dblock_floats;
    B.period = (int)(4 / std::gcd<int64_t>(dd, 4));
    if (B.period * dd / 4 > (int64_t)kBasisMaxStage / 8) return false;
    B.entries = (int)(B.period * dd / 4);
    B.per_warp = pad4(kGroup * trig_floats(L.lmax)) + pad4(kGroup * B.stride);
    const size_t table = (size_t)pad4(B.entries) * 8;
    for (int nw = kRotWarps; nw >= 1; nw--) {
        const size_t smem = table + (size_t)nw * B.per_warp * 4;
        if (smem <= (size_t)kBasisMaxStage) {
            B.nwarps = nw;
            B.smem = smem;
            return true;
        }
    }
    return false;
}

int launch_basis_stream(const float *dirs, int64_t E, const ReprLayout &L, int mfirst, float *out, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    BasisCompact B;
    if (aligned16(out) && basis_compact_plan(L, B)) {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(basis_compact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)B.smem));
        int dev = 0, sms = 148, per_sm = 1;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, basis_compact_kernel, B.nwarps * 32, B.smem) !=
                cudaSuccess || per_sm < 1)
            per_sm = 1;
        const int64_t want = (E + B.nwarps * kGroup - 1) / (B.nwarps * kGroup);
        const int grid = (int)std::max<int64_t>(1, min64(want, (int64_t)sms * per_sm));
        basis_compact_kernel<<<grid, B.nwarps * 32, B.smem, s>>>(dirs, E, L, mfirst, B, out);
        FEQ_LAUNCH_CHECK();
        return FEQ_OK;
    }
    const int scratch = rot_scratch(L).total();
    const size_t smem = (size_t)kRotWarps * scratch * 4;
    if (smem + sizeof(RotShared) > 200 * 1024) return FEQ_ERR_UNSUPPORTED;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(basis_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int grid = rot_grid((const void *)basis_warp_kernel, smem, E);
    basis_warp_kernel<<<grid, kRotWarps * 32, smem, s>>>(dirs, E, L, mfirst, scratch, out);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
