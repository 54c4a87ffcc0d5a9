// feq_rot_common.cuh -- device pieces shared by the edge-frame rotation kernels and the
// fused tensor-core edgewise kernel: bulk copies (no multicast), the per-edge trig of the
// closed-form Wigner blocks, and the generated register-resident per-degree rotations.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "feq_internal.cuh"
#include "feq_sm100.cuh"
#include "_build/feq_wigner_apply.inc"

namespace feq {
namespace rot {

constexpr float kEpsR = 1e-8f;   // get_epsilon(float32), flash_eq/utils.py:19-27

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(sm100::smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(sm100::smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_store(void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(reinterpret_cast<uint64_t>(dst)), "r"(sm100::smem_u32(src)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Per-edge trig, compact: tv = [1, cos t, sin t, cos 2t, sin 2t, ...] (2 lmax + 1 floats)
// followed by cos(m phi), sin(m phi) for m = 0..lmax.  Same float32 steps as the basis
// kernel's edge_trig.
__host__ __device__ constexpr int trig_floats(int lmax) { return 2 * lmax + 1 + 2 * (lmax + 1); }

__device__ __forceinline__ void edge_trig_compact(float vx, float vy, float vz, int lmax, float *tr) {
    float nv = sqrtf(vx * vx + vy * vy + vz * vz);
    float den = nv + kEpsR;
    float dx = vx / den, dy = vy / den, dz = vz / den;
    float n = sqrtf(dy * dy + dx * dx);
    float ax0 = -dy / (n + kEpsR), ax1 = dx / (n + kEpsR);
    float theta = acosf(fminf(fmaxf(dz, -1.0f + kEpsR), 1.0f - kEpsR));
    float rho = sqrtf(ax0 * ax0 + ax1 * ax1);
    float th = theta * rho;
    float c1p = 1.0f, s1p = 0.0f;
    if (rho > 0.0f) {
        c1p = ax0 / rho;
        s1p = ax1 / rho;
    }
    float c1t, s1t;
    sincosf(th, &s1t, &c1t);
    float *tv = tr, *cp = tr + 2 * lmax + 1, *sp = cp + lmax + 1;
    tv[0] = 1.0f;
    cp[0] = 1.0f;
    sp[0] = 0.0f;
    float ct = 1.0f, st = 0.0f, c = 1.0f, s = 0.0f;
    for (int m = 1; m <= lmax; m++) {
        float nct = ct * c1t - st * s1t, nst = st * c1t + ct * s1t;
        float nc = c * c1p - s * s1p, ns = s * c1p + c * s1p;
        ct = nct; st = nst; c = nc; s = ns;
        tv[2 * m - 1] = ct;
        tv[2 * m] = st;
        cp[m] = c;
        sp[m] = s;
    }
}

__host__ __device__ constexpr int pad4(int n) { return (n + 3) & ~3; }

// Compile-time access to the generated per-degree code.
template <int L> struct WA;
#define FEQ_DEF_WA(LL)                                                                                    \
    template <> struct WA<LL> {                                                                           \
        static constexpr int kNnz = FEQ_WM_NNZ_##LL;                                                      \
        __device__ __forceinline__ static void wm(const float *tv, float sl, float (&m)[kNnz]) {          \
            feq_wm_l##LL(tv, sl, m);                                                                      \
        }                                                                                                 \
        __device__ __forceinline__ static void wmd(const float *tv, float (&M)[(2 * LL + 1) * (2 * LL + 1)]) { \
            feq_wmd_l##LL(tv, M);                                                                         \
        }                                                                                                 \
        template <bool kT>                                                                                \
        __device__ __forceinline__ static void wa(const float (&m)[kNnz], const float (&g)[2 * LL + 1],   \
                                                  float (&h)[2 * LL + 1]) {                               \
            feq_wa_l##LL<kT>(m, g, h);                                                                    \
        }                                                                                                 \
    };
FEQ_DEF_WA(1)
FEQ_DEF_WA(2)
FEQ_DEF_WA(3)
FEQ_DEF_WA(4)
FEQ_DEF_WA(5)
FEQ_DEF_WA(6)
#undef FEQ_DEF_WA
static_assert(FEQ_WA_LMAX == 6, "generated per-degree code covers degrees 1..6");
constexpr int kFactoredLmax = 6;

// One irrep of degree Lg for two channels, entirely in registers, through the factored
// block D = R(phi) M R(phi)^T:
//   kT = false: y = x D   = ((x R) M) R^T      (rotate_in:  y[o] = sum_q x[q] D[q][o])
//   kT = true : y = x D^T = ((x R) M^T) R^T    (rotate_out: y[o] = sum_q x[q] D[o][q])
// scaled by sl (folded into M).  tr: the edge's compact trig (tv, cos m phi, sin m phi).
template <int Lg, bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot_irrep2(const float *__restrict__ tr, int lmax, float sl, Get get, Emit emit) {
    constexpr int N = 2 * Lg + 1;
    const float *tv = tr, *cp = tr + 2 * lmax + 1, *sp = cp + lmax + 1;
    float m[WA<Lg>::kNnz];
    WA<Lg>::wm(tv, sl, m);
    float g0[N], g1[N];
#pragma unroll
    for (int q = 0; q < N; q++) {
        const float2 v = get(q);
        g0[q] = v.x;
        g1[q] = v.y;
    }
#pragma unroll
    for (int mm = 1; mm <= Lg; mm++) {      // g <- g R(phi)
        const int a = Lg - mm, b = Lg + mm;
        const float c = cp[mm], s = sp[mm];
        float t0 = g0[a] * c - g0[b] * s, t1 = g0[a] * s + g0[b] * c;
        g0[a] = t0; g0[b] = t1;
        t0 = g1[a] * c - g1[b] * s; t1 = g1[a] * s + g1[b] * c;
        g1[a] = t0; g1[b] = t1;
    }
    float h0[N], h1[N];
    WA<Lg>::template wa<kT>(m, g0, h0);
    WA<Lg>::template wa<kT>(m, g1, h1);
#pragma unroll
    for (int mm = 1; mm <= Lg; mm++) {      // h <- h R(phi)^T
        const int a = Lg - mm, b = Lg + mm;
        const float c = cp[mm], s = sp[mm];
        float t0 = h0[a] * c + h0[b] * s, t1 = h0[b] * c - h0[a] * s;
        h0[a] = t0; h0[b] = t1;
        t0 = h1[a] * c + h1[b] * s; t1 = h1[b] * c - h1[a] * s;
        h1[a] = t0; h1[b] = t1;
    }
#pragma unroll
    for (int o = 0; o < N; o++) emit(o, h0[o], h1[o]);
}

template <bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot_irrep2_any(int l, const float *tr, int lmax, float sl, Get get, Emit emit) {
    switch (l) {
        case 0: {
            const float2 v = get(0);
            emit(0, v.x * sl, v.y * sl);
            break;
        }
        case 1: rot_irrep2<1, kT>(tr, lmax, sl, get, emit); break;
        case 2: rot_irrep2<2, kT>(tr, lmax, sl, get, emit); break;
        case 3: rot_irrep2<3, kT>(tr, lmax, sl, get, emit); break;
        case 4: rot_irrep2<4, kT>(tr, lmax, sl, get, emit); break;
        case 5: rot_irrep2<5, kT>(tr, lmax, sl, get, emit); break;
        default: rot_irrep2<6, kT>(tr, lmax, sl, get, emit); break;
    }
}

}  // namespace rot
}  // namespace feq
