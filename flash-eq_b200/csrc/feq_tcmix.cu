// feq_tcmix.cu -- the distance-binned block-diagonal radial mix on the 5th-gen tensor
// cores (tcgen05 + TMEM, TMA-fed).  Same mathematics as feq_mix.cu / the reference
// forward kernels (flash_eq/cuda/csrc/block_diagonal.cu:558-733).
//
// Formulation.  Edges are sorted by distance bin; a tile is 128 consecutive sorted
// rows of one bin b.  For m-block m the mix is a GEMM over K = (i, re/im, ci) with the
// m > 0 2x2 blocks [[a, b], [-b, a]] embedded as real 2x2 sub-matrices:
//     D_lo = A . B_m(b)^T,   D_hi = A . B_m(b+1)^T      (two TMEM accumulators)
//     out  = D_lo + t_e (D_hi - D_lo)                     (per-row lerp, epilogue)
// A = rotated input rows scaled by s^l_in (bf16), B = re-laid radial table (bf16).
// For float32-level accuracy every operand is split x = hi + lo into two bf16 values
// and D accumulates hi.hi + hi.lo + lo.hi (kSplit = 3): ~16 mantissa bits per product.
//
// Kernel roles (192 threads, persistent, one CTA per SM):
//   warp 0      TMA producer: A tile + B(b) tile + B(b+1) tile per 64-wide K step
//   warp 1      TMEM allocator; one elected thread issues tcgen05.mma
//   warps 2..5  epilogue: tcgen05.ld of both accumulators, lerp, store fp32 rows
// TMEM holds two accumulator pairs (2 x (128 + 128) columns) so the epilogue of one
// work item overlaps the MMAs of the next.  All TMA loads are plain (no multicast).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "feq_internal.cuh"
#include "feq_sm100.cuh"

namespace feq {

using namespace sm100;

constexpr int kTcRows = 128;     // UMMA M (rows = edges)
constexpr int kTcN = 128;        // UMMA N per work item (output columns)
constexpr int kTcK = 64;         // K per stage (one 128-byte swizzle row of bf16)
constexpr int kTcThreads = 192;
constexpr uint32_t kTcTileBytes = kTcRows * kTcK * 2;   // 16 KB (A tile and B tile alike)

struct TcGemmParams {
    int n_tiles_n;          // N_pad(m) / 128
    int k_steps;            // K_pad(m) / 64
    int a_col0;             // first A column of block m
    int npad;               // padded rows of one (bin, block) B matrix
    int n_valid;            // unpadded output columns of block m
    int h_ld;               // row stride of H (all blocks)
    int h_col0;             // first H column of block m
    const int4 *tiles;      // (start, len, bin, -) row tiles of <= 128 sorted rows
    const int *num_tiles;
    const float *tval;      // per sorted row: interpolation weight t
    float *H;               // (E, h_ld) sorted rows
    float *Hd;              // optional, same layout: D_hi - D_lo (the t-derivative of H)
    int32_t *status;        // set to 2 when a wait timed out
    uint64_t wait_ns;       // limit of each pipeline wait (wait_limit_ns())
};

template <int kSplit>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_mix_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapA2,
              const __grid_constant__ CUtensorMap mapB, const __grid_constant__ CUtensorMap mapB2,
              const __grid_constant__ TcGemmParams P) {
    constexpr int kTiles = kSplit == 1 ? 3 : 6;      // A, B(b), B(b+1) [, A.lo, B(b).lo, B(b+1).lo]
    constexpr int kStages = kSplit == 1 ? 4 : 2;
    constexpr uint32_t kStageBytes = kTiles * kTcTileBytes;
    constexpr uint32_t kIdesc = idesc_bf16_f32(kTcRows, 2 * kTcN);   // D_lo | D_hi

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full_bar[kStages], empty_bar[kStages], tfull_bar[2], tempty_bar[2], drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], 128);
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&mapA);
        prefetch_tmap(&mapB);
        if (kSplit == 3) {
            prefetch_tmap(&mapA2);
            prefetch_tmap(&mapB2);
        }
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    const int n_items = *P.num_tiles * P.n_tiles_n;
    volatile int *abort_flag = &abort_s;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        int it = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x) {
            const int tile = item / P.n_tiles_n, nt = item - tile * P.n_tiles_n;
            const int4 T = P.tiles[tile];
            const int rb0 = T.z * P.npad + nt * kTcN, rb1 = rb0 + P.npad;
            for (int ks = 0; ks < P.k_steps; ks++, it++) {
                const int s = it % kStages, r = it / kStages;
                if (r > 0 && !mbar_wait(&empty_bar[s], (r - 1) & 1, abort_flag, P.wait_ns)) break;
                uint8_t *base = smem + (size_t)s * kStageBytes;
                mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
                const int ax = P.a_col0 + ks * kTcK, bx = ks * kTcK;
                tma_load_2d(base, &mapA, ax, T.x, &full_bar[s]);
                tma_load_2d(base + kTcTileBytes, &mapB, bx, rb0, &full_bar[s]);
                tma_load_2d(base + 2 * kTcTileBytes, &mapB, bx, rb1, &full_bar[s]);
                if (kSplit == 3) {
                    tma_load_2d(base + 3 * kTcTileBytes, &mapA2, ax, T.x, &full_bar[s]);
                    tma_load_2d(base + 4 * kTcTileBytes, &mapB2, bx, rb0, &full_bar[s]);
                    tma_load_2d(base + 5 * kTcTileBytes, &mapB2, bx, rb1, &full_bar[s]);
                }
            }
        }
        // drain: the last loads of every stage must have landed before the CTA exits
        for (int k = max(0, it - kStages); k < it; k++) mbar_wait_drain(&full_bar[k % kStages], (k / kStages) & 1);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        int it = 0, j = 0;
        for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, j++) {
            const int buf = j & 1, rr = j >> 1;
            if (rr > 0 && !mbar_wait(&tempty_bar[buf], (rr - 1) & 1, abort_flag, P.wait_ns)) break;
            tc_fence_after();
            const uint32_t d_lo = tmem + buf * 2 * kTcN;
            bool ok = true;
            for (int ks = 0; ks < P.k_steps; ks++, it++) {
                const int s = it % kStages, r = it / kStages;
                if (!mbar_wait(&full_bar[s], r & 1, abort_flag, P.wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t base = smem_u32(smem + (size_t)s * kStageBytes);
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; kk++) {
                    // B(b) and B(b+1) tiles are adjacent in shared memory: one N = 256 MMA
                    // writes D_lo (columns 0..127) and D_hi (columns 128..255) together.
                    const uint32_t koff = kk * 32;   // 16 bf16 = 32 bytes along K
                    const uint64_t a = smem_desc_sw128(base + koff);
                    const uint64_t b = smem_desc_sw128(base + kTcTileBytes + koff);
                    const uint32_t acc = (ks > 0 || kk > 0) ? 1u : 0u;
                    umma_f16(d_lo, a, b, kIdesc, acc);
                    if (kSplit == 3) {
                        const uint64_t a2 = smem_desc_sw128(base + 3 * kTcTileBytes + koff);
                        const uint64_t b2 = smem_desc_sw128(base + 4 * kTcTileBytes + koff);
                        umma_f16(d_lo, a, b2, kIdesc, 1u);
                        umma_f16(d_lo, a2, b, kIdesc, 1u);
                    }
                }
                umma_commit(&empty_bar[s]);   // stage s is free once these MMAs finish
            }
            if (!ok) break;
            umma_commit(&tfull_bar[buf]);
        }
        // drain: every MMA issued above must complete before TMEM is released
        umma_commit(&drain_bar);
        mbar_wait_drain(&drain_bar, 0);
    } else if (warp >= 2) {
        // ---------------- epilogue ----------------
        const int q = warp & 3;                 // TMEM lane quadrant this warp may access
        const int row = q * 32 + lane;
        const bool vec4 = ((P.h_ld | P.h_col0 | P.n_valid) & 3) == 0;
        int j = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, j++) {
            const int buf = j & 1, rr = j >> 1;
            if (!mbar_wait(&tfull_bar[buf], rr & 1, abort_flag, P.wait_ns)) break;
            tc_fence_after();
            const int tile = item / P.n_tiles_n, nt = item - tile * P.n_tiles_n;
            const int4 T = P.tiles[tile];
            const bool valid = row < T.y;
            const int64_t p = (int64_t)T.x + row;
            const float t = valid ? P.tval[p] : 0.0f;
            const uint32_t t_lo = tmem + ((uint32_t)(q * 32) << 16) + buf * 2 * kTcN, t_hi = t_lo + kTcN;
            float *hrow = P.H + p * P.h_ld + P.h_col0;
#pragma unroll 1
            for (int c0 = 0; c0 < kTcN; c0 += 32) {
                uint32_t lo[32], hi[32];
                tmem_ld32(t_lo + c0, lo);
                tmem_ld32(t_hi + c0, hi);
                tmem_wait_ld();
                const int n0 = nt * kTcN + c0;
                if (valid) {
                    if (vec4 && n0 + 32 <= P.n_valid) {
#pragma unroll
                        for (int c = 0; c < 32; c += 4) {
                            float4 v;
                            v.x = fmaf(t, __uint_as_float(hi[c]) - __uint_as_float(lo[c]), __uint_as_float(lo[c]));
                            v.y = fmaf(t, __uint_as_float(hi[c + 1]) - __uint_as_float(lo[c + 1]), __uint_as_float(lo[c + 1]));
                            v.z = fmaf(t, __uint_as_float(hi[c + 2]) - __uint_as_float(lo[c + 2]), __uint_as_float(lo[c + 2]));
                            v.w = fmaf(t, __uint_as_float(hi[c + 3]) - __uint_as_float(lo[c + 3]), __uint_as_float(lo[c + 3]));
                            *reinterpret_cast<float4 *>(hrow + n0 + c) = v;
                            if (P.Hd) {
                                float4 dv;
                                dv.x = __uint_as_float(hi[c]) - __uint_as_float(lo[c]);
                                dv.y = __uint_as_float(hi[c + 1]) - __uint_as_float(lo[c + 1]);
                                dv.z = __uint_as_float(hi[c + 2]) - __uint_as_float(lo[c + 2]);
                                dv.w = __uint_as_float(hi[c + 3]) - __uint_as_float(lo[c + 3]);
                                *reinterpret_cast<float4 *>(P.Hd + p * P.h_ld + P.h_col0 + n0 + c) = dv;
                            }
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < 32; c++) {
                            if (n0 + c < P.n_valid) {
                                const float l = __uint_as_float(lo[c]), h = __uint_as_float(hi[c]);
                                hrow[n0 + c] = fmaf(t, h - l, l);
                                if (P.Hd) P.Hd[p * P.h_ld + P.h_col0 + n0 + c] = h - l;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty_bar[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && abort_s && P.status) atomicMax(P.status, 2);
}

// ---------------------------------------------------------------------------
// Per-bin weight-gradient reduction of the backward on the tensor cores:
//   dB_b[n][k] = sum_{p in bin b} (1 - t_p) G[p][n] A[p][k] + sum_{p in bin b-1} t_p G[p][n] A[p][k]
// The reduction runs over edges, so both operands are the transposes Gt[n][p'], At[k][p']
// (K-major over the padded sorted position p': every bin's segment starts at a multiple of
// 64, gaps are zero), with the weights folded into two copies of Gt.  Work item =
// (m-block, bin, 128 n rows, 128 k columns); roles as in tc_mix_kernel.
// ---------------------------------------------------------------------------
struct TcGramParams {
    int n_blocks, nb;
    int64_t n_items;
    TcGramBlock blk[kMaxBlocks];
    const int64_t *seg;     // (nb + 1,) padded segment starts, seg[nb] = end
    float *dB;
    int32_t *status;
    uint64_t wait_ns;       // limit of each pipeline wait (wait_limit_ns())
};

struct GramItem {
    int m, b, nt, kt, s0, s1;
    int64_t x0, x1;         // first p' of the lo segment (bin b) and of the hi segment (bin b - 1)
};

__device__ __forceinline__ GramItem gram_item(const TcGramParams &P, int64_t item) {
    GramItem g;
    int m = 0;
    while (m + 1 < P.n_blocks && P.blk[m + 1].item0 <= item) m++;
    const TcGramBlock &B = P.blk[m];
    const int64_t loc = item - B.item0, per_bin = (int64_t)B.n_tiles * B.k_tiles;
    g.m = m;
    g.b = (int)(loc / per_bin);
    const int r = (int)(loc - g.b * per_bin);
    g.nt = r / B.k_tiles;
    g.kt = r - g.nt * B.k_tiles;
    g.s0 = g.b < P.nb ? (int)((P.seg[g.b + 1] - P.seg[g.b]) / kTcK) : 0;
    g.s1 = g.b >= 1 ? (int)((P.seg[g.b] - P.seg[g.b - 1]) / kTcK) : 0;
    g.x0 = g.b < P.nb ? P.seg[g.b] : 0;
    g.x1 = g.b >= 1 ? P.seg[g.b - 1] : 0;
    return g;
}

template <int kSplit>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gram_kernel(const __grid_constant__ CUtensorMap mG0, const __grid_constant__ CUtensorMap mG0l,
               const __grid_constant__ CUtensorMap mG1, const __grid_constant__ CUtensorMap mG1l,
               const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mAl,
               const __grid_constant__ TcGramParams P) {
    constexpr int kTiles = kSplit == 1 ? 2 : 4;      // Gt, At [, Gt.lo, At.lo]
    constexpr int kStages = kSplit == 1 ? 6 : 3;
    constexpr uint32_t kStageBytes = kTiles * kTcTileBytes;
    constexpr uint32_t kIdesc = idesc_bf16_f32(kTcRows, kTcN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full_bar[kStages], empty_bar[kStages], tfull_bar[2], tempty_bar[2], drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], 128);
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&mG0);
        prefetch_tmap(&mG1);
        prefetch_tmap(&mA);
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    volatile int *abort_flag = &abort_s;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        int it = 0;
        for (int64_t item = blockIdx.x; item < P.n_items && !*abort_flag; item += gridDim.x) {
            const GramItem g = gram_item(P, item);
            const TcGramBlock &B = P.blk[g.m];
            const int gy = B.g_row0 + g.nt * kTcRows, ay = B.a_row0 + g.kt * kTcRows;
            bool ok = true;
            for (int ks = 0; ks < g.s0 + g.s1; ks++, it++) {
                const int s = it % kStages, r = it / kStages;
                if (r > 0 && !mbar_wait(&empty_bar[s], (r - 1) & 1, abort_flag, P.wait_ns)) {
                    ok = false;
                    break;
                }
                uint8_t *base = smem + (size_t)s * kStageBytes;
                const bool lo_seg = ks < g.s0;
                const int x = (int)(lo_seg ? g.x0 + (int64_t)ks * kTcK : g.x1 + (int64_t)(ks - g.s0) * kTcK);
                mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
                tma_load_2d(base, lo_seg ? &mG0 : &mG1, x, gy, &full_bar[s]);
                tma_load_2d(base + kTcTileBytes, &mA, x, ay, &full_bar[s]);
                if (kSplit == 3) {
                    tma_load_2d(base + 2 * kTcTileBytes, lo_seg ? &mG0l : &mG1l, x, gy, &full_bar[s]);
                    tma_load_2d(base + 3 * kTcTileBytes, &mAl, x, ay, &full_bar[s]);
                }
            }
            if (!ok) break;
        }
        for (int k = max(0, it - kStages); k < it; k++) mbar_wait_drain(&full_bar[k % kStages], (k / kStages) & 1);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        int it = 0, j = 0;
        for (int64_t item = blockIdx.x; item < P.n_items && !*abort_flag; item += gridDim.x, j++) {
            const GramItem g = gram_item(P, item);
            const int buf = j & 1, rr = j >> 1;
            if (rr > 0 && !mbar_wait(&tempty_bar[buf], (rr - 1) & 1, abort_flag, P.wait_ns)) break;
            tc_fence_after();
            const uint32_t d = tmem + buf * kTcN;
            bool ok = true;
            for (int ks = 0; ks < g.s0 + g.s1; ks++, it++) {
                const int s = it % kStages, r = it / kStages;
                if (!mbar_wait(&full_bar[s], r & 1, abort_flag, P.wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t base = smem_u32(smem + (size_t)s * kStageBytes);
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; kk++) {
                    const uint32_t koff = kk * 32;
                    const uint64_t a = smem_desc_sw128(base + koff);
                    const uint64_t b = smem_desc_sw128(base + kTcTileBytes + koff);
                    umma_f16(d, a, b, kIdesc, (ks > 0 || kk > 0) ? 1u : 0u);
                    if (kSplit == 3) {
                        const uint64_t a2 = smem_desc_sw128(base + 2 * kTcTileBytes + koff);
                        const uint64_t b2 = smem_desc_sw128(base + 3 * kTcTileBytes + koff);
                        umma_f16(d, a, b2, kIdesc, 1u);
                        umma_f16(d, a2, b, kIdesc, 1u);
                    }
                }
                umma_commit(&empty_bar[s]);
            }
            if (!ok) break;
            umma_commit(&tfull_bar[buf]);     // also for an item without steps: the epilogue writes zeros
        }
        umma_commit(&drain_bar);
        mbar_wait_drain(&drain_bar, 0);
    } else if (warp >= 2) {
        // ---------------- epilogue ----------------
        const int q = warp & 3;
        const int row = q * 32 + lane;         // n within the tile
        int j = 0;
        for (int64_t item = blockIdx.x; item < P.n_items; item += gridDim.x, j++) {
            const int buf = j & 1, rr = j >> 1;
            if (!mbar_wait(&tfull_bar[buf], rr & 1, abort_flag, P.wait_ns)) break;
            tc_fence_after();
            const GramItem g = gram_item(P, item);
            const TcGramBlock &B = P.blk[g.m];
            const int n = g.nt * kTcRows + row;
            const bool empty = g.s0 + g.s1 == 0;
            float *drow = P.dB + B.dboff + ((int64_t)g.b * B.N + n) * B.K;
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + buf * kTcN;
#pragma unroll 1
            for (int c0 = 0; c0 < kTcN; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                tmem_wait_ld();
                const int k0 = g.kt * kTcN + c0;
                if (n < B.N) {
#pragma unroll
                    for (int c = 0; c < 32; c++)
                        if (k0 + c < B.K) drow[k0 + c] = empty ? 0.0f : __uint_as_float(v[c]);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty_bar[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
    if (threadIdx.x == 0 && abort_s && P.status) atomicMax(P.status, 2);
}

// B operand: per block m and bin b a (npad x kpad) K-major bf16 matrix (rows = output
// columns n = (o, re/im, co), cols = k = (i, re/im, ci); channel fastest), zero padded; the m > 0 2x2
// blocks are written as [[a, b], [-b, a]].  With a second buffer the float32 weight is
// split hi + lo.
__global__ void tc_relayout_b_kernel(const float *__restrict__ T, __nv_bfloat16 *__restrict__ Bhi,
                                     __nv_bfloat16 *__restrict__ Blo, int nb1, int Cin, int Cout, int wdim,
                                     const __grid_constant__ TcGeom G, int64_t total) {
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int q = 0;
        while (q + 1 < G.n_blocks && G.g[q + 1].boff <= idx) q++;
        const TcBlockGeom &B = G.g[q];
        const int64_t r = idx - B.boff;
        const int64_t rowi = r / B.kpad;
        const int k = (int)(r - rowi * B.kpad);
        const int b = (int)(rowi / B.npad);
        const int n = (int)(rowi - (int64_t)b * B.npad);
        float v = 0.0f;
        const int kin = B.mult * B.n_in, kout = B.mult * B.n_out;
        if (B.n_in > 0 && B.n_out > 0 && b < nb1 && n < Cout * kout && k < Cin * kin) {
            // channel fastest: n = (o * mult + oc) * Cout + co, k = (i * mult + ic) * Cin + ci
            const int co = n % Cout, rn = n / Cout, o = rn / B.mult, oc = rn - o * B.mult;
            const int ci = k % Cin, rk = k / Cin, i = rk / B.mult, ic = rk - i * B.mult;
            const float *w = T + ((int64_t)(b * Cout + co) * Cin + ci) * wdim + B.w_off;
            if (B.mult == 1) {
                v = __ldg(w + o * B.n_in + i);
            } else {
                const float a = __ldg(w + 2 * (o * B.n_in + i)), bb = __ldg(w + 2 * (o * B.n_in + i) + 1);
                v = (oc == ic) ? a : (oc == 0 ? bb : -bb);   // (re,im) -> b, (im,re) -> -b
            }
        }
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        Bhi[idx] = hi;
        if (Blo) Blo[idx] = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
}

// Same layout, one block per (output channel co, bin b): the block's weights
// T[b][co][:][:] (Cin x wdim floats, contiguous) are staged in shared memory with
// coalesced loads, then every B row of that channel is written with consecutive
// threads on consecutive k (input channel fastest).  Blocks with co = 0 also zero the
// N-padding rows of their bin.
__global__ void tc_relayout_b_rows_kernel(const float *__restrict__ T, __nv_bfloat16 *__restrict__ Bhi,
                                          __nv_bfloat16 *__restrict__ Blo, int Cin, int Cout, int wdim,
                                          const __grid_constant__ TcGeom G) {
    extern __shared__ float tw[];
    const int co = blockIdx.x, b = blockIdx.y;
    const int64_t slice = (int64_t)Cin * wdim;
    const float *src = T + ((int64_t)b * Cout + co) * slice;
    if ((slice & 3) == 0 && (reinterpret_cast<uintptr_t>(T) & 15) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        for (int64_t i = threadIdx.x; i < slice / 4; i += blockDim.x) reinterpret_cast<float4 *>(tw)[i] = __ldg(s4 + i);
    } else {
        for (int64_t i = threadIdx.x; i < slice; i += blockDim.x) tw[i] = __ldg(src + i);
    }
    __syncthreads();
    for (int q = 0; q < G.n_blocks; q++) {
        const TcBlockGeom &B = G.g[q];
        const int kin = B.mult * B.n_in, kout = B.mult * B.n_out;
        const int kvalid = (B.n_in > 0 && B.n_out > 0) ? Cin * kin : 0;
        const int nreal = Cout * kout;
        const int nq = Cin >> 2;
        auto row_ptrs = [&](int n, __nv_bfloat16 *&rh, __nv_bfloat16 *&rl) {
            rh = Bhi + B.boff + ((int64_t)b * B.npad + n) * B.kpad;
            rl = Blo ? Blo + B.boff + ((int64_t)b * B.npad + n) * B.kpad : nullptr;
        };
        auto put4 = [&](__nv_bfloat16 *rh, __nv_bfloat16 *rl, int k0, const float (&v)[4]) {
            const __nv_bfloat162 h01 = __floats2bfloat162_rn(v[0], v[1]), h23 = __floats2bfloat162_rn(v[2], v[3]);
            uint2 hv;
            hv.x = *reinterpret_cast<const uint32_t *>(&h01);
            hv.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(rh + k0) = hv;
            if (rl) {
                const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
                const __nv_bfloat162 l01 = __floats2bfloat162_rn(v[0] - f01.x, v[1] - f01.y);
                const __nv_bfloat162 l23 = __floats2bfloat162_rn(v[2] - f23.x, v[3] - f23.y);
                uint2 lv;
                lv.x = *reinterpret_cast<const uint32_t *>(&l01);
                lv.y = *reinterpret_cast<const uint32_t *>(&l23);
                *reinterpret_cast<uint2 *>(rl + k0) = lv;
            }
        };
        // real rows rr * Cout + co: items (rr, rk, cq) = 4 input channels 4cq..4cq+3 of K row rk
        if (kvalid > 0) {
            const int items = kout * kin * nq;
            for (int it = threadIdx.x; it < items; it += blockDim.x) {
                const int cq = it % nq, t = it / nq, rk = t % kin, rr = t / kin;
                const int o = rr / B.mult, oc = rr - o * B.mult, i = rk / B.mult, ic = rk - i * B.mult;
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const float *w = tw + (4 * cq + u) * wdim + B.w_off;
                    if (B.mult == 1) {
                        v[u] = w[o * B.n_in + i];
                    } else {
                        const float a = w[2 * (o * B.n_in + i)], bb = w[2 * (o * B.n_in + i) + 1];
                        v[u] = (oc == ic) ? a : (oc == 0 ? bb : -bb);   // (re,im) -> b, (im,re) -> -b
                    }
                }
                __nv_bfloat16 *rh, *rl;
                row_ptrs(rr * Cout + co, rh, rl);
                put4(rh, rl, rk * Cin + 4 * cq, v);
            }
        }
        // zeros: K padding of the real rows, and (co == 0) the N padding rows
        const float z4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const int kz = B.kpad - kvalid;           // multiple of 4
        if (kvalid > 0 && kz > 0) {
            const int zq = kz >> 2;
            for (int it = threadIdx.x; it < kout * zq; it += blockDim.x) {
                const int rr = it / zq, k0 = kvalid + 4 * (it - rr * zq);
                __nv_bfloat16 *rh, *rl;
                row_ptrs(rr * Cout + co, rh, rl);
                put4(rh, rl, k0, z4);
            }
        }
        const int zrows = (kvalid > 0 ? 0 : kout) + (co == 0 ? B.npad - nreal : 0);
        for (int it = threadIdx.x; it < zrows * (B.kpad >> 2); it += blockDim.x) {
            const int zr = it / (B.kpad >> 2), k0 = 4 * (it - zr * (B.kpad >> 2));
            const int n = (kvalid > 0 || zr >= kout) ? nreal + (zr - (kvalid > 0 ? 0 : kout)) : zr * Cout + co;
            __nv_bfloat16 *rh, *rl;
            row_ptrs(n, rh, rl);
            put4(rh, rl, k0, z4);
        }
    }
}

// ---------------------------------------------------------------------------
// Host
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2D bf16 K-major tensor (inner = cols), box 64 x 128, 128-byte swizzle, zero OOB fill.
static int make_map(CUtensorMap *m, const void *base, int64_t cols, int64_t rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return FEQ_ERR_CUDA;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16) return FEQ_ERR_INVALID_ARGUMENT;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {(cuuint32_t)kTcK, (cuuint32_t)kTcRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FEQ_OK : FEQ_ERR_INVALID_ARGUMENT;
}

int launch_tc_relayout_b(const float *T, __nv_bfloat16 *Bhi, __nv_bfloat16 *Blo, int nb1, int Cin, int Cout,
                         int wdim, const TcGeom &G, int64_t total, cudaStream_t s) {
    if (total == 0) return FEQ_OK;
    const size_t smem = (size_t)Cin * wdim * 4;
    if (smem <= 96 * 1024 && Cout <= 65535 && nb1 <= 65535 && Cin % 4 == 0 && Cin / 4 <= 256) {
        if (smem > 48 * 1024)
            FEQ_CUDA_TRY(cudaFuncSetAttribute(tc_relayout_b_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem));
        tc_relayout_b_rows_kernel<<<dim3((unsigned)Cout, (unsigned)nb1), 256, smem, s>>>(T, Bhi, Blo, Cin, Cout,
                                                                                       wdim, G);
        FEQ_LAUNCH_CHECK();
        return FEQ_OK;
    }
    const int64_t grid = min64((total + 255) / 256, 148 * 32);
    tc_relayout_b_kernel<<<(unsigned)grid, 256, 0, s>>>(T, Bhi, Blo, nb1, Cin, Cout, wdim, G, total);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// One persistent launch per m-block.
int launch_tc_mix(int split, const __nv_bfloat16 *A, const __nv_bfloat16 *A2, int64_t a_rows, int a_cols,
                  const __nv_bfloat16 *Bm, const __nv_bfloat16 *Bm2, int64_t b_rows, const TcBlockGeom &B,
                  int a_col0, int n_valid, int h_ld, int h_col0, const int4 *tiles, const int *num_tiles,
                  int64_t max_tiles, const float *tval, float *H, int32_t *status, cudaStream_t s, float *Hd) {
    CUtensorMap mA, mA2, mB, mB2;
    int rc;
    if ((rc = make_map(&mA, A, a_cols, a_rows)) != FEQ_OK) return rc;
    if ((rc = make_map(&mB, Bm, B.kpad, b_rows)) != FEQ_OK) return rc;
    if (split == 3) {
        if ((rc = make_map(&mA2, A2, a_cols, a_rows)) != FEQ_OK) return rc;
        if ((rc = make_map(&mB2, Bm2, B.kpad, b_rows)) != FEQ_OK) return rc;
    } else {
        mA2 = mA;
        mB2 = mB;
    }
    TcGemmParams P;
    P.n_tiles_n = B.npad / kTcN;
    P.k_steps = B.kpad / kTcK;
    P.a_col0 = a_col0;
    P.npad = B.npad;
    P.n_valid = n_valid;
    P.h_ld = h_ld;
    P.h_col0 = h_col0;
    P.tiles = tiles;
    P.num_tiles = num_tiles;
    P.tval = tval;
    P.H = H;
    P.Hd = Hd;
    P.status = status;
    P.wait_ns = wait_limit_ns();
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t items = max_tiles * P.n_tiles_n;
    const int grid = (int)min64(sms, max64(items, 1));
    const size_t smem = (size_t)(split == 1 ? 4 * 3 : 2 * 6) * kTcTileBytes + 1024;
    if (split == 1) {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(tc_mix_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        tc_mix_kernel<1><<<grid, kTcThreads, smem, s>>>(mA, mA2, mB, mB2, P);
    } else {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(tc_mix_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        tc_mix_kernel<3><<<grid, kTcThreads, smem, s>>>(mA, mA2, mB, mB2, P);
    }
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq

namespace feq {

// Per-bin gradient reduction (see tc_gram_kernel).  Gt0 / Gt1: (1 - t) and t weighted
// transposes of G (g_rows x p_cols), At: transpose of A (a_rows x p_cols); blk[m] holds the
// block geometry (item0 is filled here); seg: device (nb + 1,) segment starts.
int launch_tc_gram(int split, const __nv_bfloat16 *Gt0, const __nv_bfloat16 *Gt0l, const __nv_bfloat16 *Gt1,
                   const __nv_bfloat16 *Gt1l, int64_t g_rows, const __nv_bfloat16 *At, const __nv_bfloat16 *Atl,
                   int64_t a_rows, int64_t p_cols, int n_blocks, const TcGramBlock *blk, int nb, const int64_t *seg,
                   float *dB, int32_t *status, cudaStream_t s) {
    TcGramParams P;
    memset(&P, 0, sizeof(P));
    P.n_blocks = n_blocks;
    P.nb = nb;
    int64_t items = 0;
    for (int m = 0; m < n_blocks; m++) {
        P.blk[m] = blk[m];
        P.blk[m].item0 = items;
        items += (int64_t)(nb + 1) * blk[m].n_tiles * blk[m].k_tiles;
    }
    P.n_items = items;
    P.seg = seg;
    P.dB = dB;
    P.status = status;
    P.wait_ns = wait_limit_ns();
    if (items == 0) return FEQ_OK;
    CUtensorMap m0, m0l, m1, m1l, ma, mal;
    int rc;
    if ((rc = make_map(&m0, Gt0, p_cols, g_rows)) != FEQ_OK) return rc;
    if ((rc = make_map(&m1, Gt1, p_cols, g_rows)) != FEQ_OK) return rc;
    if ((rc = make_map(&ma, At, p_cols, a_rows)) != FEQ_OK) return rc;
    if (split == 3) {
        if ((rc = make_map(&m0l, Gt0l, p_cols, g_rows)) != FEQ_OK) return rc;
        if ((rc = make_map(&m1l, Gt1l, p_cols, g_rows)) != FEQ_OK) return rc;
        if ((rc = make_map(&mal, Atl, p_cols, a_rows)) != FEQ_OK) return rc;
    } else {
        m0l = m0;
        m1l = m1;
        mal = ma;
    }
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = (int)min64(sms, items);
    const size_t smem = (size_t)(split == 1 ? 6 * 2 : 3 * 4) * kTcTileBytes + 1024;
    if (split == 1) {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(tc_gram_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        tc_gram_kernel<1><<<grid, kTcThreads, smem, s>>>(m0, m0l, m1, m1l, ma, mal, P);
    } else {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(tc_gram_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        tc_gram_kernel<3><<<grid, kTcThreads, smem, s>>>(m0, m0l, m1, m1l, ma, mal, P);
    }
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
