// feq_mixout.cu -- the radial mix and the rotation back out of the edge frame in one
// persistent tensor-core kernel (bf16 mix), for representations whose A rows of a
// 128-edge tile fit in shared memory.
//
// Reference behaviour replaced: the second half of EquivariantEdgewiseLinear.forward
// (flash_eq/layers/linear.py:100-160): block_diagonal_cuda (block_diagonal.cu:558-733)
// followed by bmm(., Q^T).  The input side (gather, rotation into the edge frame, bf16 A
// rows) is rot_in_kernel (feq_rotate_tc.cu); this kernel replaces tc_mix_kernel + the
// fp32 H round trip + rot_out_kernel.
//
// Per tile of <= 128 sorted edges of one distance bin:
//   warp 0 (A loader)    TMA-loads the tile's whole A block (all K chunks) once;
//   warp 1 (B loader)    TMA-loads, per 8-output-channel chunk and m-block, the weight rows
//                        of bins b and b+1 (adjacent rows, one box) through a ring;
//   warp 2 (MMA)         tcgen05.mma M = 128, N = both bins, one TMEM buffer per chunk
//                        (three buffers, so chunk q+1..q+2 overlap chunk q's epilogue);
//   warps 3..10 (epilogue) two warps per TMEM lane quadrant, thread = edge (its TMEM lane)
//                        and 4 of the chunk's 8 channels: lerp the two bins, rotate back out
//                        of the edge frame in registers (the edge's trig and scaled M blocks
//                        computed once per tile), stage the 4 channels of the output row in
//                        shared memory; each warp then writes its 32 row parts to the edges'
//                        original rows with coalesced stores.
// HBM traffic per edge: the A row (bf16) and the output row (fp32); weight tiles come from
// L2.  All waits are bounded; no TMA multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>

#include "feq_internal.cuh"
#include "feq_rot_common.cuh"
#include "feq_sm100.cuh"

namespace feq {

int tc_make_map_box(CUtensorMap *m, const void *base, int64_t cols, int64_t rows, int box_rows);
int tc_make_map_a(CUtensorMap *m, const void *base, int64_t cols, int64_t rows);

namespace {

using namespace sm100;
using namespace rot;

constexpr int kMoThreads = 352;     // A loader, B loader, MMA, 8 epilogue warps
constexpr int kMoEpiWarp0 = 3;
constexpr int kMoEpiThreads = 256;  // two warps per TMEM lane quadrant, 4 channels of a chunk each
constexpr int kMoCC = 8;            // output channels per TMEM chunk
constexpr int kMoEC = 4;            // output channels per epilogue thread and chunk
constexpr int kMoMaxBlocks = 5;     // m-blocks (output lmax <= 4)
constexpr int kMoMaxStages = 8;
constexpr int kMoTrigL = 4;        // highest output degree
constexpr int kMoMaxOut = 32;       // output positions
constexpr int kMoStT = 33;          // staging stride between a lane's values (conflict-free banks)

struct MoBlock {
    int kc0, kc;          // first 64-column chunk of the block in the A row, and count
    int R;                // weight rows per bin per channel chunk: n_out * mult * 8
    int col;              // TMEM column of the block inside a chunk buffer
};

struct MoParams {
    int n_blocks, nq, nb1, cols_per_chunk, n_kc, n_bufs, n_stages;
    uint32_t stage_bytes;       // 2 bins x max R rows x 128 B, multiple of 1024
    int stage_stride;           // floats per epilogue warp in the output staging area
    int16_t out_col[kMoMaxOut]; // std output position -> TMEM column of bin lo (channel 0) in a chunk
    int16_t out_R[kMoMaxOut];   // ... and the offset of bin hi
    int n_irr_out;
    int8_t irr_out_l[kMoMaxOut];
    int8_t irr_out_off[kMoMaxOut];
    MoBlock blk[kMoMaxBlocks];
    int C_out, d_out;
    const float *dirs, *dist, *tval;
    const int64_t *perm;
    const int4 *tiles;
    const int *num_tiles;
    float sh_scale;
    float *out;                 // (E, C_out, d_out)
    int32_t *status;
};

struct MoSmem {
    uint32_t a, b, st, ro, total;
};
// stage_stride: floats of one epilogue warp's staging area
__host__ __device__ inline MoSmem mo_smem(int n_kc, int n_stages, uint32_t stage_bytes, int stage_stride) {
    MoSmem m;
    m.a = 0;
    m.b = (uint32_t)n_kc * 16384u;
    m.st = m.b + (uint32_t)n_stages * stage_bytes;
    m.ro = m.st + (uint32_t)(kMoEpiThreads / 32) * (uint32_t)stage_stride * 4u;
    m.ro = (m.ro + 15u) & ~15u;
    m.total = m.ro + (uint32_t)kMoEpiThreads * 8u;
    return m;
}

// Per-edge rotation constants of the epilogue: cos / sin(m phi) and, per degree l <= Lm,
// the scaled sparse M block s^l M_l(theta) (computed once per edge and tile).
template <int Lm>
struct MoEdge {
    float cp[Lm + 1], sp[Lm + 1];
    float m1[WA<1>::kNnz];
    float m2[Lm >= 2 ? WA<2>::kNnz : 1];
    float m3[Lm >= 3 ? WA<3>::kNnz : 1];
    float m4[Lm >= 4 ? WA<4>::kNnz : 1];
};

template <int Lm>
__device__ __forceinline__ void mo_edge_setup(const float *dir, float s, MoEdge<Lm> &E) {
    float tr[trig_floats(Lm)];
    edge_trig_compact(dir[0], dir[1], dir[2], Lm, tr);
    const float *tv = tr, *cp = tr + 2 * Lm + 1, *sp = cp + Lm + 1;
#pragma unroll
    for (int m = 0; m <= Lm; m++) {
        E.cp[m] = cp[m];
        E.sp[m] = sp[m];
    }
    WA<1>::wm(tv, s, E.m1);
    if constexpr (Lm >= 2) WA<2>::wm(tv, s * s, E.m2);
    if constexpr (Lm >= 3) WA<3>::wm(tv, s * s * s, E.m3);
    if constexpr (Lm >= 4) WA<4>::wm(tv, (s * s) * (s * s), E.m4);
}

template <int Lg, int Lm>
__device__ __forceinline__ const float (&mo_m(const MoEdge<Lm> &E))[WA<Lg>::kNnz] {
    if constexpr (Lg == 1) return E.m1;
    else if constexpr (Lg == 2) return E.m2;
    else if constexpr (Lg == 3) return E.m3;
    else return E.m4;
}

// One output irrep of degree Lg, this thread's 4 channels of a chunk: read bins lo / hi of
// every position (one 4-column TMEM load each), lerp with t, rotate back two channels at a
// time and write the results into this lane's column of the warp's staging area: value x
// of the lane's output row part (channel-major, d_out per channel) at st[x * kMoStT].
template <int Lg, int Lm>
__device__ __forceinline__ void mo_epi_irrep(const MoParams &P, uint32_t tbuf, int off, const MoEdge<Lm> &E,
                                             float t, float *st) {
    constexpr int N = 2 * Lg + 1;
    float h[N][kMoEC];
    uint32_t lo[N][kMoEC], hi[N][kMoEC];
#pragma unroll
    for (int i = 0; i < N; i++) {
        const int col = P.out_col[off + i];
        const uint32_t c0 = col < 0 ? 0u : (uint32_t)col;
        tmem_ld4(tbuf + c0, lo[i]);
        tmem_ld4(tbuf + c0 + (uint32_t)(col < 0 ? 0 : P.out_R[off + i]), hi[i]);
    }
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < N; i++) {
        const bool z = P.out_col[off + i] < 0;
#pragma unroll
        for (int c = 0; c < kMoEC; c++) {
            const float a = __uint_as_float(lo[i][c]), b = __uint_as_float(hi[i][c]);
            h[i][c] = z ? 0.0f : fmaf(t, b - a, a);
        }
    }
    const int dout = P.d_out;
#pragma unroll
    for (int c = 0; c < kMoEC; c += 2) {
        float *o0 = st + (c * dout + off) * kMoStT, *o1 = o0 + dout * kMoStT;
        auto get = [&](int i) { return make_float2(h[i][c], h[i][c + 1]); };
        auto emit = [&](int o, float y0, float y1) {
            o0[o * kMoStT] = y0;
            o1[o * kMoStT] = y1;
        };
        if constexpr (Lg == 0)
            emit(0, h[0][c], h[0][c + 1]);
        else
            rot_irrep2_pre<Lg, true>(mo_m<Lg, Lm>(E), E.cp, E.sp, get, emit);
    }
}

template <int Lm>
__global__ void __launch_bounds__(kMoThreads, 1)
tc_mix_out_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mB0,
                  const __grid_constant__ CUtensorMap mB1, const __grid_constant__ CUtensorMap mB2,
                  const __grid_constant__ CUtensorMap mB3, const __grid_constant__ CUtensorMap mB4,
                  const __grid_constant__ MoParams P) {
    extern __shared__ uint8_t msm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(msm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t a_full, a_empty, b_full[kMoMaxStages], b_empty[kMoMaxStages], t_full[4], t_empty[4];
    __shared__ uint64_t drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const MoSmem L = mo_smem(P.n_kc, P.n_stages, P.stage_bytes, P.stage_stride);
    const int nst = P.n_stages, nbuf = P.n_bufs;
    const uint32_t stage_bytes = P.stage_bytes;
    if (threadIdx.x == 0) {
        mbar_init(&a_full, 1);
        mbar_init(&a_empty, 1);
        for (int i = 0; i < nst; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < nbuf; i++) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], kMoEpiThreads);
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(&mA);
    if (warp == 2) {
        tmem_alloc(&tmem_base_s, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    volatile int *abort_flag = &abort_s;
    const int n_tiles = *P.num_tiles;
    const CUtensorMap *mB[kMoMaxBlocks] = {&mB0, &mB1, &mB2, &mB3, &mB4};

    if (warp == 0 && lane == 0) {
        // ---------------- A loader: the whole A block of the tile ----------------
        int tc = 0;
        for (int it = blockIdx.x; it < n_tiles && !*abort_flag; it += gridDim.x, tc++) {
            if (tc > 0 && !mbar_wait(&a_empty, (tc - 1) & 1, abort_flag)) break;
            const int4 T = P.tiles[it];
            mbar_arrive_expect_tx(&a_full, (uint32_t)P.n_kc * 16384u);
            for (int kc = 0; kc < P.n_kc; kc++) tma_load_2d(sm + L.a + (size_t)kc * 16384u, &mA, kc * 64, T.x, &a_full);
        }
        // drain: the last A block must have landed before the CTA exits
        if (tc > 0) mbar_wait_drain(&a_full, (tc - 1) & 1);
    } else if (warp == 1 && lane == 0) {
        // ---------------- B loader: weight rows of bins b and b + 1 ----------------
        int it_s = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_tiles && !*abort_flag; it += gridDim.x) {
            const int bin = P.tiles[it].z;
            for (int q = 0; ok && q < P.nq; q++)
                for (int m = 0; ok && m < P.n_blocks; m++) {
                    const MoBlock &B = P.blk[m];
                    const int y = (q * P.nb1 + bin) * B.R;      // bins b and b + 1: 2R adjacent rows
                    for (int ks = 0; ks < B.kc; ks++, it_s++) {
                        const int st = it_s % nst, r = it_s / nst;
                        if (r > 0 && !mbar_wait(&b_empty[st], (r - 1) & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        uint8_t *base = sm + L.b + (size_t)st * stage_bytes;
                        mbar_arrive_expect_tx(&b_full[st], 2u * (uint32_t)B.R * 128u);
                        tma_load_2d(base, mB[m], ks * 64, y, &b_full[st]);
                    }
                }
        }
        for (int k = max(0, it_s - nst); k < it_s; k++) mbar_wait_drain(&b_full[k % nst], (k / nst) & 1);
    } else if (warp == 2 && lane == 0) {
        // ---------------- MMA issuer ----------------
        int it_s = 0, cq = 0, tc = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_tiles && !*abort_flag; it += gridDim.x, tc++) {
            if (!mbar_wait(&a_full, tc & 1, abort_flag)) break;
            tc_fence_after();
            for (int q = 0; ok && q < P.nq; q++, cq++) {
                const int buf = cq % nbuf, rr = cq / nbuf;
                if (rr > 0 && !mbar_wait(&t_empty[buf], (rr - 1) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int m = 0; ok && m < P.n_blocks; m++) {
                    const MoBlock &B = P.blk[m];
                    const uint32_t d = tmem + (uint32_t)(buf * P.cols_per_chunk + B.col);
                    const uint32_t idesc = idesc_bf16_f32(128, 2 * B.R);
                    for (int ks = 0; ks < B.kc; ks++, it_s++) {
                        const int st = it_s % nst, r = it_s / nst;
                        if (!mbar_wait(&b_full[st], r & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t abase = smem_u32(sm + L.a) + (uint32_t)(B.kc0 + ks) * 16384u;
                        const uint32_t bbase = smem_u32(sm + L.b + (size_t)st * stage_bytes);
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_f16(d, smem_desc_sw128(abase + kk * 32), smem_desc_sw128(bbase + kk * 32), idesc,
                                     (ks > 0 || kk > 0) ? 1u : 0u);
                        umma_commit(&b_empty[st]);
                    }
                }
                if (ok) umma_commit(&t_full[buf]);
            }
            if (ok) umma_commit(&a_empty);
        }
        umma_commit(&drain_bar);
        mbar_wait_drain(&drain_bar, 0);
    } else if (warp >= kMoEpiWarp0) {
        // ---------------- epilogue: lerp, rotate back, stage, coalesced stores ----------------
        const int ew = warp - kMoEpiWarp0;
        const int qd = warp & 3, half = ew >> 2, row = qd * 32 + lane;
        float *st_w = reinterpret_cast<float *>(sm + L.st) + (size_t)ew * P.stage_stride;
        float *st = st_w + lane;
        int64_t *rowoff_w = reinterpret_cast<int64_t *>(sm + L.ro) + ew * 32;
        const int F = kMoEC * P.d_out;              // floats of one row part
        MoEdge<Lm> E;
        int cq = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_tiles; it += gridDim.x) {
            const int4 T = P.tiles[it];
            const bool valid = row < T.y;
            int64_t e = 0;
            float t = 0.0f;
            float dir[3] = {0.0f, 0.0f, 1.0f}, s = 0.0f;
            if (valid) {
                const int64_t p = (int64_t)T.x + row;
                e = P.perm[p];
                const float dd = P.dist[e];
                s = dd / (dd + P.sh_scale);
                t = P.tval[p];
                dir[0] = P.dirs[e * 3];
                dir[1] = P.dirs[e * 3 + 1];
                dir[2] = P.dirs[e * 3 + 2];
            }
            mo_edge_setup<Lm>(dir, s, E);
            __syncwarp();
            rowoff_w[lane] = valid ? e * (int64_t)P.C_out * P.d_out + half * kMoEC * P.d_out : -1;
            for (int q = 0; q < P.nq; q++, cq++) {
                const int buf = cq % nbuf, rr = cq / nbuf;
                if (!mbar_wait(&t_full[buf], rr & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tbuf = tmem + ((uint32_t)(qd * 32) << 16) +
                                      (uint32_t)(buf * P.cols_per_chunk + half * kMoEC);
                for (int ir = 0; ir < P.n_irr_out; ir++) {
                    const int l = P.irr_out_l[ir], off = P.irr_out_off[ir];
                    if (l == 0) mo_epi_irrep<0, Lm>(P, tbuf, off, E, t, st);
                    else if (l == 1) mo_epi_irrep<1, Lm>(P, tbuf, off, E, t, st);
                    else if constexpr (Lm >= 2) {
                        if (l == 2) mo_epi_irrep<2, Lm>(P, tbuf, off, E, t, st);
                        else if constexpr (Lm >= 3) {
                            if (l == 3) mo_epi_irrep<3, Lm>(P, tbuf, off, E, t, st);
                            else if constexpr (Lm >= 4) mo_epi_irrep<4, Lm>(P, tbuf, off, E, t, st);
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&t_empty[buf]);
                // the warp writes its 32 row parts with coalesced stores (consecutive lanes,
                // consecutive floats of one row)
                __syncwarp();
                float *outq = P.out + q * kMoCC * P.d_out;
                for (int i = lane; i < 32 * F; i += 32) {
                    const int r = i / F, x = i - r * F;
                    const int64_t ro = rowoff_w[r];
                    if (ro >= 0) outq[ro + x] = st_w[x * kMoStT + r];
                }
                __syncwarp();
            }
        }
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && abort_s && P.status) atomicMax(P.status, 2);
}

// Chunk-major copy of the tensor-core weight matrix of one block:
//   Bq[(q * nb1 + b) * R + (u * 8 + c)][k] = B[b * npad + u * Cout + q * 8 + c][k]
// for channel chunk q, bin b, output slot u = (o, re/im), channel c (rows are kpad bf16):
// the rows of bins b and b + 1 of one chunk are adjacent, one TMA box.
__global__ void tc_chunk_b_kernel(const __nv_bfloat16 *__restrict__ B, int npad, int kpad, int Cout, int nslots,
                                  int nb1, __nv_bfloat16 *__restrict__ Bq) {
    const int nq = Cout / kMoCC, R = nslots * kMoCC;
    const int64_t rows = (int64_t)nb1 * nq * R;
    const int v_per_row = kpad / 8;            // 16-byte vectors
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * v_per_row;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / v_per_row;
        const int v = (int)(i - row * v_per_row);
        const int r = (int)(row % R);
        const int64_t qb = row / R;
        const int64_t b = qb % nb1;
        const int q = (int)(qb / nb1);
        const int u = r / kMoCC, c = r - u * kMoCC;
        const int64_t srow = b * npad + (int64_t)u * Cout + q * kMoCC + c;
        reinterpret_cast<uint4 *>(Bq + row * kpad)[v] = reinterpret_cast<const uint4 *>(B + srow * kpad)[v];
    }
}

// Host description of the launch; false when the shapes do not fit the kernel.
bool mo_params(const TcPlan &T, const ReprLayout &Lo, MoParams &P, size_t &smem) {
    memset(&P, 0, sizeof(P));
    if (T.G.n_blocks < 1 || T.G.n_blocks > kMoMaxBlocks || Lo.lmax > kMoTrigL) return false;
    if (T.c_out % kMoCC || Lo.dim > kMoMaxOut || Lo.n_irreps > kMoMaxOut) return false;
    if (T.k_total % 64) return false;
    P.n_blocks = T.G.n_blocks;
    P.nq = T.c_out / kMoCC;
    P.n_kc = T.k_total / 64;
    int col = 0, maxr = 0;
    for (int m = 0; m < P.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        MoBlock &B = P.blk[m];
        B.kc0 = T.koff[m] / 64;
        B.kc = g.kpad / 64;
        B.R = g.n_out * g.mult * kMoCC;
        if (2 * B.R > 256 || (2 * B.R) % 16) return false;       // MMA N of both bins
        B.col = col;
        col += (2 * B.R + 31) / 32 * 32;
        maxr = std::max(maxr, B.R);
    }
    P.cols_per_chunk = col;
    P.n_bufs = std::min(4, 512 / col);
    if (P.n_bufs < 2) return false;
    P.stage_bytes = (uint32_t)((2 * maxr * 128 + 1023) / 1024 * 1024);
    P.stage_stride = kMoEC * Lo.dim * kMoStT;
    for (int k = 0; k < Lo.dim; k++) {
        const int j = Lo.inv_perm[k], b = T.out_map.base[j];
        P.out_col[k] = -1;
        P.out_R[k] = 0;
        if (b < 0) continue;
        for (int m = 0; m < P.n_blocks; m++)
            if (b >= T.noff[m] && b < T.noff[m] + T.nvalid[m]) {
                const int u = (b - T.noff[m]) / T.c_out;
                P.out_col[k] = (int16_t)(P.blk[m].col + u * kMoCC);
                P.out_R[k] = (int16_t)P.blk[m].R;
            }
    }
    P.n_irr_out = Lo.n_irreps;
    for (int r = 0; r < Lo.n_irreps; r++) {
        P.irr_out_l[r] = Lo.irrep_l[r];
        P.irr_out_off[r] = (int8_t)Lo.irrep_off[r];
    }
    P.C_out = T.c_out;
    P.d_out = Lo.dim;
    for (P.n_stages = kMoMaxStages; P.n_stages >= 2; P.n_stages--) {
        smem = mo_smem(P.n_kc, P.n_stages, P.stage_bytes, P.stage_stride).total + 1024;
        if (smem <= 225 * 1024) return true;     // 227 KB per block, static barriers included
    }
    return false;
}

template <int Lm>
int launch_mo(int grid, size_t smem, cudaStream_t s, const CUtensorMap &mA, const CUtensorMap *maps,
              const MoParams &P) {
    FEQ_CUDA_TRY(cudaFuncSetAttribute(tc_mix_out_kernel<Lm>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    tc_mix_out_kernel<Lm><<<grid, kMoThreads, smem, s>>>(mA, maps[0], maps[1], maps[2], maps[3], maps[4], P);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace

bool tc_mix_out_supported(const TcPlan &T, const ReprLayout &Lo) {
    MoParams P;
    size_t smem;
    return mo_params(T, Lo, P, smem);
}

// bf16 elements of the chunk-major weight copies of all blocks.
int64_t tc_mix_out_bq_elems(const TcPlan &T, int nb1) {
    int64_t n = 0;
    for (int m = 0; m < T.G.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        n += (int64_t)nb1 * (T.c_out / kMoCC) * (g.n_out * g.mult * kMoCC) * g.kpad;
    }
    return n;
}

// Chunk-major weights (from the tensor-core layout B) into Bq; one call per forward.
int launch_tc_chunk_b(const TcPlan &T, const __nv_bfloat16 *B, __nv_bfloat16 *Bq, int nb, cudaStream_t s) {
    int64_t off = 0;
    for (int m = 0; m < T.G.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        const int nslots = g.n_out * g.mult;
        const int64_t rows = (int64_t)(nb + 1) * (T.c_out / kMoCC) * nslots * kMoCC;
        const int64_t total = rows * (g.kpad / 8);
        if (total == 0) continue;
        tc_chunk_b_kernel<<<(unsigned)min64((total + 255) / 256, 148 * 16), 256, 0, s>>>(
            B + g.boff, g.npad, g.kpad, T.c_out, nslots, nb + 1, Bq + off);
        FEQ_LAUNCH_CHECK();
        off += rows * g.kpad;
    }
    return FEQ_OK;
}

int launch_tc_mix_out(const TcPlan &T, const ReprLayout &Lo, const __nv_bfloat16 *A, int64_t E,
                      const __nv_bfloat16 *Bq, int nb, const float *dirs, const float *dist, const float *tval,
                      const int64_t *perm, const int4 *tiles, const int *num_tiles, int64_t max_tiles,
                      float sh_scale, float *out, int32_t *status, cudaStream_t s) {
    MoParams P;
    size_t smem;
    if (!mo_params(T, Lo, P, smem)) return FEQ_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(out) & 15) || !dirs) return FEQ_ERR_UNSUPPORTED;
    if (E == 0) return FEQ_OK;
    CUtensorMap mA, maps[kMoMaxBlocks];
    int rc;
    if ((rc = tc_make_map_a(&mA, A, T.k_total, E)) != FEQ_OK) return rc;
    int64_t off = 0;
    for (int m = 0; m < P.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        const int64_t rows = (int64_t)(nb + 1) * P.nq * P.blk[m].R;
        if ((rc = tc_make_map_box(&maps[m], Bq + off, g.kpad, rows, 2 * P.blk[m].R)) != FEQ_OK) return rc;
        off += rows * g.kpad;
    }
    for (int m = P.n_blocks; m < kMoMaxBlocks; m++) maps[m] = maps[0];
    P.nb1 = nb + 1;
    P.dirs = dirs;
    P.dist = dist;
    P.tval = tval;
    P.perm = perm;
    P.tiles = tiles;
    P.num_tiles = num_tiles;
    P.sh_scale = sh_scale;
    P.out = out;
    P.status = status;
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = (int)std::max<int64_t>(1, min64(sms, max_tiles));
    switch (std::max(1, Lo.lmax)) {
        case 1: rc = launch_mo<1>(grid, smem, s, mA, maps, P); break;
        case 2: rc = launch_mo<2>(grid, smem, s, mA, maps, P); break;
        case 3: rc = launch_mo<3>(grid, smem, s, mA, maps, P); break;
        default: rc = launch_mo<4>(grid, smem, s, mA, maps, P); break;
    }
    if (rc != FEQ_OK) return rc;
    return FEQ_OK;
}

}  // namespace feq
