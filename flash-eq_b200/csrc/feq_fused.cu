// feq_fused.cu -- the whole edgewise linear in one persistent tensor-core kernel, for
// representations whose rotated rows of a 128-edge tile fit in shared memory (bf16 mix).
//
// Reference behaviour replaced (the same mathematics as the 3-kernel pipeline of
// feq_rotate_tc.cu + feq_tcmix.cu): EquivariantEdgewiseLinear.forward,
// flash_eq/layers/linear.py:100-160 -- bmm(f, P), block_diagonal_cuda
// (block_diagonal.cu:558-733), bmm(., Q^T).
//
// Per tile of <= 128 sorted edges of one distance bin:
//   rotation warps (0..3)   bulk-load each edge row (gathered by src), rotate it into the
//                           edge frame in registers, and write bf16 A rows straight into
//                           the 128-byte-swizzled K-major A tile in shared memory;
//   loader warp (4)         TMA-loads the weight tiles of bins b and b+1 (adjacent rows);
//   MMA warp (5)            tcgen05.mma M = 128, N = both bins, per output-channel chunk of
//                           8 channels and per m-block, accumulators in TMEM (2 buffers);
//   epilogue warps (6..9)   thread = edge: tcgen05.ld the chunk, lerp the two bins, rotate
//                           back out of the edge frame in registers, store the output.
// A never reaches HBM, nor does the mix result: HBM traffic is the input row, the output
// row and the weight tiles (L2-resident).  All waits are bounded; no TMA multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>

#include "feq_internal.cuh"
#include "feq_rot_common.cuh"
#include "feq_sm100.cuh"

namespace feq {
namespace {

using namespace sm100;
using namespace rot;

constexpr int kFRotWarps = 4;        // rotation warps: 32 tile rows each
constexpr int kFThreads = 320;       // 4 rotation + loader + MMA + 4 epilogue warps
constexpr int kFCC = 8;              // output channels per TMEM chunk
constexpr int kFMaxBlocks = 5;       // m-blocks (lmax <= 4)
constexpr int kFMaxStages = 8;       // weight-tile ring depth (as many as fit)
constexpr int kFTrigL = 4;           // trig layout of every edge: cos/sin of m theta', m phi for m <= 4
constexpr int kFTF = 2 * kFTrigL + 1 + 2 * (kFTrigL + 1);
constexpr int kFMaxIn = 32, kFMaxOut = 16;   // positions of the input / output representation

struct FusedBlock {
    int n_in, n_out, mult;
    int kc0, kc;          // first 64-column chunk of the block in the A tile, and count
    int R;                // weight rows per bin per channel chunk: n_out * mult * 8
    int col;              // TMEM column of the block inside a chunk buffer
};

struct FusedParams {
    int n_blocks, nq, cols_per_chunk, n_kc;
    int n_stages;
    uint32_t stage_bytes;      // 2 bins x max R rows x 128 B, multiple of 1024
    int16_t in_col[kFMaxIn];   // std input position -> A column (-1: no block takes it)
    int16_t out_col[kFMaxOut]; // std output position -> TMEM column of bin lo (channel 0) in a chunk
    int16_t out_R[kFMaxOut];   // ... and the offset of bin hi
    int n_irr_in, n_irr_out;
    int8_t irr_in_l[kFMaxIn], irr_in_off[kFMaxIn], irr_out_l[kFMaxOut], irr_out_off[kFMaxOut];
    FusedBlock blk[kFMaxBlocks];
    int C_in, C_out, d_in, d_out;
    const float *x;            // node or edge rows (N_src or E, C_in, d_in)
    const int64_t *src;        // nullable: gather rows by src
    int64_t nsrc;
    const float *dirs, *dist;
    const int64_t *perm;
    const int4 *tiles;
    const int *num_tiles;
    Binning bins;
    float sh_scale;
    float *out;                // (E, C_out, d_out)
    int32_t *status;
};

// Byte offset of bf16 element (row r, column k) in a stack of 128 x 64 K-major tiles with
// the 128-byte swizzle (16-byte chunk index XOR row mod 8), as TMA SWIZZLE_128B writes it.
__device__ __forceinline__ uint32_t a_tile_offset(int r, int k) {
    const int kc = k >> 6, kin = k & 63;
    return (uint32_t)kc * 16384u + (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u +
           (uint32_t)(((kin >> 3) ^ (r & 7)) << 4) + (uint32_t)(kin & 7) * 2u;
}

// Shared-memory map of the fused kernel (bytes from the 1024-aligned base).
struct FusedSmem {
    uint32_t a, b, rows, trig, total;
};
__host__ __device__ inline FusedSmem fused_smem(int n_kc, int row_floats, int n_stages, uint32_t stage_bytes) {
    FusedSmem m;
    m.a = 0;
    m.b = (uint32_t)n_kc * 16384u;
    m.rows = m.b + (uint32_t)n_stages * stage_bytes;
    const uint32_t rb = (uint32_t)((row_floats * 4 + 15) & ~15);
    m.trig = m.rows + kFRotWarps * 2 * rb;
    m.total = m.trig + (uint32_t)(kFRotWarps * 32 + 128) * kFTF * 4u;
    return m;
}

// Epilogue for one output irrep of degree Lg: 8 channels of one edge (this thread's TMEM
// lane).  Positions i = 0..2Lg of the irrep read bins lo / hi with one 8-column load each,
// lerp with t, then rotate back two channels at a time and store.
template <int Lg>
__device__ __forceinline__ void fused_epi_irrep(const FusedParams &P, uint32_t tbuf, int off, const float *tr,
                                                float sl, float t, bool valid, float *orow, int q) {
    constexpr int N = 2 * Lg + 1;
    float h[N][kFCC];
#pragma unroll
    for (int i = 0; i < N; i++) {
        const int col = P.out_col[off + i];
        uint32_t lo[8], hi[8];
        const uint32_t c0 = col < 0 ? 0u : (uint32_t)col;
        tmem_ld8(tbuf + c0, lo);
        tmem_ld8(tbuf + c0 + (uint32_t)(col < 0 ? 0 : P.out_R[off + i]), hi);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kFCC; c++) {
            const float a = __uint_as_float(lo[c]), b = __uint_as_float(hi[c]);
            h[i][c] = col < 0 ? 0.0f : fmaf(t, b - a, a);
        }
    }
    if (!valid) return;
    const int dout = P.d_out;
#pragma unroll
    for (int c = 0; c < kFCC; c += 2) {
        float *o0 = orow + (q * kFCC + c) * dout + off, *o1 = o0 + dout;
        auto get = [&](int i) { return make_float2(h[i][c], h[i][c + 1]); };
        auto emit = [&](int o, float y0, float y1) {
            o0[o] = y0;
            o1[o] = y1;
        };
        if constexpr (Lg == 0)
            emit(0, h[0][c] * sl, h[0][c + 1] * sl);
        else
            rot_irrep2<Lg, true>(tr, kFTrigL, sl, get, emit);
    }
}

__global__ void __launch_bounds__(kFThreads, 1)
fused_edgewise_kernel(const __grid_constant__ CUtensorMap mB0, const __grid_constant__ CUtensorMap mB1,
                      const __grid_constant__ CUtensorMap mB2, const __grid_constant__ CUtensorMap mB3,
                      const __grid_constant__ CUtensorMap mB4, const __grid_constant__ FusedParams P) {
    extern __shared__ uint8_t fsm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(fsm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t a_full, a_empty, b_full[kFMaxStages], b_empty[kFMaxStages], t_full[2], t_empty[2];
    __shared__ uint64_t row_bar[kFRotWarps][2], drain_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_floats = P.C_in * P.d_in;
    const FusedSmem L = fused_smem(P.n_kc, row_floats, P.n_stages, P.stage_bytes);
    const int nst = P.n_stages;
    const uint32_t stage_bytes = P.stage_bytes;
    const uint32_t row_bytes = (uint32_t)row_floats * 4u, rb = (row_bytes + 15u) & ~15u;
    if (threadIdx.x == 0) {
        mbar_init(&a_full, kFRotWarps);
        mbar_init(&a_empty, 1);
        for (int i = 0; i < nst; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], 128);
        }
        for (int w = 0; w < kFRotWarps; w++) {
            mbar_init(&row_bar[w][0], 1);
            mbar_init(&row_bar[w][1], 1);
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    // zero the A tile once: its K padding columns are never written afterwards
    for (uint32_t i = threadIdx.x; i < (uint32_t)P.n_kc * 16384u / 16u; i += blockDim.x)
        reinterpret_cast<uint4 *>(sm + L.a)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_async_smem();
    if (warp == 5) {
        tmem_alloc(&tmem_base_s, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    volatile int *abort_flag = &abort_s;
    const int n_tiles = *P.num_tiles;
    const CUtensorMap *mB[kFMaxBlocks] = {&mB0, &mB1, &mB2, &mB3, &mB4};

    if (warp < kFRotWarps) {
        // ---------------- rotation into the edge frame -> A tile ----------------
        float *trig = reinterpret_cast<float *>(sm + L.trig) + (size_t)warp * 32 * kFTF;
        uint8_t *rowbuf = sm + L.rows + (size_t)warp * 2 * rb;
        uint32_t phase_bits = 0;
        int pending = 0;
        bool alive = true;
        int tc = 0;
        for (int it = blockIdx.x; alive && it < n_tiles; it += gridDim.x, tc++) {
            const int4 T = P.tiles[it];
            const int r0 = warp * 32, nr = min(32, T.y - r0);
            int64_t e_l = 0, xr_l = -1;
            float s_l = 0.0f;
            if (lane < nr) {
                const int64_t p = (int64_t)T.x + r0 + lane;
                e_l = P.perm[p];
                const float dd = P.dist[e_l];
                s_l = dd / (dd + P.sh_scale);
                edge_trig_compact(P.dirs[e_l * 3], P.dirs[e_l * 3 + 1], P.dirs[e_l * 3 + 2], kFTrigL,
                                  trig + lane * kFTF);
                xr_l = e_l;
                if (P.src) {
                    xr_l = P.src[e_l];
                    if (xr_l < 0 || xr_l >= P.nsrc) {
                        set_status(P.status, 1);
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
                    mbar_arrive_expect_tx(&row_bar[warp][b], row_bytes);
                    bulk_load(rowbuf + b * rb, P.x + xr * (int64_t)row_floats, row_bytes, &row_bar[warp][b]);
                }
                if (xr >= 0) pending |= 1 << b;
            };
            if (nr > 0) issue(0);
            // the previous tile's MMAs must be done reading the A tile
            if (tc > 0 && !mbar_wait(&a_empty, (tc - 1) & 1, abort_flag)) {
                set_status(P.status, 2);
                alive = false;
            }
            __syncwarp();
            for (int j = 0; alive && j < nr; j++) {
                const int64_t xr = __shfl_sync(0xffffffffu, xr_l, j);
                const float s = __shfl_sync(0xffffffffu, s_l, j);
                const int b = j & 1;
                if (j + 1 < nr) issue(j + 1);
                const float *fb = reinterpret_cast<const float *>(rowbuf + b * rb);
                if (xr >= 0) {
                    if (!mbar_wait(&row_bar[warp][b], (phase_bits >> b) & 1u, abort_flag)) {
                        set_status(P.status, 2);
                        alive = false;
                        break;
                    }
                    phase_bits ^= 1u << b;
                    pending &= ~(1 << b);
                }
                const float *trj = trig + j * kFTF;
                const int row = r0 + j;
                const bool have = xr >= 0;
                for (int c = 2 * lane; c < P.C_in; c += 64) {
                    const float *f0 = fb + c * P.d_in, *f1 = f0 + P.d_in;
                    for (int ir = 0; ir < P.n_irr_in; ir++) {
                        const int l = P.irr_in_l[ir], off = P.irr_in_off[ir];
                        auto get = [&](int q2) {
                            return have ? make_float2(f0[off + q2], f1[off + q2]) : make_float2(0.0f, 0.0f);
                        };
                        auto emit = [&](int o, float y0, float y1) {
                            const int col = P.in_col[off + o];
                            if (col < 0) return;
                            *reinterpret_cast<__nv_bfloat162 *>(sm + L.a + a_tile_offset(row, col + c)) =
                                __floats2bfloat162_rn(y0, y1);
                        };
                        rot_irrep2_any<false>(l, trj, kFTrigL, ipowf(s, l), get, emit);
                    }
                }
                __syncwarp();
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full);
        }
        for (int b = 0; b < 2; b++)
            if (pending & (1 << b)) mbar_wait_drain(&row_bar[warp][b], (phase_bits >> b) & 1u);
    }
    else if (warp == 4 && lane == 0) {
        // ---------------- TMA loader: weight tiles of bins b and b + 1 ----------------
        int it_s = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_tiles && !*abort_flag; it += gridDim.x) {
            const int bin = P.tiles[it].z;
            for (int q = 0; ok && q < P.nq; q++)
                for (int m = 0; ok && m < P.n_blocks; m++) {
                    const FusedBlock &B = P.blk[m];
                    const int y = (bin * P.nq + q) * B.R;
                    for (int ks = 0; ks < B.kc; ks++, it_s++) {
                        const int st = it_s % nst, r = it_s / nst;
                        if (r > 0 && !mbar_wait(&b_empty[st], (r - 1) & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        uint8_t *base = sm + L.b + (size_t)st * stage_bytes;
                        mbar_arrive_expect_tx(&b_full[st], 2u * (uint32_t)B.R * 128u);
                        tma_load_2d(base, mB[m], ks * 64, y, &b_full[st]);
                        tma_load_2d(base + B.R * 128, mB[m], ks * 64, y + P.nq * B.R, &b_full[st]);
                    }
                }
        }
        for (int k = max(0, it_s - nst); k < it_s; k++) mbar_wait_drain(&b_full[k % nst], (k / nst) & 1);
    } else if (warp == 5 && lane == 0) {
        // ---------------- MMA issuer ----------------
        int it_s = 0, cq = 0, tc = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_tiles && !*abort_flag; it += gridDim.x, tc++) {
            if (!mbar_wait(&a_full, tc & 1, abort_flag)) break;
            tc_fence_after();
            for (int q = 0; ok && q < P.nq; q++, cq++) {
                const int buf = cq & 1, rr = cq >> 1;
                if (rr > 0 && !mbar_wait(&t_empty[buf], (rr - 1) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int m = 0; ok && m < P.n_blocks; m++) {
                    const FusedBlock &B = P.blk[m];
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
    } else if (warp >= 6) {
        // ---------------- epilogue: lerp, rotate back, store ----------------
        const int qd = warp & 3, row = qd * 32 + lane;
        float *tr = reinterpret_cast<float *>(sm + L.trig) + (size_t)(kFRotWarps * 32 + row) * kFTF;
        int cq = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_tiles; it += gridDim.x) {
            const int4 T = P.tiles[it];
            const bool valid = row < T.y;
            int64_t e = 0;
            float s = 0.0f, t = 0.0f;
            if (valid) {
                e = P.perm[(int64_t)T.x + row];
                const float dd = P.dist[e];
                s = dd / (dd + P.sh_scale);
                int lo;
                bin_of(dd, P.bins, lo, t);
                edge_trig_compact(P.dirs[e * 3], P.dirs[e * 3 + 1], P.dirs[e * 3 + 2], kFTrigL, tr);
            }
            float *orow = P.out + e * (int64_t)P.C_out * P.d_out;
            for (int q = 0; q < P.nq; q++, cq++) {
                const int buf = cq & 1, rr = cq >> 1;
                if (!mbar_wait(&t_full[buf], rr & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tbuf = tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)(buf * P.cols_per_chunk);
                for (int ir = 0; ir < P.n_irr_out; ir++) {
                    const int l = P.irr_out_l[ir], off = P.irr_out_off[ir];
                    const float sl = ipowf(s, l);
                    switch (l) {
                        case 0: fused_epi_irrep<0>(P, tbuf, off, tr, sl, t, valid, orow, q); break;
                        case 1: fused_epi_irrep<1>(P, tbuf, off, tr, sl, t, valid, orow, q); break;
                        case 2: fused_epi_irrep<2>(P, tbuf, off, tr, sl, t, valid, orow, q); break;
                        case 3: fused_epi_irrep<3>(P, tbuf, off, tr, sl, t, valid, orow, q); break;
                        default: fused_epi_irrep<4>(P, tbuf, off, tr, sl, t, valid, orow, q); break;
                    }
                }
                tc_fence_before();
                mbar_arrive(&t_empty[buf]);
            }
        }
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && abort_s && P.status) atomicMax(P.status, 2);
}

}  // namespace
}  // namespace feq

namespace feq {

int tc_make_map_box(CUtensorMap *m, const void *base, int64_t cols, int64_t rows, int box_rows);

// Chunk-major copy of the tensor-core weight matrix of one block:
//   Bq[(b * nq + q) * R + (u * 8 + c)][k] = B[b * npad + u * Cout + q * 8 + c][k]
// for bin b, channel chunk q, output slot u = (o, re/im), channel c.  Rows are kpad bf16.
__global__ void fused_chunk_b_kernel(const __nv_bfloat16 *__restrict__ B, int npad, int kpad, int Cout, int nslots,
                                     int nb1, __nv_bfloat16 *__restrict__ Bq) {
    const int nq = Cout / kFCC, R = nslots * kFCC;
    const int64_t rows = (int64_t)nb1 * nq * R;
    const int v_per_row = kpad / 8;            // 16-byte vectors
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * v_per_row;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / v_per_row;
        const int v = (int)(i - row * v_per_row);
        const int r = (int)(row % R);
        const int64_t bq = row / R;
        const int q = (int)(bq % nq);
        const int64_t b = bq / nq;
        const int u = r / kFCC, c = r - u * kFCC;
        const int64_t srow = b * npad + (int64_t)u * Cout + q * kFCC + c;
        reinterpret_cast<uint4 *>(Bq + row * kpad)[v] = reinterpret_cast<const uint4 *>(B + srow * kpad)[v];
    }
}

// Host description of the fused launch; false when the shapes do not fit the kernel.
static bool fused_params(const TcPlan &T, const ReprLayout &Li, const ReprLayout &Lo, FusedParams &P, size_t &smem) {
    memset(&P, 0, sizeof(P));
    if (T.G.n_blocks < 1 || T.G.n_blocks > kFMaxBlocks || Li.lmax > kFTrigL || Lo.lmax > kFTrigL) return false;
    if (T.c_out % kFCC || (T.c_in & 1) || Li.dim > kFMaxIn || Lo.dim > kFMaxOut) return false;
    if (Li.n_irreps > kFMaxIn || Lo.n_irreps > kFMaxOut) return false;
    if (((int64_t)T.c_in * Li.dim * 4) % 16) return false;
    P.n_blocks = T.G.n_blocks;
    P.nq = T.c_out / kFCC;
    P.n_kc = T.k_total / 64;
    int col = 0, maxr = 0;
    for (int m = 0; m < P.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        FusedBlock &B = P.blk[m];
        B.n_in = g.n_in;
        B.n_out = g.n_out;
        B.mult = g.mult;
        B.kc0 = T.koff[m] / 64;
        B.kc = g.kpad / 64;
        B.R = g.n_out * g.mult * kFCC;
        if (2 * B.R > 256) return false;                     // MMA N of both bins
        B.col = col;
        col += (2 * B.R + 31) / 32 * 32;
        maxr = std::max(maxr, B.R);
    }
    P.cols_per_chunk = col;
    if (2 * col > 512) return false;
    P.stage_bytes = (uint32_t)((2 * maxr * 128 + 1023) / 1024 * 1024);
    for (int k = 0; k < Li.dim; k++) P.in_col[k] = (int16_t)T.in_map.base_std[k];
    for (int k = 0; k < Lo.dim; k++) {
        const int j = Lo.inv_perm[k], b = T.out_map.base[j];
        P.out_col[k] = -1;
        P.out_R[k] = 0;
        if (b < 0) continue;
        for (int m = 0; m < P.n_blocks; m++)
            if (b >= T.noff[m] && b < T.noff[m] + T.nvalid[m]) {
                const int u = (b - T.noff[m]) / T.c_out;
                P.out_col[k] = (int16_t)(P.blk[m].col + u * kFCC);
                P.out_R[k] = (int16_t)P.blk[m].R;
            }
    }
    P.n_irr_in = Li.n_irreps;
    for (int r = 0; r < Li.n_irreps; r++) {
        P.irr_in_l[r] = Li.irrep_l[r];
        P.irr_in_off[r] = (int8_t)Li.irrep_off[r];
    }
    P.n_irr_out = Lo.n_irreps;
    for (int r = 0; r < Lo.n_irreps; r++) {
        P.irr_out_l[r] = Lo.irrep_l[r];
        P.irr_out_off[r] = (int8_t)Lo.irrep_off[r];
    }
    P.C_in = T.c_in;
    P.C_out = T.c_out;
    P.d_in = Li.dim;
    P.d_out = Lo.dim;
    for (P.n_stages = kFMaxStages; P.n_stages >= 2; P.n_stages--) {
        smem = fused_smem(P.n_kc, T.c_in * Li.dim, P.n_stages, P.stage_bytes).total + 1024;
        if (smem <= 227 * 1024) return true;
    }
    return false;
}

bool fused_edgewise_supported(const TcPlan &T, const ReprLayout &Li, const ReprLayout &Lo) {
    FusedParams P;
    size_t smem;
    return fused_params(T, Li, Lo, P, smem);
}

// bf16 elements of the chunk-major weight copies of all blocks.
int64_t fused_bq_elems(const TcPlan &T, int nb1) {
    int64_t n = 0;
    for (int m = 0; m < T.G.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        n += (int64_t)nb1 * (T.c_out / kFCC) * (g.n_out * g.mult * kFCC) * g.kpad;
    }
    return n;
}

int launch_fused_edgewise(const TcPlan &T, const ReprLayout &Li, const ReprLayout &Lo, const __nv_bfloat16 *B,
                          __nv_bfloat16 *Bq, int nb, const float *x, const int64_t *src, int64_t nsrc,
                          const float *dirs, const float *dist, const int64_t *perm, const int4 *tiles,
                          const int *num_tiles, int64_t max_tiles, Binning bins, float sh_scale, float *out,
                          int32_t *status, cudaStream_t s) {
    FusedParams P;
    size_t smem;
    if (!fused_params(T, Li, Lo, P, smem)) return FEQ_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || !dirs) return FEQ_ERR_UNSUPPORTED;
    CUtensorMap maps[kFMaxBlocks];
    int64_t off = 0;
    int rc;
    for (int m = 0; m < P.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        const int64_t rows = (int64_t)(nb + 1) * P.nq * P.blk[m].R;
        const int64_t total = rows * (g.kpad / 8);
        fused_chunk_b_kernel<<<(unsigned)min64((total + 255) / 256, 148 * 16), 256, 0, s>>>(
            B + g.boff, g.npad, g.kpad, T.c_out, g.n_out * g.mult, nb + 1, Bq + off);
        FEQ_LAUNCH_CHECK();
        if ((rc = tc_make_map_box(&maps[m], Bq + off, g.kpad, rows, P.blk[m].R)) != FEQ_OK) return rc;
        off += rows * g.kpad;
    }
    for (int m = P.n_blocks; m < kFMaxBlocks; m++) maps[m] = maps[0];
    P.x = x;
    P.src = src;
    P.nsrc = nsrc;
    P.dirs = dirs;
    P.dist = dist;
    P.perm = perm;
    P.tiles = tiles;
    P.num_tiles = num_tiles;
    P.bins = bins;
    P.sh_scale = sh_scale;
    P.out = out;
    P.status = status;
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int grid = (int)std::max<int64_t>(1, min64(sms, max_tiles));
    FEQ_CUDA_TRY(cudaFuncSetAttribute(fused_edgewise_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    fused_edgewise_kernel<<<grid, kFThreads, smem, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], P);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
