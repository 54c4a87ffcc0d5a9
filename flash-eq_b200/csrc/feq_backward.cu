// feq_backward.cu -- backward of the block-diagonal radial mix (grad_features,
// grad_table, grad_distances), deterministic and atomics-free.
//
// Reference behaviour replaced: _block_diagonal_cuda.backward
// (flash_eq/cuda/csrc/block_diagonal.cu:747-1161, :1543-1758), which accumulates
// grad_table and grad_distances with atomics.
//
// With A[p][k] = s^l_i f[k] and G[p][n] = s^l_o go[n] for the sorted row p of an edge
// (the tensor-core layouts of feq_tcmix.cu, column = block offset + member/re-im
// position * C + channel), W_t = (1 - t) W[lo] + t W[lo + 1] and W the real-embedded
// block matrix:
//   grad_f[k]       = s^l_i  (G W_t)[k]                       tensor-core mix of G with W^T
//   grad_W[bin b]   = sum_{p in b} (1 - t_p) G_p^T A_p + sum_{p in b-1} t_p G_p^T A_p
//                                                              per-bin tensor-core reduction over the
//                                                              transposed, bin-padded G and A (tc_gram)
//   dL/dt           = sum_k A[k] (G (W[lo+1] - W[lo]))[k]      second epilogue output of the mix
//   dL/ds * s       = sum_k l_i A[k] (G W_t)[k] + sum_n l_o G[n] (W_t A)[n]
//   grad_d          = dL/dt dt/dd + (dL/ds * s) * scale / (d (d + scale))
// The last line is the reference's grad_sh expression (block_diagonal.cu:990-1036):
// a zero distance gives inf * 0 = NaN whenever some l_i + l_o > 0, as there.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "feq_internal.cuh"

namespace feq {

// Sorted row p of m-first rows X (E, C, D): M[p][base[j] + c] = s^l(j) X[e][c][j] as bf16
// hi (+ lo), K padding zeroed; also t[p] when tval is given.  One warp per row; the row
// is staged in shared memory with coalesced loads.
__global__ void bwd_prep_rows_kernel(const float *__restrict__ X, const float *__restrict__ dist,
                                     const int64_t *__restrict__ perm, int64_t E, int C, int D,
                                     const __grid_constant__ TcPosMap Mp, int ld, Binning bins, float sh_scale,
                                     __nv_bfloat16 *__restrict__ Mhi, __nv_bfloat16 *__restrict__ Mlo,
                                     float *__restrict__ tval) {
    extern __shared__ float rows_s[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int row = C * D;
    float *rs = rows_s + (size_t)w * row;
    for (int64_t p = (int64_t)blockIdx.x * nw + w; p < E; p += (int64_t)gridDim.x * nw) {
        const int64_t e = perm[p];
        const float dd = dist[e];
        const float s = dd / (dd + sh_scale);
        if (lane == 0 && tval) {
            int lo;
            float t;
            bin_of(dd, bins, lo, t);
            tval[p] = t;
        }
        const float *xr = X + e * (int64_t)row;
        for (int i = lane; i < row; i += 32) rs[i] = __ldg(xr + i);
        __syncwarp();
        __nv_bfloat16 *mh = Mhi + p * (int64_t)ld;
        __nv_bfloat16 *ml = Mlo ? Mlo + p * (int64_t)ld : nullptr;
        for (int r = 0; r < Mp.n_pad; r++)
            for (int i = Mp.pad_lo[r] + lane; i < Mp.pad_hi[r]; i += 32) {
                mh[i] = __float2bfloat16_rn(0.0f);
                if (ml) ml[i] = __float2bfloat16_rn(0.0f);
            }
        for (int j = 0; j < D; j++) {
            const int b = Mp.base[j];
            if (b < 0) continue;
            const float sl = ipowf(s, Mp.l[j]);
            for (int c = lane; c < C; c += 32) {
                const float v = rs[c * D + j] * sl;
                const __nv_bfloat16 h = __float2bfloat16_rn(v);
                mh[b + c] = h;
                if (ml) ml[b + c] = __float2bfloat16_rn(v - __bfloat162float(h));
            }
        }
        __syncwarp();
    }
}

// Table of the transposed mix: T'[b][ci][co][w'] from T[b][co][ci][w] with the in/out
// roles of every block swapped (w' = w_off + i n_out + o for m = 0, pairs 2(i n_out + o)
// + {a, -b} for m > 0).  blk holds (m, n_in, n_out, w_off) of the original layout.
__global__ void bwd_transpose_table_kernel(const float *__restrict__ T, float *__restrict__ Tt, int nb1, int Cout,
                                           int Cin, int W, const __grid_constant__ MixLayout M) {
    const int64_t total = (int64_t)nb1 * Cout * Cin * W;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int w = (int)(idx % W);
        int64_t r = idx / W;
        const int ci = (int)(r % Cin);
        r /= Cin;
        const int co = (int)(r % Cout);
        const int64_t b = r / Cout;
        int q = -1;
        for (int m = 0; m < M.n_blocks; m++) {
            const MixBlock &B = M.blk[m];
            const int sz = B.n_in * B.n_out * (B.m == 0 ? 1 : 2);
            if (B.n_in > 0 && B.n_out > 0 && w >= B.w_off && w < B.w_off + sz) q = m;
        }
        if (q < 0) continue;                     // weight slot of an empty block: never read
        const MixBlock &B = M.blk[q];
        const int lw = w - B.w_off;
        float v = T[idx];
        int wt;
        if (B.m == 0) {
            const int o = lw / B.n_in, i = lw - o * B.n_in;
            wt = B.w_off + i * B.n_out + o;
        } else {
            const int pr = lw >> 1, c = lw & 1;
            const int o = pr / B.n_in, i = pr - o * B.n_in;
            wt = B.w_off + 2 * (i * B.n_out + o) + c;
            if (c) v = -v;
        }
        Tt[((b * Cin + ci) * Cout + co) * (int64_t)W + wt] = v;
    }
}

// dt/dd of the bin an edge falls in (block_diagonal.cu:117-139, float steps).
__device__ __forceinline__ float bwd_dt_dd(float d, const Binning &b) {
    if (!b.log_bins) return b.p2;
    int lo;
    float t;
    bin_of(d, b, lo, t);
    const float inv_lbw = b.p2 * b.num_bins;
    const float log_edge_lo = b.p1 + (float)lo / inv_lbw;
    const float edge_lo = (float)exp((double)log_edge_lo);
    const float edge_hi = (float)exp((double)(log_edge_lo + 1.0f / inv_lbw));
    return 1.0f / (edge_hi - edge_lo);
}

// Per sorted row p (one warp): grad_f rows (m-first, the features' layout) and grad_d.
//   gA, gAd : (E, ld_g) transposed-mix outputs G W_t and G (W[hi] - W[lo]), columns out2.base + c
//   A       : (E, ld_a) bf16 hi + lo, columns in1.base + c        (s^l_i f)
//   G       : (E, ld_gg) bf16 hi + lo, columns in2.base + c       (s^l_o go)
//   H       : (E, ld_h) forward mix W_t A, columns out1.base + c
__global__ void bwd_rows_kernel(const float *__restrict__ gA, const float *__restrict__ gAd, int ld_g,
                                const __nv_bfloat16 *__restrict__ Ahi, const __nv_bfloat16 *__restrict__ Alo,
                                int ld_a, const __nv_bfloat16 *__restrict__ Ghi,
                                const __nv_bfloat16 *__restrict__ Glo, int ld_gg, const float *__restrict__ H,
                                int ld_h, const float *__restrict__ dist, const int64_t *__restrict__ perm, int64_t E,
                                int Cin, int Din, int Cout, int Dout, const __grid_constant__ TcPosMap in1,
                                const __grid_constant__ TcPosMap out1, const __grid_constant__ TcPosMap in2,
                                const __grid_constant__ TcPosMap out2, Binning bins, float sh_scale, int any_l,
                                float *__restrict__ grad_f, float *__restrict__ grad_d) {
    extern __shared__ float gf_s[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int row = Cin * Din;
    float *rs = gf_s + (size_t)w * row;
    auto bf2f = [](const __nv_bfloat16 *h, const __nv_bfloat16 *l, int64_t i) {
        float v = __bfloat162float(h[i]);
        if (l) v += __bfloat162float(l[i]);
        return v;
    };
    for (int64_t p = (int64_t)blockIdx.x * nw + w; p < E; p += (int64_t)gridDim.x * nw) {
        const int64_t e = perm[p];
        const float dd = dist[e];
        const float s = dd / (dd + sh_scale);
        float gt = 0.0f, sh = 0.0f;
        const float *ga = gA + p * (int64_t)ld_g, *gad = gAd + p * (int64_t)ld_g;
        const int64_t ar = p * (int64_t)ld_a;
        for (int j = 0; j < Din; j++) {
            const int bo = out2.base[j], ba = in1.base[j];
            const float sl = ipowf(s, in1.l[j]);
            for (int c = lane; c < Cin; c += 32) {
                float g = 0.0f;
                if (bo >= 0) {
                    g = ga[bo + c];
                    const float a = bf2f(Ahi, Alo, ar + ba + c);
                    gt = fmaf(a, gad[bo + c], gt);
                    sh = fmaf((float)in1.l[j] * a, g, sh);
                }
                rs[c * Din + j] = g * sl;
            }
        }
        const float *hr = H + p * (int64_t)ld_h;
        const int64_t gr = p * (int64_t)ld_gg;
        for (int j = 0; j < Dout; j++) {
            const int bh = out1.base[j], bg = in2.base[j];
            if (bh < 0 || bg < 0 || out1.l[j] == 0) continue;
            const float lo_ = (float)out1.l[j];
            for (int c = lane; c < Cout; c += 32) sh = fmaf(lo_ * bf2f(Ghi, Glo, gr + bg + c), hr[bh + c], sh);
        }
        for (int o = 16; o > 0; o >>= 1) {
            gt += __shfl_xor_sync(0xffffffffu, gt, o);
            sh += __shfl_xor_sync(0xffffffffu, sh, o);
        }
        __syncwarp();
        float *gfr = grad_f + e * (int64_t)row;
        for (int i = lane; i < row; i += 32) gfr[i] = rs[i];
        if (lane == 0) {
            float g = gt * bwd_dt_dd(dd, bins);
            if (any_l) g += sh * (sh_scale / (dd * (dd + sh_scale)));
            grad_d[e] = g;
        }
        __syncwarp();
    }
}

// dB (per block m: (nb + 1, N_m, K_m) at dboff[m]) -> grad_table (nb + 1, Cout, Cin, W):
// m = 0: dT[co][ci][w_off + o n_in + i] = dB[o Cout + co][i Cin + ci];
// m > 0: a = dB[re][re] + dB[im][im], b = dB[re][im] - dB[im][re] with n = (2o + re/im) Cout + co,
//        k = (2i + re/im) Cin + ci (the transposes of the [[a, b], [-b, a]] embedding).
__global__ void bwd_table_convert_kernel(const float *__restrict__ dB, const __grid_constant__ DbOff dboff,
                                         int nb1, int Cout, int Cin, int W, const __grid_constant__ MixLayout M,
                                         float *__restrict__ grad_table) {
    const int64_t total = (int64_t)nb1 * Cout * Cin * W;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int w = (int)(idx % W);
        int64_t r = idx / W;
        const int ci = (int)(r % Cin);
        r /= Cin;
        const int co = (int)(r % Cout);
        const int64_t b = r / Cout;
        float v = 0.0f;
        for (int m = 0; m < M.n_blocks; m++) {
            const MixBlock &B = M.blk[m];
            if (B.n_in == 0 || B.n_out == 0) continue;
            const int mult = B.m == 0 ? 1 : 2;
            const int sz = B.n_in * B.n_out * mult;
            if (w < B.w_off || w >= B.w_off + sz) continue;
            const int N = Cout * mult * B.n_out, K = Cin * mult * B.n_in;
            const float *D = dB + dboff.off[m] + b * (int64_t)N * K;
            const int lw = w - B.w_off;
            if (mult == 1) {
                const int o = lw / B.n_in, i = lw - o * B.n_in;
                v = D[(int64_t)(o * Cout + co) * K + i * Cin + ci];
            } else {
                const int pr = lw >> 1, c = lw & 1;
                const int o = pr / B.n_in, i = pr - o * B.n_in;
                const int nre = (2 * o) * Cout + co, nim = (2 * o + 1) * Cout + co;
                const int kre = (2 * i) * Cin + ci, kim = (2 * i + 1) * Cin + ci;
                v = c == 0 ? D[(int64_t)nre * K + kre] + D[(int64_t)nim * K + kim]
                           : D[(int64_t)nre * K + kim] - D[(int64_t)nim * K + kre];
            }
        }
        grad_table[idx] = v;
    }
}

static int rows_warps(size_t row_floats) {
    const size_t per = row_floats * 4;
    int w = 8;
    while (w > 1 && per * w > 150 * 1024) w--;
    return per > 150 * 1024 ? 0 : w;
}

static int grid_for(int64_t work, int per_block) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return (int)std::max<int64_t>(1, min64((work + per_block - 1) / per_block, (int64_t)sms * 16));
}

int launch_bwd_prep_rows(const float *X, const float *dist, const int64_t *perm, int64_t E, int C, int D,
                         const TcPosMap &Mp, int ld, Binning bins, float sh_scale, __nv_bfloat16 *Mhi,
                         __nv_bfloat16 *Mlo, float *tval, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const int nw = rows_warps((size_t)C * D);
    if (nw == 0) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = (size_t)nw * C * D * 4;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(bwd_prep_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    bwd_prep_rows_kernel<<<grid_for(E, nw), nw * 32, smem, s>>>(X, dist, perm, E, C, D, Mp, ld, bins, sh_scale, Mhi,
                                                                Mlo, tval);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_bwd_transpose_table(const float *T, float *Tt, int nb1, int Cout, int Cin, int W, const MixLayout &M,
                               cudaStream_t s) {
    const int64_t total = (int64_t)nb1 * Cout * Cin * W;
    if (total == 0) return FEQ_OK;
    bwd_transpose_table_kernel<<<grid_for(total, 256), 256, 0, s>>>(T, Tt, nb1, Cout, Cin, W, M);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_bwd_rows(const float *gA, const float *gAd, int ld_g, const __nv_bfloat16 *Ahi, const __nv_bfloat16 *Alo,
                    int ld_a, const __nv_bfloat16 *Ghi, const __nv_bfloat16 *Glo, int ld_gg, const float *H, int ld_h,
                    const float *dist, const int64_t *perm, int64_t E, int Cin, int Din, int Cout, int Dout,
                    const TcPosMap &in1, const TcPosMap &out1, const TcPosMap &in2, const TcPosMap &out2,
                    Binning bins, float sh_scale, int any_l, float *grad_f, float *grad_d, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const int nw = rows_warps((size_t)Cin * Din);
    if (nw == 0) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = (size_t)nw * Cin * Din * 4;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(bwd_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    bwd_rows_kernel<<<grid_for(E, nw), nw * 32, smem, s>>>(gA, gAd, ld_g, Ahi, Alo, ld_a, Ghi, Glo, ld_gg, H, ld_h,
                                                           dist, perm, E, Cin, Din, Cout, Dout, in1, out1, in2, out2,
                                                           bins, sh_scale, any_l, grad_f, grad_d);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_bwd_table_convert(const float *dB, const DbOff &dboff, int nb1, int Cout, int Cin, int W,
                             const MixLayout &M, float *grad_table, cudaStream_t s) {
    const int64_t total = (int64_t)nb1 * Cout * Cin * W;
    if (total == 0) return FEQ_OK;
    bwd_table_convert_kernel<<<grid_for(total, 256), 256, 0, s>>>(dB, dboff, nb1, Cout, Cin, W, M, grad_table);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// Padded segment starts: bin b occupies [seg[b], seg[b] + count_b) of the padded sorted
// order, seg[b + 1] = seg[b] + count_b rounded up to 64; seg[nb] = total.
__global__ void bwd_segments_kernel(const int64_t *__restrict__ offsets, int nb, int64_t *__restrict__ seg) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    int64_t acc = 0;
    for (int b = 0; b < nb; b++) {
        seg[b] = acc;
        acc += (offsets[b + 1] - offsets[b] + 63) / 64 * 64;
    }
    seg[nb] = acc;
}

// Y[c][p'] = w(p) X[p][c] for c < ncols and every padded position p' < pcols (zero where p'
// holds no row), X and Y bf16 hi (+ lo).  wmode: 0 -> 1, 1 -> 1 - t_p, 2 -> t_p.
__global__ void bwd_transpose_rows_kernel(const __nv_bfloat16 *__restrict__ Xhi, const __nv_bfloat16 *__restrict__ Xlo,
                                          int ld, int ncols, const int64_t *__restrict__ offsets,
                                          const int64_t *__restrict__ seg, int nb, const float *__restrict__ tval,
                                          int wmode, int64_t pcols, __nv_bfloat16 *__restrict__ Yhi,
                                          __nv_bfloat16 *__restrict__ Ylo) {
    __shared__ float tile[32][33];
    __shared__ int64_t rowp[32];
    __shared__ float roww[32];
    const int64_t p0 = (int64_t)blockIdx.x * 32;
    const int c0 = blockIdx.y * 32;
    if (threadIdx.y == 0) {
        const int64_t pp = p0 + threadIdx.x;
        int64_t prow = -1;
        float wt = 0.0f;
        if (pp < seg[nb]) {
            int lo = 0, hi = nb - 1;                 // last b with seg[b] <= pp
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (seg[mid] <= pp) lo = mid; else hi = mid - 1;
            }
            const int64_t local = pp - seg[lo];
            if (local < offsets[lo + 1] - offsets[lo]) {
                prow = offsets[lo] + local;
                const float t = tval[prow];
                wt = wmode == 0 ? 1.0f : (wmode == 1 ? 1.0f - t : t);
            }
        }
        rowp[threadIdx.x] = prow;
        roww[threadIdx.x] = wt;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int64_t prow = rowp[r];
        const int c = c0 + threadIdx.x;
        float v = 0.0f;
        if (prow >= 0 && c < ncols) {
            const int64_t i = prow * (int64_t)ld + c;
            v = __bfloat162float(Xhi[i]);
            if (Xlo) v += __bfloat162float(Xlo[i]);
            v *= roww[r];
        }
        tile[r][threadIdx.x] = v;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int c = c0 + r;
        const int64_t pp = p0 + threadIdx.x;
        if (c >= ncols || pp >= pcols) continue;
        const float v = tile[threadIdx.x][r];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        Yhi[(int64_t)c * pcols + pp] = h;
        if (Ylo) Ylo[(int64_t)c * pcols + pp] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

int launch_bwd_segments(const int64_t *offsets, int nb, int64_t *seg, cudaStream_t s) {
    bwd_segments_kernel<<<1, 32, 0, s>>>(offsets, nb, seg);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_bwd_transpose_rows(const __nv_bfloat16 *Xhi, const __nv_bfloat16 *Xlo, int ld, int ncols,
                              const int64_t *offsets, const int64_t *seg, int nb, const float *tval, int wmode,
                              int64_t pcols, __nv_bfloat16 *Yhi, __nv_bfloat16 *Ylo, cudaStream_t s) {
    if (pcols == 0 || ncols == 0) return FEQ_OK;
    if ((pcols + 31) / 32 > 0x7fffffffll || (ncols + 31) / 32 > 65535) return FEQ_ERR_UNSUPPORTED;
    dim3 grid((unsigned)((pcols + 31) / 32), (unsigned)((ncols + 31) / 32));
    bwd_transpose_rows_kernel<<<grid, dim3(32, 8), 0, s>>>(Xhi, Xlo, ld, ncols, offsets, seg, nb, tval, wmode, pcols,
                                                          Yhi, Ylo);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// out[e][c][j] = s^l(j) H[p][base[j] + c] (0 where base < 0): sorted mix rows back to m-first
// edge rows (E, C, D).  One warp per row, staged in shared memory for coalesced stores.
__global__ void unprep_rows_kernel(const float *__restrict__ H, int ld, const float *__restrict__ dist,
                                   const int64_t *__restrict__ perm, int64_t E, int C, int D,
                                   const __grid_constant__ TcPosMap Mp, float sh_scale, float *__restrict__ out) {
    extern __shared__ float un_s[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int row = C * D;
    float *rs = un_s + (size_t)w * row;
    for (int64_t p = (int64_t)blockIdx.x * nw + w; p < E; p += (int64_t)gridDim.x * nw) {
        const int64_t e = perm[p];
        const float dd = dist[e];
        const float s = dd / (dd + sh_scale);
        const float *hr = H + p * (int64_t)ld;
        for (int j = 0; j < D; j++) {
            const int b = Mp.base[j];
            const float sl = ipowf(s, Mp.l[j]);
            for (int c = lane; c < C; c += 32) rs[c * D + j] = b < 0 ? 0.0f : hr[b + c] * sl;
        }
        __syncwarp();
        float *orow = out + e * (int64_t)row;
        for (int i = lane; i < row; i += 32) orow[i] = rs[i];
        __syncwarp();
    }
}

int launch_unprep_rows(const float *H, int ld, const float *dist, const int64_t *perm, int64_t E, int C, int D,
                       const TcPosMap &Mp, float sh_scale, float *out, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const int nw = rows_warps((size_t)C * D);
    if (nw == 0) return FEQ_ERR_UNSUPPORTED;
    const size_t smem = (size_t)nw * C * D * 4;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(unprep_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    unprep_rows_kernel<<<grid_for(E, nw), nw * 32, smem, s>>>(H, ld, dist, perm, E, C, D, Mp, sh_scale, out);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
