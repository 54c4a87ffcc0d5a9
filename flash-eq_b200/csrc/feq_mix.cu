// feq_mix.cu -- the distance-binned block-diagonal radial mix (fp32, CUDA cores).
//
// Reference behaviour replaced: forward_m0_kernel / forward_mpos_kernel
// (flash_eq/cuda/csrc/block_diagonal.cu:558-733).  Per edge e and m-block m:
//   h_m[e, co, o] = sum_ci sum_i s_e^(l_i + l_o) * W(t_e)[co, ci, m, o, i] (x) g_m[e, ci, i]
//   W(t) = (1 - t) T[lo] + t T[lo + 1]
// with (x) the 2x2 [[a, b], [-b, a]] action on (+m, -m) pairs for m > 0.
//
// The reference runs one CTA per edge and reloads two table values per
// multiply-add.  Here edges are grouped by distance bin (all edges of a tile share
// lo), so one CTA = (tile of up to kTileE edges of one bin) x (one m-block): each
// weight pair is loaded once per tile and reused for every edge of the tile from
// registers; the per-edge interpolation is one FMA per weight per edge.  The
// solid-harmonic factor s^(l_i + l_o) is split into s^l_i (applied while staging
// the inputs) and s^l_o (applied in the epilogue).
//
// The table is first re-laid per bin as [block][ci][i][co][o][re/im] so that
// neighbouring threads (neighbouring outputs) read neighbouring weights.
#include <cuda_runtime.h>

#include "feq_internal.cuh"

namespace feq {

constexpr int kTileE = 32;
constexpr int kMixThreads = 128;

// Re-layout of the radial table: native (nb1, Cout, Cin, W) -> per bin
// [block m][ci][i][co*n_out + o][comp] with each (ci, i) row padded to an even count.
__global__ void relayout_table_kernel(const float *__restrict__ T, float *__restrict__ Wt, int nb1,
                                      int Cin, int Cout, const __grid_constant__ MixLayout M) {
    const int64_t per_bin = M.relaid_row;
    const int64_t total = per_bin * nb1;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = idx / per_bin;
        int64_t r = idx - b * per_bin;
        int blk = -1;
        for (int q = 0; q < M.n_blocks; q++) {
            const MixBlock &B = M.blk[q];
            if (B.n_in == 0 || B.n_out == 0) continue;
            const int64_t sz = (int64_t)Cin * B.n_in * B.relaid_stride;
            if (r >= B.relaid_off && r < B.relaid_off + sz) {
                blk = q;
                break;
            }
        }
        float v = 0.0f;
        if (blk >= 0) {
            const MixBlock &B = M.blk[blk];
            const int mult = B.m == 0 ? 1 : 2;
            const int64_t rr = r - B.relaid_off;
            const int row = (int)(rr / B.relaid_stride);       // ci * n_in + i
            const int col = (int)(rr - (int64_t)row * B.relaid_stride);
            const int ci = row / B.n_in, i = row - ci * B.n_in;
            if (col < Cout * B.n_out * mult) {
                const int q = col / mult, comp = col - q * mult;
                const int co = q / B.n_out, o = q - co * B.n_out;
                const int w = B.w_off + mult * (o * B.n_in + i) + comp;
                v = __ldg(T + ((b * Cout + co) * Cin + ci) * (int64_t)M.wdim + w);
            }
        }
        Wt[idx] = v;
    }
}

// One CTA per (tile, m-block).  kCplx: m > 0 (complex pairs); else m = 0 (reals).
// Each thread owns one "unit" of outputs: two consecutive real outputs (m = 0) or
// one complex output (m > 0), for all kTileE edges of the tile.
template <bool kCplx>
__global__ void __launch_bounds__(kMixThreads)
mix_kernel(const float *__restrict__ g, const float *__restrict__ Wt, const float *__restrict__ dist,
           const int64_t *__restrict__ perm, const int4 *__restrict__ tiles,
           const int *__restrict__ num_tiles, int Cin, int Cout, int din, int dout, int blk_id,
           int ci_chunk, const __grid_constant__ MixLayout M, Binning bins, float sh_scale,
           float *__restrict__ h) {
    const int tile_id = blockIdx.x;
    if (tile_id >= *num_tiles) return;
    const MixBlock &B = M.blk[blk_id];
    const int mult = kCplx ? 2 : 1;
    const int n_in = B.n_in, n_out = B.n_out;
    const int4 tl = tiles[tile_id];   // (start, len, bin, -)
    const int len = tl.y, bin = tl.z;

    extern __shared__ float smem[];
    __shared__ float t_s[kTileE];
    __shared__ float sp_s[kTileE][kMaxL + 1];
    __shared__ int64_t eid_s[kTileE];
    __shared__ int8_t lin_s[kMaxIrreps], lout_s[kMaxIrreps];   // degrees, staged off the param bank
    float *g_s = smem;   // [ci_chunk * n_in][kTileE][mult]
    if (threadIdx.x < kMaxIrreps) {
        lin_s[threadIdx.x] = B.l_in[threadIdx.x];
        lout_s[threadIdx.x] = B.l_out[threadIdx.x];
    }

    const int lmax = max(M.lmax_in, M.lmax_out);
    if (threadIdx.x < kTileE) {
        const int k = threadIdx.x;
        float t = 0.0f;
        int64_t e = -1;
        float s = 0.0f;
        if (k < len) {
            e = perm[(int64_t)tl.x + k];
            const float d = dist[e];
            int lo;
            bin_of(d, bins, lo, t);
            s = d / (d + sh_scale);
        }
        t_s[k] = t;
        eid_s[k] = e;
        for (int l = 0; l <= lmax; l++) sp_s[k][l] = (k < len) ? ipowf(s, l) : 0.0f;
    }
    __syncthreads();

    float tr[kTileE];
#pragma unroll
    for (int k = 0; k < kTileE; k++) tr[k] = t_s[k];

    const int n_units = kCplx ? Cout * n_out : (Cout * n_out + 1) / 2;
    const int n_groups = (n_units + kMixThreads - 1) / kMixThreads;
    const int n_chunks = (Cin + ci_chunk - 1) / ci_chunk;
    const int64_t bin_row = M.relaid_row;
    const float *W0 = Wt + (int64_t)bin * bin_row + B.relaid_off;
    const float *W1 = W0 + bin_row;
    const int wstride = B.relaid_stride;

    auto stage = [&](int c0, int cn) {
        const int items = cn * n_in * kTileE * mult;
        for (int idx = threadIdx.x; idx < items; idx += kMixThreads) {
            int comp = kCplx ? (idx & 1) : 0;
            int rest = kCplx ? (idx >> 1) : idx;
            const int k = rest % kTileE;
            rest /= kTileE;
            const int i = rest % n_in, cl = rest / n_in;
            float v = 0.0f;
            const int64_t e = eid_s[k];
            if (e >= 0) {
                v = __ldg(g + (e * Cin + c0 + cl) * (int64_t)din + B.in_off + mult * i + comp);
                v *= sp_s[k][lin_s[i]];
            }
            g_s[idx] = v;
        }
    };

    if (n_chunks == 1) {
        stage(0, Cin);
        __syncthreads();
    }
    for (int grp = 0; grp < n_groups; grp++) {
        const int u = grp * kMixThreads + threadIdx.x;
        const bool active = u < n_units;
        float acc0[kTileE], acc1[kTileE];
#pragma unroll
        for (int k = 0; k < kTileE; k++) {
            acc0[k] = 0.0f;
            acc1[k] = 0.0f;
        }
        for (int ch = 0; ch < n_chunks; ch++) {
            const int c0 = ch * ci_chunk, cn = min(ci_chunk, Cin - c0);
            if (n_chunks > 1) {
                __syncthreads();
                stage(c0, cn);
                __syncthreads();
            }
            if (active) {
                const int rows = cn * n_in;
                const float2 *wp0 = reinterpret_cast<const float2 *>(W0 + (int64_t)(c0 * n_in) * wstride + 2 * u);
                const float2 *wp1 = reinterpret_cast<const float2 *>(W1 + (int64_t)(c0 * n_in) * wstride + 2 * u);
                const int wstep = wstride / 2;   // float2 per (ci, i) row
                float2 nw0 = __ldg(wp0), nw1 = __ldg(wp1);
                for (int row = 0; row < rows; row++) {
                    const float2 w0 = nw0, w1 = nw1;
                    if (row + 1 < rows) {   // prefetch the next row's weights (hides L2 latency)
                        nw0 = __ldg(wp0 + (int64_t)(row + 1) * wstep);
                        nw1 = __ldg(wp1 + (int64_t)(row + 1) * wstep);
                    }
                    const float dx = w1.x - w0.x, dy = w1.y - w0.y;
                    if (kCplx) {
                        const float4 *gr = reinterpret_cast<const float4 *>(g_s + row * kTileE * 2);
#pragma unroll
                        for (int k2 = 0; k2 < kTileE / 2; k2++) {
                            const float4 gv = gr[k2];
                            {
                                const int k = 2 * k2;
                                const float a = fmaf(tr[k], dx, w0.x), b = fmaf(tr[k], dy, w0.y);
                                acc0[k] = fmaf(a, gv.x, fmaf(b, gv.y, acc0[k]));
                                acc1[k] = fmaf(a, gv.y, fmaf(-b, gv.x, acc1[k]));
                            }
                            {
                                const int k = 2 * k2 + 1;
                                const float a = fmaf(tr[k], dx, w0.x), b = fmaf(tr[k], dy, w0.y);
                                acc0[k] = fmaf(a, gv.z, fmaf(b, gv.w, acc0[k]));
                                acc1[k] = fmaf(a, gv.w, fmaf(-b, gv.z, acc1[k]));
                            }
                        }
                    } else {
                        const float4 *gr = reinterpret_cast<const float4 *>(g_s + row * kTileE);
#pragma unroll
                        for (int k4 = 0; k4 < kTileE / 4; k4++) {
                            const float4 gv = gr[k4];
                            const float gg[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                const int k = 4 * k4 + q;
                                acc0[k] = fmaf(fmaf(tr[k], dx, w0.x), gg[q], acc0[k]);
                                acc1[k] = fmaf(fmaf(tr[k], dy, w0.y), gg[q], acc1[k]);
                            }
                        }
                    }
                }
            }
        }
        if (active) {
            if (kCplx) {
                const int co = u / n_out, o = u - co * n_out;
                const int lo_ = lout_s[o];
#pragma unroll
                for (int k = 0; k < kTileE; k++) {
                    if (k < len) {
                        const float sc = sp_s[k][lo_];
                        // out_off may be odd: two scalar stores, never a float2
                        float *dstp = h + (eid_s[k] * Cout + co) * (int64_t)dout + B.out_off + 2 * o;
                        dstp[0] = acc0[k] * sc;
                        dstp[1] = acc1[k] * sc;
                    }
                }
            } else {
                const int q0 = 2 * u, q1 = 2 * u + 1;
                const int co0 = q0 / n_out, o0 = q0 - co0 * n_out;
                const int co1 = q1 / n_out, o1 = q1 - co1 * n_out;
                const bool has1 = q1 < Cout * n_out;
                const int l0 = lout_s[o0], l1 = has1 ? lout_s[o1] : 0;
#pragma unroll
                for (int k = 0; k < kTileE; k++) {
                    if (k < len) {
                        const int64_t e = eid_s[k];
                        h[(e * Cout + co0) * (int64_t)dout + B.out_off + o0] = acc0[k] * sp_s[k][l0];
                        if (has1) h[(e * Cout + co1) * (int64_t)dout + B.out_off + o1] = acc1[k] * sp_s[k][l1];
                    }
                }
            }
        }
    }
}

// Zero the output components of blocks that have no input (the reference output is
// torch::zeros and such blocks are never written, block_diagonal.cu:1309).
__global__ void zero_blocks_kernel(float *__restrict__ h, int64_t E, int Cout, int dout,
                                   const __grid_constant__ MixLayout M, int first_zero_off) {
    const int64_t total = E * Cout;
    const int width = dout - first_zero_off;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total * width;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t rowi = idx / width;
        const int c = (int)(idx - rowi * width);
        h[rowi * dout + first_zero_off + c] = 0.0f;
    }
}

// Tile list: for each bin, ceil(count / kTileE) tiles (start, len, bin).
__global__ void build_tiles_kernel(const int64_t *__restrict__ offsets, int nb, int te, int4 *__restrict__ tiles,
                                   int *__restrict__ num_tiles) {
    __shared__ int partial[1024];
    const int T = blockDim.x;
    const int per = (nb + T - 1) / T;
    const int b0 = threadIdx.x * per, b1 = min(nb, b0 + per);
    int cnt = 0;
    for (int b = b0; b < b1; b++) {
        const int64_t c = offsets[b + 1] - offsets[b];
        cnt += (int)((c + te - 1) / te);
    }
    partial[threadIdx.x] = cnt;
    __syncthreads();
    for (int off = 1; off < T; off <<= 1) {   // inclusive Hillis-Steele scan
        int v = threadIdx.x >= off ? partial[threadIdx.x - off] : 0;
        __syncthreads();
        partial[threadIdx.x] += v;
        __syncthreads();
    }
    int t = partial[threadIdx.x] - cnt;
    for (int b = b0; b < b1; b++) {
        const int64_t s = offsets[b], c = offsets[b + 1] - s;
        for (int64_t k = 0; k < c; k += te) {
            tiles[t++] = make_int4((int)(s + k), (int)min64(te, c - k), b, 0);
        }
    }
    if (threadIdx.x == T - 1) *num_tiles = partial[T - 1];
}

// ---------------------------------------------------------------------------
// Host
// ---------------------------------------------------------------------------
int64_t mix_max_tiles(int64_t E, int nb, int te) { return E / (te > 0 ? te : kTileE) + nb + 1; }

int launch_relayout(const float *T, float *Wt, int nb1, int Cin, int Cout, const MixLayout &M,
                    cudaStream_t s) {
    const int64_t total = M.relaid_row * nb1;
    if (total == 0) return FEQ_OK;
    const int64_t grid = min64((total + 255) / 256, 148 * 16);
    relayout_table_kernel<<<(unsigned)grid, 256, 0, s>>>(T, Wt, nb1, Cin, Cout, M);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_build_tiles(const int64_t *offsets, int nb, int te, int4 *tiles, int *num_tiles, cudaStream_t s) {
    build_tiles_kernel<<<1, 1024, 0, s>>>(offsets, nb, te > 0 ? te : kTileE, tiles, num_tiles);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

constexpr size_t kMixSmemBudget = 96 * 1024;

int launch_mix(const float *g, const float *Wt, const float *dist, const int64_t *perm,
               const int4 *tiles, const int *num_tiles, int64_t max_tiles, int64_t E, int Cin,
               int Cout, int din, int dout, const MixLayout &M, Binning bins, float sh_scale,
               float *h, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    int first_zero = dout;   // out_off of the first block that has outputs but no inputs
    for (int q = 0; q < M.n_blocks; q++) {
        const MixBlock &B = M.blk[q];
        if (B.n_out > 0 && B.n_in == 0) {
            first_zero = B.out_off;
            break;
        }
    }
    if (first_zero < dout) {
        const int64_t work = E * Cout * (int64_t)(dout - first_zero);
        const int64_t grid = min64((work + 255) / 256, 148 * 32);
        zero_blocks_kernel<<<(unsigned)grid, 256, 0, s>>>(h, E, Cout, dout, M, first_zero);
        FEQ_LAUNCH_CHECK();
    }
    for (int q = 0; q < M.n_blocks; q++) {
        const MixBlock &B = M.blk[q];
        if (B.n_in == 0 || B.n_out == 0) continue;
        const int mult = B.m == 0 ? 1 : 2;
        const size_t per_ci = (size_t)B.n_in * kTileE * mult * sizeof(float);
        int ci_chunk = (int)std::min<size_t>((size_t)Cin, kMixSmemBudget / per_ci);
        if (ci_chunk < 1) return FEQ_ERR_UNSUPPORTED;
        const size_t smem = per_ci * ci_chunk;
        if (B.m == 0) {
            FEQ_CUDA_TRY(cudaFuncSetAttribute(mix_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            mix_kernel<false><<<(unsigned)max_tiles, kMixThreads, smem, s>>>(
                g, Wt, dist, perm, tiles, num_tiles, Cin, Cout, din, dout, q, ci_chunk, M, bins, sh_scale, h);
        } else {
            FEQ_CUDA_TRY(cudaFuncSetAttribute(mix_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            mix_kernel<true><<<(unsigned)max_tiles, kMixThreads, smem, s>>>(
                g, Wt, dist, perm, tiles, num_tiles, Cin, Cout, din, dout, q, ci_chunk, M, bins, sh_scale, h);
        }
        FEQ_LAUNCH_CHECK();
    }
    return FEQ_OK;
}

}  // namespace feq
