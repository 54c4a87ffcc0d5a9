// feq_rotate.cu -- per-edge Wigner-D blocks and the rotations into / out of the
// edge frame.
//
// Reference behaviour replaced:
//   WignerDBasis.forward / WignerD.rot_to_ez   flash_eq/representations/wigner.py:198-240, 341-370
//   torch.bmm(edge_features, P)                flash_eq/layers/linear.py:135
//   torch.bmm(out_diag, Q.mT)                  flash_eq/layers/linear.py:160
//   node_features[graph.src] (+ edge_features) flash_eq/layers/attention.py:307-309
//
// The reference evaluates every block with a batched dense matrix exponential of
// the whole (dim x dim) generator.  Here each degree's block is the closed form
//   D_l = R(phi) M_l(theta') R(phi)^T,  M_l = sum_k coef_k(theta') T_l[:, :, k]
// (derivation and tables: gen_wigner_tables.py), evaluated in shared memory per
// edge.  The direction is reduced to (theta, phi) with the reference's own float32
// steps (normalise with +eps, axis (-d_y, d_x) / (|.| + eps), theta = acos of the
// clamped d_z) so degenerate inputs land where the reference does: d = 0 and
// d = -e_z give the identity, as matrix_exp of a zero generator does.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "feq_internal.cuh"
#include "_build/feq_wigner_tables.inc"

namespace feq {

constexpr float kEps = 1e-8f;   // get_epsilon(float32), flash_eq/utils.py:19-27

// Per-edge trig state: cos/sin(m theta') and cos/sin(m phi) for m = 0..lmax.
struct EdgeTrig {
    float ct[kMaxL + 1], st[kMaxL + 1], cp[kMaxL + 1], sp[kMaxL + 1];
};

__device__ __forceinline__ void edge_trig(float vx, float vy, float vz, int lmax, EdgeTrig &tr) {
    float nv = sqrtf(vx * vx + vy * vy + vz * vz);
    float den = nv + kEps;
    float dx = vx / den, dy = vy / den, dz = vz / den;
    float n = sqrtf(dy * dy + dx * dx);
    float ax0 = -dy / (n + kEps), ax1 = dx / (n + kEps);
    float theta = acosf(fminf(fmaxf(dz, -1.0f + kEps), 1.0f - kEps));
    float rho = sqrtf(ax0 * ax0 + ax1 * ax1);
    float th = theta * rho;
    float c1p = 1.0f, s1p = 0.0f;
    if (rho > 0.0f) {
        c1p = ax0 / rho;
        s1p = ax1 / rho;
    }
    float c1t, s1t;
    sincosf(th, &s1t, &c1t);
    tr.ct[0] = 1.0f; tr.st[0] = 0.0f; tr.cp[0] = 1.0f; tr.sp[0] = 0.0f;
    float ct = 1.0f, st = 0.0f, cp = 1.0f, sp = 0.0f;
    for (int m = 1; m <= lmax; m++) {
        float nct = ct * c1t - st * s1t, nst = st * c1t + ct * s1t;
        float ncp = cp * c1p - sp * s1p, nsp = sp * c1p + cp * s1p;
        ct = nct; st = nst; cp = ncp; sp = nsp;
        tr.ct[m] = ct; tr.st[m] = st; tr.cp[m] = cp; tr.sp[m] = sp;
    }
}

// Cooperative build of every distinct-degree block of `nedges` edges.
//   trig_s : nedges EdgeTrig
//   m_s    : nedges * L.dblock_floats scratch (M blocks)
//   d_s    : nedges * L.dblock_floats output (D blocks, row-major (2l+1)^2 each)
// Ends with __syncthreads().
__device__ void build_dblocks(const ReprLayout &L, int nedges, const EdgeTrig *trig_s, float *m_s,
                              float *d_s) {
    const int per = L.dblock_floats;
    const int total = nedges * per;
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        int e = idx / per, r = idx - e * per;
        int u = 0;
        while (u + 1 < L.n_unique && L.unique_doff[u + 1] <= r) u++;
        const int l = L.unique_l[u], n = 2 * l + 1;
        const int pq = r - L.unique_doff[u];
        const float *t = feq_wt_data + feq_wt_offset[l] + pq * n;
        const EdgeTrig &tr = trig_s[e];
        float acc = __ldg(t);
        for (int m = 1; m <= l; m++) {
            acc = fmaf(__ldg(t + 2 * m - 1), tr.ct[m], acc);
            acc = fmaf(__ldg(t + 2 * m), tr.st[m], acc);
        }
        m_s[idx] = acc;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        int e = idx / per, r = idx - e * per;
        int u = 0;
        while (u + 1 < L.n_unique && L.unique_doff[u + 1] <= r) u++;
        const int l = L.unique_l[u], n = 2 * l + 1;
        const int pq = r - L.unique_doff[u];
        const int a = pq / n, b = pq - a * n;
        const int ma = a < l ? l - a : a - l, mb = b < l ? l - b : b - l;
        const int abar = 2 * l - a, bbar = 2 * l - b;
        const EdgeTrig &tr = trig_s[e];
        const float ca = tr.cp[ma], cb = tr.cp[mb];
        const float sa = a < l ? tr.sp[ma] : -tr.sp[ma];   // R[a][abar]; zero when a == l
        const float sb = b < l ? tr.sp[mb] : -tr.sp[mb];
        const float *M = m_s + e * per + L.unique_doff[u];
        float v = ca * cb * M[a * n + b];
        if (mb) v = fmaf(ca * sb, M[a * n + bbar], v);
        if (ma) v = fmaf(sa * cb, M[abar * n + b], v);
        if (ma && mb) v = fmaf(sa * sb, M[abar * n + bbar], v);
        d_s[idx] = v;
    }
    __syncthreads();
}

// Kernel parameters live in the constant bank: indexing them with a per-thread index
// serialises a warp's reads.  Each kernel therefore copies its layout struct into
// shared memory once and reads it from there.
static_assert(sizeof(ReprLayout) % 4 == 0, "ReprLayout is copied as 32-bit words");
__device__ __forceinline__ void stage_layout(const ReprLayout &src, ReprLayout &dst) {
    const int *s = reinterpret_cast<const int *>(&src);
    int *d = reinterpret_cast<int *>(&dst);
    for (int i = threadIdx.x; i < (int)(sizeof(ReprLayout) / 4); i += blockDim.x) d[i] = s[i];
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Dense basis output (API compatibility with WignerDBasis / rot_to_ez).
// ---------------------------------------------------------------------------
__global__ void basis_kernel(const float *__restrict__ dirs, int64_t E, const __grid_constant__ ReprLayout Lp,
                             int layout, int epb, float *__restrict__ out) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    stage_layout(Lp, L);
    EdgeTrig *trig_s = reinterpret_cast<EdgeTrig *>(smem);
    float *m_s = reinterpret_cast<float *>(trig_s + epb);
    float *d_s = m_s + epb * L.dblock_floats;
    const int64_t e0 = (int64_t)blockIdx.x * epb;
    const int ne = (int)min64(epb, E - e0);
    if (threadIdx.x < ne) {
        const float *v = dirs + (e0 + threadIdx.x) * 3;
        edge_trig(v[0], v[1], v[2], L.lmax, trig_s[threadIdx.x]);
    }
    __syncthreads();
    build_dblocks(L, ne, trig_s, m_s, d_s);
    const int d = L.dim, dd = d * d;
    for (int idx = threadIdx.x; idx < ne * dd; idx += blockDim.x) {
        int e = idx / dd, r = idx - e * dd;
        int k = r / d, j = r - k * d;
        float v = 0.0f;
        int row_std, col_std;
        if (layout == FEQ_BASIS_MFIRST) {          // M[k][j] = D[k][perm[j]]
            row_std = k;
            col_std = L.perm[j];
        } else {                                   // rot_to_ez = D^T in std order
            row_std = j;
            col_std = k;
        }
        const int ir = L.std_irrep[row_std];
        if (L.std_irrep[col_std] == ir) {
            const int l = L.irrep_l[ir], n = 2 * l + 1, off = L.irrep_off[ir];
            const float *D = d_s + e * L.dblock_floats + L.unique_doff[L.irrep_slot[ir]];
            v = D[(row_std - off) * n + (col_std - off)];
        }
        out[(e0 + e) * dd + r] = v;
    }
}

// ---------------------------------------------------------------------------
// Rotate into the edge frame: g[e][c][j] = sum_k f[e][c][k] P[e][k][j]
// (P = D[:, perm], block sparse when built from the direction).
// ---------------------------------------------------------------------------
template <bool kDense, bool kGather>
__global__ void rotate_in_kernel(const float *__restrict__ x, const int64_t *__restrict__ src,
                                 int64_t nsrc, const float *__restrict__ edge_add,
                                 const float *__restrict__ dirs, const float *__restrict__ P,
                                 int64_t E, int C, const __grid_constant__ ReprLayout Lp, int epb,
                                 float *__restrict__ g, int32_t *status) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    stage_layout(Lp, L);
    const int d = L.dim, row = C * d;
    float *f_s = smem;                                   // epb * row
    float *b_s = f_s + epb * row;                        // basis area
    const int64_t e0 = (int64_t)blockIdx.x * epb;
    const int ne = (int)min64(epb, E - e0);

    // stage input rows (gather by src, add edge_add)
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        int e = idx / row, r = idx - e * row;
        int64_t ge = e0 + e;
        float v;
        if (kGather) {
            int64_t s = src[ge];
            if (s < 0 || s >= nsrc) {
                set_status(status, 1);
                v = 0.0f;
            } else {
                v = __ldg(x + s * row + r);
            }
        } else {
            v = __ldg(x + ge * row + r);
        }
        if (edge_add) v += __ldg(edge_add + ge * row + r);
        f_s[idx] = v;
    }
    const float *D_s;
    if (kDense) {
        float *p_s = b_s;
        const int dd = d * d;
        for (int idx = threadIdx.x; idx < ne * dd; idx += blockDim.x)
            p_s[idx] = __ldg(P + e0 * dd + idx);
        __syncthreads();
        D_s = p_s;
    } else {
        EdgeTrig *trig_s = reinterpret_cast<EdgeTrig *>(b_s);
        float *m_s = reinterpret_cast<float *>(trig_s + epb);
        float *d_s = m_s + epb * L.dblock_floats;
        if (threadIdx.x < ne) {
            const float *v = dirs + (e0 + threadIdx.x) * 3;
            edge_trig(v[0], v[1], v[2], L.lmax, trig_s[threadIdx.x]);
        }
        __syncthreads();
        build_dblocks(L, ne, trig_s, m_s, d_s);
        D_s = d_s;
    }
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        int e = idx / row, r = idx - e * row;
        int c = r / d, j = r - c * d;
        const float *fr = f_s + e * row + c * d;
        float acc = 0.0f;
        if (kDense) {
            const float *Pe = D_s + e * d * d;
            for (int k = 0; k < d; k++) acc = fmaf(fr[k], Pe[k * d + j], acc);
        } else {
            const int ps = L.perm[j];
            const int ir = L.std_irrep[ps];
            const int l = L.irrep_l[ir], n = 2 * l + 1, off = L.irrep_off[ir];
            const int col = ps - off;
            const float *De = D_s + e * L.dblock_floats + L.unique_doff[L.irrep_slot[ir]];
            for (int k = 0; k < n; k++) acc = fmaf(fr[off + k], De[k * n + col], acc);
        }
        g[(e0 + e) * row + r] = acc;
    }
}

// ---------------------------------------------------------------------------
// Rotate back: out[e][c][k] = sum_j h[e][c][j] Q[e][k][j].
// ---------------------------------------------------------------------------
template <bool kDense>
__global__ void rotate_out_kernel(const float *__restrict__ h, const float *__restrict__ dirs,
                                  const float *__restrict__ Q, int64_t E, int C,
                                  const __grid_constant__ ReprLayout Lp, int epb, float *__restrict__ out) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    stage_layout(Lp, L);
    const int d = L.dim, row = C * d;
    float *h_s = smem;
    float *b_s = h_s + epb * row;
    const int64_t e0 = (int64_t)blockIdx.x * epb;
    const int ne = (int)min64(epb, E - e0);
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) h_s[idx] = __ldg(h + e0 * row + idx);
    const float *D_s;
    if (kDense) {
        const int dd = d * d;
        for (int idx = threadIdx.x; idx < ne * dd; idx += blockDim.x) b_s[idx] = __ldg(Q + e0 * dd + idx);
        __syncthreads();
        D_s = b_s;
    } else {
        EdgeTrig *trig_s = reinterpret_cast<EdgeTrig *>(b_s);
        float *m_s = reinterpret_cast<float *>(trig_s + epb);
        float *d_s = m_s + epb * L.dblock_floats;
        if (threadIdx.x < ne) {
            const float *v = dirs + (e0 + threadIdx.x) * 3;
            edge_trig(v[0], v[1], v[2], L.lmax, trig_s[threadIdx.x]);
        }
        __syncthreads();
        build_dblocks(L, ne, trig_s, m_s, d_s);
        D_s = d_s;
    }
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        int e = idx / row, r = idx - e * row;
        int c = r / d, k = r - c * d;
        const float *hr = h_s + e * row + c * d;
        float acc = 0.0f;
        if (kDense) {
            const float *Qe = D_s + e * d * d + k * d;
            for (int j = 0; j < d; j++) acc = fmaf(hr[j], Qe[j], acc);
        } else {
            const int ir = L.std_irrep[k];
            const int l = L.irrep_l[ir], n = 2 * l + 1, off = L.irrep_off[ir];
            const float *De = D_s + e * L.dblock_floats + L.unique_doff[L.irrep_slot[ir]] + (k - off) * n;
            for (int col = 0; col < n; col++) acc = fmaf(hr[L.inv_perm[off + col]], De[col], acc);
        }
        out[(e0 + e) * row + r] = acc;
    }
}

// ---------------------------------------------------------------------------
// Launchers (host)
// ---------------------------------------------------------------------------
static size_t basis_area_floats(const ReprLayout &L, int epb, bool dense) {
    if (dense) return (size_t)epb * L.dim * L.dim;
    return (size_t)epb * (sizeof(EdgeTrig) / sizeof(float)) + 2 * (size_t)epb * L.dblock_floats;
}

static int pick_epb(size_t per_edge_floats, size_t fixed_floats, size_t budget_bytes, int max_epb) {
    int epb = max_epb;
    while (epb > 1 && (fixed_floats + per_edge_floats * epb) * 4 > budget_bytes) epb--;
    return epb;
}

constexpr size_t kSmemBudget = 96 * 1024;

int launch_basis(const float *dirs, int64_t E, const ReprLayout &L, int layout, float *out,
                 cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const size_t per = sizeof(EdgeTrig) / sizeof(float) + 2 * (size_t)L.dblock_floats;
    const int epb = pick_epb(per, 0, kSmemBudget, 16);
    const size_t smem = per * epb * 4;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(basis_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t grid = (E + epb - 1) / epb;
    basis_kernel<<<(unsigned)grid, 256, smem, s>>>(dirs, E, L, layout, epb, out);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_rotate_in(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add,
                     const float *dirs, const float *P, int64_t E, int C, const ReprLayout &L,
                     float *g, int32_t *status, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const bool dense = dirs == nullptr;
    const size_t row = (size_t)C * L.dim;
    const size_t per = row + basis_area_floats(L, 1, dense);
    if (per * 4 > kSmemBudget) return FEQ_ERR_UNSUPPORTED;
    const int epb = pick_epb(per, 0, kSmemBudget, 8);
    const size_t smem = per * epb * 4;
    const int64_t grid = (E + epb - 1) / epb;
#define FEQ_ROT_IN(D, G)                                                                               \
    do {                                                                                               \
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_in_kernel<D, G>,                                      \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));    \
        rotate_in_kernel<D, G><<<(unsigned)grid, 256, smem, s>>>(x, src, nsrc, edge_add, dirs, P, E, C, \
                                                                 L, epb, g, status);                  \
    } while (0)
    if (dense) {
        if (src) FEQ_ROT_IN(true, true); else FEQ_ROT_IN(true, false);
    } else {
        if (src) FEQ_ROT_IN(false, true); else FEQ_ROT_IN(false, false);
    }
#undef FEQ_ROT_IN
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_rotate_out(const float *h, const float *dirs, const float *Q, int64_t E, int C,
                      const ReprLayout &L, float *out, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const bool dense = dirs == nullptr;
    const size_t row = (size_t)C * L.dim;
    const size_t per = row + basis_area_floats(L, 1, dense);
    if (per * 4 > kSmemBudget) return FEQ_ERR_UNSUPPORTED;
    const int epb = pick_epb(per, 0, kSmemBudget, 8);
    const size_t smem = per * epb * 4;
    const int64_t grid = (E + epb - 1) / epb;
    if (dense) {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_out_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        rotate_out_kernel<true><<<(unsigned)grid, 256, smem, s>>>(h, dirs, Q, E, C, L, epb, out);
    } else {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_out_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        rotate_out_kernel<false><<<(unsigned)grid, 256, smem, s>>>(h, dirs, Q, E, C, L, epb, out);
    }
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq

// ===========================================================================
// Tensor-core path: producer of the GEMM's A rows and consumer of its output rows.
// One warp per edge; rows are in bin-sorted order p, edge e = perm[p].  A and H
// columns put the channel fastest, so lane = channel touches consecutive addresses.
// ===========================================================================
namespace feq {

static_assert(sizeof(TcPosMap) % 4 == 0, "TcPosMap is copied as 32-bit words");
constexpr int kTcWarps = 8;

__device__ __forceinline__ void stage_posmap(const TcPosMap &src, TcPosMap &dst) {
    const int *s = reinterpret_cast<const int *>(&src);
    int *d = reinterpret_cast<int *>(&dst);
    for (int i = threadIdx.x; i < (int)(sizeof(TcPosMap) / 4); i += blockDim.x) d[i] = s[i];
}

// Warp-cooperative version of build_dblocks for one edge.
__device__ void build_dblocks_warp(const ReprLayout &L, const EdgeTrig &tr, float *m_s, float *d_s, int lane) {
    const int per = L.dblock_floats;
    for (int r = lane; r < per; r += 32) {
        int u = 0;
        while (u + 1 < L.n_unique && L.unique_doff[u + 1] <= r) u++;
        const int l = L.unique_l[u], n = 2 * l + 1;
        const float *t = feq_wt_data + feq_wt_offset[l] + (r - L.unique_doff[u]) * n;
        float acc = __ldg(t);
        for (int m = 1; m <= l; m++) {
            acc = fmaf(__ldg(t + 2 * m - 1), tr.ct[m], acc);
            acc = fmaf(__ldg(t + 2 * m), tr.st[m], acc);
        }
        m_s[r] = acc;
    }
    __syncwarp();
    for (int r = lane; r < per; r += 32) {
        int u = 0;
        while (u + 1 < L.n_unique && L.unique_doff[u + 1] <= r) u++;
        const int l = L.unique_l[u], n = 2 * l + 1;
        const int pq = r - L.unique_doff[u];
        const int a = pq / n, b = pq - a * n;
        const int ma = a < l ? l - a : a - l, mb = b < l ? l - b : b - l;
        const float ca = tr.cp[ma], cb = tr.cp[mb];
        const float sa = a < l ? tr.sp[ma] : -tr.sp[ma];
        const float sb = b < l ? tr.sp[mb] : -tr.sp[mb];
        const float *M = m_s + L.unique_doff[u];
        float v = ca * cb * M[a * n + b];
        if (mb) v = fmaf(ca * sb, M[a * n + (2 * l - b)], v);
        if (ma) v = fmaf(sa * cb, M[(2 * l - a) * n + b], v);
        if (ma && mb) v = fmaf(sa * sb, M[(2 * l - a) * n + (2 * l - b)], v);
        d_s[r] = v;
    }
    __syncwarp();
}

// Floats of the per-warp basis area (trig + M + D blocks, or a dense d x d matrix).
__host__ __device__ inline int tc_warp_basis_floats(const ReprLayout &L, bool dense) {
    return dense ? L.dim * L.dim : (int)(sizeof(EdgeTrig) / sizeof(float)) + 2 * L.dblock_floats;
}

// y[col] = sum_q f[q] D[q*N + col] (kIn: rotate into the edge frame, D^T applied) or
// y[kk] = sum_col f[col] D[kk*N + col] (rotate back).  f in registers, D broadcast.
template <int N, bool kIn, typename Emit>
__device__ __forceinline__ void rotate_block(const float *__restrict__ fsrc, const float *__restrict__ D, Emit emit) {
    float f[N];
#pragma unroll
    for (int q = 0; q < N; q++) f[q] = fsrc[q];
#pragma unroll
    for (int o = 0; o < N; o++) {
        float acc = 0.0f;
#pragma unroll
        for (int q = 0; q < N; q++) acc = fmaf(f[q], kIn ? D[q * N + o] : D[o * N + q], acc);
        emit(o, acc);
    }
}

template <bool kIn, typename Emit>
__device__ __forceinline__ void rotate_block_any(int l, const float *__restrict__ fsrc, const float *__restrict__ D,
                                                 Emit emit) {
    switch (l) {
        case 0: rotate_block<1, kIn>(fsrc, D, emit); break;
        case 1: rotate_block<3, kIn>(fsrc, D, emit); break;
        case 2: rotate_block<5, kIn>(fsrc, D, emit); break;
        case 3: rotate_block<7, kIn>(fsrc, D, emit); break;
        case 4: rotate_block<9, kIn>(fsrc, D, emit); break;
        default: {
            const int n = 2 * l + 1;
            for (int o = 0; o < n; o++) {
                float acc = 0.0f;
                for (int q = 0; q < n; q++) acc = fmaf(fsrc[q], kIn ? D[q * n + o] : D[o * n + q], acc);
                emit(o, acc);
            }
        }
    }
}

// A[p][base(k) + c] = (f[e][c] . P)[k] * s_e^l(k) as bf16 (hi [, lo]); tval[p] = t_e.
// Lane = channel: each column store of the warp covers 32 consecutive bf16.
template <bool kDense, bool kGather, bool kSplit>
__global__ void __launch_bounds__(kTcWarps * 32)
rotate_in_tc_kernel(const float *__restrict__ x, const int64_t *__restrict__ src, int64_t nsrc,
                    const float *__restrict__ edge_add, const float *__restrict__ dirs, const float *__restrict__ P,
                    const float *__restrict__ dist, const int64_t *__restrict__ perm, int64_t E, int C,
                    const __grid_constant__ ReprLayout Lp, const __grid_constant__ TcPosMap Mp, int k_total,
                    Binning bins, float sh_scale, int per_warp, __nv_bfloat16 *__restrict__ A_hi,
                    __nv_bfloat16 *__restrict__ A_lo, float *__restrict__ tval, int32_t *status) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    __shared__ TcPosMap Mm;
    stage_posmap(Mp, Mm);
    stage_layout(Lp, L);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int d = L.dim, ds = d | 1, row = C * d;
    float *ws = smem + (size_t)w * per_warp;
    float *fs = ws + tc_warp_basis_floats(L, kDense);        // 32 x ds
    EdgeTrig *trig = reinterpret_cast<EdgeTrig *>(ws);
    float *m_s = ws + sizeof(EdgeTrig) / sizeof(float);
    float *d_s = m_s + L.dblock_floats;
    for (int64_t p = (int64_t)blockIdx.x * kTcWarps + w; p < E; p += (int64_t)gridDim.x * kTcWarps) {
        const int64_t e = perm[p];
        const float dd = dist[e];
        const float s = dd / (dd + sh_scale);
        int64_t xrow = e;
        if (kGather) {
            xrow = src[e];
            if (xrow < 0 || xrow >= nsrc) {
                if (lane == 0) set_status(status, 1);
                xrow = -1;
            }
        }
        if (lane == 0) {
            int lo;
            float t;
            bin_of(dd, bins, lo, t);
            tval[p] = t;
            if (!kDense) edge_trig(dirs[e * 3], dirs[e * 3 + 1], dirs[e * 3 + 2], L.lmax, *trig);
        }
        if (kDense) {
            for (int i = lane; i < d * d; i += 32) ws[i] = __ldg(P + e * d * d + i);
        }
        __nv_bfloat16 *ah = A_hi + p * (int64_t)k_total;
        __nv_bfloat16 *al = kSplit ? A_lo + p * (int64_t)k_total : nullptr;
        for (int r = 0; r < Mm.n_pad; r++)
            for (int i = Mm.pad_lo[r] + lane; i < Mm.pad_hi[r]; i += 32) {
                ah[i] = __float2bfloat16_rn(0.0f);
                if (kSplit) al[i] = __float2bfloat16_rn(0.0f);
            }
        __syncwarp();
        if (!kDense) build_dblocks_warp(L, *trig, m_s, d_s, lane);
        for (int c0 = 0; c0 < C; c0 += 32) {
            const int nch = min(32, C - c0);
            for (int i = lane; i < nch * d; i += 32) {
                const int c = i / d, q = i - c * d;
                float v = xrow >= 0 ? __ldg(x + xrow * row + (c0 + c) * d + q) : 0.0f;
                if (edge_add) v += __ldg(edge_add + e * row + (c0 + c) * d + q);
                fs[c * ds + q] = v;
            }
            __syncwarp();
            if (lane < nch) {
                const float *fr = fs + lane * ds;
                const int c = c0 + lane;
                auto put = [&](int b, float v) {
                    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
                    ah[b + c] = hi;
                    if (kSplit) al[b + c] = __float2bfloat16_rn(v - __bfloat162float(hi));
                };
                if (kDense) {
                    for (int j = 0; j < d; j++) {
                        const int b = Mm.base[j];
                        if (b < 0) continue;
                        float acc = 0.0f;
                        for (int q = 0; q < d; q++) acc = fmaf(fr[q], ws[q * d + j], acc);
                        put(b, acc * ipowf(s, Mm.l[j]));
                    }
                } else {
                    for (int r = 0; r < L.n_irreps; r++) {
                        const int l = L.irrep_l[r], off = L.irrep_off[r];
                        const float *D = d_s + L.unique_doff[L.irrep_slot[r]];
                        const float sl = ipowf(s, l);
                        const int32_t *bstd = Mm.base_std + off;
                        rotate_block_any<true>(l, fr + off, D, [&](int col, float v) {
                            const int b = bstd[col];
                            if (b >= 0) put(b, v * sl);
                        });
                    }
                }
            }
            __syncwarp();
        }
    }
}

// out[e][c][k] = sum_j h[c][j] Q[e][k][j], h[c][j] = H[p][base(j) + c] * s_e^l(j)
// (0 where base < 0: output blocks that receive no input).  Output rows are staged
// per 32-channel chunk and written contiguously.
template <bool kDense>
__global__ void __launch_bounds__(kTcWarps * 32)
rotate_out_tc_kernel(const float *__restrict__ H, int h_ld, const float *__restrict__ dirs,
                     const float *__restrict__ Q, const float *__restrict__ dist, const int64_t *__restrict__ perm,
                     int64_t E, int C, const __grid_constant__ ReprLayout Lp, const __grid_constant__ TcPosMap Mp,
                     float sh_scale, int per_warp, float *__restrict__ out) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    __shared__ TcPosMap Mm;
    stage_posmap(Mp, Mm);
    stage_layout(Lp, L);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int d = L.dim, ds = d | 1, row = C * d;
    float *ws = smem + (size_t)w * per_warp;
    float *hs = ws + tc_warp_basis_floats(L, kDense);        // 32 x ds (standard order)
    float *os = hs + 32 * ds;                                 // 32 x ds
    EdgeTrig *trig = reinterpret_cast<EdgeTrig *>(ws);
    float *m_s = ws + sizeof(EdgeTrig) / sizeof(float);
    float *d_s = m_s + L.dblock_floats;
    for (int64_t p = (int64_t)blockIdx.x * kTcWarps + w; p < E; p += (int64_t)gridDim.x * kTcWarps) {
        const int64_t e = perm[p];
        const float dd = dist[e];
        const float s = dd / (dd + sh_scale);
        if (kDense) {
            for (int i = lane; i < d * d; i += 32) ws[i] = __ldg(Q + e * d * d + i);
        } else if (lane == 0) {
            edge_trig(dirs[e * 3], dirs[e * 3 + 1], dirs[e * 3 + 2], L.lmax, *trig);
        }
        __syncwarp();
        if (!kDense) build_dblocks_warp(L, *trig, m_s, d_s, lane);
        const float *hp = H + p * (int64_t)h_ld;
        float *op = out + e * (int64_t)row;
        for (int c0 = 0; c0 < C; c0 += 32) {
            const int nch = min(32, C - c0);
            if (lane < nch) {
                for (int k = 0; k < d; k++) {
                    const int b = Mm.base_std[k];
                    hs[lane * ds + k] = b < 0 ? 0.0f : __ldg(hp + b + c0 + lane) * ipowf(s, L.irrep_l[L.std_irrep[k]]);
                }
                const float *hr = hs + lane * ds;
                float *orow = os + lane * ds;
                if (kDense) {
                    // dense Q is indexed by m-first columns: h in m-first order is hr[perm[j]]
                    for (int k = 0; k < d; k++) {
                        float acc = 0.0f;
                        for (int j = 0; j < d; j++) acc = fmaf(hr[L.perm[j]], ws[k * d + j], acc);
                        orow[k] = acc;
                    }
                } else {
                    for (int r = 0; r < L.n_irreps; r++) {
                        const int l = L.irrep_l[r], off = L.irrep_off[r];
                        const float *D = d_s + L.unique_doff[L.irrep_slot[r]];
                        rotate_block_any<false>(l, hr + off, D, [&](int kk, float v) { orow[off + kk] = v; });
                    }
                }
            }
            __syncwarp();
            for (int i = lane; i < nch * d; i += 32) {
                const int c = i / d, k = i - c * d;
                op[c0 * d + i] = os[c * ds + k];
            }
            __syncwarp();
        }
    }
}

static int tc_grid(int64_t E, size_t smem) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int per_sm = (int)std::max<size_t>(1, std::min<size_t>(4, (200 * 1024) / (smem + 12 * 1024)));
    return (int)min64((E + kTcWarps - 1) / kTcWarps, (int64_t)sms * per_sm * 8);
}

int launch_rotate_in_tc(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add, const float *dirs,
                        const float *P, const float *dist, const int64_t *perm, int64_t E, int C,
                        const ReprLayout &L, const TcPosMap &M, int k_total, Binning bins, float sh_scale,
                        bool split, __nv_bfloat16 *A_hi, __nv_bfloat16 *A_lo, float *tval, int32_t *status,
                        cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const bool dense = dirs == nullptr;
    const int per_warp = (tc_warp_basis_floats(L, dense) + 32 * (L.dim | 1) + 3) & ~3;
    const size_t smem = (size_t)per_warp * kTcWarps * 4;
    if (smem > 200 * 1024) return FEQ_ERR_UNSUPPORTED;
    const int grid = tc_grid(E, smem);
#define FEQ_ROT_IN_TC(D, G, S)                                                                              \
    do {                                                                                                    \
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_in_tc_kernel<D, G, S>,                                     \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));         \
        rotate_in_tc_kernel<D, G, S><<<(unsigned)grid, kTcWarps * 32, smem, s>>>(                           \
            x, src, nsrc, edge_add, dirs, P, dist, perm, E, C, L, M, k_total, bins, sh_scale, per_warp, A_hi, \
            A_lo, tval, status);                                                                            \
    } while (0)
    if (dense) {
        if (src) {
            if (split) FEQ_ROT_IN_TC(true, true, true); else FEQ_ROT_IN_TC(true, true, false);
        } else {
            if (split) FEQ_ROT_IN_TC(true, false, true); else FEQ_ROT_IN_TC(true, false, false);
        }
    } else {
        if (src) {
            if (split) FEQ_ROT_IN_TC(false, true, true); else FEQ_ROT_IN_TC(false, true, false);
        } else {
            if (split) FEQ_ROT_IN_TC(false, false, true); else FEQ_ROT_IN_TC(false, false, false);
        }
    }
#undef FEQ_ROT_IN_TC
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

int launch_rotate_out_tc(const float *H, int h_ld, const float *dirs, const float *Q, const float *dist,
                         const int64_t *perm, int64_t E, int C, const ReprLayout &L, const TcPosMap &M,
                         float sh_scale, float *out, cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const bool dense = dirs == nullptr;
    const int per_warp = (tc_warp_basis_floats(L, dense) + 64 * (L.dim | 1) + 3) & ~3;
    const size_t smem = (size_t)per_warp * kTcWarps * 4;
    if (smem > 200 * 1024) return FEQ_ERR_UNSUPPORTED;
    const int grid = tc_grid(E, smem);
    if (dense) {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_out_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        rotate_out_tc_kernel<true><<<(unsigned)grid, kTcWarps * 32, smem, s>>>(H, h_ld, dirs, Q, dist, perm, E, C, L,
                                                                               M, sh_scale, per_warp, out);
    } else {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_out_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        rotate_out_tc_kernel<false><<<(unsigned)grid, kTcWarps * 32, smem, s>>>(H, h_ld, dirs, Q, dist, perm, E, C,
                                                                                L, M, sh_scale, per_warp, out);
    }
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
