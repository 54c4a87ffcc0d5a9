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
// Rows are in bin-sorted order p; edge e = perm[p].
// ===========================================================================
namespace feq {

static_assert(sizeof(TcPosMap) % 4 == 0, "TcPosMap is copied as 32-bit words");

__device__ __forceinline__ void stage_posmap(const TcPosMap &src, TcPosMap &dst) {
    const int *s = reinterpret_cast<const int *>(&src);
    int *d = reinterpret_cast<int *>(&dst);
    for (int i = threadIdx.x; i < (int)(sizeof(TcPosMap) / 4); i += blockDim.x) d[i] = s[i];
}

// A[p][map.base[j] + c * map.stride[j]] = (g[e][c][j]) * s_e^l(j), as bf16 (hi [, lo]).
// g = f . P with f = x[src[e]] (+ edge_add[e]) or x[e].  Also tval[p] = t_e.
template <bool kDense, bool kGather, bool kSplit>
__global__ void rotate_in_tc_kernel(const float *__restrict__ x, const int64_t *__restrict__ src, int64_t nsrc,
                                    const float *__restrict__ edge_add, const float *__restrict__ dirs,
                                    const float *__restrict__ P, const float *__restrict__ dist,
                                    const int64_t *__restrict__ perm, int64_t E, int C,
                                    const __grid_constant__ ReprLayout Lp, const __grid_constant__ TcPosMap Mp,
                                    int k_total, Binning bins, float sh_scale, int epb,
                                    __nv_bfloat16 *__restrict__ A_hi, __nv_bfloat16 *__restrict__ A_lo,
                                    float *__restrict__ tval, int32_t *status) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    __shared__ TcPosMap Mm;
    __shared__ float sp_s[16][kMaxL + 1];
    __shared__ int64_t eid_s[16];
    stage_posmap(Mp, Mm);
    stage_layout(Lp, L);
    const int d = L.dim, row = C * d;
    const int64_t p0 = (int64_t)blockIdx.x * epb;
    const int ne = (int)min64(epb, E - p0);
    float *f_s = smem;                          // epb * row
    float *a_s = f_s + epb * row;               // epb * k_total (fp32 staging of the A rows)
    float *b_s = a_s + epb * k_total;           // basis area
    if (threadIdx.x < ne) {
        const int64_t e = perm[p0 + threadIdx.x];
        eid_s[threadIdx.x] = e;
        const float dd = dist[e];
        int lo;
        float t;
        bin_of(dd, bins, lo, t);
        tval[p0 + threadIdx.x] = t;
        const float s = dd / (dd + sh_scale);
        for (int l = 0; l <= L.lmax; l++) sp_s[threadIdx.x][l] = ipowf(s, l);
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        const int k = idx / row, r = idx - k * row;
        const int64_t e = eid_s[k];
        float v;
        if (kGather) {
            const int64_t s = src[e];
            if (s < 0 || s >= nsrc) {
                set_status(status, 1);
                v = 0.0f;
            } else {
                v = __ldg(x + s * row + r);
            }
        } else {
            v = __ldg(x + e * row + r);
        }
        if (edge_add) v += __ldg(edge_add + e * row + r);
        f_s[idx] = v;
    }
    for (int idx = threadIdx.x; idx < ne * k_total; idx += blockDim.x) a_s[idx] = 0.0f;   // K padding
    const float *D_s;
    if (kDense) {
        const int dd2 = d * d;
        for (int idx = threadIdx.x; idx < ne * dd2; idx += blockDim.x) {
            const int k = idx / dd2;
            b_s[idx] = __ldg(P + eid_s[k] * dd2 + (idx - k * dd2));
        }
        __syncthreads();
        D_s = b_s;
    } else {
        EdgeTrig *trig_s = reinterpret_cast<EdgeTrig *>(b_s);
        float *m_s = reinterpret_cast<float *>(trig_s + epb);
        float *d_s = m_s + epb * L.dblock_floats;
        if (threadIdx.x < ne) {
            const float *v = dirs + eid_s[threadIdx.x] * 3;
            edge_trig(v[0], v[1], v[2], L.lmax, trig_s[threadIdx.x]);
        }
        __syncthreads();
        build_dblocks(L, ne, trig_s, m_s, d_s);
        D_s = d_s;
    }
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        const int k = idx / row, r = idx - k * row;
        const int c = r / d, j = r - c * d;
        const int base = Mm.base[j];
        if (base < 0) continue;                 // component not used by any non-empty block
        const float *fr = f_s + k * row + c * d;
        float acc = 0.0f;
        if (kDense) {
            const float *Pe = D_s + k * d * d;
            for (int q = 0; q < d; q++) acc = fmaf(fr[q], Pe[q * d + j], acc);
        } else {
            const int ps = L.perm[j];
            const int ir = L.std_irrep[ps];
            const int l = L.irrep_l[ir], n = 2 * l + 1, off = L.irrep_off[ir];
            const int col = ps - off;
            const float *De = D_s + k * L.dblock_floats + L.unique_doff[L.irrep_slot[ir]];
            for (int q = 0; q < n; q++) acc = fmaf(fr[off + q], De[q * n + col], acc);
        }
        a_s[k * k_total + base + c * Mm.stride[j]] = acc * sp_s[k][Mm.l[j]];
    }
    __syncthreads();
    // rows out: 8 bf16 (16 B) per store; k_total is a multiple of 64
    const int per = k_total / 8;
    for (int idx = threadIdx.x; idx < ne * per; idx += blockDim.x) {
        const int k = idx / per, q = idx - k * per;
        const float *v = a_s + k * k_total + q * 8;
        __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            hi[u] = __float2bfloat16_rn(v[u]);
            lo[u] = __float2bfloat16_rn(v[u] - __bfloat162float(hi[u]));
        }
        const int64_t off = (p0 + k) * (int64_t)k_total + q * 8;
        *reinterpret_cast<uint4 *>(A_hi + off) = *reinterpret_cast<const uint4 *>(hi);
        if (kSplit) *reinterpret_cast<uint4 *>(A_lo + off) = *reinterpret_cast<const uint4 *>(lo);
    }
}

// out[e][c][k] = sum_j h[c][j] Q[e][k][j] with h[c][j] = H[p][map.base[j] + c * map.stride[j]] * s_e^l(j)
// (0 for components of blocks without input).
template <bool kDense>
__global__ void rotate_out_tc_kernel(const float *__restrict__ H, int h_ld, const float *__restrict__ dirs,
                                     const float *__restrict__ Q, const float *__restrict__ dist,
                                     const int64_t *__restrict__ perm, int64_t E, int C,
                                     const __grid_constant__ ReprLayout Lp, const __grid_constant__ TcPosMap Mp,
                                     float sh_scale, int epb, float *__restrict__ out) {
    extern __shared__ float smem[];
    __shared__ ReprLayout L;
    __shared__ TcPosMap Mm;
    __shared__ float sp_s[16][kMaxL + 1];
    __shared__ int64_t eid_s[16];
    stage_posmap(Mp, Mm);
    stage_layout(Lp, L);
    const int d = L.dim, row = C * d;
    const int64_t p0 = (int64_t)blockIdx.x * epb;
    const int ne = (int)min64(epb, E - p0);
    float *h_s = smem;
    float *b_s = h_s + epb * row;
    if (threadIdx.x < ne) {
        const int64_t e = perm[p0 + threadIdx.x];
        eid_s[threadIdx.x] = e;
        const float dd = dist[e];
        const float s = dd / (dd + sh_scale);
        for (int l = 0; l <= L.lmax; l++) sp_s[threadIdx.x][l] = ipowf(s, l);
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        const int k = idx / row, r = idx - k * row;
        const int c = r / d, j = r - c * d;
        const int base = Mm.base[j];
        h_s[idx] = base < 0 ? 0.0f : __ldg(H + (p0 + k) * (int64_t)h_ld + base + c * Mm.stride[j]) * sp_s[k][Mm.l[j]];
    }
    const float *D_s;
    if (kDense) {
        const int dd2 = d * d;
        for (int idx = threadIdx.x; idx < ne * dd2; idx += blockDim.x) {
            const int k = idx / dd2;
            b_s[idx] = __ldg(Q + eid_s[k] * dd2 + (idx - k * dd2));
        }
        __syncthreads();
        D_s = b_s;
    } else {
        EdgeTrig *trig_s = reinterpret_cast<EdgeTrig *>(b_s);
        float *m_s = reinterpret_cast<float *>(trig_s + epb);
        float *d_s = m_s + epb * L.dblock_floats;
        if (threadIdx.x < ne) {
            const float *v = dirs + eid_s[threadIdx.x] * 3;
            edge_trig(v[0], v[1], v[2], L.lmax, trig_s[threadIdx.x]);
        }
        __syncthreads();
        build_dblocks(L, ne, trig_s, m_s, d_s);
        D_s = d_s;
    }
    for (int idx = threadIdx.x; idx < ne * row; idx += blockDim.x) {
        const int k = idx / row, r = idx - k * row;
        const int c = r / d, kk = r - c * d;
        const float *hr = h_s + k * row + c * d;
        float acc = 0.0f;
        if (kDense) {
            const float *Qe = D_s + k * d * d + kk * d;
            for (int j = 0; j < d; j++) acc = fmaf(hr[j], Qe[j], acc);
        } else {
            const int ir = L.std_irrep[kk];
            const int l = L.irrep_l[ir], n = 2 * l + 1, off = L.irrep_off[ir];
            const float *De = D_s + k * L.dblock_floats + L.unique_doff[L.irrep_slot[ir]] + (kk - off) * n;
            for (int col = 0; col < n; col++) acc = fmaf(hr[L.inv_perm[off + col]], De[col], acc);
        }
        out[eid_s[k] * row + r] = acc;
    }
}

constexpr size_t kTcRotSmemBudget = 160 * 1024;

int launch_rotate_in_tc(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add, const float *dirs,
                        const float *P, const float *dist, const int64_t *perm, int64_t E, int C,
                        const ReprLayout &L, const TcPosMap &M, int k_total, Binning bins, float sh_scale,
                        bool split, __nv_bfloat16 *A_hi, __nv_bfloat16 *A_lo, float *tval, int32_t *status,
                        cudaStream_t s) {
    if (E == 0) return FEQ_OK;
    const bool dense = dirs == nullptr;
    const size_t row = (size_t)C * L.dim;
    const size_t per = row + k_total + basis_area_floats(L, 1, dense);
    if (per * 4 > kTcRotSmemBudget) return FEQ_ERR_UNSUPPORTED;
    const int epb = pick_epb(per, 0, kTcRotSmemBudget, 8);
    const size_t smem = per * epb * 4;
    const int64_t grid = (E + epb - 1) / epb;
#define FEQ_ROT_IN_TC(D, G, S)                                                                              \
    do {                                                                                                    \
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_in_tc_kernel<D, G, S>,                                     \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));         \
        rotate_in_tc_kernel<D, G, S><<<(unsigned)grid, 256, smem, s>>>(x, src, nsrc, edge_add, dirs, P, dist, \
                                                                       perm, E, C, L, M, k_total, bins,     \
                                                                       sh_scale, epb, A_hi, A_lo, tval,     \
                                                                       status);                             \
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
    const size_t row = (size_t)C * L.dim;
    const size_t per = row + basis_area_floats(L, 1, dense);
    if (per * 4 > kSmemBudget) return FEQ_ERR_UNSUPPORTED;
    const int epb = pick_epb(per, 0, kSmemBudget, 8);
    const size_t smem = per * epb * 4;
    const int64_t grid = (E + epb - 1) / epb;
    if (dense) {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_out_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        rotate_out_tc_kernel<true><<<(unsigned)grid, 256, smem, s>>>(H, h_ld, dirs, Q, dist, perm, E, C, L, M,
                                                                     sh_scale, epb, out);
    } else {
        FEQ_CUDA_TRY(cudaFuncSetAttribute(rotate_out_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        rotate_out_tc_kernel<false><<<(unsigned)grid, 256, smem, s>>>(H, h_ld, dirs, Q, dist, perm, E, C, L, M,
                                                                      sh_scale, epb, out);
    }
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace feq
