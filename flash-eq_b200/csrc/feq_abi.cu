// feq_abi.cu -- the extern "C" entry points of libflasheq_b200.so: argument
// validation, host-side layout tables, workspace planning and kernel sequencing.
// Declarations and the reference interface each one replaces: include/flasheq_b200.h.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_bf16.h>

#include "feq_internal.cuh"

namespace feq {

// kernels (feq_rotate.cu, feq_mix.cu, feq_graph.cu)
int launch_basis(const float *dirs, int64_t E, const ReprLayout &L, int layout, float *out, cudaStream_t s);
int launch_basis_stream(const float *dirs, int64_t E, const ReprLayout &L, int mfirst, float *out, cudaStream_t s);
int launch_rotate_in(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add,
                     const float *dirs, const float *P, int64_t E, int C, const ReprLayout &L,
                     float *g, int32_t *status, cudaStream_t s);
int launch_rotate_out(const float *h, const float *dirs, const float *Q, int64_t E, int C,
                      const ReprLayout &L, float *out, cudaStream_t s);
int64_t mix_max_tiles(int64_t E, int nb, int te);
int launch_relayout(const float *T, float *Wt, int nb1, int Cin, int Cout, const MixLayout &M, cudaStream_t s);
int launch_build_tiles(const int64_t *offsets, int nb, int te, int4 *tiles, int *num_tiles, cudaStream_t s);
int launch_mix(const float *g, const float *Wt, const float *dist, const int64_t *perm, const int4 *tiles,
               const int *num_tiles, int64_t max_tiles, int64_t E, int Cin, int Cout, int din, int dout,
               const MixLayout &M, Binning bins, float sh_scale, float *h, cudaStream_t s);
int launch_binning(const float *dist, int64_t E, Binning b, int32_t *lo, float *t, cudaStream_t s);
size_t edge_sort_workspace(int64_t E, int32_t nk);
template <typename K>
int launch_edge_sort(const K *keys, int64_t E, int32_t nk, int64_t *perm, int64_t *offsets,
                     int32_t *status, void *ws, size_t ws_bytes, cudaStream_t s);
int launch_edge_logits(const float *Q, const float *K, int64_t E, int H, int D, float scale,
                       const float *dist, float decay, float *logits, cudaStream_t s);
int launch_segment_softmax(const float *logits, int64_t N, int H, const int64_t *perm,
                           const int64_t *offsets, float *weights, cudaStream_t s);
int launch_segment_pool(const float *rows, int64_t L, const float *w, int H, const int64_t *perm,
                        const int64_t *offsets, int64_t N, int reduce, float *out, cudaStream_t s);
int launch_attn_pool(const FeqAttnArgs &a, cudaStream_t s);

// tensor-core path (feq_tcmix.cu, feq_rotate.cu)
int launch_tc_relayout_b(const float *T, __nv_bfloat16 *Bhi, __nv_bfloat16 *Blo, int nb1, int Cin, int Cout,
                         int wdim, const TcGeom &G, int64_t total, cudaStream_t s);
int launch_tc_mix(int split, const __nv_bfloat16 *A, const __nv_bfloat16 *A2, int64_t a_rows, int a_cols,
                  const __nv_bfloat16 *Bm, const __nv_bfloat16 *Bm2, int64_t b_rows, const TcBlockGeom &B,
                  int a_col0, int n_valid, int h_ld, int h_col0, const int4 *tiles, const int *num_tiles,
                  int64_t max_tiles, const float *tval, float *H, int32_t *status, cudaStream_t s,
                  float *Hd = nullptr);
int launch_rotate_in_tc(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add, const float *dirs,
                        const float *P, const float *dist, const int64_t *perm, int64_t E, int C,
                        const ReprLayout &L, const TcPosMap &M, int k_total, Binning bins, float sh_scale,
                        bool split, __nv_bfloat16 *A_hi, __nv_bfloat16 *A_lo, float *tval, int32_t *status,
                        cudaStream_t s);
int launch_rotate_out_tc(const float *H, int h_ld, const float *dirs, const float *Q, const float *dist,
                         const int64_t *perm, int64_t E, int C, const ReprLayout &L, const TcPosMap &M,
                         float sh_scale, float *out, cudaStream_t s);
int launch_rot_in_stream(const float *x, const int64_t *src, int64_t nsrc, const float *edge_add, const float *dirs,
                         const float *dist, const int64_t *perm, int64_t E, int C, const ReprLayout &L,
                         const TcPosMap &M, int k_total, Binning bins, float sh_scale, bool split,
                         __nv_bfloat16 *A_hi, __nv_bfloat16 *A_lo, float *tval, int32_t *status, cudaStream_t s);
int launch_rot_out_stream(const float *H, int h_ld, const float *dirs, const float *dist, const int64_t *perm,
                          int64_t E, int C, const ReprLayout &L, const TcPosMap &M, float sh_scale, float *out,
                          int32_t *status, cudaStream_t s);

int launch_bwd_prep_rows(const float *X, const float *dist, const int64_t *perm, int64_t E, int C, int D,
                         const TcPosMap &Mp, int ld, Binning bins, float sh_scale, __nv_bfloat16 *Mhi,
                         __nv_bfloat16 *Mlo, float *tval, cudaStream_t s);
int launch_bwd_transpose_table(const float *T, float *Tt, int nb1, int Cout, int Cin, int W, const MixLayout &M,
                               cudaStream_t s);
int launch_bwd_rows(const float *gA, const float *gAd, int ld_g, const __nv_bfloat16 *Ahi, const __nv_bfloat16 *Alo,
                    int ld_a, const __nv_bfloat16 *Ghi, const __nv_bfloat16 *Glo, int ld_gg, const float *H, int ld_h,
                    const float *dist, const int64_t *perm, int64_t E, int Cin, int Din, int Cout, int Dout,
                    const TcPosMap &in1, const TcPosMap &out1, const TcPosMap &in2, const TcPosMap &out2,
                    Binning bins, float sh_scale, int any_l, float *grad_f, float *grad_d, cudaStream_t s);
int launch_bwd_table_convert(const float *dB, const DbOff &dboff, int nb1, int Cout, int Cin, int W,
                             const MixLayout &M, float *grad_table, cudaStream_t s);
int launch_bwd_segments(const int64_t *offsets, int nb, int64_t *seg, cudaStream_t s);
int launch_unprep_rows(const float *H, int ld, const float *dist, const int64_t *perm, int64_t E, int C, int D,
                       const TcPosMap &Mp, float sh_scale, float *out, cudaStream_t s);
int launch_bwd_transpose_rows(const __nv_bfloat16 *Xhi, const __nv_bfloat16 *Xlo, int ld, int ncols,
                              const int64_t *offsets, const int64_t *seg, int nb, const float *tval, int wmode,
                              int64_t pcols, __nv_bfloat16 *Yhi, __nv_bfloat16 *Ylo, cudaStream_t s);
int launch_tc_gram(int split, const __nv_bfloat16 *Gt0, const __nv_bfloat16 *Gt0l, const __nv_bfloat16 *Gt1,
                   const __nv_bfloat16 *Gt1l, int64_t g_rows, const __nv_bfloat16 *At, const __nv_bfloat16 *Atl,
                   int64_t a_rows, int64_t p_cols, int n_blocks, const TcGramBlock *blk, int nb, const int64_t *seg,
                   float *dB, int32_t *status, cudaStream_t s);

static thread_local std::string g_last_error;
static std::atomic<long long> g_launches{0};

void count_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

static std::atomic<uint64_t> g_wait_limit_ns{4000000000ull};

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

struct ProfRec {
    std::string name;
    cudaEvent_t a = nullptr, b = nullptr;
};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static std::vector<ProfRec> g_prof;

static void prof_clear_locked() {
    for (ProfRec &r : g_prof) {
        if (r.a) cudaEventDestroy(r.a);
        if (r.b) cudaEventDestroy(r.b);
    }
    g_prof.clear();
}

void prof_begin(const char *name, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on) return;
    ProfRec r;
    r.name = name;
    if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess ||
        cudaEventRecord(r.a, s) != cudaSuccess) {
        if (r.a) cudaEventDestroy(r.a);
        if (r.b) cudaEventDestroy(r.b);
        return;
    }
    g_prof.push_back(r);
}

void prof_end(cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on || g_prof.empty()) return;
    cudaEventRecord(g_prof.back().b, s);
}

void record_cuda_error(cudaError_t err) {
    g_last_error = std::string(cudaGetErrorName(err)) + ": " + cudaGetErrorString(err);
}

void record_error_text(const char *msg) { g_last_error = msg; }

int build_repr_layout(const int32_t *lv, int32_t n, ReprLayout *L) {
    if (!lv || n < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (n > kMaxIrreps) return FEQ_ERR_UNSUPPORTED;
    memset(L, 0, sizeof(*L));
    int off = 0, lmax = 0;
    bool present[kMaxL + 1] = {false};
    for (int r = 0; r < n; r++) {
        const int l = lv[r];
        if (l < 0) return FEQ_ERR_INVALID_ARGUMENT;
        if (l > kMaxL) return FEQ_ERR_UNSUPPORTED;
        L->irrep_l[r] = (int8_t)l;
        L->irrep_off[r] = (int16_t)off;
        off += 2 * l + 1;
        if (off > kMaxDim) return FEQ_ERR_UNSUPPORTED;
        lmax = std::max(lmax, l);
        present[l] = true;
    }
    L->n_irreps = n;
    L->dim = off;
    L->lmax = lmax;
    int u = 0, doff = 0;
    int slot_of[kMaxL + 1];
    for (int l = 0; l <= kMaxL; l++) {
        slot_of[l] = -1;
        if (!present[l]) continue;
        L->unique_l[u] = (int8_t)l;
        L->unique_doff[u] = (int16_t)doff;
        slot_of[l] = u;
        doff += (2 * l + 1) * (2 * l + 1);
        u++;
    }
    L->n_unique = u;
    L->dblock_floats = doff;
    for (int r = 0; r < n; r++) {
        L->irrep_slot[r] = (int8_t)slot_of[L->irrep_l[r]];
        for (int k = 0; k < 2 * L->irrep_l[r] + 1; k++) L->std_irrep[L->irrep_off[r] + k] = (int8_t)r;
    }
    // m-first order (wigner.py:243-272): all m = 0, then per m the (+m, -m) pairs.
    int j = 0;
    for (int r = 0; r < n; r++) L->perm[j++] = (int16_t)(L->irrep_off[r] + L->irrep_l[r]);
    for (int m = 1; m <= lmax; m++)
        for (int r = 0; r < n; r++)
            if (L->irrep_l[r] >= m) {
                L->perm[j++] = (int16_t)(L->irrep_off[r] + L->irrep_l[r] + m);
                L->perm[j++] = (int16_t)(L->irrep_off[r] + L->irrep_l[r] - m);
            }
    for (int q = 0; q < off; q++) L->inv_perm[L->perm[q]] = (int16_t)q;
    return FEQ_OK;
}

// Restates precompute_block_info (block_diagonal.cu:1191-1266) plus the re-laid
// table geometry used by the mix kernel.
int build_mix_layout(const int32_t *lin, int32_t nin, const int32_t *lout, int32_t nout, int c_in,
                     int c_out, MixLayout *M) {
    if (!lin || !lout || nin < 1 || nout < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (nin > kMaxIrreps || nout > kMaxIrreps) return FEQ_ERR_UNSUPPORTED;
    memset(M, 0, sizeof(*M));
    int lmi = 0, lmo = 0;
    for (int i = 0; i < nin; i++) {
        if (lin[i] < 0) return FEQ_ERR_INVALID_ARGUMENT;
        lmi = std::max<int>(lmi, lin[i]);
    }
    for (int i = 0; i < nout; i++) {
        if (lout[i] < 0) return FEQ_ERR_INVALID_ARGUMENT;
        lmo = std::max<int>(lmo, lout[i]);
    }
    const int mmax = std::max(lmi, lmo);
    if (mmax > kMaxL) return FEQ_ERR_UNSUPPORTED;   // reference: mmax < MAX_LVALS (:1298)
    M->n_blocks = mmax + 1;
    M->lmax_in = lmi;
    M->lmax_out = lmo;
    int in_off = 0, out_off = 0, w_off = 0;
    int64_t roff = 0;
    for (int m = 0; m <= mmax; m++) {
        MixBlock &B = M->blk[m];
        B.m = m;
        int ni = 0, no = 0;
        for (int i = 0; i < nin; i++)
            if (lin[i] >= m) B.l_in[ni++] = (int8_t)lin[i];
        for (int i = 0; i < nout; i++)
            if (lout[i] >= m) B.l_out[no++] = (int8_t)lout[i];
        B.n_in = ni;
        B.n_out = no;
        B.in_off = in_off;
        B.out_off = out_off;
        B.w_off = w_off;
        const int mult = m == 0 ? 1 : 2;
        if (ni > 0 && no > 0) {
            B.relaid_stride = ((c_out * no * mult) + 1) & ~1;
            roff = (roff + 3) & ~int64_t(3);
            B.relaid_off = (int)roff;
            roff += (int64_t)c_in * ni * B.relaid_stride;
            in_off += mult * ni;
            out_off += mult * no;
            w_off += mult * no * ni;
        }
    }
    M->wdim = w_off;
    M->relaid_row = (roff + 3) & ~int64_t(3);
    if (M->relaid_row > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    return FEQ_OK;
}

static int dims_of(const int32_t *lv, int32_t n) {
    int d = 0;
    for (int i = 0; i < n; i++) d += 2 * lv[i] + 1;
    return d;
}

// Radial-mix plan shared by block_diagonal_fwd and edgewise_fwd.
struct MixPlan {
    float *Wt;
    int32_t *keys;
    int64_t *perm, *offsets;
    int4 *tiles;
    int *num_tiles;
    void *sort_ws;
    size_t sort_ws_bytes;
    int64_t max_tiles;
};

static void carve_mix(WsCarver &w, int64_t E, int nb, const MixLayout &M, MixPlan &p) {
    const int64_t E1 = std::max<int64_t>(E, 1);
    p.Wt = (float *)w.take(sizeof(float) * ((size_t)M.relaid_row * (nb + 1) + 16));
    p.keys = (int32_t *)w.take(sizeof(int32_t) * E1);
    p.perm = (int64_t *)w.take(sizeof(int64_t) * E1);
    p.offsets = (int64_t *)w.take(sizeof(int64_t) * (nb + 1));
    p.max_tiles = mix_max_tiles(E, nb, 0);
    p.tiles = (int4 *)w.take(sizeof(int4) * p.max_tiles);
    p.num_tiles = (int *)w.take(sizeof(int) * 4);
    p.sort_ws_bytes = edge_sort_workspace(E, nb);
    p.sort_ws = w.take(p.sort_ws_bytes);
}

static int run_mix(const MixPlan &p, const float *g, const float *table, const float *dist, int64_t E,
                   int Cin, int Cout, int din, int dout, const MixLayout &M, Binning bins, float sh_scale,
                   float *h, cudaStream_t s) {
    int rc;
    if ((rc = launch_binning(dist, E, bins, p.keys, nullptr, s)) != FEQ_OK) return rc;
    if ((rc = launch_edge_sort<int32_t>(p.keys, E, bins.num_bins, p.perm, p.offsets, nullptr, p.sort_ws,
                                        p.sort_ws_bytes, s)) != FEQ_OK)
        return rc;
    if ((rc = launch_build_tiles(p.offsets, bins.num_bins, 0, p.tiles, p.num_tiles, s)) != FEQ_OK) return rc;
    if ((rc = launch_relayout(table, p.Wt, bins.num_bins + 1, Cin, Cout, M, s)) != FEQ_OK) return rc;
    return launch_mix(g, p.Wt, dist, p.perm, p.tiles, p.num_tiles, p.max_tiles, E, Cin, Cout, din, dout, M,
                      bins, sh_scale, h, s);
}

static bool mix_args_ok(int64_t E, int Cin, int Cout, int nb) {
    return E >= 0 && E < 0x7fffffffll && Cin >= 1 && Cout >= 1 && nb >= 1 && nb < (1 << 24);
}

// ---------------------------------------------------------------------------
// Tensor-core plan: GEMM geometry per m-block and the row maps of A and H.
// ---------------------------------------------------------------------------
struct TcPlan {
    TcGeom G;
    int koff[kMaxBlocks], noff[kMaxBlocks], nvalid[kMaxBlocks];
    int k_total, n_total;
    int c_in, c_out;
    int64_t b_total;
    TcPosMap in_map, out_map;
};

// Offset of block m in m-first order when every irrep with l >= m contributes
// (wigner.py:243-272), independent of whether the block takes part in the mix.
static void mfirst_offsets(const ReprLayout &L, int *off) {
    int o = 0;
    for (int m = 0; m <= kMaxL; m++) {
        off[m] = o;
        int n = 0;
        for (int r = 0; r < L.n_irreps; r++) n += L.irrep_l[r] >= m;
        o += (m == 0 ? 1 : 2) * n;
    }
}

static void fill_posmap(const ReprLayout &L, const TcPlan &T, const MixLayout &M, bool input, TcPosMap *map) {
    int off[kMaxL + 1];
    mfirst_offsets(L, off);
    memset(map, 0, sizeof(*map));
    for (int j = 0; j < L.dim; j++) {
        const int ps = L.perm[j], ir = L.std_irrep[ps], l = L.irrep_l[ir];
        const int col = ps - L.irrep_off[ir];
        const int m = col >= l ? col - l : l - col;
        map->l[j] = (int8_t)l;
        map->base[j] = -1;
        if (m < T.G.n_blocks) {
            const MixBlock &B = M.blk[m];
            const int mult = m == 0 ? 1 : 2;
            // columns are (member, re/im, channel) with the channel fastest
            if (input) {
                map->base[j] = T.koff[m] + (j - off[m]) * T.c_in;
            } else {
                map->base[j] = T.noff[m] + (j - off[m]) * T.c_out;
            }
            map->stride[j] = 1;
            (void)mult;
            (void)B;
        }
    }
    for (int j = 0; j < L.dim; j++) map->base_std[L.perm[j]] = map->base[j];
    map->n_pad = 0;
    if (input) {
        for (int m = 0; m < T.G.n_blocks; m++) {
            const int K = T.c_in * T.G.g[m].mult * T.G.g[m].n_in;
            if (K < T.G.g[m].kpad) {
                map->pad_lo[map->n_pad] = T.koff[m] + K;
                map->pad_hi[map->n_pad] = T.koff[m] + T.G.g[m].kpad;
                map->n_pad++;
            }
        }
    }
}

static int build_tc_plan(const MixLayout &M, const ReprLayout &Li, const ReprLayout &Lo, int Cin, int Cout, int nb,
                         TcPlan *T) {
    memset(T, 0, sizeof(*T));
    T->c_in = Cin;
    T->c_out = Cout;
    int kt = 0, nt = 0, nblk = 0;
    int64_t boff = 0;
    for (int m = 0; m < M.n_blocks; m++) {
        const MixBlock &B = M.blk[m];
        if (B.n_in == 0 || B.n_out == 0) break;   // emptiness is monotone in m
        const int mult = m == 0 ? 1 : 2;
        TcBlockGeom &g = T->G.g[m];
        g.mult = mult;
        g.n_in = B.n_in;
        g.n_out = B.n_out;
        g.w_off = B.w_off;
        const int K = Cin * mult * B.n_in, N = Cout * mult * B.n_out;
        g.kpad = (K + 63) / 64 * 64;
        g.npad = (N + 127) / 128 * 128;
        g.boff = boff;
        T->koff[m] = kt;
        T->noff[m] = nt;
        T->nvalid[m] = N;
        kt += g.kpad;
        nt += N;
        boff += (int64_t)(nb + 1) * g.npad * g.kpad;
        nblk++;
    }
    T->G.n_blocks = nblk;
    T->k_total = kt;
    T->n_total = nt;
    T->b_total = boff;
    if ((int64_t)kt > 65535 || (int64_t)nt > (1 << 20)) return FEQ_ERR_UNSUPPORTED;
    fill_posmap(Li, *T, M, true, &T->in_map);
    fill_posmap(Lo, *T, M, false, &T->out_map);
    return FEQ_OK;
}

struct TcBuffers {
    __nv_bfloat16 *A_hi, *A_lo, *B_hi, *B_lo;
    float *H, *tval;
    int32_t *keys;
    int64_t *perm, *offsets;
    int4 *tiles;
    int *num_tiles;
    void *sort_ws;
    size_t sort_ws_bytes;
    int64_t max_tiles;
};

static void carve_tc(WsCarver &w, int64_t E, int nb, const TcPlan &T, bool split, TcBuffers &b) {
    const int64_t E1 = std::max<int64_t>(E, 1);
    b.A_hi = (__nv_bfloat16 *)w.take(2 * (size_t)E1 * T.k_total);
    b.A_lo = split ? (__nv_bfloat16 *)w.take(2 * (size_t)E1 * T.k_total) : nullptr;
    b.B_hi = (__nv_bfloat16 *)w.take(2 * (size_t)T.b_total);
    b.B_lo = split ? (__nv_bfloat16 *)w.take(2 * (size_t)T.b_total) : nullptr;
    b.H = (float *)w.take(4 * (size_t)E1 * T.n_total);
    b.tval = (float *)w.take(4 * (size_t)E1);
    b.keys = (int32_t *)w.take(4 * (size_t)E1);
    b.perm = (int64_t *)w.take(8 * (size_t)E1);
    b.offsets = (int64_t *)w.take(8 * (size_t)(nb + 1));
    b.max_tiles = mix_max_tiles(E, nb, 128);
    b.tiles = (int4 *)w.take(sizeof(int4) * b.max_tiles);
    b.num_tiles = (int *)w.take(16);
    b.sort_ws_bytes = edge_sort_workspace(E, nb);
    b.sort_ws = w.take(b.sort_ws_bytes);
}

static int run_edgewise_tc(const FeqEdgewiseArgs *a, const MixLayout &M, const ReprLayout &Li,
                           const ReprLayout &Lo, const TcPlan &T, const TcBuffers &b, cudaStream_t s) {
    const int64_t E = a->num_edges;
    const bool split = a->mix_mode == FEQ_MIX_BF16X3;
    Binning bins{a->bin_param1, a->bin_param2, a->num_bins, a->log_bins ? 1 : 0};
    int rc;
    {
        ProfScope ps("bin_sort_tiles", s);
        if ((rc = launch_binning(a->distances, E, bins, b.keys, nullptr, s)) != FEQ_OK) return rc;
        if ((rc = launch_edge_sort<int32_t>(b.keys, E, a->num_bins, b.perm, b.offsets, nullptr, b.sort_ws,
                                            b.sort_ws_bytes, s)) != FEQ_OK)
            return rc;
        if ((rc = launch_build_tiles(b.offsets, a->num_bins, 128, b.tiles, b.num_tiles, s)) != FEQ_OK) return rc;
    }
    {
        ProfScope ps("relayout_table", s);
        if ((rc = launch_tc_relayout_b(a->radial_table, b.B_hi, b.B_lo, a->num_bins + 1, a->c_in, a->c_out, M.wdim,
                                       T.G, T.b_total, s)) != FEQ_OK)
            return rc;
    }
    // directions given: streaming bulk-copy kernels; dense bases or unaligned rows: general kernels
    {
    ProfScope ps("rotate_in", s);
    rc = launch_rot_in_stream(a->x, a->src, a->num_src_rows, a->edge_add, a->directions, a->distances, b.perm, E,
                              a->c_in, Li, T.in_map, T.k_total, bins, a->sh_scale, split, b.A_hi, b.A_lo, b.tval,
                              a->status, s);
    if (rc == FEQ_ERR_UNSUPPORTED)
        rc = launch_rotate_in_tc(a->x, a->src, a->num_src_rows, a->edge_add, a->directions, a->P_in, a->distances,
                                 b.perm, E, a->c_in, Li, T.in_map, T.k_total, bins, a->sh_scale, split, b.A_hi,
                                 b.A_lo, b.tval, a->status, s);
    }
    if (rc != FEQ_OK) return rc;
    for (int m = 0; m < T.G.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        const int64_t b_rows = (int64_t)(a->num_bins + 1) * g.npad;
        ProfScope ps("tc_mix", s);
        if ((rc = launch_tc_mix(split ? 3 : 1, b.A_hi, b.A_lo, E, T.k_total, b.B_hi + g.boff,
                                split ? b.B_lo + g.boff : nullptr, b_rows, g, T.koff[m], T.nvalid[m], T.n_total,
                                T.noff[m], b.tiles, b.num_tiles, b.max_tiles, b.tval, b.H, a->status, s)) != FEQ_OK)
            return rc;
    }
    ProfScope ps("rotate_out", s);
    rc = launch_rot_out_stream(b.H, T.n_total, a->directions, a->distances, b.perm, E, a->c_out, Lo, T.out_map,
                               a->sh_scale, a->out, a->status, s);
    if (rc == FEQ_ERR_UNSUPPORTED)
        rc = launch_rotate_out_tc(b.H, T.n_total, a->directions, a->Q_out, a->distances, b.perm, E, a->c_out, Lo,
                                  T.out_map, a->sh_scale, a->out, s);
    return rc;
}


// ---------------------------------------------------------------------------
// Backward of the block-diagonal mix (see feq_backward.cu for the formulation).
// ---------------------------------------------------------------------------
struct BwdPlan {
    MixLayout M, M2;          // forward layout and the in/out-swapped one
    ReprLayout Li, Lo;
    TcPlan T, T2;             // tensor-core plans: W_t A (T) and G W_t^T (T2)
    DbOff dboff;
    int64_t db_total;
    int64_t table_floats;
};

static int build_bwd_plan(const int32_t *lin, int nin, const int32_t *lout, int nout, int Cin, int Cout, int nb,
                          BwdPlan *P) {
    int rc;
    if ((rc = build_mix_layout(lin, nin, lout, nout, Cin, Cout, &P->M)) != FEQ_OK) return rc;
    if ((rc = build_mix_layout(lout, nout, lin, nin, Cout, Cin, &P->M2)) != FEQ_OK) return rc;
    if ((rc = build_repr_layout(lin, nin, &P->Li)) != FEQ_OK) return rc;
    if ((rc = build_repr_layout(lout, nout, &P->Lo)) != FEQ_OK) return rc;
    if ((rc = build_tc_plan(P->M, P->Li, P->Lo, Cin, Cout, nb, &P->T)) != FEQ_OK) return rc;
    if ((rc = build_tc_plan(P->M2, P->Lo, P->Li, Cout, Cin, nb, &P->T2)) != FEQ_OK) return rc;
    if (P->T.G.n_blocks != P->T2.G.n_blocks) return FEQ_ERR_UNSUPPORTED;
    int64_t off = 0;
    memset(&P->dboff, 0, sizeof(P->dboff));
    for (int m = 0; m < P->T.G.n_blocks; m++) {
        const TcBlockGeom &g = P->T.G.g[m];
        P->dboff.off[m] = off;
        off += (int64_t)(nb + 1) * (Cout * g.mult * g.n_out) * (Cin * g.mult * g.n_in);
    }
    P->db_total = off;
    P->table_floats = (int64_t)(nb + 1) * Cout * Cin * P->M.wdim;
    return FEQ_OK;
}

struct BwdBuffers {
    TcBuffers f;                     // A, B, H, tval, keys, perm, offsets, tiles, sort scratch
    __nv_bfloat16 *G_hi, *G_lo, *Bt_hi, *Bt_lo;
    float *Tt, *gA, *gAd, *dB;
    int64_t *seg, pcols;
    __nv_bfloat16 *Gt0_hi, *Gt0_lo, *Gt1_hi, *Gt1_lo, *At_hi, *At_lo;
};

static void carve_bwd(WsCarver &w, int64_t E, int nb, const BwdPlan &P, bool split, BwdBuffers &b) {
    carve_tc(w, E, nb, P.T, split, b.f);
    const int64_t E1 = std::max<int64_t>(E, 1);
    b.G_hi = (__nv_bfloat16 *)w.take(2 * (size_t)E1 * P.T2.k_total);
    b.G_lo = split ? (__nv_bfloat16 *)w.take(2 * (size_t)E1 * P.T2.k_total) : nullptr;
    b.Bt_hi = (__nv_bfloat16 *)w.take(2 * (size_t)P.T2.b_total);
    b.Bt_lo = split ? (__nv_bfloat16 *)w.take(2 * (size_t)P.T2.b_total) : nullptr;
    b.Tt = (float *)w.take(4 * (size_t)P.table_floats);
    b.gA = (float *)w.take(4 * (size_t)E1 * P.T2.n_total);
    b.gAd = (float *)w.take(4 * (size_t)E1 * P.T2.n_total);
    b.dB = (float *)w.take(4 * (size_t)std::max<int64_t>(P.db_total, 1));
    b.seg = (int64_t *)w.take(8 * (size_t)(nb + 1));
    b.pcols = (E1 + 63) / 64 * 64 + 64 * (int64_t)nb;        // every bin padded to a multiple of 64
    const size_t gsz = 2 * (size_t)P.T2.k_total * b.pcols, asz = 2 * (size_t)P.T.k_total * b.pcols;
    b.Gt0_hi = (__nv_bfloat16 *)w.take(gsz);
    b.Gt0_lo = split ? (__nv_bfloat16 *)w.take(gsz) : nullptr;
    b.Gt1_hi = (__nv_bfloat16 *)w.take(gsz);
    b.Gt1_lo = split ? (__nv_bfloat16 *)w.take(gsz) : nullptr;
    b.At_hi = (__nv_bfloat16 *)w.take(asz);
    b.At_lo = split ? (__nv_bfloat16 *)w.take(asz) : nullptr;
}

static int run_bwd(const BwdPlan &P, const BwdBuffers &b, const float *go, const float *f, const float *table,
                   const float *dist, int64_t E, int Cin, int Cout, int nb, Binning bins, float sh_scale, bool split,
                   float *grad_f, float *grad_table, float *grad_d, int32_t *status, cudaStream_t s) {
    const TcBuffers &t = b.f;
    const TcPlan &T = P.T, &T2 = P.T2;
    int rc;
    {
        ProfScope ps("bwd_sort", s);
        if ((rc = launch_binning(dist, E, bins, t.keys, nullptr, s)) != FEQ_OK) return rc;
        if ((rc = launch_edge_sort<int32_t>(t.keys, E, nb, t.perm, t.offsets, nullptr, t.sort_ws, t.sort_ws_bytes,
                                            s)) != FEQ_OK)
            return rc;
        if ((rc = launch_build_tiles(t.offsets, nb, 128, t.tiles, t.num_tiles, s)) != FEQ_OK) return rc;
    }
    {
        ProfScope ps("bwd_prep", s);
        if ((rc = launch_bwd_prep_rows(f, dist, t.perm, E, Cin, P.Li.dim, T.in_map, T.k_total, bins, sh_scale, t.A_hi,
                                       t.A_lo, t.tval, s)) != FEQ_OK)
            return rc;
        if ((rc = launch_bwd_prep_rows(go, dist, t.perm, E, Cout, P.Lo.dim, T2.in_map, T2.k_total, bins, sh_scale,
                                       b.G_hi, b.G_lo, nullptr, s)) != FEQ_OK)
            return rc;
        if ((rc = launch_tc_relayout_b(table, t.B_hi, t.B_lo, nb + 1, Cin, Cout, P.M.wdim, T.G, T.b_total, s)) !=
            FEQ_OK)
            return rc;
        if ((rc = launch_bwd_transpose_table(table, b.Tt, nb + 1, Cout, Cin, P.M.wdim, P.M, s)) != FEQ_OK) return rc;
        if ((rc = launch_tc_relayout_b(b.Tt, b.Bt_hi, b.Bt_lo, nb + 1, Cout, Cin, P.M2.wdim, T2.G, T2.b_total, s)) !=
            FEQ_OK)
            return rc;
    }
    {
        ProfScope ps("bwd_mix", s);
        for (int m = 0; m < T.G.n_blocks; m++) {
            const TcBlockGeom &g = T.G.g[m], &g2 = T2.G.g[m];
            if ((rc = launch_tc_mix(split ? 3 : 1, t.A_hi, t.A_lo, E, T.k_total, t.B_hi + g.boff,
                                    split ? t.B_lo + g.boff : nullptr, (int64_t)(nb + 1) * g.npad, g, T.koff[m],
                                    T.nvalid[m], T.n_total, T.noff[m], t.tiles, t.num_tiles, t.max_tiles, t.tval, t.H,
                                    status, s)) != FEQ_OK)
                return rc;
            if ((rc = launch_tc_mix(split ? 3 : 1, b.G_hi, b.G_lo, E, T2.k_total, b.Bt_hi + g2.boff,
                                    split ? b.Bt_lo + g2.boff : nullptr, (int64_t)(nb + 1) * g2.npad, g2, T2.koff[m],
                                    T2.nvalid[m], T2.n_total, T2.noff[m], t.tiles, t.num_tiles, t.max_tiles, t.tval,
                                    b.gA, status, s, b.gAd)) != FEQ_OK)
                return rc;
        }
    }
    {
        ProfScope ps("bwd_rows", s);
        const int any_l = (P.Li.lmax > 0 || P.Lo.lmax > 0) ? 1 : 0;
        if ((rc = launch_bwd_rows(b.gA, b.gAd, T2.n_total, t.A_hi, t.A_lo, T.k_total, b.G_hi, b.G_lo, T2.k_total, t.H,
                                  T.n_total, dist, t.perm, E, Cin, P.Li.dim, Cout, P.Lo.dim, T.in_map, T.out_map,
                                  T2.in_map, T2.out_map, bins, sh_scale, any_l, grad_f, grad_d, s)) != FEQ_OK)
            return rc;
    }
    ProfScope ps("bwd_table", s);
    if ((rc = launch_bwd_segments(t.offsets, nb, b.seg, s)) != FEQ_OK) return rc;
    if ((rc = launch_bwd_transpose_rows(b.G_hi, b.G_lo, T2.k_total, T2.k_total, t.offsets, b.seg, nb, t.tval, 1,
                                        b.pcols, b.Gt0_hi, b.Gt0_lo, s)) != FEQ_OK)
        return rc;
    if ((rc = launch_bwd_transpose_rows(b.G_hi, b.G_lo, T2.k_total, T2.k_total, t.offsets, b.seg, nb, t.tval, 2,
                                        b.pcols, b.Gt1_hi, b.Gt1_lo, s)) != FEQ_OK)
        return rc;
    if ((rc = launch_bwd_transpose_rows(t.A_hi, t.A_lo, T.k_total, T.k_total, t.offsets, b.seg, nb, t.tval, 0,
                                        b.pcols, b.At_hi, b.At_lo, s)) != FEQ_OK)
        return rc;
    TcGramBlock gb[kMaxBlocks];
    for (int m = 0; m < T.G.n_blocks; m++) {
        const TcBlockGeom &g = T.G.g[m];
        gb[m].N = Cout * g.mult * g.n_out;
        gb[m].K = Cin * g.mult * g.n_in;
        gb[m].n_tiles = (gb[m].N + 127) / 128;
        gb[m].k_tiles = (gb[m].K + 127) / 128;
        gb[m].g_row0 = T2.koff[m];
        gb[m].a_row0 = T.koff[m];
        gb[m].dboff = P.dboff.off[m];
        gb[m].item0 = 0;
    }
    if ((rc = launch_tc_gram(split ? 3 : 1, b.Gt0_hi, b.Gt0_lo, b.Gt1_hi, b.Gt1_lo, T2.k_total, b.At_hi, b.At_lo,
                             T.k_total, b.pcols, T.G.n_blocks, gb, nb, b.seg, b.dB, status, s)) != FEQ_OK)
        return rc;
    return launch_bwd_table_convert(b.dB, P.dboff, nb + 1, Cout, Cin, P.M.wdim, P.M, grad_table, s);
}

}  // namespace feq

using namespace feq;

extern "C" {

const char *feq_status_string(int status) {
    switch (status) {
        case FEQ_OK: return "ok";
        case FEQ_ERR_INVALID_ARGUMENT: return "invalid argument";
        case FEQ_ERR_UNSUPPORTED: return "unsupported by this build (limits: l <= 16, <= 64 irreps, dim <= 512)";
        case FEQ_ERR_WORKSPACE: return "workspace missing or too small";
        case FEQ_ERR_CUDA: return "CUDA error";
        case FEQ_ERR_NO_DEVICE: return "no usable CUDA device";
        default: return "unknown status";
    }
}

int feq_abi_version(void) { return 4; }

uint64_t feq_set_wait_limit_ns(uint64_t limit_ns) {
    return feq::g_wait_limit_ns.exchange(limit_ns ? limit_ns : 4000000000ull);
}

const char *feq_last_error(void) { return g_last_error.c_str(); }

int64_t feq_launch_count(void) { return (int64_t)g_launches.load(); }

int feq_profile_enable(int32_t on) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (on) {
        for (ProfRec &r : g_prof) cudaEventSynchronize(r.b);
        prof_clear_locked();
    }
    g_prof_on = on != 0;
    return FEQ_OK;
}

int feq_profile_read(int32_t index, char *name, int32_t name_capacity, double *total_ms, int64_t *launches) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    std::vector<std::string> names;
    std::vector<double> ms;
    std::vector<int64_t> cnt;
    for (ProfRec &r : g_prof) {
        float t = 0.0f;
        cudaError_t e = cudaEventSynchronize(r.b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t, r.a, r.b);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return -FEQ_ERR_CUDA;
        }
        size_t k = 0;
        while (k < names.size() && names[k] != r.name) k++;
        if (k == names.size()) {
            names.push_back(r.name);
            ms.push_back(0.0);
            cnt.push_back(0);
        }
        ms[k] += t;
        cnt[k] += 1;
    }
    if (index >= 0 && index < (int32_t)names.size()) {
        if (name && name_capacity > 0) {
            strncpy(name, names[index].c_str(), (size_t)name_capacity - 1);
            name[name_capacity - 1] = 0;
        }
        if (total_ms) *total_ms = ms[index];
        if (launches) *launches = cnt[index];
    }
    return (int)names.size();
}

int feq_wigner_basis(const float *directions, int64_t num_edges, const int32_t *lvals, int32_t num_lvals,
                     int32_t layout, float *out, feq_stream_t stream) {
    if (num_edges < 0 || (layout != FEQ_BASIS_MFIRST && layout != FEQ_BASIS_ROT_TO_EZ))
        return FEQ_ERR_INVALID_ARGUMENT;
    ReprLayout L;
    int rc = build_repr_layout(lvals, num_lvals, &L);
    if (rc != FEQ_OK) return rc;
    if (num_edges == 0) return FEQ_OK;
    if (!directions || !out) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges > 0x7fffffffll * 8) return FEQ_ERR_UNSUPPORTED;
    ProfScope ps("basis", (cudaStream_t)stream);
    rc = launch_basis_stream(directions, num_edges, L, layout == FEQ_BASIS_MFIRST ? 1 : 0, out, (cudaStream_t)stream);
    if (rc == FEQ_ERR_UNSUPPORTED) rc = launch_basis(directions, num_edges, L, layout, out, (cudaStream_t)stream);
    return rc;
}

int feq_edge_binning(const float *distances, int64_t num_edges, float bin_param1, float bin_param2,
                     int32_t num_bins, int32_t log_bins, int32_t *bin_lo, float *t, feq_stream_t stream) {
    if (num_edges < 0 || num_bins < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0) return FEQ_OK;
    if (!distances || (!bin_lo && !t)) return FEQ_ERR_INVALID_ARGUMENT;
    Binning b{bin_param1, bin_param2, num_bins, log_bins ? 1 : 0};
    return launch_binning(distances, num_edges, b, bin_lo, t, (cudaStream_t)stream);
}

size_t feq_edge_sort_workspace_bytes(int64_t num_edges, int32_t num_keys) {
    if (num_edges < 0 || num_keys < 1) return 0;
    return edge_sort_workspace(num_edges, num_keys);
}

int feq_edge_sort(const int32_t *keys, int64_t num_edges, int32_t num_keys, int64_t *perm, int64_t *offsets,
                  int32_t *status, void *workspace, size_t workspace_bytes, feq_stream_t stream) {
    if (num_edges < 0 || num_keys < 1 || !offsets || (num_edges > 0 && (!keys || !perm)))
        return FEQ_ERR_INVALID_ARGUMENT;
    return launch_edge_sort<int32_t>(keys, num_edges, num_keys, perm, offsets, status, workspace,
                                     workspace_bytes, (cudaStream_t)stream);
}

int feq_edge_sort_i64(const int64_t *keys, int64_t num_edges, int32_t num_keys, int64_t *perm,
                      int64_t *offsets, int32_t *status, void *workspace, size_t workspace_bytes,
                      feq_stream_t stream) {
    if (num_edges < 0 || num_keys < 1 || !offsets || (num_edges > 0 && (!keys || !perm)))
        return FEQ_ERR_INVALID_ARGUMENT;
    return launch_edge_sort<int64_t>(keys, num_edges, num_keys, perm, offsets, status, workspace,
                                     workspace_bytes, (cudaStream_t)stream);
}

size_t feq_block_diagonal_workspace_bytes(int64_t num_edges, int32_t c_in, int32_t c_out,
                                          const int32_t *lvals_in, int32_t n_lvals_in,
                                          const int32_t *lvals_out, int32_t n_lvals_out, int32_t num_bins) {
    MixLayout M;
    if (!mix_args_ok(num_edges, c_in, c_out, num_bins)) return 0;
    if (build_mix_layout(lvals_in, n_lvals_in, lvals_out, n_lvals_out, c_in, c_out, &M) != FEQ_OK) return 0;
    WsCarver w{nullptr, 0, 0};
    MixPlan p;
    carve_mix(w, num_edges, num_bins, M, p);
    return w.used + 256;
}

int feq_block_diagonal_fwd(const float *features, const float *radial_table, const float *distances,
                           int64_t num_edges, int32_t c_in, int32_t c_out, const int32_t *lvals_in,
                           int32_t n_lvals_in, const int32_t *lvals_out, int32_t n_lvals_out, float sh_scale,
                           float bin_param1, float bin_param2, int32_t num_bins, int32_t log_bins,
                           float *output, void *workspace, size_t workspace_bytes, feq_stream_t stream) {
    if (!mix_args_ok(num_edges, c_in, c_out, num_bins)) return FEQ_ERR_INVALID_ARGUMENT;
    MixLayout M;
    int rc = build_mix_layout(lvals_in, n_lvals_in, lvals_out, n_lvals_out, c_in, c_out, &M);
    if (rc != FEQ_OK) return rc;
    if (num_edges == 0) return FEQ_OK;
    if (!features || !radial_table || !distances || !output) return FEQ_ERR_INVALID_ARGUMENT;
    WsCarver w{(char *)workspace, 0, workspace_bytes};
    MixPlan p;
    carve_mix(w, num_edges, num_bins, M, p);
    if (!workspace || w.used > workspace_bytes) return FEQ_ERR_WORKSPACE;
    const int din = dims_of(lvals_in, n_lvals_in), dout = dims_of(lvals_out, n_lvals_out);
    Binning b{bin_param1, bin_param2, num_bins, log_bins ? 1 : 0};
    return run_mix(p, features, radial_table, distances, num_edges, c_in, c_out, din, dout, M, b, sh_scale,
                   output, (cudaStream_t)stream);
}

size_t feq_block_diagonal_fwd_mix_workspace_bytes(int64_t num_edges, int32_t c_in, int32_t c_out,
                                                  const int32_t *lvals_in, int32_t n_lvals_in,
                                                  const int32_t *lvals_out, int32_t n_lvals_out, int32_t num_bins,
                                                  int32_t mix_mode) {
    if (mix_mode == FEQ_MIX_FP32)
        return feq_block_diagonal_workspace_bytes(num_edges, c_in, c_out, lvals_in, n_lvals_in, lvals_out,
                                                  n_lvals_out, num_bins);
    if (!mix_args_ok(num_edges, c_in, c_out, num_bins)) return 0;
    if (mix_mode != FEQ_MIX_BF16 && mix_mode != FEQ_MIX_BF16X3) return 0;
    static thread_local BwdPlan P;
    if (build_bwd_plan(lvals_in, n_lvals_in, lvals_out, n_lvals_out, c_in, c_out, num_bins, &P) != FEQ_OK) return 0;
    WsCarver w{nullptr, 0, 0};
    TcBuffers b;
    carve_tc(w, num_edges, num_bins, P.T, mix_mode == FEQ_MIX_BF16X3, b);
    return w.used + 256;
}

int feq_block_diagonal_fwd_mix(const float *features, const float *radial_table, const float *distances,
                               int64_t num_edges, int32_t c_in, int32_t c_out, const int32_t *lvals_in,
                               int32_t n_lvals_in, const int32_t *lvals_out, int32_t n_lvals_out, float sh_scale,
                               float bin_param1, float bin_param2, int32_t num_bins, int32_t log_bins,
                               int32_t mix_mode, float *output, void *workspace, size_t workspace_bytes,
                               feq_stream_t stream) {
    if (mix_mode == FEQ_MIX_FP32)
        return feq_block_diagonal_fwd(features, radial_table, distances, num_edges, c_in, c_out, lvals_in,
                                      n_lvals_in, lvals_out, n_lvals_out, sh_scale, bin_param1, bin_param2, num_bins,
                                      log_bins, output, workspace, workspace_bytes, stream);
    if (!mix_args_ok(num_edges, c_in, c_out, num_bins)) return FEQ_ERR_INVALID_ARGUMENT;
    if (mix_mode != FEQ_MIX_BF16 && mix_mode != FEQ_MIX_BF16X3) return FEQ_ERR_UNSUPPORTED;
    static thread_local BwdPlan P;
    int rc = build_bwd_plan(lvals_in, n_lvals_in, lvals_out, n_lvals_out, c_in, c_out, num_bins, &P);
    if (rc != FEQ_OK) return rc;
    if (num_edges == 0) return FEQ_OK;
    if (!features || !radial_table || !distances || !output) return FEQ_ERR_INVALID_ARGUMENT;
    const bool split = mix_mode == FEQ_MIX_BF16X3;
    WsCarver w{(char *)workspace, 0, workspace_bytes};
    TcBuffers b;
    carve_tc(w, num_edges, num_bins, P.T, split, b);
    if (!workspace || w.used > workspace_bytes) return FEQ_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    const TcPlan &T = P.T;
    const int64_t E = num_edges;
    Binning bins{bin_param1, bin_param2, num_bins, log_bins ? 1 : 0};
    {
        ProfScope ps("bin_sort_tiles", s);
        if ((rc = launch_binning(distances, E, bins, b.keys, nullptr, s)) != FEQ_OK) return rc;
        if ((rc = launch_edge_sort<int32_t>(b.keys, E, num_bins, b.perm, b.offsets, nullptr, b.sort_ws,
                                            b.sort_ws_bytes, s)) != FEQ_OK)
            return rc;
        if ((rc = launch_build_tiles(b.offsets, num_bins, 128, b.tiles, b.num_tiles, s)) != FEQ_OK) return rc;
    }
    {
        ProfScope ps("prep_rows", s);
        if ((rc = launch_bwd_prep_rows(features, distances, b.perm, E, c_in, P.Li.dim, T.in_map, T.k_total, bins,
                                       sh_scale, b.A_hi, b.A_lo, b.tval, s)) != FEQ_OK)
            return rc;
        if ((rc = launch_tc_relayout_b(radial_table, b.B_hi, b.B_lo, num_bins + 1, c_in, c_out, P.M.wdim, T.G,
                                       T.b_total, s)) != FEQ_OK)
            return rc;
    }
    for (int m = 0; m < T.G.n_blocks; m++) {
        ProfScope ps("tc_mix", s);
        const TcBlockGeom &g = T.G.g[m];
        if ((rc = launch_tc_mix(split ? 3 : 1, b.A_hi, b.A_lo, E, T.k_total, b.B_hi + g.boff,
                                split ? b.B_lo + g.boff : nullptr, (int64_t)(num_bins + 1) * g.npad, g, T.koff[m],
                                T.nvalid[m], T.n_total, T.noff[m], b.tiles, b.num_tiles, b.max_tiles, b.tval, b.H,
                                nullptr, s)) != FEQ_OK)
            return rc;
    }
    ProfScope ps("unprep_rows", s);
    if (T.G.n_blocks == 0 || T.n_total == 0) {
        FEQ_CUDA_TRY(cudaMemsetAsync(output, 0, sizeof(float) * (size_t)E * c_out * P.Lo.dim, s));
        return FEQ_OK;
    }
    return launch_unprep_rows(b.H, T.n_total, distances, b.perm, E, c_out, P.Lo.dim, T.out_map, sh_scale, output, s);
}

size_t feq_block_diagonal_bwd_workspace_bytes(int64_t num_edges, int32_t c_in, int32_t c_out,
                                              const int32_t *lvals_in, int32_t n_lvals_in,
                                              const int32_t *lvals_out, int32_t n_lvals_out, int32_t num_bins,
                                              int32_t mix_mode) {
    if (!mix_args_ok(num_edges, c_in, c_out, num_bins)) return 0;
    if (mix_mode != FEQ_MIX_BF16 && mix_mode != FEQ_MIX_BF16X3) return 0;
    static thread_local BwdPlan P;
    if (build_bwd_plan(lvals_in, n_lvals_in, lvals_out, n_lvals_out, c_in, c_out, num_bins, &P) != FEQ_OK) return 0;
    WsCarver w{nullptr, 0, 0};
    BwdBuffers b;
    carve_bwd(w, num_edges, num_bins, P, mix_mode == FEQ_MIX_BF16X3, b);
    return w.used + 256;
}

int feq_block_diagonal_bwd(const float *grad_output, const float *features, const float *radial_table,
                           const float *distances, int64_t num_edges, int32_t c_in, int32_t c_out,
                           const int32_t *lvals_in, int32_t n_lvals_in, const int32_t *lvals_out,
                           int32_t n_lvals_out, float sh_scale, float bin_param1, float bin_param2,
                           int32_t num_bins, int32_t log_bins, int32_t mix_mode, float *grad_features,
                           float *grad_table, float *grad_distances, void *workspace, size_t workspace_bytes,
                           feq_stream_t stream) {
    if (!mix_args_ok(num_edges, c_in, c_out, num_bins)) return FEQ_ERR_INVALID_ARGUMENT;
    if (mix_mode != FEQ_MIX_BF16 && mix_mode != FEQ_MIX_BF16X3) return FEQ_ERR_UNSUPPORTED;
    static thread_local BwdPlan P;
    int rc = build_bwd_plan(lvals_in, n_lvals_in, lvals_out, n_lvals_out, c_in, c_out, num_bins, &P);
    if (rc != FEQ_OK) return rc;
    if (!radial_table || !grad_table) return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (num_edges == 0) {
        FEQ_CUDA_TRY(cudaMemsetAsync(grad_table, 0, sizeof(float) * (size_t)P.table_floats, s));
        return FEQ_OK;
    }
    if (!grad_output || !features || !distances || !grad_features || !grad_distances) return FEQ_ERR_INVALID_ARGUMENT;
    WsCarver w{(char *)workspace, 0, workspace_bytes};
    BwdBuffers b;
    const bool split = mix_mode == FEQ_MIX_BF16X3;
    carve_bwd(w, num_edges, num_bins, P, split, b);
    if (!workspace || w.used > workspace_bytes) return FEQ_ERR_WORKSPACE;
    Binning bins{bin_param1, bin_param2, num_bins, log_bins ? 1 : 0};
    return run_bwd(P, b, grad_output, features, radial_table, distances, num_edges, c_in, c_out, num_bins, bins,
                   sh_scale, split, grad_features, grad_table, grad_distances, nullptr, s);
}

size_t feq_edgewise_workspace_bytes(const FeqEdgewiseArgs *a) {
    if (!a || !mix_args_ok(a->num_edges, a->c_in, a->c_out, a->num_bins)) return 0;
    MixLayout M;
    ReprLayout Li, Lo;
    if (build_mix_layout(a->lvals_in, a->n_lvals_in, a->lvals_out, a->n_lvals_out, a->c_in, a->c_out, &M) !=
        FEQ_OK)
        return 0;
    if (build_repr_layout(a->lvals_in, a->n_lvals_in, &Li) != FEQ_OK) return 0;
    if (build_repr_layout(a->lvals_out, a->n_lvals_out, &Lo) != FEQ_OK) return 0;
    if (a->mix_mode == FEQ_MIX_BF16 || a->mix_mode == FEQ_MIX_BF16X3) {
        static thread_local TcPlan T;
        if (build_tc_plan(M, Li, Lo, a->c_in, a->c_out, a->num_bins, &T) != FEQ_OK) return 0;
        WsCarver w{nullptr, 0, 0};
        TcBuffers b;
        carve_tc(w, a->num_edges, a->num_bins, T, a->mix_mode == FEQ_MIX_BF16X3, b);
        return w.used + 256;
    }
    const int64_t E1 = std::max<int64_t>(a->num_edges, 1);
    WsCarver w{nullptr, 0, 0};
    w.take(sizeof(float) * (size_t)E1 * a->c_in * Li.dim);
    w.take(sizeof(float) * (size_t)E1 * a->c_out * Lo.dim);
    MixPlan p;
    carve_mix(w, a->num_edges, a->num_bins, M, p);
    return w.used + 256;
}

int feq_edgewise_fwd(const FeqEdgewiseArgs *a, void *workspace, size_t workspace_bytes, feq_stream_t stream) {
    if (!a || !mix_args_ok(a->num_edges, a->c_in, a->c_out, a->num_bins)) return FEQ_ERR_INVALID_ARGUMENT;
    MixLayout M;
    ReprLayout Li, Lo;
    int rc = build_mix_layout(a->lvals_in, a->n_lvals_in, a->lvals_out, a->n_lvals_out, a->c_in, a->c_out, &M);
    if (rc != FEQ_OK) return rc;
    if ((rc = build_repr_layout(a->lvals_in, a->n_lvals_in, &Li)) != FEQ_OK) return rc;
    if ((rc = build_repr_layout(a->lvals_out, a->n_lvals_out, &Lo)) != FEQ_OK) return rc;
    const int64_t E = a->num_edges;
    if (E == 0) return FEQ_OK;
    if (!a->x || !a->distances || !a->radial_table || !a->out) return FEQ_ERR_INVALID_ARGUMENT;
    if (!a->directions && (!a->P_in || !a->Q_out)) return FEQ_ERR_INVALID_ARGUMENT;
    if (a->src && a->num_src_rows < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (a->mix_mode < FEQ_MIX_FP32 || a->mix_mode > FEQ_MIX_BF16X3) return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (a->mix_mode != FEQ_MIX_FP32) {
        static thread_local TcPlan T;
        if ((rc = build_tc_plan(M, Li, Lo, a->c_in, a->c_out, a->num_bins, &T)) != FEQ_OK) return rc;
        WsCarver w{(char *)workspace, 0, workspace_bytes};
        TcBuffers b;
        carve_tc(w, E, a->num_bins, T, a->mix_mode == FEQ_MIX_BF16X3, b);
        if (!workspace || w.used > workspace_bytes) return FEQ_ERR_WORKSPACE;
        return run_edgewise_tc(a, M, Li, Lo, T, b, s);
    }
    WsCarver w{(char *)workspace, 0, workspace_bytes};
    float *g = (float *)w.take(sizeof(float) * (size_t)E * a->c_in * Li.dim);
    float *h = (float *)w.take(sizeof(float) * (size_t)E * a->c_out * Lo.dim);
    MixPlan p;
    carve_mix(w, E, a->num_bins, M, p);
    if (!workspace || w.used > workspace_bytes) return FEQ_ERR_WORKSPACE;
    Binning b{a->bin_param1, a->bin_param2, a->num_bins, a->log_bins ? 1 : 0};
    if ((rc = launch_rotate_in(a->x, a->src, a->num_src_rows, a->edge_add, a->directions, a->P_in, E, a->c_in,
                               Li, g, a->status, s)) != FEQ_OK)
        return rc;
    if ((rc = run_mix(p, g, a->radial_table, a->distances, E, a->c_in, a->c_out, Li.dim, Lo.dim, M, b,
                      a->sh_scale, h, s)) != FEQ_OK)
        return rc;
    return launch_rotate_out(h, a->directions, a->Q_out, E, a->c_out, Lo, a->out, s);
}

int feq_segment_softmax(const float *logits, int64_t num_edges, int32_t num_heads, const int64_t *perm,
                        const int64_t *offsets, int64_t num_nodes, float *weights, feq_stream_t stream) {
    if (num_edges < 0 || num_nodes < 0 || num_heads < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0 || num_nodes == 0) return FEQ_OK;
    if (!logits || !perm || !offsets || !weights) return FEQ_ERR_INVALID_ARGUMENT;
    return launch_segment_softmax(logits, num_nodes, num_heads, perm, offsets, weights, (cudaStream_t)stream);
}

int feq_edge_attention_weights(const float *Q, const float *K, int64_t num_edges, int32_t num_heads,
                               int32_t qk_dim, float scale, const float *distances, float decay_scale,
                               const int64_t *perm, const int64_t *offsets, int64_t num_nodes, float *weights,
                               feq_stream_t stream) {
    if (num_edges < 0 || num_nodes < 0 || num_heads < 1 || qk_dim < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0) return FEQ_OK;
    if (!Q || !K || !perm || !offsets || !weights || (decay_scale > 0.0f && !distances))
        return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    int rc = launch_edge_logits(Q, K, num_edges, num_heads, qk_dim, scale, distances, decay_scale, weights, s);
    if (rc != FEQ_OK) return rc;
    return launch_segment_softmax(weights, num_nodes, num_heads, perm, offsets, weights, s);
}

int feq_segment_pool(const float *edge_rows, int64_t row_len, const float *weights, int32_t num_heads,
                     const int64_t *perm, const int64_t *offsets, int64_t num_nodes, int32_t reduce, float *out,
                     feq_stream_t stream) {
    if (row_len < 0 || num_nodes < 0 || reduce < FEQ_REDUCE_SUM || reduce > FEQ_REDUCE_MAX)
        return FEQ_ERR_INVALID_ARGUMENT;
    if (weights && (num_heads < 1 || row_len % num_heads)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_nodes == 0 || row_len == 0) return FEQ_OK;
    if (!perm || !offsets || !out) return FEQ_ERR_INVALID_ARGUMENT;
    return launch_segment_pool(edge_rows, row_len, weights, weights ? num_heads : 0, perm, offsets, num_nodes,
                               reduce, out, (cudaStream_t)stream);
}

int feq_attn_pool_fwd(const FeqAttnArgs *a, feq_stream_t stream) {
    if (!a || a->num_nodes < 0 || a->num_edges < 0 || a->num_heads < 1 || a->c_qk < 1 || a->d_qk < 1 ||
        a->c_v < 1 || a->d_v < 1)
        return FEQ_ERR_INVALID_ARGUMENT;
    if (a->c_qk % a->num_heads || a->c_v % a->num_heads) return FEQ_ERR_INVALID_ARGUMENT;
    if (a->reduce != FEQ_REDUCE_SUM && a->reduce != FEQ_REDUCE_MEAN) return FEQ_ERR_UNSUPPORTED;
    if (a->num_nodes == 0) return FEQ_OK;
    if (!a->qk || !a->perm || !a->offsets || !a->out || (a->num_edges > 0 && (!a->v || !a->src)))
        return FEQ_ERR_INVALID_ARGUMENT;
    if (a->decay_scale > 0.0f && !a->distances) return FEQ_ERR_INVALID_ARGUMENT;
    if (a->k && a->num_src_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    ProfScope ps("attn_pool", (cudaStream_t)stream);
    return launch_attn_pool(*a, (cudaStream_t)stream);
}

}  // extern "C"
