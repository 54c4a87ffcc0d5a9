/*
 * TEST INFRASTRUCTURE ONLY -- the parity checker and the timed CPU baseline.
 * Nothing in the product (flash-eq_b200/) links, loads or calls this file.
 *
 * CPU restatement of the forward pass of flash-eq's block-diagonal kernel
 * (flash_eq/cuda/csrc/block_diagonal.cu in hmblair/flash-eq):
 *
 *   out_m[e, co, o] = sum_ci sum_i  s(e)^(l_i + l_o) *
 *                     ((1 - t_e) T[lo_e, co, ci, w] + t_e T[lo_e + 1, co, ci, w]) * f_m[e, ci, i]
 *
 * with the m > 0 blocks acting as 2x2 [[a, b], [-b, a]] on (+m, -m) pairs.
 *
 * Followed line by line:
 *   compute_binning          block_diagonal.cu:82-115   (float32 bin index, t in the
 *                                                       feature type, t NOT clamped in
 *                                                       linear mode)
 *   ipow / solid harmonic    block_diagonal.cu:202-232
 *   setup_edge               block_diagonal.cu:307-319  (sh_weight = d / (d + scale))
 *   precompute_scales        block_diagonal.cu:325-344  (scale = sh_weight^(l_in+l_out))
 *   lerp_weight              block_diagonal.cu:277-287
 *   forward_m0_kernel        block_diagonal.cu:558-632  (w index w_off + o*n_in + i)
 *   forward_mpos_kernel      block_diagonal.cu:645-733  (w index w_off + 2(o*n_in+i) + c)
 *   precompute_block_info    block_diagonal.cu:1191-1266 (offsets advance only when
 *                                                        n_in > 0 and n_out > 0)
 *   output zero-initialised  block_diagonal.cu:1309
 *
 * Built with -ffp-contract=off so the float32 variant rounds every step the way
 * the source expressions read.  Parallel over edges with plain pthreads (no
 * OpenMP runtime, so it cannot clash with the one torch loads).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define ORACLE_MAX_L 17      /* block_diagonal.cu:172 MAX_LVALS */
#define ORACLE_BP_STRIDE 6   /* block_diagonal.cu:179 */
#define ORACLE_MAX_THREADS 512

static int count_geq(const int *lv, int n, int m) {
    int c = 0;
    for (int i = 0; i < n; i++) c += lv[i] >= m;
    return c;
}

/* Block layout restating precompute_block_info (block_diagonal.cu:1191-1266).
 * params: (mmax+1) x 6 ints [m, n_in, n_out, in_off, out_off, w_off]
 * lk_in / lk_out: (mmax+1) x ORACLE_MAX_L l-values of the i-th / o-th member of
 * block m.  Returns mmax, or -1 when mmax >= ORACLE_MAX_L. */
int oracle_block_layout(const int *lin, int nlin, const int *lout, int nlout,
                        int *params, int *lk_in, int *lk_out) {
    int mmax = 0;
    for (int i = 0; i < nlin; i++) if (lin[i] > mmax) mmax = lin[i];
    for (int i = 0; i < nlout; i++) if (lout[i] > mmax) mmax = lout[i];
    if (mmax >= ORACLE_MAX_L) return -1;
    int in_off = 0, out_off = 0, w_off = 0;
    for (int m = 0; m <= mmax; m++) {
        int n_in = count_geq(lin, nlin, m), n_out = count_geq(lout, nlout, m);
        int *bp = params + m * ORACLE_BP_STRIDE;
        bp[0] = m; bp[1] = n_in; bp[2] = n_out; bp[3] = in_off; bp[4] = out_off; bp[5] = w_off;
        for (int i = 0; i < ORACLE_MAX_L; i++) {
            lk_in[m * ORACLE_MAX_L + i] = 0;
            lk_out[m * ORACLE_MAX_L + i] = 0;
        }
        int k = 0;
        for (int i = 0; i < nlin; i++)
            if (lin[i] >= m && k < ORACLE_MAX_L) lk_in[m * ORACLE_MAX_L + k++] = lin[i];
        k = 0;
        for (int i = 0; i < nlout; i++)
            if (lout[i] >= m && k < ORACLE_MAX_L) lk_out[m * ORACLE_MAX_L + k++] = lout[i];
        if (n_in > 0 && n_out > 0) {
            int mult = (m == 0) ? 1 : 2;
            in_off += mult * n_in;
            out_off += mult * n_out;
            w_off += mult * n_out * n_in;
        }
    }
    return mmax;
}

/* compute_binning (block_diagonal.cu:82-115), float32 index math. */
static void binning_index(float dist, float p1, float p2, int nb, int log_bins,
                          int *lo, int *hi) {
    float normalized;
    if (log_bins)
        normalized = (logf(fmaxf(dist, expf(p1))) - p1) * p2 * nb;
    else
        normalized = (dist - p1) * p2;
    normalized = fminf(fmaxf(normalized, 0.0f), (float)nb);
    int l = (int)floorf(normalized);
    if (l > nb - 1) l = nb - 1;
    *lo = l;
    *hi = (l + 1 < nb) ? l + 1 : nb;
}

/* Bin index and interpolation weight for every edge (float32 variant). */
void oracle_binning_f32(const float *dist, int64_t E, float p1, float p2, int nb,
                        int log_bins, int32_t *lo_out, float *t_out) {
    for (int64_t e = 0; e < E; e++) {
        int lo, hi;
        float d = dist[e];
        binning_index(d, p1, p2, nb, log_bins, &lo, &hi);
        float t;
        if (log_bins) {
            float inv_lbw = (float)(p2 * nb);
            float log_edge_lo = p1 + (float)lo / inv_lbw;
            float edge_lo = (float)exp((double)log_edge_lo);
            float edge_hi = (float)exp((double)(log_edge_lo + 1.0f / inv_lbw));
            float cd = d > edge_lo ? d : edge_lo;
            t = (cd - edge_lo) / (edge_hi - edge_lo);
            t = t < 1.0f ? t : 1.0f;
        } else {
            float bw = 1.0f / p2;
            float edge_lo = p1 + (float)lo * bw;
            t = (d - edge_lo) / bw;
        }
        lo_out[e] = lo;
        t_out[e] = t;
    }
}

/* ---- minimal pthread parallel-for over [0, n) ---------------------------- */
typedef void (*range_fn)(const void *job, int64_t e0, int64_t e1);
struct par_chunk { range_fn fn; const void *job; int64_t e0, e1; };

static void *par_entry(void *p) {
    struct par_chunk *c = (struct par_chunk *)p;
    c->fn(c->job, c->e0, c->e1);
    return NULL;
}

static void run_parallel(int64_t n, int nthreads, range_fn fn, const void *job) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > ORACLE_MAX_THREADS) nthreads = ORACLE_MAX_THREADS;
    if ((int64_t)nthreads > n) nthreads = (int)(n > 0 ? n : 1);
    if (nthreads == 1) { fn(job, 0, n); return; }
    pthread_t th[ORACLE_MAX_THREADS];
    struct par_chunk ch[ORACLE_MAX_THREADS];
    int started[ORACLE_MAX_THREADS];
    for (int i = 0; i < nthreads; i++) {
        ch[i].fn = fn; ch[i].job = job;
        ch[i].e0 = n * i / nthreads; ch[i].e1 = n * (i + 1) / nthreads;
        started[i] = pthread_create(&th[i], NULL, par_entry, &ch[i]) == 0;
        if (!started[i]) fn(job, ch[i].e0, ch[i].e1);   /* run inline if no thread */
    }
    for (int i = 0; i < nthreads; i++) if (started[i]) pthread_join(th[i], NULL);
}

/* ---- the forward restatement, for float and double ------------------------ */
#define DEFINE_BD_FWD(NAME, T)                                                              \
struct NAME##_job {                                                                         \
    const T *features, *table, *dist;                                                       \
    int Cin, Cout, Din, Dout, Wdim;                                                         \
    float sh_scale, p1, p2;                                                                 \
    int nb, log_bins, mmax;                                                                 \
    int64_t tstride;                                                                        \
    const int *params, *lk_in, *lk_out;                                                     \
    T *out;                                                                                 \
};                                                                                          \
static T NAME##_ipow(T base, int ex) {                                                      \
    T r = (T)1;                                                                             \
    while (ex > 0) { if (ex & 1) r *= base; base *= base; ex >>= 1; }                       \
    return r;                                                                               \
}                                                                                           \
static void NAME##_range(const void *jv, int64_t e0, int64_t e1) {                          \
    const struct NAME##_job *J = (const struct NAME##_job *)jv;                             \
    const int Cin = J->Cin, Cout = J->Cout, Din = J->Din, Dout = J->Dout, Wdim = J->Wdim;   \
    for (int64_t e = e0; e < e1; e++) {                                                     \
        const T d = J->dist[e];                                                             \
        const T shw = d / (d + (T)J->sh_scale);                                             \
        int lo, hi;                                                                         \
        binning_index((float)d, J->p1, J->p2, J->nb, J->log_bins, &lo, &hi);                \
        T t;                                                                                \
        if (J->log_bins) {                                                                  \
            T inv_lbw = (T)(J->p2 * J->nb);                                                 \
            T log_edge_lo = (T)J->p1 + (T)lo / inv_lbw;                                     \
            T edge_lo = (T)exp((double)log_edge_lo);                                        \
            T edge_hi = (T)exp((double)(log_edge_lo + (T)1 / inv_lbw));                     \
            T cd = d > edge_lo ? d : edge_lo;                                               \
            t = (cd - edge_lo) / (edge_hi - edge_lo);                                       \
            t = t < (T)1 ? t : (T)1;                                                        \
        } else {                                                                            \
            T bw = (T)1 / (T)J->p2;                                                         \
            T edge_lo = (T)J->p1 + (T)lo * bw;                                              \
            t = (d - edge_lo) / bw;                                                         \
        }                                                                                   \
        const T omt = (T)1 - t;                                                             \
        const T *f = J->features + e * (int64_t)Cin * Din;                                  \
        T *o_e = J->out + e * (int64_t)Cout * Dout;                                         \
        for (int m = 0; m <= J->mmax; m++) {                                                \
            const int *bp = J->params + m * ORACLE_BP_STRIDE;                               \
            const int n_in = bp[1], n_out = bp[2], in_off = bp[3], out_off = bp[4];         \
            const int w_off = bp[5];                                                        \
            if (n_in == 0 || n_out == 0) continue;                                          \
            const int *lki = J->lk_in + m * ORACLE_MAX_L, *lko = J->lk_out + m * ORACLE_MAX_L; \
            for (int co = 0; co < Cout; co++) {                                             \
                const T *tl = J->table + lo * J->tstride + (int64_t)co * Cin * Wdim + w_off; \
                const T *th = J->table + hi * J->tstride + (int64_t)co * Cin * Wdim + w_off; \
                for (int oo = 0; oo < n_out; oo++) {                                        \
                    if (m == 0) {                                                           \
                        T acc = 0;                                                          \
                        for (int ci = 0; ci < Cin; ci++) {                                  \
                            const T *fp = f + (int64_t)ci * Din + in_off;                   \
                            for (int ii = 0; ii < n_in; ii++) {                             \
                                const int w = ci * Wdim + oo * n_in + ii;                   \
                                T wt = omt * tl[w] + t * th[w];                             \
                                wt *= NAME##_ipow(shw, lki[ii] + lko[oo]);                  \
                                acc += wt * fp[ii];                                         \
                            }                                                               \
                        }                                                                   \
                        o_e[(int64_t)co * Dout + out_off + oo] = acc;                       \
                    } else {                                                                \
                        T are = 0, aim = 0;                                                 \
                        for (int ci = 0; ci < Cin; ci++) {                                  \
                            const T *fp = f + (int64_t)ci * Din + in_off;                   \
                            for (int ii = 0; ii < n_in; ii++) {                             \
                                const int w = ci * Wdim + 2 * (oo * n_in + ii);             \
                                T a = omt * tl[w] + t * th[w];                              \
                                T b = omt * tl[w + 1] + t * th[w + 1];                      \
                                const T sc = NAME##_ipow(shw, lki[ii] + lko[oo]);           \
                                a *= sc; b *= sc;                                           \
                                const T fre = fp[2 * ii], fim = fp[2 * ii + 1];             \
                                are += a * fre + b * fim;                                   \
                                aim += a * fim - b * fre;                                   \
                            }                                                               \
                        }                                                                   \
                        o_e[(int64_t)co * Dout + out_off + 2 * oo] = are;                   \
                        o_e[(int64_t)co * Dout + out_off + 2 * oo + 1] = aim;               \
                    }                                                                       \
                }                                                                           \
            }                                                                               \
        }                                                                                   \
    }                                                                                       \
}                                                                                           \
int NAME(const T *features, const T *table, const T *dist, int64_t E, int Cin, int Cout,   \
         int Din, int Dout, int Wdim, const int *lin, int nlin, const int *lout, int nlout, \
         float sh_scale, float p1, float p2, int nb, int log_bins, T *out, int nthreads) {  \
    int params[ORACLE_MAX_L * ORACLE_BP_STRIDE];                                            \
    int lk_in[ORACLE_MAX_L * ORACLE_MAX_L], lk_out[ORACLE_MAX_L * ORACLE_MAX_L];            \
    int mmax = oracle_block_layout(lin, nlin, lout, nlout, params, lk_in, lk_out);          \
    if (mmax < 0) return -1;                                                                \
    memset(out, 0, sizeof(T) * (size_t)E * Cout * Dout);                                    \
    struct NAME##_job job;                                                                  \
    job.features = features; job.table = table; job.dist = dist;                            \
    job.Cin = Cin; job.Cout = Cout; job.Din = Din; job.Dout = Dout; job.Wdim = Wdim;        \
    job.sh_scale = sh_scale; job.p1 = p1; job.p2 = p2;                                      \
    job.nb = nb; job.log_bins = log_bins; job.mmax = mmax;                                  \
    job.tstride = (int64_t)Cout * Cin * Wdim;                                               \
    job.params = params; job.lk_in = lk_in; job.lk_out = lk_out; job.out = out;             \
    run_parallel(E, nthreads, NAME##_range, &job);                                          \
    return mmax;                                                                            \
}

DEFINE_BD_FWD(oracle_bd_fwd_f32, float)
DEFINE_BD_FWD(oracle_bd_fwd_f64, double)

int oracle_num_cpus(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
