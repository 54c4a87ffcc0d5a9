/*
 * TEST INFRASTRUCTURE ONLY -- the parity checker for the backward pass.
 * Nothing in the product (flash-eq_b200/) links, loads or calls this file.
 *
 * CPU restatement (float64, one thread, edges in order, so grad_table sums are
 * deterministic) of the backward of flash-eq's block-diagonal kernel
 * (flash_eq/cuda/csrc/block_diagonal.cu in hmblair/flash-eq):
 *
 *   backward_features_m0_kernel    block_diagonal.cu:748-830
 *       grad_f[e, ci, i] = sum_co sum_o s^(l_i+l_o) W_t[co, ci, w(o,i)] go[e, co, o]
 *   backward_features_mpos_kernel  block_diagonal.cu:832-923
 *       the transpose of [[a, b], [-b, a]]:  d/df_re = a go_re - b go_im,
 *                                            d/df_im = b go_re + a go_im
 *   backward_table_m0_kernel       block_diagonal.cu:925-1039
 *   backward_table_mpos_kernel     block_diagonal.cu:1041-1161
 *       grad_w = s^L f go (m = 0); for m > 0  grad_a = s^L (f_re go_re + f_im go_im),
 *       grad_b = s^L (f_im go_re - f_re go_im);
 *       grad_T[lo] += (1 - t) grad_w,  grad_T[hi] += t grad_w
 *       grad_t    += (T[hi] - T[lo]) grad_w
 *       grad_sh   += W_t grad_w L * scale / (d (d + scale))     (only for L = l_i + l_o > 0)
 *       grad_d     = grad_t * dt/dd + grad_sh
 *   binning_derivative             block_diagonal.cu:117-139   (linear: param2;
 *                                  log: 1 / (edge_hi - edge_lo) of the bin)
 *
 * The expression for grad_sh is kept as the reference writes it, so a zero
 * distance with L > 0 gives 0 * inf = NaN there, as in the reference.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORACLE_MAX_L 17
#define ORACLE_BP_STRIDE 6

int oracle_block_layout(const int *lin, int nlin, const int *lout, int nlout, int *params, int *lk_in,
                        int *lk_out);

static void bwd_binning(double d, float p1, float p2, int nb, int log_bins, int *lo, int *hi, double *t,
                        double *dtdd) {
    float normalized;
    const float df = (float)d;
    if (log_bins)
        normalized = (logf(fmaxf(df, expf(p1))) - p1) * p2 * nb;
    else
        normalized = (df - p1) * p2;
    normalized = fminf(fmaxf(normalized, 0.0f), (float)nb);
    int l = (int)floorf(normalized);
    if (l > nb - 1) l = nb - 1;
    *lo = l;
    *hi = (l + 1 < nb) ? l + 1 : nb;
    if (log_bins) {
        const double inv_lbw = (double)(p2 * nb);
        const double log_edge_lo = (double)p1 + (double)l / inv_lbw;
        const double edge_lo = exp(log_edge_lo);
        const double edge_hi = exp(log_edge_lo + 1.0 / inv_lbw);
        const double cd = d > edge_lo ? d : edge_lo;
        double tt = (cd - edge_lo) / (edge_hi - edge_lo);
        *t = tt < 1.0 ? tt : 1.0;
        *dtdd = 1.0 / (edge_hi - edge_lo);
    } else {
        const double bw = 1.0 / (double)p2;
        const double edge_lo = (double)p1 + (double)l * bw;
        *t = (d - edge_lo) / bw;
        *dtdd = (double)p2;
    }
}

static double ipow_d(double b, int ex) {
    double r = 1.0;
    while (ex > 0) {
        if (ex & 1) r *= b;
        b *= b;
        ex >>= 1;
    }
    return r;
}

/* features (E, Cin, Din) m-first, grad_out (E, Cout, Dout) m-first, table (nb+1, Cout, Cin, W).
 * Writes grad_features (E, Cin, Din), grad_table (nb+1, Cout, Cin, W), grad_dist (E). */
int oracle_bd_bwd_f64(const double *grad_out, const double *features, const double *table, const double *dist,
                      int64_t E, int Cin, int Cout, int Din, int Dout, int Wdim, const int *lin, int nlin,
                      const int *lout, int nlout, float sh_scale, float p1, float p2, int nb, int log_bins,
                      double *grad_features, double *grad_table, double *grad_dist) {
    int params[ORACLE_MAX_L * ORACLE_BP_STRIDE];
    int lk_in[ORACLE_MAX_L * ORACLE_MAX_L], lk_out[ORACLE_MAX_L * ORACLE_MAX_L];
    const int mmax = oracle_block_layout(lin, nlin, lout, nlout, params, lk_in, lk_out);
    if (mmax < 0) return -1;
    const int64_t tstride = (int64_t)Cout * Cin * Wdim;
    memset(grad_features, 0, sizeof(double) * (size_t)E * Cin * Din);
    memset(grad_table, 0, sizeof(double) * (size_t)(nb + 1) * tstride);
    memset(grad_dist, 0, sizeof(double) * (size_t)E);
    for (int64_t e = 0; e < E; e++) {
        const double d = dist[e];
        const double shw = d / (d + (double)sh_scale);
        const double deriv = (double)sh_scale / (d * (d + (double)sh_scale));
        int lo, hi;
        double t, dtdd;
        bwd_binning(d, p1, p2, nb, log_bins, &lo, &hi, &t, &dtdd);
        const double omt = 1.0 - t;
        const double *f = features + e * (int64_t)Cin * Din;
        const double *go = grad_out + e * (int64_t)Cout * Dout;
        double *gf = grad_features + e * (int64_t)Cin * Din;
        double gt = 0.0, gsh = 0.0;
        for (int m = 0; m <= mmax; m++) {
            const int *bp = params + m * ORACLE_BP_STRIDE;
            const int n_in = bp[1], n_out = bp[2], in_off = bp[3], out_off = bp[4], w_off = bp[5];
            if (n_in == 0 || n_out == 0) continue;
            const int *lki = lk_in + m * ORACLE_MAX_L, *lko = lk_out + m * ORACLE_MAX_L;
            for (int co = 0; co < Cout; co++) {
                const double *tl = table + lo * tstride + (int64_t)co * Cin * Wdim + w_off;
                const double *th = table + hi * tstride + (int64_t)co * Cin * Wdim + w_off;
                double *gl = grad_table + lo * tstride + (int64_t)co * Cin * Wdim + w_off;
                double *gh = grad_table + hi * tstride + (int64_t)co * Cin * Wdim + w_off;
                for (int ci = 0; ci < Cin; ci++) {
                    for (int oo = 0; oo < n_out; oo++) {
                        for (int ii = 0; ii < n_in; ii++) {
                            const int L = lki[ii] + lko[oo];
                            const double sc = ipow_d(shw, L);
                            if (m == 0) {
                                const int w = ci * Wdim + oo * n_in + ii;
                                const double fv = f[(int64_t)ci * Din + in_off + ii];
                                const double g = go[(int64_t)co * Dout + out_off + oo];
                                const double wt = omt * tl[w] + t * th[w];
                                gf[(int64_t)ci * Din + in_off + ii] += sc * wt * g;
                                const double grad_w = sc * fv * g;
                                gl[w] += omt * grad_w;
                                gh[w] += t * grad_w;
                                gt += (th[w] - tl[w]) * grad_w;
                                if (L > 0) gsh += wt * fv * g * sc * (double)L * deriv;
                            } else {
                                const int w = ci * Wdim + 2 * (oo * n_in + ii);
                                const double fre = f[(int64_t)ci * Din + in_off + 2 * ii];
                                const double fim = f[(int64_t)ci * Din + in_off + 2 * ii + 1];
                                const double gre = go[(int64_t)co * Dout + out_off + 2 * oo];
                                const double gim = go[(int64_t)co * Dout + out_off + 2 * oo + 1];
                                const double a = omt * tl[w] + t * th[w];
                                const double b = omt * tl[w + 1] + t * th[w + 1];
                                gf[(int64_t)ci * Din + in_off + 2 * ii] += sc * (a * gre - b * gim);
                                gf[(int64_t)ci * Din + in_off + 2 * ii + 1] += sc * (b * gre + a * gim);
                                const double ga_u = fre * gre + fim * gim;   /* before the s^L factor */
                                const double gb_u = fim * gre - fre * gim;
                                const double ga = sc * ga_u, gb = sc * gb_u;
                                gl[w] += omt * ga;
                                gl[w + 1] += omt * gb;
                                gh[w] += t * ga;
                                gh[w + 1] += t * gb;
                                gt += (th[w] - tl[w]) * ga + (th[w + 1] - tl[w + 1]) * gb;
                                if (L > 0) gsh += (a * ga_u + b * gb_u) * sc * (double)L * deriv;
                            }
                        }
                    }
                }
            }
        }
        grad_dist[e] = gt * dtdd + gsh;
    }
    return mmax;
}
