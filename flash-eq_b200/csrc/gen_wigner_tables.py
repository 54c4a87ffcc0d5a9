"""Build step: write the constant tables of the closed-form Wigner-D evaluation.

The reference builds every per-edge basis block as
    D_l = exp(theta * (a0 G0 + a1 G1)),   (a0, a1) = (-d_y, d_x) / |.|
with torch.linalg.matrix_exp (flash_eq/representations/wigner.py:144-240), where
[G0, G1, G2] are the so(3) generators in the reference's real spherical-harmonic
basis, ordered [Lz, Lx, Ly] (flash_eq/representations/types.py:86-135).

They satisfy [G0, G1] = G2, [G1, G2] = G0, [G2, G0] = G1, and G2 is "m-diagonal"
(it only couples index l-m with l+m).  Hence, with phi the polar angle of
(a0, a1) and R(a) = exp(a G2) (2x2 rotations by m*a on each (l-m, l+m) pair):
    a0 G0 + a1 G1 = |a| R(phi) G0 R(-phi)
    exp(theta G0) = U R(theta) U^T,           U = exp(pi/2 G1)
    D_l = R(phi) M(theta') R(phi)^T,          theta' = theta |a|
    M(theta') = sum_m cos(m theta') C_m + sin(m theta') S_m
with C_0 = u_l u_l^T, C_m = u_{l-m} u_{l-m}^T + u_{l+m} u_{l+m}^T,
S_m = u_{l-m} u_{l+m}^T - u_{l+m} u_{l-m}^T (u_j = column j of U).

This script evaluates U in float64 and emits, for l = 0..FEQ_MAX_L, the tensor
T_l[p][q][k] (k = 0: C_0; k = 2m-1: C_m; k = 2m: S_m) as device constants, so
a kernel evaluates M with 2l+1 multiply-adds per entry.  It also checks the
algebra it relies on and fails the build if any identity is off by > 1e-12.

Usage: python gen_wigner_tables.py OUT.inc [--lmax 16]
"""
from __future__ import annotations

import argparse
import sys

import numpy as np


def _so3_real_generators(l: int) -> np.ndarray:
    """[G0, G1, G2] = [Lz, Lx, Ly] in the reference's real SH basis, float64."""
    n = 2 * l + 1
    mm = np.arange(-l, l + 1)
    up = np.zeros((n, n), dtype=np.complex128)      # J+ below the diagonal (types.py:74-78)
    dn = np.zeros((n, n), dtype=np.complex128)      # J- above the diagonal (types.py:80-84)
    for i in range(n - 1):
        m = mm[i]
        up[i + 1, i] = -np.sqrt(l * (l + 1) - m * (m + 1))
        m2 = mm[i + 1]
        dn[i, i + 1] = np.sqrt(l * (l + 1) - m2 * (m2 - 1))
    jx = 0.5 * (up + dn)
    jy = -0.5j * (up - dn)
    jz = 1j * np.diag(mm.astype(np.complex128))
    # complex -> real change of basis (types.py:114-135)
    q = np.zeros((n, n), dtype=np.complex128)
    r2 = 1.0 / np.sqrt(2.0)
    for m in range(1, l + 1):
        q[l - m, l + m] = r2
        q[l - m, l - m] = -1j * r2
        q[l + m, l + m] = (-1) ** m * r2
        q[l + m, l - m] = 1j * (-1) ** m * r2
    q[l, l] = 1.0
    q = (-1j) ** l * q
    qh = q.conj().T
    conv = lambda j: (qh @ j @ q)
    gx, gy, gz = conv(jx), conv(jy), conv(jz)
    for g in (gx, gy, gz):
        assert np.abs(g.imag).max() < 1e-12
    # ordering [Lz, Lx, Ly] = [real(Q^H Jy Q), real(Q^H Jx Q), real(Q^H Jz Q)]
    return np.stack([gy.real, gx.real, gz.real])


def _expm(a: np.ndarray) -> np.ndarray:
    """exp(a) by scaling and squaring with a Taylor series (float64)."""
    nrm = np.abs(a).sum(axis=1).max()
    s = max(0, int(np.ceil(np.log2(max(nrm, 1e-300)))) + 4)
    x = a / (2.0 ** s)
    out = np.eye(a.shape[0])
    term = np.eye(a.shape[0])
    for k in range(1, 30):
        term = term @ x / k
        out = out + term
    for _ in range(s):
        out = out @ out
    return out


def tables_for(l: int) -> np.ndarray:
    n = 2 * l + 1
    if l == 0:
        return np.ones((1, 1, 1))
    g0, g1, g2 = _so3_real_generators(l)
    comm = lambda a, b: a @ b - b @ a
    for lhs, rhs in ((comm(g0, g1), g2), (comm(g1, g2), g0), (comm(g2, g0), g1)):
        assert np.abs(lhs - rhs).max() < 1e-12, l
    for m in range(1, l + 1):   # m-diagonal structure of G2
        assert abs(g2[l - m, l + m] - m) < 1e-12 and abs(g2[l + m, l - m] + m) < 1e-12, l
    u = _expm(0.5 * np.pi * g1)
    assert np.abs(u @ g2 @ u.T - g0).max() < 1e-12, l
    t = np.zeros((n, n, n))
    t[:, :, 0] = np.outer(u[:, l], u[:, l])
    for m in range(1, l + 1):
        a, b = l - m, l + m
        t[:, :, 2 * m - 1] = np.outer(u[:, a], u[:, a]) + np.outer(u[:, b], u[:, b])
        t[:, :, 2 * m] = np.outer(u[:, a], u[:, b]) - np.outer(u[:, b], u[:, a])
    # self-check against a direct exponential at a random angle pair
    rng = np.random.default_rng(l)
    th, ph = rng.uniform(0, np.pi), rng.uniform(-np.pi, np.pi)
    coef = np.zeros(n)
    coef[0] = 1.0
    for m in range(1, l + 1):
        coef[2 * m - 1], coef[2 * m] = np.cos(m * th), np.sin(m * th)
    mth = t @ coef
    r = np.zeros((n, n))
    r[l, l] = 1.0
    for m in range(1, l + 1):
        a, b = l - m, l + m
        c, s = np.cos(m * ph), np.sin(m * ph)
        r[a, a], r[b, b], r[a, b], r[b, a] = c, c, s, -s
    d = r @ mth @ r.T
    ref = _expm(th * (np.cos(ph) * g0 + np.sin(ph) * g1))
    assert np.abs(d - ref).max() < 1e-10, (l, np.abs(d - ref).max())
    return t


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("out")
    ap.add_argument("--lmax", type=int, default=16)
    ap.add_argument("--apply-out", default=None, help="also write the unrolled sparse M_l products here")
    args = ap.parse_args()
    offs, chunks, total = [], [], 0
    for l in range(args.lmax + 1):
        t = tables_for(l).astype(np.float32).reshape(-1)
        offs.append(total)
        chunks.append(t)
        total += t.size
    data = np.concatenate(chunks)
    with open(args.out, "w") as fh:
        fh.write("/* generated by gen_wigner_tables.py -- closed-form Wigner-D tables */\n")
        fh.write(f"#define FEQ_WT_LMAX {args.lmax}\n")
        fh.write(f"#define FEQ_WT_SIZE {total}\n")
        fh.write("__device__ const int feq_wt_offset[%d] = {%s};\n"
                 % (len(offs), ", ".join(str(o) for o in offs)))
        fh.write("__device__ const float feq_wt_data[FEQ_WT_SIZE] = {\n")
        for i in range(0, total, 8):
            fh.write("  " + ", ".join("%.9ef" % v for v in data[i:i + 8]) + ",\n")
        fh.write("};\n")
        # Compressed form: each M entry is a short sum over the few trig terms whose
        # coefficient is not zero (float32 round-off of exact zeros is dropped); every
        # entry of degree l carries exactly K_l (coefficient, term) slots, unused ones 0.
        coefs, qs, coffs, ks, ctotal = [], [], [], [], 0
        for l in range(args.lmax + 1):
            n = 2 * l + 1
            t = tables_for(l).reshape(n * n, n)
            keep = np.abs(t) > 1e-7
            k = max(1, int(keep.sum(axis=1).max()))
            c = np.zeros((n * n, k), dtype=np.float32)
            q = np.zeros((n * n, k), dtype=np.int64)
            for i in range(n * n):
                idx = np.nonzero(keep[i])[0]
                c[i, :len(idx)] = t[i, idx]
                q[i, :len(idx)] = idx
            coffs.append(ctotal)
            ks.append(k)
            coefs.append(c.reshape(-1))
            qs.append(q.reshape(-1))
            ctotal += n * n * k
        cdata, qdata = np.concatenate(coefs), np.concatenate(qs)
        fh.write(f"#define FEQ_WTC_SIZE {ctotal}\n")
        fh.write("__device__ const int feq_wtc_offset[%d] = {%s};\n" % (len(coffs), ", ".join(map(str, coffs))))
        fh.write("__device__ const int feq_wtc_k[%d] = {%s};\n" % (len(ks), ", ".join(map(str, ks))))
        fh.write("#define FEQ_WTC_K_UPTO4 {%s}\n" % ", ".join(map(str, ks[:5])))
        fh.write("__device__ const float feq_wtc_coef[FEQ_WTC_SIZE] = {\n")
        for i in range(0, ctotal, 8):
            fh.write("  " + ", ".join("%.9ef" % v for v in cdata[i:i + 8]) + ",\n")
        fh.write("};\n")
        fh.write("__device__ const unsigned char feq_wtc_term[FEQ_WTC_SIZE] = {\n")
        for i in range(0, ctotal, 32):
            fh.write("  " + ", ".join(str(int(v)) for v in qdata[i:i + 32]) + ",\n")
        fh.write("};\n")
    if args.apply_out:
        write_apply(args.apply_out, min(args.lmax, 6))
    return 0


def write_apply(path: str, lgen: int) -> None:
    """Unrolled per-degree code for the factored rotation D_l = R(phi) M_l R(phi)^T.

    feq_wm_l<l>(tv, sl, m):  the nonzero entries of s^l M_l(theta'), each a short sum of
                              the trig terms tv[k] with constant coefficients;
    feq_wmd_l<l>(tv, M):      all (2l+1)^2 entries of M_l(theta'), row-major (dense);
    feq_wa_l<l><kT>(m, g, h): h = g M_l (kT = false) or h = g M_l^T (kT = true), row
                              vectors, only the nonzero entries of M_l.
    """
    out = ["/* generated by gen_wigner_tables.py -- unrolled sparse M_l products */",
           f"#define FEQ_WA_LMAX {lgen}"]
    for l in range(1, lgen + 1):
        n = 2 * l + 1
        t = tables_for(l).astype(np.float32).astype(np.float64).reshape(n * n, n)
        ents = [i for i in range(n * n) if (np.abs(t[i]) > 1e-7).any()]
        slot = {e: k for k, e in enumerate(ents)}
        out.append(f"#define FEQ_WM_NNZ_{l} {len(ents)}")
        out.append(f"__device__ __forceinline__ void feq_wm_l{l}(const float *tv, float sl, float (&m)[{len(ents)}]) {{")
        for k, e in enumerate(ents):
            terms = [f"{t[e, q]:.9e}f * tv[{q}]" for q in range(n) if abs(t[e, q]) > 1e-7]
            out.append(f"    m[{k}] = sl * ({' + '.join(terms)});")
        out.append("}")
        out.append(f"__device__ __forceinline__ void feq_wmd_l{l}(const float *tv, float (&M)[{n * n}]) {{")
        for e in range(n * n):
            terms = [f"{t[e, q]:.9e}f * tv[{q}]" for q in range(n) if abs(t[e, q]) > 1e-7]
            out.append(f"    M[{e}] = {' + '.join(terms) if terms else '0.0f'};")
        out.append("}")
        out.append(f"template <bool kT> __device__ __forceinline__ void feq_wa_l{l}("
                   f"const float (&m)[{len(ents)}], const float (&g)[{n}], float (&h)[{n}]) {{")
        for tr in (False, True):
            out.append("    if (%skT) {" % ("" if tr else "!"))
            for o in range(n):
                terms = []
                for q in range(n):
                    e = (o * n + q) if tr else (q * n + o)   # g M: h[o] = sum_q g[q] M[q][o]
                    if e in slot:
                        terms.append(f"g[{q}] * m[{slot[e]}]")
                out.append(f"        h[{o}] = {' + '.join(terms) if terms else '0.0f'};")
            out.append("    }")
        out.append("}")
    with open(path, "w") as fh:
        fh.write("\n".join(out) + "\n")


if __name__ == "__main__":
    sys.exit(main())
