// feq_sepmix.cu -- the edgewise linear out = Q . Lambda(r) . P^T . f as ONE kernel, for the
// radial tables that EquivariantEdgewiseLinear builds: gather by src, rotation into the edge
// frame, the distance-interpolated block-diagonal mix and the rotation back, with neither
// the rotated rows nor the mix output ever leaving the SM.
//
// Reference behaviour replaced (flash_eq/layers/linear.py:100-160 with its radial net):
//   table[b, o, i, w] = sum_k C[k, o, i] f[b, k, w]        SeparableRadialNet.forward,
//                                                          flash_eq/layers/radial.py:259-275
//   f_diag = bmm(x[src], P)                                 linear.py:135-140
//   out_diag = block_diagonal_cuda(f_diag, table, r)        block_diagonal.cu:558-733
//   out = bmm(out_diag, Q^T)                                linear.py:160
//
// Formulation.  The table is separable with rank R (the module's ``rank``), so the
// interpolated weight of an edge is lerp_t(table)[o, i, w] = sum_k C[k, o, i] g_k[w] with
// g_k = (1 - t) f[lo, k] + t f[lo + 1, k].  The mix therefore factors into
//   Z_k[o, j] = sum_i C[k, o, i] a[i, j]         a = s^l_in (f . D) (rotated input, m-first)
//   h[o, q]   = sum_k sum_j G_k[q, j] Z_k[o, j]  G_k = the block-diagonal position mix of g_k
// The first step is one GEMM whose weight C is the same for every edge (kept in shared
// memory for the whole kernel): tcgen05.mma with C as the M side (rows (o, k)) and the
// rotated rows of a tile of edges as the N side, accumulating Z in TMEM.  No bin sort, no
// re-laid table, no two-bin doubling.  The second step is per-edge CUDA-core work in the
// epilogue, straight from TMEM, followed by the rotation back (s^l_out folded in) and one
// bulk store per output row.
//
// Roles (persistent, one CTA per SM, one edge tile after another):
//   warp 0      TMEM allocator; one thread issues tcgen05.mma
//   warp 1      loader: lane per edge, up to 32 edges ahead of the rotation warps: the
//               edge's scalars (bin, t, s = d / (d + sh_scale)) and a bulk copy of its input
//               row x[src[e]] into a ring of row buffers, so that enough bytes are in flight
//               to cover the HBM latency.  At L <= 2 it also forms the trig of the rotations
//               and the M_l nonzeros and copies the edge's two radial-feature rows into the
//               ring; at L >= 3 the rotation warp forms those with all 32 lanes and reads the
//               feature rows from L2 (a short ring of large rows would leave the
//               lane-per-edge loader only a few edges at a time)
//   next NROT   rotation in: rotate two channels per lane with the factored Wigner blocks,
//               write bf16 (hi, and lo in bf16x3 mode) into the K-major 128-byte-swizzled
//               N-side tile; per edge also the lerped g_k for the epilogue
//   then EWG    epilogue warpgroups: tcgen05.ld of Z, position mix, sum over k across lane
//               pairs, rotation back, bulk store
//   (L <= 2: 8 rotation warps, 3 epilogue warpgroups; L >= 3: 4 and 2)
// Rings: input rows, 2 N-side tiles, 2 TMEM accumulator sets, 4 (L <= 2) or 2 per-tile
// slots.  Every wait is bounded (limit from the launch); on time-out the kernel sets status
// 2, drains its copies and MMAs, frees TMEM and returns.  No TMA multicast anywhere.
//
// bf16x3 (float32-level accuracy): both operands split x = hi + lo, Z accumulates
// hi.hi + hi.lo + lo.hi.  bf16: hi only.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "feq_internal.cuh"
#include "feq_rot_common.cuh"
#include "feq_sm100.cuh"

namespace feq {
namespace sep {

using namespace sm100;
using namespace rot;

constexpr int kLoadWarp = 1;
constexpr int kRotWarp0 = 2;
constexpr int kNumEpi = 4;   // warps per epilogue warpgroup (one per TMEM lane quadrant)
// NROT rotation warps (warps 2 .. 2 + NROT - 1), then EWG epilogue warpgroups
__host__ __device__ constexpr int threads_for(int ewg, int nrot) { return (kRotWarp0 + nrot + kNumEpi * ewg) * 32; }
constexpr int kMaxRing = 32;    // input rows in flight per CTA (bulk copies), at most
constexpr int kStages = 2;      // N-side tiles
constexpr int kMaxSlots = 4;    // per-tile edge scalars (Geo::SLOTS of them)
constexpr int kBufs = 2;        // TMEM accumulator sets
constexpr int kCin = 64;        // K (one 128-byte swizzle row of bf16)
constexpr int kCout = 64;
constexpr int kRank = 4;
constexpr int kG = 128 / kCout;             // k values per 128-row slice and output channel
constexpr int kSlices = kRank / kG;         // 128-row M slices
constexpr uint32_t kTileBytes = 128 * 128;  // 128 rows x 128 B
static_assert(kRank % kG == 0, "rank must split evenly over the slices");
static_assert(kG == 2, "the lane-pair exchange below assumes two k values per slice");

// Compile-time geometry of lvals_in = [0..LIN] -> lvals_out = [0..LOUT].
template <int LIN, int LOUT>
struct Geo {
    static constexpr int LI = LIN, LO = LOUT;
    static constexpr int DIN = (LIN + 1) * (LIN + 1);
    static constexpr int DOUT = (LOUT + 1) * (LOUT + 1);
    static constexpr int MB = LIN < LOUT ? LIN : LOUT;     // last m-block with inputs and outputs
    static constexpr int LMAX = LIN > LOUT ? LIN : LOUT;
    static constexpr int ES = DIN <= 16 ? 16 : 32;          // TMEM columns / N rows per edge
    static constexpr int TE = 128 / ES;                     // edges per tile
    static constexpr int TF = trig_floats(LMAX);
    __host__ __device__ static constexpr int nin(int m) { return LIN - m + 1; }
    __host__ __device__ static constexpr int nout(int m) { return LOUT - m + 1; }
    __host__ __device__ static constexpr int mul(int m) { return m == 0 ? 1 : 2; }
    // block_diagonal.cu:1191-1266: offsets of block m (every block up to MB is non-empty)
    __host__ __device__ static constexpr int in_off(int m) {
        int o = 0;
        for (int q = 0; q < m; q++) o += mul(q) * nin(q);
        return o;
    }
    __host__ __device__ static constexpr int out_off(int m) {
        int o = 0;
        for (int q = 0; q < m; q++) o += mul(q) * nout(q);
        return o;
    }
    __host__ __device__ static constexpr int w_off(int m) {
        int o = 0;
        for (int q = 0; q < m; q++) o += mul(q) * nin(q) * nout(q);
        return o;
    }
    __host__ __device__ static constexpr int gsize(int m) { return mul(m) * nin(m) * nout(m); }
    __host__ __device__ static constexpr int gpad(int m) { return (gsize(m) + 3) & ~3; }
    __host__ __device__ static constexpr int goff(int m) {
        int o = 0;
        for (int q = 0; q < m; q++) o += gpad(q);
        return o;
    }
    static constexpr int W = w_off(MB + 1);      // ProductRepr(in, out).nreps()
    static constexpr int GP = goff(MB + 1);      // floats of one k's g, each block padded to 4
    // m-first position of (l, m) (flash_eq/representations/wigner.py:243-272)
    __host__ __device__ static constexpr int mf_in(int l, int m) {
        return m == 0 ? l : in_off(m < 0 ? -m : m) + 2 * (l - (m < 0 ? -m : m)) + (m < 0 ? 1 : 0);
    }
    __host__ __device__ static constexpr int mf_out(int l, int m) {
        return m == 0 ? l : out_off(m < 0 ? -m : m) + 2 * (l - (m < 0 ? -m : m)) + (m < 0 ? 1 : 0);
    }
    // the nonzeros of the factored Wigner block M_l (s^l folded in) of every degree 1..LMAX,
    // each degree's run padded to 4 floats
    __host__ __device__ static constexpr int mnnz(int l) {
        return l == 1 ? FEQ_WM_NNZ_1 : l == 2 ? FEQ_WM_NNZ_2 : l == 3 ? FEQ_WM_NNZ_3 : l == 4 ? FEQ_WM_NNZ_4 : 0;
    }
    __host__ __device__ static constexpr int moff(int l) {
        int o = 0;
        for (int q = 1; q < l; q++) o += pad4(mnnz(q));
        return o;
    }
    static constexpr int MF = moff(LMAX + 1);
    // per-edge record shared by the loader (writes), the rotation warps and the epilogue:
    // trig (cos / sin of the polar multiples and of m phi), s, t, bin (int), row flag (int),
    // then the M_l nonzeros
    static constexpr int REC_TRIG = 0;
    static constexpr int REC_S = TF, REC_T = TF + 1, REC_LO = TF + 2, REC_FLAG = TF + 3;
    static constexpr int REC_M = pad4(TF + 4);
    static constexpr int REC_FLOATS = REC_M + MF;
    // per-tile slot of one edge for the epilogue: the record, then g for every k
    static constexpr int SLOT_G = REC_FLOATS;
    static constexpr int SLOT_EDGE = SLOT_G + kRank * GP;     // floats per edge
    static constexpr int STAGE_ROW = ((kCout * DOUT + 15) / 32) * 32 + 16;   // == 16 mod 32 floats
    // L >= 3 (ROTREC): the rotation warp forms the trig and the M_l nonzeros of its edge and
    // reads the edge's two rows of radial features from L2 itself, so a ring entry carries only
    // the input row and a short job (direction, s, t, bin, flag).  This keeps entries small
    // enough for a ring that prefetches (8 rows at L = 4, bf16x3).  Below, the loader forms the
    // whole record and the feature rows travel in the ring.
    static constexpr bool ROTREC = LMAX >= 3;
    static constexpr int J_S = ROTREC ? 3 : REC_S, J_T = J_S + 1, J_LO = J_S + 2, J_FLAG = J_S + 3;
    static constexpr int JOB_FLOATS = ROTREC ? 8 : REC_FLOATS;
    static constexpr int FR = ROTREC ? 0 : (2 * kRank * W + 3) & ~3;     // feature-row floats per entry
    // per-tile slots of edge scalars: 4, or 2 at L >= 3 where shared memory is short (the
    // rotation warps then run at most 2 tiles ahead of the epilogue; the memory goes to the
    // row ring instead: at L = 4 with two epilogue warpgroups 8 rows instead of 4, 6.1 -> 5.4 ms
    // on 640 000 edges)
    static constexpr int SLOTS = ROTREC ? 2 : 4;
};

struct SepParams {
    const float *x;
    const int64_t *src;
    int64_t nsrc;
    const float *edge_add;
    const float *dirs;
    const float *dist;
    const float *cpat;        // (rank, c_out, c_in)
    const float *ftab;        // (num_bins + 1, rank, W)
    float *out;
    int32_t *status;
    int64_t E;
    int64_t num_tiles;
    Binning bins;
    float sh_scale;
    uint64_t wait_ns;
    int nr;                   // input-row ring size (<= kMaxRing)
};

// Byte offset of element (row r, column c) in a 128-row K-major tile of 64 bf16 per row with
// the 128-byte swizzle (16-byte chunk index XOR row % 8; 8-row atoms of 1024 B).
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7))) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ void named_bar(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t (&r)[32]) {
    tmem_ld32(taddr, r);
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// One channel of one irrep of degree Lg, in registers, through D = R(phi) M R(phi)^T
// (as rot::rot_irrep2, for a single channel): kT = false y = x D, kT = true y = x D^T.
template <int Lg, bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot_irrep1(const float *__restrict__ tr, int lmax, float sl, Get get, Emit emit) {
    if constexpr (Lg == 0) {
        emit(0, get(0) * sl);
    } else {
        constexpr int N = 2 * Lg + 1;
        const float *tv = tr, *cp = tr + 2 * lmax + 1, *sp = cp + lmax + 1;
        float m[WA<Lg>::kNnz];
        WA<Lg>::wm(tv, sl, m);
        float g[N];
#pragma unroll
        for (int q = 0; q < N; q++) g[q] = get(q);
#pragma unroll
        for (int mm = 1; mm <= Lg; mm++) {
            const int a = Lg - mm, b = Lg + mm;
            const float c = cp[mm], s = sp[mm];
            const float t0 = g[a] * c - g[b] * s, t1 = g[a] * s + g[b] * c;
            g[a] = t0;
            g[b] = t1;
        }
        float h[N];
        WA<Lg>::template wa<kT>(m, g, h);
#pragma unroll
        for (int mm = 1; mm <= Lg; mm++) {
            const int a = Lg - mm, b = Lg + mm;
            const float c = cp[mm], s = sp[mm];
            const float t0 = h[a] * c + h[b] * s, t1 = h[b] * c - h[a] * s;
            h[a] = t0;
            h[b] = t1;
        }
#pragma unroll
        for (int o = 0; o < N; o++) emit(o, h[o]);
    }
}

template <int Lg, bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot_irrep2c(const float *__restrict__ tr, int lmax, float sl, Get get, Emit emit) {
    if constexpr (Lg == 0) {
        const float2 v = get(0);
        emit(0, v.x * sl, v.y * sl);
    } else {
        rot_irrep2<Lg, kT>(tr, lmax, sl, get, emit);
    }
}

// n floats from 16-byte aligned shared memory into registers (float4 loads).
template <int NZ>
__device__ __forceinline__ void load_m(const float *__restrict__ src, float (&m)[NZ]);

template <int NZ>
__device__ __forceinline__ void load_regs(const float *__restrict__ src, float (&m)[NZ]) {
    load_m<NZ>(src, m);
}

template <int NZ>
__device__ __forceinline__ void load_m(const float *__restrict__ src, float (&m)[NZ]) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int v = 0; v < NZ / 4; v++) {
        const float4 t = s4[v];
        m[4 * v] = t.x;
        m[4 * v + 1] = t.y;
        m[4 * v + 2] = t.z;
        m[4 * v + 3] = t.w;
    }
#pragma unroll
    for (int v = (NZ / 4) * 4; v < NZ; v++) m[v] = src[v];
}

// One irrep of degree Lg through D = R(phi) M R(phi)^T with the nonzeros of M (s^l folded
// in) given in registers; cp / sp: cos / sin of m phi.  Two channels (emit(o, y0, y1)).
template <int Lg, bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot2_m(const float (&m)[Lg == 0 ? 1 : WA<(Lg > 0 ? Lg : 1)>::kNnz],
                                       const float *__restrict__ cp, const float *__restrict__ sp, Get get,
                                       Emit emit) {
    if constexpr (Lg == 0) {
        const float2 v = get(0);
        emit(0, v.x, v.y);
    } else {
        constexpr int N = 2 * Lg + 1;
        float g0[N], g1[N];
#pragma unroll
        for (int q = 0; q < N; q++) {
            const float2 v = get(q);
            g0[q] = v.x;
            g1[q] = v.y;
        }
#pragma unroll
        for (int mm = 1; mm <= Lg; mm++) {
            const int a = Lg - mm, b = Lg + mm;
            const float c = cp[mm], sn = sp[mm];
            float t0 = g0[a] * c - g0[b] * sn, t1 = g0[a] * sn + g0[b] * c;
            g0[a] = t0;
            g0[b] = t1;
            t0 = g1[a] * c - g1[b] * sn;
            t1 = g1[a] * sn + g1[b] * c;
            g1[a] = t0;
            g1[b] = t1;
        }
        float h0[N], h1[N];
        WA<Lg>::template wa<kT>(m, g0, h0);
        WA<Lg>::template wa<kT>(m, g1, h1);
#pragma unroll
        for (int mm = 1; mm <= Lg; mm++) {
            const int a = Lg - mm, b = Lg + mm;
            const float c = cp[mm], sn = sp[mm];
            float t0 = h0[a] * c + h0[b] * sn, t1 = h0[b] * c - h0[a] * sn;
            h0[a] = t0;
            h0[b] = t1;
            t0 = h1[a] * c + h1[b] * sn;
            t1 = h1[b] * c - h1[a] * sn;
            h1[a] = t0;
            h1[b] = t1;
        }
#pragma unroll
        for (int o = 0; o < N; o++) emit(o, h0[o], h1[o]);
    }
}

// The same with the nonzeros of M read from msm (shared memory).
template <int Lg, bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot2_pre(const float *__restrict__ msm, const float *__restrict__ cp,
                                         const float *__restrict__ sp, Get get, Emit emit) {
    if constexpr (Lg == 0) {
        const float2 v = get(0);
        emit(0, v.x, v.y);
    } else {
        float m[WA<Lg>::kNnz];
        load_m(msm, m);
        rot2_m<Lg, kT>(m, cp, sp, get, emit);
    }
}

// The same for one channel.
template <int Lg, bool kT, typename Get, typename Emit>
__device__ __forceinline__ void rot1_pre(const float *__restrict__ msm, const float *__restrict__ cp,
                                         const float *__restrict__ sp, Get get, Emit emit) {
    if constexpr (Lg == 0) {
        emit(0, get(0));
    } else {
        constexpr int N = 2 * Lg + 1;
        float m[WA<Lg>::kNnz];
        load_m(msm, m);
        float g[N];
#pragma unroll
        for (int q = 0; q < N; q++) g[q] = get(q);
#pragma unroll
        for (int mm = 1; mm <= Lg; mm++) {
            const int a = Lg - mm, b = Lg + mm;
            const float c = cp[mm], sn = sp[mm];
            const float t0 = g[a] * c - g[b] * sn, t1 = g[a] * sn + g[b] * c;
            g[a] = t0;
            g[b] = t1;
        }
        float h[N];
        WA<Lg>::template wa<kT>(m, g, h);
#pragma unroll
        for (int mm = 1; mm <= Lg; mm++) {
            const int a = Lg - mm, b = Lg + mm;
            const float c = cp[mm], sn = sp[mm];
            const float t0 = h[a] * c + h[b] * sn, t1 = h[b] * c - h[a] * sn;
            h[a] = t0;
            h[b] = t1;
        }
#pragma unroll
        for (int o = 0; o < N; o++) emit(o, h[o]);
    }
}

// M_l nonzeros of every degree 1..LMAX of one edge (s^l folded in) into rec + REC_M.
template <class GE, int L>
__device__ __forceinline__ void fill_m(const float *__restrict__ tv, float s, float *__restrict__ rec) {
    if constexpr (L <= GE::LMAX) {
        float m[WA<L>::kNnz];
        WA<L>::wm(tv, ipowf(s, L), m);
#pragma unroll
        for (int v = 0; v < WA<L>::kNnz; v++) rec[GE::REC_M + GE::moff(L) + v] = m[v];
        fill_m<GE, L + 1>(tv, s, rec);
    }
}

// h[q] += sum_j G[q, j] Z[j] for the blocks m = M..MB of one k (G in shared memory, padded
// per block; Z this thread's TMEM row for one edge).  m = 0: out[o] += g[o n_in + i] z[i];
// m > 0: 2x2 [[a, b], [-b, a]] on the (+m, -m) pairs (block_diagonal.cu:558-733).
template <class GE, int M, int ES>
__device__ __forceinline__ void pos_mix(const uint32_t (&Z)[ES], const float *__restrict__ G,
                                        float (&h)[GE::DOUT]) {
    if constexpr (M <= GE::MB) {
        constexpr int ni = GE::nin(M), no = GE::nout(M), io = GE::in_off(M), oo_ = GE::out_off(M);
        constexpr int np = GE::gpad(M);
        float g[np];
        const float4 *g4 = reinterpret_cast<const float4 *>(G + GE::goff(M));
#pragma unroll
        for (int v = 0; v < np / 4; v++) {
            const float4 t = g4[v];
            g[4 * v] = t.x;
            g[4 * v + 1] = t.y;
            g[4 * v + 2] = t.z;
            g[4 * v + 3] = t.w;
        }
        if constexpr (M == 0) {
#pragma unroll
            for (int o = 0; o < no; o++) {
                float acc = h[oo_ + o];
#pragma unroll
                for (int i = 0; i < ni; i++) acc = fmaf(g[o * ni + i], __uint_as_float(Z[io + i]), acc);
                h[oo_ + o] = acc;
            }
        } else {
#pragma unroll
            for (int o = 0; o < no; o++) {
                float re = h[oo_ + 2 * o], im = h[oo_ + 2 * o + 1];
#pragma unroll
                for (int i = 0; i < ni; i++) {
                    const float a = g[2 * (o * ni + i)], b = g[2 * (o * ni + i) + 1];
                    const float zr = __uint_as_float(Z[io + 2 * i]), zi = __uint_as_float(Z[io + 2 * i + 1]);
                    re = fmaf(a, zr, fmaf(b, zi, re));
                    im = fmaf(a, zi, fmaf(-b, zr, im));
                }
                h[oo_ + 2 * o] = re;
                h[oo_ + 2 * o + 1] = im;
            }
        }
        pos_mix<GE, M + 1, ES>(Z, G, h);
    }
}

// Input rotation of one irrep degree L (recursing to LIN) for the channel pair (c, c + 1);
// rec: the edge's record (trig, M_l nonzeros).
// The N-side rows of an edge start at a multiple of 8 rows (ES is 16 or 32), so the 128-byte
// swizzle of row r = row0 + j depends on j only: byte offset j * 128 + xo[j & 7], with
// xo[k] = ((c / 8) ^ k) * 16 + (c % 8) * 2 for this lane's channel pair c (swz above).
template <class GE, int L, bool kSplit>
__device__ __forceinline__ void rotate_in_all(const float *__restrict__ rec, const float *__restrict__ cp,
                                              const float *__restrict__ sp, const float *__restrict__ f0,
                                              const float *__restrict__ f1, uint8_t *bhi, uint8_t *blo,
                                              const uint32_t (&xo)[8]) {
    if constexpr (L <= GE::LI) {
        constexpr int off = L * L;    // standard offset of degree L in [0..LIN]
        auto get = [&](int q) { return make_float2(f0[off + q], f1[off + q]); };
        auto emit = [&](int o, float y0, float y1) {
            const int jm = GE::mf_in(L, o - L);
            const uint32_t bo = (uint32_t)jm * 128u + xo[jm & 7];
            const __nv_bfloat162 hi = __floats2bfloat162_rn(y0, y1);
            *reinterpret_cast<__nv_bfloat162 *>(bhi + bo) = hi;
            if (kSplit) {
                const float2 hf = __bfloat1622float2(hi);
                *reinterpret_cast<__nv_bfloat162 *>(blo + bo) = __floats2bfloat162_rn(y0 - hf.x, y1 - hf.y);
            }
        };
        rot2_pre<L, false>(rec + GE::REC_M + GE::moff(L), cp, sp, get, emit);
        rotate_in_all<GE, L + 1, kSplit>(rec, cp, sp, f0, f1, bhi, blo, xo);
    }
}

// As rotate_in_all, but the warp forms the M_l nonzeros of every degree itself from the edge's
// trig (tv) and s (every lane the same values), rotates with them from registers and stores them
// at rec + REC_M for the epilogue's rotation back.
template <class GE, int L, bool kSplit>
__device__ __forceinline__ void rotate_in_all_m(const float *__restrict__ tv, float s, float *__restrict__ rec,
                                                const float *__restrict__ cp, const float *__restrict__ sp,
                                                const float *__restrict__ f0, const float *__restrict__ f1,
                                                uint8_t *bhi, uint8_t *blo, const uint32_t (&xo)[8]) {
    if constexpr (L <= GE::LI) {
        constexpr int off = L * L;
        auto get = [&](int q) { return make_float2(f0[off + q], f1[off + q]); };
        auto emit = [&](int o, float y0, float y1) {
            const int jm = GE::mf_in(L, o - L);
            const uint32_t bo = (uint32_t)jm * 128u + xo[jm & 7];
            const __nv_bfloat162 hi = __floats2bfloat162_rn(y0, y1);
            *reinterpret_cast<__nv_bfloat162 *>(bhi + bo) = hi;
            if (kSplit) {
                const float2 hf = __bfloat1622float2(hi);
                *reinterpret_cast<__nv_bfloat162 *>(blo + bo) = __floats2bfloat162_rn(y0 - hf.x, y1 - hf.y);
            }
        };
        if constexpr (L == 0) {
            float m0[1] = {1.0f};
            rot2_m<0, false>(m0, cp, sp, get, emit);
        } else {
            constexpr int NZ = WA<L>::kNnz;
            float m[NZ];
            WA<L>::wm(tv, ipowf(s, L), m);
            float *dst = rec + GE::REC_M + GE::moff(L);
#pragma unroll
            for (int v = 0; v + 3 < NZ; v += 4) *reinterpret_cast<float4 *>(dst + v) = make_float4(m[v], m[v + 1], m[v + 2], m[v + 3]);
#pragma unroll
            for (int v = (NZ / 4) * 4; v < NZ; v++) dst[v] = m[v];
            rot2_m<L, false>(m, cp, sp, get, emit);
        }
        rotate_in_all_m<GE, L + 1, kSplit>(tv, s, rec, cp, sp, f0, f1, bhi, blo, xo);
    }
}

// Output rotation of every degree of [0..LOUT] for one channel of one edge, into the
// staging row (standard order).
template <class GE, int L>
__device__ __forceinline__ void rotate_out_all(const float *__restrict__ rec, const float *__restrict__ cp,
                                               const float *__restrict__ sp, const float (&h)[GE::DOUT],
                                               float *__restrict__ orow) {
    if constexpr (L <= GE::LO) {
        constexpr int off = L * L;
        auto get = [&](int q) { return h[GE::mf_out(L, q - L)]; };
        auto emit = [&](int o, float y) { orow[off + o] = y; };
        rot1_pre<L, true>(rec + GE::REC_M + GE::moff(L), cp, sp, get, emit);
        rotate_out_all<GE, L + 1>(rec, cp, sp, h, orow);
    }
}

// EWG epilogue warpgroups (1 or 2): with 2 the groups of a tile alternate between them, so each
// SM sub-partition runs two epilogue warps and one hides the other's latencies.  NROT rotation
// warps (4 or 8) share the edges of a tile the same way.  Every warp runs long dependent chains,
// so where the registers allow, more warps per sub-partition is what keeps the issue slots busy.
template <int LIN, int LOUT, bool kSplit, int EWG, int NROT>
__global__ void __launch_bounds__(threads_for(EWG, NROT), 1)
sep_edgewise_kernel(const __grid_constant__ SepParams P) {
    using GE = Geo<LIN, LOUT>;
    constexpr int kThreads = threads_for(EWG, NROT);
    constexpr int kNumRot = NROT;
    constexpr int kEpiWarp0 = kRotWarp0 + NROT;
    constexpr int ES = GE::ES, TE = GE::TE, DIN = GE::DIN, DOUT = GE::DOUT;
    constexpr int ROWF = kCin * DIN;                       // input row floats
    constexpr int ROWF_PAD = (ROWF + 3) & ~3;
    constexpr int OUTF = kCout * DOUT;                     // output row floats
    constexpr uint32_t kIdesc = idesc_bf16_f32(128, 128);
    constexpr int kSplitN = kSplit ? 2 : 1;
    constexpr int JS = GE::JOB_FLOATS;
    constexpr int FRB = 2 * kRank * GE::W * 4;                        // bytes of two rows of f
    constexpr int FR = GE::FR;
    // L >= 3: the per-edge trig and M_l nonzeros are formed by the rotation warp (32 lanes per
    // edge) instead of the loader (a lane per edge): with a short row ring of large rows the
    // loader would otherwise prepare only a few edges at a time.
    constexpr bool kRotRec = GE::ROTREC;
    static_assert(TE % kNumRot == 0 && TE % kG == 0, "tile edges split over the warps");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *a_hi = smem;                                            // kSlices tiles
    uint8_t *a_lo = a_hi + kSlices * kTileBytes;                      // (split only)
    uint8_t *b_base = a_hi + kSplitN * kSlices * kTileBytes;          // kStages x (hi [, lo])
    float *slots = reinterpret_cast<float *>(b_base + kStages * kSplitN * kTileBytes);
    float *stage = slots + GE::SLOTS * TE * GE::SLOT_EDGE;
    float *jobs = stage + EWG * kG * GE::STAGE_ROW;                   // nr x JS per-edge records
    float *frows = jobs + (size_t)P.nr * JS;                          // nr x FR: rows lo, lo + 1 of f
    float *rows = frows + (size_t)P.nr * FR;                          // nr input rows

    __shared__ uint64_t b_full[kStages], b_empty[kStages], t_full[kBufs], t_empty[kBufs], s_empty[kMaxSlots];
    __shared__ uint64_t r_full[kMaxRing], r_free[kMaxRing], drain_bar;
    __shared__ int64_t r_issued[kMaxRing];
    __shared__ int16_t gidx_s[kRank * GE::GP];     // g slot -> index into one bin row of f (-1: pad)
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s, epi_stop_s[4];    // per epilogue warpgroup

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NR = P.nr;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; i++) epi_stop_s[i] = 0;
        for (int i = 0; i < kStages; i++) {
            mbar_init(&b_full[i], kNumRot);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kBufs; i++) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], kNumEpi * EWG);
        }
        for (int i = 0; i < GE::SLOTS; i++) mbar_init(&s_empty[i], kNumEpi * EWG);
        for (int i = 0; i < kMaxRing; i++) {
            mbar_init(&r_full[i], 1);
            mbar_init(&r_free[i], 1);
            r_issued[i] = -1;
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base_s, 512);
        tmem_relinquish();
    }
    // Channel patterns -> M-side tiles: slice s, row r = co * kG + kk holds C[s * kG + kk][co][:].
    for (int idx = threadIdx.x; idx < kSlices * 128 * kCin; idx += kThreads) {
        const int s = idx / (128 * kCin), rem = idx - s * 128 * kCin;
        const int r = rem / kCin, c = rem - r * kCin;
        const int co = r / kG, k = s * kG + (r % kG);
        const float v = __ldg(P.cpat + ((int64_t)k * kCout + co) * kCin + c);
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        *reinterpret_cast<__nv_bfloat16 *>(a_hi + s * kTileBytes + swz(r, c)) = hi;
        if (kSplit)
            *reinterpret_cast<__nv_bfloat16 *>(a_lo + s * kTileBytes + swz(r, c)) =
                __float2bfloat16_rn(v - __bfloat162float(hi));
    }
    // N-side tiles start at zero: rows of the padding positions (j >= d_in of every edge)
    // are never written again.
    for (int i = threadIdx.x; i < (int)(kStages * kSplitN * kTileBytes / 16); i += kThreads)
        reinterpret_cast<uint4 *>(b_base)[i] = make_uint4(0u, 0u, 0u, 0u);
    // g layout: per k, per m-block, the block's weights padded to 4 floats
    for (int idx = threadIdx.x; idx < kRank * GE::GP; idx += kThreads) {
        const int k = idx / GE::GP, p = idx - k * GE::GP;
        int wi = -1;
        for (int m = 0; m <= GE::MB; m++)
            if (p >= GE::goff(m) && p - GE::goff(m) < GE::gsize(m)) wi = k * GE::W + GE::w_off(m) + (p - GE::goff(m));
        gidx_s[idx] = (int16_t)wi;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    volatile int *abort_flag = &abort_s;
    const int64_t n_local = P.num_tiles > blockIdx.x ? (P.num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int64_t n_jobs = n_local * TE;     // job j = edge j % TE of this CTA's tile j / TE
    auto edge_of_job = [&](int64_t j) -> int64_t {
        return (blockIdx.x + (j / TE) * gridDim.x) * TE + (j % TE);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            for (int64_t i = 0; i < n_local && !*abort_flag; i++) {
                const int st = (int)(i % kStages), buf = (int)(i % kBufs);
                if (!mbar_wait(&b_full[st], (uint32_t)((i / kStages) & 1), abort_flag, P.wait_ns)) break;
                if (i >= kBufs && !mbar_wait(&t_empty[buf], (uint32_t)((i / kBufs - 1) & 1), abort_flag, P.wait_ns))
                    break;
                tc_fence_after();
                const uint32_t bh = smem_u32(b_base + st * kSplitN * kTileBytes);
                const uint32_t bl = bh + kTileBytes;
#pragma unroll
                for (int s = 0; s < kSlices; s++) {
                    const uint32_t d = tmem + (uint32_t)(buf * kSlices * 128 + s * 128);
                    const uint32_t ah = smem_u32(a_hi + s * kTileBytes), al = smem_u32(a_lo + s * kTileBytes);
#pragma unroll
                    for (int ks = 0; ks < kCin / 16; ks++) {
                        const uint32_t ko = ks * 32;
                        umma_f16(d, smem_desc_sw128(ah + ko), smem_desc_sw128(bh + ko), kIdesc, ks > 0 ? 1u : 0u);
                        if (kSplit) {
                            umma_f16(d, smem_desc_sw128(ah + ko), smem_desc_sw128(bl + ko), kIdesc, 1u);
                            umma_f16(d, smem_desc_sw128(al + ko), smem_desc_sw128(bh + ko), kIdesc, 1u);
                        }
                    }
                }
                umma_commit(&b_empty[st]);
                umma_commit(&t_full[buf]);
            }
            umma_commit(&drain_bar);
            mbar_wait_drain(&drain_bar, 0);
        }
    } else if (warp == kLoadWarp) {
        // ---------------- loader: edge scalars + input rows, lane per edge ----------------
        // Batches of NB = nr / 2 jobs: a batch only waits for the buffers of the batch two back,
        // so one batch is always in flight while the next is prepared.  The next batch's edge
        // inputs (distance, direction, src) are fetched before this batch is processed.
        const int NB = NR / 2 < 32 ? NR / 2 : 32;
        float nd = 0.0f, nx = 0.0f, ny = 0.0f, nz = 0.0f;
        int64_t nrow = -1;
        auto fetch = [&](int64_t b0) {
            const int64_t j = b0 + lane;
            if (lane < NB && j < n_jobs) {
                const int64_t e = edge_of_job(j);
                if (e < P.E) {
                    nd = P.dist[e];
                    nx = P.dirs[e * 3];
                    ny = P.dirs[e * 3 + 1];
                    nz = P.dirs[e * 3 + 2];
                    nrow = P.src ? P.src[e] : e;
                }
            }
        };
        fetch(0);
        uint32_t bidx = 0;
        for (int64_t base = 0; base < n_jobs; base += NB, bidx++) {
            const float dd = nd, vx = nx, vy = ny, vz = nz;
            const int64_t row = nrow;
            fetch(base + NB);
            const int64_t j = base + lane;
            bool ok = true;
            if (lane < NB && j < n_jobs) {
                const int r = (int)(bidx & 1u) * NB + lane;
                if (bidx >= 2) ok = mbar_wait(&r_free[r], ((bidx >> 1) - 1u) & 1u, abort_flag, P.wait_ns);
                if (ok) {
                    float *sc = jobs + (size_t)r * JS;
                    int *sci = reinterpret_cast<int *>(sc);
                    const int64_t e = edge_of_job(j);
                    int flag = 2;                         // 0 row copied, 1 bad src (zero row), 2 no edge
                    int lo = 0;
                    if (e < P.E) {
                        float t;
                        bin_of(dd, P.bins, lo, t);
                        const float sw = dd / (dd + P.sh_scale);
                        if constexpr (kRotRec) {          // the rotation warp derives the rest
                            sc[GE::REC_TRIG] = vx;
                            sc[GE::REC_TRIG + 1] = vy;
                            sc[GE::REC_TRIG + 2] = vz;
                        } else {
                            float tr[GE::TF];
                            edge_trig_compact(vx, vy, vz, GE::LMAX, tr);
#pragma unroll
                            for (int q = 0; q < GE::TF; q++) sc[GE::REC_TRIG + q] = tr[q];
                            fill_m<GE, 1>(tr, sw, sc);
                        }
                        sc[GE::J_S] = sw;
                        sc[GE::J_T] = t;
                        sci[GE::J_LO] = lo;
                        if (row < 0 || row >= P.nsrc) {
                            set_status(P.status, 1);
                            flag = 1;
                        } else {
                            flag = 0;
                        }
                    }
                    sci[GE::J_FLAG] = flag;
                    r_issued[r] = j;
                    constexpr uint32_t kFrb = FR > 0 ? FRB : 0;
                    if (flag == 0 || (flag == 1 && FR > 0)) {
                        // the edge's input row, and (L <= 2) its two rows of radial features
                        // (bins lo, lo + 1)
                        fence_async_smem();
                        mbar_arrive_expect_tx(&r_full[r], kFrb + (flag == 0 ? ROWF * 4 : 0));
                        if constexpr (FR > 0)
                            bulk_load(frows + (size_t)r * FR, P.ftab + (int64_t)lo * kRank * GE::W, FRB, &r_full[r]);
                        if (flag == 0)
                            bulk_load(rows + (size_t)r * ROWF_PAD, P.x + row * (int64_t)ROWF, ROWF * 4, &r_full[r]);
                    } else {
                        mbar_arrive(&r_full[r]);
                    }
                }
            }
            if (__any_sync(0xffffffffu, !ok)) break;
        }
        __syncwarp();
        // drain: every copy issued must have landed before the CTA exits
        if (lane == 0)
            for (int r = 0; r < NR; r++)
                if (r_issued[r] >= 0) mbar_wait_drain(&r_full[r], (uint32_t)((r_issued[r] / NR) & 1));
    } else if (warp < kEpiWarp0) {
        // ---------------- rotation in ----------------
        const int w = warp - kRotWarp0;
        constexpr int EPW = TE / kNumRot;                  // edges of one tile per rotation warp
        uint32_t xo[8];
#pragma unroll
        for (int k = 0; k < 8; k++) xo[k] = (uint32_t)((((lane >> 2) ^ k) << 4) + ((2 * lane) & 7) * 2);
        const int64_t n_mine = n_local * EPW;
        const int NT = NR / TE;
        int ti = 0;
        uint32_t pass = 0;
        for (int64_t q = 0; q < n_mine; q++) {
            const int64_t i = q / EPW;
            const int st = (int)(i % kStages), slot = (int)(i % GE::SLOTS);
            const int sub = (int)(q - i * EPW);
            const int el = w + kNumRot * sub;
            if (q > 0 && sub == 0 && ++ti == NT) {
                ti = 0;
                pass++;
            }
            const int r = ti * TE + el;
            if (q % EPW == 0) {       // first edge of this warp in tile i: wait for its buffers
                if (i >= kStages &&
                    !mbar_wait(&b_empty[st], (uint32_t)((i / kStages - 1) & 1), abort_flag, P.wait_ns))
                    break;
                if (i >= GE::SLOTS &&
                    !mbar_wait(&s_empty[slot], (uint32_t)((i / GE::SLOTS - 1) & 1), abort_flag, P.wait_ns))
                    break;
            }
            if (!mbar_wait(&r_full[r], pass & 1u, abort_flag, P.wait_ns)) {
                set_status(P.status, 2);
                break;
            }
            const float *sc = jobs + (size_t)r * JS;
            const int flag = reinterpret_cast<const int *>(sc)[GE::J_FLAG];
            if (flag != 2) {
                const int64_t e = edge_of_job(i * TE + el);
                float *sl = slots + (size_t)(slot * TE + el) * GE::SLOT_EDGE;
                float tr[GE::TF];
                const float t = sc[GE::J_T];
                if constexpr (kRotRec) {
                    // every lane forms the edge's trig (the same values); the record for the
                    // epilogue gets it here and the M_l nonzeros in rotate_in_all_m
                    edge_trig_compact(sc[GE::REC_TRIG], sc[GE::REC_TRIG + 1], sc[GE::REC_TRIG + 2], GE::LMAX, tr);
#pragma unroll
                    for (int q = 0; q < GE::TF; q++) sl[GE::REC_TRIG + q] = tr[q];
                    if (lane < 4) sl[GE::REC_S + lane] = sc[GE::J_S + lane];     // s, t, bin, flag
                } else {
                    load_regs<GE::TF>(sc + GE::REC_TRIG, tr);
                    for (int qq = lane; qq < GE::REC_FLOATS; qq += 32) sl[qq] = sc[qq];   // record for the epilogue
                }
                // g_k = (1 - t) f[lo, k] + t f[lo + 1, k], per block padded to 4 floats
                constexpr int GI = (kRank * GE::GP + 31) / 32;
                float gl[GI], gh[GI];
                {
                    const float *f_lo;
                    if constexpr (FR > 0)           // arrived with the input row
                        f_lo = frows + (size_t)r * FR;
                    else                            // read from L2 (the table is small)
                        f_lo = P.ftab + (int64_t)reinterpret_cast<const int *>(sc)[GE::J_LO] * kRank * GE::W;
                    const float *f_hi = f_lo + kRank * GE::W;
#pragma unroll
                    for (int u = 0; u < GI; u++) {
                        const int idx = lane + 32 * u;
                        const int wi = idx < kRank * GE::GP ? gidx_s[idx] : -1;
                        gl[u] = wi >= 0 ? f_lo[wi] : 0.0f;
                        gh[u] = wi >= 0 ? f_hi[wi] : 0.0f;
                    }
                }
                float *fb = rows + (size_t)r * ROWF_PAD;
                if (flag == 1)
                    for (int qq = lane; qq < ROWF; qq += 32) fb[qq] = 0.0f;
                if (P.edge_add) {
                    const float4 *ea = reinterpret_cast<const float4 *>(P.edge_add + e * (int64_t)ROWF);
                    float4 *f4 = reinterpret_cast<float4 *>(fb);
                    for (int qq = lane; qq < ROWF / 4; qq += 32) {
                        const float4 a = __ldg(ea + qq);
                        float4 v = f4[qq];
                        v.x += a.x;
                        v.y += a.y;
                        v.z += a.z;
                        v.w += a.w;
                        f4[qq] = v;
                    }
                }
                __syncwarp();
                uint8_t *bh = b_base + st * kSplitN * kTileBytes;
                const int c = 2 * lane;
                const float *cp = tr + 2 * GE::LMAX + 1, *sp = cp + GE::LMAX + 1;
                uint8_t *rb = bh + el * ES * 128;
                if constexpr (kRotRec)
                    rotate_in_all_m<GE, 0, kSplit>(tr, sc[GE::J_S], sl, cp, sp, fb + c * DIN, fb + (c + 1) * DIN, rb,
                                                   rb + kTileBytes, xo);
                else
                    rotate_in_all<GE, 0, kSplit>(sc, cp, sp, fb + c * DIN, fb + (c + 1) * DIN, rb, rb + kTileBytes, xo);
                {
                    const float omt = 1.0f - t;
#pragma unroll
                    for (int u = 0; u < GI; u++) {
                        const int idx = lane + 32 * u;
                        if (idx < kRank * GE::GP) sl[GE::SLOT_G + idx] = omt * gl[u] + t * gh[u];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&r_free[r]);       // the row buffer may be refilled
            if (q % EPW == EPW - 1) {     // this warp's part of tile i is in shared memory
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[st]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int q4 = warp & 3;                       // TMEM lane quadrant of this warp
        const int row = q4 * 32 + lane;                // M row: co * kG + kk
        const int co = row / kG, kk = row % kG;
        const int wg = (warp - kEpiWarp0) / kNumEpi;   // this warp's epilogue warpgroup
        const int bar_id = 3 + wg;                     // named barrier of the warpgroup
        const bool leader = warp == kEpiWarp0 + kNumEpi * wg && lane == 0;
        float *my_stage = stage + wg * kG * GE::STAGE_ROW;
        // When the groups of a tile split evenly over the warpgroups, warpgroup wg takes groups
        // wg, wg + EWG, ... of every tile and all epilogue warps meet once per tile.  Otherwise
        // (three warpgroups, four groups per tile) the groups go round-robin over all tiles
        // (group i * GPT + gi to warpgroup (i * GPT + gi) mod EWG) and each warpgroup meets only
        // itself, so none waits for the others.  Either way every warp waits for every tile's
        // accumulators and releases them, so a release never precedes the tile's MMAs.
        constexpr int GPT = TE / kG;
        constexpr bool kRoundRobin = GPT % EWG != 0;
        const int stop_ix = kRoundRobin ? wg : 0;
        int rr = 0;
        for (int64_t i = 0; i < n_local; i++) {
            const int buf = (int)(i % kBufs), slot = (int)(i % GE::SLOTS);
            // The warps that meet at named barriers below must leave the loop together: a failed
            // wait in any of them stops all of them.
            if (!mbar_wait(&t_full[buf], (uint32_t)((i / kBufs) & 1), abort_flag, P.wait_ns) && lane == 0)
                epi_stop_s[stop_ix] = 1;
            if (kRoundRobin)
                named_bar(bar_id, kNumEpi * 32);
            else
                named_bar(2, EWG * kNumEpi * 32);
            if (*reinterpret_cast<volatile int *>(&epi_stop_s[stop_ix])) break;
            tc_fence_after();
            const int64_t e0 = (blockIdx.x + i * gridDim.x) * TE;
            const float *slot_base = slots + (size_t)slot * TE * GE::SLOT_EDGE;
            const uint32_t tbase = tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(buf * kSlices * 128);
#pragma unroll 1
            for (int gi = kRoundRobin ? 0 : wg; gi < GPT; gi += kRoundRobin ? 1 : EWG) {
                if (kRoundRobin) {
                    const bool mine = rr == wg;
                    rr = rr + 1 == EWG ? 0 : rr + 1;
                    if (!mine) continue;
                }
                // every lane of a pair computes its k's share of both edges of the group; the
                // pair sums its shares, and lane kk keeps edge gi * kG + kk
                float hf[DOUT];
#pragma unroll 1
                for (int ee = 0; ee < kG; ee++) {
                    const int el = gi * kG + ee;
                    const float *G = slot_base + el * GE::SLOT_EDGE + GE::SLOT_G;
                    float h[DOUT];
#pragma unroll
                    for (int q = 0; q < DOUT; q++) h[q] = 0.0f;
                    if constexpr (ES == 16) {          // both slices' rows in one round trip
                        uint32_t Z[kSlices][ES];
#pragma unroll
                        for (int s = 0; s < kSlices; s++) tmem_ld<ES>(tbase + (uint32_t)(s * 128 + el * ES), Z[s]);
                        tmem_wait_ld();
#pragma unroll
                        for (int s = 0; s < kSlices; s++) pos_mix<GE, 0, ES>(Z[s], G + (s * kG + kk) * GE::GP, h);
                    } else {
#pragma unroll 1
                        for (int s = 0; s < kSlices; s++) {
                            uint32_t Z[ES];
                            tmem_ld<ES>(tbase + (uint32_t)(s * 128 + el * ES), Z);
                            tmem_wait_ld();
                            pos_mix<GE, 0, ES>(Z, G + (s * kG + kk) * GE::GP, h);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < DOUT; q++) {
                        const float v = h[q] + __shfl_xor_sync(0xffffffffu, h[q], 1);
                        if (kk == ee) hf[q] = v;
                    }
                }
                const int el = gi * kG + kk;
                const float *es = slot_base + el * GE::SLOT_EDGE;
                float tr[GE::TF];
                load_regs<GE::TF>(es + GE::REC_TRIG, tr);
                const float *cp = tr + 2 * GE::LMAX + 1, *sp = cp + GE::LMAX + 1;
                if (leader) bulk_wait_read0();           // the previous group's rows have left
                named_bar(bar_id, kNumEpi * 32);
                rotate_out_all<GE, 0>(es, cp, sp, hf, my_stage + kk * GE::STAGE_ROW + co * DOUT);
                fence_async_smem();
                named_bar(bar_id, kNumEpi * 32);
                if (leader) {
#pragma unroll
                    for (int ee = 0; ee < kG; ee++) {
                        const int64_t e = e0 + gi * kG + ee;
                        if (e < P.E) bulk_store(P.out + e * (int64_t)OUTF, my_stage + ee * GE::STAGE_ROW, OUTF * 4);
                    }
                    bulk_commit();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&t_empty[buf]);
                mbar_arrive(&s_empty[slot]);
            }
        }
        if (leader) bulk_wait0();
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && abort_s) set_status(P.status, 2);
}

// Shared memory without the input-row ring, and the bytes of one ring entry (row + scalars).
template <int LIN, int LOUT, bool kSplit, int EWG>
size_t smem_fixed_bytes() {
    using GE = Geo<LIN, LOUT>;
    constexpr int kSplitN = kSplit ? 2 : 1;
    size_t b = 1024;                                                     // alignment slack
    b += (size_t)kSplitN * kSlices * kTileBytes;                         // M side
    b += (size_t)kStages * kSplitN * kTileBytes;                         // N side
    b += (size_t)GE::SLOTS * GE::TE * GE::SLOT_EDGE * 4;                 // per-tile slots
    b += (size_t)EWG * kG * GE::STAGE_ROW * 4;                           // output staging
    return b;
}
template <int LIN, int LOUT>
size_t ring_entry_bytes() {
    using GE = Geo<LIN, LOUT>;
    return ((size_t)((kCin * GE::DIN + 3) & ~3) + GE::JOB_FLOATS + GE::FR) * 4;
}

constexpr size_t kSmemPerBlock = 227 * 1024;     // dynamic + static shared memory of one CTA

template <int LIN, int LOUT, bool kSplit, int EWG, int NROT>
int launch(SepParams P, cudaStream_t stream) {
    auto kern = sep_edgewise_kernel<LIN, LOUT, kSplit, EWG, NROT>;
    constexpr int kThreads = threads_for(EWG, NROT);
    cudaFuncAttributes fa;
    FEQ_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
    const size_t cap = kSmemPerBlock - fa.sharedSizeBytes;
    const size_t fixed = smem_fixed_bytes<LIN, LOUT, kSplit, EWG>(), entry = ring_entry_bytes<LIN, LOUT>();
    // The ring size is a multiple of the tile's edge count: then job j and job j + nr are the
    // same edge slot of their tiles, so every ring buffer is only ever read by one rotation
    // warp, which takes its jobs in order.  Each wait on a buffer's "full" barrier is then for
    // the phase right after the one that warp last consumed, and a parity wait cannot match a
    // phase two ahead.  (With another size a warp could run two phases ahead of the loader on
    // a buffer another warp still owes, and its parity wait would pass early.)
    int nr = (int)((cap - fixed) / entry);
    nr = nr < kMaxRing ? nr : kMaxRing;
    nr -= nr % Geo<LIN, LOUT>::TE;
    if (nr < Geo<LIN, LOUT>::TE || fixed + (size_t)nr * entry > cap) return FEQ_ERR_UNSUPPORTED;
    P.nr = nr;
    size_t smem = fixed + (size_t)P.nr * entry;
    // more than half of the SM's shared memory: one CTA per SM, so one TMEM allocation
    if (smem < 120 * 1024) smem = 120 * 1024;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t grid = P.num_tiles < sms ? P.num_tiles : sms;
    kern<<<(unsigned)grid, kThreads, smem, stream>>>(P);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// (LIN, LOUT) pairs this build instantiates: lvals [0..L] in and out, L <= 4.
template <bool kSplit>
int dispatch(int lin, int lout, const SepParams &P, cudaStream_t s) {
    // as many warps as the registers allow: L <= 2 (80 registers) 8 rotation warps and three
    // epilogue warpgroups, L >= 3 (128) 4 and two
    if (lin == 1 && lout == 1) return launch<1, 1, kSplit, 3, 8>(P, s);
    if (lin == 2 && lout == 2) return launch<2, 2, kSplit, 3, 8>(P, s);
    if (lin == 3 && lout == 3) return launch<3, 3, kSplit, 2, 4>(P, s);
    if (lin == 4 && lout == 4) return launch<4, 4, kSplit, 2, 4>(P, s);
    return FEQ_ERR_UNSUPPORTED;
}

// lvals == [0, 1, ..., L]?  Returns L, or -1.
int contiguous_lmax(const int32_t *lv, int32_t n) {
    if (!lv || n < 1 || n > 5) return -1;
    for (int i = 0; i < n; i++)
        if (lv[i] != i) return -1;
    return n - 1;
}

}  // namespace sep
}  // namespace feq

using namespace feq;

extern "C" int feq_edgewise_separable_supported(const FeqSeparableArgs *a) {
    if (!a) return 0;
    const int lin = sep::contiguous_lmax(a->lvals_in, a->n_lvals_in);
    const int lout = sep::contiguous_lmax(a->lvals_out, a->n_lvals_out);
    if (lin < 1 || lin != lout) return 0;
    if (a->c_in != sep::kCin || a->c_out != sep::kCout || a->rank != sep::kRank) return 0;
    if (a->mix_mode != FEQ_MIX_BF16 && a->mix_mode != FEQ_MIX_BF16X3) return 0;
    if (!a->directions) return 0;
    return 1;
}

extern "C" int feq_edgewise_separable_fwd(const FeqSeparableArgs *a, feq_stream_t stream) {
    if (!a) return FEQ_ERR_INVALID_ARGUMENT;
    if (a->num_edges < 0 || a->num_bins < 1) return FEQ_ERR_INVALID_ARGUMENT;
    if (!feq_edgewise_separable_supported(a)) return FEQ_ERR_UNSUPPORTED;
    if (a->num_edges == 0) return FEQ_OK;
    if (!a->x || !a->distances || !a->channel_patterns || !a->radial_features || !a->out)
        return FEQ_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->out) |
         reinterpret_cast<uintptr_t>(a->edge_add) | reinterpret_cast<uintptr_t>(a->radial_features)) & 15)
        return FEQ_ERR_INVALID_ARGUMENT;      // bulk copies need 16-byte aligned rows
    const int L = a->n_lvals_in - 1;
    sep::SepParams P;
    P.x = a->x;
    P.src = a->src;
    P.nsrc = a->src ? a->num_src_rows : a->num_edges;
    P.edge_add = a->edge_add;
    P.dirs = a->directions;
    P.dist = a->distances;
    P.cpat = a->channel_patterns;
    P.ftab = a->radial_features;
    P.out = a->out;
    P.status = a->status;
    P.E = a->num_edges;
    P.bins.p1 = a->bin_param1;
    P.bins.p2 = a->bin_param2;
    P.bins.num_bins = a->num_bins;
    P.bins.log_bins = a->log_bins;
    P.sh_scale = a->sh_scale;
    P.wait_ns = wait_limit_ns();
    const int te = 128 / ((L + 1) * (L + 1) <= 16 ? 16 : 32);
    P.num_tiles = (a->num_edges + te - 1) / te;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    ProfScope prof("sep_edgewise", s);
    return a->mix_mode == FEQ_MIX_BF16X3 ? sep::dispatch<true>(L, L, P, s) : sep::dispatch<false>(L, L, P, s);
}
