// feq_nodelin.cu -- EquivariantLinear (flash_eq/layers/linear.py:172-268) on the tcgen05
// tensor cores: y[n, co, p] = sum_ci W[irrep(p)][co, ci] x[n, ci, p] (+ bias[co] at the l = 0
// position), for node-major rows x (N, C_in, d) and y (N, C_out, d).
//
// The reference forms weight @ f for every irrep at every position and gathers the matching
// one (linear.py:230-268).  Here each irrep's positions form their own GEMM, in one kernel
// that reads every node row once and writes every output row once:
//   - a tile is 16 nodes; its rows (node, position) are grouped by irrep, so irrep r owns
//     16 (2r + 1) consecutive rows -- a legal MMA N (a multiple of 16) for every degree;
//   - the weights, re-laid once per call into 128-byte-swizzled bf16 tiles (hi / lo) by
//     nodelin_wtiles_kernel, stay in shared memory for the whole kernel;
//   - converter warps (4, 8 or 16, a few nodes each) load their node rows with 16-byte loads
//     (the next tile's while the MMAs run) and write them as the K-major swizzled bf16 operand
//     (hi, and lo for bf16x3) into one of two operand stages;
//   - one thread issues tcgen05.mma kind::f16 per irrep (M = C_out rows of W_r, or 64),
//     into one of two TMEM accumulator sets; bf16x3 accumulates hi.hi + hi.lo + lo.hi;
//   - four epilogue warps (one per TMEM lane quadrant, lane = output channel) add the bias,
//     stage four nodes' rows of their 32 (or 16) channels and bulk-store them;
// so one tile's operand is written while the previous tile's MMAs run and the one before is
// stored.  Every wait is bounded; on time-out the kernel sets status 2, drains and leaves.
// No TMA multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "feq_internal.cuh"
#include "feq_rot_common.cuh"
#include "feq_sm100.cuh"

namespace feq {
namespace nlin {

using namespace sm100;
using namespace rot;

constexpr int TN = 16;            // nodes per tile

template <int L, int CIN, int COUT>
struct NG {
    static constexpr int D = (L + 1) * (L + 1);
    static constexpr int NR = L + 1;                            // irreps (lvals 0..L)
    static constexpr int ROWS = TN * D;                         // operand rows (node, position)
    static constexpr int KC = CIN / 64;                         // K chunks of 64 channels
    static constexpr int MROWS = COUT >= 128 ? 128 : 64;        // UMMA M
    static constexpr int MT = COUT / MROWS;                     // M tiles
    static constexpr uint32_t WTILE = MROWS * 128;              // one weight tile: MROWS x 64 bf16
    static constexpr uint32_t BCHUNK = ROWS * 128;              // one operand chunk: ROWS x 64 bf16
    static constexpr int TCOLS = MT * ROWS;                     // TMEM columns in use
    static constexpr uint32_t TALLOC = TCOLS <= 32 ? 32 : TCOLS <= 64 ? 64 : TCOLS <= 128 ? 128
                                     : TCOLS <= 256 ? 256 : 512;
    static constexpr int ROWF = CIN * D;                        // floats of one input row
    __host__ __device__ static constexpr int roff(int r) { return TN * r * r; }     // first row of irrep r
};

// Byte offset of (row, k) in a K-major tile of 64 bf16 per row, 128-byte swizzle.
__host__ __device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7))) << 4) + ((c & 7) << 1));
}

template <int L, int CIN, int COUT, bool kSplit>
constexpr uint32_t w_bytes() {
    using G = NG<L, CIN, COUT>;
    return (uint32_t)G::NR * G::KC * G::MT * (kSplit ? 2 : 1) * G::WTILE;
}

// Weights (NR, COUT, CIN) float32 -> swizzled bf16 tiles [r][kc][mt][hi, lo].
template <int L, int CIN, int COUT, bool kSplit>
__global__ void nodelin_wtiles_kernel(const float *__restrict__ w, uint8_t *__restrict__ wt) {
    using G = NG<L, CIN, COUT>;
    constexpr int SP = kSplit ? 2 : 1;
    const int total = G::NR * COUT * CIN;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = i / (COUT * CIN), rem = i - r * COUT * CIN;
        const int co = rem / CIN, ci = rem - co * CIN;
        const int mt = co / G::MROWS, row = co - mt * G::MROWS, kc = ci >> 6, k = ci & 63;
        uint8_t *base = wt + (size_t)(((r * G::KC + kc) * G::MT + mt) * SP) * G::WTILE;
        const float v = w[i];
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        *reinterpret_cast<__nv_bfloat16 *>(base + swz(row, k)) = hi;
        if (kSplit) *reinterpret_cast<__nv_bfloat16 *>(base + G::WTILE + swz(row, k)) = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
}

// Warp roles of the pipelined kernel: warp 0 issues the MMAs (and allocates TMEM), NCONV
// converter warps turn node rows into the operand (TN / NCONV nodes each), four epilogue
// warps (one per TMEM lane quadrant) turn accumulators into output rows.
template <int L, int CIN>
struct Roles {
    static constexpr int ROWF = CIN * (L + 1) * (L + 1);
    static constexpr int NCONV = ROWF <= 512 ? 4 : ROWF <= 576 ? 8 : 16;
    static constexpr int NPC = TN / NCONV;                       // nodes per converter warp
    static constexpr int VPL = NPC * ROWF / 4 / 32;              // float4s per lane per tile
    static constexpr bool XDB = NCONV == 4 && VPL <= 8;          // next tile's rows double-buffered (small rows)
    static constexpr int THREADS = (1 + NCONV + 4) * 32;
    static constexpr int CONV0 = 1, EPI0 = 1 + NCONV;
    static_assert(NPC * ROWF % 128 == 0, "a converter warp's rows split into float4s over 32 lanes");
};

__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

// 4 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

template <int L, int CIN, int COUT, bool kSplit>
constexpr uint32_t bufcols() {           // TMEM columns of one accumulator set, 256-aligned sets
    return (uint32_t)NG<L, CIN, COUT>::TCOLS <= 256 ? 256u : 512u;
}

template <int L, int CIN, int COUT, bool kSplit>
constexpr size_t smem_bytes_for(int bstages) {
    using G = NG<L, CIN, COUT>;
    constexpr int CW = G::MROWS == 128 ? 32 : 16;                 // output channels per epilogue warp
    return 1024 + (size_t)w_bytes<L, CIN, COUT, kSplit>() + (size_t)bstages * G::KC * (kSplit ? 2 : 1) * G::BCHUNK
         + (size_t)4 * 2 * 4 * CW * G::D * 4;
}
// operand stages: two where shared memory allows (the converters fill one while the MMAs read
// the other), else one
template <int L, int CIN, int COUT, bool kSplit>
constexpr int bstages() { return smem_bytes_for<L, CIN, COUT, kSplit>(2) <= 227 * 1024 ? 2 : 1; }
template <int L, int CIN, int COUT, bool kSplit>
constexpr size_t smem_bytes() { return smem_bytes_for<L, CIN, COUT, kSplit>(bstages<L, CIN, COUT, kSplit>()); }

// The kernel, pipelined: converter warps fill operand stage i % 2 for tile i while the MMA warp
// works on tile i - 1 and the epilogue warps drain the accumulators of tile i - 2 (two
// accumulator sets).  mbarriers: b_full (converters -> MMA), b_empty (MMA -> converters),
// t_full (MMA -> epilogue), t_empty (epilogue -> MMA).  No role waits at a barrier shared with
// another role, so a time-out in one lets the others time out in turn and leave.
template <int L, int CIN, int COUT, bool kSplit>
__global__ void __launch_bounds__(Roles<L, CIN>::THREADS, 1)
nodelin_kernel(const float *__restrict__ x, int64_t N, const uint8_t *__restrict__ wt, const float *__restrict__ bias,
               float *__restrict__ y, int64_t ntiles, int32_t *status, uint64_t wait_ns) {
    using G = NG<L, CIN, COUT>;
    using R = Roles<L, CIN>;
    constexpr int SP = kSplit ? 2 : 1;
    constexpr int D = G::D;
    constexpr uint32_t WB = w_bytes<L, CIN, COUT, kSplit>();
    constexpr uint32_t BSTAGE = G::KC * SP * G::BCHUNK;
    constexpr int BST = bstages<L, CIN, COUT, kSplit>();
    constexpr uint32_t BUFC = bufcols<L, CIN, COUT, kSplit>();
    constexpr uint32_t TALLOC = 2 * BUFC;
    constexpr int CW = G::MROWS == 128 ? 32 : 16;
    constexpr int GROUP = 4;                                   // nodes per epilogue store group
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *wsm = smem;                                       // weight tiles [r][kc][mt][s]
    uint8_t *bsm = wsm + WB;                                   // BST operand stages [kc][s]
    float *stg = reinterpret_cast<float *>(bsm + BST * BSTAGE);  // per epilogue warp 2 x GROUP x CW x D

    __shared__ uint64_t w_bar, b_full[2], b_empty[2], t_full[2], t_empty[2], drain_bar;
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&w_bar, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&b_full[i], R::NCONV);
            mbar_init(&b_empty[i], 1);
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], 4);
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_s, TALLOC);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    volatile int *abort_flag = &abort_s;
    const int64_t n_local = ntiles > blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (warp == 0) {
        // ---------------- weights in, MMA issuer ----------------
        if (lane == 0) {
            mbar_arrive_expect_tx(&w_bar, WB);
            for (uint32_t o = 0; o < WB; o += G::WTILE) bulk_load(wsm + o, wt + o, G::WTILE, &w_bar);
            bool ok = mbar_wait(&w_bar, 0, abort_flag, wait_ns);
            for (int64_t i = 0; ok && i < n_local; i++) {
                const int s = (int)(i & 1), sb = (int)(i % BST);
                if (!mbar_wait(&b_full[sb], (uint32_t)((i / BST) & 1), abort_flag, wait_ns)) break;
                if (i >= 2 && !mbar_wait(&t_empty[s], (uint32_t)(((i >> 1) - 1) & 1), abort_flag, wait_ns)) break;
                tc_fence_after();
                const uint8_t *bst = bsm + (size_t)sb * BSTAGE;
#pragma unroll
                for (int r = 0; r < G::NR; r++) {
                    const uint32_t idesc = idesc_bf16_f32(G::MROWS, TN * (2 * r + 1));
#pragma unroll
                    for (int mt = 0; mt < G::MT; mt++) {
                        const uint32_t d = tmem + (uint32_t)s * BUFC + (uint32_t)(mt * G::ROWS + G::roff(r));
#pragma unroll
                        for (int kc = 0; kc < G::KC; kc++) {
                            const uint32_t ah = smem_u32(wsm + (size_t)(((r * G::KC + kc) * G::MT + mt) * SP) * G::WTILE);
                            const uint32_t bh = smem_u32(bst + (size_t)(kc * SP) * G::BCHUNK) + (uint32_t)G::roff(r) * 128u;
#pragma unroll
                            for (int ks = 0; ks < 4; ks++) {
                                const uint32_t ko = ks * 32;
                                umma_f16(d, smem_desc_sw128(ah + ko), smem_desc_sw128(bh + ko), idesc, (kc | ks) ? 1u : 0u);
                                if (kSplit) {
                                    umma_f16(d, smem_desc_sw128(ah + ko), smem_desc_sw128(bh + G::BCHUNK + ko), idesc, 1u);
                                    umma_f16(d, smem_desc_sw128(ah + G::WTILE + ko), smem_desc_sw128(bh + ko), idesc, 1u);
                                }
                            }
                        }
                    }
                }
                umma_commit(&b_empty[sb]);             // the operand stage may be refilled
                umma_commit(&t_full[s]);               // the accumulators are ready
            }
            // everything in flight lands before TMEM and shared memory are released
            mbar_wait_drain(&w_bar, 0);
            umma_commit(&drain_bar);
            mbar_wait_drain(&drain_bar, 0);
        }
    } else if (warp < R::EPI0) {
        // ---------------- converters: node rows -> operand ----------------
        const int cw = warp - R::CONV0;
        const int nb = cw * R::NPC;                            // first node of this warp in a tile
        if constexpr (CIN >= 128) {
            // 128 input channels: lane l takes channels 4 l .. 4 l + 3 of each of the warp's
            // nodes, whose 4 D floats are contiguous in the node row (16-byte loads); the lane
            // then holds every position of two channel pairs, so each (pair, position) is one
            // packed bf16x2 store per operand half with compile-time row arithmetic, instead of
            // a per-element decode and 2-byte stores (1 M nodes 128 -> 64: 2.53 -> 2.03 ms).
            constexpr int CPL = CIN / 32;                          // channels per lane
            constexpr int FPN = CPL * D;                           // floats per lane per node
            constexpr int VF = R::NPC * FPN;                       // floats per lane per tile
            static_assert(VF == 4 * R::VPL, "the same floats per lane as the float4 view");
            auto load = [&](int64_t i, float (&v)[VF]) {
                const int64_t n0 = (blockIdx.x + i * gridDim.x) * (int64_t)TN + nb;
#pragma unroll
                for (int nl = 0; nl < R::NPC; nl++) {
                    const bool in = i < n_local && n0 + nl < N;
                    const float *src = x + (n0 + nl) * R::ROWF + lane * FPN;
                    if constexpr (FPN % 4 == 0) {
#pragma unroll
                        for (int u = 0; u < FPN / 4; u++) {
                            const float4 t = in ? __ldg(reinterpret_cast<const float4 *>(src) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
                            v[nl * FPN + 4 * u] = t.x;
                            v[nl * FPN + 4 * u + 1] = t.y;
                            v[nl * FPN + 4 * u + 2] = t.z;
                            v[nl * FPN + 4 * u + 3] = t.w;
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < FPN / 2; u++) {
                            const float2 t = in ? __ldg(reinterpret_cast<const float2 *>(src) + u) : make_float2(0.f, 0.f);
                            v[nl * FPN + 2 * u] = t.x;
                            v[nl * FPN + 2 * u + 1] = t.y;
                        }
                    }
                }
            };
            auto convert = [&](int64_t i, const float (&v)[VF]) -> bool {
                const int sb = (int)(i % BST);
                if (i >= BST && !mbar_wait(&b_empty[sb], (uint32_t)((i / BST - 1) & 1), abort_flag, wait_ns)) return false;
                uint8_t *bst = bsm + (size_t)sb * BSTAGE;
#pragma unroll
                for (int nl = 0; nl < R::NPC; nl++) {
#pragma unroll
                    for (int p = 0; p < D; p++) {
                        const int r = p >= 9 ? 3 : p >= 4 ? 2 : p >= 1 ? 1 : 0;
                        const int row = G::roff(r) + (nb + nl) * (2 * r + 1) + (p - r * r);
#pragma unroll
                        for (int j = 0; j < CPL / 2; j++) {
                            const int c = lane * CPL + 2 * j;
                            const float y0 = v[nl * FPN + (2 * j) * D + p], y1 = v[nl * FPN + (2 * j + 1) * D + p];
                            uint8_t *chunk = bst + (size_t)((c >> 6) * SP) * G::BCHUNK;
                            const uint32_t o = swz(row, c & 63);
                            const __nv_bfloat162 hi = __floats2bfloat162_rn(y0, y1);
                            *reinterpret_cast<__nv_bfloat162 *>(chunk + o) = hi;
                            if (kSplit) {
                                const float2 hf = __bfloat1622float2(hi);
                                *reinterpret_cast<__nv_bfloat162 *>(chunk + G::BCHUNK + o) =
                                    __floats2bfloat162_rn(y0 - hf.x, y1 - hf.y);
                            }
                        }
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[sb]);
                return true;
            };
            if constexpr (R::XDB) {
                float va[VF], vb[VF];
                load(0, va);
                for (int64_t i = 0; i < n_local; i += 2) {
                    load(i + 1, vb);                           // in flight while tile i is converted
                    if (!convert(i, va)) break;
                    if (i + 1 >= n_local) break;
                    load(i + 2, va);
                    if (!convert(i + 1, vb)) break;
                }
            } else {
                // the next tile's rows are loaded right after this tile's operand is handed over, so
                // they are in flight while the MMAs run
                float va[VF];
                load(0, va);
                for (int64_t i = 0; i < n_local; i++) {
                    if (!convert(i, va)) break;
                    load(i + 1, va);
                }
            }
        } else {
            // 64 input channels: float4 loads along the node row (coalesced); each element is
            // placed on its own (the lane's four floats are consecutive positions).  The
            // channel-pair mapping above measured slower here (8-byte loads at a 72-byte lane
            // stride): 1 M nodes 64 -> 128 1.46 -> 1.59 ms.
            auto load = [&](int64_t i, float4 (&v)[R::VPL]) {
                const int64_t n0 = (blockIdx.x + i * gridDim.x) * (int64_t)TN + nb;
                const int64_t lim = (N - n0) * (int64_t)R::ROWF;   // valid floats from n0 on
                const float4 *src = reinterpret_cast<const float4 *>(x + n0 * R::ROWF);
#pragma unroll
                for (int k = 0; k < R::VPL; k++) {
                    const int j = lane + 32 * k;
                    v[k] = (i < n_local && 4 * j < lim) ? __ldg(src + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            };
            auto convert = [&](int64_t i, const float4 (&v)[R::VPL]) -> bool {
                const int sb = (int)(i % BST);
                if (i >= BST && !mbar_wait(&b_empty[sb], (uint32_t)((i / BST - 1) & 1), abort_flag, wait_ns)) return false;
                uint8_t *bst = bsm + (size_t)sb * BSTAGE;
#pragma unroll
                for (int k = 0; k < R::VPL; k++) {
                    const float vv[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const int e = 4 * (lane + 32 * k) + q;
                        const int nl = e / R::ROWF, rem = e - nl * R::ROWF;
                        const int c = rem / D, p = rem - c * D;
                        const float val = vv[q];
                        const int r = p >= 9 ? 3 : p >= 4 ? 2 : p >= 1 ? 1 : 0;
                        const int row = G::roff(r) + (nb + nl) * (2 * r + 1) + (p - r * r);
                        uint8_t *chunk = bst + (size_t)((c >> 6) * SP) * G::BCHUNK;
                        const uint32_t o = swz(row, c & 63);
                        const __nv_bfloat16 hi = __float2bfloat16_rn(val);
                        *reinterpret_cast<__nv_bfloat16 *>(chunk + o) = hi;
                        if (kSplit)
                            *reinterpret_cast<__nv_bfloat16 *>(chunk + G::BCHUNK + o) =
                                __float2bfloat16_rn(val - __bfloat162float(hi));
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[sb]);
                return true;
            };
            if constexpr (R::XDB) {
                float4 va[R::VPL], vb[R::VPL];
                load(0, va);
                for (int64_t i = 0; i < n_local; i += 2) {
                    load(i + 1, vb);                           // in flight while tile i is converted
                    if (!convert(i, va)) break;
                    if (i + 1 >= n_local) break;
                    load(i + 2, va);
                    if (!convert(i + 1, vb)) break;
                }
            } else {
                // the next tile's rows are loaded right after this tile's operand is handed over, so
                // they are in flight while the MMAs run
                float4 va[R::VPL];
                load(0, va);
                for (int64_t i = 0; i < n_local; i++) {
                    if (!convert(i, va)) break;
                    load(i + 1, va);
                }
            }
        }
    } else {
        // ---------------- epilogue: accumulators -> output rows ----------------
        const int q4 = warp & 3;
        const bool live = G::MROWS == 128 || lane < 16;
        const int co_l = G::MROWS == 128 ? q4 * 32 + lane : q4 * 16 + lane;
        const int co0 = q4 * CW;                               // first channel of this warp
        float *wst = stg + (size_t)(warp - R::EPI0) * 2 * GROUP * CW * D;
        uint32_t groups = 0;
        for (int64_t i = 0; i < n_local; i++) {
            const int s = (int)(i & 1);
            if (!mbar_wait(&t_full[s], (uint32_t)((i >> 1) & 1), abort_flag, wait_ns)) break;
            tc_fence_after();
            const int64_t n0 = (blockIdx.x + i * gridDim.x) * (int64_t)TN;
#pragma unroll
            for (int mt = 0; mt < G::MT; mt++) {
                const int co = mt * G::MROWS + co_l;
                const float b0 = (bias && live) ? bias[co] : 0.0f;
#pragma unroll 1
                for (int g = 0; g < TN / GROUP; g++, groups++) {
                    float *sb = wst + (size_t)(groups & 1) * GROUP * CW * D;
                    if (groups >= 2) {                    // the store from two groups back has read sb
                        if (lane == 0) bulk_wait_read1();
                        __syncwarp();
                    }
#pragma unroll
                    for (int r = 0; r < G::NR; r++) {
                        const int w = 2 * r + 1;
                        uint32_t v[4 * 7];                     // 4 nodes x (2r + 1) columns, r <= 3
                        const uint32_t col = (uint32_t)s * BUFC + (uint32_t)(mt * G::ROWS + G::roff(r) + g * GROUP * w);
#pragma unroll
                        for (int piece = 0; piece < 7; piece++)
                            if (piece < w) tmem_ld4(tmem + ((uint32_t)(q4 * 32) << 16) + col + piece * 4, v + piece * 4);
                        tmem_wait_ld();
                        if (live) {
#pragma unroll
                            for (int jj = 0; jj < 4 * 7; jj++) {
                                if (jj < GROUP * w) {
                                    const int nl = jj / w, p = r * r + jj % w;
                                    float val = __uint_as_float(v[jj]);
                                    if (r == 0) val += b0;
                                    sb[((size_t)nl * CW + (co - mt * G::MROWS - co0)) * D + p] = val;
                                }
                            }
                        }
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
#pragma unroll
                        for (int nl = 0; nl < GROUP; nl++) {
                            const int64_t node = n0 + g * GROUP + nl;
                            if (node < N)
                                bulk_store(y + (node * COUT + mt * G::MROWS + co0) * (int64_t)D, sb + (size_t)nl * CW * D,
                                           (uint32_t)CW * D * 4);
                        }
                        bulk_commit();
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_empty[s]);
        }
        if (lane == 0) bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TALLOC);
    }
    if (threadIdx.x == 0 && abort_s) set_status(status, 2);
}

template <int L, int CIN, int COUT, bool kSplit>
int run(const float *x, int64_t N, const float *w, const float *bias, float *y, void *ws, size_t ws_bytes,
        int32_t *status, cudaStream_t s) {
    constexpr size_t smem = smem_bytes<L, CIN, COUT, kSplit>();
    static_assert(smem <= 227 * 1024, "shared memory of one CTA");
    if (ws_bytes < w_bytes<L, CIN, COUT, kSplit>() || !ws) return FEQ_ERR_WORKSPACE;
    uint8_t *wt = static_cast<uint8_t *>(ws);
    const int total = NG<L, CIN, COUT>::NR * COUT * CIN;
    nodelin_wtiles_kernel<L, CIN, COUT, kSplit><<<(total + 255) / 256, 256, 0, s>>>(w, wt);
    FEQ_LAUNCH_CHECK();
    auto kern = nodelin_kernel<L, CIN, COUT, kSplit>;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t ntiles = (N + TN - 1) / TN;
    const int64_t grid = ntiles < sms ? ntiles : sms;
    kern<<<(unsigned)grid, Roles<L, CIN>::THREADS, smem, s>>>(x, N, wt, bias, y, ntiles, status, wait_limit_ns());
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

// lvals == [0, 1, ..., L]?  Returns L, or -1.
int contiguous_lmax(const int32_t *lv, int32_t n) {
    if (!lv || n < 1 || n > 4) return -1;
    for (int i = 0; i < n; i++)
        if (lv[i] != i) return -1;
    return n - 1;
}

template <bool kSplit>
size_t wbytes_for(int L, int cin, int cout) {
#define FEQ_NL_CASE(LL, CI, CO) \
    if (L == LL && cin == CI && cout == CO) return w_bytes<LL, CI, CO, kSplit>();
    FEQ_NL_CASE(1, 64, 64) FEQ_NL_CASE(1, 64, 128) FEQ_NL_CASE(1, 128, 64)
    FEQ_NL_CASE(2, 64, 64) FEQ_NL_CASE(2, 64, 128) FEQ_NL_CASE(2, 128, 64)
#undef FEQ_NL_CASE
    return 0;
}

template <bool kSplit>
int dispatch(int L, int cin, int cout, const float *x, int64_t N, const float *w, const float *bias, float *y,
             void *ws, size_t wsb, int32_t *status, cudaStream_t s) {
#define FEQ_NL_CASE(LL, CI, CO) \
    if (L == LL && cin == CI && cout == CO) return run<LL, CI, CO, kSplit>(x, N, w, bias, y, ws, wsb, status, s);
    FEQ_NL_CASE(1, 64, 64) FEQ_NL_CASE(1, 64, 128) FEQ_NL_CASE(1, 128, 64)
    FEQ_NL_CASE(2, 64, 64) FEQ_NL_CASE(2, 64, 128) FEQ_NL_CASE(2, 128, 64)
#undef FEQ_NL_CASE
    return FEQ_ERR_UNSUPPORTED;
}

}  // namespace nlin
}  // namespace feq

using namespace feq;

extern "C" size_t feq_node_linear_tc_workspace_bytes(int32_t c_in, int32_t c_out, const int32_t *lvals,
                                                     int32_t n_lvals, int32_t mix_mode) {
    const int L = nlin::contiguous_lmax(lvals, n_lvals);
    if (L < 0) return 0;
    if (mix_mode == FEQ_MIX_BF16X3) return nlin::wbytes_for<true>(L, c_in, c_out);
    if (mix_mode == FEQ_MIX_BF16) return nlin::wbytes_for<false>(L, c_in, c_out);
    return 0;
}

extern "C" int feq_node_linear_tc(const float *x, int64_t num_nodes, int32_t c_in, int32_t c_out,
                                  const int32_t *lvals, int32_t n_lvals, const float *weight, const float *bias,
                                  int32_t mix_mode, float *y, void *workspace, size_t workspace_bytes,
                                  int32_t *status, feq_stream_t stream) {
    if (num_nodes < 0) return FEQ_ERR_INVALID_ARGUMENT;
    const size_t need = feq_node_linear_tc_workspace_bytes(c_in, c_out, lvals, n_lvals, mix_mode);
    if (need == 0) return FEQ_ERR_UNSUPPORTED;
    if (num_nodes == 0) return FEQ_OK;
    if (!x || !weight || !y) return FEQ_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(workspace)) & 15)
        return FEQ_ERR_INVALID_ARGUMENT;     // 16-byte loads, bulk copies
    const int L = n_lvals - 1;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    ProfScope prof("node_linear", s);
    return mix_mode == FEQ_MIX_BF16X3
               ? nlin::dispatch<true>(L, c_in, c_out, x, num_nodes, weight, bias, y, workspace, workspace_bytes, status, s)
               : nlin::dispatch<false>(L, c_in, c_out, x, num_nodes, weight, bias, y, workspace, workspace_bytes, status, s);
}
