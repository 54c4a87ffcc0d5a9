// feq_nodelin.cu -- EquivariantLinear (flash_eq/layers/linear.py:172-268) on the tcgen05
// tensor cores: y[n, co, p] = sum_ci W[irrep(p)][co, ci] x[n, ci, p] (+ bias[co] at the l = 0
// position), for node-major rows x (N, C_in, d) and y (N, C_out, d).
//
// The reference forms weight @ f for every irrep at every position and gathers the matching
// one (linear.py:230-268).  Here each irrep's positions form their own GEMM, in one kernel
// that reads every node row once and writes every output row once:
//   - a tile is 16 nodes; its rows (node, position) are grouped by irrep, so irrep r owns
//     16 (2r + 1) consecutive rows -- a legal MMA N (a multiple of 16) for every degree;
//   - the node rows are loaded with 16-byte loads (the next tile's while this one is in the
//     MMAs and the epilogue) and written by the CUDA cores as the K-major, 128-byte-swizzled
//     bf16 operand (hi, and lo for bf16x3);
//   - the weights, re-laid once per call into the same swizzled tiles (hi / lo) by
//     nodelin_wtiles_kernel, stay in shared memory for the whole kernel;
//   - one thread issues tcgen05.mma kind::f16 per irrep (M = C_out rows of W_r, or 64),
//     accumulating in TMEM; bf16x3 accumulates hi.hi + hi.lo + lo.hi;
//   - the epilogue reads TMEM (lane = output channel), adds the bias, stages the tile's output
//     rows in shared memory and writes them with one bulk store (16 node rows are contiguous).
// Every wait is bounded; on time-out the kernel sets status 2 and every thread leaves.  No
// TMA multicast.
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
constexpr int kThreads = 256;     // 8 warps: two per TMEM lane quadrant in the epilogue

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
    static constexpr int VPT = TN * ROWF / 4 / kThreads;        // float4 loads per thread per tile
    static_assert((TN * ROWF) % (4 * kThreads) == 0, "tile loads split evenly over the threads");
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

template <int L, int CIN, int COUT, bool kSplit>
constexpr size_t smem_bytes() {
    using G = NG<L, CIN, COUT>;
    return 1024 + (size_t)w_bytes<L, CIN, COUT, kSplit>() + (size_t)G::KC * (kSplit ? 2 : 1) * G::BCHUNK
         + (size_t)TN * COUT * G::D * 4;
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

// 8 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

template <int L, int CIN, int COUT, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
nodelin_kernel(const float *__restrict__ x, int64_t N, const uint8_t *__restrict__ wt, const float *__restrict__ bias,
               float *__restrict__ y, int64_t ntiles, int32_t *status, uint64_t wait_ns) {
    using G = NG<L, CIN, COUT>;
    constexpr int SP = kSplit ? 2 : 1;
    constexpr int D = G::D;
    constexpr uint32_t WB = w_bytes<L, CIN, COUT, kSplit>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *wsm = smem;                                        // weight tiles [r][kc][mt][s]
    uint8_t *bsm = wsm + WB;                                    // operand chunks [kc][s]
    float *stg = reinterpret_cast<float *>(bsm + G::KC * SP * G::BCHUNK);   // TN x COUT x D output rows

    __shared__ uint64_t w_bar, mma_bar, drain_bar;
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        mbar_init(&w_bar, 1);
        mbar_init(&mma_bar, 1);
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_s, G::TALLOC);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    volatile int *abort_flag = &abort_s;
    if (tid == 0) {
        mbar_arrive_expect_tx(&w_bar, WB);
        for (uint32_t o = 0; o < WB; o += G::WTILE) bulk_load(wsm + o, wt + o, G::WTILE, &w_bar);
    }

    // this thread's share of a tile: VPT float4s at element 4 (tid + v kThreads)
    float4 xv[G::VPT];
    auto load_tile = [&](int64_t t) {
        const int64_t n0 = t * TN;
        const int64_t lim = (N - n0) * G::ROWF;                 // valid floats of the tile
        const float4 *src = reinterpret_cast<const float4 *>(x + n0 * G::ROWF);
#pragma unroll
        for (int v = 0; v < G::VPT; v++) {
            const int e = 4 * (tid + v * kThreads);
            xv[v] = (t < ntiles && e < lim) ? __ldg(src + tid + v * kThreads) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto put = [&](int e, float val) {
        const int n = e / G::ROWF, rem = e - n * G::ROWF;
        const int c = rem / D, p = rem - c * D;
        const int r = p >= 9 ? 3 : p >= 4 ? 2 : p >= 1 ? 1 : 0;
        const int row = G::roff(r) + n * (2 * r + 1) + (p - r * r);
        uint8_t *chunk = bsm + (size_t)((c >> 6) * SP) * G::BCHUNK;
        const uint32_t o = swz(row, c & 63);
        const __nv_bfloat16 hi = __float2bfloat16_rn(val);
        *reinterpret_cast<__nv_bfloat16 *>(chunk + o) = hi;
        if (kSplit) *reinterpret_cast<__nv_bfloat16 *>(chunk + G::BCHUNK + o) = __float2bfloat16_rn(val - __bfloat162float(hi));
    };

    int64_t t = blockIdx.x;
    load_tile(t);
    uint32_t phase = 0;
    bool stored = false;
    if (!mbar_wait(&w_bar, 0, abort_flag, wait_ns)) set_status(status, 2);
    __syncthreads();
    for (; t < ntiles && !*abort_flag; t += gridDim.x) {
        const int64_t n0 = t * TN;
        const int nv = (int)((N - n0) < TN ? (N - n0) : TN);
        // (1) rows -> K-major bf16 operand
#pragma unroll
        for (int v = 0; v < G::VPT; v++) {
            const int e = 4 * (tid + v * kThreads);
            put(e, xv[v].x);
            put(e + 1, xv[v].y);
            put(e + 2, xv[v].z);
            put(e + 3, xv[v].w);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        // (2) one MMA group per irrep and M tile
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int r = 0; r < G::NR; r++) {
                const uint32_t idesc = idesc_bf16_f32(G::MROWS, TN * (2 * r + 1));
#pragma unroll
                for (int mt = 0; mt < G::MT; mt++) {
                    const uint32_t d = tmem + (uint32_t)(mt * G::ROWS + G::roff(r));
#pragma unroll
                    for (int kc = 0; kc < G::KC; kc++) {
                        const uint32_t ah = smem_u32(wsm + (size_t)(((r * G::KC + kc) * G::MT + mt) * SP) * G::WTILE);
                        const uint32_t bh = smem_u32(bsm + (size_t)(kc * SP) * G::BCHUNK) + (uint32_t)G::roff(r) * 128u;
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
            umma_commit(&mma_bar);
        }
        // the next tile's rows are in flight during the MMAs and the epilogue
        load_tile(t + gridDim.x);
        if (!mbar_wait(&mma_bar, phase, abort_flag, wait_ns)) set_status(status, 2);
        phase ^= 1;
        if (tid == 0 && stored) bulk_wait_read0();          // the previous tile's rows have left
        __syncthreads();
        if (*abort_flag) break;
        tc_fence_after();
        // (3) epilogue: warp w reads lane quadrant w % 4 for nodes [8 (w / 4), 8 (w / 4) + 8)
        {
            const int q4 = warp & 3, hn = warp >> 2;
            const bool live = G::MROWS == 128 || lane < 16;
            const int co_l = G::MROWS == 128 ? q4 * 32 + lane : q4 * 16 + lane;   // M row of this lane
#pragma unroll
            for (int mt = 0; mt < G::MT; mt++) {
                const int co = mt * G::MROWS + co_l;
                const float b0 = (bias && live) ? bias[co] : 0.0f;
#pragma unroll
                for (int r = 0; r < G::NR; r++) {
                    const int w = 2 * r + 1;
#pragma unroll
                    for (int piece = 0; piece < w; piece++) {        // 8 columns a piece
                        uint32_t v[8];
                        const uint32_t col = (uint32_t)(mt * G::ROWS + G::roff(r) + hn * 8 * w + piece * 8);
                        tmem_ld8(tmem + ((uint32_t)(q4 * 32) << 16) + col, v);
                        tmem_wait_ld();
                        if (live) {
#pragma unroll
                            for (int j = 0; j < 8; j++) {
                                const int jj = piece * 8 + j;                 // column within the 8 w of this half
                                const int n = hn * 8 + jj / w, p = r * r + jj % w;
                                float val = __uint_as_float(v[j]);
                                if (r == 0) val += b0;
                                stg[((size_t)n * COUT + co) * D + p] = val;
                            }
                        }
                    }
                }
            }
        }
        tc_fence_before();
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            bulk_store(y + n0 * (int64_t)COUT * D, stg, (uint32_t)nv * COUT * D * 4);
            bulk_commit();
            stored = true;
        }
    }
    if (tid == 0) {
        // before TMEM and shared memory are released, everything in flight lands, also after a
        // wait ran out: the weight copies, every MMA issued (this thread issued them all) and the
        // last output rows
        mbar_wait_drain(&w_bar, 0);
        umma_commit(&drain_bar);
        mbar_wait_drain(&drain_bar, 0);
        bulk_wait0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, G::TALLOC);
    }
}

template <int L, int CIN, int COUT, bool kSplit>
int run(const float *x, int64_t N, const float *w, const float *bias, float *y, void *ws, size_t ws_bytes,
        int32_t *status, cudaStream_t s) {
    constexpr size_t smem = smem_bytes<L, CIN, COUT, kSplit>();
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
    kern<<<(unsigned)grid, kThreads, smem, s>>>(x, N, wt, bias, y, ntiles, status, wait_limit_ns());
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
