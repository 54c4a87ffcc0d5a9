// feq_dense.cu -- a dense linear Y = X W^T + b on the tcgen05 tensor cores (bf16x3 or bf16),
// for the plain nn.Linear of EquivariantGating (flash_eq/layers/gating.py:17-76 of the
// reference: the (C * n_irreps)^2 mix of the irrep norms before the sigmoid gate).
//
// X (N, K) and Y (N, M) float32 row-major, W (M, K) float32 (nn.Linear's weight), b (M,).
// M a multiple of 128 up to 512, K a multiple of 64 up to 512.  A tile is 64 rows of X.
// Warp-specialised, persistent (one CTA per SM), every role on its own mbarriers:
//   warp 0      W producer: W is re-laid once per call into swizzled bf16 tiles of 128 x 64
//               (hi / lo) by dense_wtiles_kernel and streamed from L2, tile pair after tile
//               pair in the MMA's order, through a shared-memory ring (bulk copies)
//   warp 1      one thread issues tcgen05.mma kind::f16 (M = 128 rows of W, N = 64 rows of X,
//               K = 16), bf16x3 accumulating hi.hi + hi.lo + lo.hi, K chunk by K chunk (all
//               M tiles of a chunk before the next chunk), into one of two TMEM accumulator
//               sets
//   warps 2..5  converters: each takes 16 rows of every 64-column K chunk of X (16-byte
//               loads, the next two chunks' in flight while this one is converted) and writes the
//               K-major, 128-byte-swizzled bf16 operand (hi, and lo for bf16x3) into a ring of
//               chunk slots, so the conversion of a tile overlaps the MMAs of the one before
//   warps 6..9  epilogue: tcgen05.ld (lane = output feature), + b, coalesced stores (a warp
//               writes 32 consecutive features of a row), overlapping the next tile's MMAs
// Every wait is bounded; on time-out the kernel sets status 2, drains and leaves.  No TMA
// multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "feq_internal.cuh"
#include "feq_rot_common.cuh"
#include "feq_sm100.cuh"

namespace feq {
namespace dense {

using namespace sm100;
using namespace rot;

constexpr int TR = 64;                    // rows of X per tile (UMMA N)
constexpr int kConvWarps = 4, kEpiWarps = 4;
constexpr int kThreads = (2 + kConvWarps + kEpiWarps) * 32;   // producer, MMA, converters, epilogue
constexpr int kMaxStages = 12;            // W tile-pair ring
constexpr int kMaxXSlots = 8;             // X chunk ring
constexpr uint32_t kWTile = 128 * 128;    // 128 rows x 64 bf16
constexpr uint32_t kXChunk = TR * 128;    // 64 rows x 64 bf16
constexpr int kMaxM = 512, kMaxK = 512;

__host__ __device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7))) << 4) + ((c & 7) << 1));
}

// W (M, K) -> tiles [mt][kc][hi, lo] of 128 x 64 swizzled bf16.
template <bool kSplit>
__global__ void dense_wtiles_kernel(const float *__restrict__ w, int M, int K, uint8_t *__restrict__ wt) {
    constexpr int SP = kSplit ? 2 : 1;
    const int KC = K / 64;
    const int total = M * K;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int j = i / K, k = i - j * K;
        const int mt = j >> 7, row = j & 127, kc = k >> 6, kk = k & 63;
        uint8_t *base = wt + (size_t)((mt * KC + kc) * SP) * kWTile;
        const float v = w[i];
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        *reinterpret_cast<__nv_bfloat16 *>(base + swz(row, kk)) = hi;
        if (kSplit) *reinterpret_cast<__nv_bfloat16 *>(base + kWTile + swz(row, kk)) = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
}


template <bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
dense_kernel(const float *__restrict__ x, int64_t N, int M, int K, const uint8_t *__restrict__ wt,
             const float *__restrict__ bias, float *__restrict__ y, int64_t ntiles, int stages, int xslots,
             int32_t *status, uint64_t wait_ns) {
    constexpr int SP = kSplit ? 2 : 1;
    const int MT = M >> 7, KC = K >> 6;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *wring = smem;                                    // stages x SP x kWTile
    uint8_t *xring = wring + (size_t)stages * SP * kWTile;   // xslots x SP x kXChunk

    __shared__ uint64_t w_full[kMaxStages], w_empty[kMaxStages], x_full[kMaxXSlots], x_empty[kMaxXSlots];
    __shared__ uint64_t t_full[2], t_empty[2], drain_bar;
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], 1);
        }
        for (int s = 0; s < xslots; s++) {
            mbar_init(&x_full[s], kConvWarps);
            mbar_init(&x_empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&t_full[b], 1);
            mbar_init(&t_empty[b], kEpiWarps);
        }
        mbar_init(&drain_bar, 1);
        abort_s = 0;
        fence_mbar_init();
    }
    const uint32_t tcols = (uint32_t)(2 * MT * TR) <= 256 ? 256u : 512u;
    if (warp == 0) {
        tmem_alloc(&tmem_s, tcols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    volatile int *abort_flag = &abort_s;
    const int64_t n_local = ntiles > blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (warp == 0) {
        // ---------------- W producer: pairs in the MMA's order (chunk kc, then tile mt) ----------------
        if (lane == 0) {
            uint32_t u = 0;
            for (int64_t i = 0; i < n_local && !*abort_flag; i++) {
                bool ok = true;
                for (int kc = 0; kc < KC && ok; kc++)
                    for (int mt = 0; mt < MT; mt++, u++) {
                        const int s = (int)(u % stages);
                        if (u >= (uint32_t)stages &&
                            !mbar_wait(&w_empty[s], ((u / stages) - 1) & 1u, abort_flag, wait_ns)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&w_full[s], SP * kWTile);
                        bulk_load(wring + (size_t)s * SP * kWTile, wt + (size_t)(mt * KC + kc) * SP * kWTile,
                                  SP * kWTile, &w_full[s]);
                    }
                if (!ok) break;
            }
            // every copy issued has landed before the CTA leaves
            const uint32_t last = u;
            for (uint32_t v = last > (uint32_t)stages ? last - stages : 0; v < last; v++)
                mbar_wait_drain(&w_full[v % stages], (v / stages) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, TR);
            uint32_t u = 0, c = 0;
            bool ok = true;
            for (int64_t i = 0; i < n_local && ok && !*abort_flag; i++) {
                const int buf = (int)(i & 1);
                if (i >= 2 && !mbar_wait(&t_empty[buf], (uint32_t)(((i >> 1) - 1) & 1), abort_flag, wait_ns)) break;
                for (int kc = 0; kc < KC && ok; kc++, c++) {
                    const int xs = (int)(c % xslots);
                    if (!mbar_wait(&x_full[xs], (c / xslots) & 1u, abort_flag, wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bh = smem_u32(xring + (size_t)xs * SP * kXChunk);
                    for (int mt = 0; mt < MT; mt++, u++) {
                        const int s = (int)(u % stages);
                        if (!mbar_wait(&w_full[s], (u / stages) & 1u, abort_flag, wait_ns)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tmem + (uint32_t)(buf * MT * TR + mt * TR);
                        const uint32_t ah = smem_u32(wring + (size_t)s * SP * kWTile);
#pragma unroll
                        for (int ks = 0; ks < 4; ks++) {
                            const uint32_t ko = ks * 32;
                            umma_f16(d, smem_desc_sw128(ah + ko), smem_desc_sw128(bh + ko), idesc, (kc | ks) ? 1u : 0u);
                            if (kSplit) {
                                umma_f16(d, smem_desc_sw128(ah + ko), smem_desc_sw128(bh + kXChunk + ko), idesc, 1u);
                                umma_f16(d, smem_desc_sw128(ah + kWTile + ko), smem_desc_sw128(bh + ko), idesc, 1u);
                            }
                        }
                        umma_commit(&w_empty[s]);
                    }
                    if (ok) umma_commit(&x_empty[xs]);        // the chunk slot may be rewritten
                }
                if (ok) umma_commit(&t_full[buf]);
            }
            umma_commit(&drain_bar);
            mbar_wait_drain(&drain_bar, 0);
        }
    } else if (warp < 2 + kConvWarps) {
        // ---------------- converters: 16 rows of every chunk per warp ----------------
        const int cw = warp - 2;
        const int64_t n_chunks = n_local * KC;
        // float4 f = lane + 32 u of this warp's 16 x 64 block: row cw * 16 + f / 16, column 4 (f % 16)
        auto load = [&](int64_t c, float4 (&v)[8]) {
            const int64_t i = c / KC;
            const int kc = (int)(c - i * KC);
            const int64_t r0 = (blockIdx.x + i * gridDim.x) * TR + cw * 16;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int f = lane + 32 * u;
                const int64_t r = r0 + (f >> 4);
                v[u] = r < N ? __ldg(reinterpret_cast<const float4 *>(x + r * (int64_t)K + kc * 64) + (f & 15))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        auto store = [&](int64_t c, const float4 (&v)[8]) -> bool {
            const int xs = (int)(c % xslots);
            if (c >= xslots && !mbar_wait(&x_empty[xs], (uint32_t)(((c / xslots) - 1) & 1), abort_flag, wait_ns))
                return false;
            uint8_t *hi = xring + (size_t)xs * SP * kXChunk;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int f = lane + 32 * u;
                const int row = cw * 16 + (f >> 4), col = (f & 15) * 4;
                const uint32_t o = swz(row, col);         // 4 bf16 in one 16-byte chunk: one 8-byte store
                const __nv_bfloat162 h01 = __floats2bfloat162_rn(v[u].x, v[u].y);
                const __nv_bfloat162 h23 = __floats2bfloat162_rn(v[u].z, v[u].w);
                uint2 hv;
                hv.x = *reinterpret_cast<const uint32_t *>(&h01);
                hv.y = *reinterpret_cast<const uint32_t *>(&h23);
                *reinterpret_cast<uint2 *>(hi + o) = hv;
                if (kSplit) {
                    const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
                    const __nv_bfloat162 l01 = __floats2bfloat162_rn(v[u].x - f01.x, v[u].y - f01.y);
                    const __nv_bfloat162 l23 = __floats2bfloat162_rn(v[u].z - f23.x, v[u].w - f23.y);
                    uint2 lv;
                    lv.x = *reinterpret_cast<const uint32_t *>(&l01);
                    lv.y = *reinterpret_cast<const uint32_t *>(&l23);
                    *reinterpret_cast<uint2 *>(hi + kXChunk + o) = lv;
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&x_full[xs]);
            return true;
        };
        // three register buffers: while chunk c is converted, chunks c + 1 and c + 2 are in
        // flight (48 KB of X per SM with the four converter warps)
        float4 va[8], vb[8], vc[8];
        if (n_chunks > 0) load(0, va);
        if (n_chunks > 1) load(1, vb);
        for (int64_t c = 0; c < n_chunks; c += 3) {
            if (c + 2 < n_chunks) load(c + 2, vc);
            if (!store(c, va) || c + 1 >= n_chunks) break;
            if (c + 3 < n_chunks) load(c + 3, va);
            if (!store(c + 1, vb) || c + 2 >= n_chunks) break;
            if (c + 4 < n_chunks) load(c + 4, vb);
            if (!store(c + 2, vc)) break;
        }
    } else {
        // ---------------- epilogue ----------------
        const int q4 = warp & 3;                              // TMEM lane quadrant
        for (int64_t i = 0; i < n_local; i++) {
            const int buf = (int)(i & 1);
            if (!mbar_wait(&t_full[buf], (uint32_t)((i >> 1) & 1), abort_flag, wait_ns)) break;
            tc_fence_after();
            const int64_t r0 = (blockIdx.x + i * gridDim.x) * TR;
            for (int mt = 0; mt < MT; mt++) {
                const int j = mt * 128 + q4 * 32 + lane;
                const float bj = bias ? bias[j] : 0.0f;
#pragma unroll 1
                for (int c0 = 0; c0 < TR; c0 += 16) {
                    uint32_t v[16];
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                          "=r"(v[14]), "=r"(v[15])
                        : "r"(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(buf * MT * TR + mt * TR + c0)));
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 16; c++) {
                        const int64_t r = r0 + c0 + c;
                        if (r < N) y[r * (int64_t)M + j] = __uint_as_float(v[c]) + bj;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_empty[buf]);
        }
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, tcols);
    }
    if (threadIdx.x == 0 && abort_s) set_status(status, 2);
}

size_t wbytes(int M, int K, bool split) { return (size_t)M * K * 2 * (split ? 2 : 1); }

template <bool kSplit>
int run(const float *x, int64_t N, int M, int K, const float *w, const float *b, float *y, void *ws, size_t wsb,
        int32_t *status, cudaStream_t s) {
    if (!ws || wsb < wbytes(M, K, kSplit)) return FEQ_ERR_WORKSPACE;
    uint8_t *wt = static_cast<uint8_t *>(ws);
    dense_wtiles_kernel<kSplit><<<(M * K + 255) / 256, 256, 0, s>>>(w, M, K, wt);
    FEQ_LAUNCH_CHECK();
    // shared memory: W ring (tile pairs) + X chunk ring, bf16x3 5 + 3 (208 KB), bf16 10 + 6
    // (208 KB).  At a million rows the split does not matter (4 + 6, 6 + 2, 2 + 6 all within
    // 1 %); at a few thousand rows, one tile per CTA, the deeper W ring shortens the chain.
    const size_t xchunk = (size_t)(kSplit ? 2 : 1) * kXChunk, wpair = (size_t)(kSplit ? 2 : 1) * kWTile;
    const int stages = kSplit ? 5 : 10, xslots = kSplit ? 3 : 6;
    const size_t smem = 1024 + (size_t)stages * wpair + (size_t)xslots * xchunk;
    auto kern = dense_kernel<kSplit>;
    FEQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, sms = 148;
    FEQ_CUDA_TRY(cudaGetDevice(&dev));
    FEQ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t ntiles = (N + TR - 1) / TR;
    const int64_t grid = ntiles < sms ? ntiles : sms;
    kern<<<(unsigned)grid, kThreads, smem, s>>>(x, N, M, K, wt, b, y, ntiles, stages, xslots, status, wait_limit_ns());
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // namespace dense
}  // namespace feq

using namespace feq;

extern "C" size_t feq_dense_linear_tc_workspace_bytes(int32_t m, int32_t k, int32_t mix_mode) {
    if (m < 128 || m > dense::kMaxM || m % 128 || k < 64 || k > dense::kMaxK || k % 64) return 0;
    if (mix_mode != FEQ_MIX_BF16X3 && mix_mode != FEQ_MIX_BF16) return 0;
    return dense::wbytes(m, k, mix_mode == FEQ_MIX_BF16X3);
}

extern "C" int feq_dense_linear_tc(const float *x, int64_t n, int32_t m, int32_t k, const float *weight,
                                   const float *bias, int32_t mix_mode, float *y, void *workspace,
                                   size_t workspace_bytes, int32_t *status, feq_stream_t stream) {
    if (n < 0) return FEQ_ERR_INVALID_ARGUMENT;
    if (feq_dense_linear_tc_workspace_bytes(m, k, mix_mode) == 0) return FEQ_ERR_UNSUPPORTED;
    if (n == 0) return FEQ_OK;
    if (!x || !weight || !y) return FEQ_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(workspace)) & 15) return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    ProfScope prof("dense_linear", s);
    return mix_mode == FEQ_MIX_BF16X3
               ? dense::run<true>(x, n, m, k, weight, bias, y, workspace, workspace_bytes, status, s)
               : dense::run<false>(x, n, m, k, weight, bias, y, workspace, workspace_bytes, status, s);
}
