// feq_internal.cuh -- shared host/device definitions of libflasheq_b200.
//
// Layout structs are built once on the host from the lvals lists and passed to
// kernels by value (__grid_constant__), so no launch needs a host->device copy
// or a device->host sync.  The reference instead rebuilds its block table on
// the CPU and copies it to the GPU on every call
// (flash_eq/cuda/csrc/block_diagonal.cu:1191-1266, :1296).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "flasheq_b200.h"

namespace feq {

constexpr int kMaxL = FEQ_MAX_L;
constexpr int kMaxIrreps = FEQ_MAX_IRREPS;
constexpr int kMaxDim = FEQ_MAX_DIM;
constexpr int kMaxBlocks = FEQ_MAX_L + 1;

// ---------------------------------------------------------------------------
// One representation (a list of irreps with degrees lvals), both orders.
// std order: irreps in list order, each m = -l..l  (types.py:178-305)
// m-first order: wigner.py:243-272
// ---------------------------------------------------------------------------
struct ReprLayout {
    int n_irreps;
    int dim;
    int lmax;
    int n_unique;                    // distinct l values
    int dblock_floats;               // sum over distinct l of (2l+1)^2
    int8_t irrep_l[kMaxIrreps];
    int16_t irrep_off[kMaxIrreps];   // std offset of irrep r
    int8_t irrep_slot[kMaxIrreps];   // index into unique_l of irrep r's degree
    int8_t unique_l[kMaxL + 1];
    int16_t unique_doff[kMaxL + 1];  // float offset of that degree's (2l+1)^2 block
    int16_t perm[kMaxDim];           // m-first position -> std position
    int16_t inv_perm[kMaxDim];       // std position -> m-first position
    int8_t std_irrep[kMaxDim];       // std position -> irrep
};

// One m-block of the block-diagonal weight (block_diagonal.cu:143-157).
struct MixBlock {
    int m, n_in, n_out, in_off, out_off, w_off;
    int relaid_off;                  // float offset of the block inside one re-laid bin row
    int relaid_stride;               // floats per (ci, i) row: c_out * n_out * mult, rounded up to even
    int8_t l_in[kMaxIrreps];         // degree of the i-th input member
    int8_t l_out[kMaxIrreps];        // degree of the o-th output member
};

struct MixLayout {
    int n_blocks;                    // mmax + 1
    int wdim;                        // ProductRepr.nreps()
    int lmax_in, lmax_out;
    int64_t relaid_row;              // floats per bin in the re-laid table (multiple of 4)
    MixBlock blk[kMaxBlocks];
};

// Tensor-core path: where component j (m-first order) of channel c lives in a GEMM
// row (A for the input repr, H for the output repr): base[j] + c * stride[j] (stride 1:
// the channel is the fastest column index), or
// base[j] = -1 when j belongs to a block that does not take part in the mix; l[j] is
// the degree of j (solid-harmonic scaling).
struct TcPosMap {
    int32_t base[kMaxDim];
    int32_t base_std[kMaxDim];       // base of the component at standard position k
    int16_t stride[kMaxDim];
    int8_t l[kMaxDim];
    int n_pad;                       // zero-padding column ranges of the A row
    int pad_lo[kMaxBlocks], pad_hi[kMaxBlocks];
};

// Tensor-core radial mix: per m-block GEMM geometry.  B (the re-laid table) holds, per
// block, (num_bins + 1) matrices of npad x kpad bf16 (K-major) starting at element boff.
struct TcBlockGeom {
    int mult, n_in, n_out, w_off, kpad, npad;
    int64_t boff;
};
struct TcGeom {
    int n_blocks;                    // non-empty blocks (a prefix of m = 0..mmax)
    TcBlockGeom g[kMaxBlocks];
};

struct Binning {
    float p1, p2;
    int num_bins;
    int log_bins;
};

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// compute_binning (block_diagonal.cu:82-115): bin index in float32, bit-exact;
// t in float32, unclamped in linear mode, clamped to <= 1 in log mode.
__device__ __forceinline__ void bin_of(float d, const Binning &b, int &lo, float &t) {
    float normalized;
    if (b.log_bins) {
        normalized = (logf(fmaxf(d, expf(b.p1))) - b.p1) * b.p2 * b.num_bins;
    } else {
        normalized = (d - b.p1) * b.p2;
    }
    normalized = fminf(fmaxf(normalized, 0.0f), (float)b.num_bins);
    lo = min((int)floorf(normalized), b.num_bins - 1);
    if (b.log_bins) {
        float inv_lbw = b.p2 * b.num_bins;
        float log_edge_lo = b.p1 + (float)lo / inv_lbw;
        float edge_lo = (float)exp((double)log_edge_lo);
        float edge_hi = (float)exp((double)(log_edge_lo + 1.0f / inv_lbw));
        float cd = d > edge_lo ? d : edge_lo;
        t = (cd - edge_lo) / (edge_hi - edge_lo);
        t = t < 1.0f ? t : 1.0f;
    } else {
        float bw = 1.0f / b.p2;
        float edge_lo = b.p1 + (float)lo * bw;
        t = (d - edge_lo) / bw;
    }
}

// (r / (r + scale))^l by squaring, as block_diagonal.cu:202-232.
__device__ __forceinline__ float ipowf(float base, int e) {
    float r = 1.0f;
    while (e > 0) {
        if (e & 1) r *= base;
        base *= base;
        e >>= 1;
    }
    return r;
}

__device__ __forceinline__ void set_status(int32_t *status, int32_t code) {
    if (status) atomicMax(status, code);
}

// ---------------------------------------------------------------------------
// Host helpers (defined in feq_abi.cu)
// ---------------------------------------------------------------------------
int build_repr_layout(const int32_t *lvals, int32_t n, ReprLayout *out);
int build_mix_layout(const int32_t *lin, int32_t nin, const int32_t *lout, int32_t nout,
                     int c_in, int c_out, MixLayout *out);
void record_cuda_error(cudaError_t err);
// Limit of every pipeline wait in the tensor-core kernels, in ns (feq_set_wait_limit_ns).
uint64_t wait_limit_ns();
void record_error_text(const char *msg);
void count_launches(int n);

// Stage timing: while profiling is enabled, ProfScope records an event pair around
// the work enqueued during its lifetime on stream s.
void prof_begin(const char *name, cudaStream_t s);
void prof_end(cudaStream_t s);
struct ProfScope {
    cudaStream_t s;
    ProfScope(const char *name, cudaStream_t st) : s(st) { prof_begin(name, s); }
    ~ProfScope() { prof_end(s); }
};

// Workspace carving: every region 256-byte aligned.
// Per-block float offsets of the backward's per-bin reduction buffer.
struct DbOff {
    int64_t off[kMaxBlocks];
};

// One m-block of the backward's tensor-core per-bin reduction.
struct TcGramBlock {
    int N, K, n_tiles, k_tiles, g_row0, a_row0;
    int64_t dboff, item0;
};

struct WsCarver {
    char *base;
    size_t used, cap;
    __host__ void *take(size_t bytes) {
        size_t off = (used + 255) & ~size_t(255);
        used = off + bytes;
        return base ? (void *)(base + off) : nullptr;
    }
};

}  // namespace feq

#define FEQ_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) {                             \
            ::feq::record_cuda_error(_e);                    \
            return FEQ_ERR_CUDA;                             \
        }                                                    \
    } while (0)

#define FEQ_LAUNCH_CHECK()                                   \
    do {                                                     \
        ::feq::count_launches(1);                            \
        cudaError_t _e = cudaGetLastError();                 \
        if (_e != cudaSuccess) {                             \
            ::feq::record_cuda_error(_e);                    \
            return FEQ_ERR_CUDA;                             \
        }                                                    \
    } while (0)
