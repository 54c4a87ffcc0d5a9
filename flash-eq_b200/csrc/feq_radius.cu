// feq_radius.cu -- radius graph construction on the GPU (cell lists): every ordered pair
// (i, j), i != j (or i == j too with `loop`), of points of the same batch entry with
// |x_j - x_i| < r.  No counterpart in the reference, which leaves graph building to the user
// (README.md:49-52); the reference's benchmark configuration "all pairs within 5 A" is such a
// graph.
//
// Points are binned into cubic cells of side h >= r keyed by (batch, cell x, cell y, cell z)
// and sorted by key (CUB radix sort), so the points of one graph in one cell are contiguous
// and points of different graphs never meet.  Every neighbour within r lies in one of the 27
// cells around a point's own.  Two passes over those cells: count, then (after an exclusive
// scan gives each point its output range) write the pairs; a final radix sort of the
// (i << 32 | j) keys puts the edges in (src, dst) order, the order of torch.nonzero on the
// dense (N, N) mask.  The squared distance is formed with separately rounded multiplies and
// adds (no FMA contraction) so the cut-off test is the same float32 arithmetic as a CPU
// evaluation of (dx*dx + dy*dy) + dz*dz: the edge set is bit-exact against brute force.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "feq_internal.cuh"

namespace feq {
namespace {

constexpr int kCellBits = 14;                       // per axis
constexpr int kCellMax = (1 << kCellBits) - 1;
constexpr int64_t kBatchMax = (int64_t)1 << (64 - 1 - 3 * kCellBits);   // 2^21 graphs

struct RadiusGrid {
    float x0, y0, z0, inv_h, r2;
    int64_t n;
    int loop;
};

__device__ __forceinline__ int64_t rkey(int64_t b, int cx, int cy, int cz) {
    return (b << (3 * kCellBits)) | ((int64_t)cx << (2 * kCellBits)) | ((int64_t)cy << kCellBits) | (int64_t)cz;
}

__device__ __forceinline__ float dist2_rn(float ax, float ay, float az, float bx, float by, float bz) {
    const float dx = __fsub_rn(bx, ax), dy = __fsub_rn(by, ay), dz = __fsub_rn(bz, az);
    return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
}

__device__ __forceinline__ void rcell(const RadiusGrid &g, float x, float y, float z, int &cx, int &cy, int &cz) {
    cx = (int)floorf((x - g.x0) * g.inv_h);
    cy = (int)floorf((y - g.y0) * g.inv_h);
    cz = (int)floorf((z - g.z0) * g.inv_h);
}

__global__ void radius_keys_kernel(const float *__restrict__ xyz, const int64_t *__restrict__ batch, RadiusGrid g,
                                   int64_t *__restrict__ keys, int64_t *__restrict__ ids, int32_t *status) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < g.n; i += (int64_t)gridDim.x * blockDim.x) {
        int cx, cy, cz;
        rcell(g, xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], cx, cy, cz);
        const int64_t b = batch ? batch[i] : 0;
        if (cx < 0 || cy < 0 || cz < 0 || cx > kCellMax || cy > kCellMax || cz > kCellMax || b < 0 ||
            b >= kBatchMax || !isfinite(xyz[3 * i]) || !isfinite(xyz[3 * i + 1]) || !isfinite(xyz[3 * i + 2])) {
            set_status(status, 1);
            cx = cy = cz = 0;
        }
        keys[i] = rkey(b < 0 ? 0 : (b >= kBatchMax ? kBatchMax - 1 : b), cx, cy, cz);
        ids[i] = i;
    }
}

__device__ __forceinline__ int64_t first_at(const int64_t *__restrict__ sk, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (sk[mid] < key) lo = mid + 1;
        else hi = mid;
    }
    return (lo < n && sk[lo] == key) ? lo : -1;
}

// kFill = false: counts[i] = number of neighbours of i.  kFill = true: write (i << 32 | j)
// for every neighbour j of i at out[offsets[i] ...] (cell order; sorted afterwards).
template <bool kFill>
__global__ void radius_scan_kernel(const float *__restrict__ xyz, const int64_t *__restrict__ batch, RadiusGrid g,
                                   const int64_t *__restrict__ sk, const int64_t *__restrict__ sid,
                                   int64_t *__restrict__ counts, const int64_t *__restrict__ offsets,
                                   uint64_t *__restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < g.n; i += (int64_t)gridDim.x * blockDim.x) {
        const float qx = xyz[3 * i], qy = xyz[3 * i + 1], qz = xyz[3 * i + 2];
        int cx, cy, cz;
        rcell(g, qx, qy, qz, cx, cy, cz);
        int64_t b = batch ? batch[i] : 0;
        b = b < 0 ? 0 : (b >= kBatchMax ? kBatchMax - 1 : b);     // (flagged by the keys kernel)
        int64_t c = 0, w = kFill ? offsets[i] : 0;
        for (int dx = -1; dx <= 1; dx++)
            for (int dy = -1; dy <= 1; dy++)
                for (int dz = -1; dz <= 1; dz++) {
                    const int x = cx + dx, y = cy + dy, z = cz + dz;
                    if (x < 0 || y < 0 || z < 0 || x > kCellMax || y > kCellMax || z > kCellMax) continue;
                    const int64_t key = rkey(b, x, y, z);
                    int64_t p = first_at(sk, g.n, key);
                    if (p < 0) continue;
                    for (; p < g.n && sk[p] == key; p++) {
                        const int64_t j = sid[p];
                        if (j == i && !g.loop) continue;
                        if (dist2_rn(qx, qy, qz, xyz[3 * j], xyz[3 * j + 1], xyz[3 * j + 2]) < g.r2) {
                            if (kFill) out[w++] = ((uint64_t)i << 32) | (uint64_t)j;
                            else c++;
                        }
                    }
                }
        if (!kFill) counts[i] = c;
    }
}

__global__ void radius_split_kernel(const uint64_t *__restrict__ pairs, int64_t E, int64_t *__restrict__ src,
                                    int64_t *__restrict__ dst) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E; e += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t v = pairs[e];
        src[e] = (int64_t)(v >> 32);
        dst[e] = (int64_t)(v & 0xffffffffull);
    }
}

struct RadiusWs {
    int64_t *keys, *ids, *sk, *sid, *counts;
    void *tmp;
    size_t tmp_bytes;
};

size_t radius_tmp_bytes(int64_t n) {
    size_t a = 0, b = 0;
    const int m = (int)std::max<int64_t>(n, 1);
    cub::DeviceRadixSort::SortPairs(nullptr, a, (const int64_t *)nullptr, (int64_t *)nullptr,
                                    (const int64_t *)nullptr, (int64_t *)nullptr, m);
    cub::DeviceScan::ExclusiveSum(nullptr, b, (const int64_t *)nullptr, (int64_t *)nullptr, m + 1);
    return std::max(a, b);
}

bool carve_radius(void *ws, size_t bytes, int64_t n, RadiusWs &R) {
    WsCarver w{(char *)ws, 0, bytes};
    const int64_t m = std::max<int64_t>(n, 1);
    R.keys = (int64_t *)w.take(sizeof(int64_t) * m);
    R.ids = (int64_t *)w.take(sizeof(int64_t) * m);
    R.sk = (int64_t *)w.take(sizeof(int64_t) * m);
    R.sid = (int64_t *)w.take(sizeof(int64_t) * m);
    R.counts = (int64_t *)w.take(sizeof(int64_t) * (m + 1));
    R.tmp_bytes = radius_tmp_bytes(n);
    R.tmp = w.take(R.tmp_bytes);
    return w.used <= bytes;
}

}  // namespace
}  // namespace feq

using namespace feq;

extern "C" {

size_t feq_radius_workspace_bytes(int64_t num_points) {
    WsCarver w{nullptr, 0, 0};
    const int64_t m = std::max<int64_t>(num_points, 1);
    for (int i = 0; i < 4; i++) w.take(sizeof(int64_t) * m);
    w.take(sizeof(int64_t) * (m + 1));
    w.take(radius_tmp_bytes(num_points));
    return w.used + 256;
}

size_t feq_radius_pairs_workspace_bytes(int64_t num_edges) {
    size_t tmp = 0;
    cub::DeviceRadixSort::SortKeys(nullptr, tmp, (const uint64_t *)nullptr, (uint64_t *)nullptr,
                                   (int)std::max<int64_t>(num_edges, 1));
    return 2 * sizeof(uint64_t) * (size_t)std::max<int64_t>(num_edges, 1) + tmp + 1024;
}

int feq_radius_count(const float *xyz, const int64_t *batch, int64_t num_points, float r, int32_t loop, float cell,
                     float x0, float y0, float z0, int64_t *offsets, int32_t *status, void *workspace,
                     size_t workspace_bytes, feq_stream_t stream) {
    if (num_points < 0 || !(r > 0.0f) || !(cell >= r)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_points > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    if (!offsets) return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (num_points == 0) {
        FEQ_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int64_t), s));
        return FEQ_OK;
    }
    if (!xyz || !workspace) return FEQ_ERR_INVALID_ARGUMENT;
    RadiusWs R;
    if (workspace_bytes < feq_radius_workspace_bytes(num_points) || !carve_radius(workspace, workspace_bytes,
                                                                                   num_points, R))
        return FEQ_ERR_WORKSPACE;
    const int64_t n = num_points;
    RadiusGrid g{x0, y0, z0, 1.0f / cell, r * r, n, loop ? 1 : 0};
    const int grid = (int)min64((n + 255) / 256, 148 * 16);
    radius_keys_kernel<<<grid, 256, 0, s>>>(xyz, batch, g, R.keys, R.ids, status);
    FEQ_LAUNCH_CHECK();
    size_t tb = R.tmp_bytes;
    FEQ_CUDA_TRY(cub::DeviceRadixSort::SortPairs(R.tmp, tb, R.keys, R.sk, R.ids, R.sid, (int)n, 0, 63, s));
    count_launches(3);
    const int qgrid = (int)min64((n + 127) / 128, 148 * 32);
    radius_scan_kernel<false><<<qgrid, 128, 0, s>>>(xyz, batch, g, R.sk, R.sid, R.counts, nullptr, nullptr);
    FEQ_LAUNCH_CHECK();
    FEQ_CUDA_TRY(cudaMemsetAsync(R.counts + n, 0, sizeof(int64_t), s));
    tb = R.tmp_bytes;
    FEQ_CUDA_TRY(cub::DeviceScan::ExclusiveSum(R.tmp, tb, R.counts, offsets, (int)n + 1, s));
    count_launches(1);
    return FEQ_OK;
}

int feq_radius_fill(const float *xyz, const int64_t *batch, int64_t num_points, float r, int32_t loop, float cell,
                    float x0, float y0, float z0, const int64_t *offsets, int64_t num_edges, int64_t *src,
                    int64_t *dst, const void *workspace, size_t workspace_bytes, void *pair_workspace,
                    size_t pair_workspace_bytes, feq_stream_t stream) {
    if (num_points < 0 || num_edges < 0 || !(r > 0.0f) || !(cell >= r)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges == 0) return FEQ_OK;
    if (!xyz || !offsets || !src || !dst || !workspace || !pair_workspace) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_edges > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    RadiusWs R;
    if (workspace_bytes < feq_radius_workspace_bytes(num_points) ||
        !carve_radius(const_cast<void *>(workspace), workspace_bytes, num_points, R))
        return FEQ_ERR_WORKSPACE;
    if (pair_workspace_bytes < feq_radius_pairs_workspace_bytes(num_edges)) return FEQ_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t n = num_points, E = num_edges;
    WsCarver w{(char *)pair_workspace, 0, pair_workspace_bytes};
    uint64_t *pairs = (uint64_t *)w.take(sizeof(uint64_t) * E), *sorted = (uint64_t *)w.take(sizeof(uint64_t) * E);
    size_t tmp = 0;
    FEQ_CUDA_TRY(cub::DeviceRadixSort::SortKeys(nullptr, tmp, pairs, sorted, (int)E));
    void *tmpp = w.take(tmp);
    if (w.used > pair_workspace_bytes) return FEQ_ERR_WORKSPACE;
    RadiusGrid g{x0, y0, z0, 1.0f / cell, r * r, n, loop ? 1 : 0};
    const int qgrid = (int)min64((n + 127) / 128, 148 * 32);
    radius_scan_kernel<true><<<qgrid, 128, 0, s>>>(xyz, batch, g, R.sk, R.sid, nullptr, offsets, pairs);
    FEQ_LAUNCH_CHECK();
    int end_bit = 32;
    while (end_bit < 64 && ((int64_t)1 << (end_bit - 32)) < n) end_bit++;
    FEQ_CUDA_TRY(cub::DeviceRadixSort::SortKeys(tmpp, tmp, pairs, sorted, (int)E, 0, end_bit, s));
    count_launches(3);
    const int egrid = (int)min64((E + 255) / 256, 148 * 16);
    radius_split_kernel<<<egrid, 256, 0, s>>>(sorted, E, src, dst);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // extern "C"
