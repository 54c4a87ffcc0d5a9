// feq_knn.cu -- k-nearest-neighbour graph construction on the GPU (cell lists).
//
// No counterpart in the reference, which leaves graph construction to the user (its
// README builds graphs with torch.cdist + topk, O(N^2)).  Here points are binned into
// cubic cells of side h, the cells are sorted by a 64-bit key (CUB radix sort), and one
// thread per query point scans the cells in growing cubic shells around its own cell,
// keeping the k best (distance, index) pairs in registers.  A cell at Chebyshev cell
// distance s + 1 from the query's cell only holds points farther than s * h from the
// query, so after the shells 0..s the scan stops as soon as k candidates are known and the
// k-th best distance is <= s * h: the result is exact whatever h is (h only sets the cost).
//
// Output: for every query q the indices of its k nearest other points, ordered by
// distance (ties by index), in nbr[q * k + j]; -1 where fewer than k points exist.
#include <cub/device/device_radix_sort.cuh>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "feq_internal.cuh"

namespace feq {
namespace {

constexpr int kKnnMax = 64;
constexpr int kKnnMaxShell = 16;     // the scan also stops here (cell far too small): status 1

struct KnnGrid {
    float x0, y0, z0, inv_h, h;
    int64_t n;
};

__device__ __forceinline__ int64_t cell_key(int cx, int cy, int cz) {
    // 21 bits per axis, offset so that negative cells order correctly
    return ((int64_t)(cx + (1 << 20)) << 42) | ((int64_t)(cy + (1 << 20)) << 21) | (int64_t)(cz + (1 << 20));
}

__device__ __forceinline__ void cell_of(const KnnGrid &g, float x, float y, float z, int &cx, int &cy, int &cz) {
    cx = (int)floorf((x - g.x0) * g.inv_h);
    cy = (int)floorf((y - g.y0) * g.inv_h);
    cz = (int)floorf((z - g.z0) * g.inv_h);
}

__global__ void knn_keys_kernel(const float *__restrict__ xyz, KnnGrid g, int64_t *__restrict__ keys,
                                int64_t *__restrict__ ids) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < g.n; i += (int64_t)gridDim.x * blockDim.x) {
        int cx, cy, cz;
        cell_of(g, xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], cx, cy, cz);
        keys[i] = cell_key(cx, cy, cz);
        ids[i] = i;
    }
}

// first sorted position of the cell with key `key`, or -1 (binary search over sorted keys)
__device__ __forceinline__ int64_t cell_start(const int64_t *__restrict__ sk, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (sk[mid] < key) lo = mid + 1;
        else hi = mid;
    }
    return (lo < n && sk[lo] == key) ? lo : -1;
}

// keep the K best (distance, index) pairs, sorted ascending: the new pair is carried
// through the array, swapping with every larger entry (the largest falls off the end)
template <int K>
__device__ __forceinline__ void insert(float (&bd)[K], int32_t (&bi)[K], float d, int32_t j) {
    if (!(d < bd[K - 1] || (d == bd[K - 1] && j < bi[K - 1]))) return;
#pragma unroll
    for (int q = 0; q < K; q++) {
        if (d < bd[q] || (d == bd[q] && j < bi[q])) {
            const float td = bd[q];
            const int32_t tj = bi[q];
            bd[q] = d;
            bi[q] = j;
            d = td;
            j = tj;
        }
    }
}

template <int K>
__global__ void knn_query_kernel(const float *__restrict__ xyz, KnnGrid g, const int64_t *__restrict__ sk,
                                 const int64_t *__restrict__ sid, int k, int64_t *__restrict__ nbr,
                                 int32_t *status) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < g.n; q += (int64_t)gridDim.x * blockDim.x) {
        const float qx = xyz[3 * q], qy = xyz[3 * q + 1], qz = xyz[3 * q + 2];
        int cx, cy, cz;
        cell_of(g, qx, qy, qz, cx, cy, cz);
        float bd[K];
        int32_t bi[K];
#pragma unroll
        for (int j = 0; j < K; j++) {
            bd[j] = INFINITY;
            bi[j] = INT32_MAX;
        }
        int found = 0;
        bool done = false;
        for (int s = 0; s <= kKnnMaxShell && !done; s++) {
            // cells at Chebyshev distance exactly s from the query's cell
            for (int dx = -s; dx <= s; dx++)
                for (int dy = -s; dy <= s; dy++) {
                    const bool face = dx == -s || dx == s || dy == -s || dy == s;
                    const int step = face ? 1 : 2 * s;     // interior columns: only the two z faces
                    for (int dz = -s; dz <= s; dz += step) {
                        int64_t p = cell_start(sk, g.n, cell_key(cx + dx, cy + dy, cz + dz));
                        if (p < 0) continue;
                        const int64_t key = sk[p];
                        for (; p < g.n && sk[p] == key; p++) {
                            const int64_t j = sid[p];
                            if (j == q) continue;
                            const float ex = xyz[3 * j] - qx, ey = xyz[3 * j + 1] - qy, ez = xyz[3 * j + 2] - qz;
                            const float d2 = ex * ex + ey * ey + ez * ez;
                            insert<K>(bd, bi, d2, (int32_t)j);
                            found++;
                        }
                    }
                }
            // every point in shells > s is farther than s * h
            const float bound = (float)s * g.h;
            if (found >= k && bd[k - 1] <= bound * bound) done = true;
            if (found >= g.n - 1) done = true;
        }
        if (!done) set_status(status, 1);
#pragma unroll
        for (int j = 0; j < K; j++)
            if (j < k) nbr[q * k + j] = bi[j] == INT32_MAX ? -1 : (int64_t)bi[j];
    }
}

}  // namespace
}  // namespace feq

using namespace feq;

extern "C" {

size_t feq_knn_workspace_bytes(int64_t num_points) {
    size_t tmp = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tmp, (const int64_t *)nullptr, (int64_t *)nullptr,
                                    (const int64_t *)nullptr, (int64_t *)nullptr, (int)std::max<int64_t>(num_points, 1));
    return 4 * sizeof(int64_t) * (size_t)std::max<int64_t>(num_points, 1) + tmp + 1024;
}

int feq_knn_graph(const float *xyz, int64_t num_points, int32_t k, float cell, float x0, float y0, float z0,
                  int64_t *nbr, int32_t *status, void *workspace, size_t workspace_bytes, feq_stream_t stream) {
    if (num_points < 0 || k < 1 || k > kKnnMax || !(cell > 0.0f)) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_points == 0) return FEQ_OK;
    if (!xyz || !nbr || !workspace) return FEQ_ERR_INVALID_ARGUMENT;
    if (num_points > 0x7fffffffll) return FEQ_ERR_UNSUPPORTED;
    if (workspace_bytes < feq_knn_workspace_bytes(num_points)) return FEQ_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    WsCarver w{(char *)workspace, 0, workspace_bytes};
    const int64_t n = num_points;
    int64_t *keys = (int64_t *)w.take(sizeof(int64_t) * n), *ids = (int64_t *)w.take(sizeof(int64_t) * n);
    int64_t *sk = (int64_t *)w.take(sizeof(int64_t) * n), *sid = (int64_t *)w.take(sizeof(int64_t) * n);
    size_t tmp_bytes = 0;
    FEQ_CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, keys, sk, ids, sid, (int)n));
    void *tmp = w.take(tmp_bytes);
    if (w.used > workspace_bytes) return FEQ_ERR_WORKSPACE;
    KnnGrid g{x0, y0, z0, 1.0f / cell, cell, n};
    const int grid = (int)min64((n + 255) / 256, 148 * 16);
    knn_keys_kernel<<<grid, 256, 0, s>>>(xyz, g, keys, ids);
    FEQ_LAUNCH_CHECK();
    FEQ_CUDA_TRY(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys, sk, ids, sid, (int)n, 0, 63, s));
    count_launches(3);
    const int qgrid = (int)min64((n + 127) / 128, 148 * 32);
    if (k <= 16) knn_query_kernel<16><<<qgrid, 128, 0, s>>>(xyz, g, sk, sid, k, nbr, status);
    else if (k <= 32) knn_query_kernel<32><<<qgrid, 128, 0, s>>>(xyz, g, sk, sid, k, nbr, status);
    else knn_query_kernel<64><<<qgrid, 128, 0, s>>>(xyz, g, sk, sid, k, nbr, status);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}

}  // extern "C"
