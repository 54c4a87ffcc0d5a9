// feq_radial_net.cu -- the radial features of SeparableRadialNet in one launch.
//
// Reference behaviour replaced (flash_eq/layers/radial.py:226-267, SeparableRadialNet):
//   x   = clamp((r_b - min) / (max - min), 0, 1)                       at every bin edge r_b
//   env = 1 - 10 x^3 + 15 x^4 - 6 x^5                                  (DimeNet envelope, p = 5)
//   e   = [sin(x f_j) env, cos(x f_j) env]_j                           (2 num_freqs values)
//   f   = head(SiLU(W2 SiLU(W1 e + b1) + b2))                          (rank * weight_dim values)
// In PyTorch that is about twenty small launches (the basis elementwise ops, three GEMMs, two
// SiLUs) per edgewise layer call, each a few microseconds of launch and ramp for a few hundred
// kilobytes of work; here one CTA per bin edge computes the whole chain in shared memory.
// Float32 throughout, each dot product accumulated in input order.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "feq_internal.cuh"

namespace feq {
namespace {

constexpr int kRnThreads = 128;
constexpr int kRnMaxFreqs = 64;
constexpr int kRnMaxHidden = 256;

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

__global__ void __launch_bounds__(kRnThreads)
radial_features_kernel(const float *__restrict__ edges, float lo, float range, const float *__restrict__ freqs,
                       int nf, const float *__restrict__ w1, const float *__restrict__ b1, int hidden,
                       const float *__restrict__ w2, const float *__restrict__ b2, const float *__restrict__ w3,
                       const float *__restrict__ b3, int out_dim, float *__restrict__ out) {
    __shared__ float basis[2 * kRnMaxFreqs];
    __shared__ float h1[kRnMaxHidden], h2[kRnMaxHidden];
    const int b = blockIdx.x, t = threadIdx.x;
    {
        float x = (edges[b] - lo) / range;
        x = fminf(fmaxf(x, 0.0f), 1.0f);
        const float x3 = x * x * x, x4 = x3 * x, x5 = x4 * x;
        const float env = 1.0f - 10.0f * x3 + 15.0f * x4 - 6.0f * x5;
        for (int j = t; j < nf; j += kRnThreads) {
            const float ang = x * freqs[j];
            basis[j] = sinf(ang) * env;
            basis[nf + j] = cosf(ang) * env;
        }
    }
    __syncthreads();
    const int n0 = 2 * nf;
    for (int j = t; j < hidden; j += kRnThreads) {
        const float *w = w1 + (int64_t)j * n0;
        float acc = 0.0f;
        for (int i = 0; i < n0; i++) acc = fmaf(w[i], basis[i], acc);
        h1[j] = silu(acc + b1[j]);
    }
    __syncthreads();
    for (int j = t; j < hidden; j += kRnThreads) {
        const float *w = w2 + (int64_t)j * hidden;
        float acc = 0.0f;
        for (int i = 0; i < hidden; i++) acc = fmaf(w[i], h1[i], acc);
        h2[j] = silu(acc + b2[j]);
    }
    __syncthreads();
    for (int o = t; o < out_dim; o += kRnThreads) {
        const float *w = w3 + (int64_t)o * hidden;
        float acc = 0.0f;
        for (int i = 0; i < hidden; i++) acc = fmaf(w[i], h2[i], acc);
        out[(int64_t)b * out_dim + o] = acc + b3[o];
    }
}

}  // namespace
}  // namespace feq

using namespace feq;

extern "C" int feq_radial_features(const float *bin_edges, int32_t num_edges, float min_val, float max_val,
                                   const float *frequencies, int32_t num_freqs, const float *w1, const float *b1,
                                   int32_t hidden, const float *w2, const float *b2, const float *w3,
                                   const float *b3, int32_t out_dim, float *out, feq_stream_t stream) {
    if (num_edges < 0 || num_freqs < 1 || hidden < 1 || out_dim < 1 || !(max_val > min_val))
        return FEQ_ERR_INVALID_ARGUMENT;
    if (num_freqs > kRnMaxFreqs || hidden > kRnMaxHidden) return FEQ_ERR_UNSUPPORTED;
    if (num_edges == 0) return FEQ_OK;
    if (!bin_edges || !frequencies || !w1 || !b1 || !w2 || !b2 || !w3 || !b3 || !out) return FEQ_ERR_INVALID_ARGUMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    ProfScope prof("radial_features", s);
    radial_features_kernel<<<(unsigned)num_edges, kRnThreads, 0, s>>>(bin_edges, min_val, max_val - min_val,
                                                                       frequencies, num_freqs, w1, b1, hidden, w2, b2,
                                                                       w3, b3, out_dim, out);
    FEQ_LAUNCH_CHECK();
    return FEQ_OK;
}
