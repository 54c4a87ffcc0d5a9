// feq_noalloc.cu -- feq_block_diagonal_fwd for callers that cannot allocate.
//
// Some callers have no way to obtain device memory for a workspace: code that runs
// inside a host framework which owns every allocation, a plugin handed raw pointers
// but no allocator, or a context where allocating is not allowed at all.  This entry
// point gives them the block-diagonal radial mix with its scratch taken from a fixed
// array that lives in the library's own device memory.
//
// The array's name is only a host-side stand-in in host code, so on every call the
// host looks up its device address with cudaGetSymbolAddress (with the caller's device
// current) and passes that address as the workspace of the ordinary entry point.  The
// lookup allocates nothing; doing it per call (instead of caching it) keeps the address
// right after a device reset or a new primary context on that device.
// Every call shares the array; overlapping calls race (see include/flasheq_b200.h).
#include <cuda_runtime.h>
#include <stdio.h>

#include "feq_internal.cuh"

namespace feq {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FEQ_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device.
static int scratch_address(void **addr) {
    void *p = nullptr;
    FEQ_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    *addr = p;
    return FEQ_OK;
}

}  // namespace feq

extern "C" int feq_block_diagonal_fwd_noalloc(const float *features, const float *radial_table,
                                              const float *distances, int64_t num_edges, int32_t c_in,
                                              int32_t c_out, const int32_t *lvals_in, int32_t n_lvals_in,
                                              const int32_t *lvals_out, int32_t n_lvals_out, float sh_scale,
                                              float bin_param1, float bin_param2, int32_t num_bins,
                                              int32_t log_bins, float *output, feq_stream_t stream) {
    const size_t need = feq_block_diagonal_workspace_bytes(num_edges, c_in, c_out, lvals_in, n_lvals_in,
                                                           lvals_out, n_lvals_out, num_bins);
    if (need == 0) return FEQ_ERR_INVALID_ARGUMENT;   // layout or sizes rejected
    if (need > FEQ_NOALLOC_SCRATCH_BYTES) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "no-alloc block-diagonal: this problem needs %zu bytes of scratch, the built-in "
                 "scratch holds %zu bytes (use feq_block_diagonal_fwd with a workspace)",
                 need, (size_t)FEQ_NOALLOC_SCRATCH_BYTES);
        feq::record_error_text(msg);
        return FEQ_ERR_WORKSPACE;
    }
    void *scratch = nullptr;
    const int rc = feq::scratch_address(&scratch);
    if (rc != FEQ_OK) return rc;
    return feq_block_diagonal_fwd(features, radial_table, distances, num_edges, c_in, c_out, lvals_in,
                                  n_lvals_in, lvals_out, n_lvals_out, sh_scale, bin_param1, bin_param2,
                                  num_bins, log_bins, output, scratch, FEQ_NOALLOC_SCRATCH_BYTES, stream);
}
