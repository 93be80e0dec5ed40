// Internal declarations of the tensor-core (tcgen05) decode path of libnqb.
#pragma once

#include "nqb_common.cuh"

namespace nqb {

// True when the tcgen05 path takes this call (shapes, dtypes, token count).
bool tc_eligible(const nqb_linear_desc *layers, int count, int32_t x_dtype, int64_t tokens);
// Extra workspace (beyond the fp32 latent) the tcgen05 path needs; 0 if not eligible.
size_t tc_extra_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens);
// Runs 1..3 layers sharing x through the tcgen05 kernels.
int run_tc(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
           float *const *ys, void *extra, size_t extra_bytes, float *latent, cudaStream_t stream);

}  // namespace nqb
