// Internal declarations of the tensor-core (tcgen05, fp16) prefill path of libnqb.
#pragma once

#include "nqb_common.cuh"

namespace nqb {

// True when the prefill tensor-core path takes this call (more than 16 tokens, tiles present).
bool prefill_eligible(const nqb_linear_desc *layers, int count, int32_t x_dtype, int64_t tokens);
// Workspace for the fp16 activations and per-token exponents; 0 if not eligible.
size_t prefill_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens);
// Runs 1..3 layers sharing x; `latent` is the fp32 [tokens, total rank] buffer.
int run_prefill(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
                float *const *ys, float *latent, void *extra, size_t extra_bytes, cudaStream_t stream);
// Reads and clears the prefill kernels' device status word.
int prefill_device_error(int32_t *out);

}  // namespace nqb
