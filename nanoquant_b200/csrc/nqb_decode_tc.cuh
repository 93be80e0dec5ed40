// Internal declarations of the tensor-core (tcgen05) decode path of libnqb.
#pragma once

#include "nqb_common.cuh"

namespace nqb {

constexpr int kMaxMembersTc = 3;
// Fixed-size region of completion counters at the start of every workspace.
constexpr size_t kCounterRegionBytes = 16384;
constexpr int kMaxCounters = static_cast<int>(kCounterRegionBytes / sizeof(int32_t));

// True when the tcgen05 path takes this call (shapes, dtypes, token count).
bool tc_eligible(const nqb_linear_desc *layers, int count, int32_t x_dtype, int64_t tokens);
// Workspace for the tcgen05 path's K-split partials (beyond the counter region
// and the fp32 latent); 0 if not eligible.
size_t tc_extra_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens);
// Runs 1..3 layers sharing x through the tcgen05 kernels.
// `counters` is the zero-on-entry counter region; `extra` holds the partials.
int run_tc(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
           float *const *ys, int32_t *counters, void *extra, size_t extra_bytes, float *latent, float *patch,
           cudaStream_t stream);

// Row-interleaved tile copy of a sign matrix (see nqb_repack_signs).
int32_t repack_chunks(int64_t columns);
size_t repack_bytes(int64_t rows, int64_t columns);
int launch_repack(const uint32_t *words, int64_t rows, int64_t columns, uint32_t *tiles, cudaStream_t stream);
// Reads and clears the tensor-core kernels' device status word.
int tc_device_error(int32_t *out);

}  // namespace nqb
