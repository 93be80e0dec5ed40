// Tensor-core (tcgen05) decode path of libnqb.  Not enabled yet: every call
// takes the generic path.
#include "nqb_decode_tc.cuh"

namespace nqb {

bool tc_eligible(const nqb_linear_desc *, int, int32_t, int64_t) { return false; }

size_t tc_extra_workspace_bytes(const nqb_linear_desc *, int, int64_t) { return 0; }

int run_tc(const nqb_linear_desc *, int, const void *, int32_t, int64_t, float *const *, void *, size_t,
           float *, cudaStream_t) {
  return fail(NQB_ERR_UNSUPPORTED, "tensor-core decode path is not built");
}

}  // namespace nqb
