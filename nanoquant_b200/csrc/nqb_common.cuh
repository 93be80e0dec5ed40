// Shared helpers for libnqb: status reporting, dtype-generic loads, small
// device utilities.  Internal header; the public ABI is include/nqb.h.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/nqb.h"

namespace nqb {

// ---------------------------------------------------------------- status ---

// Records a printf-style message for nqb_last_error() and returns `code`.
int fail(int code, const char *fmt, ...);
// Clears the calling thread's message; returns NQB_OK.
int ok();
// Maps a CUDA error (after a launch or API call) to NQB_ERR_CUDA with context.
int cuda_status(cudaError_t err, const char *what);

#define NQB_CHECK(expr)                                                        \
  do {                                                                         \
    int _nqb_rc = (expr);                                                      \
    if (_nqb_rc != NQB_OK) return _nqb_rc;                                     \
  } while (0)

#define NQB_CUDA(expr, what)                                                   \
  do {                                                                         \
    cudaError_t _nqb_err = (expr);                                             \
    if (_nqb_err != cudaSuccess) return ::nqb::cuda_status(_nqb_err, what);    \
  } while (0)

// Raises a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute is set once per (kernel, device, size
// increase), so calls made during CUDA-graph capture do not touch it again.
int ensure_dynamic_smem(const void *kernel, size_t bytes);

inline bool is_float_dtype(int32_t dt) { return dt == NQB_F32 || dt == NQB_F16 || dt == NQB_BF16; }
__host__ __device__ inline size_t dtype_size(int32_t dt) {
  switch (dt) {
    case NQB_F32: return 4;
    case NQB_F16: return 2;
    case NQB_BF16: return 2;
    case NQB_I8: return 1;
    case NQB_I32: return 4;
  }
  return 0;
}
inline int64_t words_for(int64_t columns) { return (columns + 31) / 32; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ------------------------------------------------------------ device side ---

// Load element i of a buffer whose dtype is only known at run time.  The
// dtype is uniform across a launch, so the switch does not diverge.
__device__ __forceinline__ float load_as_float(const void *p, int64_t i, int32_t dt) {
  switch (dt) {
    case NQB_F32: return __ldg(reinterpret_cast<const float *>(p) + i);
    case NQB_F16: return __half2float(reinterpret_cast<const __half *>(p)[i]);
    case NQB_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    case NQB_I8: return static_cast<float>(reinterpret_cast<const int8_t *>(p)[i]);
    default: return 0.0f;
  }
}

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Flip the sign of `v` when `neg` is 1 (exact: only the sign bit changes).
__device__ __forceinline__ float apply_sign(float v, uint32_t neg) {
  return __uint_as_float(__float_as_uint(v) ^ (neg << 31));
}

}  // namespace nqb
