// Device building blocks of the tcgen05 int8 decode arithmetic, shared by the
// per-call stage kernels (nqb_decode_tc.cu) and the persistent decode
// program (nqb_program.cu).  Internal header.
//
// A sign-matrix product out[row, t] = sum_k sign(S[row, k]) * a[t, k] runs as
// kind::i8 MMAs (M = 128 rows, K = 32):
// * B: the activations of a K slice, per token quantised to 22-bit fixed point
//   q = rint(a * 2^e) (e from the slice maximum) and split into three signed
//   base-256 digits, the N columns (3 per token) of an int8 matrix.
// * A: the raw sign bits (sign = 1 - 2*bit) as uint8 0/1 in tensor memory;
//   sum_k sign_k q_k = Q - 2 * sum_k bit_k q_k with Q = sum_k q_k.  A sign word
//   w becomes eight registers (w & 0x01010101<<j) and ((w>>4) & 0x01010101<<j),
//   j = 0..3, whose bytes are bit * 2^j; each j has its own accumulator and the
//   drain adds D_j >> j (exact).
// The sign words come in 4 KB slices: 256 input columns (8 words) of one
// 128-row tile in the row-interleaved layout of nqb_repack_signs.
#pragma once

#include "nqb_common.cuh"
#include "nqb_tc_ptx.cuh"

namespace nqb {
namespace tc {

constexpr int kThreads = 128;       // one thread per tile row (TMEM lane)
constexpr int kTileRows = 128;      // MMA M
constexpr int kStageWords = 8;      // sign words per row per slice
constexpr int kStageCols = 256;     // input columns per slice
constexpr int kChunkBytes = 16;     // one 4-word chunk of one row
constexpr int kStageWeightBytes = kTileRows * 2 * kChunkBytes;  // 4 KB per slice
constexpr int kClasses = 4;         // accumulators (bit weight 2^j)
constexpr int kAStageCols = 64;     // TMEM columns of A per slice
constexpr int kDCol = 2 * kAStageCols;  // first accumulator column (after two A buffers)
constexpr int kMaxTokens = 16;
constexpr int kMaxStagesPerCta = 8;  // <= 2048 input columns quantised at once
constexpr int kQuadsPerThread = kMaxStagesPerCta * 64 / kThreads;
constexpr int kDigits = 3;
constexpr int kMaxNPad = 48;

__host__ __device__ constexpr int n_pad_for(int tokens) { return ((kDigits * tokens + 15) / 16) * 16; }

// Bytes of one (slice, class, half) block of the B image for MMA width n_pad.
__host__ __device__ constexpr uint32_t b_block_bytes(int n_pad) { return 32u * n_pad; }

// Splits four fixed-point values into three signed base-256 digits each
// (q = d0 + 256*d1 + 65536*d2, every digit in [-128, 127]) and packs digit k
// of the four values, one byte per value, into w[k].
__device__ __forceinline__ void split_digits(const int32_t (&q)[4], uint32_t (&w)[kDigits]) {
  w[0] = w[1] = w[2] = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    int32_t v = q[b];
    const int32_t d0 = static_cast<int8_t>(v & 0xFF);
    v = (v - d0) >> 8;
    const int32_t d1 = static_cast<int8_t>(v & 0xFF);
    const int32_t d2 = (v - d1) >> 8;
    w[0] |= (static_cast<uint32_t>(d0) & 0xFFu) << (8 * b);
    w[1] |= (static_cast<uint32_t>(d1) & 0xFFu) << (8 * b);
    w[2] |= (static_cast<uint32_t>(d2) & 0xFFu) << (8 * b);
  }
}

// Input column of byte b of quad (slice sl, word i, bit class j, nibble s).
__device__ __forceinline__ int quad_column(int sl, int i, int j, int s, int b) {
  return sl * kStageCols + 32 * i + 8 * b + j + 4 * s;
}

// 2^e as a float, exactly, for e in [-126, 127].
__device__ __forceinline__ float exp2_int(int e) { return __int_as_float((e + 127) << 23); }

// Copies the K slice [k0, k0 + ncols) of x * pre of every token into shared
// memory as fp32 (zero past k_valid).  Each thread keeps 16 loads in flight
// before it stores any of them; activations are read through L2 (.cg) since
// an earlier grid stage may have written them.
constexpr int kStageBatch = 16;

template <typename XT, typename ST>
__device__ __forceinline__ void stage_input_slice(const XT *x, const ST *pre, int64_t n, int64_t k0, int ncols,
                                                  int tokens, int64_t k_valid, float *out, int nthreads) {
  const int total = tokens * ncols;
  for (int base = threadIdx.x; base < total; base += kStageBatch * nthreads) {
    float xv[kStageBatch], pv[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = base + u * nthreads;
      xv[u] = 0.0f;
      pv[u] = 0.0f;
      if (i < total) {
        const int t = i / ncols;
        const int64_t col = k0 + (i - t * ncols);
        if (col < k_valid) {
          xv[u] = to_f32(__ldcg(x + static_cast<int64_t>(t) * n + col));
          pv[u] = to_f32(pre[col]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = base + u * nthreads;
      if (i < total) out[i] = xv[u] * pv[u];
    }
  }
}

template <typename XT>
__device__ __forceinline__ void stage_input_slice_pre(const XT *x, const void *pre, int32_t scale_dtype, int64_t n,
                                                      int64_t k0, int ncols, int tokens, int64_t k_valid,
                                                      float *out, int nthreads) {
  switch (scale_dtype) {
    case NQB_F32:
      stage_input_slice(x, static_cast<const float *>(pre), n, k0, ncols, tokens, k_valid, out, nthreads);
      break;
    case NQB_F16:
      stage_input_slice(x, static_cast<const __half *>(pre), n, k0, ncols, tokens, k_valid, out, nthreads);
      break;
    default:
      stage_input_slice(x, static_cast<const __nv_bfloat16 *>(pre), n, k0, ncols, tokens, k_valid, out, nthreads);
      break;
  }
}

// Stage-1 activations: x * pre (dtype dispatch outside the loops), by the
// first `nthreads` threads of the block.
__device__ __forceinline__ void stage_x_slice(const void *x, int32_t x_dtype, const void *pre, int32_t scale_dtype,
                                              int64_t n, int64_t k0, int ncols, int tokens, int64_t k_valid,
                                              float *out, int nthreads = kThreads) {
  switch (x_dtype) {
    case NQB_F32:
      stage_input_slice_pre(static_cast<const float *>(x), pre, scale_dtype, n, k0, ncols, tokens, k_valid, out,
                            nthreads);
      break;
    case NQB_F16:
      stage_input_slice_pre(static_cast<const __half *>(x), pre, scale_dtype, n, k0, ncols, tokens, k_valid, out,
                            nthreads);
      break;
    default:
      stage_input_slice_pre(static_cast<const __nv_bfloat16 *>(x), pre, scale_dtype, n, k0, ncols, tokens, k_valid,
                            out, nthreads);
      break;
  }
}

// Stage-2 activations: latent[t * stride + offset + col] (read through L2).
__device__ __forceinline__ void stage_latent_slice(const float *latent, int64_t stride, int64_t offset, int64_t k0,
                                                   int ncols, int tokens, int64_t k_valid, float *out,
                                                   int nthreads = kThreads) {
  const int total = tokens * ncols;
  for (int base = threadIdx.x; base < total; base += kStageBatch * nthreads) {
    float v[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = base + u * nthreads;
      v[u] = 0.0f;
      if (i < total) {
        const int t = i / ncols;
        const int64_t col = k0 + (i - t * ncols);
        if (col < k_valid) v[u] = __ldcg(latent + static_cast<int64_t>(t) * stride + offset + col);
      }
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = base + u * nthreads;
      if (i < total) out[i] = v[u];
    }
  }
}

// Scratch of build_b_image in static shared memory.
template <int kT>
struct BImageScratch {
  int exp[kT];
  long long qsum[kT];
  float red_f[4 * kT];
  long long red_q[4 * kT];
};

// Quantises the staged activations s_act[T][nst * 256] into the B image
// (nst slices x 4 classes x 2 halves of b_block bytes, K-major no-swizzle
// core matrices) and records per token the exponent e and Q = sum q.  Ends
// with the async-proxy fence and a CTA barrier, so MMAs may read the image.
// Column-padding rows of N (>= 3T) are left as they are; their accumulator
// columns are never read.
template <int kT>
__device__ __forceinline__ void build_b_image(const float *s_act, int nst, int T, uint8_t *smem_b, uint32_t b_block,
                                              BImageScratch<kT> &sc) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int ncols = nst * kStageCols;
  const int nquads = nst * 64;
  // per-token maximum over the slice -> power-of-two scale 2^e
  float mx[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) mx[t] = 0.0f;
  for (int c = tid; c < ncols; c += kThreads) {
#pragma unroll
    for (int t = 0; t < kT; ++t)
      if (t < T) mx[t] = fmaxf(mx[t], fabsf(s_act[t * ncols + c]));
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    if (t < T) {
      float v = mx[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
      if (lane == 0) sc.red_f[warp * kT + t] = v;
    }
  }
  __syncthreads();
  if (tid < T) {
    const float v = fmaxf(fmaxf(sc.red_f[tid], sc.red_f[kT + tid]), fmaxf(sc.red_f[2 * kT + tid], sc.red_f[3 * kT + tid]));
    int e = 0;
    if (v > 0.0f && isfinite(v)) {
      int ex;
      frexpf(v, &ex);   // v < 2^ex
      e = 22 - ex;      // |a * 2^e| < 2^22
      e = min(e, 126);  // keep 2^e and 2^-e normal floats (only |a| < 2^-104 loses bits)
    }
    sc.exp[tid] = e;
  }
  __syncthreads();
  // quantise, split into digits, scatter into the MMA's K order
  long long qsum[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) qsum[t] = 0;
#pragma unroll
  for (int i = 0; i < kQuadsPerThread; ++i) {
    const int qd = tid + i * kThreads;
    if (qd < nquads) {
      const int sl = qd >> 6;
      const int r = qd & 63;
      const int wi = r >> 3, j = (r >> 1) & 3, s = r & 1;
      const uint32_t block = (static_cast<uint32_t>(sl) * 4 + j) * 2 + (wi >> 2);
      const uint32_t pk = 4 * ((wi & 3) * 2 + s);  // first K position of the quad in its MMA
      const int c0 = quad_column(sl, wi, j, s, 0);
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        if (t < T) {
          const float scale = exp2_int(sc.exp[t]);  // exact power of two
          int32_t q[4];
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) {
            q[bb] = __float2int_rn(s_act[t * ncols + c0 + 8 * bb] * scale);
            qsum[t] += q[bb];
          }
          uint32_t digits[kDigits];
          split_digits(q, digits);
#pragma unroll
          for (int d = 0; d < kDigits; ++d) {
            const uint32_t nrow = 3 * t + d;
            const uint32_t offset = block * b_block + (nrow >> 3) * 256 + (pk >> 4) * 128 + (nrow & 7) * 16 + (pk & 15);
            *reinterpret_cast<uint32_t *>(smem_b + offset) = digits[d];
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    if (t < T) {
      long long v = qsum[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) sc.red_q[warp * kT + t] = v;
    }
  }
  __syncthreads();
  if (tid < T) sc.qsum[tid] = sc.red_q[tid] + sc.red_q[kT + tid] + sc.red_q[2 * kT + tid] + sc.red_q[3 * kT + tid];
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B image -> tensor core (async proxy)
  __syncthreads();
}

// The 64 A registers (bit classes x halves) of one row's 8 sign words.
__device__ __forceinline__ void expand_slice(uint4 c0, uint4 c1, uint32_t (&a)[kAStageCols]) {
  const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w = words[i];
    const uint32_t hi = w >> 4;
#pragma unroll
    for (int j = 0; j < kClasses; ++j) {
      const uint32_t mask = 0x01010101u << j;
      const int col = j * 16 + (i >> 2) * 8 + (i & 3) * 2;
      a[col] = w & mask;
      a[col + 1] = hi & mask;
    }
  }
}

// The eight MMAs of one slice (4 classes x 2 halves of K = 32), one thread.
// The four accumulators start at TMEM column d_col (kDCol for one set).
__device__ __forceinline__ void issue_slice_mmas(uint32_t tmem, int buf, int sl, uint32_t b_base, uint32_t b_block,
                                                 uint32_t idesc, int n_pad, bool first, uint32_t d_col = kDCol) {
#pragma unroll
  for (int j = 0; j < kClasses; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t block = (static_cast<uint32_t>(sl) * 4 + j) * 2 + h;
      const uint64_t bdesc = ptx::smem_desc_kmajor(b_base + block * b_block, 128, 256);
      ptx::mma_i8_ts(tmem + d_col + j * n_pad, tmem + buf * kAStageCols + j * 16 + h * 8, bdesc, idesc,
                     (!first || h > 0) ? 1u : 0u);
    }
  }
}

// Reads this thread's row of the four accumulators (starting at TMEM column
// d_col) and combines the classes: sacc[c] = sum_j D_j[c] >> j for the
// first n_pad columns.
template <int kNP>
__device__ __forceinline__ void drain_accumulators(uint32_t tmem, uint32_t lane_base, int32_t (&sacc)[kNP],
                                                   uint32_t d_col = kDCol) {
#pragma unroll
  for (int n = 0; n < kNP; ++n) sacc[n] = 0;
#pragma unroll
  for (int j = 0; j < kClasses; ++j) {
    uint32_t v[kNP];
#pragma unroll
    for (int qb = 0; qb < kNP / 16; ++qb) ptx::tmem_ld16(tmem + lane_base + d_col + j * kNP + qb * 16, v + qb * 16);
    ptx::tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < kNP; ++e) sacc[e] += static_cast<int32_t>(v[e]) >> j;
  }
}

// fp32 value of token t from the combined accumulators: one rounding
// (int64 -> fp32), then the exact power-of-two unscale.
template <int kNP>
__device__ __forceinline__ float token_value(const int32_t (&sacc)[kNP], int t, long long qsum, int e) {
  const long long st = static_cast<long long>(sacc[3 * t]) + 256ll * sacc[3 * t + 1] + 65536ll * sacc[3 * t + 2];
  return __ll2float_rn(qsum - 2 * st) * exp2_int(-e);
}

}  // namespace tc
}  // namespace nqb
