// Tensor-core (tcgen05) decode path of libnqb: batch 1..16 tokens.
//
// Both stages of the packed linear are sign-matrix products
//     out[row, t] = sum_k sign(S[row, k]) * a[t, k]
// (stage 1: S = V, a = x * pre; stage 2: S = U, a = latent).  This path runs
// them on the 5th-generation tensor cores with exact integer arithmetic:
//
// * Activations -> B operand.  Each CTA quantises its K-slice of `a` per token
//   to 22-bit fixed point with a power-of-two scale 2^e (e from the slice
//   maximum), q = rint(a * 2^e), split into three signed base-256 digits; the
//   digits are the N columns (3 per token) of an int8 B matrix in shared memory.
// * Signs -> A operand in tensor memory.  With sign = 1 - 2*bit,
//     sum_k sign_k q_k = Q - 2 * sum_k bit_k q_k,   Q = sum_k q_k,
//   so A only needs the raw bits as uint8 0/1 values.  A 32-bit sign word w
//   becomes eight A registers with one LOP3 each: (w & 0x01010101<<j) and
//   ((w>>4) & 0x01010101<<j), j = 0..3, whose bytes are bit*2^j.  Registers of
//   the same j share a power of two, so each j has its own accumulator and the
//   epilogue adds D_j >> j (exact).  K order inside an MMA is therefore a fixed
//   permutation of the input columns, which the B image follows.
// * tcgen05.mma kind::i8, M = 128 rows, N = 16..48, K = 32, A from TMEM
//   (written with tcgen05.st), B from shared memory, int32 accumulators in TMEM.
//
// The sign words arrive in a row-interleaved tile layout made at prepare time
// (nqb_repack_signs): per 128-row tile and per 4-word chunk, the 128 rows'
// 16-byte chunks are contiguous, so one CTA's whole K-slice is one contiguous
// block that a single bulk copy (cp.async.bulk) brings into shared memory.
//
// Integer accumulation is exact, so the only rounding is the 22-bit
// quantisation of the activations and the final conversion to fp32; results
// are deterministic.  Stage 1 writes per-K-split fp32 partials; stage 2 reads
// them in a fixed order (times scale_mid) as its activations and the last CTA
// of each output tile reduces its partials, applies scale_post, salient
// columns, the int8 row overlay and bias, and writes y.
#include <cstring>

#include "nqb_decode_tc.cuh"
#include "nqb_tc_ptx.cuh"

namespace nqb {
namespace tc {

constexpr int kThreads = 128;       // one thread per tile row (TMEM lane)
constexpr int kTileRows = 128;      // MMA M
constexpr int kStageWords = 8;      // sign words per row per pipeline stage
constexpr int kStageCols = 256;     // input columns per stage
constexpr int kChunkBytes = 16;     // one 4-word chunk of one row
constexpr int kStageWeightBytes = kTileRows * 2 * kChunkBytes;  // 4 KB per stage
constexpr int kClasses = 4;         // accumulators (bit weight 2^j)
constexpr int kAStageCols = 64;     // TMEM columns of A per stage
constexpr int kDCol = 2 * kAStageCols;  // first accumulator column
constexpr int kMaxTokens = 16;
constexpr int kMaxStagesPerCta = 8;  // <= 2048 input columns per CTA
constexpr int kDigits = 3;
constexpr int kMaxNPad = 48;
constexpr uint32_t kSpinLimit = 1u << 28;

struct Member {
  const uint4 *tiles;    // row-interleaved tiles of the sign matrix
  int64_t rows;          // valid rows (rank for stage 1, out_features for stage 2)
  int32_t wc;            // 4-word chunks per row (even)
  int32_t row_tiles;
  int32_t k_stages;      // wc / 2
  int32_t splits;        // K splits
  int32_t stages_per_split;
  int32_t cta_begin;
  int64_t k_valid;       // valid K columns (in_features, or rank for stage 2)
  const void *pre;       // stage 1 activation scale
  const void *mid;       // stage 2: latent scale
  int64_t act_offset;    // stage 2: first latent column of this member
  int64_t out_offset;    // first row of this member in the partial buffer
  // stage 2 epilogue
  const void *post;
  const void *bias;
  int32_t bias_dtype;
  int64_t outlier_count;
  const int32_t *outlier_indices;
  const void *outlier_values;
  int32_t outlier_value_dtype;
  const void *outlier_scales;
  int64_t overlay_rows;
  const int32_t *overlay_row_ids;
  const int8_t *overlay_values;
  const void *overlay_scales;
  int32_t overlay_scale_dtype;
  float *y;
  int32_t *counters;  // [row_tiles]
};

struct Params {
  Member m[kMaxMembersTc];
  int32_t count;
  const void *x;
  int32_t x_dtype;
  int32_t scale_dtype;
  int64_t n;           // in_features
  int32_t tokens;
  int32_t n_pad;       // MMA N
  uint32_t tmem_cols;
  float *partial;      // this stage's output partials [splits][tokens][part_stride]
  int64_t part_stride;
  const float *act_partial;  // stage 2: stage-1 partials [s1_splits][tokens][act_stride]
  int32_t act_splits;
  int64_t act_stride;
};

__device__ int g_tc_error;  // first bounded-wait failure (0 = none), for diagnostics

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_tc_error, 0, code); }

// Value of activation column k (CTA-relative K range already applied) of token t.
template <bool kStage2>
__device__ __forceinline__ float activation(const Params &p, const Member &m, int t, int64_t k) {
  if (k >= m.k_valid) return 0.0f;
  if constexpr (!kStage2) {
    return load_as_float(p.x, static_cast<int64_t>(t) * p.n + k, p.x_dtype) *
           load_as_float(m.pre, k, p.scale_dtype);
  } else {
    float sum = 0.0f;
    const float *src = p.act_partial + static_cast<int64_t>(t) * p.act_stride + m.act_offset + k;
    for (int s = 0; s < p.act_splits; ++s)
      sum += __ldcg(src + static_cast<int64_t>(s) * p.tokens * p.act_stride);
    return sum * load_as_float(m.mid, k, p.scale_dtype);
  }
}

__device__ __forceinline__ uint32_t pack_digit_bytes(const int32_t (&q)[4], int digit) {
  uint32_t out = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    int32_t v = q[b];
    int32_t d = 0;
    for (int i = 0; i <= digit; ++i) {
      d = static_cast<int8_t>(v & 0xFF);
      v = (v - d) >> 8;
    }
    out |= (static_cast<uint32_t>(d) & 0xFFu) << (8 * b);
  }
  return out;
}

template <bool kStage2>
__global__ void __launch_bounds__(kThreads, 1) tc_stage_kernel(const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t s_bar_a[2];                    // A buffer b free again
  __shared__ uint64_t s_bar_done;                    // all MMAs complete
  __shared__ uint64_t s_bar_w[kMaxStagesPerCta];     // stage weights landed
  __shared__ uint32_t s_tmem;
  __shared__ int s_exp[kMaxTokens];
  __shared__ long long s_qsum[kMaxTokens];
  __shared__ float s_warp_max[4][kMaxTokens];
  __shared__ long long s_warp_q[4];
  __shared__ int s_last;
  __shared__ int s_failed;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  int g = 0;
  for (int i = 1; i < p.count; ++i)
    if (static_cast<int32_t>(blockIdx.x) >= p.m[i].cta_begin) g = i;
  const Member &m = p.m[g];
  const int local = static_cast<int>(blockIdx.x) - m.cta_begin;
  const int tile = local / m.splits;
  const int split = local - tile * m.splits;
  const int st_begin = split * m.stages_per_split;
  const int st_end = min(st_begin + m.stages_per_split, m.k_stages);
  const int nst = st_end - st_begin;
  const int T = p.tokens;
  const int NP = p.n_pad;
  const uint32_t b_block = 32u * NP;  // bytes of one (stage, class, half) B block

  uint8_t *smem_w = smem;                                   // nst * 4 KB weights
  uint8_t *smem_b = smem + nst * kStageWeightBytes;         // nst * 8 * b_block digits

  if (tid == 0) {
    s_failed = 0;
    ptx::mbar_init(&s_bar_a[0], 1);
    ptx::mbar_init(&s_bar_a[1], 1);
    ptx::mbar_init(&s_bar_done, 1);
    for (int s = 0; s < nst; ++s) ptx::mbar_init(&s_bar_w[s], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();

  // 1. start streaming this CTA's sign words: one bulk copy per stage
  if (tid == 0) {
    const uint8_t *src = reinterpret_cast<const uint8_t *>(m.tiles) +
                         (static_cast<size_t>(tile) * m.wc + 2 * st_begin) * (kTileRows * kChunkBytes);
    for (int s = 0; s < nst; ++s) {
      const uint32_t bar = ptx::smem_u32(&s_bar_w[s]);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kStageWeightBytes)
                   : "memory");
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              ptx::smem_u32(smem_w + s * kStageWeightBytes)),
          "l"(src + static_cast<size_t>(s) * kStageWeightBytes), "r"(kStageWeightBytes), "r"(bar)
          : "memory");
    }
  }
  // 2. tensor memory
  if (warp == 0) {
    ptx::tmem_alloc(&s_tmem, p.tmem_cols);
    ptx::tmem_relinquish();
  }
  // 3. clear the B image (unused N rows and K positions must be zero)
  {
    uint4 *b4 = reinterpret_cast<uint4 *>(smem_b);
    const int count = nst * 8 * static_cast<int>(b_block) / 16;
    for (int i = tid; i < count; i += kThreads) b4[i] = make_uint4(0, 0, 0, 0);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = s_tmem;

  // 4. quantise this K slice of the activations into the B image
  const int64_t k0 = static_cast<int64_t>(st_begin) * kStageCols;
  const int ncols = nst * kStageCols;
  {
    float mx[kMaxTokens];
#pragma unroll
    for (int t = 0; t < kMaxTokens; ++t) mx[t] = 0.0f;
    for (int c = tid; c < ncols; c += kThreads) {
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t)
        if (t < T) mx[t] = fmaxf(mx[t], fabsf(activation<kStage2>(p, m, t, k0 + c)));
    }
#pragma unroll
    for (int t = 0; t < kMaxTokens; ++t) {
      float v = mx[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
      if (lane == 0) s_warp_max[warp][t] = v;
    }
    __syncthreads();
    if (tid < T) {
      const float v = fmaxf(fmaxf(s_warp_max[0][tid], s_warp_max[1][tid]), fmaxf(s_warp_max[2][tid], s_warp_max[3][tid]));
      int e = 0;
      if (v > 0.0f && isfinite(v)) {
        int ex;
        frexpf(v, &ex);  // v < 2^ex
        e = 22 - ex;     // |a * 2^e| < 2^22
      }
      s_exp[tid] = e;
    }
    __syncthreads();

    const int nquads = nst * 64;
    for (int t = 0; t < T; ++t) {
      const int e = s_exp[t];
      long long qsum = 0;
      for (int qd = tid; qd < nquads; qd += kThreads) {
        const int sl = qd >> 6;
        const int r = qd & 63;
        const int i = r >> 3;        // word in stage
        const int j = (r >> 1) & 3;  // bit class
        const int s = r & 1;         // low / high nibble
        int32_t q[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int64_t col = k0 + sl * kStageCols + 32 * i + 8 * b + j + 4 * s;
          q[b] = __float2int_rn(ldexpf(activation<kStage2>(p, m, t, col), e));
          qsum += q[b];
        }
        const uint32_t block = (static_cast<uint32_t>(sl) * 4 + j) * 2 + (i >> 2);
        const uint32_t pk = 4 * ((i & 3) * 2 + s);  // first K position of the quad in its MMA
#pragma unroll
        for (int d = 0; d < kDigits; ++d) {
          const uint32_t nrow = 3 * t + d;
          const uint32_t offset = block * b_block + (nrow >> 3) * 256 + (pk >> 4) * 128 + (nrow & 7) * 16 + (pk & 15);
          *reinterpret_cast<uint32_t *>(smem_b + offset) = pack_digit_bytes(q, d);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, off);
      if (lane == 0) s_warp_q[warp] = qsum;
      __syncthreads();
      if (tid == 0) s_qsum[t] = s_warp_q[0] + s_warp_q[1] + s_warp_q[2] + s_warp_q[3];
      __syncthreads();
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B image -> tensor core (async proxy)
  __syncthreads();

  // 5. main loop: bits -> TMEM (A), one tcgen05.mma per (class, half) per stage
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t idesc = ptx::idesc_i8_m128(static_cast<uint32_t>(NP));
  const uint32_t b_base = ptx::smem_u32(smem_b);
  bool ok = true;
  for (int sl = 0; sl < nst; ++sl) {
    const int buf = sl & 1;
    if (!ptx::mbar_wait_bounded(&s_bar_w[sl], 0, kSpinLimit)) ok = false;
    const uint4 *wsrc = reinterpret_cast<const uint4 *>(smem_w + sl * kStageWeightBytes);
    const uint4 c0 = wsrc[tid];
    const uint4 c1 = wsrc[kTileRows + tid];
    const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    uint32_t a[kAStageCols];
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
    if (sl >= 2) {
      if (!ptx::mbar_wait_bounded(&s_bar_a[buf], ((sl - 2) >> 1) & 1, kSpinLimit)) ok = false;
      ptx::tc_fence_after();
    }
    const uint32_t a_addr = tmem + lane_base + buf * kAStageCols;
#pragma unroll
    for (int q = 0; q < kAStageCols / 16; ++q) ptx::tmem_st16(a_addr + q * 16, a + q * 16);
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int j = 0; j < kClasses; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t block = (static_cast<uint32_t>(sl) * 4 + j) * 2 + h;
          const uint64_t bdesc = ptx::smem_desc_kmajor(b_base + block * b_block, 128, 256);
          ptx::mma_i8_ts(tmem + kDCol + j * NP, tmem + buf * kAStageCols + j * 16 + h * 8, bdesc, idesc,
                         (sl > 0 || h > 0) ? 1u : 0u);
        }
      }
      ptx::mma_commit(&s_bar_a[buf]);
    }
  }
  if (tid == 0) ptx::mma_commit(&s_bar_done);
  if (!ptx::mbar_wait_bounded(&s_bar_done, 0, kSpinLimit)) ok = false;
  ptx::tc_fence_after();
  if (!ok) {
    s_failed = 1;
    record_error(NQB_ERR_TIMEOUT);
  }

  // 6. epilogue: combine classes and digits, convert to fp32 partials
  const int64_t row = static_cast<int64_t>(tile) * kTileRows + tid;
  {
    int32_t sacc[kMaxNPad];
#pragma unroll
    for (int n = 0; n < kMaxNPad; ++n) sacc[n] = 0;
#pragma unroll
    for (int j = 0; j < kClasses; ++j) {
#pragma unroll
      for (int qb = 0; qb < kMaxNPad / 16; ++qb) {
        if (qb * 16 < NP) {
          uint32_t v[16];
          ptx::tmem_ld16(tmem + lane_base + kDCol + j * NP + qb * 16, v);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) sacc[qb * 16 + e] += static_cast<int32_t>(v[e]) >> j;
        }
      }
    }
    if (row < m.rows) {
#pragma unroll
      for (int t = 0; t < kMaxTokens; ++t) {
        if (t < T) {
          const long long st = static_cast<long long>(sacc[3 * t]) + 256ll * sacc[3 * t + 1] +
                               65536ll * sacc[3 * t + 2];
          const double value = ldexp(static_cast<double>(s_qsum[t] - 2 * st), -s_exp[t]);
          p.partial[(static_cast<int64_t>(split) * T + t) * p.part_stride + m.out_offset + row] =
              static_cast<float>(value);
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, p.tmem_cols);

  if constexpr (kStage2) {
    // 7. the last CTA of this output tile reduces the K-split partials
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int previous = atomicAdd(m.counters + tile, 1);
      s_last = (previous == m.splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (row < m.rows) {
      const float post = load_as_float(m.post, row, p.scale_dtype);
      const float bias = m.bias != nullptr ? load_as_float(m.bias, row, m.bias_dtype) : 0.0f;
      const int64_t out_features = m.rows;
      for (int t = 0; t < T; ++t) {
        float acc = 0.0f;
        for (int s = 0; s < m.splits; ++s)
          acc += __ldcg(p.partial + (static_cast<int64_t>(s) * T + t) * p.part_stride + m.out_offset + row);
        float v = acc * post;
        if (m.outlier_count > 0) {
          float sal = 0.0f;
          for (int64_t s = 0; s < m.outlier_count; ++s) {
            float w = load_as_float(m.outlier_values, row * m.outlier_count + s, m.outlier_value_dtype);
            if (m.outlier_scales != nullptr) w *= load_as_float(m.outlier_scales, s, p.scale_dtype);
            sal += load_as_float(p.x, static_cast<int64_t>(t) * p.n + m.outlier_indices[s], p.x_dtype) * w;
          }
          v += sal;
        }
        m.y[static_cast<int64_t>(t) * out_features + row] = v + bias;
      }
    }
    if (m.overlay_rows > 0) {
      // residual rows of this tile: the whole CTA computes each dot product
      __syncthreads();
      const int64_t first = static_cast<int64_t>(tile) * kTileRows;
      const int64_t last = min(first + kTileRows, m.rows);
      int64_t lo = 0, hi = m.overlay_rows;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (m.overlay_row_ids[mid] < first) lo = mid + 1; else hi = mid;
      }
      for (int64_t jrow = lo; jrow < m.overlay_rows && m.overlay_row_ids[jrow] < last; ++jrow) {
        const int64_t orow = m.overlay_row_ids[jrow];
        const float scale = load_as_float(m.overlay_scales, jrow, m.overlay_scale_dtype);
        const int8_t *rv = m.overlay_values + jrow * p.n;
        for (int t = 0; t < T; ++t) {
          float part = 0.0f;
          for (int64_t i = tid; i < p.n; i += kThreads)
            part += static_cast<float>(rv[i]) * load_as_float(p.x, static_cast<int64_t>(t) * p.n + i, p.x_dtype);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
          if (lane == 0) s_warp_max[warp][0] = part;
          __syncthreads();
          if (tid == 0) {
            const float dot = (s_warp_max[0][0] + s_warp_max[1][0]) + (s_warp_max[2][0] + s_warp_max[3][0]);
            m.y[static_cast<int64_t>(t) * m.rows + orow] += dot * scale;
          }
          __syncthreads();
        }
      }
    }
    if (tid == 0) m.counters[tile] = 0;  // ready for the next call
  }
}

// ------------------------------------------------------------- repack ---

__global__ void repack_kernel(const uint32_t *words, int64_t rows, int64_t wpr, int32_t wc, int32_t row_tiles,
                              uint32_t *out) {
  const int64_t total = static_cast<int64_t>(row_tiles) * wc * kTileRows * 4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t wi = i & 3;
    const int64_t rr = (i >> 2) % kTileRows;
    const int64_t chunk_tile = (i >> 2) / kTileRows;  // tile * wc + c
    const int64_t c = chunk_tile % wc;
    const int64_t tile = chunk_tile / wc;
    const int64_t row = tile * kTileRows + rr;
    const int64_t word = c * 4 + wi;
    out[i] = (row < rows && word < wpr) ? words[row * wpr + word] : 0u;
  }
}

}  // namespace tc

// --------------------------------------------------------------- host ---

using tc::kMaxStagesPerCta;
using tc::kMaxTokens;

int32_t repack_chunks(int64_t columns) {
  const int64_t wpr = words_for(columns);
  return static_cast<int32_t>(2 * ((wpr + tc::kStageWords - 1) / tc::kStageWords));
}

size_t repack_bytes(int64_t rows, int64_t columns) {
  const int64_t tiles = (rows + tc::kTileRows - 1) / tc::kTileRows;
  return static_cast<size_t>(tiles) * repack_chunks(columns) * tc::kTileRows * tc::kChunkBytes;
}

int launch_repack(const uint32_t *words, int64_t rows, int64_t columns, uint32_t *tiles, cudaStream_t stream) {
  const int32_t wc = repack_chunks(columns);
  const int32_t row_tiles = static_cast<int32_t>((rows + tc::kTileRows - 1) / tc::kTileRows);
  const int64_t total = static_cast<int64_t>(row_tiles) * wc * tc::kTileRows * 4;
  const int64_t blocks = (total + 255) / 256;
  tc::repack_kernel<<<static_cast<unsigned>(blocks < 65535 * 16 ? blocks : 65535 * 16), 256, 0, stream>>>(
      words, rows, words_for(columns), wc, row_tiles, tiles);
  NQB_CUDA(cudaGetLastError(), "repack_kernel launch");
  return NQB_OK;
}

struct Plan {
  int32_t splits[kMaxMembersTc];
  int32_t sps[kMaxMembersTc];
  int32_t ctas;
};

// Split each member's K stages so the grid fills the GPU about twice.
static Plan plan_stage(const int32_t *row_tiles, const int32_t *k_stages, int count, bool uniform, int sms) {
  Plan plan{};
  int64_t tiles = 0;
  for (int i = 0; i < count; ++i) tiles += row_tiles[i];
  const int64_t target = 2 * static_cast<int64_t>(sms);
  int32_t want = static_cast<int32_t>((target + tiles - 1) / tiles);
  if (want < 1) want = 1;
  plan.ctas = 0;
  for (int i = 0; i < count; ++i) {
    int32_t splits = want < k_stages[i] ? want : k_stages[i];
    int32_t sps = (k_stages[i] + splits - 1) / splits;
    if (sps > kMaxStagesPerCta) sps = kMaxStagesPerCta;
    splits = (k_stages[i] + sps - 1) / sps;
    plan.splits[i] = splits;
    plan.sps[i] = sps;
  }
  if (uniform) {  // stage 1: every member shares K, keep one split count
    for (int i = 1; i < count; ++i) {
      plan.splits[i] = plan.splits[0];
      plan.sps[i] = plan.sps[0];
    }
  }
  for (int i = 0; i < count; ++i) plan.ctas += row_tiles[i] * plan.splits[i];
  return plan;
}

static int sm_count() {
  int device = 0, sms = 148;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms;
}

bool tc_eligible(const nqb_linear_desc *layers, int count, int32_t x_dtype, int64_t tokens) {
  if (tokens < 1 || tokens > kMaxTokens || count < 1 || count > kMaxMembersTc) return false;
  if (!is_float_dtype(x_dtype)) return false;
  for (int i = 0; i < count; ++i) {
    if (layers[i].right_tiles == nullptr || layers[i].left_tiles == nullptr) return false;
    if (reinterpret_cast<uintptr_t>(layers[i].right_tiles) % 16 || reinterpret_cast<uintptr_t>(layers[i].left_tiles) % 16)
      return false;
  }
  return true;
}

struct Sizes {
  size_t partial1, partial2, counters;
};

static Sizes tc_sizes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  const int sms = sm_count();
  int32_t rt[kMaxMembersTc], ks[kMaxMembersTc];
  int64_t total_rank = 0, total_out = 0;
  for (int i = 0; i < count; ++i) {
    rt[i] = static_cast<int32_t>((layers[i].rank + tc::kTileRows - 1) / tc::kTileRows);
    ks[i] = repack_chunks(layers[i].in_features) / 2;
    total_rank += layers[i].rank;
  }
  const Plan p1 = plan_stage(rt, ks, count, true, sms);
  int32_t max_s2 = 0;
  int64_t counters = 0;
  for (int i = 0; i < count; ++i) {
    rt[i] = static_cast<int32_t>((layers[i].out_features + tc::kTileRows - 1) / tc::kTileRows);
    ks[i] = repack_chunks(layers[i].rank) / 2;
    total_out += layers[i].out_features;
    counters += rt[i];
  }
  const Plan p2 = plan_stage(rt, ks, count, false, sms);
  for (int i = 0; i < count; ++i) max_s2 = p2.splits[i] > max_s2 ? p2.splits[i] : max_s2;
  Sizes s;
  s.partial1 = align_up(static_cast<size_t>(p1.splits[0]) * tokens * total_rank * sizeof(float), 256);
  s.partial2 = align_up(static_cast<size_t>(max_s2) * tokens * total_out * sizeof(float), 256);
  s.counters = align_up(static_cast<size_t>(counters) * sizeof(int32_t), 256);
  return s;
}

size_t tc_extra_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  if (!tc_eligible(layers, count, NQB_F32, tokens)) return 0;
  const Sizes s = tc_sizes(layers, count, tokens);
  return s.partial1 + s.partial2 + s.counters;
}

static int smem_bytes(int stages, int n_pad) {
  return stages * tc::kStageWeightBytes + stages * 8 * 32 * n_pad;
}

int run_tc(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
           float *const *ys, void *extra, size_t extra_bytes, float * /*latent*/, cudaStream_t stream) {
  const Sizes sizes = tc_sizes(layers, count, tokens);
  if (extra_bytes < sizes.partial1 + sizes.partial2 + sizes.counters)
    return fail(NQB_ERR_WORKSPACE, "tensor-core path workspace too small");
  char *ws = static_cast<char *>(extra);
  float *partial1 = reinterpret_cast<float *>(ws);
  float *partial2 = reinterpret_cast<float *>(ws + sizes.partial1);
  int32_t *counters = reinterpret_cast<int32_t *>(ws + sizes.partial1 + sizes.partial2);
  const int sms = sm_count();
  const int32_t n_pad = static_cast<int32_t>(((3 * tokens + 15) / 16) * 16);
  const uint32_t tmem_cols = (tc::kDCol + tc::kClasses * n_pad) <= 256 ? 256u : 512u;

  int64_t total_rank = 0, total_out = 0;
  for (int i = 0; i < count; ++i) {
    total_rank += layers[i].rank;
    total_out += layers[i].out_features;
  }

  // ---- stage 1: latent partials = V x (x * pre)
  tc::Params p1;
  std::memset(&p1, 0, sizeof(p1));
  {
    int32_t rt[kMaxMembersTc], ks[kMaxMembersTc];
    for (int i = 0; i < count; ++i) {
      rt[i] = static_cast<int32_t>((layers[i].rank + tc::kTileRows - 1) / tc::kTileRows);
      ks[i] = repack_chunks(layers[i].in_features) / 2;
    }
    const Plan plan = plan_stage(rt, ks, count, true, sms);
    int32_t cta = 0;
    int64_t offset = 0;
    for (int i = 0; i < count; ++i) {
      tc::Member &m = p1.m[i];
      m.tiles = static_cast<const uint4 *>(layers[i].right_tiles);
      m.rows = layers[i].rank;
      m.wc = repack_chunks(layers[i].in_features);
      m.row_tiles = rt[i];
      m.k_stages = ks[i];
      m.splits = plan.splits[i];
      m.stages_per_split = plan.sps[i];
      m.cta_begin = cta;
      m.k_valid = layers[i].in_features;
      m.pre = layers[i].scale_pre;
      m.out_offset = offset;
      cta += rt[i] * plan.splits[i];
      offset += layers[i].rank;
    }
    p1.count = count;
    p1.x = x;
    p1.x_dtype = x_dtype;
    p1.scale_dtype = layers[0].scale_dtype;
    p1.n = layers[0].in_features;
    p1.tokens = static_cast<int32_t>(tokens);
    p1.n_pad = n_pad;
    p1.tmem_cols = tmem_cols;
    p1.partial = partial1;
    p1.part_stride = total_rank;
    const int smem = smem_bytes(plan.sps[0], n_pad);
    NQB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(tc::tc_stage_kernel<false>), smem));
    tc::tc_stage_kernel<false><<<cta, tc::kThreads, smem, stream>>>(p1);
    NQB_CUDA(cudaGetLastError(), "tc stage 1 launch");
  }

  // ---- stage 2: y = post * U x latent (+ salient, overlay, bias)
  {
    tc::Params p2;
    std::memset(&p2, 0, sizeof(p2));
    int32_t rt[kMaxMembersTc], ks[kMaxMembersTc];
    for (int i = 0; i < count; ++i) {
      rt[i] = static_cast<int32_t>((layers[i].out_features + tc::kTileRows - 1) / tc::kTileRows);
      ks[i] = repack_chunks(layers[i].rank) / 2;
    }
    const Plan plan = plan_stage(rt, ks, count, false, sms);
    int32_t cta = 0, max_sps = 1;
    int64_t out_offset = 0, act_offset = 0, counter_offset = 0;
    for (int i = 0; i < count; ++i) {
      const nqb_linear_desc &d = layers[i];
      tc::Member &m = p2.m[i];
      m.tiles = static_cast<const uint4 *>(d.left_tiles);
      m.rows = d.out_features;
      m.wc = repack_chunks(d.rank);
      m.row_tiles = rt[i];
      m.k_stages = ks[i];
      m.splits = plan.splits[i];
      m.stages_per_split = plan.sps[i];
      m.cta_begin = cta;
      m.k_valid = d.rank;
      m.mid = d.scale_mid;
      m.act_offset = act_offset;
      m.out_offset = out_offset;
      m.post = d.scale_post;
      m.bias = d.bias;
      m.bias_dtype = d.bias_dtype;
      m.outlier_count = d.outlier_count;
      m.outlier_indices = d.outlier_indices;
      m.outlier_values = d.outlier_values;
      m.outlier_value_dtype = d.outlier_value_dtype;
      m.outlier_scales = d.outlier_scales;
      m.overlay_rows = d.overlay_rows;
      m.overlay_row_ids = d.overlay_row_ids;
      m.overlay_values = d.overlay_values;
      m.overlay_scales = d.overlay_scales;
      m.overlay_scale_dtype = d.overlay_scale_dtype;
      m.y = ys[i];
      m.counters = counters + counter_offset;
      cta += rt[i] * plan.splits[i];
      out_offset += d.out_features;
      act_offset += d.rank;
      counter_offset += rt[i];
      if (plan.sps[i] > max_sps) max_sps = plan.sps[i];
    }
    p2.count = count;
    p2.x = x;
    p2.x_dtype = x_dtype;
    p2.scale_dtype = layers[0].scale_dtype;
    p2.n = layers[0].in_features;
    p2.tokens = static_cast<int32_t>(tokens);
    p2.n_pad = n_pad;
    p2.tmem_cols = tmem_cols;
    p2.partial = partial2;
    p2.part_stride = total_out;
    p2.act_partial = partial1;
    p2.act_splits = p1.m[0].splits;
    p2.act_stride = total_rank;
    NQB_CUDA(cudaMemsetAsync(counters, 0, sizes.counters, stream), "counter reset");
    const int smem = smem_bytes(max_sps, n_pad);
    NQB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(tc::tc_stage_kernel<true>), smem));
    tc::tc_stage_kernel<true><<<cta, tc::kThreads, smem, stream>>>(p2);
    NQB_CUDA(cudaGetLastError(), "tc stage 2 launch");
  }
  return NQB_OK;
}

int tc_device_error(int32_t *out) {
  int value = 0;
  NQB_CUDA(cudaMemcpyFromSymbol(&value, tc::g_tc_error, sizeof(int)), "read tc error flag");
  *out = value;
  const int zero = 0;
  NQB_CUDA(cudaMemcpyToSymbol(tc::g_tc_error, &zero, sizeof(int)), "clear tc error flag");
  return NQB_OK;
}

}  // namespace nqb
