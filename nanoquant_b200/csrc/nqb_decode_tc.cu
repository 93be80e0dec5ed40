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
// 16-byte chunks are contiguous, so one CTA's K-slice is one contiguous block
// that bulk copies (cp.async.bulk) bring into shared memory.
//
// Kernels are launched with programmatic dependent launch: everything that
// does not read the previous kernel's output (mbarrier set-up, the bulk copies
// of the sign tiles, TMEM allocation, clearing the B image) runs before
// griddepcontrol.wait, overlapping the previous kernel's tail.
//
// Integer accumulation is exact, so the only rounding is the 22-bit
// quantisation of the activations and the final conversion to fp32; results
// are deterministic.  Each stage writes per-K-split fp32 partials; the last
// CTA of every row tile (atomic counter) reduces them in a fixed order:
// stage 1 into the latent (times scale_mid), stage 2 into y (times
// scale_post, plus salient columns, the int8 row overlay, the low-rank patch
// and bias).  A patched layer's patch latent R x is formed in stage 1 by the
// member's CTAs (patch rows spread over them, while their MMAs run) and
// stage 2's reducing CTA adds L times it per row.
#include <cstring>

#include "nqb_decode_tc.cuh"
#include "nqb_tc_decode.cuh"
#include "nqb_tc_ptx.cuh"

namespace nqb {
namespace tc {

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
  const void *pre;       // stage 1: activation scale
  const void *mid;       // stage 1: latent scale, applied by the reducing CTA
  int64_t act_offset;    // stage 2: first latent column of this member
  int64_t out_offset;    // first row of this member in the partial / latent buffers
  int32_t *counters;     // [row_tiles], zero on entry, left zero
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
  // low-rank patch: stage 1 reads R [p, n], stage 2 L [m, p]
  int64_t patch_rank;
  const void *patch_factor;
  int32_t patch_dtype;
  float *patch_latent;   // [tokens][patch_rank]: written by stage 1, read by stage 2
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
  float *partial;      // this stage's K-split partials [splits][tokens][part_stride]
  int64_t part_stride;
  float *latent;       // [tokens][latent_stride]: written by stage 1, read by stage 2
  int64_t latent_stride;
};

__device__ int g_tc_error;  // first bounded-wait failure (0 = none), for diagnostics

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_tc_error, 0, code); }

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <bool kStage2>
__device__ __forceinline__ void stage_activations(const Params &p, const Member &m, int64_t k0, int ncols,
                                                  float *out) {
  if constexpr (kStage2) {
    stage_latent_slice(p.latent, p.latent_stride, m.act_offset, k0, ncols, p.tokens, m.k_valid, out);
  } else {
    stage_x_slice(p.x, p.x_dtype, m.pre, p.scale_dtype, p.n, k0, ncols, p.tokens, m.k_valid, out);
  }
}

// Patch latent rows q = first, first + step, ... of member m (whole CTA):
// patch_latent[t][q] = sum_i x[t, i] R[q, i], fp32, fixed summation order.
// (Plain arguments: a reference to the kernel's parameters would make the
// kernel copy them to local memory.)
template <int kT>
__device__ __noinline__ void patch_latent_rows(const void *x, int32_t x_dtype, int64_t n, int T, int64_t rows,
                                               const void *factor, int32_t dtype, float *out, int64_t first,
                                               int64_t step, float *s_part) {
  constexpr int kW = kThreads / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int64_t q = first; q < rows; q += step) {
    float part[kT];
#pragma unroll
    for (int t = 0; t < kT; ++t) part[t] = 0.0f;
    for (int64_t i = tid; i < n; i += kThreads) {
      const float r = load_as_float(factor, q * n + i, dtype);
#pragma unroll
      for (int t = 0; t < kT; ++t)
        if (t < T) part[t] += load_as_float(x, static_cast<int64_t>(t) * n + i, x_dtype) * r;
    }
#pragma unroll
    for (int t = 0; t < kT; ++t) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part[t] += __shfl_xor_sync(0xffffffffu, part[t], off);
      if (lane == 0) s_part[warp * kT + t] = part[t];
    }
    __syncthreads();
    if (tid < T) {
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kW; ++w) v += s_part[w * kT + tid];
      out[static_cast<int64_t>(tid) * rows + q] = v;
    }
    __syncthreads();
  }
}

// kPatch: some member has a low-rank patch; calls without one run an instance
// with the patch steps compiled out.
template <bool kStage2, int kT, bool kPatch>
__global__ void __launch_bounds__(kThreads, 1) tc_stage_kernel(const Params p) {
  constexpr int kNP = n_pad_for(kT);  // MMA N: 3 digit columns per token, multiple of 16
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t s_bar_a[2];                    // A buffer b free again
  __shared__ uint64_t s_bar_done;                    // all MMAs complete
  __shared__ uint64_t s_bar_w[kMaxStagesPerCta];     // stage weights landed
  __shared__ uint32_t s_tmem;
  __shared__ BImageScratch<kT> s_bi;
  __shared__ float s_red_f[4];
  __shared__ float s_patch[(kThreads / 32) * kT];
  __shared__ int s_last;

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
  constexpr int NP = kNP;
  const uint32_t b_block = 32u * NP;  // bytes of one (stage, class, half) B block

  uint8_t *smem_w = smem;                                   // nst * 4 KB weights
  uint8_t *smem_b = smem + nst * kStageWeightBytes;         // nst * 8 * b_block digits

  // ---- prologue: nothing here reads the previous kernel's output ----------
  if (tid == 0) {
    ptx::mbar_init(&s_bar_a[0], 1);
    ptx::mbar_init(&s_bar_a[1], 1);
    ptx::mbar_init(&s_bar_done, 1);
    for (int s = 0; s < nst; ++s) ptx::mbar_init(&s_bar_w[s], 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    // stream this CTA's sign words: one bulk copy per 256-column stage
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
  if (warp == 0) {
    ptx::tmem_alloc(&s_tmem, p.tmem_cols);
    ptx::tmem_relinquish();
  }
  {
    uint4 *b4 = reinterpret_cast<uint4 *>(smem_b);
    const int count = nst * 8 * static_cast<int>(b_block) / 16;
    for (int i = tid; i < count; i += kThreads) b4[i] = make_uint4(0, 0, 0, 0);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = s_tmem;
  allow_dependent_launch();
  grid_dependency_wait();

  // ---- quantise this K slice of the activations into the B image ---------
  const int64_t k0 = static_cast<int64_t>(st_begin) * kStageCols;
  {
    float *s_act = reinterpret_cast<float *>(smem_b + nst * 8 * b_block);  // [T][ncols] fp32
    stage_activations<kStage2>(p, m, k0, nst * kStageCols, s_act);
    __syncthreads();
    build_b_image<kT>(s_act, nst, T, smem_b, b_block, s_bi);
  }

  // ---- main loop: bits -> TMEM (A), one tcgen05.mma per (class, half) per stage
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t idesc = ptx::idesc_i8_m128(static_cast<uint32_t>(NP));
  const uint32_t b_base = ptx::smem_u32(smem_b);
  bool ok = true;
  for (int sl = 0; sl < nst; ++sl) {
    const int buf = sl & 1;
    if (!ptx::mbar_wait_bounded(&s_bar_w[sl], 0, kSpinLimit)) ok = false;
    const uint4 *wsrc = reinterpret_cast<const uint4 *>(smem_w + sl * kStageWeightBytes);
    uint32_t a[kAStageCols];
    expand_slice(wsrc[tid], wsrc[kTileRows + tid], a);
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
      issue_slice_mmas(tmem, buf, sl, b_base, b_block, idesc, NP, sl == 0);
      ptx::mma_commit(&s_bar_a[buf]);
    }
  }
  if (tid == 0) ptx::mma_commit(&s_bar_done);
  if constexpr (!kStage2 && kPatch) {
    // this CTA's share of the patch latent while the tensor cores finish
    if (m.patch_rank > 0)
      patch_latent_rows<kT>(p.x, p.x_dtype, p.n, T, m.patch_rank, m.patch_factor, m.patch_dtype, m.patch_latent, local,
                            static_cast<int64_t>(m.row_tiles) * m.splits, s_patch);
  }
  if (!ptx::mbar_wait_bounded(&s_bar_done, 0, kSpinLimit)) ok = false;
  ptx::tc_fence_after();
  if (!ok) record_error(NQB_ERR_TIMEOUT);

  // ---- epilogue: combine classes and digits, write fp32 partials ---------
  const int64_t row = static_cast<int64_t>(tile) * kTileRows + tid;
  {
    int32_t sacc[kNP];
    drain_accumulators<kNP>(tmem, lane_base, sacc);
    if (row < m.rows) {
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        if (t < T)
          p.partial[(static_cast<int64_t>(split) * T + t) * p.part_stride + m.out_offset + row] =
              token_value<kNP>(sacc, t, s_bi.qsum[t], s_bi.exp[t]);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, p.tmem_cols);

  // ---- the last CTA of this row tile reduces the K-split partials --------
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int previous = atomicAdd(m.counters + tile, 1);
    s_last = (previous == m.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if constexpr (!kStage2) {
    if (row < m.rows) {
      const float mid = load_as_float(m.mid, row, p.scale_dtype);
      for (int t = 0; t < T; ++t) {
        float acc = 0.0f;
        for (int s = 0; s < m.splits; ++s)
          acc += __ldcg(p.partial + (static_cast<int64_t>(s) * T + t) * p.part_stride + m.out_offset + row);
        p.latent[static_cast<int64_t>(t) * p.latent_stride + m.out_offset + row] = acc * mid;
      }
    }
  } else {
    if (row < m.rows) {
      const float post = load_as_float(m.post, row, p.scale_dtype);
      const float bias = m.bias != nullptr ? load_as_float(m.bias, row, m.bias_dtype) : 0.0f;
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
        if constexpr (kPatch) {
          if (m.patch_rank > 0) {
            float pv = 0.0f;
            for (int64_t q = 0; q < m.patch_rank; ++q)
              pv += load_as_float(m.patch_factor, row * m.patch_rank + q, m.patch_dtype) *
                    __ldcg(m.patch_latent + static_cast<int64_t>(t) * m.patch_rank + q);
            v += pv;
          }
        }
        m.y[static_cast<int64_t>(t) * m.rows + row] = v + bias;
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
          if (lane == 0) s_red_f[warp] = part;
          __syncthreads();
          if (tid == 0) {
            const float dot = (s_red_f[0] + s_red_f[1]) + (s_red_f[2] + s_red_f[3]);
            m.y[static_cast<int64_t>(t) * m.rows + orow] += dot * scale;
          }
          __syncthreads();
        }
      }
    }
  }
  if (tid == 0) m.counters[tile] = 0;  // zero again for the next call
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
// Largest K slice (in 256-column stages) per CTA for `tokens` tokens: keeps the
// staged activations (tokens x slice fp32) and the B image within ~64 KB.
static int max_stages_for(int64_t tokens) { return tokens <= 4 ? kMaxStagesPerCta : (tokens <= 8 ? 4 : 2); }

static Plan plan_stage(const int32_t *row_tiles, const int32_t *k_stages, int count, bool uniform, int sms,
                       int max_sps) {
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
    if (sps > max_sps) sps = max_sps;
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
  int64_t tiles = 0;
  for (int i = 0; i < count; ++i)
    tiles += (layers[i].rank + tc::kTileRows - 1) / tc::kTileRows +
             (layers[i].out_features + tc::kTileRows - 1) / tc::kTileRows;
  if (tiles > kMaxCounters) return false;
  for (int i = 0; i < count; ++i) {
    if (layers[i].right_tiles == nullptr || layers[i].left_tiles == nullptr) return false;
    if (reinterpret_cast<uintptr_t>(layers[i].right_tiles) % 16 || reinterpret_cast<uintptr_t>(layers[i].left_tiles) % 16)
      return false;
  }
  return true;
}

struct Layout {
  Plan s1, s2;
  int32_t rt1[kMaxMembersTc], ks1[kMaxMembersTc], rt2[kMaxMembersTc], ks2[kMaxMembersTc];
  int64_t total_rank, total_out;
  int64_t counters;                     // completion counters used (row tiles of both stages)
  size_t partial1, partial2;            // section sizes (256-aligned)
};

static Layout tc_layout(const nqb_linear_desc *layers, int count, int64_t tokens) {
  const int sms = sm_count();
  Layout l{};
  int64_t counters = 0;
  int32_t max_s2 = 0;
  for (int i = 0; i < count; ++i) {
    l.rt1[i] = static_cast<int32_t>((layers[i].rank + tc::kTileRows - 1) / tc::kTileRows);
    l.ks1[i] = repack_chunks(layers[i].in_features) / 2;
    l.rt2[i] = static_cast<int32_t>((layers[i].out_features + tc::kTileRows - 1) / tc::kTileRows);
    l.ks2[i] = repack_chunks(layers[i].rank) / 2;
    l.total_rank += layers[i].rank;
    l.total_out += layers[i].out_features;
    counters += l.rt1[i] + l.rt2[i];
  }
  l.s1 = plan_stage(l.rt1, l.ks1, count, true, sms, max_stages_for(tokens));
  l.s2 = plan_stage(l.rt2, l.ks2, count, false, sms, max_stages_for(tokens));
  for (int i = 0; i < count; ++i) max_s2 = l.s2.splits[i] > max_s2 ? l.s2.splits[i] : max_s2;
  l.counters = counters;
  l.partial1 = align_up(static_cast<size_t>(l.s1.splits[0]) * tokens * l.total_rank * sizeof(float), 256);
  l.partial2 = align_up(static_cast<size_t>(max_s2) * tokens * l.total_out * sizeof(float), 256);
  return l;
}

size_t tc_extra_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  if (!tc_eligible(layers, count, NQB_F32, tokens)) return 0;
  const Layout l = tc_layout(layers, count, tokens);
  return l.partial1 + l.partial2;
}

// Dynamic shared memory of one CTA: sign tiles, B image, staged activations.
static int smem_bytes(int stages, int n_pad, int64_t tokens) {
  return stages * tc::kStageWeightBytes + stages * 8 * 32 * n_pad +
         static_cast<int>(tokens) * stages * tc::kStageCols * static_cast<int>(sizeof(float));
}

template <bool kStage2, int kT, bool kPatch>
static int launch_stage_t(const tc::Params &params, int ctas, int smem, cudaStream_t stream) {
  const void *fn = reinterpret_cast<const void *>(tc::tc_stage_kernel<kStage2, kT, kPatch>);
  NQB_CHECK(ensure_dynamic_smem(fn, smem));
  cudaLaunchConfig_t config;
  std::memset(&config, 0, sizeof(config));
  config.gridDim = dim3(ctas);
  config.blockDim = dim3(tc::kThreads);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  NQB_CUDA(cudaLaunchKernelEx(&config, tc::tc_stage_kernel<kStage2, kT, kPatch>, params),
           kStage2 ? "tc stage 2 launch" : "tc stage 1 launch");
  return NQB_OK;
}

// Token buckets: each kernel instance is compiled for at most kT tokens.
static int token_bucket(int64_t tokens) { return tokens <= 1 ? 1 : tokens <= 2 ? 2 : tokens <= 4 ? 4 : tokens <= 8 ? 8 : 16; }

template <bool kStage2, bool kPatch>
static int launch_stage_p(const tc::Params &params, int ctas, int smem, cudaStream_t stream) {
  switch (token_bucket(params.tokens)) {
    case 1: return launch_stage_t<kStage2, 1, kPatch>(params, ctas, smem, stream);
    case 2: return launch_stage_t<kStage2, 2, kPatch>(params, ctas, smem, stream);
    case 4: return launch_stage_t<kStage2, 4, kPatch>(params, ctas, smem, stream);
    case 8: return launch_stage_t<kStage2, 8, kPatch>(params, ctas, smem, stream);
    default: return launch_stage_t<kStage2, 16, kPatch>(params, ctas, smem, stream);
  }
}

template <bool kStage2>
static int launch_stage(const tc::Params &params, int ctas, int smem, bool patch, cudaStream_t stream) {
  return patch ? launch_stage_p<kStage2, true>(params, ctas, smem, stream)
               : launch_stage_p<kStage2, false>(params, ctas, smem, stream);
}

int run_tc(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
           float *const *ys, int32_t *counters, void *extra, size_t extra_bytes, float *latent, float *patch,
           cudaStream_t stream) {
  const Layout l = tc_layout(layers, count, tokens);
  if (extra_bytes < l.partial1 + l.partial2) return fail(NQB_ERR_WORKSPACE, "tensor-core path workspace too small");
  char *ws = static_cast<char *>(extra);
  float *partial1 = reinterpret_cast<float *>(ws);
  float *partial2 = reinterpret_cast<float *>(ws + l.partial1);
  const int32_t n_pad = tc::n_pad_for(token_bucket(tokens));
  const uint32_t tmem_cols = (tc::kDCol + tc::kClasses * n_pad) <= 256 ? 256u : 512u;

  tc::Params p1;
  std::memset(&p1, 0, sizeof(p1));
  tc::Params p2;
  std::memset(&p2, 0, sizeof(p2));
  int32_t cta1 = 0, cta2 = 0, max_sps2 = 1;
  int64_t rank_offset = 0, out_offset = 0, counter_offset = 0, patch_offset = 0;
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    tc::Member &a = p1.m[i];
    a.tiles = static_cast<const uint4 *>(d.right_tiles);
    a.rows = d.rank;
    a.wc = repack_chunks(d.in_features);
    a.row_tiles = l.rt1[i];
    a.k_stages = l.ks1[i];
    a.splits = l.s1.splits[i];
    a.stages_per_split = l.s1.sps[i];
    a.cta_begin = cta1;
    a.k_valid = d.in_features;
    a.pre = d.scale_pre;
    a.mid = d.scale_mid;
    a.out_offset = rank_offset;
    a.counters = counters + counter_offset;
    cta1 += l.rt1[i] * a.splits;
    counter_offset += l.rt1[i];

    tc::Member &b = p2.m[i];
    b.tiles = static_cast<const uint4 *>(d.left_tiles);
    b.rows = d.out_features;
    b.wc = repack_chunks(d.rank);
    b.row_tiles = l.rt2[i];
    b.k_stages = l.ks2[i];
    b.splits = l.s2.splits[i];
    b.stages_per_split = l.s2.sps[i];
    b.cta_begin = cta2;
    b.k_valid = d.rank;
    b.act_offset = rank_offset;
    b.out_offset = out_offset;
    b.counters = counters + counter_offset;
    b.post = d.scale_post;
    b.bias = d.bias;
    b.bias_dtype = d.bias_dtype;
    b.outlier_count = d.outlier_count;
    b.outlier_indices = d.outlier_indices;
    b.outlier_values = d.outlier_values;
    b.outlier_value_dtype = d.outlier_value_dtype;
    b.outlier_scales = d.outlier_scales;
    b.overlay_rows = d.overlay_rows;
    b.overlay_row_ids = d.overlay_row_ids;
    b.overlay_values = d.overlay_values;
    b.overlay_scales = d.overlay_scales;
    b.overlay_scale_dtype = d.overlay_scale_dtype;
    b.y = ys[i];
    if (d.patch_rank > 0) {
      float *pl = patch + tokens * patch_offset;
      a.patch_rank = b.patch_rank = d.patch_rank;
      a.patch_dtype = b.patch_dtype = d.patch_dtype;
      a.patch_factor = d.patch_right;
      b.patch_factor = d.patch_left;
      a.patch_latent = b.patch_latent = pl;
      patch_offset += d.patch_rank;
    }
    cta2 += l.rt2[i] * b.splits;
    counter_offset += l.rt2[i];
    if (b.stages_per_split > max_sps2) max_sps2 = b.stages_per_split;
    rank_offset += d.rank;
    out_offset += d.out_features;
  }
  for (tc::Params *p : {&p1, &p2}) {
    p->count = count;
    p->x = x;
    p->x_dtype = x_dtype;
    p->scale_dtype = layers[0].scale_dtype;
    p->n = layers[0].in_features;
    p->tokens = static_cast<int32_t>(tokens);
    p->n_pad = n_pad;
    p->tmem_cols = tmem_cols;
    p->latent = latent;
    p->latent_stride = l.total_rank;
  }
  p1.partial = partial1;
  p1.part_stride = l.total_rank;
  p2.partial = partial2;
  p2.part_stride = l.total_out;

  const bool patched = patch_offset > 0;
  NQB_CHECK(launch_stage<false>(p1, cta1, smem_bytes(l.s1.sps[0], n_pad, tokens), patched, stream));
  NQB_CHECK(launch_stage<true>(p2, cta2, smem_bytes(max_sps2, n_pad, tokens), patched, stream));
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
