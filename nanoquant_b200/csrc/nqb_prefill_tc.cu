// Tensor-core (tcgen05) prefill path of libnqb: more than 16 tokens.
//
// Stage 1 computes latent[t, k] = mid[k] * sum_i sign(V[k, i]) * (x * pre)[t, i]
// and stage 2 y[t, o] = post[o] * sum_k sign(U[o, k]) * latent[t, k] + extras;
// both are GEMMs D[rows x tokens] = S[rows x K] * A[tokens x K]^T with a
// +/-1 matrix S.  Here they run as fp16 tcgen05.mma (kind::f16, fp32
// accumulate, M = 128, N = 128 tokens, K = 16 per instruction):
//
// * The signs are the A operand and live in tensor memory.  Each of 128
//   threads owns one row (its TMEM lane) and turns a 32-bit sign word into 16
//   TMEM columns of fp16 pairs with one shift and one LOP3 per pair:
//       ((w << (15 - j)) & 0x80008000) | 0x3C003C00      (j = 0..15)
//   i.e. the pair (+/-1 for bit j, +/-1 for bit j+16).  The expanded signs
//   never touch shared memory.
// * The activations are the B operand: a pre-pass scales each token's row by
//   a power of two (max |a| * 2^e < 2^15, exact), converts it to fp16 and
//   stores it with the same pair order (position 2j <- column j, 2j+1 <-
//   column j+16 of every 32-column group); TMA (128-byte swizzle) brings
//   128-token x 64-column boxes into shared memory.
// * One CTA owns one 128-row sign tile and one 256-token tile (MMA
//   128 x 256 x 16); the K loop (128 columns per step) is pipelined over 3
//   shared-memory stages of 64 KB: warp 4 issues TMA and the sign-chunk bulk
//   copy, warps 0-3 expand signs into a double-buffered A region of TMEM, one
//   thread of warp 5 issues the 8 MMAs of a step and commits them to the
//   stage's "empty" barriers.  The 128 x 256 fp32 accumulator stays in TMEM
//   until the epilogue multiplies by 2^-e and the row scale and writes fp32.
// Every mbarrier wait is bounded; a timeout sets the device status word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "nqb_decode_tc.cuh"
#include "nqb_prefill_tc.cuh"
#include "nqb_tc_ptx.cuh"

namespace nqb {
namespace pf {

constexpr int kTileRows = 128;     // sign rows per CTA (MMA M)
constexpr int kTokTile = 256;      // tokens per CTA (MMA N)
constexpr int kKStep = 128;        // K columns per pipeline step = one 4-word sign chunk
constexpr int kStages = 3;
constexpr int kAtomBytes = kTokTile * 128;             // 256 tokens x 64 fp16 (one 128-byte swizzle column)
constexpr int kBStageBytes = 2 * kAtomBytes;           // 128 K columns
constexpr int kChunkBytes = kTileRows * 16;            // one 4-word chunk of a 128-row tile
constexpr int kStageBytes = kBStageBytes + kChunkBytes;
constexpr int kACols = kKStep / 2;                     // TMEM columns of A per step
constexpr int kDCol = 2 * kACols;                      // accumulator after 2 buffers of A
constexpr uint32_t kTmemCols = 512;
constexpr int kThreads = 192;
constexpr uint32_t kSpinLimit = 1u << 28;
constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // +1024 for the swizzle alignment

struct Member {
  const uint4 *tiles;   // row-interleaved sign tiles (nqb_repack_signs)
  int64_t rows;
  int32_t wc;           // 4-word chunks per row
  int32_t row_tiles;
  int32_t cta_begin;    // first blockIdx.x of this member (one CTA per row tile)
  int32_t k_steps;      // K steps of 128 columns
  const void *row_scale;  // mid (stage 1) / post (stage 2)
  const int32_t *exps;    // per-token exponent e of the fp16 activations
  float *out;
  int64_t out_stride;
  int64_t out_offset;
  // stage 2 extras
  const void *bias;
  int32_t bias_dtype;
  int64_t outlier_count;
  const int32_t *outlier_indices;
  const void *outlier_values;
  int32_t outlier_value_dtype;
  const void *outlier_scales;
  int32_t tma_store;  // 1: write the tile with one TMA store through shared memory
};

struct Params {
  Member m[kMaxMembersTc];
  int32_t count;
  int64_t tokens;
  int32_t scale_dtype;
  const void *x;  // original input (stage-2 salient columns)
  int32_t x_dtype;
  int64_t n;
};

__device__ int g_pf_error;

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;              // LBO (unused for 128-byte swizzle K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;      // SBO: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;              // sm_100 descriptor version
  d |= static_cast<uint64_t>(2) << 61;              // SWIZZLE_128B
  return d;
}

__host__ __device__ constexpr uint32_t idesc_f16_m128(uint32_t n) {
  return (1u << 4)                // D: f32
         | (0u << 7) | (0u << 10)  // A, B: f16
         | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int32_t x, int32_t y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ptx::smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ptx::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ float exp2_int(int e) { return __int_as_float((e + 127) << 23); }

// Expands the four sign words of one row for one K step into 64 TMEM
// columns (fp16 pairs) of this thread's lane.
__device__ __forceinline__ void expand_and_store(uint4 chunk, uint32_t taddr) {
  const uint32_t words[4] = {chunk.x, chunk.y, chunk.z, chunk.w};
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t v[32];
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
      const uint32_t w = words[half * 2 + wi];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[wi * 16 + j] = ((w << (15 - j)) & 0x80008000u) | 0x3C003C00u;
    }
    ptx::tmem_st16(taddr + half * 32, v);
    ptx::tmem_st16(taddr + half * 32 + 16, v + 16);
  }
}

template <bool kStage2>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map0,
                        const __grid_constant__ CUtensorMap map1, const __grid_constant__ CUtensorMap map2,
                        const __grid_constant__ CUtensorMap out0, const __grid_constant__ CUtensorMap out1,
                        const __grid_constant__ CUtensorMap out2) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], a_full[2], a_empty[2], d_full;
  __shared__ uint32_t s_tmem;
  __shared__ float s_unscale[kTokTile];  // 2^-e of each token of the tile (0 past the last token)

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  int g = 0;
  for (int i = 1; i < p.count; ++i)
    if (static_cast<int32_t>(blockIdx.x) >= p.m[i].cta_begin) g = i;
  const Member &m = p.m[g];
  const CUtensorMap *map = g == 0 ? &map0 : (g == 1 ? &map1 : &map2);
  const CUtensorMap *out_map = g == 0 ? &out0 : (g == 1 ? &out1 : &out2);
  const int tile0 = static_cast<int>(blockIdx.x) - m.cta_begin;
  const int tok0 = static_cast<int>(blockIdx.y) * kTokTile;
  const int K = m.k_steps;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&a_full[b], 128);
      ptx::mbar_init(&a_empty[b], 1);
    }
    ptx::mbar_init(&d_full, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&s_tmem, kTmemCols);
    ptx::tmem_relinquish();
  }
  for (int i = tid; i < kTokTile; i += kThreads) {
    const int64_t tok = tok0 + i;
    s_unscale[i] = tok < p.tokens ? exp2_int(-m.exps[tok]) : 0.0f;
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = s_tmem;
  bool ok = true;

  if (warp == 4) {
    if (lane == 0) {  // producer
      const uint32_t bytes = kStageBytes;
      for (int s = 0; s < K; ++s) {
        const int slot = s % kStages;
        if (s >= kStages && !ptx::mbar_wait_bounded(&empty[slot], ((s / kStages) - 1) & 1, kSpinLimit)) ok = false;
        const uint32_t base = ptx::smem_u32(smem + slot * kStageBytes);
        const uint32_t bar = ptx::smem_u32(&full[slot]);
        expect_tx(&full[slot], bytes);
        tma_load_2d(base, map, s * kKStep, tok0, bar);
        tma_load_2d(base + kAtomBytes, map, s * kKStep + 64, tok0, bar);
        const uint8_t *src =
            reinterpret_cast<const uint8_t *>(m.tiles) + (static_cast<size_t>(tile0) * m.wc + s) * kChunkBytes;
        bulk_load(base + kBStageBytes, src, kChunkBytes, bar);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = idesc_f16_m128(kTokTile);
      for (int s = 0; s < K; ++s) {
        const int slot = s % kStages;
        const int buf = s & 1;
        if (!ptx::mbar_wait_bounded(&full[slot], (s / kStages) & 1, kSpinLimit)) ok = false;
        if (!ptx::mbar_wait_bounded(&a_full[buf], (s >> 1) & 1, kSpinLimit)) ok = false;
        ptx::tc_fence_after();
        const uint32_t bbase = ptx::smem_u32(smem + slot * kStageBytes);
#pragma unroll
        for (int k16 = 0; k16 < kKStep / 16; ++k16) {
          const uint64_t bdesc = desc_sw128(bbase + (k16 >> 2) * kAtomBytes + (k16 & 3) * 32);
          mma_f16_ts(tmem + kDCol, tmem + buf * kACols + k16 * 8, bdesc, idesc, (s > 0 || k16 > 0) ? 1u : 0u);
        }
        ptx::mma_commit(&empty[slot]);
        ptx::mma_commit(&a_empty[buf]);
      }
      ptx::mma_commit(&d_full);
    }
  } else {  // warps 0-3: sign expansion, then the epilogue
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    for (int s = 0; s < K; ++s) {
      const int slot = s % kStages;
      const int buf = s & 1;
      if (!ptx::mbar_wait_bounded(&full[slot], (s / kStages) & 1, kSpinLimit)) ok = false;
      const uint4 *chunks = reinterpret_cast<const uint4 *>(smem + slot * kStageBytes + kBStageBytes);
      const uint4 c0 = chunks[tid];
      if (s >= 2) {
        if (!ptx::mbar_wait_bounded(&a_empty[buf], ((s >> 1) - 1) & 1, kSpinLimit)) ok = false;
        ptx::tc_fence_after();
      }
      expand_and_store(c0, tmem + lane_base + buf * kACols);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      mbar_arrive(&a_full[buf]);
    }
    if (!ptx::mbar_wait_bounded(&d_full, 0, kSpinLimit)) ok = false;
    ptx::tc_fence_after();
    // Epilogue.  Every value an output needs besides the accumulator is read
    // from shared memory or registers: a global load between the global
    // stores would be ordered behind them (possible aliasing) and serialise.
    const int64_t row = static_cast<int64_t>(tile0) * kTileRows + tid;
    const bool live = row < m.rows;
    const float rscale = live ? load_as_float(m.row_scale, row, p.scale_dtype) : 0.0f;
    float bias = 0.0f;
    // stage 2 salient columns: x[tok0 + t][idx_s] staged (fp32) into the now idle
    // pipeline buffers by the epilogue warps; this row's weights into registers
    constexpr int kMaxStagedSalient = 64;  // 64 KB of the idle pipeline buffers
    float *s_xs = reinterpret_cast<float *>(smem);
    float *s_out = reinterpret_cast<float *>(smem + kMaxStagedSalient * kTokTile * 4);  // [token][row], 128 KB
    int64_t staged = 0;
    if constexpr (kStage2) {
      if (live && m.bias != nullptr) bias = load_as_float(m.bias, row, m.bias_dtype);
      staged = m.outlier_count <= kMaxStagedSalient ? m.outlier_count : 0;
      for (int64_t i = tid; i < staged * kTokTile; i += kTileRows) {
        const int64_t t = i / staged, sidx = i - t * staged;
        const int64_t tok = tok0 + t;
        s_xs[i] = tok < p.tokens ? load_as_float(p.x, tok * p.n + m.outlier_indices[sidx], p.x_dtype) : 0.0f;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps only
    }
#pragma unroll 1
    for (int c = 0; c < kTokTile / 16; ++c) {
      uint32_t v[16];
      ptx::tmem_ld16(tmem + lane_base + kDCol + c * 16, v);
      ptx::tmem_wait_ld();
      float out[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) out[e] = __uint_as_float(v[e]) * s_unscale[c * 16 + e] * rscale + bias;
      if constexpr (kStage2) {
        if (live && m.outlier_count > 0) {
          for (int64_t sidx = 0; sidx < m.outlier_count; ++sidx) {
            float w = load_as_float(m.outlier_values, row * m.outlier_count + sidx, m.outlier_value_dtype);
            if (m.outlier_scales != nullptr) w *= load_as_float(m.outlier_scales, sidx, p.scale_dtype);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int t = c * 16 + e;
              const int64_t tok = tok0 + t;
              const float xv = sidx < staged ? s_xs[t * staged + sidx]
                                             : (tok < p.tokens ? load_as_float(p.x, tok * p.n + m.outlier_indices[sidx],
                                                                               p.x_dtype)
                                                               : 0.0f);
              out[e] += xv * w;
            }
          }
        }
      }
      if (m.tma_store) {
#pragma unroll
        for (int e = 0; e < 16; ++e) s_out[(c * 16 + e) * kTileRows + tid] = out[e];
        continue;
      }
      if (!live) continue;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int64_t tok = tok0 + c * 16 + e;
        if (tok < p.tokens) m.out[tok * m.out_stride + m.out_offset + row] = out[e];
      }
    }
    if (m.tma_store) {
      // The member's map starts at its first output column; rows past the
      // member and tokens past `tokens` are clipped by the TMA unit.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tid == 0) tma_store_2d(out_map, tile0 * kTileRows, tok0, ptx::smem_u32(s_out));
    }
  }
  if (!ok) atomicCAS(&g_pf_error, 0, NQB_ERR_TIMEOUT);
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, kTmemCols);
}

// Pre-pass: per token, scale the activation row of one member by 2^e
// (max |a| * 2^e < 2^15), convert to fp16 in pair order, record e.
// Stage 1 reads x * pre, stage 2 the fp32 latent.
template <bool kLatent>
__global__ void __launch_bounds__(256) quantise_kernel(const void *x, int32_t x_dtype, int64_t n, const void *pre,
                                                       int32_t scale_dtype, const float *latent, int64_t latent_stride,
                                                       int64_t latent_offset, int64_t k_valid, int64_t k_pad,
                                                       __half *out, int32_t *exps) {
  __shared__ float s_max[8];
  const int64_t t = blockIdx.x;
  auto value = [&](int64_t col) -> float {
    if (col >= k_valid) return 0.0f;
    if constexpr (kLatent) {
      return latent[t * latent_stride + latent_offset + col];
    } else {
      return load_as_float(x, t * n + col, x_dtype) * load_as_float(pre, col, scale_dtype);
    }
  };
  float mx = 0.0f;
  for (int64_t c = threadIdx.x; c < k_valid; c += blockDim.x) mx = fmaxf(mx, fabsf(value(c)));
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = mx;
  __syncthreads();
  float v = s_max[0];
  for (int i = 1; i < 8; ++i) v = fmaxf(v, s_max[i]);
  int e = 0;
  if (v > 0.0f && isfinite(v)) {
    int ex;
    frexpf(v, &ex);
    e = min(15 - ex, 126);
  }
  const float scale = exp2_int(e);
  for (int64_t pos = threadIdx.x; pos < k_pad; pos += blockDim.x) {
    const int64_t group = pos & ~int64_t(31);
    const int64_t col = group + ((pos & 31) >> 1) + ((pos & 1) << 4);
    out[t * k_pad + pos] = __float2half_rn(value(col) * scale);
  }
  if (threadIdx.x == 0) exps[t] = e;
}

// Int8 residual rows for the prefill path: y[t, ids[j]] += s[j] * sum_i R[j, i] x[t, i].
__global__ void overlay_kernel(const void *x, int32_t x_dtype, int64_t n, int64_t tokens, const int32_t *ids,
                               const int8_t *values, const void *scales, int32_t scale_dtype, int64_t rows,
                               float *y, int64_t y_stride) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows * tokens) return;
  const int64_t j = warp / tokens, t = warp - j * tokens;
  float acc = 0.0f;
  for (int64_t i = lane; i < n; i += 32) acc += static_cast<float>(values[j * n + i]) * load_as_float(x, t * n + i, x_dtype);
  acc = warp_sum(acc);
  if (lane == 0) y[t * y_stride + ids[j]] += acc * load_as_float(scales, j, scale_dtype);
}

}  // namespace pf

// --------------------------------------------------------------- host ---

static int64_t k_pad_of(int64_t k) { return ((k + pf::kKStep - 1) / pf::kKStep) * pf::kKStep; }

bool prefill_eligible(const nqb_linear_desc *layers, int count, int32_t x_dtype, int64_t tokens) {
  if (tokens <= 16 || tokens > (1 << 22) || count < 1 || count > kMaxMembersTc || !is_float_dtype(x_dtype)) return false;
  for (int i = 0; i < count; ++i) {
    if (layers[i].right_tiles == nullptr || layers[i].left_tiles == nullptr) return false;
    if (reinterpret_cast<uintptr_t>(layers[i].right_tiles) % 16 || reinterpret_cast<uintptr_t>(layers[i].left_tiles) % 16)
      return false;
  }
  return true;
}

size_t prefill_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  if (!prefill_eligible(layers, count, NQB_F32, tokens)) return 0;
  size_t total = 0;
  for (int i = 0; i < count; ++i) {
    total += align_up(static_cast<size_t>(tokens) * k_pad_of(layers[i].in_features) * 2, 256);  // stage-1 fp16
    total += align_up(static_cast<size_t>(tokens) * k_pad_of(layers[i].rank) * 2, 256);         // stage-2 fp16
    total += 2 * align_up(static_cast<size_t>(tokens) * 4, 256);                                 // exponents
  }
  return total;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library has no link-time dependency on libcuda (it loads on CPU-only hosts).
static int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000 *out) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *sym = nullptr;
    cudaDriverEntryPointQueryResult status;
    NQB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &status),
             "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (status != cudaDriverEntryPointSuccess || sym == nullptr)
      return fail(NQB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(sym);
  }
  *out = fn;
  return NQB_OK;
}

// fp32 output [tokens][columns] with row stride `stride` floats, written as
// 128-column x 256-token boxes from shared memory (no swizzle).
static int encode_out_map(CUtensorMap *map, float *base, int64_t columns, int64_t stride, int64_t tokens) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  NQB_CHECK(tensor_map_encoder(&encode));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(columns), static_cast<cuuint64_t>(tokens)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 4};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(pf::kTileRows), static_cast<cuuint32_t>(pf::kTokTile)};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, elem,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NQB_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", static_cast<int>(r));
  return NQB_OK;
}

// The TMA store needs a 16-byte aligned base and a row stride of whole 16-byte units.
static bool tma_storable(const float *base, int64_t stride) {
  return reinterpret_cast<uintptr_t>(base) % 16 == 0 && stride % 4 == 0;
}

static int encode_map(CUtensorMap *map, const void *base, int64_t k_pad, int64_t tokens) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  NQB_CHECK(tensor_map_encoder(&encode));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_pad), static_cast<cuuint64_t>(tokens)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k_pad) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(pf::kTokTile)};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                                            strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NQB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return NQB_OK;
}

template <bool kStage2>
static int launch_gemm(const pf::Params &params, const CUtensorMap *maps, int ctas_x, int64_t tokens,
                       cudaStream_t stream) {
  const void *fn = reinterpret_cast<const void *>(pf::prefill_gemm_kernel<kStage2>);
  NQB_CHECK(ensure_dynamic_smem(fn, pf::kSmemBytes));
  const dim3 grid(ctas_x, static_cast<unsigned>((tokens + pf::kTokTile - 1) / pf::kTokTile));
  pf::prefill_gemm_kernel<kStage2><<<grid, pf::kThreads, pf::kSmemBytes, stream>>>(params, maps[0], maps[1], maps[2],
                                                                                   maps[3], maps[4], maps[5]);
  NQB_CUDA(cudaGetLastError(), kStage2 ? "prefill stage 2 launch" : "prefill stage 1 launch");
  return NQB_OK;
}

int run_prefill(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
                float *const *ys, float *latent, void *extra, size_t extra_bytes, cudaStream_t stream) {
  if (tokens > 65535ll * pf::kTokTile) return fail(NQB_ERR_UNSUPPORTED, "prefill token count too large");
  if (extra_bytes < prefill_workspace_bytes(layers, count, tokens))
    return fail(NQB_ERR_WORKSPACE, "prefill workspace too small");
  char *ws = static_cast<char *>(extra);
  __half *act1[kMaxMembersTc], *act2[kMaxMembersTc];
  int32_t *exp1[kMaxMembersTc], *exp2[kMaxMembersTc];
  for (int i = 0; i < count; ++i) {
    act1[i] = reinterpret_cast<__half *>(ws);
    ws += align_up(static_cast<size_t>(tokens) * k_pad_of(layers[i].in_features) * 2, 256);
    act2[i] = reinterpret_cast<__half *>(ws);
    ws += align_up(static_cast<size_t>(tokens) * k_pad_of(layers[i].rank) * 2, 256);
    exp1[i] = reinterpret_cast<int32_t *>(ws);
    ws += align_up(static_cast<size_t>(tokens) * 4, 256);
    exp2[i] = reinterpret_cast<int32_t *>(ws);
    ws += align_up(static_cast<size_t>(tokens) * 4, 256);
  }
  // latent members start on 16-byte boundaries (the workspace reserves each
  // member's rank rounded up to 4 columns)
  int64_t latent_stride = 0;
  for (int i = 0; i < count; ++i) latent_stride += (layers[i].rank + 3) & ~int64_t(3);
  const int64_t n = layers[0].in_features;

  // ---- stage 1
  CUtensorMap maps[6];
  std::memset(maps, 0, sizeof(maps));
  pf::Params p1;
  std::memset(&p1, 0, sizeof(p1));
  int ctas = 0;
  int64_t offset = 0;
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    const int64_t kp = k_pad_of(d.in_features);
    pf::quantise_kernel<false><<<static_cast<unsigned>(tokens), 256, 0, stream>>>(
        x, x_dtype, n, d.scale_pre, d.scale_dtype, nullptr, 0, 0, d.in_features, kp, act1[i], exp1[i]);
    NQB_CUDA(cudaGetLastError(), "prefill quantise (stage 1) launch");
    NQB_CHECK(encode_map(&maps[i], act1[i], kp, tokens));
    pf::Member &m = p1.m[i];
    m.tiles = static_cast<const uint4 *>(d.right_tiles);
    m.rows = d.rank;
    m.wc = repack_chunks(d.in_features);
    m.row_tiles = static_cast<int32_t>((d.rank + pf::kTileRows - 1) / pf::kTileRows);
    m.cta_begin = ctas;
    m.k_steps = static_cast<int32_t>(kp / pf::kKStep);
    m.row_scale = d.scale_mid;
    m.exps = exp1[i];
    m.out = latent;
    m.out_stride = latent_stride;
    m.out_offset = offset;
    m.tma_store = tma_storable(latent + offset, latent_stride) ? 1 : 0;
    if (m.tma_store) NQB_CHECK(encode_out_map(&maps[3 + i], latent + offset, d.rank, latent_stride, tokens));
    ctas += m.row_tiles;
    offset += (d.rank + 3) & ~int64_t(3);
  }
  for (int i = count; i < 3; ++i) maps[i] = maps[0];
  for (int i = count; i < 3; ++i) maps[3 + i] = maps[3];
  p1.count = count;
  p1.tokens = tokens;
  p1.scale_dtype = layers[0].scale_dtype;
  p1.x = x;
  p1.x_dtype = x_dtype;
  p1.n = n;
  NQB_CHECK(launch_gemm<false>(p1, maps, ctas, tokens, stream));

  // ---- stage 2
  pf::Params p2;
  std::memset(&p2, 0, sizeof(p2));
  ctas = 0;
  offset = 0;
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    const int64_t kp = k_pad_of(d.rank);
    pf::quantise_kernel<true><<<static_cast<unsigned>(tokens), 256, 0, stream>>>(
        nullptr, 0, 0, nullptr, 0, latent, latent_stride, offset, d.rank, kp, act2[i], exp2[i]);
    NQB_CUDA(cudaGetLastError(), "prefill quantise (stage 2) launch");
    NQB_CHECK(encode_map(&maps[i], act2[i], kp, tokens));
    pf::Member &m = p2.m[i];
    m.tiles = static_cast<const uint4 *>(d.left_tiles);
    m.rows = d.out_features;
    m.wc = repack_chunks(d.rank);
    m.row_tiles = static_cast<int32_t>((d.out_features + pf::kTileRows - 1) / pf::kTileRows);
    m.cta_begin = ctas;
    m.k_steps = static_cast<int32_t>(kp / pf::kKStep);
    m.row_scale = d.scale_post;
    m.exps = exp2[i];
    m.out = ys[i];
    m.out_stride = d.out_features;
    m.out_offset = 0;
    m.bias = d.bias;
    m.bias_dtype = d.bias_dtype;
    m.outlier_count = d.outlier_count;
    m.outlier_indices = d.outlier_indices;
    m.outlier_values = d.outlier_values;
    m.outlier_value_dtype = d.outlier_value_dtype;
    m.outlier_scales = d.outlier_scales;
    m.tma_store = tma_storable(ys[i], d.out_features) ? 1 : 0;
    if (m.tma_store) NQB_CHECK(encode_out_map(&maps[3 + i], ys[i], d.out_features, d.out_features, tokens));
    ctas += m.row_tiles;
    offset += (d.rank + 3) & ~int64_t(3);
  }
  for (int i = count; i < 3; ++i) maps[i] = maps[0];
  for (int i = count; i < 3; ++i) maps[3 + i] = maps[3];
  p2.count = count;
  p2.tokens = tokens;
  p2.scale_dtype = layers[0].scale_dtype;
  p2.x = x;
  p2.x_dtype = x_dtype;
  p2.n = n;
  NQB_CHECK(launch_gemm<true>(p2, maps, ctas, tokens, stream));

  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    if (d.overlay_rows > 0) {
      const int64_t warps = d.overlay_rows * tokens;
      pf::overlay_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
          x, x_dtype, n, tokens, d.overlay_row_ids, d.overlay_values, d.overlay_scales, d.overlay_scale_dtype,
          d.overlay_rows, ys[i], d.out_features);
      NQB_CUDA(cudaGetLastError(), "prefill overlay launch");
    }
  }
  return NQB_OK;
}

int prefill_device_error(int32_t *out) {
  int value = 0;
  NQB_CUDA(cudaMemcpyFromSymbol(&value, pf::g_pf_error, sizeof(int)), "read prefill error flag");
  *out = value;
  const int zero = 0;
  NQB_CUDA(cudaMemcpyToSymbol(pf::g_pf_error, &zero, sizeof(int)), "clear prefill error flag");
  return NQB_OK;
}

}  // namespace nqb
