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
//   shared-memory stages of 66 KB: warp 4 issues TMA and the sign-chunk bulk
//   copy, warps 0-3 expand signs into a double-buffered A region of TMEM, one
//   thread of warp 5 issues the 8 MMAs of a step and commits them to the
//   stage's "empty" barriers.  The 128 x 256 fp32 accumulator stays in TMEM
//   until the epilogue multiplies by 2^-e and the row scale, transposes the
//   tile through the idle stage buffers and writes it with one TMA store.
//   (Two co-resident 128 x 128 CTAs per SM measured slower: their main
//   loops lose more than the overlapped epilogues gain.)
// Every mbarrier wait is bounded; a timeout sets the device status word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "nqb_decode_tc.cuh"
#include "nqb_prefill_tc.cuh"
#include "nqb_tc_ptx.cuh"

namespace nqb {
namespace pf {

constexpr int kTileRows = 128;     // sign rows per tile (MMA M)
constexpr int kTokTile = 192;      // tokens per tile (MMA N): two accumulators + two A buffers fill TMEM
constexpr int kKStep = 128;        // K columns per pipeline step = one 4-word sign chunk
constexpr int kStages = 4;
constexpr int kAtomBytes = kTokTile * 128;             // 192 tokens x 64 fp16 (one 128-byte swizzle column)
constexpr int kBStageBytes = 2 * kAtomBytes;           // 128 K columns
constexpr int kChunkBytes = kTileRows * 16;            // one 4-word chunk of a 128-row tile
constexpr int kACols = kKStep / 2;                     // TMEM columns of A per step
constexpr int kDCol = 2 * kACols;                      // accumulator 0; accumulator 1 follows
constexpr uint32_t kTmemCols = 512;                    // 2 x 64 (A) + 2 x 192 (D)
constexpr int kThreads = 320;                          // 10 warps: 4 expand, 1 TMA, 1 MMA, 4 epilogue
constexpr uint32_t kSpinLimit = 1u << 26;
constexpr int kPreBytes = kKStep * 2;  // fp16 pre scales of one K step, pair order
constexpr int kOutTok = 16;                            // tokens per output box (TMA store)
constexpr int kOutBytes = kOutTok * kTileRows * 4;     // one fp32 [16 tokens][128 rows] box
constexpr int kSmemBytes =
    kStages * (kBStageBytes + kChunkBytes + kPreBytes) + 2 * kOutBytes + 1024;  // +1024: swizzle alignment
static_assert(kDCol + 2 * kTokTile <= static_cast<int>(kTmemCols), "two accumulators must fit tensor memory");
static_assert(kSmemBytes + 4096 <= 227 * 1024, "the stage ring must fit shared memory");
static_assert(kAtomBytes % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");

struct Member {
  const uint4 *tiles;   // row-interleaved sign tiles (nqb_repack_signs)
  const __half *pre_pairs;  // stage 1: fp16 pre scales [k_pad] in pair order, folded into the signs; or nullptr
  int64_t rows;
  int32_t wc;           // 4-word chunks per row
  int32_t row_tiles;
  int32_t cta_begin;    // first row tile of this member among all members
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
  int32_t tma_store;  // 1: output boxes leave through shared memory by TMA store
};

struct Params {
  Member m[kMaxMembersTc];
  int32_t count;
  int32_t total_row_tiles;  // row tiles of all members
  int32_t tok_tiles;
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

// Issues one TMA store of a shared-memory box as its own bulk group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int32_t x, int32_t y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
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
// columns (fp16 pairs) of this thread's lane.  Each pair is the fp16 pair
// (s_j, s_j+16) with its sign bits flipped where the sign bit is 1: s = 1.0
// without folded scales, else the pre scales of those two columns, so that
// the MMA multiplies by +/-pre exactly (fp16 x fp16 products are exact in
// the fp32 accumulator).
__device__ __forceinline__ void expand_and_store(uint4 chunk, uint32_t taddr, const uint4 *pre) {
  const uint32_t words[4] = {chunk.x, chunk.y, chunk.z, chunk.w};
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t v[32];
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
      const uint32_t w = words[half * 2 + wi];
      uint32_t pp[16];
      if (pre != nullptr) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = pre[(half * 2 + wi) * 4 + q];
          pp[4 * q] = u.x;
          pp[4 * q + 1] = u.y;
          pp[4 * q + 2] = u.z;
          pp[4 * q + 3] = u.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) pp[j] = 0x3C003C00u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) v[wi * 16 + j] = ((w << (15 - j)) & 0x80008000u) ^ pp[j];
    }
    ptx::tmem_st16(taddr + half * 32, v);
    ptx::tmem_st16(taddr + half * 32 + 16, v + 16);
  }
}

// Persistent tile loop.  Tile t (of Σ row tiles × token tiles, token-tile
// major so concurrent CTAs share their activations in L2) goes to CTA
// t mod gridDim.x.  Four roles run concurrently over the CTA's tiles:
//   warps 0-3  expand each K step's sign words into TMEM (A, double buffer);
//              lane 0 of each warp arrives for the warp;
//   warp 4     streams B boxes, sign chunks and pre pairs into the stage ring;
//   warp 5     issues the MMAs of a tile into accumulator d = tile & 1;
//   warps 6-9  drain accumulator d of the previous tile (epilogue) while the
//              MMAs fill the other one.
// Every wait is bounded and gives up early once any wait has failed.
struct TileRef {
  int g;      // member
  int tile0;  // row tile within the member
  int tok0;   // first token
};

__device__ __forceinline__ TileRef tile_ref(const Params &p, int t) {
  const int tok_tile = t / p.total_row_tiles;
  const int rt = t - tok_tile * p.total_row_tiles;
  int g = 0;
  for (int i = 1; i < p.count; ++i)
    if (rt >= p.m[i].cta_begin) g = i;
  return TileRef{g, rt - p.m[g].cta_begin, tok_tile * kTokTile};
}

__device__ __forceinline__ bool pf_failed() { return *reinterpret_cast<volatile int *>(&g_pf_error) != 0; }

__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && pf_failed()) return false;
  }
  atomicCAS(&g_pf_error, 0, NQB_ERR_TIMEOUT);
  return false;
}

// Bounded wait with back-off by one lane, then the warp: for the epilogue
// warps, which wait out a whole main loop and must not load the shared-memory
// pipe the expansion warps use.
__device__ __forceinline__ void pf_wait_warp(uint64_t *bar, uint32_t parity) {
  if ((threadIdx.x & 31) == 0) {
    uint32_t i = 0;
    while (!ptx::mbar_try_wait(bar, parity)) {
      if (++i >= kSpinLimit) {
        atomicCAS(&g_pf_error, 0, NQB_ERR_TIMEOUT);
        break;
      }
      if ((i & 255) == 255 && pf_failed()) break;
      __nanosleep(200);
    }
  }
  __syncwarp();
}

template <bool kStage2>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap map0,
                        const __grid_constant__ CUtensorMap map1, const __grid_constant__ CUtensorMap map2,
                        const __grid_constant__ CUtensorMap out0, const __grid_constant__ CUtensorMap out1,
                        const __grid_constant__ CUtensorMap out2) {
  extern __shared__ uint8_t smem_raw[];
  // full[s]: stage s landed; empty[s]: the MMAs of the step that used stage s
  // are done (also frees that step's A buffer); a_full[b]: A buffer b expanded
  __shared__ uint64_t full[kStages], empty[kStages], a_full[2], d_full[2], d_empty[2];
  __shared__ uint32_t s_tmem;
  __shared__ float s_unscale[2][kTokTile];  // 2^-e of each token of the tile in accumulator d (0 past the end)

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *s_b = smem;                                   // [kStages][kBStageBytes], 1024-aligned atoms
  uint8_t *s_chunk = smem + kStages * kBStageBytes;      // [kStages][kChunkBytes]
  uint8_t *s_pre = s_chunk + kStages * kChunkBytes;      // [kStages][kPreBytes]
  float *s_out = reinterpret_cast<float *>(s_pre + kStages * kPreBytes);  // [2][kOutTok][kTileRows] fp32
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int tiles = p.total_row_tiles * p.tok_tiles;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&a_full[b], 4);  // one arrival per expansion warp
      ptx::mbar_init(&d_full[b], 1);
      ptx::mbar_init(&d_empty[b], 128);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&s_tmem, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 4) {
    if (lane == 0) {  // ---- producer
      uint32_t it = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        const TileRef tr = tile_ref(p, t);
        const Member &m = p.m[tr.g];
        const CUtensorMap *map = tr.g == 0 ? &map0 : (tr.g == 1 ? &map1 : &map2);
        const uint32_t bytes = kBStageBytes + kChunkBytes + (m.pre_pairs != nullptr ? kPreBytes : 0);
        for (int s = 0; s < m.k_steps; ++s, ++it) {
          const int slot = static_cast<int>(it % kStages);
          if (it >= kStages) pf_wait(&empty[slot], ((it / kStages) - 1) & 1);
          const uint32_t bar = ptx::smem_u32(&full[slot]);
          expect_tx(&full[slot], bytes);
          const uint32_t base = ptx::smem_u32(s_b + slot * kBStageBytes);
          tma_load_2d(base, map, s * kKStep, tr.tok0, bar);
          tma_load_2d(base + kAtomBytes, map, s * kKStep + 64, tr.tok0, bar);
          const uint8_t *src =
              reinterpret_cast<const uint8_t *>(m.tiles) + (static_cast<size_t>(tr.tile0) * m.wc + s) * kChunkBytes;
          bulk_load(ptx::smem_u32(s_chunk + slot * kChunkBytes), src, kChunkBytes, bar);
          if (m.pre_pairs != nullptr)
            bulk_load(ptx::smem_u32(s_pre + slot * kPreBytes), m.pre_pairs + s * kKStep, kPreBytes, bar);
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = idesc_f16_m128(kTokTile);
      uint32_t it = 0, tc = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tc) {
        const TileRef tr = tile_ref(p, t);
        const int k_steps = p.m[tr.g].k_steps;
        const uint32_t d = tc & 1;
        if (tc >= 2) pf_wait(&d_empty[d], ((tc >> 1) - 1) & 1);
        ptx::tc_fence_after();
        for (int s = 0; s < k_steps; ++s, ++it) {
          // a_full implies full: the expansion warps waited for this stage
          // before they arrived (one wait and one commit per step keep the
          // issuing thread's work below the MMAs' 768 cycles)
          const int slot = static_cast<int>(it % kStages);
          const uint32_t buf = it & 1;
          pf_wait(&a_full[buf], (it >> 1) & 1);
          ptx::tc_fence_after();
          const uint32_t bbase = ptx::smem_u32(s_b + slot * kBStageBytes);
#pragma unroll
          for (int k16 = 0; k16 < kKStep / 16; ++k16) {
            const uint64_t bdesc = desc_sw128(bbase + (k16 >> 2) * kAtomBytes + (k16 & 3) * 32);
            mma_f16_ts(tmem + kDCol + d * kTokTile, tmem + buf * kACols + k16 * 8, bdesc, idesc,
                       (s > 0 || k16 > 0) ? 1u : 0u);
          }
          ptx::mma_commit(&empty[slot]);
        }
        ptx::mma_commit(&d_full[d]);
      }
    }
  } else if (warp < 4) {
    // ---- sign expansion into TMEM: thread tid owns tile row tid (TMEM lane tid)
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const TileRef tr = tile_ref(p, t);
      const Member &m = p.m[tr.g];
      for (int s = 0; s < m.k_steps; ++s, ++it) {
        const int slot = static_cast<int>(it % kStages);
        pf_wait(&full[slot], (it / kStages) & 1);
        const uint4 c0 = reinterpret_cast<const uint4 *>(s_chunk + slot * kChunkBytes)[tid];
        const uint32_t buf = it & 1;
        if (it >= 2) {  // A buffer `buf` is free once step it - 2's MMAs are done
          pf_wait(&empty[(it - 2) % kStages], ((it - 2) / kStages) & 1);
          ptx::tc_fence_after();
        }
        const uint4 *pre = m.pre_pairs != nullptr ? reinterpret_cast<const uint4 *>(s_pre + slot * kPreBytes) : nullptr;
        expand_and_store(c0, tmem + lane_base + buf * kACols, pre);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[buf]);
      }
    }
  } else {
    // ---- epilogue warps 6-9: warp w reads TMEM lanes 32 * (w % 4) .. +32.
    // Each 16-token half of a 32-column TMEM load becomes one fp32
    // [16 tokens][128 rows] box in shared memory (two buffers) that thread 0
    // of the group writes out with a TMA store; the store of the box two
    // halves back must have finished reading its buffer first.  Rows past the
    // member and tokens past the end are clipped by the store.
    const int et = tid - 6 * 32;  // 0..127
    const int quarter = warp & 3;
    const int lrow = quarter * 32 + lane;  // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t tc = 0;
    uint32_t boxes = 0;  // boxes staged so far; buffer = boxes & 1
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tc) {
      const TileRef tr = tile_ref(p, t);
      const Member &m = p.m[tr.g];
      const CUtensorMap *out_map = tr.g == 0 ? &out0 : (tr.g == 1 ? &out1 : &out2);
      const uint32_t d = tc & 1;
      // the four epilogue warps are past tile tc - 2: s_unscale[d] is free
      asm volatile("bar.sync 2, 128;" ::: "memory");
      for (int i = et; i < kTokTile; i += 128) {
        const int64_t tok = tr.tok0 + i;
        s_unscale[d][i] = tok < p.tokens ? exp2_int(-m.exps[tok]) : 0.0f;
      }
      const int64_t row = static_cast<int64_t>(tr.tile0) * kTileRows + lrow;
      const bool live = row < m.rows;
      const float rscale = live ? load_as_float(m.row_scale, row, p.scale_dtype) : 0.0f;
      const float bias = (kStage2 && live && m.bias != nullptr) ? load_as_float(m.bias, row, m.bias_dtype) : 0.0f;
      asm volatile("bar.sync 2, 128;" ::: "memory");
      pf_wait_warp(&d_full[d], (tc >> 1) & 1);
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c2 = 0; c2 < kTokTile / 32; ++c2) {
        if (tr.tok0 + c2 * 32 >= p.tokens) break;  // uniform over the group
        uint32_t v[32];
        ptx::tmem_ld16(tmem + lane_base + kDCol + d * kTokTile + c2 * 32, v);
        ptx::tmem_ld16(tmem + lane_base + kDCol + d * kTokTile + c2 * 32 + 16, v + 16);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t0 = c2 * 32 + h * 16;  // first token of the box within the tile
          float out[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) out[e] = __uint_as_float(v[h * 16 + e]) * s_unscale[d][t0 + e] * rscale + bias;
          if constexpr (kStage2) {
            if (live && m.outlier_count > 0) {
              for (int64_t sidx = 0; sidx < m.outlier_count; ++sidx) {
                float w = load_as_float(m.outlier_values, row * m.outlier_count + sidx, m.outlier_value_dtype);
                if (m.outlier_scales != nullptr) w *= load_as_float(m.outlier_scales, sidx, p.scale_dtype);
                const int32_t col = m.outlier_indices[sidx];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                  const int64_t tok = tr.tok0 + t0 + e;
                  if (tok < p.tokens) out[e] += load_as_float(p.x, tok * p.n + col, p.x_dtype) * w;
                }
              }
            }
          }
          if (m.tma_store) {
            if (tr.tok0 + t0 >= p.tokens) continue;  // uniform over the group
            float *buf = s_out + (boxes & 1) * (kOutTok * kTileRows);
            ++boxes;
            if (et == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            asm volatile("bar.sync 2, 128;" ::: "memory");
#pragma unroll
            for (int e = 0; e < 16; ++e) buf[e * kTileRows + lrow] = out[e];
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (et == 0)
              tma_store_2d(out_map, tr.tile0 * kTileRows, static_cast<int32_t>(tr.tok0 + t0), ptx::smem_u32(buf));
          } else if (live) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int64_t tok = tr.tok0 + t0 + e;
              if (tok < p.tokens) m.out[tok * m.out_stride + m.out_offset + row] = out[e];
            }
          }
        }
      }
      ptx::tc_fence_before();
      mbar_arrive(&d_empty[d]);
    }
    if (et == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) ptx::tmem_dealloc(tmem, kTmemCols);
}

// Pre-pass: per token and member, scale the activation row by 2^e
// (max |a| * 2^e < 2^15, exact), convert to fp16 in pair order, record e.
// Stage 1 reads x * pre (all members share x), stage 2 the fp32 latent
// slice of each member.  One warp per token; lane l owns the 32-column
// groups l, l + 32, ...; a group is read with 16-byte loads when it lies
// whole inside the row and the row is 16-byte aligned.
struct PrepMember {
  const void *scale;   // per-column scale (stage 1: pre), nullptr for none
  int64_t src_offset;  // first source column of the member
  int64_t k_valid;     // source columns
  int64_t k_pad;       // fp16 columns written (multiple of 128, zero past k_valid)
  __half *out;         // [tokens][k_pad]
  int32_t *exps;       // [tokens]
};

struct PrepParams {
  PrepMember m[kMaxMembersTc];
  int32_t count;
  const void *src;
  int32_t src_dtype;
  int64_t src_stride;  // elements per token row
  int32_t scale_dtype;
  int32_t vec_src;     // token rows and member offsets are 16-byte aligned
  int32_t vec_scale;   // every scale vector is 16-byte aligned
  int64_t tokens;
  // fp16 pre scales rewritten in pair order for the stage-1 sign expansion
  // (CTA row i writes member i's copy; pairs_count = 0 for none)
  int32_t pairs_count;
  const __half *pairs_src[kMaxMembersTc];
  __half *pairs_out[kMaxMembersTc];
  int64_t pairs_valid;
  int64_t pairs_pad;
};

__device__ __forceinline__ void unpack8(uint4 u, int32_t dt, float *v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (dt == NQB_BF16) {
      v[2 * q] = __uint_as_float(w[q] << 16);
      v[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[q]));
      v[2 * q] = f.x;
      v[2 * q + 1] = f.y;
    }
  }
}

// 32 consecutive values base[idx .. idx + 31] as float; entries at or past
// `valid` read as 0.
__device__ __forceinline__ void load_group(const void *base, int64_t idx, int32_t dt, int64_t valid, bool vec,
                                           float *v) {
  if (vec && valid >= 32) {
    if (dt == NQB_F32) {
      const float4 *p4 = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 f = __ldg(p4 + q);
        v[4 * q] = f.x;
        v[4 * q + 1] = f.y;
        v[4 * q + 2] = f.z;
        v[4 * q + 3] = f.w;
      }
    } else {
      const uint4 *p4 = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + idx);
      uint4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) u[q] = __ldg(p4 + q);
#pragma unroll
      for (int q = 0; q < 4; ++q) unpack8(u[q], dt, v + 8 * q);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = e < valid ? load_as_float(base, idx + e, dt) : 0.0f;
  }
}

__global__ void __launch_bounds__(256) prepare_kernel(const __grid_constant__ PrepParams p) {
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= p.tokens) return;
  const bool vsrc = p.vec_src != 0, vscale = p.vec_scale != 0;
  for (int i = 0; i < p.count; ++i) {
    const PrepMember &m = p.m[i];
    const int64_t row = t * p.src_stride + m.src_offset;
    float mx = 0.0f;
#pragma unroll 2
    for (int64_t g = lane; g * 32 < m.k_valid; g += 32) {
      float v[32], sc[32];
      load_group(p.src, row + g * 32, p.src_dtype, m.k_valid - g * 32, vsrc, v);
      if (m.scale != nullptr) {
        load_group(m.scale, g * 32, p.scale_dtype, m.k_valid - g * 32, vscale, sc);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= sc[e];
      }
#pragma unroll
      for (int e = 0; e < 32; ++e) mx = fmaxf(mx, fabsf(v[e]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    int e2 = 0;
    if (mx > 0.0f && isfinite(mx)) {
      int ex;
      frexpf(mx, &ex);
      e2 = min(15 - ex, 126);
    }
    const float scale = exp2_int(e2);
    uint4 *out = reinterpret_cast<uint4 *>(m.out + t * m.k_pad);
#pragma unroll 2
    for (int64_t g = lane; g * 32 < m.k_pad; g += 32) {
      float v[32], sc[32];
      const int64_t valid = m.k_valid - g * 32;
      load_group(p.src, row + g * 32, p.src_dtype, valid, vsrc, v);
      if (m.scale != nullptr) {
        load_group(m.scale, g * 32, p.scale_dtype, valid, vscale, sc);
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] *= sc[e];
      }
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const __half2 h = __floats2half2_rn(v[j] * scale, v[j + 16] * scale);
        w[j] = *reinterpret_cast<const uint32_t *>(&h);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) out[g * 4 + q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
    if (lane == 0) m.exps[t] = e2;
  }
}

// 8 consecutive values base[idx .. idx + 7] as float; entries at or past
// `valid` read as 0.  The vector form needs base + idx 16-byte aligned.
__device__ __forceinline__ void load8(const void *base, int64_t idx, int32_t dt, int64_t valid, bool vec, float *v) {
  if (vec && valid >= 8) {
    if (dt == NQB_F32) {
      const float4 *p4 = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx);
      const float4 a = __ldg(p4), b = __ldg(p4 + 1);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
      unpack8(__ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + idx)), dt, v);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = e < valid ? load_as_float(base, idx + e, dt) : 0.0f;
  }
}

// Row pre-pass, one CTA per (token, member) row held in registers.  Unit u
// of a row is the 16 columns {32g + 8h + j, 32g + 16 + 8h + j : j < 8}
// (g = u / 2, h = u % 2): exactly the fp16 positions [32g + 16h, +16) of the
// pair order, so every thread loads and stores whole 16-byte vectors.
constexpr int kPrepThreads = 128;  // threads per row for rows up to 512 units (8192 columns)

template <int kUnits, int kRowThreads = kPrepThreads>
__global__ void __launch_bounds__(kRowThreads) prepare_rows_kernel(const __grid_constant__ PrepParams p) {
  __shared__ float s_max[kRowThreads / 32];
  const int64_t t = blockIdx.x;
  const PrepMember &m = p.m[blockIdx.y];
  const int64_t row = t * p.src_stride + m.src_offset;
  const int64_t units = m.k_pad / 16;
  const bool vsrc = p.vec_src != 0, vscale = p.vec_scale != 0;
  const int tid = threadIdx.x;
  float v[kUnits][16];
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < kUnits; ++i) {
    const int64_t u = tid + i * kRowThreads;
    if (u < units) {
      const int64_t c0 = (u >> 1) * 32 + (u & 1) * 8;
      load8(p.src, row + c0, p.src_dtype, m.k_valid - c0, vsrc, v[i]);
      load8(p.src, row + c0 + 16, p.src_dtype, m.k_valid - c0 - 16, vsrc, v[i] + 8);
      if (m.scale != nullptr) {
        float sc[16];
        load8(m.scale, c0, p.scale_dtype, m.k_valid - c0, vscale, sc);
        load8(m.scale, c0 + 16, p.scale_dtype, m.k_valid - c0 - 16, vscale, sc + 8);
#pragma unroll
        for (int e = 0; e < 16; ++e) v[i][e] *= sc[e];
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) mx = fmaxf(mx, fabsf(v[i][e]));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((tid & 31) == 0) s_max[tid >> 5] = mx;
  __syncthreads();
  mx = s_max[0];
#pragma unroll
  for (int w = 1; w < kRowThreads / 32; ++w) mx = fmaxf(mx, s_max[w]);
  int e2 = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);
    e2 = min(15 - ex, 126);
  }
  const float scale = exp2_int(e2);
  uint4 *out = reinterpret_cast<uint4 *>(m.out + t * m.k_pad);
#pragma unroll
  for (int i = 0; i < kUnits; ++i) {
    const int64_t u = tid + i * kRowThreads;
    if (u < units) {
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half2 h = __floats2half2_rn(v[i][j] * scale, v[i][j + 8] * scale);
        w[j] = *reinterpret_cast<const uint32_t *>(&h);
      }
      out[2 * u] = make_uint4(w[0], w[1], w[2], w[3]);
      out[2 * u + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
  if (tid == 0) m.exps[t] = e2;
  if (blockIdx.y == 0 && t < p.pairs_count) {
    const __half *src = p.pairs_src[t];
    __half *dst = p.pairs_out[t];
    for (int64_t pos = tid; pos < p.pairs_pad; pos += kRowThreads) {
      const int64_t col = (pos & ~int64_t(31)) + ((pos & 31) >> 1) + ((pos & 1) << 4);
      dst[pos] = col < p.pairs_valid ? src[col] : __float2half_rn(0.0f);
    }
  }
}

// 8 consecutive 16-bit values base[idx .. idx + 7], raw; entries at or past
// `valid` read as 0.  The vector form needs base + idx 16-byte aligned.
__device__ __forceinline__ uint4 load8_raw16(const uint16_t *base, int64_t idx, int64_t valid) {
  if (valid >= 8) return __ldg(reinterpret_cast<const uint4 *>(base + idx));
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  for (int e = 0; e < 8 && e < valid; ++e) w[e >> 1] |= static_cast<uint32_t>(base[idx + e]) << (16 * (e & 1));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// The row pre-pass for 16-bit sources without a per-column scale (bf16 / f16
// x with pre folded into the sign expansion): the same units and output as
// prepare_rows_kernel, but each thread keeps its units as the loaded 16-byte
// vectors (8 registers a unit instead of 16 floats), so twice as many rows
// stay in flight per SM; the values are widened once for the maximum and
// again for the fp16 stores.
template <int kUnits, int kRowThreads = kPrepThreads>
__global__ void __launch_bounds__(kRowThreads) prepare_rows16_kernel(const __grid_constant__ PrepParams p) {
  __shared__ float s_max[kRowThreads / 32];
  const int64_t t = blockIdx.x;
  const PrepMember &m = p.m[blockIdx.y];
  const uint16_t *src = static_cast<const uint16_t *>(p.src) + t * p.src_stride + m.src_offset;
  const int64_t units = m.k_pad / 16;
  const int tid = threadIdx.x;
  uint4 raw[kUnits][2];
#pragma unroll
  for (int i = 0; i < kUnits; ++i) {
    const int64_t u = tid + i * kRowThreads;
    const int64_t c0 = (u >> 1) * 32 + (u & 1) * 8;
    raw[i][0] = raw[i][1] = make_uint4(0u, 0u, 0u, 0u);
    if (u < units) {
      raw[i][0] = load8_raw16(src, c0, m.k_valid - c0);
      raw[i][1] = load8_raw16(src, c0 + 16, m.k_valid - c0 - 16);
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < kUnits; ++i) {
    float v[16];
    unpack8(raw[i][0], p.src_dtype, v);
    unpack8(raw[i][1], p.src_dtype, v + 8);
#pragma unroll
    for (int e = 0; e < 16; ++e) mx = fmaxf(mx, fabsf(v[e]));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((tid & 31) == 0) s_max[tid >> 5] = mx;
  __syncthreads();
  mx = s_max[0];
#pragma unroll
  for (int w = 1; w < kRowThreads / 32; ++w) mx = fmaxf(mx, s_max[w]);
  int e2 = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);
    e2 = min(15 - ex, 126);
  }
  const float scale = exp2_int(e2);
  uint4 *out = reinterpret_cast<uint4 *>(m.out + t * m.k_pad);
#pragma unroll
  for (int i = 0; i < kUnits; ++i) {
    const int64_t u = tid + i * kRowThreads;
    if (u < units) {
      float v[16];
      unpack8(raw[i][0], p.src_dtype, v);
      unpack8(raw[i][1], p.src_dtype, v + 8);
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half2 h = __floats2half2_rn(v[j] * scale, v[j + 8] * scale);
        w[j] = *reinterpret_cast<const uint32_t *>(&h);
      }
      out[2 * u] = make_uint4(w[0], w[1], w[2], w[3]);
      out[2 * u + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  }
  if (tid == 0) m.exps[t] = e2;
  if (blockIdx.y == 0 && t < p.pairs_count) {
    const __half *ps = p.pairs_src[t];
    __half *dst = p.pairs_out[t];
    for (int64_t pos = tid; pos < p.pairs_pad; pos += kRowThreads) {
      const int64_t col = (pos & ~int64_t(31)) + ((pos & 31) >> 1) + ((pos & 1) << 4);
      dst[pos] = col < p.pairs_valid ? ps[col] : __float2half_rn(0.0f);
    }
  }
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

// Longest row the register-resident pre-pass takes (8 units per thread, 256 threads).
constexpr int64_t kRowKernelMaxCols = 8 * 256 * 16;

// With fp16 pre scales (and rows the row pre-pass takes) stage 1 folds pre
// into the sign expansion, so all members read one fp16 copy of x.
static bool fold_pre(const nqb_linear_desc *layers) {
  return layers[0].scale_dtype == NQB_F16 && k_pad_of(layers[0].in_features) <= kRowKernelMaxCols;
}

// Byte offsets of the prefill buffers inside the path workspace.
struct PrefillLayout {
  size_t act1[kMaxMembersTc], exp1[kMaxMembersTc];    // stage-1 fp16 activations, exponents (one set if folded)
  size_t act2[kMaxMembersTc], exp2[kMaxMembersTc];    // stage-2 fp16 latent, exponents
  size_t pairs[kMaxMembersTc];                        // pair-ordered fp16 pre scales (folded only)
  bool fold;
  size_t total;
};

static PrefillLayout prefill_layout(const nqb_linear_desc *layers, int count, int64_t tokens) {
  PrefillLayout l{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align_up(bytes, 256);
    return at;
  };
  const size_t t = static_cast<size_t>(tokens);
  l.fold = fold_pre(layers);
  for (int i = 0; i < (l.fold ? 1 : count); ++i) {
    l.act1[i] = take(t * k_pad_of(layers[i].in_features) * 2);
    l.exp1[i] = take(t * 4);
  }
  for (int i = 0; i < count; ++i) {
    l.act2[i] = take(t * k_pad_of(layers[i].rank) * 2);
    l.exp2[i] = take(t * 4);
    if (l.fold) l.pairs[i] = take(k_pad_of(layers[i].in_features) * 2);
  }
  l.total = off;
  return l;
}

size_t prefill_workspace_bytes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  if (!prefill_eligible(layers, count, NQB_F32, tokens)) return 0;
  return prefill_layout(layers, count, tokens).total;
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

// fp32 output [tokens][columns] with a row stride of `stride` floats, written
// as [16 tokens][128 columns] boxes from shared memory (no swizzle).
static int encode_out_map(CUtensorMap *map, float *base, int64_t columns, int64_t stride, int64_t tokens) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  NQB_CHECK(tensor_map_encoder(&encode));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(columns), static_cast<cuuint64_t>(tokens)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 4};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(pf::kTileRows), static_cast<cuuint32_t>(pf::kOutTok)};
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

// Row pre-pass for rows up to kRowKernelMaxCols columns, else the warp-per-token one.
static int launch_prepare(const pf::PrepParams &params, cudaStream_t stream, const char *what) {
  int64_t units = 0;
  for (int i = 0; i < params.count; ++i) units = std::max<int64_t>(units, params.m[i].k_pad / 16);
  const dim3 grid(static_cast<unsigned>(params.tokens), static_cast<unsigned>(params.count));
  bool raw16 = (params.src_dtype == NQB_BF16 || params.src_dtype == NQB_F16) && params.vec_src != 0;
  for (int i = 0; i < params.count; ++i) raw16 = raw16 && params.m[i].scale == nullptr;
  if (raw16 && units <= 8 * 256) {
    if (units <= pf::kPrepThreads) {
      pf::prepare_rows16_kernel<1><<<grid, pf::kPrepThreads, 0, stream>>>(params);
    } else if (units <= 2 * pf::kPrepThreads) {
      pf::prepare_rows16_kernel<2><<<grid, pf::kPrepThreads, 0, stream>>>(params);
    } else if (units <= 4 * pf::kPrepThreads) {
      pf::prepare_rows16_kernel<4><<<grid, pf::kPrepThreads, 0, stream>>>(params);
    } else if (units <= 4 * 256) {
      pf::prepare_rows16_kernel<4, 256><<<grid, 256, 0, stream>>>(params);
    } else {
      pf::prepare_rows16_kernel<8, 256><<<grid, 256, 0, stream>>>(params);
    }
  } else if (units <= pf::kPrepThreads) {
    pf::prepare_rows_kernel<1><<<grid, pf::kPrepThreads, 0, stream>>>(params);
  } else if (units <= 2 * pf::kPrepThreads) {
    pf::prepare_rows_kernel<2><<<grid, pf::kPrepThreads, 0, stream>>>(params);
  } else if (units <= 4 * pf::kPrepThreads) {
    pf::prepare_rows_kernel<4><<<grid, pf::kPrepThreads, 0, stream>>>(params);
  } else if (units <= 4 * 256) {  // wide rows: 256 threads per row keep 16 warps per SM
    pf::prepare_rows_kernel<4, 256><<<grid, 256, 0, stream>>>(params);
  } else if (units <= 8 * 256) {
    pf::prepare_rows_kernel<8, 256><<<grid, 256, 0, stream>>>(params);
  } else {
    if (params.pairs_count != 0) return fail(NQB_ERR_UNSUPPORTED, "folded pre scales need the row pre-pass");
    pf::prepare_kernel<<<static_cast<unsigned>((params.tokens + 7) / 8), 256, 0, stream>>>(params);  // warp per token
  }
  NQB_CUDA(cudaGetLastError(), what);
  return NQB_OK;
}

// Persistent launch: one CTA per SM (or per tile when there are fewer tiles).
template <bool kStage2>
static int launch_gemm(pf::Params &params, const CUtensorMap *maps, int row_tiles, int64_t tokens,
                       cudaStream_t stream) {
  const void *fn = reinterpret_cast<const void *>(pf::prefill_gemm_kernel<kStage2>);
  NQB_CHECK(ensure_dynamic_smem(fn, pf::kSmemBytes));
  params.total_row_tiles = row_tiles;
  params.tok_tiles = static_cast<int32_t>((tokens + pf::kTokTile - 1) / pf::kTokTile);
  const int64_t tiles = static_cast<int64_t>(row_tiles) * params.tok_tiles;
  int device = 0, sms = 148;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const unsigned grid = static_cast<unsigned>(tiles < sms ? tiles : sms);
  pf::prefill_gemm_kernel<kStage2><<<grid, pf::kThreads, pf::kSmemBytes, stream>>>(params, maps[0], maps[1], maps[2],
                                                                                   maps[3], maps[4], maps[5]);
  NQB_CUDA(cudaGetLastError(), kStage2 ? "prefill stage 2 launch" : "prefill stage 1 launch");
  return NQB_OK;
}

int run_prefill(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
                float *const *ys, float *latent, void *extra, size_t extra_bytes, cudaStream_t stream) {
  if (tokens > (1ll << 22)) return fail(NQB_ERR_UNSUPPORTED, "prefill token count too large");
  if (extra_bytes < prefill_workspace_bytes(layers, count, tokens))
    return fail(NQB_ERR_WORKSPACE, "prefill workspace too small");
  char *ws = static_cast<char *>(extra);
  const PrefillLayout lay = prefill_layout(layers, count, tokens);
  __half *act1[kMaxMembersTc], *act2[kMaxMembersTc], *pairs[kMaxMembersTc];
  int32_t *exp1[kMaxMembersTc], *exp2[kMaxMembersTc];
  for (int i = 0; i < count; ++i) {
    const int i1 = lay.fold ? 0 : i;
    act1[i] = reinterpret_cast<__half *>(ws + lay.act1[i1]);
    exp1[i] = reinterpret_cast<int32_t *>(ws + lay.exp1[i1]);
    act2[i] = reinterpret_cast<__half *>(ws + lay.act2[i]);
    exp2[i] = reinterpret_cast<int32_t *>(ws + lay.exp2[i]);
    pairs[i] = lay.fold ? reinterpret_cast<__half *>(ws + lay.pairs[i]) : nullptr;
  }
  // latent members start on 16-byte boundaries (the workspace reserves each
  // member's rank rounded up to 4 columns)
  int64_t latent_stride = 0;
  for (int i = 0; i < count; ++i) latent_stride += (layers[i].rank + 3) & ~int64_t(3);
  const int64_t n = layers[0].in_features;

  // ---- stage 1
  CUtensorMap maps[6];  // activation maps of up to three members, then their output maps
  std::memset(maps, 0, sizeof(maps));
  pf::Params p1;
  std::memset(&p1, 0, sizeof(p1));
  int ctas = 0;
  int64_t offset = 0;
  pf::PrepParams q1;
  std::memset(&q1, 0, sizeof(q1));
  q1.count = count;
  q1.src = x;
  q1.src_dtype = x_dtype;
  q1.src_stride = n;
  q1.scale_dtype = layers[0].scale_dtype;
  q1.tokens = tokens;
  q1.vec_src = (reinterpret_cast<uintptr_t>(x) % 16 == 0 && (n * dtype_size(x_dtype)) % 16 == 0) ? 1 : 0;
  q1.vec_scale = 1;
  if (lay.fold) {  // x alone; the pre scales go to the sign expansion in pair order
    q1.count = 1;
    q1.m[0] = pf::PrepMember{nullptr, 0, n, k_pad_of(n), act1[0], exp1[0]};
    q1.pairs_count = count;
    q1.pairs_valid = n;
    q1.pairs_pad = k_pad_of(n);
    for (int i = 0; i < count; ++i) {
      q1.pairs_src[i] = static_cast<const __half *>(layers[i].scale_pre);
      q1.pairs_out[i] = pairs[i];
    }
  } else {
    for (int i = 0; i < count; ++i) {
      const nqb_linear_desc &d = layers[i];
      q1.m[i] = pf::PrepMember{d.scale_pre, 0, d.in_features, k_pad_of(d.in_features), act1[i], exp1[i]};
      if (reinterpret_cast<uintptr_t>(d.scale_pre) % 16) q1.vec_scale = 0;
    }
  }
  NQB_CHECK(launch_prepare(q1, stream, "prefill activation pre-pass (stage 1) launch"));
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    const int64_t kp = k_pad_of(d.in_features);
    NQB_CHECK(encode_map(&maps[i], act1[i], kp, tokens));
    pf::Member &m = p1.m[i];
    m.tiles = static_cast<const uint4 *>(d.right_tiles);
    m.pre_pairs = pairs[i];
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
  pf::PrepParams q2;
  std::memset(&q2, 0, sizeof(q2));
  q2.count = count;
  q2.src = latent;
  q2.src_dtype = NQB_F32;
  q2.src_stride = latent_stride;
  q2.tokens = tokens;
  q2.vec_src = reinterpret_cast<uintptr_t>(latent) % 16 == 0 ? 1 : 0;
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    q2.m[i] = pf::PrepMember{nullptr, offset, d.rank, k_pad_of(d.rank), act2[i], exp2[i]};
    offset += (d.rank + 3) & ~int64_t(3);
  }
  NQB_CHECK(launch_prepare(q2, stream, "prefill activation pre-pass (stage 2) launch"));
  offset = 0;
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    const int64_t kp = k_pad_of(d.rank);
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
    m.tma_store = tma_storable(ys[i], d.out_features) ? 1 : 0;
    if (m.tma_store) NQB_CHECK(encode_out_map(&maps[3 + i], ys[i], d.out_features, d.out_features, tokens));
    m.bias = d.bias;
    m.bias_dtype = d.bias_dtype;
    m.outlier_count = d.outlier_count;
    m.outlier_indices = d.outlier_indices;
    m.outlier_values = d.outlier_values;
    m.outlier_value_dtype = d.outlier_value_dtype;
    m.outlier_scales = d.outlier_scales;
    ctas += m.row_tiles;
    offset += (d.rank + 3) & ~int64_t(3);
  }
  for (int i = count; i < 3; ++i) maps[i] = maps[0];
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
