// Persistent decode program of libnqb: a whole sequence of packed-linear
// calls (1..16 tokens) in one cooperative launch.
//
// A decode step is a chain of small sign-matrix products; launched one kernel
// per stage, each pays a launch, a prologue and several global-memory round
// trips while the weights it streams take well under a microsecond.  Here one
// CTA per SM runs every stage of every op in order:
//
// * Work.  The CTAs form clusters of 4.  For each stage the host assigns the
//   128-row tiles to clusters (balanced by sign bytes); the 4 CTAs of a
//   cluster split every tile's K range in quarters, so each tile's partial
//   sums meet in distributed shared memory: CTA q writes its quarter into the
//   tile's leader CTA (tile index mod 4), which adds the four in a fixed order
//   and runs the epilogue (scale_mid -> latent; scale_post, salient columns,
//   low-rank patch, bias, int8 overlay rows -> y).  No global atomics,
//   deterministic.  A patched layer's patch latent R x is formed in stage 1
//   (its rows spread over all CTAs, after their tiles) in latent columns
//   after the op's ranks.
// * Arithmetic.  Exact integer MMAs with register operands
//   (nqb_mma_decode.cuh): activations quantised per (token, K chunk) to 22-bit
//   fixed-point digits (B fragments in shared memory), sign bits expanded by
//   one LOP3 per A-fragment register; 8 consumer warps x 16 rows per tile.
// * Weights.  Sign words do not depend on activations, so a producer warp
//   streams each CTA's 4 KB slices (256 columns x 128 rows) through a ring of
//   bulk copies as far ahead as the ring allows, across stage barriers.  The
//   host precomputes each CTA's slice addresses in consumption order; the
//   addresses themselves arrive by bulk copy, 64 at a time.
// * Order.  After every stage a grid barrier (one release add per CTA on a
//   global counter, an acquire poll).  Activations are read through L2 after
//   the barrier, so an op may consume an earlier op's output.  The producer
//   warp never joins a barrier: cluster exchanges use mbarriers with remote
//   arrivals, CTA-wide steps a named barrier of the consumer warps.
// Every wait is bounded.  Only the grid barriers depend on other clusters:
// when one gives up, it sets the device status word and every later grid
// barrier gives up at once, so a failed run ends (with wrong results and
// NQB_ERR_TIMEOUT) instead of hanging.  The CTA-local and cluster waits (sign
// copies, stage tables, partial-sum exchange) always complete, so they do not
// give up early: a failed run still consumes every slice it copied and keeps
// its stage tables consistent, and no copy is in flight when a CTA exits.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <new>
#include <vector>

#include "nqb_decode_tc.cuh"
#include "nqb_mma_decode.cuh"
#include "nqb_program.cuh"
#include "nqb_tc_decode.cuh"
#include "nqb_tc_ptx.cuh"

namespace nqb {
namespace prog {

using namespace tc;

constexpr int kClusterSize = 4;
constexpr int kMaxRing = 48;            // ring slots (4 KB each)
constexpr int kAddrChunk = 64;          // slice addresses per bulk copy
constexpr int kAddrSlots = 4;           // address chunks in flight
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kBarrierSpinLimit = 1u << 22;  // default polls of the grid-barrier counter
constexpr int kMaxDynamicSmem = 220 * 1024;  // + static shared memory <= 227 KB
// Coded mixed-V slices (nqb_repack_mixed_v): 128 rows x 8 20-bit records
// (codebook index | a << 10 | b << 15), row r's from bit 160 r; a member's
// 1024-word codebook is staged in shared memory per stage 1.
constexpr uint32_t kCodedSliceBytes = 2560;
constexpr uint32_t kCodedRowBits = 160;
// Coded product-codebook slices (nqb_repack_product_codebook): 128 rows x 8
// 16-bit records, row r's at byte 16 r; the member's 1024-word decode table
// (first half words, second half words << 16) is staged like a codebook.
constexpr uint32_t kCodebookSliceBytes = 2048;
constexpr int kCodebookWords = 1024;
constexpr int64_t kOverlaySegCols = 1024;  // columns of one int8 overlay row segment (a multiple of 16)

struct MemberDev {
  const uint8_t *tiles;  // row-interleaved sign tiles
  int64_t rows;
  int32_t wc;            // 4-word chunks per row
  int32_t ks;            // 256-column slices per row
  int64_t k_valid;
  const float *pre;       // stage 1: activation scale (fp32 copy owned by the program)
  const float *row_scale;  // stage 1: scale_mid; stage 2: scale_post (fp32 copies)
  int64_t act_offset;    // stage 2: first latent column of the member
  int64_t out_offset;    // stage 1: first latent column written
  const float *bias;     // fp32 copy or nullptr
  int64_t outlier_count;
  const int32_t *outlier_indices;
  const void *outlier_values;
  int32_t outlier_value_dtype;
  const void *outlier_scales;
  int32_t outlier_scale_dtype;
  int64_t overlay_rows;
  const int32_t *overlay_row_ids;
  const int8_t *overlay_values;
  const void *overlay_scales;
  int32_t overlay_scale_dtype;
  const int32_t *overlay_slot;  // stage 2: [rows] overlay row index of each output row, -1 without (program-owned)
  int64_t overlay_offset;       // first latent column of the member's overlay partial dot products
  float *y;
  int64_t patch_rank;         // low-rank patch: stage 1 reads R [p, n], stage 2 L [m, p]
  const void *patch_factor;
  int32_t patch_dtype;
  int64_t patch_offset;       // first latent column of the member's patch latent
  // stage 1 of a coded member: tiles from coded_from on stream as records
  const uint8_t *coded_tiles;
  const uint32_t *codebook;   // [1024] words, bulk-copied into shared memory per stage
  int32_t coded_from;         // first coded tile (INT32_MAX: none)
  int32_t coded_format;       // NQB_CODED_MIXED_V / NQB_CODED_PRODUCT_CODEBOOK
};

// The decoder-step extensions of an op (nqb_program_op_ext), staged into
// shared memory with the op's other tables.
struct __align__(8) StepDev {
  int32_t kind;            // NQB_OP_LINEAR / NQB_OP_ATTENTION
  int32_t epilogue;        // NQB_EPI_*
  const float *norm_stats;  // residual-stream input: [stat_tiles][tokens] partial sums of h^2
  int32_t stat_tiles;
  float eps;
  float inv_n;
  float *out_stats;        // NQB_EPI_RESIDUAL: [tiles][tokens]
  int32_t q_heads, kv_heads;
  const float *q_norm, *k_norm;  // fp32 copies, or nullptr
  const float *cos_t, *sin_t;    // [tokens][128]
  __nv_bfloat16 *q;              // [tokens][q_heads * 128]
  __nv_bfloat16 *k_cache, *v_cache;
  int64_t cache_len, position;
  int64_t seq_stride;            // 0: one sequence; else token t's caches start t * seq_stride elements in
  __nv_bfloat16 *attn_out;
  int32_t att_splits;
  int32_t att_parts;         // partials per (token, q head): splits, or 2 x splits from 8 tokens on (key halves)
  int32_t att_ring_blocks;   // at most this many 16-row K/V blocks of a unit arrive through the sign ring
  int64_t att_chunk;         // keys per split, a multiple of 16
};

struct OpDev {
  MemberDev s[2][kMaxMembersTc];  // [stage][member]
  int32_t count;
  const void *x;
  const void *x2;  // NQB_X_SWIGLU / NQB_X_GEGLU: the up projection (x is the gate)
  int32_t x_dtype;
  int32_t side_rows;  // patch rows and int8 overlay row segments of all members (stage 1 forms their latents)
  int32_t ovl_segs;   // segments (kOverlaySegCols columns each) per int8 overlay row
  int64_t n;
  int64_t latent_stride;
  StepDev step;  // decoder-step extensions
};

// 16-row K and V blocks of attention unit (split sp) that stream through the
// sign ring: the unit's rows before this step's tokens (they do not change
// during the program), whole blocks only, at most op.att_ring_blocks.  The
// host lists the same blocks in the CTA's slice addresses.
__host__ __device__ inline int att_unit_ring_blocks(const StepDev &op, int sp) {
  const int64_t k0 = static_cast<int64_t>(sp) * op.att_chunk;
  const int64_t old_end = op.position < k0 + op.att_chunk ? op.position : k0 + op.att_chunk;
  const int64_t blocks = old_end > k0 ? (old_end - k0) / 16 : 0;
  return static_cast<int>(blocks < op.att_ring_blocks ? blocks : op.att_ring_blocks);
}

struct Item {
  int32_t member;
  int32_t tile;
};

// Everything a CTA's consumers read about one stage, staged into shared
// memory by the producer warp one stage ahead: the op's fields, the members'
// descriptors of that stage and the cluster's tile list.
constexpr int kMaxStageItems = 64;
struct __align__(16) StageInfo {
  MemberDev md[kMaxMembersTc];
  const void *x;
  const void *x2;
  int64_t n;
  int64_t latent_stride;
  int32_t x_dtype;
  int32_t n_items;
  int32_t side_rows;
  int32_t ovl_segs;
  StepDev step;
  Item items[kMaxStageItems];
};

struct Params {
  const OpDev *ops;
  int32_t stages;              // 2 * ops
  int32_t clusters;
  const int32_t *stage_items;  // [stages * clusters + 1] offsets into items
  const Item *items;
  const uint64_t *slice_addrs;  // per-CTA lists (each padded to kAddrChunk entries)
  const int64_t *slice_begin;   // [ctas]
  const int32_t *slice_count;   // [ctas]
  const uint64_t *pf_lines;     // L2 lines each CTA reads in each stage besides signs and activations
  const int32_t *pf_begin;      // [stages * ctas + 1]
  float *latent;
  uint32_t *counters;           // [0] grid barrier arrivals, [1] finished clusters
  uint32_t barrier_limit;       // polls before a grid barrier gives up
  uint32_t barrier_skew;        // added to every barrier target (tests: a barrier that cannot complete)
  int32_t tokens;
  int32_t ring;                 // ring slots
  int32_t sc;                   // slices quantised at once
  int32_t group;                // items per exchange group (4 x leader slots)
  // dynamic shared memory offsets
  uint32_t off_addr, off_b, off_acc, off_exch;
  uint32_t off_cb;              // mixed-V codebooks [kMaxMembersTc][1024]
  uint32_t off_epi;             // decoder-step epilogue scratch: [tokens][128] + [4][tokens] floats
  float *att_part;              // attention partials [tokens * q_heads][splits][kAttRow]
  // 8 and 16 tokens: each linear stage's activation chunks are quantised once,
  // by all CTAs, into qbuf (one slot of qunit_bytes per chunk), before a grid
  // barrier; the stage's consumers then copy the digits instead of
  // re-quantising them in every cluster
  uint8_t *qbuf;
  int32_t qunit_bytes;
  const int32_t *bar_end;       // [stages] index of the grid barrier that ends each stage
};

__device__ int g_prog_error;

// Phase trace (built with NQB_PHASE_TRACE only): per CTA and stage, the SM
// cycles consumer thread 0 spent in each phase of the stage.
enum TracePhase {
  kTraceTables = 0,   // stage start -> first quantisation (tables, accumulator reset)
  kTraceQuantise,     // activation loads, maxima, digit scatter
  kTraceWaitSigns,    // waiting for sign slices in the ring
  kTraceMma,          // sign-word loads + MMA issue
  kTraceDrain,        // accumulators -> fp32 partials
  kTraceSend,         // partials -> leaders (st.async), row-scale loads
  kTraceWaitQuarters, // waiting for the four quarters
  kTraceSum,          // fixed-order sum
  kTraceRelease,      // exchange buffers handed back
  kTraceEpilogue,     // scales, bias, salient columns, stores
  kTraceGridBarrier,  // grid barrier after the stage
  kTracePhases
};
constexpr int kTraceMaxCtas = 160;
constexpr int kTraceMaxStages = 512;
#ifdef NQB_PHASE_TRACE
__device__ long long g_trace[kTraceMaxCtas][kTraceMaxStages][kTracePhases];
#define NQB_TRACE_BEGIN            \
  long long trace_t = clock64();   \
  long long trace_c[kTracePhases]; \
  for (int trace_k = 0; trace_k < kTracePhases; ++trace_k) trace_c[trace_k] = 0;
#define NQB_TRACE(phase)             \
  do {                               \
    const long long now = clock64(); \
    trace_c[phase] += now - trace_t; \
    trace_t = now;                   \
  } while (0)
#define NQB_TRACE_RESET() trace_t = clock64()
#define NQB_TRACE_FLUSH(stage)                                                                 \
  do {                                                                                         \
    if (threadIdx.x == 0 && blockIdx.x < kTraceMaxCtas && (stage) < kTraceMaxStages)           \
      for (int trace_k = 0; trace_k < kTracePhases; ++trace_k)                                 \
        g_trace[blockIdx.x][stage][trace_k] = trace_c[trace_k];                                \
  } while (0)
#else
#define NQB_TRACE_BEGIN
#define NQB_TRACE(phase) \
  do {                   \
  } while (0)
#define NQB_TRACE_FLUSH(stage) \
  do {                         \
  } while (0)
#define NQB_TRACE_RESET() \
  do {                    \
  } while (0)
#endif

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_prog_error, 0, code); }

__device__ __forceinline__ bool program_failed() { return *reinterpret_cast<volatile int *>(&g_prog_error) != 0; }

// Bounded wait with back-off, for the producer warps (they run ahead and are
// not on the critical path; sleeping leaves the issue slots to the MMA warps).
__device__ __forceinline__ bool wait_local_backoff(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    __nanosleep(32);
  }
  record_error(NQB_ERR_TIMEOUT);
  return false;
}

// Bounded wait for phase `parity` of a CTA-local mbarrier; on timeout it
// records NQB_ERR_TIMEOUT.  The phases it waits for are completed by this CTA
// (or by its copies), so it never gives up early.
__device__ __forceinline__ bool wait_local(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
  }
  record_error(NQB_ERR_TIMEOUT);
  return false;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_addr(const void *local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(ptx::smem_u32(local)), "r"(rank));
  return remote;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}


__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ptx::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ptx::smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   ptx::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(ptx::smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Arrive (relaxed, cluster scope) on the mbarrier at the same offset in CTA
// `rank`.  Used to hand back exchange buffers whose values this thread's CTA
// has already consumed, so no ordering of earlier memory operations is needed.
__device__ __forceinline__ void remote_arrive_relaxed(uint64_t *bar, uint32_t rank) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr(bar, rank))
               : "memory");
}

// Waits (acquire, cluster scope) for phase `parity` of a local mbarrier; bounded.
__device__ __forceinline__ bool wait_cluster(uint64_t *bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(ptx::smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  record_error(NQB_ERR_TIMEOUT);
  return false;
}

// Asynchronous 16-byte store into the shared memory of CTA `rank` (same
// offset as `local`); completion is counted on that CTA's mbarrier `bar`.
__device__ __forceinline__ void st_async_v4(const float *local, uint32_t rank, float4 v, uint64_t *bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          cluster_addr(local, rank)),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cluster_addr(bar, rank))
      : "memory");
}

// L2 prefetch of [p, p + bytes) by the consumer threads (one line each).
__device__ __forceinline__ void prefetch_range(const void *ptr, int64_t bytes) {
  const char *base = static_cast<const char *>(ptr);
  for (int64_t off = static_cast<int64_t>(threadIdx.x) * 128; off < bytes; off += static_cast<int64_t>(mmad::kThreads) * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
}

// L2 prefetch of the lines stage g of this CTA reads besides sign words and
// activations (pre and row scales, bias, input rows), from the host-built
// list; the 32 lanes of the info warp.
__device__ __forceinline__ void prefetch_stage(const Params &p, int g, int lane) {
  if (g >= p.stages) return;
  const int cta = static_cast<int>(blockIdx.x);
  const int b = p.pf_begin[g * static_cast<int>(gridDim.x) + cta];
  const int e = p.pf_begin[g * static_cast<int>(gridDim.x) + cta + 1];
  for (int i = b + lane; i < e; i += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(p.pf_lines[i]));
}

// Until the grid-barrier counter reaches `target`; false after `limit` polls
// (or at once when a grid barrier has failed).
__device__ __forceinline__ bool wait_counter(const uint32_t *counter, uint32_t target, uint32_t limit) {
  for (uint32_t polls = 0; polls < limit; ++polls) {
    if (ld_acquire_gpu(counter) >= target) return true;
    if (program_failed()) return false;
    __nanosleep(64);
  }
  record_error(NQB_ERR_TIMEOUT);
  return false;
}

// Copies stage g's tables for this CTA's cluster into `info` (the 32 lanes of
// the info warp; 4-byte words).
__device__ __forceinline__ void stage_info_copy(const Params &p, int g, uint32_t cluster, int lane, StageInfo &info) {
  const OpDev &op = p.ops[g >> 1];
  const int st = g & 1;
  const int ib = p.stage_items[g * p.clusters + cluster];
  const int ie = p.stage_items[g * p.clusters + cluster + 1];
  const int n_items = min(ie - ib, kMaxStageItems);
  const uint32_t *md_src = reinterpret_cast<const uint32_t *>(&op.s[st][0]);
  uint32_t *md_dst = reinterpret_cast<uint32_t *>(&info.md[0]);
  constexpr int kMdWords = static_cast<int>(sizeof(MemberDev) * kMaxMembersTc / 4);
  for (int i = lane; i < kMdWords; i += 32) md_dst[i] = md_src[i];
  const uint32_t *it_src = reinterpret_cast<const uint32_t *>(p.items + ib);
  uint32_t *it_dst = reinterpret_cast<uint32_t *>(&info.items[0]);
  for (int i = lane; i < n_items * 2; i += 32) it_dst[i] = it_src[i];
  {
    const uint32_t *sd_src = reinterpret_cast<const uint32_t *>(&op.step);
    uint32_t *sd_dst = reinterpret_cast<uint32_t *>(&info.step);
    for (int i = lane; i < static_cast<int>(sizeof(StepDev) / 4); i += 32) sd_dst[i] = sd_src[i];
  }
  if (lane == 0) {
    info.x = op.x;
    info.x2 = op.x2;
    info.n = op.n;
    info.latent_stride = op.latent_stride;
    info.x_dtype = op.x_dtype;
    info.n_items = n_items;
    info.side_rows = op.side_rows;
    info.ovl_segs = op.ovl_segs;
  }
}

// Grid barrier number `index` over every CTA of the grid (consumer warps;
// thread 0 adds and polls).  At a stage's end every consumer is done with the
// stage's tables: thread 0 first hands their buffer back (`info_free`; NULL
// for the barrier after a pre-quantisation pass).
__device__ __forceinline__ void grid_barrier(const Params &p, uint32_t index, uint64_t *info_free) {
  uint32_t *counter = p.counters;
  const uint32_t ctas = gridDim.x;
  mmad::consumer_sync();
  if (threadIdx.x == 0) {
    if (info_free != nullptr) mbar_arrive_cta(info_free);
    // release: this CTA's stores (ordered before this thread by the named
    // barrier) are visible to every CTA that acquires the count
    red_release_gpu_add(counter, 1);
    // acquire polls (relaxed polls with one acquire fence at the end
    // measured slower on B200)
    const uint32_t target = (index + 1) * ctas + p.barrier_skew;
    uint32_t polls = 0;
    while (ld_acquire_gpu(counter) < target) {
      if (program_failed()) break;
      if (++polls > p.barrier_limit) {
        record_error(NQB_ERR_TIMEOUT);
        break;
      }
    }
  }
  mmad::consumer_sync();
}

// Stage 1's side latents, formed by the two side warps of every CTA while
// the consumer warps run the stage's tiles.  Rows numbered across the op --
// the patched members' patch rows, then the stage-2 members' int8 overlay
// rows -- go to the grid's side warps round-robin:
//   patch row q of member k:   latent[t][patch_offset_k + q]   = sum_i x[t, i] R_k[q, i]
//   overlay row j of member k, segment s (columns [s S, s S + S), S = kOverlaySegCols):
//     latent[t][overlay_offset_k + j segs + s] = scale_j sum_i x[t, i] v_k[j, i]
// (fp32, each lane's share then the warp's sum in fixed order).  Stage 2's
// epilogue adds L_k P and each overlay row's segments in order.  Inputs are read through
// L2: an earlier op of the program may have written them.
__device__ __forceinline__ float load_x_cg(const void *x, int64_t i, int32_t dtype) {
  if (dtype == NQB_F32) return __ldcg(static_cast<const float *>(x) + i);
  if (dtype == NQB_BF16) return __bfloat162float(__ldcg(static_cast<const __nv_bfloat16 *>(x) + i));
  return __half2float(__ldcg(static_cast<const __half *>(x) + i));
}

__device__ __forceinline__ float dot_i8x4(uint32_t w, float a0, float a1, float a2, float a3) {
  return static_cast<float>(static_cast<int8_t>(w & 0xFFu)) * a0 +
         static_cast<float>(static_cast<int8_t>((w >> 8) & 0xFFu)) * a1 +
         static_cast<float>(static_cast<int8_t>((w >> 16) & 0xFFu)) * a2 +
         static_cast<float>(static_cast<int8_t>(w >> 24)) * a3;
}

__device__ __forceinline__ float2 unpack_pair(uint32_t v, int32_t dtype) {
  if (dtype == NQB_BF16) return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  return __half22float2(*reinterpret_cast<const __half2 *>(&v));
}

// sum over 16 elements of int8 w (one 16-byte word) times x[i0 .. i0 + 16)
// (x 16-byte aligned there), read through L2
__device__ __forceinline__ float dot_i8x16(uint4 w, const void *x, int64_t i0, int32_t dtype) {
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
  float s = 0.0f;
  if (dtype == NQB_F32) {
    const float4 *xv = reinterpret_cast<const float4 *>(static_cast<const float *>(x) + i0);
    float4 a[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) a[q] = __ldcg(xv + q);
#pragma unroll
    for (int q = 0; q < 4; ++q) s += dot_i8x4(ww[q], a[q].x, a[q].y, a[q].z, a[q].w);
  } else {
    const uint4 *xv = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + i0);
    const uint4 h0 = __ldcg(xv), h1 = __ldcg(xv + 1);
    const uint32_t hh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 lo = unpack_pair(hh[2 * q], dtype), hi = unpack_pair(hh[2 * q + 1], dtype);
      s += dot_i8x4(ww[q], lo.x, lo.y, hi.x, hi.y);
    }
  }
  return s;
}

__device__ __forceinline__ void side_rows_warp(const Params &p, const OpDev &op, int worker, int workers, int lane) {
  const int T = p.tokens;
  int64_t base = 0;  // side rows of earlier members
  for (int k = 0; k < op.count; ++k) {
    const MemberDev &md = op.s[0][k];
    if (md.patch_rank <= 0) continue;
    for (int64_t q = ((worker - base) % workers + workers) % workers; q < md.patch_rank; q += workers) {
      for (int t0 = 0; t0 < T; t0 += 4) {  // four tokens at a time: few registers beside the consumers'
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t i = lane; i < op.n; i += 32) {
          const float r = load_as_float(md.patch_factor, q * op.n + i, md.patch_dtype);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (t0 + u >= T) break;
            part[u] += load_x_cg(op.x, static_cast<int64_t>(t0 + u) * op.n + i, op.x_dtype) * r;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) part[u] += __shfl_xor_sync(0xffffffffu, part[u], off);
          if (lane == 0 && t0 + u < T)
            p.latent[static_cast<int64_t>(t0 + u) * op.latent_stride + md.patch_offset + q] = part[u];
        }
      }
    }
    base += md.patch_rank;
  }
  for (int k = 0; k < op.count; ++k) {
    const MemberDev &md = op.s[1][k];
    if (md.overlay_rows <= 0) continue;
    // 16-element chunks: one 16-byte load of int8 values and 16-byte loads of x
    const bool vec = op.n % 16 == 0 && reinterpret_cast<uintptr_t>(op.x) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(md.overlay_values) % 16 == 0;
    const int segs = op.ovl_segs;
    const int n = static_cast<int>(op.n);
    const int items = static_cast<int>(md.overlay_rows) * segs;
    for (int it = ((worker - static_cast<int>(base)) % workers + workers) % workers; it < items; it += workers) {
      const int j = it / segs;
      const int c0 = (it - j * segs) * static_cast<int>(kOverlaySegCols);
      const int c1 = min(c0 + static_cast<int>(kOverlaySegCols), n);
      const int8_t *row = md.overlay_values + static_cast<int64_t>(j) * n;
      for (int t = 0; t < T; ++t) {
        float part = 0.0f;
        if (vec) {
#pragma unroll 1
          for (int c = c0 / 16 + lane; c < c1 / 16; c += 32)
            part += dot_i8x16(__ldg(reinterpret_cast<const uint4 *>(row) + c), op.x,
                              static_cast<int64_t>(t) * n + 16 * c, op.x_dtype);
        } else {
#pragma unroll 4
          for (int i = c0 + lane; i < c1; i += 32)
            part += load_x_cg(op.x, static_cast<int64_t>(t) * n + i, op.x_dtype) * static_cast<float>(row[i]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        if (lane == 0)
          p.latent[static_cast<int64_t>(t) * op.latent_stride + md.overlay_offset + it] =
              part * load_as_float(md.overlay_scales, j, md.overlay_scale_dtype);
      }
    }
    base += items;
  }
}

__device__ __forceinline__ uint32_t coded_record(const uint32_t *w, int row, int j) {
  const uint32_t bit = static_cast<uint32_t>(row) * kCodedRowBits + static_cast<uint32_t>(j) * 20u;
  const uint32_t i = bit >> 5;  // i + 1 <= 640 stays inside the 4 KB ring slot
  return __funnelshift_r(w[i], w[i + 1], bit & 31u) & 0xFFFFFu;
}

// Record -> sign word: codebook word with bits a and b flipped.
__device__ __forceinline__ uint32_t decode_record(const uint32_t *cb, uint32_t rec) {
  return cb[rec & 1023u] ^ (1u << ((rec >> 10) & 31u)) ^ (1u << (rec >> 15));
}

// Product-codebook record (16 bits, row r's record j at halfword 8 r + j of
// the slice) -> sign word: the two half words from the staged table.
__device__ __forceinline__ uint32_t decode_product_record(const uint32_t *tab, const uint8_t *slice, int row,
                                                          int j) {
  const uint32_t rec = reinterpret_cast<const uint16_t *>(slice)[row * 8 + j];
  return tab[rec & 255u] | tab[256u + (rec >> 8)];
}

// The producer lane's view of this CTA's slice-address list.
struct Producer {
  const uint64_t *addrs;
  int32_t count;
  int32_t padded;
  uint64_t *cache;      // [kAddrSlots][kAddrChunk]
  uint64_t *addr_bar;   // [kAddrSlots]
  uint8_t *ring;
  uint64_t *full;       // [ring]
  int32_t ring_slots;

  __device__ void issue_addr_chunk(int chunk) const {
    if (chunk * kAddrChunk >= padded) return;
    uint64_t *bar = addr_bar + (chunk % kAddrSlots);
    expect_tx(bar, kAddrChunk * 8);
    bulk_load(cache + (chunk % kAddrSlots) * kAddrChunk, addrs + static_cast<int64_t>(chunk) * kAddrChunk,
              kAddrChunk * 8, bar);
  }

  // Fill ring position `pos` (slot pos % ring) with slice `pos` of this CTA's
  // list.  With kMixed, bit 0 of an address marks a coded mixed-V slice
  // (2560 bytes) and bit 1 a coded product-codebook slice (2048 bytes).
  template <bool kMixed>
  __device__ bool produce(int pos, int slot) const {
    const int chunk = pos / kAddrChunk;
    if (pos % kAddrChunk == 0 && chunk >= 1) issue_addr_chunk(chunk + kAddrSlots - 1);
    const bool ok = wait_local(addr_bar + (chunk % kAddrSlots), (chunk / kAddrSlots) & 1);
    uint64_t src = cache[(chunk % kAddrSlots) * kAddrChunk + pos % kAddrChunk];
    uint32_t bytes = kStageWeightBytes;
    if constexpr (kMixed) {
      if (src & 3u) {
        bytes = (src & 2u) ? kCodebookSliceBytes : kCodedSliceBytes;
        src &= ~uint64_t(3);
      }
    }
    expect_tx(full + slot, bytes);
    bulk_load(ring + static_cast<size_t>(slot) * kStageWeightBytes, reinterpret_cast<const void *>(src), bytes,
              full + slot);
    return ok;
  }
};

// 8 consumer warps (warpgroups 0 and 1), then warpgroup 2: the sign-ring
// producer warp, a warp that stages each stage's tables and prefetches its
// scales (two warps, so that neither role's waiting can starve the other
// within one warp) and two idle warps.  Twelve warps launch with 168
// registers each (65536 / 384, rounded down to 8); warpgroup 2 then hands
// registers back (setmaxnreg) so each consumer thread holds up to 224:
// 256 x 224 + 128 x 56 = 64512 = 384 x 168, and per SM sub-partition (two
// consumer warps and one of warpgroup 2) 32 x (2 x 224 + 56) <= 16384.  The
// host launches an instance only if it was built with exactly 168 registers
// (a smaller launch could not serve the consumers' increase).
constexpr int kBlockThreads = mmad::kThreads + 128;
constexpr int kProducerWarp = mmad::kWarps;
constexpr int kInfoWarp = mmad::kWarps + 1;
constexpr int kSideWarp = mmad::kWarps + 2;  // and kSideWarp + 1: stage 1's patch and overlay rows
constexpr int kLaunchRegs = 168;
constexpr int kConsumerRegs = 224;
constexpr int kHelperRegs = 56;
static_assert(mmad::kThreads * kConsumerRegs + (kBlockThreads - mmad::kThreads) * kHelperRegs <=
                  kBlockThreads * kLaunchRegs,
              "register split exceeds the launch's registers");
static_assert(32 * (2 * kConsumerRegs + kHelperRegs) <= 16384, "register split exceeds a sub-partition");

// Instances whose linear stages quantise their activation chunks once, over
// the grid, before the stage (a grid barrier more per stage; each cluster
// re-quantising every chunk itself costs more from 8 tokens on).
__host__ __device__ constexpr bool pre_quantised(int bucket) { return bucket >= 8; }

// Slices quantised at once (B fragments and activations held for them).
__host__ __device__ constexpr int slices_per_chunk(int bucket) {
  return bucket <= 2 ? 16 : (bucket <= 4 ? 8 : 4);
}

// Tiles each CTA leads per exchange group: 16 KB of exchange buffer.
__host__ __device__ constexpr int leader_slots(int bucket) {
  return 16384 / (kClusterSize * bucket * kTileRows * 4) > 1 ? 16384 / (kClusterSize * bucket * kTileRows * 4) : 1;
}

// Pre-quantised stages (8 and 16 tokens): the stage's activation chunks in a
// fixed order -- member k, then K quarter q (slices [ks q / 4, ks (q + 1) / 4)),
// then chunks of sc slices -- are units 0, 1, ..; unit u's digits, exponents
// and digit sums go to qbuf slot u.
__host__ __device__ inline int quarter_chunks(int ks, int q, int sc) {
  const int lo = ks * q / kClusterSize, hi = ks * (q + 1) / kClusterSize;
  return (hi - lo + sc - 1) / sc;
}

__host__ __device__ inline int member_chunks(int ks, int sc) {
  int n = 0;
  for (int q = 0; q < kClusterSize; ++q) n += quarter_chunks(ks, q, sc);
  return n;
}

// The unit of member k's quarter q starting at slice c0.
__device__ __forceinline__ int unit_of(const StageInfo &op, int k, int q, int c0, int sc) {
  int u = 0;
  for (int m = 0; m < k; ++m) u += member_chunks(op.md[m].ks, sc);
  for (int r = 0; r < q; ++r) u += quarter_chunks(op.md[k].ks, r, sc);
  return u + (c0 - op.md[k].ks * q / kClusterSize) / sc;
}

// Unit u -> member, first slice and slice count; false past the stage's units.
__device__ __forceinline__ bool unit_at(const StageInfo &op, int u, int sc, int &k, int &c0, int &nst) {
  for (k = 0; k < kMaxMembersTc; ++k) {
    const int ks = op.md[k].ks;
    for (int q = 0; q < kClusterSize; ++q) {
      const int n = quarter_chunks(ks, q, sc);
      if (u < n) {
        const int lo = ks * q / kClusterSize, hi = ks * (q + 1) / kClusterSize;
        c0 = lo + u * sc;
        nst = min(sc, hi - c0);
        return true;
      }
      u -= n;
    }
  }
  return false;
}

// Advances (j0, j1, c0, hi) to the next (member run, chunk) unit of the
// group [.., ge) with a non-empty K range for this cluster rank: items
// [j0, j1) share a member; chunk c0 covers slices [c0, min(c0 + sc, hi)).
// Start with j0 = j1 = first item, c0 = hi = 0.  False once the group is done.
__device__ __forceinline__ bool next_unit(const StageInfo &op, int ge, int rank, int sc, int &j0, int &j1, int &c0,
                                          int &hi) {
  c0 += sc;
  while (c0 >= hi) {
    j0 = j1;
    if (j0 >= ge) return false;
    const int mi = op.items[j0].member;
    j1 = j0 + 1;
    while (j1 < ge && op.items[j1].member == mi) ++j1;
    const int ks = op.md[mi].ks;
    c0 = ks * rank / kClusterSize;
    hi = ks * (rank + 1) / kClusterSize;
  }
  return true;
}

// ------------------------------------------------------ decoder-step ops ---

constexpr int kAttHd = 128;                 // head_dim of the fused attention and q/k epilogue
constexpr int kAttGroup = 4;                // q heads per kv head
constexpr int kAttSub = 32 / kAttGroup;     // keys per warp sub-block (group x keys = 32 lanes)
constexpr int kAttRow = kAttHd + 4;         // a partial: acc[128], m, l, two pad floats (16-byte rows)
constexpr int kAttPadRow = kAttHd * 2 + 16;  // staged K/V row stride of the tensor-core path (conflict-free ldmatrix)
// the tensor-core path stages two halves x (K, V) x 16 rows in the consumers'
// accumulator and exchange buffers, which are idle during attention stages
constexpr int kAttStageBytes = 2 * 2 * 16 * kAttPadRow;
constexpr int64_t kAttPrefetchRows = 512;  // K/V rows per attention unit on the L2 prefetch list

// Attention units: (kv head, key split), and with independent sequences
// (seq_stride > 0) one set per token; unit u -> token tu (0 for one
// sequence), kv head, split.
__host__ __device__ inline int att_units(const StepDev &op, int tokens) {
  return (op.seq_stride != 0 ? tokens : 1) * op.kv_heads * op.att_splits;
}
__host__ __device__ inline void att_unit_of(const StepDev &op, int u, int &tu, int &kvh, int &sp) {
  const int per = op.kv_heads * op.att_splits;
  tu = u / per;
  const int r = u - tu * per;
  kvh = r / op.att_splits;
  sp = r - kvh * op.att_splits;
}
// Element offset of kv head `head`'s cache row `row` in the caches of token tu's sequence.
__host__ __device__ inline int64_t att_cache_offset(const StepDev &op, int tu, int head, int64_t row) {
  return static_cast<int64_t>(tu) * op.seq_stride + (static_cast<int64_t>(head) * op.cache_len + row) * kAttHd;
}
// Element offset of token t's new row of kv head `head`.
__host__ __device__ inline int64_t att_new_row(const StepDev &op, int t, int head) {
  return op.seq_stride != 0 ? att_cache_offset(op, t, head, op.position) : att_cache_offset(op, 0, head, op.position + t);
}

// Named barrier of the 128 leader threads (consumer warps 0..3).
__device__ __forceinline__ void leader_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// Sum over the 32 lanes of v[i] for i < 32, transposed: afterwards lane l holds
// the total of v[l] (31 shuffles instead of 32 x 5).
__device__ __forceinline__ float transposed_sum32(float (&v)[32], int lane) {
  // step `half`: 2 * half values are live; this lane keeps the half of them
  // that matches its lane bit and adds its partner's copy of the same indices
#pragma unroll
  for (int half = 16; half >= 1; half >>= 1) {
    const bool upper = (lane & half) != 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < half) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
      }
    }
  }
  return v[0];
}

__device__ __forceinline__ void bf16x4_to_float(uint2 raw, float (&out)[4]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.y));
  out[0] = a.x;
  out[1] = a.y;
  out[2] = b.x;
  out[3] = b.y;
}

// Tensor-core pieces of the many-token attention path: one m16n8k16 bf16 MMA
// with fp32 accumulators, 8x8 b16 matrix loads from shared memory (four
// matrices; .trans transposes each) and the named barrier of one key half's
// four consumer warps (threads 128 hf .. +127).
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(ptx::smem_u32(row)));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(ptx::smem_u32(row)));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

__device__ __forceinline__ void half_sync(int hf) { asm volatile("bar.sync %0, 128;" ::"r"(4 + hf) : "memory"); }

// Attention partials of one CTA: unit `blockIdx.x` = (kv head, key split),
// for every token of the step.  The 8 consumer warps take 8-key sub-blocks in
// turn; per sub-block a lane loads its 4 dims of the 8 K and V rows (all
// loads in flight together), the 4 heads x 8 keys dot products are summed
// across the warp in one transposed reduction (lane = head * 8 + key), and an
// online softmax updates each head's (m, l, acc).  The warps' partials meet in
// shared memory (fixed order) and one partial per (token, q head, split) goes
// to the workspace.  K/V rows are read through L2 (.cg): this step's rows were
// written by the preceding stage.
//
// The unit's rows before this step's tokens arrive ahead of time as 16-row
// blocks through the sign ring (K block, then V block; the producer streams
// them with the sign slices, across the stage barriers), so most K/V reads
// come from shared memory; the remaining rows (this step's, and any past the
// ring's share) are read from global memory.  The consumers wait for the
// unit's ring slots first and every warp hands them back after the last token.
// Inlined, like attention_join: a call would make the kernel keep its stage
// loop's state across the call (spills), slowing every linear stage.
template <bool kMany>  // kMany: the instance may run 8 or more tokens (the tensor-core path is compiled in)
__device__ __forceinline__ void attention_partials(const Params &p, const StepDev &op, float *scratch,
                                                const uint8_t *ring, uint64_t *s_full, uint64_t *s_empty,
                                                int &slot, uint32_t &phase, bool &ok, long long *trace) {
#ifdef NQB_PHASE_TRACE
  // trace build: ring waits -> wait-signs, q loads and the key loop -> mma, the
  // warps' join and the partial stores -> drain (consumer thread 0's cycles)
  long long tr_t = clock64();
#define NQB_ATT_TRACE(phase)                         \
  do {                                               \
    const long long tr_now = clock64();              \
    if (trace != nullptr) trace[phase] += tr_now - tr_t; \
    tr_t = tr_now;                                   \
  } while (0)
#else
  (void)trace;
#define NQB_ATT_TRACE(phase) \
  do {                       \
  } while (0)
#endif
  const int T = p.tokens;
  const int units = att_units(op, T);
  const int cta = static_cast<int>(blockIdx.x);
  if (cta >= units) return;  // uniform over the CTA
  int tu, kvh, sp;
  att_unit_of(op, cta, tu, kvh, sp);
  const bool seqs = op.seq_stride != 0;  // independent sequences: this unit serves token tu only
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R = p.ring;
  const int nb = att_unit_ring_blocks(op, sp);
  // one consumer thread per ring slot of the unit waits, then a consumer
  // barrier: every warp polling every slot in turn cost microseconds
  if (tid < 2 * nb) {
    const int sj = (slot + tid) % R;
    const uint32_t ph = phase + static_cast<uint32_t>((slot + tid) / R);
    if (!wait_local(&s_full[sj], ph & 1)) ok = false;
  }
  mmad::consumer_sync();
  NQB_ATT_TRACE(kTraceWaitSigns);
  const int64_t ring_rows = 16 * static_cast<int64_t>(nb);
  const float scale = rsqrtf(static_cast<float>(kAttHd));
  const __nv_bfloat16 *kbase = op.k_cache + att_cache_offset(op, tu, kvh, 0) + lane * 4;
  const __nv_bfloat16 *vbase = op.v_cache + att_cache_offset(op, tu, kvh, 0) + lane * 4;
  // one 8-key sub-block [b0, b0 + nk) of the split's K and V rows: from the
  // ring where the unit's blocks are, else from global memory (L2)
  auto load_block = [&](int64_t k0, int64_t b0, int nk, uint2 (&kr)[kAttSub], uint2 (&vr)[kAttSub]) {
    if (b0 - k0 < ring_rows) {  // a whole sub-block inside a ring block (16 nb is a multiple of 8)
      const int blk = static_cast<int>((b0 - k0) >> 4), within = static_cast<int>((b0 - k0) & 15);
      const uint8_t *kslot = ring + static_cast<size_t>((slot + 2 * blk) % R) * kStageWeightBytes;
      const uint8_t *vslot = ring + static_cast<size_t>((slot + 2 * blk + 1) % R) * kStageWeightBytes;
#pragma unroll
      for (int j = 0; j < kAttSub; ++j) {
        kr[j] = *reinterpret_cast<const uint2 *>(kslot + (within + j) * (kAttHd * 2) + lane * 8);
        vr[j] = *reinterpret_cast<const uint2 *>(vslot + (within + j) * (kAttHd * 2) + lane * 8);
      }
    } else {
#pragma unroll
      for (int j = 0; j < kAttSub; ++j) {
        const int64_t row = b0 + (j < nk ? j : 0);  // rows past the block re-read row b0 (masked below)
        kr[j] = __ldcg(reinterpret_cast<const uint2 *>(kbase + row * kAttHd));
        vr[j] = __ldcg(reinterpret_cast<const uint2 *>(vbase + row * kAttHd));
      }
    }
  };
  // one sub-block's scores, online-softmax step and P V for one token (q in
  // qv; state acc, m, l of the unit's four q heads, lane: 4 dims)
  auto block_update = [&](const uint2 (&kr)[kAttSub], const uint2 (&vr)[kAttSub], int nk,
                          const float (&qv)[kAttGroup][4], float (&acc)[kAttGroup][4], float (&m)[kAttGroup],
                          float (&l)[kAttGroup]) {
    float sv[32];
#pragma unroll
    for (int j = 0; j < kAttSub; ++j) {
      float kf[4];
      bf16x4_to_float(kr[j], kf);
#pragma unroll
      for (int h = 0; h < kAttGroup; ++h)
        sv[h * kAttSub + j] = qv[h][0] * kf[0] + qv[h][1] * kf[1] + qv[h][2] * kf[2] + qv[h][3] * kf[3];
    }
    const int own_h = lane / kAttSub, own_j = lane % kAttSub;
    float sc = transposed_sum32(sv, lane);
    if (own_j >= nk) sc = -INFINITY;
    float mb = sc;
#pragma unroll
    for (int off = 1; off < kAttSub; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
    float mn[kAttGroup], corr[kAttGroup];
#pragma unroll
    for (int h = 0; h < kAttGroup; ++h) {
      mn[h] = fmaxf(m[h], __shfl_sync(0xffffffffu, mb, h * kAttSub));  // finite: the block has a key
      corr[h] = __expf(m[h] - mn[h]);  // exp(-inf) = 0 on the first block
    }
    const float pr = own_j < nk ? __expf(sc - mn[own_h]) : 0.0f;
    float ps = pr;
#pragma unroll
    for (int off = 1; off < kAttSub; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
#pragma unroll
    for (int h = 0; h < kAttGroup; ++h) {
      l[h] = l[h] * corr[h] + __shfl_sync(0xffffffffu, ps, h * kAttSub);
      m[h] = mn[h];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[h][e] *= corr[h];
    }
#pragma unroll
    for (int j = 0; j < kAttSub; ++j) {
      float vf[4];
      bf16x4_to_float(vr[j], vf);
#pragma unroll
      for (int h = 0; h < kAttGroup; ++h) {
        const float pj = __shfl_sync(0xffffffffu, pr, h * kAttSub + j);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] += pj * vf[e];
      }
    }
  };
  auto load_q = [&](int t, float (&qv)[kAttGroup][4], float (&acc)[kAttGroup][4], float (&m)[kAttGroup],
                    float (&l)[kAttGroup]) {
#pragma unroll
    for (int h = 0; h < kAttGroup; ++h) {
      const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(
          op.q + (static_cast<int64_t>(t) * op.q_heads + kvh * kAttGroup + h) * kAttHd + lane * 4));
      bf16x4_to_float(raw, qv[h]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qv[h][e] *= scale;
        acc[h][e] = 0.0f;
      }
      m[h] = -INFINITY;
      l[h] = 0.0f;
    }
  };
  // token t over this split's keys b0 = first, first + step, .. (8-key sub-blocks)
  auto token_keys = [&](int t, int64_t k0, int64_t k1, int64_t first, int64_t step, float (&acc)[kAttGroup][4],
                        float (&m)[kAttGroup], float (&l)[kAttGroup]) {
    float qv[kAttGroup][4];
    load_q(t, qv, acc, m, l);
    for (int64_t b0 = first; b0 < k1; b0 += step) {
      const int nk = static_cast<int>(min(static_cast<int64_t>(kAttSub), k1 - b0));
      uint2 kr[kAttSub], vr[kAttSub];
      load_block(k0, b0, nk, kr, vr);
      block_update(kr, vr, nk, qv, acc, m, l);
    }
  };
  if (kMany && T >= mmad::kWarps && !seqs) {
    // many tokens, on the tensor cores (mma.sync m16n8k16 bf16, fp32
    // accumulators): the unit's query rows r = 4 tl + h (token 4 rb + tl, q
    // head h of this kv head) in 16-row blocks rb; warp w < 4 takes block w
    // over the split's first key half, warp w + 4 the same rows over the
    // second half, and each writes its own partial (the join takes 2 per
    // split).  Per 16-key block: the half's four warps stage K and V into
    // shared memory (272-byte rows: the ring's 256-byte rows put the eight
    // rows of every 8x8 matrix load on the same banks), then S = Q K^T, an
    // online softmax and O += P V.
    const int rbs = (T + 3) / 4;
    const int rb = warp & 3, hf = warp >> 2;
    const int g = lane >> 2, c = lane & 3;
    const int64_t k0 = static_cast<int64_t>(sp) * op.att_chunk;
    const int64_t kend = min(k0 + op.att_chunk, op.position + T);  // past the last key any token sees
    const int64_t kmid = k0 + (kend > k0 ? ((kend - k0 + 31) / 32) * 16 : 0);
    const int64_t ka = hf == 0 ? k0 : kmid, kb = hf == 0 ? min(kmid, kend) : kend;
    const int t_lo = 4 * rb + (g >> 2), t_hi = t_lo + 2, hq = g & 3;
    const int64_t k1_lo = min(k0 + op.att_chunk, op.position + 1 + t_lo);
    const int64_t k1_hi = min(k0 + op.att_chunk, op.position + 1 + t_hi);
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.0f, l_hi = 0.0f;
    uint32_t qa[8][4];  // A fragments of Q: 8 steps of 16 dims (rows of this warp's block)
    if (rb < rbs) {
      const __nv_bfloat16 *q_lo = op.q + (static_cast<int64_t>(t_lo) * op.q_heads + kvh * kAttGroup + hq) * kAttHd;
      const __nv_bfloat16 *q_hi = op.q + (static_cast<int64_t>(t_hi) * op.q_heads + kvh * kAttGroup + hq) * kAttHd;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d0 = 16 * kk + 2 * c;
        qa[kk][0] = t_lo < T ? __ldcg(reinterpret_cast<const uint32_t *>(q_lo + d0)) : 0u;
        qa[kk][1] = t_hi < T ? __ldcg(reinterpret_cast<const uint32_t *>(q_hi + d0)) : 0u;
        qa[kk][2] = t_lo < T ? __ldcg(reinterpret_cast<const uint32_t *>(q_lo + d0 + 8)) : 0u;
        qa[kk][3] = t_hi < T ? __ldcg(reinterpret_cast<const uint32_t *>(q_hi + d0 + 8)) : 0u;
      }
    }
    const __nv_bfloat16 *kg = op.k_cache + static_cast<int64_t>(kvh) * op.cache_len * kAttHd;
    const __nv_bfloat16 *vg = op.v_cache + static_cast<int64_t>(kvh) * op.cache_len * kAttHd;
    uint8_t *sk = reinterpret_cast<uint8_t *>(scratch) + hf * (2 * 16 * kAttPadRow);
    uint8_t *sv = sk + 16 * kAttPadRow;
    const int ht = tid & 127;  // thread within the half
    for (int64_t b0 = ka; b0 < kb; b0 += 16) {
      const bool in_ring = b0 - k0 < ring_rows;  // 16-key blocks from k0 coincide with the ring's blocks
      const int blk = static_cast<int>((b0 - k0) >> 4);
      const uint8_t *kslot = ring + static_cast<size_t>((slot + 2 * blk) % R) * kStageWeightBytes;
      const uint8_t *vslot = ring + static_cast<size_t>((slot + 2 * blk + 1) % R) * kStageWeightBytes;
#pragma unroll
      for (int u = 0; u < 2; ++u) {  // 16 rows x 16 chunks of 16 bytes, two per thread
        const int q = ht + 128 * u, row = q >> 4, col = q & 15;
        uint4 kv, vv;
        if (in_ring) {
          kv = *reinterpret_cast<const uint4 *>(kslot + row * (kAttHd * 2) + col * 16);
          vv = *reinterpret_cast<const uint4 *>(vslot + row * (kAttHd * 2) + col * 16);
        } else {  // rows past the last key re-read the last key (their scores are masked)
          const int64_t r = min(b0 + row, kend - 1);
          kv = __ldcg(reinterpret_cast<const uint4 *>(kg + r * kAttHd) + col);
          vv = __ldcg(reinterpret_cast<const uint4 *>(vg + r * kAttHd) + col);
        }
        *reinterpret_cast<uint4 *>(sk + row * kAttPadRow + col * 16) = kv;
        *reinterpret_cast<uint4 *>(sv + row * kAttPadRow + col * 16) = vv;
      }
      half_sync(hf);
      if (rb < rbs) {
        float sc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
        const int mi = lane >> 3, mr = lane & 7;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t kb4[4];  // B fragments: keys 0-7 (dims lo, hi), keys 8-15 (dims lo, hi)
          ldsm_x4(kb4, sk + ((mi >> 1) * 8 + mr) * kAttPadRow + (16 * kk + (mi & 1) * 8) * 2);
          mma_bf16(sc[0], qa[kk], kb4[0], kb4[1]);
          mma_bf16(sc[1], qa[kk], kb4[2], kb4[3]);
        }
        // scores -> online softmax of rows lo (regs 0, 1) and hi (regs 2, 3)
        float pv[2][4];
        float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t key = b0 + 8 * nt + 2 * c + e;
            sc[nt][e] = key < k1_lo ? sc[nt][e] * scale : -INFINITY;
            sc[nt][2 + e] = key < k1_hi ? sc[nt][2 + e] * scale : -INFINITY;
            mx_lo = fmaxf(mx_lo, sc[nt][e]);
            mx_hi = fmaxf(mx_hi, sc[nt][2 + e]);
          }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
          mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
          mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
        }
        const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
        // a row that has seen no key yet keeps m = -inf, l = 0 and zero probabilities
        const float cr_lo = mn_lo == -INFINITY ? 1.0f : __expf(m_lo - mn_lo);
        const float cr_hi = mn_hi == -INFINITY ? 1.0f : __expf(m_hi - mn_hi);
        float rs_lo = 0.0f, rs_hi = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            pv[nt][e] = mn_lo == -INFINITY ? 0.0f : __expf(sc[nt][e] - mn_lo);
            pv[nt][2 + e] = mn_hi == -INFINITY ? 0.0f : __expf(sc[nt][2 + e] - mn_hi);
            rs_lo += pv[nt][e];
            rs_hi += pv[nt][2 + e];
          }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {
          rs_lo += __shfl_xor_sync(0xffffffffu, rs_lo, off);
          rs_hi += __shfl_xor_sync(0xffffffffu, rs_hi, off);
        }
        l_lo = l_lo * cr_lo + rs_lo;
        l_hi = l_hi * cr_hi + rs_hi;
        m_lo = mn_lo;
        m_hi = mn_hi;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          o[j][0] *= cr_lo;
          o[j][1] *= cr_lo;
          o[j][2] *= cr_hi;
          o[j][3] *= cr_hi;
        }
        // P (the scores' accumulator layout is the next MMA's A layout) x V
        const uint32_t pa[4] = {pack_bf16(pv[0][0], pv[0][1]), pack_bf16(pv[0][2], pv[0][3]),
                                pack_bf16(pv[1][0], pv[1][1]), pack_bf16(pv[1][2], pv[1][3])};
#pragma unroll
        for (int j2 = 0; j2 < 8; ++j2) {  // dims 16 j2 .. +15: two N tiles
          uint32_t vb[4];  // (keys 0-7, keys 8-15) for dims +0..7, then for dims +8..15
          ldsm_x4_trans(vb, sv + ((mi & 1) * 8 + mr) * kAttPadRow + (16 * j2 + (mi >> 1) * 8) * 2);
          mma_bf16(o[2 * j2], pa, vb[0], vb[1]);
          mma_bf16(o[2 * j2 + 1], pa, vb[2], vb[3]);
        }
      }
      half_sync(hf);  // the half's staged block is free again
    }
    if (rb < rbs) {
      // this half's partial of rows lo and hi (tokens past T write nothing)
      const int part = sp * 2 + hf;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int t = rr == 0 ? t_lo : t_hi;
        if (t >= T) continue;
        float *out = p.att_part +
                     ((static_cast<int64_t>(t) * op.q_heads + kvh * kAttGroup + hq) * op.att_parts + part) * kAttRow;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          *reinterpret_cast<float2 *>(out + 8 * j + 2 * c) = make_float2(o[j][2 * rr], o[j][2 * rr + 1]);
        if (c == 0) {
          out[kAttHd] = rr == 0 ? m_lo : m_hi;
          out[kAttHd + 1] = rr == 0 ? l_lo : l_hi;
        }
      }
    }
    NQB_ATT_TRACE(kTraceMma);
  } else {
  for (int t = seqs ? tu : 0; t < (seqs ? tu + 1 : T); ++t) {
    const int64_t k0 = static_cast<int64_t>(sp) * op.att_chunk;
    const int64_t k1 = min(k0 + op.att_chunk, op.position + 1 + (seqs ? 0 : t));
    float acc[kAttGroup][4], m[kAttGroup], l[kAttGroup];
    token_keys(t, k0, k1, k0 + warp * kAttSub, static_cast<int64_t>(kAttSub) * mmad::kWarps, acc, m, l);
    NQB_ATT_TRACE(kTraceMma);
    // the warps' partials -> shared memory [warp][head][kAttRow]
#pragma unroll
    for (int h = 0; h < kAttGroup; ++h) {
      float *row = scratch + (warp * kAttGroup + h) * kAttRow;
      *reinterpret_cast<float4 *>(row + lane * 4) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
      if (lane == 0) {
        row[kAttHd] = m[h];
        row[kAttHd + 1] = l[h];
      }
    }
    mmad::consumer_sync();
    {
      // thread tid: head tid / 64, dims 2 (tid % 64) .. +1; warps joined in index order
      const int h = tid >> 6, d = (tid & 63) * 2;
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < mmad::kWarps; ++w) mx = fmaxf(mx, scratch[(w * kAttGroup + h) * kAttRow + kAttHd]);
      float a0 = 0.0f, a1 = 0.0f, ls = 0.0f;
#pragma unroll
      for (int w = 0; w < mmad::kWarps; ++w) {
        const float *row = scratch + (w * kAttGroup + h) * kAttRow;
        const float mw = row[kAttHd];
        const float f = mw == -INFINITY ? 0.0f : __expf(mw - mx);
        a0 += f * row[d];
        a1 += f * row[d + 1];
        ls += f * row[kAttHd + 1];
      }
      float *out = p.att_part +
                   ((static_cast<int64_t>(t) * op.q_heads + kvh * kAttGroup + h) * op.att_parts + sp) * kAttRow;
      *reinterpret_cast<float2 *>(out + d) = make_float2(a0, a1);
      if ((tid & 63) == 0) {
        out[kAttHd] = mx;
        out[kAttHd + 1] = ls;
      }
    }
    mmad::consumer_sync();  // the scratch is reused by the next token
    NQB_ATT_TRACE(kTraceDrain);
  }
  }
#undef NQB_ATT_TRACE
  // every warp is done with the unit's ring blocks: hand them back
  if (lane == 0)
    for (int j = 0; j < 2 * nb; ++j) mbar_arrive_cta(&s_empty[(slot + j) % R]);
  phase += static_cast<uint32_t>((slot + 2 * nb) / R);
  slot = (slot + 2 * nb) % R;
}

// Joins the splits' partials of every (token, q head) in split order, one
// warp per row (lane: 4 dims), and writes the bf16 attention output.
__device__ __forceinline__ void attention_join(const Params &p, const StepDev &op) {
  const int rows = p.tokens * op.q_heads;
  const int lane = threadIdx.x & 31;
  const int stride = static_cast<int>(gridDim.x) * mmad::kWarps;
  for (int r = static_cast<int>(blockIdx.x) * mmad::kWarps + (threadIdx.x >> 5); r < rows; r += stride) {
    const float *base = p.att_part + static_cast<int64_t>(r) * op.att_parts * kAttRow;
    const float m0 = lane < op.att_parts ? __ldcg(base + lane * kAttRow + kAttHd) : -INFINITY;
    const float l0 = lane < op.att_parts ? __ldcg(base + lane * kAttRow + kAttHd + 1) : 0.0f;
    // the splits' vectors, kJoin at a time, all in flight together (issued before the weights are known)
    constexpr int kJoin = 16;
    float4 v[kJoin];
#pragma unroll
    for (int u = 0; u < kJoin; ++u)
      v[u] = __ldcg(reinterpret_cast<const float4 *>(base + min(u, op.att_parts - 1) * kAttRow + lane * 4));
    float mx = m0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float f0 = m0 == -INFINITY ? 0.0f : __expf(m0 - mx);
    float den = f0 * l0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
    float num[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int s0 = 0; s0 < op.att_parts; s0 += kJoin) {
      if (s0 > 0) {
#pragma unroll
        for (int u = 0; u < kJoin; ++u)
          v[u] = __ldcg(
              reinterpret_cast<const float4 *>(base + min(s0 + u, op.att_parts - 1) * kAttRow + lane * 4));
      }
#pragma unroll
      for (int u = 0; u < kJoin; ++u) {
        const float f = __shfl_sync(0xffffffffu, f0, (s0 + u) & 31);
        if (s0 + u < op.att_parts) {
          num[0] += f * v[u].x;
          num[1] += f * v[u].y;
          num[2] += f * v[u].z;
          num[3] += f * v[u].w;
        }
      }
    }
    const float inv = den > 0.0f ? 1.0f / den : 0.0f;
    __nv_bfloat16 *o = op.attn_out + static_cast<int64_t>(r) * kAttHd + lane * 4;
    *reinterpret_cast<__nv_bfloat162 *>(o) = __floats2bfloat162_rn(num[0] * inv, num[1] * inv);
    *reinterpret_cast<__nv_bfloat162 *>(o + 2) = __floats2bfloat162_rn(num[2] * inv, num[3] * inv);
  }
}

// NQB_EPI_RESIDUAL for one tile (the 128 leader threads): h += out, and the
// tile's sums of squares of the new h per token to out_stats.
template <int kT>
__device__ __forceinline__ void residual_epilogue(const StepDev &op, const MemberDev &md, int tile, const float (&outv)[kT],
                                                  const float (&hprev)[kT], int T, float *red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = static_cast<int64_t>(tile) * kTileRows + tid;
  float sq[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    sq[t] = 0.0f;
    if (t < T && row < md.rows) {
      const float hn = hprev[t] + outv[t];  // hprev: h of this row, loaded with the row scales
      md.y[static_cast<int64_t>(t) * md.rows + row] = hn;
      sq[t] = hn * hn;
    }
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    const float w = warp_sum(sq[t]);
    if (lane == 0) red[warp * kT + t] = w;
  }
  leader_sync();
  if (tid < T) op.out_stats[static_cast<int64_t>(tile) * T + tid] = (red[tid] + red[kT + tid]) + (red[2 * kT + tid] + red[3 * kT + tid]);
  leader_sync();  // red is reused by the next tile
}

// NQB_EPI_QK_ROPE for one tile = one head (the 128 leader threads, d = tid):
// q and k heads get RMSNorm and rotate-half RoPE, v heads are copied; all go
// out as bf16 (q to op.q, k and v to the caches at row position + t).
template <int kT>
__device__ __forceinline__ void qk_rope_epilogue(const StepDev &op, int member, int tile, const float (&outv)[kT], int T,
                                                 float *xs, float *red) {
  const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
  if (member == 2) {
#pragma unroll
    for (int t = 0; t < kT; ++t)
      if (t < T)
        op.v_cache[att_new_row(op, t, tile) + d] = __float2bfloat16_rn(outv[t]);
    return;
  }
  const float *w = member == 0 ? op.q_norm : op.k_norm;
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    const float ss = warp_sum(t < T ? outv[t] * outv[t] : 0.0f);
    if (lane == 0) red[warp * kT + t] = ss;
  }
  leader_sync();
  const float wd = w != nullptr ? w[d] : 1.0f;
  float xn[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    xn[t] = outv[t];
    if (t < T && w != nullptr) {
      const float ss = (red[t] + red[kT + t]) + (red[2 * kT + t] + red[3 * kT + t]);
      xn[t] = outv[t] * rsqrtf(ss / static_cast<float>(kAttHd) + op.eps) * wd;
    }
    if (t < T) xs[t * kAttHd + d] = xn[t];
  }
  leader_sync();
  const float sign = d < kAttHd / 2 ? -1.0f : 1.0f;  // rotate_half: (-x2, x1)
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    if (t >= T) break;
    const float partner = xs[t * kAttHd + (d ^ (kAttHd / 2))];
    const float o = xn[t] * op.cos_t[t * kAttHd + d] + sign * partner * op.sin_t[t * kAttHd + d];
    if (member == 0)
      op.q[(static_cast<int64_t>(t) * op.q_heads + tile) * kAttHd + d] = __float2bfloat16_rn(o);
    else
      op.k_cache[att_new_row(op, t, tile) + d] = __float2bfloat16_rn(o);
  }
  leader_sync();  // xs and red are reused by the next tile
}

// A CTA's exit steps, run by every warp: a failed wait is recorded, every CTA
// stays until its cluster peers have made their last remote arrivals, and the
// last CTA of the grid zeroes the barrier counters for the next run.
__device__ __forceinline__ void finish_cta(const Params &p, bool ok) {
  if (!ok) record_error(NQB_ERR_TIMEOUT);
  cluster_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t finished = atomicAdd(p.counters + 1, 1u);
    if (finished == gridDim.x - 1) {
      p.counters[0] = 0;
      p.counters[1] = 0;
      __threadfence();
    }
  }
}

// kPatch: some op has a patched member or int8 overlay rows; kMixed: some member streams coded
// mixed-V tiles; kStep: some op uses the decoder-step extensions (residual
// input norm, fused epilogues, attention).  Programs without them run
// instances with those steps compiled out (the steps cost time in the stage
// loop even when never taken).
template <int kT, bool kPatch, bool kMixed, bool kStep>
__global__ void __launch_bounds__(kBlockThreads, 1) program_kernel(const __grid_constant__ Params p) {
  constexpr int kNT = mmad::n_tiles(kT);
  constexpr int kSets = mmad::acc_sets(kNT);
  constexpr int kQPT = mmad::quads_per_thread(slices_per_chunk(kT));
  constexpr bool kPrefetchUnits = kT == 1;  // two chunks of activations in registers only at one token
  constexpr bool kPreQ = pre_quantised(kT);  // linear stages quantise their activation chunks once, grid-wide
  constexpr int kLead = leader_slots(kT);  // tiles this CTA leads per exchange group
  constexpr int kC = mmad::kThreads;  // consumer threads
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t s_full[kMaxRing], s_empty[kMaxRing];
  __shared__ uint64_t s_addr_bar[kAddrSlots];
  __shared__ uint64_t s_x_full;  // this CTA's leader buffers hold every quarter (own expect_tx + st.async bytes)
  __shared__ uint64_t s_x_free;  // every leader has read this CTA's quarters (one arrival per leader)
  __shared__ uint64_t s_info_full[2];  // s_info[b] holds the next stage of parity b
  __shared__ uint64_t s_info_free[2];  // the consumers are done with s_info[b]'s stage
  __shared__ StageInfo s_info[2];
  __shared__ mmad::Scratch<kT> s_sc;
  __shared__ uint64_t s_patch_done;  // the side warps formed this CTA's side rows of the current stage 1
  __shared__ float s_rms[kT];        // residual-stream input: the stage's per-token norm factors

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t cluster = cluster_id();
  const int cta = static_cast<int>(blockIdx.x);
  const int T = p.tokens;
  const int R = p.ring;

  uint8_t *ring = smem;
  uint64_t *addr_cache = reinterpret_cast<uint64_t *>(smem + p.off_addr);
  uint8_t *smem_b = smem + p.off_b;
  float *s_acc = reinterpret_cast<float *>(smem + p.off_acc);    // [group][T][128]
  float *s_exch = reinterpret_cast<float *>(smem + p.off_exch);  // [group / 4][4][T][128]
  float *s_epi = reinterpret_cast<float *>(smem + p.off_epi);    // [T][128] then [4][kT] (fused epilogues)

  if (tid == 0) {
    for (int s = 0; s < R; ++s) {
      ptx::mbar_init(&s_full[s], 1);
      ptx::mbar_init(&s_empty[s], mmad::kWarps);
    }
    for (int s = 0; s < kAddrSlots; ++s) ptx::mbar_init(&s_addr_bar[s], 1);
    ptx::mbar_init(&s_x_full, 1);
    ptx::mbar_init(&s_x_free, kClusterSize);
    ptx::mbar_init(&s_info_full[0], 1);
    ptx::mbar_init(&s_info_full[1], 1);
    ptx::mbar_init(&s_info_free[0], 1);
    ptx::mbar_init(&s_info_free[1], 1);
    ptx::mbar_init(&s_patch_done, 1);
    ptx::fence_mbar_init();
  }
  cluster_sync();  // every CTA's barriers exist before any remote arrive
  // Each warpgroup runs its roles inside one branch that starts with its
  // register split (setmaxnreg is warpgroup-uniform) and ends with the CTA's
  // exit steps, so no code is shared between the two register budgets.
  //
  // Run by nqb_program_run_dependent, the program is a programmatic dependent
  // of the preceding kernel: only the producer warp runs ahead (sign words,
  // which no kernel writes); every other warp first waits for the preceding
  // kernel to complete (its outputs are this program's inputs).  After a
  // plain launch the wait returns at once.  The split comes first, so the
  // producer's warpgroup never waits on that dependency.
  bool ok = true;
  if (warp >= mmad::kWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kHelperRegs));
    if (warp != kProducerWarp) asm volatile("griddepcontrol.wait;" ::: "memory");
    if (warp == kProducerWarp) {
      // ---- producer: stream this CTA's sign slices through the ring, as far
      // ahead as the ring allows, independent of the stage barriers
      if (lane == 0) {
        Producer prod;
        prod.addrs = p.slice_addrs + p.slice_begin[cta];
        prod.count = p.slice_count[cta];
        prod.padded = ((prod.count + kAddrChunk - 1) / kAddrChunk) * kAddrChunk;
        prod.cache = addr_cache;
        prod.addr_bar = s_addr_bar;
        prod.ring = ring;
        prod.full = s_full;
        prod.ring_slots = R;
        for (int c = 0; c < kAddrSlots; ++c) prod.issue_addr_chunk(c);
        int slot = 0;
        uint32_t phase = 0;  // ring passes completed
        for (int pos = 0; pos < prod.count; ++pos) {
          if (phase > 0 && !wait_local_backoff(&s_empty[slot], (phase - 1) & 1)) ok = false;
          ok &= prod.template produce<kMixed>(pos, slot);
          if (++slot == R) {
            slot = 0;
            ++phase;
          }
        }
      }
      __syncwarp();
    } else if (warp == kInfoWarp) {
      // ---- stage g's tables into s_info[g % 2] and an L2 prefetch of its
      // scales and inputs, once stage g - 1 has started (so stage g - 2, the
      // buffer's previous user, is finished everywhere)
      for (int g = 0; g < p.stages; ++g) {
        if (g >= 2) {
          // stage g - 2 (the buffer's previous user) finished everywhere, so
          // stage g - 1's inputs are complete; then, even when that grid wait
          // gave up, this CTA's consumers are done with the buffer
          if (lane == 0) {
            if (!wait_counter(p.counters, static_cast<uint32_t>(p.bar_end[g - 2] + 1) * gridDim.x + p.barrier_skew,
                              p.barrier_limit))
              ok = false;
            if (!wait_local(&s_info_free[g & 1], ((g >> 1) - 1) & 1)) ok = false;
          }
          __syncwarp();
        }
        stage_info_copy(p, g, cluster, lane, s_info[g & 1]);
        __syncwarp();
        if (lane == 0) {
          // a stage 1 with coded members also brings their tables (the
          // previous stage 1, their last reader, has finished everywhere)
          uint32_t coded = 0;
          if constexpr (kMixed) {
            if ((g & 1) == 0)
              for (int k = 0; k < kMaxMembersTc; ++k) coded += s_info[g & 1].md[k].coded_tiles != nullptr ? 1u : 0u;
          }
          if (coded == 0) {
            mbar_arrive_cta(&s_info_full[g & 1]);
          } else {
            uint32_t *cb = reinterpret_cast<uint32_t *>(smem + p.off_cb);
            expect_tx(&s_info_full[g & 1], coded * kCodebookWords * 4u);
            for (int k = 0; k < kMaxMembersTc; ++k)
              if (s_info[g & 1].md[k].coded_tiles != nullptr)
                bulk_load(cb + k * kCodebookWords, s_info[g & 1].md[k].codebook, kCodebookWords * 4u,
                          &s_info_full[g & 1]);
          }
        }
        prefetch_stage(p, g, lane);
      }
    } else if (kPatch && warp >= kSideWarp) {
      // ---- side warps: for each stage 1 with side rows (patch or overlay
      // rows), once its inputs are complete (the stage before it finished
      // everywhere), this CTA's share of them; then one arrival on s_patch_done
      const int worker = cta * 2 + (warp - kSideWarp);
      for (int g = 0; g < p.stages; g += 2) {
        const OpDev &op = p.ops[g >> 1];
        if (op.side_rows <= 0) continue;
        if (g >= 2) {
          if (lane == 0 &&
              !wait_counter(p.counters, static_cast<uint32_t>(p.bar_end[g - 1] + 1) * gridDim.x + p.barrier_skew,
                            p.barrier_limit))
            ok = false;
          __syncwarp();
        }
        side_rows_warp(p, op, worker, 2 * static_cast<int>(gridDim.x), lane);
        __threadfence();  // the rows are visible GPU-wide before the consumers' barrier release
        asm volatile("bar.sync 3, 64;" ::: "memory");  // both side warps are done
        if (warp == kSideWarp && lane == 0) mbar_arrive_cta(&s_patch_done);
      }
    }
    finish_cta(p, ok);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
    asm volatile("griddepcontrol.wait;" ::: "memory");
    {
      // ---- consumers: 8 warps x 16 rows of the current 128-row tile
      int slot = 0;         // ring slot of the next slice
      uint32_t phase = 0;   // ring passes completed
      uint32_t xg = 0;      // exchange groups done
      uint32_t patched = 0;  // patched stage 1s done
      for (int g = 0; g < p.stages; ++g) {
        const int st = g & 1;
        if (!wait_local(&s_info_full[g & 1], (g >> 1) & 1)) ok = false;
        const StageInfo &op = s_info[g & 1];
        const int ib = 0;
        const int ie = op.n_items;
        NQB_TRACE_BEGIN
        const StepDev &gop = op.step;  // the op's decoder-step fields (staged in shared memory)
        int op_kind = NQB_OP_LINEAR, op_epi = NQB_EPI_STORE;
        bool normed = false;
        float rms_part[kT];  // residual-stream input: warp 0's partial sums of h^2 (lane: tiles lane, lane + 32, ..)
        float rms_next[kT];  // up to two tokens: tile lane + 32, loaded without waiting, added at the reduction
  #pragma unroll
        for (int t = 0; t < kT; ++t) rms_part[t] = rms_next[t] = 0.0f;
        bool rms_pending = false;
        if constexpr (kStep) {
          op_kind = gop.kind;
          op_epi = st == 1 ? gop.epilogue : NQB_EPI_STORE;
          normed = st == 0 && gop.norm_stats != nullptr;
          if (op_kind == NQB_OP_ATTENTION) {
            // split-K partials over the CTAs (stage 1 of the op), then their join;
            // the CTA's exchange buffers are idle during these stages
            NQB_TRACE(kTraceTables);
            if (st == 0)
  #ifdef NQB_PHASE_TRACE
              attention_partials<(kT >= mmad::kWarps)>(p, gop, s_acc, ring, s_full, s_empty, slot, phase, ok, tid == 0 ? trace_c : nullptr);
  #else
              attention_partials<(kT >= mmad::kWarps)>(p, gop, s_acc, ring, s_full, s_empty, slot, phase, ok, nullptr);
  #endif
            else
              attention_join(p, gop);
            if (st == 0) {
              NQB_TRACE_RESET();  // attention_partials added its own phases
            } else {
              NQB_TRACE(kTraceMma);
            }
          } else if (normed) {
            // h's per-tile sums of squares (written before this stage): warp 0
            // issues the loads now and reduces them while the quarters land
            rms_pending = true;
            if (warp == 0) {
              if (kT <= 2 && gop.stat_tiles <= 64) {
                // two independent loads per token, no arithmetic on them before the reduction
  #pragma unroll
                for (int t = 0; t < kT; ++t) {
                  if (t < T && lane < gop.stat_tiles) rms_part[t] = __ldcg(gop.norm_stats + static_cast<int64_t>(lane) * T + t);
                  if (t < T && lane + 32 < gop.stat_tiles)
                    rms_next[t] = __ldcg(gop.norm_stats + static_cast<int64_t>(lane + 32) * T + t);
                }
              } else {
                for (int i = lane; i < gop.stat_tiles; i += 32)
  #pragma unroll
                  for (int t = 0; t < kT; ++t)
                    if (t < T) rms_part[t] += __ldcg(gop.norm_stats + static_cast<int64_t>(i) * T + t);
              }
            }
          }
        }
        // kMixed: item j's slices, the records of a coded tile decoded where a
        // plain tile's words are loaded (whether item j is coded is read once)
        auto mixed_slices = [&](int j, int nst, auto &d) {
          const Item item = op.items[j];
          const uint32_t *cb = (st == 0 && item.tile >= op.md[item.member].coded_from)
                                   ? reinterpret_cast<const uint32_t *>(smem + p.off_cb) + item.member * kCodebookWords
                                   : nullptr;
          const bool product = op.md[item.member].coded_format == NQB_CODED_PRODUCT_CODEBOOK;
          for (int sl = 0; sl < nst; ++sl) {
            if (!wait_local(&s_full[slot], phase & 1)) ok = false;
            const uint8_t *src = ring + static_cast<size_t>(slot) * kStageWeightBytes;
            mmad::SliceWords w;
            if (cb != nullptr) {
              const int r0 = warp * 16 + (lane >> 2), tig = lane & 3;
              if (product) {
                w.w00 = decode_product_record(cb, src, r0, tig);
                w.w10 = decode_product_record(cb, src, r0 + 8, tig);
                w.w01 = decode_product_record(cb, src, r0, 4 + tig);
                w.w11 = decode_product_record(cb, src, r0 + 8, 4 + tig);
              } else {
                const uint32_t *rw = reinterpret_cast<const uint32_t *>(src);
                w.w00 = decode_record(cb, coded_record(rw, r0, tig));
                w.w10 = decode_record(cb, coded_record(rw, r0 + 8, tig));
                w.w01 = decode_record(cb, coded_record(rw, r0, 4 + tig));
                w.w11 = decode_record(cb, coded_record(rw, r0 + 8, 4 + tig));
              }
            } else {
              w = mmad::load_slice_words(src, warp, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(&s_empty[slot]);
            if (++slot == R) {
              slot = 0;
              ++phase;
            }
            mmad::slice_mmas<kNT>(w, smem_b + static_cast<size_t>(sl) * mmad::slice_frag_bytes(kNT), lane, d);
          }
        };
        // one chunk of this stage's activations -> B fragments in smem_b, with
        // per-token exponents e and digit sums Q
        auto quantize_input = [&](const MemberDev &md, int c0, int nst, int (&e)[kT], long long (&Q)[kT]) {
          const int64_t k0 = static_cast<int64_t>(c0) * kStageCols;
          if (st == 1) {
            const mmad::LatentLoader ld{p.latent, op.latent_stride, md.act_offset, k0, md.k_valid};
            mmad::quantize_chunk<kT, kQPT>(ld, nst, T, smem_b, s_sc, e, Q);
          } else if (op.x_dtype == NQB_X_SWIGLU) {
            const mmad::SwigluLoader ld{static_cast<const float *>(op.x), static_cast<const float *>(op.x2), md.pre,
                                        op.n, k0, md.k_valid};
            mmad::quantize_chunk<kT, kQPT>(ld, nst, T, smem_b, s_sc, e, Q);
          } else if (op.x_dtype == NQB_X_GEGLU) {
            const mmad::GegluLoader ld{static_cast<const float *>(op.x), static_cast<const float *>(op.x2), md.pre,
                                       op.n, k0, md.k_valid};
            mmad::quantize_chunk<kT, kQPT>(ld, nst, T, smem_b, s_sc, e, Q);
          } else if (op.x_dtype == NQB_BF16) {
            const mmad::XLoader<__nv_bfloat16> ld{static_cast<const __nv_bfloat16 *>(op.x), md.pre, op.n, k0,
                                                  md.k_valid};
            mmad::quantize_chunk<kT, kQPT>(ld, nst, T, smem_b, s_sc, e, Q);
          } else if (op.x_dtype == NQB_F16) {
            const mmad::XLoader<__half> ld{static_cast<const __half *>(op.x), md.pre, op.n, k0, md.k_valid};
            mmad::quantize_chunk<kT, kQPT>(ld, nst, T, smem_b, s_sc, e, Q);
          } else {
            const mmad::XLoader<float> ld{static_cast<const float *>(op.x), md.pre, op.n, k0, md.k_valid};
            mmad::quantize_chunk<kT, kQPT>(ld, nst, T, smem_b, s_sc, e, Q);
          }
        };
        const uint32_t q_frag = static_cast<uint32_t>(p.sc) * mmad::slice_frag_bytes(kNT);  // e, then Q follow
        if constexpr (kPreQ) {
          if (op_kind == NQB_OP_LINEAR) {
            // ---- the stage's activation chunks, quantised once over the grid:
            // unit u = (chunk u / groups, tokens 2 (u % groups) ..) by CTA u mod
            // grid, each writing its half N tile of the chunk's fragments and
            // its tokens' e and Q into the chunk's slot; then a grid barrier
            constexpr int kG = 2;
            constexpr int kGroups = kT / kG;
            int k = 0, c0 = 0, nst = 0;
            for (int u = cta;; u += static_cast<int>(gridDim.x)) {
              const int cu = u / kGroups, t0 = (u - cu * kGroups) * kG;
              if (!unit_at(op, cu, p.sc, k, c0, nst)) break;
              if (t0 >= T) continue;
              const MemberDev &md = op.md[k];
              const int64_t k0 = static_cast<int64_t>(c0) * kStageCols;
              int e[kG];
              long long Q[kG];
              if (st == 1) {
                const mmad::LatentLoader ld{p.latent, op.latent_stride, md.act_offset, k0, md.k_valid};
                mmad::quantize_tokens<kT, kG, kQPT>(ld, nst, t0, T, smem_b, s_sc, e, Q);
              } else if (op.x_dtype == NQB_X_SWIGLU) {
                const mmad::SwigluLoader ld{static_cast<const float *>(op.x), static_cast<const float *>(op.x2),
                                            md.pre, op.n, k0, md.k_valid};
                mmad::quantize_tokens<kT, kG, kQPT>(ld, nst, t0, T, smem_b, s_sc, e, Q);
              } else if (op.x_dtype == NQB_X_GEGLU) {
                const mmad::GegluLoader ld{static_cast<const float *>(op.x), static_cast<const float *>(op.x2),
                                           md.pre, op.n, k0, md.k_valid};
                mmad::quantize_tokens<kT, kG, kQPT>(ld, nst, t0, T, smem_b, s_sc, e, Q);
              } else if (op.x_dtype == NQB_BF16) {
                const mmad::XLoader<__nv_bfloat16> ld{static_cast<const __nv_bfloat16 *>(op.x), md.pre, op.n, k0,
                                                      md.k_valid};
                mmad::quantize_tokens<kT, kG, kQPT>(ld, nst, t0, T, smem_b, s_sc, e, Q);
              } else if (op.x_dtype == NQB_F16) {
                const mmad::XLoader<__half> ld{static_cast<const __half *>(op.x), md.pre, op.n, k0, md.k_valid};
                mmad::quantize_tokens<kT, kG, kQPT>(ld, nst, t0, T, smem_b, s_sc, e, Q);
              } else {
                const mmad::XLoader<float> ld{static_cast<const float *>(op.x), md.pre, op.n, k0, md.k_valid};
                mmad::quantize_tokens<kT, kG, kQPT>(ld, nst, t0, T, smem_b, s_sc, e, Q);
              }
              // (the quantiser ends with a consumer barrier after its fragment writes)
              uint8_t *dst = p.qbuf + static_cast<size_t>(cu) * p.qunit_bytes;
              const int n0 = 2 * t0;  // first N column of the group (two digits per token)
              const uint32_t part = static_cast<uint32_t>(n0 >> 3) * mmad::kFragBytes + ((n0 & 7) >> 2) * 128u;
              for (int i = tid; i < nst * 8 * 8; i += kC) {  // 8 fragment blocks per slice, 8 x 16 bytes each
                const uint32_t off = static_cast<uint32_t>(i >> 3) * kNT * mmad::kFragBytes + part + (i & 7) * 16u;
                *reinterpret_cast<uint4 *>(dst + off) = *reinterpret_cast<const uint4 *>(smem_b + off);
              }
              if (tid == 0) {
#pragma unroll
                for (int t = 0; t < kG; ++t) {
                  reinterpret_cast<int32_t *>(dst + q_frag)[t0 + t] = e[t];
                  reinterpret_cast<long long *>(dst + q_frag + 4 * kT)[t0 + t] = Q[t];
                }
              }
            }
            grid_barrier(p, static_cast<uint32_t>(p.bar_end[g] - 1), nullptr);
            NQB_TRACE(kTraceQuantise);
          }
        }
        // this CTA's pre-quantised unit u: fragments -> smem_b, e and Q
        auto load_quantised = [&](int u, int nst, int (&e)[kT], long long (&Q)[kT]) {
          mmad::consumer_sync();  // every warp is done with the previous chunk's fragments
          const uint8_t *src = p.qbuf + static_cast<size_t>(u) * p.qunit_bytes;
          const uint32_t fb = static_cast<uint32_t>(nst) * mmad::slice_frag_bytes(kNT);
          for (uint32_t i = static_cast<uint32_t>(tid) * 16; i < fb; i += kC * 16)
            *reinterpret_cast<uint4 *>(smem_b + i) = __ldcg(reinterpret_cast<const uint4 *>(src + i));
#pragma unroll
          for (int t = 0; t < kT; ++t) {
            e[t] = __ldcg(reinterpret_cast<const int32_t *>(src + q_frag) + t);
            Q[t] = __ldcg(reinterpret_cast<const long long *>(src + q_frag + 4 * kT) + t);
          }
          mmad::consumer_sync();
        };
        for (int gb = ib; gb < ie; gb += p.group) {
          const int ge = min(gb + p.group, ie);
          for (int i = tid; i < (ge - gb) * T * kTileRows; i += kC) s_acc[i] = 0.0f;
          if constexpr (kPrefetchUnits) {
            // ---- this CTA's quarter of every item of the group, one (member run,
            // chunk) unit at a time.  At one token the next unit's activation
            // loads are issued before this unit's MMAs, so their L2 round trip
            // is hidden behind the MMAs instead of opening the next unit.
            auto load_unit = [&](int j, int c0, int hi, mmad::ChunkValues<kT, kQPT> &cv) {
              const MemberDev &md = op.md[op.items[j].member];
              const int nst = min(p.sc, hi - c0);
              const int64_t k0 = static_cast<int64_t>(c0) * kStageCols;
              if (st == 1) {
                mmad::load_chunk<kT, kQPT>(mmad::LatentLoader{p.latent, op.latent_stride, md.act_offset, k0, md.k_valid},
                                           nst, T, cv);
              } else if (op.x_dtype == NQB_X_SWIGLU) {
                mmad::load_chunk<kT, kQPT>(mmad::SwigluLoader{static_cast<const float *>(op.x),
                                                              static_cast<const float *>(op.x2), md.pre, op.n, k0,
                                                              md.k_valid},
                                           nst, T, cv);
              } else if (op.x_dtype == NQB_X_GEGLU) {
                mmad::load_chunk<kT, kQPT>(mmad::GegluLoader{static_cast<const float *>(op.x),
                                                             static_cast<const float *>(op.x2), md.pre, op.n, k0,
                                                             md.k_valid},
                                           nst, T, cv);
              } else if (op.x_dtype == NQB_BF16) {
                mmad::load_chunk<kT, kQPT>(mmad::XLoader<__nv_bfloat16>{static_cast<const __nv_bfloat16 *>(op.x), md.pre,
                                                                       op.n, k0, md.k_valid},
                                           nst, T, cv);
              } else if (op.x_dtype == NQB_F16) {
                mmad::load_chunk<kT, kQPT>(
                    mmad::XLoader<__half>{static_cast<const __half *>(op.x), md.pre, op.n, k0, md.k_valid}, nst, T, cv);
              } else {
                mmad::load_chunk<kT, kQPT>(
                    mmad::XLoader<float>{static_cast<const float *>(op.x), md.pre, op.n, k0, md.k_valid}, nst, T, cv);
              }
            };
            int j0 = gb, j1 = gb, c0 = 0, hi = 0;
            bool have = next_unit(op, ge, static_cast<int>(rank), p.sc, j0, j1, c0, hi);
            mmad::ChunkValues<kT, kQPT> cur;
            if (have) load_unit(j0, c0, hi, cur);
            while (have) {
              int nj0 = j0, nj1 = j1, nc0 = c0, nhi = hi;
              const bool more = next_unit(op, ge, static_cast<int>(rank), p.sc, nj0, nj1, nc0, nhi);
              mmad::ChunkValues<kT, kQPT> nxt;
              if (kPrefetchUnits && more) load_unit(nj0, nc0, nhi, nxt);
              const int nst = min(p.sc, hi - c0);
              int e[kT];
              long long Q[kT];
              NQB_TRACE(kTraceTables);
              mmad::quantize_loaded<kT, kQPT>(cur, nst, T, smem_b, s_sc, e, Q);
              NQB_TRACE(kTraceQuantise);
              for (int j = j0; j < j1; ++j) {
                int32_t d[kSets][kNT][4];
    #pragma unroll
                for (int c = 0; c < kSets; ++c)
    #pragma unroll
                  for (int nt = 0; nt < kNT; ++nt)
    #pragma unroll
                    for (int r = 0; r < 4; ++r) d[c][nt][r] = 0;
                if constexpr (kMixed) {
                  mixed_slices(j, nst, d);
                } else {
                  for (int sl = 0; sl < nst; ++sl) {
                    NQB_TRACE(kTraceMma);
                    if (!wait_local(&s_full[slot], phase & 1)) ok = false;
                    NQB_TRACE(kTraceWaitSigns);
                    const mmad::SliceWords w =
                        mmad::load_slice_words(ring + static_cast<size_t>(slot) * kStageWeightBytes, warp, lane);
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cta(&s_empty[slot]);
                    if (++slot == R) {
                      slot = 0;
                      ++phase;
                    }
                    mmad::slice_mmas<kNT>(w, smem_b + static_cast<size_t>(sl) * mmad::slice_frag_bytes(kNT), lane, d);
                  }
                }
                NQB_TRACE(kTraceMma);
                mmad::drain_to_acc<kT>(d, T, warp, lane, e, Q, s_acc + static_cast<size_t>(j - gb) * T * kTileRows);
                NQB_TRACE(kTraceDrain);
              }
              j0 = nj0;
              j1 = nj1;
              c0 = nc0;
              hi = nhi;
              have = more;
              if (have) {
                if constexpr (kPrefetchUnits) {
                  cur = nxt;
                } else {
                  load_unit(j0, c0, hi, cur);
                }
              }
            }
          } else {
            // ---- this CTA's quarter of every item of the group, member by member
            for (int j0 = gb; j0 < ge;) {
              const int mi = op.items[j0].member;
              int j1 = j0 + 1;
              while (j1 < ge && op.items[j1].member == mi) ++j1;
              const MemberDev &md = op.md[mi];
              const int lo = md.ks * static_cast<int>(rank) / kClusterSize;
              const int hi = md.ks * (static_cast<int>(rank) + 1) / kClusterSize;
              for (int c0 = lo; c0 < hi; c0 += p.sc) {
                const int nst = min(p.sc, hi - c0);
                int e[kT];
                long long Q[kT];
                NQB_TRACE(kTraceTables);
                if constexpr (kPreQ)
                  load_quantised(unit_of(op, mi, static_cast<int>(rank), c0, p.sc), nst, e, Q);
                else
                  quantize_input(md, c0, nst, e, Q);
                NQB_TRACE(kTraceQuantise);
                for (int j = j0; j < j1; ++j) {
                  int32_t d[kSets][kNT][4];
    #pragma unroll
                  for (int c = 0; c < kSets; ++c)
    #pragma unroll
                    for (int nt = 0; nt < kNT; ++nt)
    #pragma unroll
                      for (int r = 0; r < 4; ++r) d[c][nt][r] = 0;
                  if constexpr (kMixed) {
                    mixed_slices(j, nst, d);
                  } else {
                    for (int sl = 0; sl < nst; ++sl) {
                      NQB_TRACE(kTraceMma);
                      if (!wait_local(&s_full[slot], phase & 1)) ok = false;
                      NQB_TRACE(kTraceWaitSigns);
                      const mmad::SliceWords w =
                          mmad::load_slice_words(ring + static_cast<size_t>(slot) * kStageWeightBytes, warp, lane);
                      __syncwarp();
                      if (lane == 0) mbar_arrive_cta(&s_empty[slot]);
                      if (++slot == R) {
                        slot = 0;
                        ++phase;
                      }
                      mmad::slice_mmas<kNT>(w, smem_b + static_cast<size_t>(sl) * mmad::slice_frag_bytes(kNT), lane, d);
                    }
                  }
                  NQB_TRACE(kTraceMma);
                  mmad::drain_to_acc<kT>(d, T, warp, lane, e, Q, s_acc + static_cast<size_t>(j - gb) * T * kTileRows);
                  NQB_TRACE(kTraceDrain);
                }
              }
              j0 = j1;
            }
          }
          // ---- quarters -> leaders: asynchronous stores into their shared
          // memory, counted on each leader's s_x_full
          if (xg > 0 && !wait_cluster(&s_x_free, (xg - 1) & 1)) ok = false;
          mmad::consumer_sync();  // every lane's accumulation is in s_acc
          const int per_item = T * kTileRows;
          if (tid == 0) {
            const int led = (ge - gb - static_cast<int>(rank) + kClusterSize - 1) / kClusterSize;
            expect_tx(&s_x_full, static_cast<uint32_t>(led > 0 ? led : 0) * kClusterSize * per_item * 4);
          }
          for (int i = tid * 4; i < (ge - gb) * per_item; i += kC * 4) {
            const int jj = i / per_item;
            const int rest = i - jj * per_item;
            float *dst = s_exch + (static_cast<size_t>(jj / kClusterSize) * kClusterSize + rank) * per_item + rest;
            st_async_v4(dst, static_cast<uint32_t>(jj % kClusterSize), *reinterpret_cast<const float4 *>(s_acc + i),
                        &s_x_full);
          }
          // leaders load the row scales and bias of their tiles while the quarters land
          float lead_scale[kLead], lead_bias[kLead];
          float lead_h[kStep ? kLead : 1][kT];  // residual epilogues: h of the led rows, loaded early
          int lead_slot[kPatch ? kLead : 1];    // int8 overlay rows: the led rows' overlay row index (-1: none)
  #pragma unroll
          for (int sidx = 0; sidx < kLead; ++sidx) {
            lead_scale[sidx] = 0.0f;
            lead_bias[sidx] = 0.0f;
            if constexpr (kPatch) lead_slot[sidx] = -1;
            if constexpr (kStep) {
  #pragma unroll
              for (int t = 0; t < kT; ++t) lead_h[sidx][t] = 0.0f;
            }
            const int jj = static_cast<int>(rank) + sidx * kClusterSize;
            if (jj < ge - gb && tid < kTileRows) {
              const Item item = op.items[gb + jj];
              const MemberDev &md = op.md[item.member];
              const int64_t row = static_cast<int64_t>(item.tile) * kTileRows + tid;
              if (row < md.rows) {
                lead_scale[sidx] = __ldg(md.row_scale + row);
                if (md.bias != nullptr) lead_bias[sidx] = __ldg(md.bias + row);
                if constexpr (kPatch) {
                  if (md.overlay_slot != nullptr) lead_slot[sidx] = __ldg(md.overlay_slot + row);
                }
                if constexpr (kStep) {
                  if (op_epi == NQB_EPI_RESIDUAL)
  #pragma unroll
                    for (int t = 0; t < kT; ++t)
                      if (t < T) lead_h[sidx][t] = __ldcg(md.y + static_cast<int64_t>(t) * md.rows + row);
                }
              }
            }
          }
          if constexpr (kStep) {
            if (rms_pending) {  // the norm factors, read by the leader epilogue after the next consumer barrier
              if (warp == 0) {
  #pragma unroll
                for (int t = 0; t < kT; ++t) {
                  const float ss = warp_sum(rms_part[t] + rms_next[t]);
                  if (lane == 0 && t < T) s_rms[t] = rsqrtf(ss * gop.inv_n + gop.eps);
                }
              }
              rms_pending = false;
            }
          }
          NQB_TRACE(kTraceSend);
          if (!wait_cluster(&s_x_full, xg & 1)) ok = false;
          NQB_TRACE(kTraceWaitQuarters);
          // ---- leaders: fixed-order sum of the four quarters into registers,
          // then release the exchange buffers before any global store
          float vsum[kLead][kT];
  #pragma unroll
          for (int sidx = 0; sidx < kLead; ++sidx) {
            const int jj = static_cast<int>(rank) + sidx * kClusterSize;
            const float *ex = s_exch + static_cast<size_t>(sidx) * kClusterSize * per_item;
  #pragma unroll
            for (int t = 0; t < kT; ++t) {
              float v = 0.0f;
              if (jj < ge - gb && t < T && tid < kTileRows) {
  #pragma unroll
                for (int q = 0; q < kClusterSize; ++q) v += ex[(q * T + t) * kTileRows + tid];
              }
              vsum[sidx][t] = v;
            }
          }
          NQB_TRACE(kTraceSum);
          mmad::consumer_sync();  // done reading this CTA's leader buffers
          if (tid == 0)
            for (uint32_t r = 0; r < kClusterSize; ++r) remote_arrive_relaxed(&s_x_free, r);
          ++xg;
          NQB_TRACE(kTraceRelease);
          // ---- epilogue of the led tiles
  #pragma unroll
          for (int sidx = 0; sidx < kLead; ++sidx) {
            const int jj = static_cast<int>(rank) + sidx * kClusterSize;
            if (jj >= ge - gb) break;
            const Item item = op.items[gb + jj];
            const MemberDev &md = op.md[item.member];
            float outv[kT];  // stage-2 values for the fused epilogues
  #pragma unroll
            for (int t = 0; t < kT; ++t) outv[t] = 0.0f;
            if (tid < kTileRows) {
              const int64_t row = static_cast<int64_t>(item.tile) * kTileRows + tid;
              if (row < md.rows) {
  #pragma unroll
                for (int t = 0; t < kT; ++t) {
                  if (t >= T) break;
                  float v = vsum[sidx][t];
                  if (st == 0) {
                    float f = lead_scale[sidx];
                    if constexpr (kStep) {
                      if (normed) f *= s_rms[t];
                    }
                    p.latent[static_cast<int64_t>(t) * op.latent_stride + md.out_offset + row] = v * f;
                  } else {
                    v *= lead_scale[sidx];
                    if (md.outlier_count > 0) {
                      float sal = 0.0f;
                      for (int64_t s = 0; s < md.outlier_count; ++s) {
                        float w = load_as_float(md.outlier_values, row * md.outlier_count + s, md.outlier_value_dtype);
                        if (md.outlier_scales != nullptr) w *= load_as_float(md.outlier_scales, s, md.outlier_scale_dtype);
                        sal += load_as_float(op.x, static_cast<int64_t>(t) * op.n + md.outlier_indices[s], op.x_dtype) *
                               w;
                      }
                      v += sal;
                    }
                    if constexpr (kPatch) {
                      if (md.patch_rank > 0) {
                        const float *pl = p.latent + static_cast<int64_t>(t) * op.latent_stride + md.patch_offset;
                        float pv = 0.0f;
                        for (int64_t q = 0; q < md.patch_rank; ++q)
                          pv += load_as_float(md.patch_factor, row * md.patch_rank + q, md.patch_dtype) * __ldcg(pl + q);
                        v += pv;
                      }
                      // the row's int8 overlay value (formed in stage 1 by the side-row warps)
                      if (lead_slot[sidx] >= 0) {
                        const float *ov = p.latent + static_cast<int64_t>(t) * op.latent_stride + md.overlay_offset +
                                          static_cast<int64_t>(lead_slot[sidx]) * op.ovl_segs;
                        float o = 0.0f;
                        for (int sg = 0; sg < op.ovl_segs; ++sg) o += __ldcg(ov + sg);
                        v += o;
                      }
                    }
                    if (kStep && op_epi != NQB_EPI_STORE)
                      outv[t] = v + lead_bias[sidx];
                    else
                      md.y[static_cast<int64_t>(t) * md.rows + row] = v + lead_bias[sidx];
                  }
                }
              }
            }
            if constexpr (kStep) {
              if (op_epi == NQB_EPI_RESIDUAL && tid < kTileRows)
                residual_epilogue<kT>(gop, md, item.tile, outv, lead_h[kStep ? sidx : 0], T, s_epi + kT * kTileRows);
              else if (op_epi == NQB_EPI_QK_ROPE && tid < kTileRows)
                qk_rope_epilogue<kT>(gop, item.member, item.tile, outv, T, s_epi, s_epi + kT * kTileRows);
            }
          }
        }
        NQB_TRACE(kTraceEpilogue);
        if constexpr (kPatch) {
          if (st == 0 && op.side_rows > 0) {
            // this CTA's side rows (side warps) are written before its barrier arrival
            if (tid == 0 && !wait_local(&s_patch_done, patched & 1)) ok = false;
            ++patched;
          }
        }
        if (g + 1 < p.stages) grid_barrier(p, static_cast<uint32_t>(p.bar_end[g]), &s_info_free[g & 1]);
        NQB_TRACE(kTraceGridBarrier);
        NQB_TRACE_FLUSH(g);
      }
    }

    finish_cta(p, ok);
  }
}

// dst[i] *= w[i] (program create time: a norm weight folded into an input scale).
__global__ void mul_f32_kernel(float *dst, const float *w, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] *= w[i];
}

// stats[i][t] = sum over the 128 rows i*128 .. of h[t][row]^2: one warp per (tile, token), fixed order.
__global__ void residual_stats_kernel(const float *h, int64_t tokens, int64_t hidden, float *stats) {
  const int64_t tiles = (hidden + kTileRows - 1) / kTileRows;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= tiles * tokens) return;
  const int64_t tile = w / tokens, t = w - tile * tokens;
  float s = 0.0f;
  for (int64_t r = tile * kTileRows + lane; r < min((tile + 1) * kTileRows, hidden); r += 32) {
    const float v = h[t * hidden + r];
    s += v * v;
  }
  s = warp_sum(s);
  if (lane == 0) stats[tile * tokens + t] = s;
}

// fp32 copy of a scale / bias vector (program create time).
__global__ void to_f32_kernel(const void *src, int32_t dtype, int64_t n, float *dst) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = load_as_float(src, i, dtype);
}

}  // namespace prog
}  // namespace nqb

// --------------------------------------------------------------- host ---

using namespace nqb;

struct nqb_program {
  int device = 0;
  float *scales = nullptr;  // fp32 copies of every pre / mid / post / bias vector
  int64_t tokens = 0;
  int bucket = 1;
  bool patch = false;  // runs the patch-capable kernel instance
  bool mixed = false;  // runs the coded mixed-V instance
  bool step = false;   // runs the decoder-step instance
  size_t att_part_bytes = 0;  // attention partials after the latent in the workspace
  size_t qbuf_bytes = 0;      // pre-quantised activation chunks after the partials
  int ctas = 0;
  int clusters = 0;
  int smem = 0;
  void *arena = nullptr;
  size_t latent_bytes = 0;
  uint32_t barrier_skew = 0;  // tests only: extra arrivals every grid barrier waits for
  prog::Params params{};
};

namespace nqb {
namespace prog {

static int token_bucket(int64_t tokens) {
  return tokens <= 1 ? 1 : tokens <= 2 ? 2 : tokens <= 4 ? 4 : tokens <= 8 ? 8 : 16;
}

// The caches of a step op: one sequence (rows position .. position + tokens
// - 1 new) or `tokens` independent sequences of sequence_stride elements
// each (row `position` new in every one).
static bool cache_layout_ok(const nqb_program_op_ext *e, int64_t tokens) {
  if (e->position < 0) return false;
  if (e->sequence_stride == 0) return e->position + tokens <= e->cache_len;
  return e->sequence_stride > 0 && e->sequence_stride % 8 == 0 && e->position + 1 <= e->cache_len &&
         e->sequence_stride >= static_cast<int64_t>(e->kv_heads) * e->cache_len * kAttHd;
}

struct SmemPlan {
  int sc, group, ring;
  uint32_t off_addr, off_b, off_acc, off_exch, off_cb, off_epi, total;
};

static SmemPlan smem_plan(int bucket, bool mixed) {
  SmemPlan s{};
  s.sc = slices_per_chunk(bucket);
  const int lead = leader_slots(bucket);
  s.group = kClusterSize * lead;
  const uint32_t addr = kAddrSlots * kAddrChunk * 8;
  const uint32_t b = static_cast<uint32_t>(s.sc) * mmad::slice_frag_bytes(mmad::n_tiles(bucket));
  const uint32_t acc = static_cast<uint32_t>(s.group) * bucket * kTileRows * 4;
  const uint32_t exch = static_cast<uint32_t>(lead) * kClusterSize * bucket * kTileRows * 4;
  const uint32_t cb = mixed ? kMaxMembersTc * kCodebookWords * 4u : 0u;
  // fused decoder-step epilogues: [tokens][128] values, then [4][tokens] partial sums
  const uint32_t epi = static_cast<uint32_t>(align_up(static_cast<size_t>(bucket) * (kTileRows + 4) * 4, 16));
  const uint32_t rest = addr + b + acc + exch + cb + epi;
  s.ring = std::min<int>(kMaxRing, static_cast<int>((kMaxDynamicSmem - rest) / kStageWeightBytes));
  uint32_t off = static_cast<uint32_t>(s.ring) * kStageWeightBytes;
  s.off_addr = off;
  off += addr;
  s.off_b = off;
  off += b;
  s.off_acc = off;
  off += acc;
  s.off_exch = off;
  off += exch;
  s.off_cb = off;
  off += cb;
  s.off_epi = off;
  off += epi;
  s.total = off;
  return s;
}

template <bool kPatch, bool kMixed, bool kStep>
static const void *kernel_for_t(int bucket) {
  switch (bucket) {
    case 1: return reinterpret_cast<const void *>(program_kernel<1, kPatch, kMixed, kStep>);
    case 2: return reinterpret_cast<const void *>(program_kernel<2, kPatch, kMixed, kStep>);
    case 4: return reinterpret_cast<const void *>(program_kernel<4, kPatch, kMixed, kStep>);
    case 8: return reinterpret_cast<const void *>(program_kernel<8, kPatch, kMixed, kStep>);
    default: return reinterpret_cast<const void *>(program_kernel<16, kPatch, kMixed, kStep>);
  }
}

// Step programs (decoder-step extensions) take no patched or coded members.
static const void *kernel_for(int bucket, bool patch, bool mixed, bool step) {
  if (step) return kernel_for_t<false, false, true>(bucket);
  if (mixed) return patch ? kernel_for_t<true, true, false>(bucket) : kernel_for_t<false, true, false>(bucket);
  return patch ? kernel_for_t<true, false, false>(bucket) : kernel_for_t<false, false, false>(bucket);
}

// `pre`, `row_scale` and `bias` are the program's fp32 copies of the layer's vectors.
static void fill_member(MemberDev &m, const nqb_linear_desc &d, int stage, int64_t rank_offset, float *y,
                        const float *pre, const float *row_scale, const float *bias) {
  std::memset(&m, 0, sizeof(m));
  m.row_scale = row_scale;
  if (stage == 0) {
    m.tiles = static_cast<const uint8_t *>(d.right_tiles);
    m.rows = d.rank;
    m.wc = repack_chunks(d.in_features);
    m.k_valid = d.in_features;
    m.pre = pre;
    m.out_offset = rank_offset;
    m.patch_factor = d.patch_right;
    if (d.coded_right_tiles != nullptr) {
      m.coded_tiles = static_cast<const uint8_t *>(d.coded_right_tiles);
      m.codebook = reinterpret_cast<const uint32_t *>(d.coded_codebook);
      m.coded_from = static_cast<int32_t>((d.coded_free_rows + kTileRows - 1) / kTileRows);
      m.coded_format = d.coded_format;
    }
  } else {
    m.tiles = static_cast<const uint8_t *>(d.left_tiles);
    m.rows = d.out_features;
    m.wc = repack_chunks(d.rank);
    m.k_valid = d.rank;
    m.act_offset = rank_offset;
    m.bias = bias;
    m.outlier_count = d.outlier_count;
    m.outlier_indices = d.outlier_indices;
    m.outlier_values = d.outlier_values;
    m.outlier_value_dtype = d.outlier_value_dtype;
    m.outlier_scales = d.outlier_scales;
    m.outlier_scale_dtype = d.scale_dtype;
    m.overlay_rows = d.overlay_rows;
    m.overlay_row_ids = d.overlay_row_ids;
    m.overlay_values = d.overlay_values;
    m.overlay_scales = d.overlay_scales;
    m.overlay_scale_dtype = d.overlay_scale_dtype;
    m.y = y;
    m.patch_factor = d.patch_left;
  }
  m.patch_rank = d.patch_rank;
  m.patch_dtype = d.patch_dtype;
  if (m.coded_tiles == nullptr) m.coded_from = INT32_MAX;
  m.ks = m.wc / 2;
}

// Assigns a stage's tiles to clusters (largest cost first onto the least
// loaded cluster), then orders each cluster's tiles by member and tile.
static void assign_stage(const OpDev &op, int stage, int clusters, std::vector<std::vector<Item>> &out) {
  struct Cand {
    Item item;
    int cost;
  };
  std::vector<Cand> cands;
  for (int mi = 0; mi < op.count; ++mi) {
    const MemberDev &m = op.s[stage][mi];
    const int tiles = static_cast<int>((m.rows + kTileRows - 1) / kTileRows);
    for (int t = 0; t < tiles; ++t) cands.push_back({{mi, t}, m.ks});
  }
  std::stable_sort(cands.begin(), cands.end(), [](const Cand &a, const Cand &b) { return a.cost > b.cost; });
  std::vector<int64_t> load(clusters, 0);
  out.assign(clusters, {});
  for (const Cand &c : cands) {
    const int best = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
    load[best] += c.cost;
    out[best].push_back(c.item);
  }
  for (auto &list : out)
    std::sort(list.begin(), list.end(), [](const Item &a, const Item &b) {
      return a.member != b.member ? a.member < b.member : a.tile < b.tile;
    });
}

}  // namespace prog

int program_device_error(int32_t *out) {
  int value = 0;
  NQB_CUDA(cudaMemcpyFromSymbol(&value, prog::g_prog_error, sizeof(int)), "read program error flag");
  *out = value;
  const int zero = 0;
  NQB_CUDA(cudaMemcpyToSymbol(prog::g_prog_error, &zero, sizeof(int)), "clear program error flag");
  return NQB_OK;
}

}  // namespace nqb

extern "C" {

int nqb_program_create(const nqb_program_op *ops, int32_t op_count, int64_t tokens, nqb_program **program) {
  using namespace nqb::prog;
  if (program == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "program is NULL");
  *program = nullptr;
  if (ops == nullptr || op_count < 1) return fail(NQB_ERR_INVALID_ARGUMENT, "a program needs at least one op");
  if (tokens < 1 || tokens > kMaxTokens) return fail(NQB_ERR_UNSUPPORTED, "programs take 1 to %d tokens", kMaxTokens);
  const int bucket = token_bucket(tokens);
  std::vector<OpDev> opdev(op_count);
  int64_t latent_cols = 0;
  bool step = false;
  for (int i = 0; i < op_count; ++i) {
    const nqb_program_op &o = ops[i];
    const nqb_program_op_ext *e = o.ext;
    if (e != nullptr) {
      step = true;
      if (e->kind == NQB_OP_ATTENTION) {
        if (e->head_dim != kAttHd || e->kv_heads < 1 || e->q_heads != kAttGroup * e->kv_heads)
          return fail(NQB_ERR_UNSUPPORTED, "op %d: fused attention takes head_dim %d and %d q heads per kv head", i,
                      kAttHd, kAttGroup);
        if (e->q == nullptr || e->k_cache == nullptr || e->v_cache == nullptr || e->attn_out == nullptr ||
            !cache_layout_ok(e, tokens))
          return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: attention operands or cache position invalid", i);
        if (reinterpret_cast<uintptr_t>(e->q) % 16 || reinterpret_cast<uintptr_t>(e->k_cache) % 16 ||
            reinterpret_cast<uintptr_t>(e->v_cache) % 16 || reinterpret_cast<uintptr_t>(e->attn_out) % 16)
          return fail(NQB_ERR_ALIGNMENT, "op %d: attention operands need 16-byte alignment", i);
        continue;
      }
      if (e->kind != NQB_OP_LINEAR) return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: unknown op kind %d", i, e->kind);
    }
    if (o.layers == nullptr || o.count < 1 || o.count > kMaxMembersTc)
      return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: 1 to %d layers", i, kMaxMembersTc);
    if (o.x == nullptr || o.y == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: x or y is NULL", i);
    const bool swiglu = o.x_dtype == NQB_X_SWIGLU || o.x_dtype == NQB_X_GEGLU;
    if (swiglu && o.x2 == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: a gated input needs x2", i);
    if (swiglu)
      for (int k = 0; k < o.count; ++k)
        if (o.layers[k].outlier_count > 0 || o.layers[k].overlay_rows > 0 || o.layers[k].patch_rank > 0)
          return fail(NQB_ERR_UNSUPPORTED, "op %d: gated inputs take no salient columns, overlay rows or patch", i);
    int64_t rank_total = 0;
    for (int k = 0; k < o.count; ++k) {
      const nqb_linear_desc &d = o.layers[k];
      if (d.patch_rank < 0 || d.patch_rank > (1ll << 20) ||
          (d.patch_rank > 0 && (d.patch_left == nullptr || d.patch_right == nullptr || !is_float_dtype(d.patch_dtype))))
        return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: member %d has an invalid low-rank patch", i, k);
      if (d.overlay_rows < 0 || d.overlay_rows > d.out_features ||
          (d.overlay_rows > 0 && (d.overlay_row_ids == nullptr || d.overlay_values == nullptr ||
                                  d.overlay_scales == nullptr || !is_float_dtype(d.overlay_scale_dtype))))
        return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: member %d has invalid int8 overlay rows", i, k);
      if (d.coded_right_tiles != nullptr &&
          (d.coded_codebook == nullptr || d.coded_free_rows <= 0 || d.coded_free_rows >= d.rank ||
           (d.coded_format != NQB_CODED_MIXED_V && d.coded_format != NQB_CODED_PRODUCT_CODEBOOK) ||
           reinterpret_cast<uintptr_t>(d.coded_right_tiles) % 16 || reinterpret_cast<uintptr_t>(d.coded_codebook) % 16))
        return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: member %d has invalid coded right-factor tiles", i, k);
      if (d.in_features != o.layers[0].in_features || d.scale_dtype != o.layers[0].scale_dtype)
        return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: members must share in_features and scale dtype", i);
      if (o.y[k] == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: output %d is NULL", i, k);
      rank_total += d.rank;
    }
    if (!tc_eligible(o.layers, o.count, swiglu ? NQB_F32 : o.x_dtype, tokens))
      return fail(NQB_ERR_UNSUPPORTED, "op %d does not take the tensor-core decode path", i);
    int64_t side_total = 0;  // patch latents and overlay row segments after the ranks
    const int64_t segs = (o.layers[0].in_features + kOverlaySegCols - 1) / kOverlaySegCols;
    for (int k = 0; k < o.count; ++k) side_total += o.layers[k].patch_rank + o.layers[k].overlay_rows * segs;
    latent_cols = std::max(latent_cols, rank_total + side_total);
    if (e != nullptr) {
      for (int k = 0; k < o.count; ++k)
        if (o.layers[k].patch_rank > 0 || o.layers[k].coded_right_tiles != nullptr || o.layers[k].overlay_rows > 0)
          return fail(NQB_ERR_UNSUPPORTED, "op %d: decoder-step ops take no patch, coded right-factor tiles or overlay rows", i);
      if (e->norm_stats != nullptr) {
        if (o.x_dtype != NQB_F32 || e->norm_weight == nullptr || !is_float_dtype(e->norm_weight_dtype) ||
            !(e->eps >= 0.0f))
          return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: a residual-stream input is fp32 h with a norm weight", i);
        for (int k = 0; k < o.count; ++k)
          if (o.layers[k].outlier_count > 0)
            return fail(NQB_ERR_UNSUPPORTED, "op %d: residual-stream inputs take no salient columns", i);
      }
      if (e->epilogue == NQB_EPI_RESIDUAL) {
        if (o.count != 1 || e->out_stats == nullptr)
          return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: a residual epilogue has one member and out_stats", i);
      } else if (e->epilogue == NQB_EPI_QK_ROPE) {
        if (e->head_dim != kAttHd || o.count != 3 || e->kv_heads < 1 ||
            o.layers[0].out_features != static_cast<int64_t>(e->q_heads) * kAttHd ||
            o.layers[1].out_features != static_cast<int64_t>(e->kv_heads) * kAttHd ||
            o.layers[2].out_features != static_cast<int64_t>(e->kv_heads) * kAttHd)
          return fail(NQB_ERR_UNSUPPORTED, "op %d: the q/k epilogue takes q, k, v members of head_dim %d", i, kAttHd);
        if (e->cos_table == nullptr || e->sin_table == nullptr || e->q == nullptr || e->k_cache == nullptr ||
            e->v_cache == nullptr || !cache_layout_ok(e, tokens) ||
            ((e->q_norm_weight != nullptr || e->k_norm_weight != nullptr) && !is_float_dtype(e->qk_norm_dtype)))
          return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: q/k epilogue operands or cache position invalid", i);
      } else if (e->epilogue != NQB_EPI_STORE) {
        return fail(NQB_ERR_INVALID_ARGUMENT, "op %d: unknown epilogue %d", i, e->epilogue);
      }
    }
  }

  // fp32 copies of the scale and bias vectors, so the kernel reads them with
  // plain loads (no per-element dtype dispatch)
  struct VecCopy {
    const void *src;
    int32_t dtype;
    int64_t n;
    size_t offset;
  };
  std::vector<VecCopy> copies;
  size_t scale_floats = 0;
  auto add_copy = [&](const void *src, int32_t dtype, int64_t n) -> size_t {
    if (src == nullptr) return SIZE_MAX;
    const size_t at = (scale_floats + 63) & ~size_t(63);
    copies.push_back({src, dtype, n, at});
    scale_floats = at + static_cast<size_t>(n);
    return at;
  };
  struct MemberScales {
    size_t pre, mid, post, bias;
    size_t slot = SIZE_MAX;  // int8 overlay rows: [out_features] int32 row -> overlay row index (-1: none)
  };
  std::vector<MemberScales> member_scales;
  struct SlotMap {
    size_t at;
    std::vector<int32_t> slots;
  };
  std::vector<SlotMap> slot_maps;
  struct OpScales {
    size_t norm_weight = SIZE_MAX, q_norm = SIZE_MAX, k_norm = SIZE_MAX;
  };
  std::vector<OpScales> op_scales(op_count);
  for (int i = 0; i < op_count; ++i) {
    const nqb_program_op_ext *e = ops[i].ext;
    if (e == nullptr || e->kind != NQB_OP_LINEAR) continue;
    if (e->norm_stats != nullptr)
      op_scales[i].norm_weight = add_copy(e->norm_weight, e->norm_weight_dtype, ops[i].layers[0].in_features);
    if (e->epilogue == NQB_EPI_QK_ROPE) {
      op_scales[i].q_norm = add_copy(e->q_norm_weight, e->qk_norm_dtype, kAttHd);
      op_scales[i].k_norm = add_copy(e->k_norm_weight, e->qk_norm_dtype, kAttHd);
    }
  }
  for (int i = 0; i < op_count; ++i)
    for (int k = 0; k < (ops[i].ext != nullptr && ops[i].ext->kind == NQB_OP_ATTENTION ? 0 : ops[i].count); ++k) {
      const nqb_linear_desc &d = ops[i].layers[k];
      MemberScales ms;
      ms.pre = add_copy(d.scale_pre, d.scale_dtype, d.in_features);
      ms.mid = add_copy(d.scale_mid, d.scale_dtype, d.rank);
      ms.post = add_copy(d.scale_post, d.scale_dtype, d.out_features);
      ms.bias = add_copy(d.bias, d.bias_dtype, d.out_features);
      if (d.overlay_rows > 0) {
        // the overlay's row ids (device) -> a per-row index map owned by the program
        std::vector<int32_t> ids(static_cast<size_t>(d.overlay_rows));
        if (cudaMemcpy(ids.data(), d.overlay_row_ids, ids.size() * sizeof(int32_t), cudaMemcpyDeviceToHost) !=
            cudaSuccess) {
          cudaGetLastError();
          return fail(NQB_ERR_CUDA, "op %d member %d: reading the overlay row ids failed", i, k);
        }
        SlotMap map{(scale_floats + 63) & ~size_t(63), std::vector<int32_t>(static_cast<size_t>(d.out_features), -1)};
        for (size_t j = 0; j < ids.size(); ++j) {
          if (ids[j] < 0 || ids[j] >= d.out_features || (j > 0 && ids[j] <= ids[j - 1]))
            return fail(NQB_ERR_INVALID_ARGUMENT,
                        "op %d member %d: overlay row ids must be strictly increasing and below out_features", i, k);
          map.slots[ids[j]] = static_cast<int32_t>(j);
        }
        scale_floats = map.at + map.slots.size();
        ms.slot = map.at;
        slot_maps.push_back(std::move(map));
      }
      member_scales.push_back(ms);
    }
  float *scales = nullptr;
  if (cudaMalloc(&scales, std::max<size_t>(scale_floats, 64) * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    return fail(NQB_ERR_CUDA, "cudaMalloc of the program's fp32 scale copies failed");
  }
  for (const VecCopy &c : copies) {
    const int64_t blocks = std::min<int64_t>((c.n + 255) / 256, 1024);
    to_f32_kernel<<<static_cast<unsigned>(blocks), 256>>>(c.src, c.dtype, c.n, scales + c.offset);
  }
  for (const SlotMap &m : slot_maps)
    if (cudaMemcpy(scales + m.at, m.slots.data(), m.slots.size() * sizeof(int32_t), cudaMemcpyHostToDevice) !=
        cudaSuccess) {
      cudaGetLastError();
      cudaFree(scales);
      return fail(NQB_ERR_CUDA, "copying the overlay row maps failed");
    }
  // residual-stream inputs: the norm weight folds into each member's input scale (pre := pre * w)
  for (int i = 0, mi = 0; i < op_count; ++i) {
    const bool attention = ops[i].ext != nullptr && ops[i].ext->kind == NQB_OP_ATTENTION;
    const int members = attention ? 0 : ops[i].count;
    if (op_scales[i].norm_weight != SIZE_MAX)
      for (int k = 0; k < members; ++k) {
        const int64_t n = ops[i].layers[k].in_features;
        mul_f32_kernel<<<static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 1024)), 256>>>(
            scales + member_scales[mi + k].pre, scales + op_scales[i].norm_weight, n);
      }
    mi += members;
  }
  if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(scales);
    return fail(NQB_ERR_CUDA, "converting the program's scales to fp32 failed");
  }
  auto f32 = [&](size_t offset) -> const float * { return offset == SIZE_MAX ? nullptr : scales + offset; };
  size_t member_index = 0;
  for (int i = 0; i < op_count; ++i) {
    const nqb_program_op &o = ops[i];
    OpDev &od = opdev[i];
    std::memset(&od, 0, sizeof(od));
    const nqb_program_op_ext *e = o.ext;
    od.step.kind = e != nullptr ? e->kind : NQB_OP_LINEAR;
    if (e != nullptr) {
      od.step.epilogue = e->epilogue;
      od.step.eps = e->eps;
      od.step.out_stats = e->out_stats;
      od.step.q_heads = e->q_heads;
      od.step.kv_heads = e->kv_heads;
      od.step.cos_t = e->cos_table;
      od.step.sin_t = e->sin_table;
      od.step.q = static_cast<__nv_bfloat16 *>(e->q);
      od.step.k_cache = static_cast<__nv_bfloat16 *>(e->k_cache);
      od.step.v_cache = static_cast<__nv_bfloat16 *>(e->v_cache);
      od.step.cache_len = e->cache_len;
      od.step.position = e->position;
      od.step.seq_stride = e->sequence_stride;
      od.step.attn_out = static_cast<__nv_bfloat16 *>(e->attn_out);
      od.step.q_norm = f32(op_scales[i].q_norm);
      od.step.k_norm = f32(op_scales[i].k_norm);
      if (e->kind == NQB_OP_ATTENTION) continue;  // no members; the splits are set once the grid is known
      if (e->norm_stats != nullptr) {
        od.step.norm_stats = e->norm_stats;
        od.step.stat_tiles = static_cast<int32_t>((o.layers[0].in_features + kTileRows - 1) / kTileRows);
        od.step.inv_n = 1.0f / static_cast<float>(o.layers[0].in_features);
      }
    }
    od.count = o.count;
    od.x = o.x;
    od.x2 = (o.x_dtype == NQB_X_SWIGLU || o.x_dtype == NQB_X_GEGLU) ? o.x2 : nullptr;
    od.x_dtype = o.x_dtype;
    od.n = o.layers[0].in_features;
    int64_t offset = 0;
    for (int k = 0; k < o.count; ++k) {
      const MemberScales &ms = member_scales[member_index++];
      fill_member(od.s[0][k], o.layers[k], 0, offset, nullptr, f32(ms.pre), f32(ms.mid), nullptr);
      fill_member(od.s[1][k], o.layers[k], 1, offset, o.y[k], nullptr, f32(ms.post), f32(ms.bias));
      offset += o.layers[k].rank;
    }
    for (int k = 0; k < o.count; ++k) {  // patch latents after the ranks
      od.s[0][k].patch_offset = od.s[1][k].patch_offset = offset;
      offset += o.layers[k].patch_rank;
      od.side_rows += static_cast<int32_t>(o.layers[k].patch_rank);
    }
    od.ovl_segs = static_cast<int32_t>((od.n + kOverlaySegCols - 1) / kOverlaySegCols);
    for (int k = 0; k < o.count; ++k) {  // then the int8 overlay rows' partial dot products
      const MemberScales &ms = member_scales[member_index - o.count + k];
      if (o.layers[k].overlay_rows <= 0) continue;
      od.s[1][k].overlay_offset = offset;
      od.s[1][k].overlay_slot = reinterpret_cast<const int32_t *>(scales + ms.slot);
      offset += o.layers[k].overlay_rows * od.ovl_segs;
      od.side_rows += static_cast<int32_t>(o.layers[k].overlay_rows * od.ovl_segs);
    }
    od.latent_stride = offset;
  }

  int device = 0;
  NQB_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  bool patch = false, mixed = false;
  for (int i = 0; i < op_count; ++i) {
    patch = patch || opdev[i].side_rows > 0;
    for (int k = 0; k < opdev[i].count; ++k) mixed = mixed || opdev[i].s[0][k].coded_tiles != nullptr;
  }
  if (step && (patch || mixed)) return fail(NQB_ERR_UNSUPPORTED, "decoder-step programs take no patch or mixed-V tiles");
  const SmemPlan sp = smem_plan(bucket, mixed);
  if (sp.off_cb % 16) return fail(NQB_ERR_UNSUPPORTED, "codebook buffer is misaligned");
  if (step && bucket >= mmad::kWarps && sp.off_cb - sp.off_acc < static_cast<uint32_t>(kAttStageBytes))
    return fail(NQB_ERR_UNSUPPORTED, "the attention staging buffer does not fit the accumulator buffers");
  const void *fn = kernel_for(bucket, patch, mixed, step);
  {
    // the kernel's register split assumes the launch count (kLaunchRegs)
    cudaFuncAttributes attr;
    NQB_CUDA(cudaFuncGetAttributes(&attr, fn), "cudaFuncGetAttributes");
    if (attr.numRegs != kLaunchRegs)
      return fail(NQB_ERR_UNSUPPORTED, "program kernel built with %d registers; its register split needs %d",
                  attr.numRegs, kLaunchRegs);
  }
  NQB_CHECK(ensure_dynamic_smem(fn, static_cast<int>(sp.total)));
  int sms = 0;
  NQB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "SM count");
  int clusters = 0;
  {
    cudaLaunchConfig_t config;
    std::memset(&config, 0, sizeof(config));
    config.gridDim = dim3(kClusterSize * std::max(1, sms / kClusterSize));
    config.blockDim = dim3(kBlockThreads);
    config.dynamicSmemBytes = sp.total;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kClusterSize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    NQB_CUDA(cudaOccupancyMaxActiveClusters(&clusters, fn, &config), "cudaOccupancyMaxActiveClusters");
  }
  clusters = std::min(clusters, sms / kClusterSize);
  if (clusters < 1) return fail(NQB_ERR_UNSUPPORTED, "no cluster of %d CTAs fits this device", kClusterSize);
  const int ctas = clusters * kClusterSize;
  // fused attention: one (kv head, key split) unit per CTA, at most 32
  // partials per (token, q head) -- from 8 tokens on a unit writes one per
  // key half, so at most 16 splits
  size_t att_floats = 0;
  for (int i = 0; i < op_count; ++i) {
    OpDev &od = opdev[i];
    if (od.step.kind != NQB_OP_ATTENTION) continue;
    const bool seqs = od.step.seq_stride != 0;
    const int halves = tokens >= mmad::kWarps && !seqs ? 2 : 1;
    const int64_t split_units = (seqs ? tokens : 1) * od.step.kv_heads;  // units per key split
    if (split_units > ctas)
      return fail(NQB_ERR_UNSUPPORTED, "op %d: %lld sequences x %d kv heads exceed the program's %d CTAs", i,
                  static_cast<long long>(seqs ? tokens : 1), od.step.kv_heads, ctas);
    const int want = std::max(1, std::min(32 / halves, static_cast<int>(ctas / split_units)));
    const int64_t most = od.step.position + (seqs ? 1 : tokens);  // keys the last token sees
    od.step.att_chunk = ((most + want - 1) / want + 15) / 16 * 16;
    od.step.att_splits = static_cast<int32_t>((most + od.step.att_chunk - 1) / od.step.att_chunk);
    od.step.att_parts = od.step.att_splits * halves;
    // K and V blocks of a unit must fit the ring at once (the consumers hold them all)
    od.step.att_ring_blocks = std::max(0, sp.ring / 2 - 1);
    att_floats = std::max(att_floats, static_cast<size_t>(tokens) * od.step.q_heads * od.step.att_parts * kAttRow);
  }

  // tiles per (stage, cluster), then every CTA's slice addresses in consumption order
  // and the L2 lines it reads per stage besides sign words and activations
  const int stages = 2 * op_count;
  std::vector<std::vector<uint64_t>> pf(static_cast<size_t>(stages) * ctas);
  auto add_lines = [](std::vector<uint64_t> &out, const void *base, int64_t bytes) {
    if (base == nullptr || bytes <= 0) return;
    const uint64_t first = reinterpret_cast<uint64_t>(base) & ~uint64_t(127);
    const uint64_t end = reinterpret_cast<uint64_t>(base) + static_cast<uint64_t>(bytes);
    for (uint64_t a = first; a < end; a += 128) out.push_back(a);
  };
  // lines of the program's own tables (op descriptors, tile lists): arena
  // offsets tagged in bit 63, turned into addresses once the arena exists
  constexpr uint64_t kArenaTag = uint64_t(1) << 63;
  const size_t arena_ops = 0;
  const size_t arena_items = align_up(sizeof(OpDev) * op_count, 256) +
                             align_up(sizeof(int32_t) * (static_cast<size_t>(stages) * clusters + 1), 256);
  auto add_arena_lines = [&](std::vector<uint64_t> &out, size_t offset, size_t bytes) {
    for (size_t a = offset & ~size_t(127); a < offset + bytes; a += 128) out.push_back(kArenaTag | a);
  };
  std::vector<int32_t> stage_items(static_cast<size_t>(stages) * clusters + 1, 0);
  std::vector<Item> items;
  std::vector<std::vector<uint64_t>> lists(ctas);
  std::vector<std::vector<Item>> per_cluster;
  for (int g = 0; g < stages; ++g) {
    const OpDev &op = opdev[g >> 1];
    const int st = g & 1;
    if (op.step.kind == NQB_OP_ATTENTION && st == 0 && op.step.seq_stride == 0) {
      // each CTA's unit (kv head, key split): its K and V rows that do not
      // stream through the sign ring go on the L2 prefetch list of the stage
      // two ahead of this one (the rows before this step's tokens do not
      // change during the program)
      const int target = std::max(0, g - 2);
      for (int c = 0; c < ctas && c < att_units(op.step, static_cast<int>(tokens)); ++c) {
        int tu, kvh, spl;
        att_unit_of(op.step, c, tu, kvh, spl);
        const int64_t k0 = static_cast<int64_t>(spl) * op.step.att_chunk + 16 * att_unit_ring_blocks(op.step, spl);
        // at most kAttPrefetchRows rows: with independent sequences a step's
        // K/V rows can exceed the L2, and the tables grow with the lines
        const int64_t k1 = std::min({static_cast<int64_t>(spl) * op.step.att_chunk + op.step.att_chunk,
                                     op.step.position + (op.step.seq_stride != 0 ? 1 : tokens),
                                     k0 + kAttPrefetchRows});
        if (k1 <= k0) continue;
        const int64_t off = att_cache_offset(op.step, tu, kvh, k0);
        std::vector<uint64_t> &lines = pf[static_cast<size_t>(target) * ctas + c];
        add_lines(lines, op.step.k_cache + off, (k1 - k0) * kAttHd * 2);
        add_lines(lines, op.step.v_cache + off, (k1 - k0) * kAttHd * 2);
      }
    }
    assign_stage(op, st, clusters, per_cluster);
    for (int c = 0; c < clusters; ++c)
      if (per_cluster[c].size() > static_cast<size_t>(kMaxStageItems))
        return fail(NQB_ERR_UNSUPPORTED, "op %d stage %d: more than %d row tiles per cluster", g >> 1, st + 1,
                    kMaxStageItems);
    for (int c = 0; c < clusters; ++c) {
      stage_items[static_cast<size_t>(g) * clusters + c] = static_cast<int32_t>(items.size());
      const std::vector<Item> &list = per_cluster[c];
      items.insert(items.end(), list.begin(), list.end());
      for (int q = 0; q < kClusterSize; ++q) {
        std::vector<uint64_t> &lines = pf[static_cast<size_t>(g) * ctas + c * kClusterSize + q];
        if (st == 0) add_arena_lines(lines, arena_ops + sizeof(OpDev) * (g >> 1), sizeof(OpDev));
        add_arena_lines(lines, arena_items + sizeof(Item) * stage_items[static_cast<size_t>(g) * clusters + c],
                        sizeof(Item) * list.size());
        int last_member = -1;
        for (size_t j = 0; j < list.size(); ++j) {
          const MemberDev &md = op.s[st][list[j].member];
          if (st == 0 && list[j].member != last_member) {
            last_member = list[j].member;
            const int64_t lo = static_cast<int64_t>(md.ks) * q / kClusterSize * kStageCols;
            const int64_t hi = std::min<int64_t>(static_cast<int64_t>(md.ks) * (q + 1) / kClusterSize * kStageCols,
                                                 md.k_valid);
            if (hi > lo) {
              add_lines(lines, md.pre + lo, (hi - lo) * 4);
              const bool swiglu = op.x_dtype == NQB_X_SWIGLU || op.x_dtype == NQB_X_GEGLU;
              const int64_t xs = swiglu ? 4 : static_cast<int64_t>(dtype_size(op.x_dtype));
              for (int64_t t = 0; t < tokens; ++t) {
                add_lines(lines, static_cast<const char *>(op.x) + (t * op.n + lo) * xs, (hi - lo) * xs);
                if (swiglu)
                  add_lines(lines, static_cast<const char *>(op.x2) + (t * op.n + lo) * xs, (hi - lo) * xs);
              }
            }
          }
          if (static_cast<int>(j % kClusterSize) == q) {
            const int64_t r0 = static_cast<int64_t>(list[j].tile) * kTileRows;
            const int64_t rows = std::min<int64_t>(kTileRows, md.rows - r0);
            add_lines(lines, md.row_scale + r0, rows * 4);
            if (md.bias != nullptr) add_lines(lines, md.bias + r0, rows * 4);
          }
        }
        std::vector<uint64_t> &addrs = lists[c * kClusterSize + q];
        if (op.step.kind == NQB_OP_ATTENTION && st == 0) {
          // this CTA's attention unit: its old K and V rows as 16-row blocks (4 KB each, K then V)
          const int cta_id = c * kClusterSize + q;
          if (cta_id < att_units(op.step, static_cast<int>(tokens))) {
            int tu, kvh, spl;
            att_unit_of(op.step, cta_id, tu, kvh, spl);
            const int nb = att_unit_ring_blocks(op.step, spl);
            for (int b = 0; b < nb; ++b) {
              const int64_t off = att_cache_offset(op.step, tu, kvh, static_cast<int64_t>(spl) * op.step.att_chunk + 16 * b);
              addrs.push_back(reinterpret_cast<uint64_t>(op.step.k_cache + off));
              addrs.push_back(reinterpret_cast<uint64_t>(op.step.v_cache + off));
            }
          }
        }
        for (size_t gb = 0; gb < list.size(); gb += sp.group) {
          const size_t ge = std::min(list.size(), gb + sp.group);
          for (size_t j0 = gb; j0 < ge;) {
            size_t j1 = j0 + 1;
            while (j1 < ge && list[j1].member == list[j0].member) ++j1;
            const MemberDev &md = op.s[st][list[j0].member];
            const int lo = md.ks * q / kClusterSize, hi = md.ks * (q + 1) / kClusterSize;
            for (int c0 = lo; c0 < hi; c0 += sp.sc) {
              const int nst = std::min(sp.sc, hi - c0);
              for (size_t j = j0; j < j1; ++j)
                for (int sl = c0; sl < c0 + nst; ++sl) {
                  if (st == 0 && list[j].tile >= md.coded_from) {  // coded slice: tag bit 0 or 1
                    const bool product = md.coded_format == NQB_CODED_PRODUCT_CODEBOOK;
                    const uint64_t bytes = product ? kCodebookSliceBytes : kCodedSliceBytes;
                    addrs.push_back((reinterpret_cast<uint64_t>(md.coded_tiles) +
                                     (static_cast<uint64_t>(list[j].tile - md.coded_from) * md.ks + sl) * bytes) |
                                    (product ? 2u : 1u));
                  } else {
                    addrs.push_back(reinterpret_cast<uint64_t>(md.tiles) +
                                    (static_cast<uint64_t>(list[j].tile) * md.wc + 2ull * sl) * (kTileRows * kChunkBytes));
                  }
                }
            }
            j0 = j1;
          }
        }
      }
    }
  }
  stage_items.back() = static_cast<int32_t>(items.size());
  // grid barriers: pre-quantised instances add one before every linear stage
  // (index bar_end[g] - 1), and every stage but the last ends with bar_end[g]
  const bool pre_q = pre_quantised(bucket);
  const int32_t qunit_bytes = static_cast<int32_t>(
      align_up(static_cast<size_t>(sp.sc) * mmad::slice_frag_bytes(mmad::n_tiles(bucket)) + 12u * bucket, 16));
  size_t qbuf_bytes = 0;
  std::vector<int32_t> bar_end(stages);
  {
    int32_t index = 0;
    for (int g = 0; g < stages; ++g) {
      const OpDev &op = opdev[g >> 1];
      if (pre_q && op.step.kind == NQB_OP_LINEAR) {
        ++index;
        size_t units = 0;
        for (int k = 0; k < op.count; ++k) units += static_cast<size_t>(member_chunks(op.s[g & 1][k].ks, sp.sc));
        qbuf_bytes = std::max(qbuf_bytes, units * static_cast<size_t>(qunit_bytes));
      }
      bar_end[g] = index++;
    }
  }
  std::vector<int64_t> slice_begin(ctas);
  std::vector<int32_t> slice_count(ctas);
  std::vector<uint64_t> flat;
  for (int c = 0; c < ctas; ++c) {
    slice_begin[c] = static_cast<int64_t>(flat.size());
    slice_count[c] = static_cast<int32_t>(lists[c].size());
    flat.insert(flat.end(), lists[c].begin(), lists[c].end());
    flat.resize(((flat.size() + kAddrChunk - 1) / kAddrChunk) * kAddrChunk, 0);
  }
  if (flat.empty()) flat.resize(kAddrChunk, 0);
  std::vector<int32_t> pf_begin(static_cast<size_t>(stages) * ctas + 1, 0);
  std::vector<uint64_t> pf_lines;
  for (size_t i = 0; i < pf.size(); ++i) {
    pf_begin[i] = static_cast<int32_t>(pf_lines.size());
    pf_lines.insert(pf_lines.end(), pf[i].begin(), pf[i].end());
  }
  pf_begin.back() = static_cast<int32_t>(pf_lines.size());
  if (pf_lines.empty()) pf_lines.push_back(0);

  // one device arena for the tables
  auto section = [](size_t bytes) { return align_up(bytes, 256); };
  const size_t b_ops = section(sizeof(OpDev) * op_count);
  const size_t b_si = section(sizeof(int32_t) * stage_items.size());
  const size_t b_items = section(sizeof(Item) * std::max<size_t>(1, items.size()));
  const size_t b_addrs = section(sizeof(uint64_t) * flat.size());
  const size_t b_begin = section(sizeof(int64_t) * ctas);
  const size_t b_count = section(sizeof(int32_t) * ctas);
  const size_t b_pfb = section(sizeof(int32_t) * pf_begin.size());
  const size_t b_pfl = section(sizeof(uint64_t) * pf_lines.size());
  const size_t b_bar = section(sizeof(int32_t) * bar_end.size());
  const size_t total = b_ops + b_si + b_items + b_addrs + b_begin + b_count + b_pfb + b_pfl + b_bar;
  nqb_program *prog = new (std::nothrow) nqb_program();
  if (prog == nullptr) {
    cudaFree(scales);
    return fail(NQB_ERR_INVALID_ARGUMENT, "out of host memory");
  }
  prog->scales = scales;
  if (cudaMalloc(&prog->arena, total) != cudaSuccess) {
    cudaFree(scales);
    delete prog;
    cudaGetLastError();
    return fail(NQB_ERR_CUDA, "cudaMalloc of %zu bytes for the program tables failed", total);
  }
  char *base = static_cast<char *>(prog->arena);
  size_t off = 0;
  auto put = [&](const void *src, size_t bytes, size_t section_bytes) -> void * {
    void *dst = base + off;
    if (bytes > 0) cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    off += section_bytes;
    return dst;
  };
  Params &pp = prog->params;
  std::memset(&pp, 0, sizeof(pp));
  for (uint64_t &line : pf_lines)
    if (line & kArenaTag) line = reinterpret_cast<uint64_t>(base) + (line & ~kArenaTag);
  pp.ops = static_cast<const OpDev *>(put(opdev.data(), sizeof(OpDev) * op_count, b_ops));
  pp.stage_items = static_cast<const int32_t *>(put(stage_items.data(), sizeof(int32_t) * stage_items.size(), b_si));
  pp.items = static_cast<const Item *>(put(items.data(), sizeof(Item) * items.size(), b_items));
  pp.slice_addrs = static_cast<const uint64_t *>(put(flat.data(), sizeof(uint64_t) * flat.size(), b_addrs));
  pp.slice_begin = static_cast<const int64_t *>(put(slice_begin.data(), sizeof(int64_t) * ctas, b_begin));
  pp.slice_count = static_cast<const int32_t *>(put(slice_count.data(), sizeof(int32_t) * ctas, b_count));
  pp.pf_begin = static_cast<const int32_t *>(put(pf_begin.data(), sizeof(int32_t) * pf_begin.size(), b_pfb));
  pp.pf_lines = static_cast<const uint64_t *>(put(pf_lines.data(), sizeof(uint64_t) * pf_lines.size(), b_pfl));
  pp.bar_end = static_cast<const int32_t *>(put(bar_end.data(), sizeof(int32_t) * bar_end.size(), b_bar));
  pp.qunit_bytes = qunit_bytes;
  const cudaError_t copy_status = cudaDeviceSynchronize();
  if (copy_status != cudaSuccess) {
    cudaFree(prog->arena);
    cudaFree(scales);
    delete prog;
    return fail(NQB_ERR_CUDA, "copying the program tables failed: %s", cudaGetErrorString(copy_status));
  }
  pp.stages = stages;
  pp.clusters = clusters;
  pp.tokens = static_cast<int32_t>(tokens);
  pp.ring = sp.ring;
  pp.sc = sp.sc;
  pp.group = sp.group;
  pp.off_addr = sp.off_addr;
  pp.off_b = sp.off_b;
  pp.off_acc = sp.off_acc;
  pp.off_exch = sp.off_exch;
  pp.off_cb = sp.off_cb;
  prog->device = device;
  prog->tokens = tokens;
  prog->bucket = bucket;
  prog->patch = patch;
  prog->mixed = mixed;
  prog->ctas = ctas;
  prog->clusters = clusters;
  prog->smem = static_cast<int>(sp.total);
  prog->latent_bytes = align_up(static_cast<size_t>(tokens) * latent_cols * sizeof(float), 256);
  prog->att_part_bytes = align_up(att_floats * sizeof(float), 256);
  prog->qbuf_bytes = align_up(qbuf_bytes, 256);
  prog->step = step;
  pp.off_epi = sp.off_epi;
  *program = prog;
  return ok();
}

int nqb_program_workspace_bytes(const nqb_program *program, size_t *bytes) {
  if (program == nullptr || bytes == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "program or bytes is NULL");
  *bytes = kCounterRegionBytes + program->latent_bytes + program->att_part_bytes + program->qbuf_bytes;
  return ok();
}

}  // extern "C"

namespace nqb {
namespace prog {

// Grid-barrier poll limit of the next launches (0: kBarrierSpinLimit); tests
// shorten it to make a barrier that cannot complete give up quickly.
static std::atomic<uint32_t> g_barrier_limit{0};

static int launch_program(const nqb_program *program, void *workspace, size_t workspace_bytes, void *stream,
                          bool dependent) {
  if (program == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "program is NULL");
  const size_t need = kCounterRegionBytes + program->latent_bytes + program->att_part_bytes + program->qbuf_bytes;
  if (workspace == nullptr || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(NQB_ERR_WORKSPACE, "program workspace needs %zu bytes aligned to 256, got %zu", need, workspace_bytes);
  Params params = program->params;
  params.counters = static_cast<uint32_t *>(workspace);
  params.latent = reinterpret_cast<float *>(static_cast<char *>(workspace) + kCounterRegionBytes);
  params.att_part =
      reinterpret_cast<float *>(static_cast<char *>(workspace) + kCounterRegionBytes + program->latent_bytes);
  params.qbuf = program->qbuf_bytes > 0 ? static_cast<uint8_t *>(workspace) + kCounterRegionBytes +
                                              program->latent_bytes + program->att_part_bytes
                                        : nullptr;
  const uint32_t limit = g_barrier_limit.load();
  params.barrier_limit = limit != 0 ? limit : kBarrierSpinLimit;
  params.barrier_skew = program->barrier_skew;
  const void *fn = kernel_for(program->bucket, program->patch, program->mixed, program->step);
  NQB_CHECK(ensure_dynamic_smem(fn, program->smem));
  cudaLaunchConfig_t config;
  std::memset(&config, 0, sizeof(config));
  config.gridDim = dim3(program->ctas);
  config.blockDim = dim3(kBlockThreads);
  config.dynamicSmemBytes = program->smem;
  config.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterSize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  attr[2].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[2].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = dependent ? 3 : 2;
  void *args[] = {&params};
  NQB_CUDA(cudaLaunchKernelExC(&config, fn, args), "program launch");
  return NQB_OK;
}

}  // namespace prog
}  // namespace nqb

extern "C" {

int nqb_program_run(const nqb_program *program, void *workspace, size_t workspace_bytes, void *stream) {
  NQB_CHECK(nqb::prog::launch_program(program, workspace, workspace_bytes, stream, false));
  return ok();
}

int nqb_program_run_dependent(const nqb_program *program, void *workspace, size_t workspace_bytes, void *stream) {
  NQB_CHECK(nqb::prog::launch_program(program, workspace, workspace_bytes, stream, true));
  return ok();
}

int nqb_program_destroy(nqb_program *program) {
  if (program == nullptr) return ok();
  if (program->arena != nullptr) cudaFree(program->arena);
  if (program->scales != nullptr) cudaFree(program->scales);
  delete program;
  return ok();
}

int nqb_program_trace(const nqb_program *program, int64_t *cycles, size_t count) {
#ifdef NQB_PHASE_TRACE
  if (program == nullptr || cycles == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "program or cycles is NULL");
  const size_t need = static_cast<size_t>(program->ctas) * program->params.stages * nqb::prog::kTracePhases;
  if (count < need) return fail(NQB_ERR_INVALID_ARGUMENT, "trace buffer needs %zu entries", need);
  static long long host[nqb::prog::kTraceMaxCtas][nqb::prog::kTraceMaxStages][nqb::prog::kTracePhases];
  NQB_CUDA(cudaMemcpyFromSymbol(host, nqb::prog::g_trace, sizeof(host)), "read the phase trace");
  const int ctas = std::min(program->ctas, nqb::prog::kTraceMaxCtas);
  const int stages = std::min(program->params.stages, nqb::prog::kTraceMaxStages);
  std::memset(cycles, 0, need * sizeof(int64_t));
  for (int c = 0; c < ctas; ++c)
    for (int g = 0; g < stages; ++g)
      for (int k = 0; k < nqb::prog::kTracePhases; ++k)
        cycles[(static_cast<size_t>(c) * program->params.stages + g) * nqb::prog::kTracePhases + k] = host[c][g][k];
  return ok();
#else
  (void)program;
  (void)cycles;
  (void)count;
  return fail(NQB_ERR_UNSUPPORTED, "phase tracing needs the trace build (python -m nanoquant_b200.build --trace)");
#endif
}

int nqb_residual_stats(const float *h, int64_t tokens, int64_t hidden, float *stats, void *stream) {
  if (h == nullptr || stats == nullptr || tokens <= 0 || hidden <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "residual stats operands invalid");
  const int64_t warps = (hidden + nqb::prog::kTileRows - 1) / nqb::prog::kTileRows * tokens;
  nqb::prog::residual_stats_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0,
                                      static_cast<cudaStream_t>(stream)>>>(h, tokens, hidden, stats);
  NQB_CUDA(cudaGetLastError(), "residual stats launch");
  return ok();
}

int nqb_debug_set_barrier_limit(uint32_t polls) {
  nqb::prog::g_barrier_limit.store(polls);
  return ok();
}

int nqb_program_debug_barrier_skew(nqb_program *program, uint32_t skew) {
  if (program == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "program is NULL");
  program->barrier_skew = skew;
  return ok();
}

int nqb_program_shape(const nqb_program *program, int32_t *ctas, int32_t *cluster_size) {
  if (program == nullptr || ctas == nullptr || cluster_size == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "program, ctas or cluster_size is NULL");
  *ctas = program->ctas;
  *cluster_size = nqb::prog::kClusterSize;
  return ok();
}

}  // extern "C"
