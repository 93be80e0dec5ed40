// Register-operand decode arithmetic (mma.sync m16n8k32 s8) shared by the
// persistent decode program.  Internal header.
//
// The product out[row, t] = sum_k sign(S[row, k]) * a[t, k] for 1..16
// tokens is exact integer work on the tensor cores, like the tcgen05 decode
// kernels (nqb_tc_decode.cuh), but with the sign bits expanded straight into
// A-fragment registers instead of into tensor memory: for tiny N the tcgen05
// path spends its time writing 8 bytes of TMEM per sign byte, while here one
// LOP3 per register feeds the MMA.
//
// * A (16 rows x 32 K per MMA): lane (g, tig) = (lane/4, lane%4) holds rows g
//   and g+8.  For K block kb = 2j + h of a 256-column slice, its registers are
//   (w >> 4h) & (0x01010101 << j) of sign words tig (a0/a1) and tig + 4
//   (a2/a3): bytes bit * 2^j of columns 32*word + 8b + j + 4h.  Each j has its
//   own accumulator; the drain adds D_j >> j (exact).
// * B (32 K x 8 columns): the activations of a K chunk quantised per token to
//   fixed point, D signed base-256 digits per token, so column n = D t + d;
//   stored in shared memory as ready fragments (one 64-bit load per lane and
//   MMA).  Up to 2 tokens D = 3 (22-bit: the columns fit one 8-column N tile
//   anyway); from 3 tokens (the 4-token instance) on D = 2 (14-bit), which
//   takes the N tiles, and so the MMAs, from 2 to 1 at 4 tokens, 3 to 2 at 8
//   and 6 to 4 at 16.  Error of the 14-bit form: about 1e-4 of max|y| per
//   stage (measured against a float64 oracle), inside the 2e-3 bound.
// * sum_k sign_k q_k = Q - 2 * sum_k bit_k q_k, Q = sum_k q_k per token.
#pragma once

#include "nqb_common.cuh"
#include "nqb_tc_decode.cuh"

namespace nqb {
namespace mmad {

constexpr int kWarps = 8;                 // consumer warps, 16 rows each
constexpr int kThreads = kWarps * 32;     // consumer threads
constexpr int kTileRows = 128;
constexpr int kSliceCols = 256;
constexpr int kSliceBytes = 4096;         // 128 rows x 8 words
constexpr uint32_t kFragBytes = 256;      // one (K block, N tile) B fragment block: 32 lanes x 8 bytes
constexpr int kMaxSliceQuant = 16;        // slices quantised at once

// Digits per token and fixed-point bits of the instance for `tokens` (a token bucket: 1, 2, 4, 8 or 16).
__host__ __device__ constexpr int digits_for(int tokens) { return tokens >= 4 ? 2 : 3; }
__host__ __device__ constexpr int fixed_bits(int tokens) { return tokens >= 4 ? 14 : 22; }

__host__ __device__ constexpr int n_tiles(int tokens) { return (digits_for(tokens) * tokens + 7) / 8; }

// q (|q| < 2^(8 kD - 2)) as kD signed base-256 digits, byte b of w[d] from q[b].
template <int kD>
__device__ __forceinline__ void split_digits_n(const int32_t (&q)[4], uint32_t (&w)[kD]) {
#pragma unroll
  for (int d = 0; d < kD; ++d) w[d] = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    int32_t v = q[b];
#pragma unroll
    for (int d = 0; d < kD - 1; ++d) {
      const int32_t dk = static_cast<int8_t>(v & 0xFF);
      v = (v - dk) >> 8;
      w[d] |= (static_cast<uint32_t>(dk) & 0xFFu) << (8 * b);
    }
    w[kD - 1] |= (static_cast<uint32_t>(v) & 0xFFu) << (8 * b);
  }
}

// B-fragment bytes of one slice for kNT N tiles.
__host__ __device__ constexpr uint32_t slice_frag_bytes(int nt) { return 8u * nt * kFragBytes; }

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void mma_s8(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Where a K chunk of activations comes from.  Column indices are relative
// to k0; past k_valid reads 0.  Activations are read through L2 (.cg): an
// earlier grid stage may have written them.
//
// Each loader also splits a value into loads and arithmetic: scale(col) and
// fetch(t, col) only load (the column's factor, the token's raw element),
// finish(raw, scale) computes the value, so load_chunk can issue every load
// of a chunk before the first arithmetic waits on one.
template <typename XT>
struct XLoader {  // stage 1: x * pre, pre in fp32
  using Raw = XT;
  static constexpr bool kTwoPhase = false;
  const XT *x;
  const float *pre;
  int64_t stride;  // elements per token row
  int64_t k0;
  int64_t k_valid;
  __device__ __forceinline__ float operator()(int t, int col) const {
    const int64_t k = k0 + col;
    if (k >= k_valid) return 0.0f;
    return to_f32(__ldcg(x + static_cast<int64_t>(t) * stride + k)) * __ldg(pre + k);
  }
  __device__ __forceinline__ float scale(int col) const {
    const int64_t k = k0 + col;
    return k < k_valid ? __ldg(pre + k) : 0.0f;
  }
  __device__ __forceinline__ Raw fetch(int t, int col) const {
    const int64_t k = k0 + col;
    return k < k_valid ? __ldcg(x + static_cast<int64_t>(t) * stride + k) : Raw{};
  }
  __device__ __forceinline__ float finish(Raw r, float s) const { return to_f32(r) * s; }
};

struct SwigluLoader {  // stage 1 of a down projection: silu(gate) * up * pre, gate and up fp32
  const float *gate;
  const float *up;
  const float *pre;
  int64_t stride;
  int64_t k0;
  int64_t k_valid;
  using Raw = float2;  // (gate, up)
  static constexpr bool kTwoPhase = true;
  // fast exp and divide keep the T=1 prefetch loop free of spills; clamping
  // the exponent at 80 keeps the divisor below 2^126, inside __fdividef's
  // range (silu(g) for g < -80 is below 1e-33 either way)
  __device__ __forceinline__ static float silu(float g) { return __fdividef(g, 1.0f + __expf(fminf(-g, 80.0f))); }
  __device__ __forceinline__ float operator()(int t, int col) const {
    const int64_t k = k0 + col;
    if (k >= k_valid) return 0.0f;
    const int64_t i = static_cast<int64_t>(t) * stride + k;
    return silu(__ldcg(gate + i)) * __ldcg(up + i) * __ldg(pre + k);
  }
  __device__ __forceinline__ float scale(int col) const {
    const int64_t k = k0 + col;
    return k < k_valid ? __ldg(pre + k) : 0.0f;
  }
  __device__ __forceinline__ Raw fetch(int t, int col) const {
    const int64_t k = k0 + col;
    if (k >= k_valid) return make_float2(0.0f, 0.0f);
    const int64_t i = static_cast<int64_t>(t) * stride + k;
    return make_float2(__ldcg(gate + i), __ldcg(up + i));
  }
  __device__ __forceinline__ float finish(Raw r, float s) const { return silu(r.x) * r.y * s; }
};

// GELU (tanh form, Hendrycks & Gimpel 2016) of g: 0.5 g (1 + tanh(u)),
// u = sqrt(2/pi) (g + 0.044715 g^3), with tanh(u) = 1 - 2 / (1 + e^(2u)).  The
// exponent is clamped to +-80 so the divisor stays inside __fdividef's range
// (tanh is +-1 to float precision there).
__device__ __forceinline__ float gelu_tanh(float g) {
  const float u = 0.7978845608028654f * (g + 0.044715f * g * g * g);
  const float e = __expf(fminf(fmaxf(2.0f * u, -80.0f), 80.0f));
  return 0.5f * g * (2.0f - __fdividef(2.0f, 1.0f + e));
}

struct GegluLoader {  // stage 1 of a gated-GELU down projection: gelu_tanh(gate) * up * pre
  const float *gate;
  const float *up;
  const float *pre;
  int64_t stride;
  int64_t k0;
  int64_t k_valid;
  using Raw = float2;  // (gate, up)
  static constexpr bool kTwoPhase = true;
  __device__ __forceinline__ float operator()(int t, int col) const {
    const int64_t k = k0 + col;
    if (k >= k_valid) return 0.0f;
    const int64_t i = static_cast<int64_t>(t) * stride + k;
    return gelu_tanh(__ldcg(gate + i)) * __ldcg(up + i) * __ldg(pre + k);
  }
  __device__ __forceinline__ float scale(int col) const {
    const int64_t k = k0 + col;
    return k < k_valid ? __ldg(pre + k) : 0.0f;
  }
  __device__ __forceinline__ Raw fetch(int t, int col) const {
    const int64_t k = k0 + col;
    if (k >= k_valid) return make_float2(0.0f, 0.0f);
    const int64_t i = static_cast<int64_t>(t) * stride + k;
    return make_float2(__ldcg(gate + i), __ldcg(up + i));
  }
  __device__ __forceinline__ float finish(Raw r, float s) const { return gelu_tanh(r.x) * r.y * s; }
};

struct LatentLoader {  // stage 2: the fp32 latent slice of one member
  using Raw = float;
  static constexpr bool kTwoPhase = false;
  const float *latent;
  int64_t stride;
  int64_t offset;
  int64_t k0;
  int64_t k_valid;
  __device__ __forceinline__ float operator()(int t, int col) const {
    const int64_t k = k0 + col;
    if (k >= k_valid) return 0.0f;
    return __ldcg(latent + static_cast<int64_t>(t) * stride + offset + k);
  }
  __device__ __forceinline__ float scale(int) const { return 1.0f; }
  __device__ __forceinline__ Raw fetch(int t, int col) const { return (*this)(t, col); }
  __device__ __forceinline__ float finish(Raw r, float) const { return r; }
};

// Per-warp partials of the chunk quantiser (consumer warps).
template <int kT>
struct Scratch {
  float red_f[kWarps * kT];
  long long red_q[kWarps * kT];
};

// Quads of one chunk held per consumer thread: nst <= 16 slices x 64 quads.
__host__ __device__ constexpr int quads_per_thread(int max_slices) { return (max_slices * 64 + kThreads - 1) / kThreads; }

// This consumer thread's activations of one chunk: kQPT quads of four
// columns, kT tokens each.
template <int kT, int kQPT>
struct ChunkValues {
  float v[kQPT][4][kT];
};

// The chunk's activations.  For the gated loaders (long arithmetic per value)
// up to two tokens, every load is issued first and the arithmetic follows, so
// the chunk costs one memory round trip; otherwise each value is loaded and
// computed in turn (the compiler batches those loads itself, with fewer live
// registers).
template <int kT, int kQPT, typename Loader>
__device__ __forceinline__ void load_chunk(const Loader &src, int nst, int T, ChunkValues<kT, kQPT> &cv) {
  const int tid = threadIdx.x;
  const int nquads = nst * 64;
  if constexpr (kT >= 4 || Loader::kTwoPhase) {
    float scl[kQPT][4];
    typename Loader::Raw raw[kQPT][4][kT];
#pragma unroll
    for (int i = 0; i < kQPT; ++i) {
      const int qd = tid + i * kThreads;
      const int sl = qd >> 6, r = qd & 63;
      const int wi = r >> 3, j = (r >> 1) & 3, s = r & 1;
      const int c0 = sl * kSliceCols + 32 * wi + j + 4 * s;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        scl[i][b] = qd < nquads ? src.scale(c0 + 8 * b) : 0.0f;
#pragma unroll
        for (int t = 0; t < kT; ++t)
          raw[i][b][t] = (qd < nquads && t < T) ? src.fetch(t, c0 + 8 * b) : typename Loader::Raw{};
      }
    }
#pragma unroll
    for (int i = 0; i < kQPT; ++i)
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int t = 0; t < kT; ++t) cv.v[i][b][t] = src.finish(raw[i][b][t], scl[i][b]);
  } else {
#pragma unroll
    for (int i = 0; i < kQPT; ++i) {
      const int qd = tid + i * kThreads;
      const int sl = qd >> 6, r = qd & 63;
      const int wi = r >> 3, j = (r >> 1) & 3, s = r & 1;
      const int c0 = sl * kSliceCols + 32 * wi + j + 4 * s;
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int t = 0; t < kT; ++t) cv.v[i][b][t] = (qd < nquads && t < T) ? src(t, c0 + 8 * b) : 0.0f;
    }
  }
}

// Quantises loaded activations per token to 22-bit fixed point (2^e from the
// chunk maximum), scatters the signed base-256 digits into B fragments and
// returns per token e and Q = sum q.  Two consumer barriers; the first also
// orders this chunk's fragment writes after every warp's previous MMAs.
template <int kT, int kQPT>
__device__ __forceinline__ void quantize_loaded(const ChunkValues<kT, kQPT> &cv, int nst, int T, uint8_t *smem_b,
                                                Scratch<kT> &sc, int (&e)[kT], long long (&Q)[kT]) {
  constexpr int kNT = n_tiles(kT);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nquads = nst * 64;
  const auto &v = cv.v;
  float mx[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    mx[t] = 0.0f;
#pragma unroll
    for (int i = 0; i < kQPT; ++i)
#pragma unroll
      for (int b = 0; b < 4; ++b) mx[t] = fmaxf(mx[t], fabsf(v[i][b][t]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx[t] = fmaxf(mx[t], __shfl_xor_sync(0xffffffffu, mx[t], off));
    if (lane == 0) sc.red_f[warp * kT + t] = mx[t];
  }
  consumer_sync();
  long long qs[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, sc.red_f[w * kT + t]);
    int ex = 0, et = 0;
    if (m > 0.0f && isfinite(m)) {
      frexpf(m, &ex);  // m < 2^ex
      et = min(fixed_bits(kT) - ex, 126);
    }
    e[t] = et;
    qs[t] = 0;
  }
#pragma unroll
  for (int i = 0; i < kQPT; ++i) {
    const int qd = tid + i * kThreads;
    if (qd < nquads) {
      const int sl = qd >> 6, r = qd & 63;
      const int wi = r >> 3, j = (r >> 1) & 3, s = r & 1;
      const int tig = wi & 3, hi = wi >> 2;  // word wi feeds a0/a1 (hi = 0) or a2/a3 (hi = 1) of lane tig
      const int kb = j * 2 + s;
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        if (t < T) {
          const float scale = tc::exp2_int(e[t]);
          int32_t q[4];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            q[b] = __float2int_rn(v[i][b][t] * scale);
            qs[t] += q[b];
          }
          constexpr int kD = digits_for(kT);
          uint32_t digits[kD];
          split_digits_n<kD>(q, digits);
#pragma unroll
          for (int d = 0; d < kD; ++d) {
            const int n = kD * t + d;
            const int nt = n >> 3, gg = n & 7;
            const uint32_t offset =
                ((static_cast<uint32_t>(sl) * 8 + kb) * kNT + nt) * kFragBytes + (gg * 4 + tig) * 8 + hi * 4;
            *reinterpret_cast<uint32_t *>(smem_b + offset) = digits[d];
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    long long x = qs[t];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    if (lane == 0) sc.red_q[warp * kT + t] = x;
  }
  consumer_sync();
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    long long x = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) x += sc.red_q[w * kT + t];
    Q[t] = x;
  }
}

// load_chunk then quantize_loaded.
// quantize_chunk for the kG tokens t0 .. t0 + kG - 1 of a kT-token instance
// (two digits per token, kG x 2 = 4 N columns: one half of an N tile): the
// same exponents, digits and digit sums as quantize_chunk gives those tokens,
// written to the same fragment positions.  Used by the grid-wide
// pre-quantisation pass, which splits a chunk's tokens over several CTAs.
template <int kT, int kG, int kQPT, typename Loader>
__device__ __forceinline__ void quantize_tokens(const Loader &src, int nst, int t0, int T, uint8_t *smem_b,
                                                Scratch<kT> &sc, int (&e)[kG], long long (&Q)[kG]) {
  constexpr int kNT = n_tiles(kT);
  constexpr int kD = digits_for(kT);
  static_assert(kD * kG == 4, "a token group fills half an N tile");
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nquads = nst * 64;
  float scl[kQPT][4];
  typename Loader::Raw raw[kQPT][4][kG];
#pragma unroll
  for (int i = 0; i < kQPT; ++i) {
    const int qd = tid + i * kThreads;
    const int sl = qd >> 6, r = qd & 63;
    const int wi = r >> 3, j = (r >> 1) & 3, s = r & 1;
    const int c0 = sl * kSliceCols + 32 * wi + j + 4 * s;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      scl[i][b] = qd < nquads ? src.scale(c0 + 8 * b) : 0.0f;
#pragma unroll
      for (int t = 0; t < kG; ++t)
        raw[i][b][t] = (qd < nquads && t0 + t < T) ? src.fetch(t0 + t, c0 + 8 * b) : typename Loader::Raw{};
    }
  }
  float v[kQPT][4][kG];
  float mx[kG];
#pragma unroll
  for (int t = 0; t < kG; ++t) mx[t] = 0.0f;
#pragma unroll
  for (int i = 0; i < kQPT; ++i)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int t = 0; t < kG; ++t) {
        v[i][b][t] = src.finish(raw[i][b][t], scl[i][b]);
        mx[t] = fmaxf(mx[t], fabsf(v[i][b][t]));
      }
#pragma unroll
  for (int t = 0; t < kG; ++t) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx[t] = fmaxf(mx[t], __shfl_xor_sync(0xffffffffu, mx[t], off));
    if (lane == 0) sc.red_f[warp * kT + t] = mx[t];
  }
  consumer_sync();
  long long qs[kG];
#pragma unroll
  for (int t = 0; t < kG; ++t) {
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, sc.red_f[w * kT + t]);
    int ex = 0, et = 0;
    if (m > 0.0f && isfinite(m)) {
      frexpf(m, &ex);  // m < 2^ex
      et = min(fixed_bits(kT) - ex, 126);
    }
    e[t] = et;
    qs[t] = 0;
  }
#pragma unroll
  for (int i = 0; i < kQPT; ++i) {
    const int qd = tid + i * kThreads;
    if (qd < nquads) {
      const int sl = qd >> 6, r = qd & 63;
      const int wi = r >> 3, j = (r >> 1) & 3, s = r & 1;
      const int tig = wi & 3, hi = wi >> 2;
      const int kb = j * 2 + s;
#pragma unroll
      for (int t = 0; t < kG; ++t) {
        if (t0 + t < T) {
          const float scale = tc::exp2_int(e[t]);
          int32_t q[4];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            q[b] = __float2int_rn(v[i][b][t] * scale);
            qs[t] += q[b];
          }
          uint32_t digits[kD];
          split_digits_n<kD>(q, digits);
#pragma unroll
          for (int d = 0; d < kD; ++d) {
            const int n = kD * (t0 + t) + d;
            const int nt = n >> 3, gg = n & 7;
            const uint32_t offset =
                ((static_cast<uint32_t>(sl) * 8 + kb) * kNT + nt) * kFragBytes + (gg * 4 + tig) * 8 + hi * 4;
            *reinterpret_cast<uint32_t *>(smem_b + offset) = digits[d];
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kG; ++t) {
    long long x = qs[t];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    if (lane == 0) sc.red_q[warp * kT + t] = x;
  }
  consumer_sync();
#pragma unroll
  for (int t = 0; t < kG; ++t) {
    long long x = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) x += sc.red_q[w * kT + t];
    Q[t] = x;
  }
}

template <int kT, int kQPT, typename Loader>
__device__ __forceinline__ void quantize_chunk(const Loader &src, int nst, int T, uint8_t *smem_b, Scratch<kT> &sc,
                                               int (&e)[kT], long long (&Q)[kT]) {
  ChunkValues<kT, kQPT> cv;
  load_chunk<kT, kQPT>(src, nst, T, cv);
  quantize_loaded<kT, kQPT>(cv, nst, T, smem_b, sc, e, Q);
}

// This lane's four sign words of one slice: rows (16 warp + g) and +8, words
// tig and tig + 4 (row-interleaved slice: [2 chunks][128 rows][4 words]).
struct SliceWords {
  uint32_t w00, w10, w01, w11;  // [row g / g+8][word tig / tig+4]
};

__device__ __forceinline__ SliceWords load_slice_words(const uint8_t *slot, int warp, int lane) {
  const int g = lane >> 2, tig = lane & 3;
  const int r0 = warp * 16 + g;
  const uint32_t *c0 = reinterpret_cast<const uint32_t *>(slot);
  const uint32_t *c1 = reinterpret_cast<const uint32_t *>(slot + kSliceBytes / 2);
  SliceWords s;
  s.w00 = c0[r0 * 4 + tig];
  s.w10 = c0[(r0 + 8) * 4 + tig];
  s.w01 = c1[r0 * 4 + tig];
  s.w11 = c1[(r0 + 8) * 4 + tig];
  return s;
}

// Accumulator sets per class: separate sets for the two K halves (h) keep
// eight independent MMA chains when registers allow.
__host__ __device__ constexpr int acc_sets(int nt) { return nt <= 2 ? 8 : 4; }

// The 8 x kNT MMAs of one slice into the accumulators d[set][nt].
template <int kNT>
__device__ __forceinline__ void slice_mmas(const SliceWords &w, const uint8_t *frags, int lane,
                                           int32_t (&d)[acc_sets(kNT)][kNT][4]) {
#pragma unroll
  for (int kb = 0; kb < 8; ++kb) {
    const int j = kb >> 1, h = kb & 1;
    const int set = acc_sets(kNT) == 8 ? kb : j;
    const uint32_t m = 0x01010101u << j;
    const uint32_t a0 = (w.w00 >> (4 * h)) & m, a1 = (w.w10 >> (4 * h)) & m;
    const uint32_t a2 = (w.w01 >> (4 * h)) & m, a3 = (w.w11 >> (4 * h)) & m;
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      const uint2 b = *reinterpret_cast<const uint2 *>(frags + (kb * kNT + nt) * kFragBytes + lane * 8);
      mma_s8(d[set][nt], a0, a1, a2, a3, b.x, b.y);
    }
  }
}

// Combines classes and digits of the accumulators and adds the fp32 value of
// every token to acc[t * 128 + row] for this lane's two rows (each (row,
// token) is written by exactly one lane).
template <int kT>
__device__ __forceinline__ void drain_to_acc(int32_t (&d)[acc_sets(n_tiles(kT))][n_tiles(kT)][4], int T, int warp,
                                             int lane, const int (&e)[kT], const long long (&Q)[kT], float *acc) {
  constexpr int kNT = n_tiles(kT);
  constexpr int kSets = acc_sets(kNT);
  const int g = lane >> 2, tig = lane & 3;
  int32_t v[kNT][4];
#pragma unroll
  for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int32_t x = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int32_t dj = kSets == 8 ? d[2 * j][nt][c] + d[2 * j + 1][nt][c] : d[j][nt][c];
        x += dj >> j;
      }
      v[nt][c] = x;
    }
  const int r0 = warp * 16 + g;
  constexpr int kD = digits_for(kT);
  if constexpr (kD == 2) {
    // Two digits: columns 2t and 2t + 1 (both digits of token t = 4 nt + tig)
    // are this lane's registers c and c + 1, so every lane combines its own
    // tokens without shuffles (same arithmetic, same single writer per entry).
    static_assert(kT == 4 * kNT, "two digits per token fill whole N tiles");
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      const int t = nt * 4 + tig;
      int et = e[nt * 4];
      long long qt = Q[nt * 4];
#pragma unroll
      for (int k = 1; k < 4; ++k)
        if (tig == k) {
          et = e[nt * 4 + k];
          qt = Q[nt * 4 + k];
        }
      if (t < T) {
        const float unscale = tc::exp2_int(-et);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const long long s = static_cast<long long>(v[nt][2 * rr + 1]) * 256 + v[nt][2 * rr];
          acc[t * kTileRows + r0 + rr * 8] += __ll2float_rn(qt - 2 * s) * unscale;
        }
      }
    }
    return;
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
    // digit dd of token t sits in column kD t + dd: N tile (kD t+dd)/8, lane tig ((kD t+dd)%8)/2, register (..)%2
    int32_t dig[2][kD];
#pragma unroll
    for (int dd = 0; dd < kD; ++dd) {
      const int n = kD * t + dd;
      const int nt = n >> 3, cc = n & 7;
      const int src = g * 4 + (cc >> 1);
      dig[0][dd] = __shfl_sync(0xffffffffu, v[nt][cc & 1], src);
      dig[1][dd] = __shfl_sync(0xffffffffu, v[nt][2 + (cc & 1)], src);
    }
    if (t < T && tig == ((kD * t) & 7) >> 1) {
      const float unscale = tc::exp2_int(-e[t]);
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        long long s = 0;
#pragma unroll
        for (int dd = kD - 1; dd >= 0; --dd) s = s * 256 + dig[rr][dd];
        acc[t * kTileRows + r0 + rr * 8] += __ll2float_rn(Q[t] - 2 * s) * unscale;
      }
    }
  }
}

}  // namespace mmad
}  // namespace nqb
