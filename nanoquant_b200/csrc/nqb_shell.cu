// Decode-step shell kernels (batch 1..16): the work of a decoder step around
// its packed linears -- RMSNorm with the residual add, per-head q/k RMSNorm
// with rotate-half RoPE and the KV-cache append, split-K grouped-query
// attention over the bf16 cache, the SwiGLU product, and the bf16 output
// projection (lm head) as an HBM-streaming GEMV.
//
// Every reduction runs in a fixed order (warp shuffles, then the warps'
// partials in index order), so results are bitwise reproducible.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "nqb.h"
#include "nqb_common.cuh"

namespace nqb {
namespace shell {

__device__ __forceinline__ void store_as(void *p, int64_t i, int32_t dt, float v) {
  if (dt == NQB_F32) {
    static_cast<float *>(p)[i] = v;
  } else if (dt == NQB_BF16) {
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half *>(p)[i] = __float2half_rn(v);
  }
}

// Lets a decode program launched as this kernel's programmatic dependent
// (nqb_program_run_dependent) launch now and start streaming its sign words;
// the program still waits for this kernel's completion before reading its output.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Sum over the block (blockDim.x a multiple of 32, at most 1024 threads).
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float s = 0.0f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += scratch[w];
  __syncthreads();
  return s;
}

// One block per token: h += delta (when given, written back), then
// out = h * rsqrt(mean(h^2) + eps) * w.  Rows of up to kRmsVec * 1024 values
// (a multiple of 4, 16-byte aligned) stay in registers: every load of the row
// is issued before any is used (one memory round trip instead of one per
// loop step, which the in-place write-back otherwise forces).
constexpr int kRmsVec = 8;  // float4 pieces per thread (256 threads: hidden <= 8192)

// Elements i .. i + 3 of a float vector (16-byte aligned base, i % 4 == 0).
__device__ __forceinline__ float4 load4_as_float(const void *p, int64_t i, int32_t dt) {
  if (dt == NQB_F32) return __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(p) + i));
  const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p) + i));
  float2 a, b;
  if (dt == NQB_BF16) {
    a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.x));
    b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw.y));
  } else {
    a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
  }
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ void store4_as(void *p, int64_t i, int32_t dt, float4 v) {
  if (dt == NQB_F32) {
    *reinterpret_cast<float4 *>(static_cast<float *>(p) + i) = v;
    return;
  }
  uint2 raw;
  if (dt == NQB_BF16) {
    *reinterpret_cast<__nv_bfloat162 *>(&raw.x) = __floats2bfloat162_rn(v.x, v.y);
    *reinterpret_cast<__nv_bfloat162 *>(&raw.y) = __floats2bfloat162_rn(v.z, v.w);
  } else {
    *reinterpret_cast<__half2 *>(&raw.x) = __floats2half2_rn(v.x, v.y);
    *reinterpret_cast<__half2 *>(&raw.y) = __floats2half2_rn(v.z, v.w);
  }
  *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(p) + i) = raw;
}

//
// With `dw` (the delta's own norm weight), the delta is normalised before the
// add: h += delta * rsqrt(mean(delta^2) + eps) * dw (Gemma-3's post-attention
// and post-feedforward norms), then out is formed from the new h as above.
__global__ void __launch_bounds__(256) rmsnorm_kernel(float *h, const float *delta, const void *w, int32_t w_dt,
                                                      int64_t hidden, float eps, void *out, int32_t out_dt,
                                                      const void *dw = nullptr) {
  __shared__ float scratch[32];
  allow_dependents();
  const int64_t t = blockIdx.x;
  const bool vec = hidden % 4 == 0 && hidden <= 1024 * kRmsVec && reinterpret_cast<uintptr_t>(h) % 16 == 0 &&
                   (delta == nullptr || reinterpret_cast<uintptr_t>(delta) % 16 == 0) &&
                   reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dw) % 16 == 0;
  if (vec) {
    float4 *row4 = reinterpret_cast<float4 *>(h + t * hidden);
    const float4 *d4 = delta != nullptr ? reinterpret_cast<const float4 *>(delta + t * hidden) : nullptr;
    const int n4 = static_cast<int>(hidden / 4);
    float4 v[kRmsVec], wv[kRmsVec];  // the weights load with the row, before the reduction
#pragma unroll
    for (int j = 0; j < kRmsVec; ++j) {
      const int i = threadIdx.x + j * 256;
      v[j] = i < n4 ? row4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      wv[j] = i < n4 ? load4_as_float(w, 4 * static_cast<int64_t>(i), w_dt) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    if (d4 != nullptr) {
      float4 dv[kRmsVec], dwv[kRmsVec];
#pragma unroll
      for (int j = 0; j < kRmsVec; ++j) {
        const int i = threadIdx.x + j * 256;
        dv[j] = i < n4 ? d4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        dwv[j] = dw != nullptr && i < n4 ? load4_as_float(dw, 4 * static_cast<int64_t>(i), w_dt)
                                         : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
      }
      if (dw != nullptr) {
        float dss = 0.0f;
#pragma unroll
        for (int j = 0; j < kRmsVec; ++j)
          dss += dv[j].x * dv[j].x + dv[j].y * dv[j].y + dv[j].z * dv[j].z + dv[j].w * dv[j].w;
        const float dr = rsqrtf(block_sum(dss, scratch) / static_cast<float>(hidden) + eps);
#pragma unroll
        for (int j = 0; j < kRmsVec; ++j) {
          dv[j].x = dv[j].x * dr * dwv[j].x;
          dv[j].y = dv[j].y * dr * dwv[j].y;
          dv[j].z = dv[j].z * dr * dwv[j].z;
          dv[j].w = dv[j].w * dr * dwv[j].w;
        }
      }
#pragma unroll
      for (int j = 0; j < kRmsVec; ++j) {
        const int i = threadIdx.x + j * 256;
        if (i < n4) {
          v[j].x += dv[j].x;
          v[j].y += dv[j].y;
          v[j].z += dv[j].z;
          v[j].w += dv[j].w;
          row4[i] = v[j];
        }
      }
    }
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kRmsVec; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    const float r = rsqrtf(block_sum(ss, scratch) / static_cast<float>(hidden) + eps);
#pragma unroll
    for (int j = 0; j < kRmsVec; ++j) {
      const int i = threadIdx.x + j * 256;
      if (i < n4)
        store4_as(out, t * hidden + 4 * static_cast<int64_t>(i), out_dt,
                  make_float4(v[j].x * r * wv[j].x, v[j].y * r * wv[j].y, v[j].z * r * wv[j].z, v[j].w * r * wv[j].w));
    }
    return;
  }
  float *row = h + t * hidden;
  const float *drow = delta != nullptr ? delta + t * hidden : nullptr;
  float dr = 1.0f;
  if (drow != nullptr && dw != nullptr) {
    float dss = 0.0f;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) dss += drow[i] * drow[i];
    dr = rsqrtf(block_sum(dss, scratch) / static_cast<float>(hidden) + eps);
  }
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = row[i];
    if (drow != nullptr) {
      v += dw != nullptr ? drow[i] * dr * load_as_float(dw, i, w_dt) : drow[i];
      row[i] = v;
    }
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, scratch) / static_cast<float>(hidden) + eps);
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x)
    store_as(out, t * hidden + i, out_dt, row[i] * r * load_as_float(w, i, w_dt));
}

// One warp per (token, head) over q heads, then k heads, then v heads.  Lane
// l holds dimensions [l * kDpl, (l + 1) * kDpl); the rotate-half partner of a
// dimension is in lane l ^ 16.  q and k: RMSNorm over the head (weight
// optional), then RoPE with the token's cos/sin rows; q goes to q_out, k and
// v to the caches at position + t.
template <int kDpl>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const float *q, const float *k, const float *v, const void *qw, const void *kw, int32_t w_dt, const float *cos_t,
    const float *sin_t, int64_t tokens, int32_t q_heads, int32_t kv_heads, float eps, __nv_bfloat16 *q_out,
    __nv_bfloat16 *kcache, __nv_bfloat16 *vcache, int64_t cache_len, int64_t position) {
  constexpr int kHd = 32 * kDpl;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = q_heads + 2 * kv_heads;
  if (gw >= tokens * heads) return;  // uniform over the warp
  const int64_t t = gw / heads;
  const int hh = static_cast<int>(gw - t * heads);
  const int d0 = lane * kDpl;
  const float *src;
  const void *w = nullptr;
  __nv_bfloat16 *dst;
  bool rope = true;
  if (hh < q_heads) {
    src = q + (t * q_heads + hh) * kHd;
    w = qw;
    dst = q_out + (t * q_heads + hh) * kHd;
  } else if (hh < q_heads + kv_heads) {
    const int kh = hh - q_heads;
    src = k + (t * kv_heads + kh) * kHd;
    w = kw;
    dst = kcache + (static_cast<int64_t>(kh) * cache_len + position + t) * kHd;
  } else {
    const int vh = hh - q_heads - kv_heads;
    src = v + (t * kv_heads + vh) * kHd;
    dst = vcache + (static_cast<int64_t>(vh) * cache_len + position + t) * kHd;
    rope = false;
  }
  // the head's values, norm weights and cos/sin rows load together (one round trip)
  float x[kDpl], wv[kDpl], cv[kDpl], sv[kDpl];
  const float *c = cos_t + t * kHd;
  const float *sn = sin_t + t * kHd;
#pragma unroll
  for (int j = 0; j < kDpl; ++j) {
    x[j] = src[d0 + j];
    wv[j] = rope && w != nullptr ? load_as_float(w, d0 + j, w_dt) : 1.0f;
    cv[j] = rope ? c[d0 + j] : 0.0f;
    sv[j] = rope ? sn[d0 + j] : 0.0f;
  }
  if (rope) {  // uniform over the warp
    if (w != nullptr) {
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < kDpl; ++j) ss += x[j] * x[j];
      const float r = rsqrtf(warp_sum(ss) / static_cast<float>(kHd) + eps);
#pragma unroll
      for (int j = 0; j < kDpl; ++j) x[j] = x[j] * r * wv[j];
    }
    float partner[kDpl];
#pragma unroll
    for (int j = 0; j < kDpl; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, x[j], 16);
    const float sign = lane < 16 ? -1.0f : 1.0f;  // rotate_half: (-x2, x1)
#pragma unroll
    for (int j = 0; j < kDpl; ++j) x[j] = x[j] * cv[j] + sign * partner[j] * sv[j];
  }
#pragma unroll
  for (int j = 0; j < kDpl; ++j) dst[d0 + j] = __float2bfloat16_rn(x[j]);
}

// kDpl consecutive bf16 values (4, 8 or 16 bytes, aligned) as floats.
template <int kDpl>
__device__ __forceinline__ void load_bf16_row(const __nv_bfloat16 *p, float (&out)[kDpl]) {
  if constexpr (kDpl == 2) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(p));
    out[0] = f.x;
    out[1] = f.y;
  } else if constexpr (kDpl == 4) {
    const uint2 raw = *reinterpret_cast<const uint2 *>(p);
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  } else {
    static_assert(kDpl == 8, "2, 4 or 8 values per lane");
    const uint4 raw = *reinterpret_cast<const uint4 *>(p);
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  }
}

constexpr int kStageKeys = 64;  // K and V rows staged in shared memory at once
// A split's partial row: hd accumulators, m, l and two pad floats, so every
// row (and every lane's slice of it) starts on a 16-byte boundary.
constexpr int kPartPad = 4;

template <int kDpl>
__device__ __forceinline__ void load_f32_slice(const float *p, float (&out)[kDpl]) {
  if constexpr (kDpl == 2) {
    const float2 v = *reinterpret_cast<const float2 *>(p);
    out[0] = v.x;
    out[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < kDpl; i += 4) {
      const float4 v = *reinterpret_cast<const float4 *>(p + i);
      out[i] = v.x;
      out[i + 1] = v.y;
      out[i + 2] = v.z;
      out[i + 3] = v.w;
    }
  }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Split-K attention partials.  Grid (kv_heads, splits, tokens); one warp per
// q head of the kv head's group.  Token t sees keys [0, keys + t); split sp
// covers [sp * chunk, min((sp + 1) * chunk, keys + t)).  The block copies up
// to 64 of its K and V rows at once into shared memory (16-byte cp.async,
// all in flight together: one memory round trip, the rows of a kv head are
// contiguous) and the group's warps read them from there, keys in blocks of
// kB with the kB dot-product reductions interleaved.  Writes (acc[hd], m, l)
// of an online softmax per (token, q head, split).
template <int kDpl>
__global__ void attention_partial_kernel(const __nv_bfloat16 *q, const __nv_bfloat16 *kc, const __nv_bfloat16 *vc,
                                         int64_t cache_len, int64_t keys, int32_t q_heads, int32_t kv_heads,
                                         int32_t splits, int64_t chunk, float scale, float *part, int64_t window) {
  constexpr int kHd = 32 * kDpl;
  constexpr int kB = kDpl <= 4 ? 8 : 4;
  const int kh = blockIdx.x, sp = blockIdx.y;
  const int64_t t = blockIdx.z;
  const int group = q_heads / kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = kh * group + warp;
  const int d0 = lane * kDpl;
  const int64_t visible = keys + t;
  // a sliding window of `window` keys ends at the token's own row
  const int64_t first = window > 0 && visible > window ? visible - window : 0;
  const int64_t j0 = max(static_cast<int64_t>(sp) * chunk, first);
  const int64_t j1 = min(static_cast<int64_t>(sp) * chunk + chunk, visible);
  float qv[kDpl], acc[kDpl];
  load_bf16_row<kDpl>(q + (t * q_heads + qh) * kHd + d0, qv);
#pragma unroll
  for (int j = 0; j < kDpl; ++j) {
    qv[j] *= scale;
    acc[j] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  extern __shared__ __align__(16) uint8_t s_rows[];  // [kStageKeys][kHd] K rows, then V rows
  __nv_bfloat16 *sk = reinterpret_cast<__nv_bfloat16 *>(s_rows);
  __nv_bfloat16 *sv = sk + kStageKeys * kHd;
  const char *kg = reinterpret_cast<const char *>(kc + static_cast<int64_t>(kh) * cache_len * kHd);
  const char *vg = reinterpret_cast<const char *>(vc + static_cast<int64_t>(kh) * cache_len * kHd);
  for (int64_t s0 = j0; s0 < j1; s0 += kStageKeys) {
    const int rows = static_cast<int>(min(static_cast<int64_t>(kStageKeys), j1 - s0));
    const int chunks = rows * kHd * 2 / 16;  // 16-byte pieces per matrix
    for (int i = threadIdx.x; i < 2 * chunks; i += blockDim.x) {
      const bool is_v = i >= chunks;
      const int c = is_v ? i - chunks : i;
      cp_async16(reinterpret_cast<char *>(is_v ? sv : sk) + c * 16, (is_v ? vg : kg) + s0 * kHd * 2 + c * 16);
    }
    cp_async_wait_all();
    __syncthreads();
    for (int j = 0; j < rows; j += kB) {
      const int nb = min(kB, rows - j);
      float kv[kB][kDpl], vv[kB][kDpl];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int row = j + (b < nb ? b : 0);  // rows past the block re-read row j (masked below)
        load_bf16_row<kDpl>(sk + row * kHd + d0, kv[b]);
        load_bf16_row<kDpl>(sv + row * kHd + d0, vv[b]);
      }
      float sc[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        float d = 0.0f;
#pragma unroll
        for (int e = 0; e < kDpl; ++e) d += qv[e] * kv[b][e];
        sc[b] = d;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int b = 0; b < kB; ++b) sc[b] += __shfl_xor_sync(0xffffffffu, sc[b], off);
      }
      float mb = sc[0];
#pragma unroll
      for (int b = 1; b < kB; ++b)
        if (b < nb) mb = fmaxf(mb, sc[b]);
      const float mn = fmaxf(m, mb);
      const float corr = expf(m - mn);
      l *= corr;
#pragma unroll
      for (int e = 0; e < kDpl; ++e) acc[e] *= corr;
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        if (b < nb) {
          const float p = expf(sc[b] - mn);
          l += p;
#pragma unroll
          for (int e = 0; e < kDpl; ++e) acc[e] += p * vv[b][e];
        }
      }
      m = mn;
    }
    __syncthreads();  // every warp is done with the staged rows before the next copy
  }
  float *o = part + ((t * q_heads + qh) * splits + sp) * (kHd + kPartPad);
#pragma unroll
  for (int e = 0; e < kDpl; ++e) o[d0 + e] = acc[e];  // contiguous: the compiler vectorises
  if (lane == 0) {
    o[kHd] = m;
    o[kHd + 1] = l;
  }
}

// One warp per (token, q head): joins the splits in index order.
template <int kDpl>
__global__ void attention_combine_kernel(const float *part, int32_t splits, int64_t tokens, int32_t q_heads,
                                         __nv_bfloat16 *out) {
  constexpr int kHd = 32 * kDpl;
  allow_dependents();
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= tokens * q_heads) return;
  const float *base = part + gw * splits * (kHd + kPartPad);
  // (m, l) of split lane and lane + 32 (splits <= 64), read once in parallel
  const float m0 = lane < splits ? base[lane * (kHd + kPartPad) + kHd] : -INFINITY;
  const float m1 = lane + 32 < splits ? base[(lane + 32) * (kHd + kPartPad) + kHd] : -INFINITY;
  const float l0 = lane < splits ? base[lane * (kHd + kPartPad) + kHd + 1] : 0.0f;
  const float l1 = lane + 32 < splits ? base[(lane + 32) * (kHd + kPartPad) + kHd + 1] : 0.0f;
  float mx = fmaxf(m0, m1);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float f0 = m0 == -INFINITY ? 0.0f : expf(m0 - mx);
  const float f1 = m1 == -INFINITY ? 0.0f : expf(m1 - mx);
  float den = f0 * l0 + f1 * l1;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  // weighted sum of the splits' vectors: a lane's slice of a split is one
  // aligned vector load (rows padded to hd + 4 floats), kU splits in flight
  constexpr int kU = kDpl <= 4 ? 16 : 8;
  float num[kDpl];
#pragma unroll
  for (int e = 0; e < kDpl; ++e) num[e] = 0.0f;
  for (int s0 = 0; s0 < splits; s0 += kU) {
    float vals[kU][kDpl];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int s = min(s0 + u, splits - 1);
      load_f32_slice<kDpl>(base + s * (kHd + kPartPad) + lane * kDpl, vals[u]);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int s = s0 + u;
      const float f = __shfl_sync(0xffffffffu, (s & 32) ? f1 : f0, s & 31);
      if (s < splits) {
#pragma unroll
        for (int e = 0; e < kDpl; ++e) num[e] += f * vals[u][e];
      }
    }
  }
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;
#pragma unroll
  for (int e = 0; e < kDpl; ++e) out[gw * kHd + lane * kDpl + e] = __float2bfloat16_rn(num[e] * inv);
}

// out[t, :] = float(W[ids[t], :]) * scale: one block per token, 16-byte
// loads of the bf16 row (dim a multiple of 8, 16-byte aligned rows) or a
// scalar loop; an id outside [0, rows) gives a zero row.
__global__ void __launch_bounds__(256) embedding_bf16_kernel(const int64_t *ids, const __nv_bfloat16 *w, int64_t rows,
                                                             int64_t dim, float scale, float *out) {
  allow_dependents();
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  float *o = out + t * dim;
  const bool valid = id >= 0 && id < rows;
  if (dim % 8 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    const uint4 *src = reinterpret_cast<const uint4 *>(w + (valid ? id : 0) * dim);
    for (int64_t u = threadIdx.x; u < dim / 8; u += blockDim.x) {
      float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f), b = a;
      if (valid) {
        const uint4 raw = __ldg(src + u);
        const __nv_bfloat162 *pairs = reinterpret_cast<const __nv_bfloat162 *>(&raw);
        const float2 f0 = __bfloat1622float2(pairs[0]), f1 = __bfloat1622float2(pairs[1]);
        const float2 f2 = __bfloat1622float2(pairs[2]), f3 = __bfloat1622float2(pairs[3]);
        a = make_float4(f0.x * scale, f0.y * scale, f1.x * scale, f1.y * scale);
        b = make_float4(f2.x * scale, f2.y * scale, f3.x * scale, f3.y * scale);
      }
      reinterpret_cast<float4 *>(o)[2 * u] = a;
      reinterpret_cast<float4 *>(o)[2 * u + 1] = b;
    }
    return;
  }
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x)
    o[i] = valid ? __bfloat162float(w[id * dim + i]) * scale : 0.0f;
}

__global__ void silu_mul_kernel(const float *gate, const float *up, int64_t n, void *out, int32_t out_dt) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float g = gate[i];
  store_as(out, i, out_dt, g / (1.0f + expf(-g)) * up[i]);
}

// out[t][r] = sum_c W[r][c] x[t][c] for kT tokens; W bf16 [rows][cols] with
// cols % 8 == 0 and 16-byte aligned rows, streamed once with 16-byte loads;
// x staged in shared memory as fp32.  One warp per row, rows strided over
// the grid's warps.
template <int kT>
__global__ void __launch_bounds__(256) gemv_bf16_kernel(const __nv_bfloat16 *w, const __nv_bfloat16 *x, int64_t rows,
                                                        int64_t cols, int64_t x_stride, float *out, int64_t out_stride) {
  extern __shared__ float xs[];  // [kT][cols]
  for (int64_t i = threadIdx.x; i < kT * cols; i += blockDim.x) {
    const int64_t t = i / cols;
    xs[i] = __bfloat162float(x[t * x_stride + (i - t * cols)]);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t units = cols / 8;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(w + r * cols);
    float acc[kT];
#pragma unroll
    for (int t = 0; t < kT; ++t) acc[t] = 0.0f;
#pragma unroll 8
    for (int64_t u = lane; u < units; u += 32) {
      const uint4 raw = __ldcs(wr + u);
      const __nv_bfloat162 *pairs = reinterpret_cast<const __nv_bfloat162 *>(&raw);
      const float2 f0 = __bfloat1622float2(pairs[0]), f1 = __bfloat1622float2(pairs[1]);
      const float2 f2 = __bfloat1622float2(pairs[2]), f3 = __bfloat1622float2(pairs[3]);
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        // x as two 16-byte shared loads (cols % 8 == 0 keeps them aligned)
        const float4 *xv = reinterpret_cast<const float4 *>(xs + t * cols + u * 8);
        const float4 a = xv[0], b = xv[1];
        acc[t] += f0.x * a.x + f0.y * a.y + f1.x * a.z + f1.y * a.w + f2.x * b.x + f2.y * b.y + f3.x * b.z +
                  f3.y * b.w;
      }
    }
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const float s = warp_sum(acc[t]);
      if (lane == 0) out[t * out_stride + r] = s;
    }
  }
}

// out[t][r] = sum_c W[r][c] x[t][c] for 2 .. 8 * kNT tokens on the tensor
// cores: mma.sync m16n8k16 bf16 with fp32 accumulation, A = a 16-row tile of W,
// B = the tokens (kNT tiles of 8).  One warp per 16-row tile, tiles strided
// over the grid's warps.  K goes in 32-column blocks; lane (g, q) = (lane / 4,
// lane % 4) loads W[row g][8q .. 8q + 7] and W[row g + 8][8q .. 8q + 7] as
// 16-byte streaming loads (kU blocks in flight) and x[token][8q .. 8q + 7]
// from shared memory, and uses the eight values as its fragment elements of
// two 16-wide k-steps: columns 8q + {0,1}, 8q + {2,3} for the first and
// 8q + {4,5}, 8q + {6,7} for the second.  That is a permutation of K applied
// to A and B alike, so the sums are unchanged and every load is one
// contiguous vector.  x rows in shared memory are padded by 16 bytes, which
// spreads a fragment load's 32 lanes over the banks (4 wavefronts for 512 B).
template <int kNT>
__global__ void __launch_bounds__(256) gemv_bf16_mma_kernel(const __nv_bfloat16 *w, const __nv_bfloat16 *x,
                                                            int64_t rows, int64_t cols, int tokens, float *out,
                                                            int64_t out_stride) {
  constexpr int kU = 8;  // 32-column blocks of W in flight per lane
  extern __shared__ uint4 xs_units[];  // [kNT * 8][cols / 8 + 1] (16-byte units, one unit of padding per row)
  allow_dependents();
  const int64_t units = cols / 8;
  const int64_t stride = units + 1;
  for (int64_t i = threadIdx.x; i < kNT * 8 * units; i += blockDim.x) {
    const int64_t t = i / units, u = i - t * units;
    xs_units[t * stride + u] =
        t < tokens ? __ldg(reinterpret_cast<const uint4 *>(x + t * cols) + u) : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t blocks = cols / 32;
  for (int64_t tile = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); tile * 16 < rows;
       tile += warps) {
    const int64_t r0 = tile * 16 + g, r1 = r0 + 8;
    const uint4 *wa = reinterpret_cast<const uint4 *>(w + min(r0, rows - 1) * cols) + q;
    const uint4 *wb = reinterpret_cast<const uint4 *>(w + min(r1, rows - 1) * cols) + q;
    float acc[kNT][4];
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[nt][c] = 0.0f;
    for (int64_t b0 = 0; b0 < blocks; b0 += kU) {
      uint4 a0[kU], a1[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t b = min(b0 + u, blocks - 1);  // past the row's end: re-read its last block (unused)
        a0[u] = __ldcs(wa + 4 * b);
        a1[u] = __ldcs(wb + 4 * b);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (b0 + u >= blocks) break;
#pragma unroll
        for (int nt = 0; nt < kNT; ++nt) {
          const uint4 bx = xs_units[static_cast<int64_t>(nt * 8 + g) * stride + 4 * (b0 + u) + q];
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
              "{%0,%1,%2,%3};"
              : "+f"(acc[nt][0]), "+f"(acc[nt][1]), "+f"(acc[nt][2]), "+f"(acc[nt][3])
              : "r"(a0[u].x), "r"(a1[u].x), "r"(a0[u].y), "r"(a1[u].y), "r"(bx.x), "r"(bx.y));
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
              "{%0,%1,%2,%3};"
              : "+f"(acc[nt][0]), "+f"(acc[nt][1]), "+f"(acc[nt][2]), "+f"(acc[nt][3])
              : "r"(a0[u].z), "r"(a1[u].z), "r"(a0[u].w), "r"(a1[u].w), "r"(bx.z), "r"(bx.w));
        }
      }
    }
    // D: c0, c1 = rows g, columns (tokens) 2q, 2q + 1; c2, c3 = row g + 8
#pragma unroll
    for (int nt = 0; nt < kNT; ++nt) {
      const int t0 = nt * 8 + 2 * q;
      if (r0 < rows) {
        if (t0 < tokens) out[t0 * out_stride + r0] = acc[nt][0];
        if (t0 + 1 < tokens) out[(t0 + 1) * out_stride + r0] = acc[nt][1];
      }
      if (r1 < rows) {
        if (t0 < tokens) out[t0 * out_stride + r1] = acc[nt][2];
        if (t0 + 1 < tokens) out[(t0 + 1) * out_stride + r1] = acc[nt][3];
      }
    }
  }
}

// Splits of the attention: 64 keys each (eight blocks of eight per warp), at
// most 64.  (32-key splits measured slower: the combine over twice as many
// partials costs more than the shorter key loop saves.)
int splits_for(int64_t keys, int64_t tokens) {
  const int64_t most = keys + tokens - 1;
  const int64_t s = (most + 63) / 64;
  return static_cast<int>(s < 1 ? 1 : (s > 64 ? 64 : s));
}

size_t attention_smem_bytes(int head_dim) { return 2ull * kStageKeys * head_dim * sizeof(__nv_bfloat16); }

int launch_sm_count() {
  int device = 0, sms = 148;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms;
}

}  // namespace shell
}  // namespace nqb

using namespace nqb;

extern "C" {

int nqb_rmsnorm(float *h, const float *delta, const void *weight, int32_t weight_dtype, int64_t tokens, int64_t hidden,
                float eps, void *out, int32_t out_dtype, void *stream) {
  return nqb_rmsnorm_residual(h, delta, nullptr, weight, weight_dtype, tokens, hidden, eps, out, out_dtype, stream);
}

int nqb_rmsnorm_residual(float *h, const float *delta, const void *delta_weight, const void *weight,
                         int32_t weight_dtype, int64_t tokens, int64_t hidden, float eps, void *out, int32_t out_dtype,
                         void *stream) {
  if (h == nullptr || weight == nullptr || out == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "rmsnorm operand is NULL");
  if (delta_weight != nullptr && delta == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "rmsnorm delta weight given without a delta");
  if (tokens <= 0 || hidden <= 0 || !(eps >= 0.0f)) return fail(NQB_ERR_INVALID_ARGUMENT, "rmsnorm shape or eps invalid");
  if (!is_float_dtype(weight_dtype) || !is_float_dtype(out_dtype)) return fail(NQB_ERR_DTYPE, "rmsnorm dtype invalid");
  shell::rmsnorm_kernel<<<static_cast<unsigned>(tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      h, delta, weight, weight_dtype, hidden, eps, out, out_dtype, delta_weight);
  NQB_CUDA(cudaGetLastError(), "rmsnorm launch");
  return ok();
}

int nqb_embedding_bf16(const int64_t *ids, int64_t tokens, const void *weight, int64_t rows, int64_t dim, float scale,
                       float *out, void *stream) {
  if (ids == nullptr || weight == nullptr || out == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "embedding operand is NULL");
  if (tokens <= 0 || rows <= 0 || dim <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "embedding shape invalid");
  shell::embedding_bf16_kernel<<<static_cast<unsigned>(tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      ids, static_cast<const __nv_bfloat16 *>(weight), rows, dim, scale, out);
  NQB_CUDA(cudaGetLastError(), "embedding launch");
  return ok();
}

int nqb_qk_norm_rope(const float *q, const float *k, const float *v, const void *q_weight, const void *k_weight,
                     int32_t weight_dtype, const float *cos_table, const float *sin_table, int64_t tokens,
                     int32_t q_heads, int32_t kv_heads, int32_t head_dim, float eps, void *q_out, void *k_cache,
                     void *v_cache, int64_t cache_len, int64_t position, void *stream) {
  if (q == nullptr || k == nullptr || v == nullptr || cos_table == nullptr || sin_table == nullptr || q_out == nullptr ||
      k_cache == nullptr || v_cache == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "rope operand is NULL");
  if (tokens <= 0 || q_heads <= 0 || kv_heads <= 0 || position < 0 || position + tokens > cache_len)
    return fail(NQB_ERR_INVALID_ARGUMENT, "rope shape or cache position invalid");
  if ((q_weight != nullptr || k_weight != nullptr) && !is_float_dtype(weight_dtype))
    return fail(NQB_ERR_DTYPE, "rope norm weight dtype invalid");
  const int64_t warps = tokens * (q_heads + 2 * kv_heads);
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
  auto s = static_cast<cudaStream_t>(stream);
  auto *qo = static_cast<__nv_bfloat16 *>(q_out);
  auto *kc = static_cast<__nv_bfloat16 *>(k_cache);
  auto *vc = static_cast<__nv_bfloat16 *>(v_cache);
  switch (head_dim) {
    case 64:
      shell::qk_norm_rope_kernel<2><<<blocks, 256, 0, s>>>(q, k, v, q_weight, k_weight, weight_dtype, cos_table,
                                                            sin_table, tokens, q_heads, kv_heads, eps, qo, kc, vc,
                                                            cache_len, position);
      break;
    case 128:
      shell::qk_norm_rope_kernel<4><<<blocks, 256, 0, s>>>(q, k, v, q_weight, k_weight, weight_dtype, cos_table,
                                                            sin_table, tokens, q_heads, kv_heads, eps, qo, kc, vc,
                                                            cache_len, position);
      break;
    case 256:
      shell::qk_norm_rope_kernel<8><<<blocks, 256, 0, s>>>(q, k, v, q_weight, k_weight, weight_dtype, cos_table,
                                                            sin_table, tokens, q_heads, kv_heads, eps, qo, kc, vc,
                                                            cache_len, position);
      break;
    default:
      return fail(NQB_ERR_UNSUPPORTED, "head_dim %d is not 64, 128 or 256", head_dim);
  }
  NQB_CUDA(cudaGetLastError(), "rope launch");
  return ok();
}

int nqb_decode_attention_workspace_bytes(int64_t keys, int64_t tokens, int32_t q_heads, int32_t head_dim,
                                         size_t *bytes) {
  if (bytes == nullptr || keys <= 0 || tokens <= 0 || q_heads <= 0 || head_dim <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "attention workspace query is invalid");
  *bytes = static_cast<size_t>(tokens) * q_heads * shell::splits_for(keys, tokens) * (head_dim + shell::kPartPad) *
           sizeof(float);
  return ok();
}

int nqb_decode_attention(const void *q, const void *k_cache, const void *v_cache, int64_t cache_len, int64_t keys,
                         int64_t tokens, int32_t q_heads, int32_t kv_heads, int32_t head_dim, void *out,
                         void *workspace, size_t workspace_bytes, void *stream) {
  return nqb_decode_attention_window(q, k_cache, v_cache, cache_len, keys, tokens, q_heads, kv_heads, head_dim, 0, out,
                                     workspace, workspace_bytes, stream);
}

int nqb_decode_attention_window(const void *q, const void *k_cache, const void *v_cache, int64_t cache_len,
                                int64_t keys, int64_t tokens, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                                int64_t window, void *out, void *workspace, size_t workspace_bytes, void *stream) {
  if (window < 0) return fail(NQB_ERR_INVALID_ARGUMENT, "attention window must be >= 0");
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || workspace == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "attention operand is NULL");
  if (tokens <= 0 || keys <= 0 || keys + tokens - 1 > cache_len || kv_heads <= 0 || q_heads % kv_heads != 0 ||
      q_heads / kv_heads > 32)
    return fail(NQB_ERR_INVALID_ARGUMENT, "attention shape invalid (keys, cache length or head grouping)");
  // 16-byte cp.async of cache rows and vector loads of q and of the partials
  const uintptr_t q_align = static_cast<uintptr_t>(head_dim / 32) * 2;
  if (reinterpret_cast<uintptr_t>(k_cache) % 16 || reinterpret_cast<uintptr_t>(v_cache) % 16 ||
      reinterpret_cast<uintptr_t>(workspace) % 16 ||
      (q_align > 1 && (reinterpret_cast<uintptr_t>(q) % q_align || reinterpret_cast<uintptr_t>(out) % q_align)))
    return fail(NQB_ERR_ALIGNMENT, "attention caches and workspace need 16-byte alignment, q and out %zu-byte alignment",
                static_cast<size_t>(q_align));
  size_t need = 0;
  NQB_CHECK(nqb_decode_attention_workspace_bytes(keys, tokens, q_heads, head_dim, &need));
  if (workspace_bytes < need) return fail(NQB_ERR_WORKSPACE, "attention workspace too small");
  const int splits = shell::splits_for(keys, tokens);
  const int64_t chunk = (keys + tokens - 1 + splits - 1) / splits;
  const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
  const dim3 grid(static_cast<unsigned>(kv_heads), static_cast<unsigned>(splits), static_cast<unsigned>(tokens));
  const unsigned threads = static_cast<unsigned>(32 * (q_heads / kv_heads));
  const unsigned cblocks = static_cast<unsigned>((tokens * q_heads * 32 + 255) / 256);
  auto s = static_cast<cudaStream_t>(stream);
  auto *qp = static_cast<const __nv_bfloat16 *>(q);
  auto *kc = static_cast<const __nv_bfloat16 *>(k_cache);
  auto *vc = static_cast<const __nv_bfloat16 *>(v_cache);
  auto *part = static_cast<float *>(workspace);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  switch (head_dim) {
    case 64:
      NQB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(shell::attention_partial_kernel<2>),
                                    shell::attention_smem_bytes(64)));
      shell::attention_partial_kernel<2><<<grid, threads, shell::attention_smem_bytes(64), s>>>(
          qp, kc, vc, cache_len, keys, q_heads, kv_heads, splits, chunk, scale, part, window);
      shell::attention_combine_kernel<2><<<cblocks, 256, 0, s>>>(part, splits, tokens, q_heads, o);
      break;
    case 128:
      NQB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(shell::attention_partial_kernel<4>),
                                    shell::attention_smem_bytes(128)));
      shell::attention_partial_kernel<4><<<grid, threads, shell::attention_smem_bytes(128), s>>>(
          qp, kc, vc, cache_len, keys, q_heads, kv_heads, splits, chunk, scale, part, window);
      shell::attention_combine_kernel<4><<<cblocks, 256, 0, s>>>(part, splits, tokens, q_heads, o);
      break;
    case 256:
      NQB_CHECK(ensure_dynamic_smem(reinterpret_cast<const void *>(shell::attention_partial_kernel<8>),
                                    shell::attention_smem_bytes(256)));
      shell::attention_partial_kernel<8><<<grid, threads, shell::attention_smem_bytes(256), s>>>(
          qp, kc, vc, cache_len, keys, q_heads, kv_heads, splits, chunk, scale, part, window);
      shell::attention_combine_kernel<8><<<cblocks, 256, 0, s>>>(part, splits, tokens, q_heads, o);
      break;
    default:
      return fail(NQB_ERR_UNSUPPORTED, "head_dim %d is not 64, 128 or 256", head_dim);
  }
  NQB_CUDA(cudaGetLastError(), "attention launch");
  return ok();
}

int nqb_silu_mul(const float *gate, const float *up, int64_t count, void *out, int32_t out_dtype, void *stream) {
  if (gate == nullptr || up == nullptr || out == nullptr || count <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "silu_mul operand is NULL or empty");
  if (!is_float_dtype(out_dtype)) return fail(NQB_ERR_DTYPE, "silu_mul output dtype invalid");
  shell::silu_mul_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      gate, up, count, out, out_dtype);
  NQB_CUDA(cudaGetLastError(), "silu_mul launch");
  return ok();
}

int nqb_gemv_bf16(const void *weight, int64_t rows, int64_t cols, const void *x, int64_t tokens, float *out,
                  void *stream) {
  if (weight == nullptr || x == nullptr || out == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "gemv operand is NULL");
  if (rows <= 0 || cols <= 0 || tokens <= 0 || cols % 8 != 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "gemv needs positive sizes and a multiple of 8 columns");
  if (reinterpret_cast<uintptr_t>(weight) % 16 != 0) return fail(NQB_ERR_ALIGNMENT, "gemv weight is not 16-byte aligned");
  if (cols * 4 > 200 * 1024) return fail(NQB_ERR_UNSUPPORTED, "gemv rows longer than %d columns", 200 * 1024 / 4);
  auto s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(shell::launch_sm_count() * 8);
  auto *w = static_cast<const __nv_bfloat16 *>(weight);
  auto *xp = static_cast<const __nv_bfloat16 *>(x);
  // 2..16 tokens: tensor-core tiles of 8 tokens (16-byte aligned x, columns a multiple of 32)
  if (tokens >= 2 && cols % 32 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0) {
    for (int64_t t0 = 0; t0 < tokens; t0 += 16) {
      const int n = static_cast<int>(std::min<int64_t>(16, tokens - t0));
      const int tiles = n > 8 ? 2 : 1;
      const size_t smem = static_cast<size_t>(tiles) * 8 * (cols / 8 + 1) * 16;
      if (smem > 200 * 1024) break;  // too long a row for shared memory: the CUDA-core kernels below
      const void *fn = tiles == 2 ? reinterpret_cast<const void *>(shell::gemv_bf16_mma_kernel<2>)
                                  : reinterpret_cast<const void *>(shell::gemv_bf16_mma_kernel<1>);
      NQB_CHECK(ensure_dynamic_smem(fn, smem));
      const unsigned mma_grid = static_cast<unsigned>(shell::launch_sm_count() * (tiles == 2 ? 1 : 2));
      if (tiles == 2)
        shell::gemv_bf16_mma_kernel<2><<<mma_grid, 256, smem, s>>>(w, xp + t0 * cols, rows, cols, n, out + t0 * rows,
                                                                    rows);
      else
        shell::gemv_bf16_mma_kernel<1><<<mma_grid, 256, smem, s>>>(w, xp + t0 * cols, rows, cols, n, out + t0 * rows,
                                                                    rows);
      NQB_CUDA(cudaGetLastError(), "gemv launch");
      if (t0 + n == tokens) return ok();
    }
  }
  for (int64_t t0 = 0; t0 < tokens;) {
    const int64_t left = tokens - t0;
    const int group = left >= 8 && cols * 8 * 4 <= 200 * 1024   ? 8
                      : left >= 4 && cols * 4 * 4 <= 200 * 1024 ? 4
                      : left >= 2 && cols * 2 * 4 <= 200 * 1024 ? 2
                                                                 : 1;
    const size_t smem = static_cast<size_t>(group) * cols * sizeof(float);
    const void *fn = group == 8   ? reinterpret_cast<const void *>(shell::gemv_bf16_kernel<8>)
                     : group == 4 ? reinterpret_cast<const void *>(shell::gemv_bf16_kernel<4>)
                     : group == 2 ? reinterpret_cast<const void *>(shell::gemv_bf16_kernel<2>)
                                  : reinterpret_cast<const void *>(shell::gemv_bf16_kernel<1>);
    NQB_CHECK(ensure_dynamic_smem(fn, smem));
    const __nv_bfloat16 *xt = xp + t0 * cols;
    float *ot = out + t0 * rows;
    if (group == 8)
      shell::gemv_bf16_kernel<8><<<grid, 256, smem, s>>>(w, xt, rows, cols, cols, ot, rows);
    else if (group == 4)
      shell::gemv_bf16_kernel<4><<<grid, 256, smem, s>>>(w, xt, rows, cols, cols, ot, rows);
    else if (group == 2)
      shell::gemv_bf16_kernel<2><<<grid, 256, smem, s>>>(w, xt, rows, cols, cols, ot, rows);
    else
      shell::gemv_bf16_kernel<1><<<grid, 256, smem, s>>>(w, xt, rows, cols, cols, ot, rows);
    NQB_CUDA(cudaGetLastError(), "gemv launch");
    t0 += group;
  }
  return ok();
}

}  // extern "C"
