// Generic CUDA-core kernels of libnqb.
//
// These kernels accept every shape and dtype the ABI accepts (odd widths,
// tails, many salient columns, product-codebook V, grouped members) and are
// the path for shapes the tensor-core decode kernel does not take.  They follow
// the two-stage structure of the reference operation
// (src/nanoquant/runtime/cuda_kernels.py:65-162):
//
//   stage 1: latent[t,k] = mid[k] * sum_i sign(V[k,i]) * x[t,i] * pre[i]
//   stage 2: y[t,o]      = post[o] * sum_k sign(U[o,k]) * latent[t,k]
//                          + salient + overlay + bias
//
// Mapping: one warp per output row of the stage.  The warp loads 32 sign
// words of its row with one coalesced load, then walks them; for each word
// every lane owns one bit (column), so activation reads from shared memory
// are conflict-free.  Each warp keeps one accumulator per token of the
// block's token tile.  Sums use a fixed order, so results are deterministic.
#include "nqb_generic.cuh"

namespace nqb {

__device__ __forceinline__ uint32_t fetch_v_word(const Stage1Member &m, int64_t row, int64_t w,
                                                 int64_t wpr) {
  if (m.words != nullptr) return __ldg(m.words + row * wpr + w);
  // product-codebook right factor (reference product_codebook.py:110-143):
  // rows below free_rows are plain words; later rows hold one 16-bit record
  // per word, low byte -> first table (bits 0..15), high byte -> second.
  if (row < m.cb_free_rows) return __ldg(m.cb_free + row * wpr + w);
  const int64_t record_index = (row - m.cb_free_rows) * wpr + w;
  const uint32_t record = m.cb_payload[record_index];
  const uint32_t low = m.cb_first[record & 0xFFu];
  const uint32_t high = m.cb_second[record >> 8];
  return low | (high << 16);
}

__global__ void __launch_bounds__(kGenericThreads)
    stage1_generic_kernel(const Stage1Params p) {
  extern __shared__ float su[];  // [tok_tile][in_features] = x * pre
  int g = 0;
  for (int i = 1; i < p.count; ++i)
    if (static_cast<int32_t>(blockIdx.x) >= p.m[i].block_begin) g = i;
  const Stage1Member &m = p.m[g];
  const int64_t n = p.in_features;
  const int64_t t0 = static_cast<int64_t>(blockIdx.y) * p.tok_tile;
  const int tt = static_cast<int>(min(static_cast<int64_t>(p.tok_tile), p.tokens - t0));
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(tt) * n; i += blockDim.x) {
    const int64_t t = i / n;
    const int64_t c = i - t * n;
    su[i] = load_as_float(p.x, (t0 + t) * n + c, p.x_dtype) * load_as_float(m.pre, c, p.scale_dtype);
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x - m.block_begin) * kGenericWarps + warp;
  if (row >= m.rank) return;  // warp-uniform

  float acc[kMaxTokTile];
#pragma unroll
  for (int t = 0; t < kMaxTokTile; ++t) acc[t] = 0.0f;

  for (int64_t w0 = 0; w0 < p.wpr; w0 += 32) {
    const uint32_t mine = (w0 + lane < p.wpr) ? fetch_v_word(m, row, w0 + lane, p.wpr) : 0u;
    const int words_here = static_cast<int>(min(static_cast<int64_t>(32), p.wpr - w0));
    for (int k = 0; k < words_here; ++k) {
      const uint32_t word = __shfl_sync(0xffffffffu, mine, k);
      const int64_t c = (w0 + k) * 32 + lane;
      if (c < n) {
        const uint32_t neg = (word >> lane) & 1u;
#pragma unroll
        for (int t = 0; t < kMaxTokTile; ++t)
          if (t < tt) acc[t] += apply_sign(su[t * n + c], neg);
      }
    }
  }
  const float mid = load_as_float(m.mid, row, p.scale_dtype);
#pragma unroll
  for (int t = 0; t < kMaxTokTile; ++t) {
    const float s = warp_sum(acc[t]);
    if (lane == 0 && t < tt) p.latent[(t0 + t) * p.total_rank + m.latent_offset + row] = s * mid;
  }
}

// Index of `row` in the strictly increasing overlay row list, or -1.
__device__ __forceinline__ int64_t find_overlay(const int32_t *ids, int64_t count, int64_t row) {
  int64_t lo = 0, hi = count;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    const int32_t v = ids[mid];
    if (v == row) return mid;
    if (v < row) lo = mid + 1; else hi = mid;
  }
  return -1;
}

__global__ void __launch_bounds__(kGenericThreads)
    stage2_generic_kernel(const Stage2Params p) {
  extern __shared__ float sl[];  // [tok_tile][member rank] = latent slice
  int g = 0;
  for (int i = 1; i < p.count; ++i)
    if (static_cast<int32_t>(blockIdx.x) >= p.m[i].block_begin) g = i;
  const Stage2Member &m = p.m[g];
  const int64_t r = m.rank;
  const int64_t n = p.in_features;
  const int64_t t0 = static_cast<int64_t>(blockIdx.y) * p.tok_tile;
  const int tt = static_cast<int>(min(static_cast<int64_t>(p.tok_tile), p.tokens - t0));
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(tt) * r; i += blockDim.x) {
    const int64_t t = i / r;
    const int64_t k = i - t * r;
    sl[i] = p.latent[(t0 + t) * p.total_rank + m.latent_offset + k];
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x - m.block_begin) * kGenericWarps + warp;
  if (row >= m.out_features) return;  // warp-uniform

  float acc[kMaxTokTile];
#pragma unroll
  for (int t = 0; t < kMaxTokTile; ++t) acc[t] = 0.0f;
  for (int64_t w0 = 0; w0 < m.wpr; w0 += 32) {
    const uint32_t mine = (w0 + lane < m.wpr) ? __ldg(m.words + row * m.wpr + w0 + lane) : 0u;
    const int words_here = static_cast<int>(min(static_cast<int64_t>(32), m.wpr - w0));
    for (int k = 0; k < words_here; ++k) {
      const uint32_t word = __shfl_sync(0xffffffffu, mine, k);
      const int64_t c = (w0 + k) * 32 + lane;
      if (c < r) {
        const uint32_t neg = (word >> lane) & 1u;
#pragma unroll
        for (int t = 0; t < kMaxTokTile; ++t)
          if (t < tt) acc[t] += apply_sign(sl[t * r + c], neg);
      }
    }
  }

  // salient columns (reference cuda_kernels.py:140-156)
  float sal[kMaxTokTile];
#pragma unroll
  for (int t = 0; t < kMaxTokTile; ++t) sal[t] = 0.0f;
  for (int64_t s = lane; s < m.outlier_count; s += 32) {
    float w = load_as_float(m.outlier_values, row * m.outlier_count + s, m.outlier_value_dtype);
    if (m.outlier_scales != nullptr) w *= load_as_float(m.outlier_scales, s, p.scale_dtype);
    const int64_t column = m.outlier_indices[s];
#pragma unroll
    for (int t = 0; t < kMaxTokTile; ++t)
      if (t < tt) sal[t] += load_as_float(p.x, (t0 + t) * n + column, p.x_dtype) * w;
  }

  // int8 residual row overlay
  float ovl[kMaxTokTile];
#pragma unroll
  for (int t = 0; t < kMaxTokTile; ++t) ovl[t] = 0.0f;
  float ovl_scale = 0.0f;
  const int64_t j = m.overlay_rows > 0 ? find_overlay(m.overlay_row_ids, m.overlay_rows, row) : -1;
  if (j >= 0) {
    ovl_scale = load_as_float(m.overlay_scales, j, m.overlay_scale_dtype);
    const int8_t *rvals = m.overlay_values + j * n;
    for (int64_t i = lane; i < n; i += 32) {
      const float rv = static_cast<float>(rvals[i]);
#pragma unroll
      for (int t = 0; t < kMaxTokTile; ++t)
        if (t < tt) ovl[t] += rv * load_as_float(p.x, (t0 + t) * n + i, p.x_dtype);
    }
  }

  const float post = load_as_float(m.post, row, p.scale_dtype);
  const float bias = m.bias != nullptr ? load_as_float(m.bias, row, m.bias_dtype) : 0.0f;
#pragma unroll
  for (int t = 0; t < kMaxTokTile; ++t) {
    float v = warp_sum(acc[t]) * post;
    if (m.outlier_count > 0) v += warp_sum(sal[t]);
    if (j >= 0) v += warp_sum(ovl[t]) * ovl_scale;
    v += bias;
    if (lane == 0 && t < tt) m.y[(t0 + t) * m.out_features + row] = v;
  }
}

// ------------------------------------------------------------ patch ---

__global__ void patch_latent_kernel(const void *x, int32_t x_dtype, int64_t tokens, int64_t n,
                                    int64_t pr, const void *right, int32_t dt, float *latent) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (item >= tokens * pr) return;
  const int64_t t = item / pr, q = item - t * pr;
  float acc = 0.0f;
  for (int64_t i = lane; i < n; i += 32)
    acc += load_as_float(x, t * n + i, x_dtype) * load_as_float(right, q * n + i, dt);
  acc = warp_sum(acc);
  if (lane == 0) latent[t * pr + q] = acc;
}

__global__ void patch_output_kernel(const float *latent, int64_t tokens, int64_t m, int64_t pr,
                                    const void *left, int32_t dt, float *y) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= tokens * m) return;
  const int64_t t = i / m, o = i - t * m;
  float acc = 0.0f;
  for (int64_t q = 0; q < pr; ++q) acc += load_as_float(left, o * pr + q, dt) * latent[t * pr + q];
  y[i] += acc;
}

// ------------------------------------------------------ layout v1 tools ---

__global__ void pack_signs_kernel(const void *signs, int32_t dt, int64_t rows, int64_t cols,
                                  int64_t wpr, uint32_t *words) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * wpr) return;
  const int64_t row = i / wpr, w = i - row * wpr;
  uint32_t out = 0;
  for (int b = 0; b < 32; ++b) {
    const int64_t c = w * 32 + b;
    if (c < cols && load_as_float(signs, row * cols + c, dt) < 0.0f) out |= 1u << b;
  }
  words[i] = out;
}

__global__ void unpack_signs_kernel(const uint32_t *words, int64_t rows, int64_t cols, int64_t wpr,
                                    float *signs, int32_t *bad_rows) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < rows * cols) {
    const int64_t row = i / cols, c = i - row * cols;
    const uint32_t bit = (__ldg(words + row * wpr + (c >> 5)) >> (c & 31)) & 1u;
    signs[i] = bit ? -1.0f : 1.0f;
  }
  if (bad_rows != nullptr && i < rows) {
    const int tail = static_cast<int>(cols & 31);
    if (tail != 0) {
      const uint32_t padding = ~((1u << tail) - 1u);
      if (__ldg(words + i * wpr + wpr - 1) & padding) atomicAdd(bad_rows, 1);
    }
  }
}

__global__ void decode_codebook_kernel(const uint32_t *free_words, int64_t free_rows, int64_t rank,
                                       int64_t wpr, const uint16_t *payload, const uint16_t *first,
                                       const uint16_t *second, uint32_t *out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rank * wpr) return;
  const int64_t row = i / wpr;
  if (row < free_rows) {
    out[i] = free_words[i];
    return;
  }
  const uint32_t record = payload[i - free_rows * wpr];
  out[i] = static_cast<uint32_t>(first[record & 0xFFu]) |
           (static_cast<uint32_t>(second[record >> 8]) << 16);
}

// Mixed-V right factor: the first free_rows rows are plain words; every
// word of the remaining rows is one 19-bit record (bits 0..9: index into
// the 1024-word codebook, bits 10..18: id of the bit pair to flip), records
// packed LSB-first across consecutive uint32 words.  Pair ids enumerate
// (a, b), a < b < 32, in lexicographic order.  Shifts and the codebook index
// are masked, so any payload stays in bounds; ids 496..511 are rejected by
// the host before a launch.
__device__ __forceinline__ uint32_t pair_mask(uint32_t id) {
  uint32_t a = 0;
  while (a < 30 && id >= 31 - a) {  // pairs (a, a+1 .. 31): 31 - a of them
    id -= 31 - a;
    ++a;
  }
  const uint32_t b = a + 1 + id;
  return (1u << a) | (1u << (b & 31u));
}

__global__ void decode_mixed_v_kernel(const uint32_t *free_words, int64_t free_rows, int64_t rank, int64_t wpr,
                                      const uint32_t *payload, const uint32_t *codebook, uint32_t *out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rank * wpr) return;
  if (i < free_rows * wpr) {
    out[i] = free_words[i];
    return;
  }
  const int64_t bit = (i - free_rows * wpr) * kMixedRecordBits;
  const int64_t word = bit >> 5;
  const uint32_t shift = static_cast<uint32_t>(bit & 31);
  uint32_t record = payload[word] >> shift;
  if (shift > 32 - kMixedRecordBits) record |= payload[word + 1] << (32 - shift);
  record &= (1u << kMixedRecordBits) - 1;
  out[i] = codebook[record & 1023u] ^ pair_mask(record >> 10);
}

// Coded tiles of a mixed-V right factor (nqb_repack_mixed_v): one thread per
// (coded tile, slice, row) writes the row's 20-byte block of 8 tile records
// (index | a << 10 | b << 15: the pair id resolved, so the decode needs no
// pair table).
__global__ void repack_mixed_v_kernel(const uint32_t *payload, int64_t rank, int64_t wpr, int64_t free_rows,
                                      int64_t first_tile, int64_t coded_tiles, int32_t slices, uint8_t *out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= coded_tiles * slices * kMixedTileRows) return;
  const int64_t row_in_tile = i % kMixedTileRows;
  const int64_t ts = i / kMixedTileRows;  // coded tile * slices + slice
  const int64_t slice = ts % slices;
  const int64_t row = (first_tile + ts / slices) * kMixedTileRows + row_in_tile;
  uint8_t *dst = out + ts * kMixedSliceBytes + row_in_tile * (8 * kMixedTileRecordBits / 8);
  uint64_t acc = 0;
  int bits = 0;
  for (int j = 0; j < 8; ++j) {
    const int64_t w = slice * 8 + j;
    uint32_t tile_record = 0;
    if (row < rank && w < wpr) {
      const int64_t bit = ((row - free_rows) * wpr + w) * kMixedRecordBits;
      const uint32_t shift = static_cast<uint32_t>(bit & 31);
      uint32_t record = payload[bit >> 5] >> shift;
      if (shift > 32 - kMixedRecordBits) record |= payload[(bit >> 5) + 1] << (32 - shift);
      record &= (1u << kMixedRecordBits) - 1;
      uint32_t id = record >> 10, a = 0;
      while (a < 30 && id >= 31 - a) {  // pair id -> (a, b), as pair_mask
        id -= 31 - a;
        ++a;
      }
      const uint32_t b = (a + 1 + id) & 31u;
      tile_record = (record & 1023u) | (a << 10) | (b << 15);
    }
    acc |= static_cast<uint64_t>(tile_record) << bits;
    bits += kMixedTileRecordBits;
    while (bits >= 8) {
      *dst++ = static_cast<uint8_t>(acc & 0xFFu);
      acc >>= 8;
      bits -= 8;
    }
  }
}

// Coded tiles of a product-codebook right factor (nqb_repack_product_codebook):
// one thread per (coded tile, slice, row) writes the row's 16-byte block of 8
// records, zero past the row and past the rank; threads past the tiles write
// the 1024-word decode table (first half words, second half words << 16).
__global__ void repack_product_codebook_kernel(const uint16_t *payload, const uint16_t *first,
                                               const uint16_t *second, int64_t rank, int64_t wpr,
                                               int64_t free_rows, int64_t first_tile, int64_t coded_tiles,
                                               int32_t slices, uint8_t *out, uint32_t *table) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t items = coded_tiles * slices * kMixedTileRows;
  if (i >= items) {
    const int64_t e = i - items;
    if (e < 1024)
      table[e] = e < 256 ? static_cast<uint32_t>(first[e])
                         : (e < 512 ? static_cast<uint32_t>(second[e - 256]) << 16 : 0u);
    return;
  }
  const int64_t row_in_tile = i % kMixedTileRows;
  const int64_t ts = i / kMixedTileRows;  // coded tile * slices + slice
  const int64_t slice = ts % slices;
  const int64_t row = (first_tile + ts / slices) * kMixedTileRows + row_in_tile;
  uint32_t half[4] = {0u, 0u, 0u, 0u};
  if (row < rank) {
    const uint16_t *src = payload + (row - free_rows) * wpr;
    for (int j = 0; j < 8; ++j) {
      const int64_t w = slice * 8 + j;
      if (w < wpr) half[j >> 1] |= static_cast<uint32_t>(src[w]) << (16 * (j & 1));
    }
  }
  *reinterpret_cast<uint4 *>(out + ts * kCodebookTileSliceBytes + row_in_tile * 16) =
      make_uint4(half[0], half[1], half[2], half[3]);
}

// --------------------------------------------------------------- launch ---

static int set_smem(const void *fn, size_t bytes) { return ensure_dynamic_smem(fn, bytes); }

int choose_tok_tile(int64_t tokens, int64_t width) {
  // keep the staged activations under ~96 KB so two blocks fit per SM
  int64_t tile = (96 * 1024) / (4 * (width > 0 ? width : 1));
  if (tile > kMaxTokTile) tile = kMaxTokTile;
  if (tile < 1) tile = 1;
  if (tile > tokens) tile = tokens;
  return static_cast<int>(tile);
}

int launch_stage1_generic(Stage1Params &p, int32_t total_blocks, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(p.tok_tile) * p.in_features * sizeof(float);
  NQB_CHECK(set_smem(reinterpret_cast<const void *>(stage1_generic_kernel), smem));
  const dim3 grid(total_blocks, static_cast<unsigned>((p.tokens + p.tok_tile - 1) / p.tok_tile));
  stage1_generic_kernel<<<grid, kGenericThreads, smem, stream>>>(p);
  NQB_CUDA(cudaGetLastError(), "stage1_generic_kernel launch");
  return NQB_OK;
}

int launch_stage2_generic(Stage2Params &p, int32_t total_blocks, int64_t max_rank, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(p.tok_tile) * max_rank * sizeof(float);
  NQB_CHECK(set_smem(reinterpret_cast<const void *>(stage2_generic_kernel), smem));
  const dim3 grid(total_blocks, static_cast<unsigned>((p.tokens + p.tok_tile - 1) / p.tok_tile));
  stage2_generic_kernel<<<grid, kGenericThreads, smem, stream>>>(p);
  NQB_CUDA(cudaGetLastError(), "stage2_generic_kernel launch");
  return NQB_OK;
}

int launch_patch(const void *x, int32_t x_dtype, int64_t tokens, int64_t n, int64_t m, int64_t pr,
                 const void *left, const void *right, int32_t dt, float *y, float *latent,
                 cudaStream_t stream) {
  const int64_t items = tokens * pr;
  patch_latent_kernel<<<static_cast<unsigned>((items + 7) / 8), 256, 0, stream>>>(x, x_dtype, tokens, n, pr,
                                                                                  right, dt, latent);
  NQB_CUDA(cudaGetLastError(), "patch_latent_kernel launch");
  const int64_t outs = tokens * m;
  patch_output_kernel<<<static_cast<unsigned>((outs + 255) / 256), 256, 0, stream>>>(latent, tokens, m, pr,
                                                                                     left, dt, y);
  NQB_CUDA(cudaGetLastError(), "patch_output_kernel launch");
  return NQB_OK;
}

int launch_pack(const void *signs, int32_t dt, int64_t rows, int64_t cols, uint32_t *words,
                cudaStream_t stream) {
  const int64_t wpr = words_for(cols);
  const int64_t items = rows * wpr;
  pack_signs_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(signs, dt, rows, cols, wpr,
                                                                                    words);
  NQB_CUDA(cudaGetLastError(), "pack_signs_kernel launch");
  return NQB_OK;
}

int launch_unpack(const uint32_t *words, int64_t rows, int64_t cols, float *signs, int32_t *bad_rows,
                  cudaStream_t stream) {
  const int64_t wpr = words_for(cols);
  const int64_t items = rows * cols > rows ? rows * cols : rows;
  unpack_signs_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(words, rows, cols, wpr,
                                                                                      signs, bad_rows);
  NQB_CUDA(cudaGetLastError(), "unpack_signs_kernel launch");
  return NQB_OK;
}

int launch_decode_mixed_v(const uint32_t *free_words, int64_t free_rows, int64_t rank, int64_t cols,
                          const uint32_t *payload, const uint32_t *codebook, uint32_t *out, cudaStream_t stream) {
  const int64_t items = rank * ((cols + 31) / 32);
  decode_mixed_v_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(
      free_words, free_rows, rank, (cols + 31) / 32, payload, codebook, out);
  NQB_CUDA(cudaGetLastError(), "decode_mixed_v_kernel launch");
  return NQB_OK;
}

int64_t mixed_v_first_coded_tile(int64_t free_rows) { return (free_rows + kMixedTileRows - 1) / kMixedTileRows; }

size_t mixed_v_tiles_bytes(int64_t rank, int64_t columns, int64_t free_rows) {
  const int64_t tiles = (rank + kMixedTileRows - 1) / kMixedTileRows - mixed_v_first_coded_tile(free_rows);
  const int64_t slices = (words_for(columns) + 7) / 8;
  return tiles > 0 ? static_cast<size_t>(tiles * slices) * kMixedSliceBytes : 0;
}

int launch_repack_mixed_v(const uint32_t *payload, int64_t rank, int64_t columns, int64_t free_rows, uint8_t *out,
                          cudaStream_t stream) {
  const int64_t first = mixed_v_first_coded_tile(free_rows);
  const int64_t tiles = (rank + kMixedTileRows - 1) / kMixedTileRows - first;
  if (tiles <= 0) return NQB_OK;
  const int64_t wpr = words_for(columns);
  const int32_t slices = static_cast<int32_t>((wpr + 7) / 8);
  const int64_t items = tiles * slices * kMixedTileRows;
  repack_mixed_v_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(
      payload, rank, wpr, free_rows, first, tiles, slices, out);
  NQB_CUDA(cudaGetLastError(), "repack_mixed_v_kernel launch");
  return NQB_OK;
}

size_t product_codebook_tiles_bytes(int64_t rank, int64_t columns, int64_t free_rows) {
  const int64_t tiles = (rank + kMixedTileRows - 1) / kMixedTileRows - mixed_v_first_coded_tile(free_rows);
  const int64_t slices = (words_for(columns) + 7) / 8;
  return tiles > 0 ? static_cast<size_t>(tiles * slices) * kCodebookTileSliceBytes : 0;
}

int launch_repack_product_codebook(const uint16_t *payload, const uint16_t *first, const uint16_t *second,
                                   int64_t rank, int64_t columns, int64_t free_rows, uint8_t *tiles,
                                   uint32_t *table, cudaStream_t stream) {
  const int64_t first_tile = mixed_v_first_coded_tile(free_rows);
  const int64_t tile_count = (rank + kMixedTileRows - 1) / kMixedTileRows - first_tile;
  const int64_t coded = tile_count > 0 ? tile_count : 0;
  const int64_t wpr = words_for(columns);
  const int32_t slices = static_cast<int32_t>((wpr + 7) / 8);
  const int64_t items = coded * slices * kMixedTileRows + 1024;
  repack_product_codebook_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(
      payload, first, second, rank, wpr, free_rows, first_tile, coded, slices, tiles, table);
  NQB_CUDA(cudaGetLastError(), "repack_product_codebook_kernel launch");
  return NQB_OK;
}

int launch_decode_codebook(const uint32_t *free_words, int64_t free_rows, int64_t rank, int64_t cols,
                           const uint16_t *payload, const uint16_t *first, const uint16_t *second,
                           uint32_t *out, cudaStream_t stream) {
  const int64_t wpr = words_for(cols);
  const int64_t items = rank * wpr;
  decode_codebook_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, stream>>>(
      free_words, free_rows, rank, wpr, payload, first, second, out);
  NQB_CUDA(cudaGetLastError(), "decode_codebook_kernel launch");
  return NQB_OK;
}

}  // namespace nqb
