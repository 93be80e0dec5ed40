// Internal declarations of the generic CUDA-core path of libnqb.
#pragma once

#include "nqb_common.cuh"

namespace nqb {

constexpr int kMaxMembers = 3;    // grouped projections: QKV or gate/up
constexpr int kGenericWarps = 8;  // output rows per block (one warp per row)
constexpr int kGenericThreads = 32 * kGenericWarps;
constexpr int kMaxTokTile = 8;    // tokens accumulated per warp

struct Stage1Member {
  const uint32_t *words;  // V [rank, wpr], or nullptr for a product-codebook V
  const uint32_t *cb_free;
  const uint16_t *cb_payload;
  const uint16_t *cb_first;
  const uint16_t *cb_second;
  int64_t cb_free_rows;
  const void *pre;
  const void *mid;
  int64_t rank;
  int64_t latent_offset;  // column of this member in the [tokens, total_rank] latent
  int32_t block_begin;    // first blockIdx.x owned by this member
};

struct Stage1Params {
  Stage1Member m[kMaxMembers];
  int32_t count;
  const void *x;
  int32_t x_dtype;
  int32_t scale_dtype;
  int64_t in_features;
  int64_t wpr;  // words per V row
  int64_t tokens;
  int64_t total_rank;
  float *latent;
  int32_t tok_tile;
};

struct Stage2Member {
  const uint32_t *words;  // U [out, wpr]
  int64_t out_features;
  int64_t rank;
  int64_t wpr;
  int64_t latent_offset;
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
  float *y;  // [tokens, out_features]
  int32_t block_begin;
};

struct Stage2Params {
  Stage2Member m[kMaxMembers];
  int32_t count;
  const void *x;
  int32_t x_dtype;
  int32_t scale_dtype;
  int64_t in_features;
  int64_t tokens;
  int64_t total_rank;
  const float *latent;
  int32_t tok_tile;
};

int choose_tok_tile(int64_t tokens, int64_t width);
int launch_stage1_generic(Stage1Params &p, int32_t total_blocks, cudaStream_t stream);
int launch_stage2_generic(Stage2Params &p, int32_t total_blocks, int64_t max_rank, cudaStream_t stream);
int launch_patch(const void *x, int32_t x_dtype, int64_t tokens, int64_t n, int64_t m, int64_t pr,
                 const void *left, const void *right, int32_t dt, float *y, float *latent,
                 cudaStream_t stream);
int launch_pack(const void *signs, int32_t dt, int64_t rows, int64_t cols, uint32_t *words,
                cudaStream_t stream);
int launch_unpack(const uint32_t *words, int64_t rows, int64_t cols, float *signs, int32_t *bad_rows,
                  cudaStream_t stream);
constexpr int kMixedRecordBits = 19;  // 10-bit codebook index + 9-bit pair id
// Coded mixed-V tiles (nqb_repack_mixed_v): 128-row tiles, per 256-column
// slice 8 tile records per row, each 20 bits (codebook index, then the two
// flipped bit positions a and b, 5 bits each), row r's from bit 160 r.
constexpr int kMixedTileRows = 128;
constexpr int kMixedTileRecordBits = 20;
constexpr int kMixedSliceBytes = kMixedTileRows * 8 * kMixedTileRecordBits / 8;  // 2560
int64_t mixed_v_first_coded_tile(int64_t free_rows);
size_t mixed_v_tiles_bytes(int64_t rank, int64_t columns, int64_t free_rows);
int launch_repack_mixed_v(const uint32_t *payload, int64_t rank, int64_t columns, int64_t free_rows, uint8_t *out,
                          cudaStream_t stream);
// Coded product-codebook tiles (nqb_repack_product_codebook): 128-row tiles,
// per 256-column slice 8 16-bit records per row, row r's at byte 16 r.
constexpr int kCodebookTileSliceBytes = kMixedTileRows * 8 * 2;  // 2048
size_t product_codebook_tiles_bytes(int64_t rank, int64_t columns, int64_t free_rows);
int launch_repack_product_codebook(const uint16_t *payload, const uint16_t *first, const uint16_t *second,
                                   int64_t rank, int64_t columns, int64_t free_rows, uint8_t *tiles,
                                   uint32_t *table, cudaStream_t stream);
int launch_decode_mixed_v(const uint32_t *free_words, int64_t free_rows, int64_t rank, int64_t cols,
                          const uint32_t *payload, const uint32_t *codebook, uint32_t *out, cudaStream_t stream);
int launch_decode_codebook(const uint32_t *free_words, int64_t free_rows, int64_t rank, int64_t cols,
                           const uint16_t *payload, const uint16_t *first, const uint16_t *second,
                           uint32_t *out, cudaStream_t stream);

}  // namespace nqb
