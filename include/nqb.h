/*
 * nqb.h - C ABI of libnqb, the B200 (sm_100a) packed binary low-rank linear.
 *
 * One layer computes, per token t and output row o,
 *
 *   latent[t,k] = mid[k]  * sum_i sign(V[k,i]) * x[t,i] * pre[i]
 *   y[t,o]      = post[o] * sum_k sign(U[o,k]) * latent[t,k]
 *               + sum_s x[t,idx[s]] * w[o,s] (* wscale[s] for int8 w)
 *               + bias[o]
 *               + rscale[j] * sum_i R[j,i] * x[t,i]      (for o == row_ids[j])
 *
 * with U [out x rank] and V [rank x in] stored in NanoQuant packed layout v1:
 * int32 words, column c in word c/32 at bit c%32 (LSB first), bit 1 = -1,
 * zero tail padding.  All pointers are device pointers unless stated
 * otherwise; every call is asynchronous on the given stream (a cudaStream_t
 * passed as void*, NULL = legacy default stream).  No entry point allocates
 * device memory or synchronises the host, except the program set-up calls
 * (nqb_program_create / _destroy) and the diagnostics readers
 * (nqb_device_status, nqb_program_trace).
 *
 * Every function returns NQB_OK (0) or one of the NQB_ERR_* codes below and
 * never traps; nqb_last_error() returns a message for the calling thread.
 */
#ifndef NQB_H
#define NQB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NQB_ABI_VERSION 5

/* status codes */
#define NQB_OK 0
#define NQB_ERR_INVALID_ARGUMENT 1 /* bad shape, null pointer, inconsistent descriptor */
#define NQB_ERR_ALIGNMENT 2        /* pointer alignment below what the layout needs   */
#define NQB_ERR_DTYPE 3            /* dtype code not accepted for this operand         */
#define NQB_ERR_CUDA 4             /* a CUDA runtime call failed                       */
#define NQB_ERR_WORKSPACE 5        /* workspace missing or smaller than required       */
#define NQB_ERR_UNSUPPORTED 6      /* valid request this build does not implement      */
#define NQB_ERR_TIMEOUT 7          /* a bounded device-side wait gave up               */

/* dtype codes */
#define NQB_F32 0
#define NQB_F16 1
#define NQB_BF16 2
#define NQB_I8 3
#define NQB_I32 4

/*
 * One packed linear, described by plain device pointers.  Optional operands
 * are NULL (and their counts 0).  The layer descriptor is read on the host at
 * call time only; it may live on the stack.
 *
 * Mirrors the operands of launch_packed_linear
 * (src/nanoquant/runtime/cuda_kernels.py:816-874 in the reference) plus two
 * additions the reference runtime has no type for: the int8 residual-row
 * overlay and the product-codebook right factor.
 */
typedef struct nqb_linear_desc {
  int64_t in_features;  /* n */
  int64_t out_features; /* m */
  int64_t rank;         /* r */

  const int32_t *left_words;  /* U, [m, ceil(r/32)] layout v1                */
  const int32_t *right_words; /* V, [r, ceil(n/32)] layout v1; NULL when the
                                 product-codebook fields below are used.
                                 A tiles-only layer sets both word pointers
                                 and codebook_payload NULL and gives both tile
                                 copies below: it runs on the tensor-core
                                 decode, prefill and program paths, and a call
                                 that would take the generic path returns
                                 NQB_ERR_UNSUPPORTED                          */

  const void *scale_pre;  /* [n] */
  const void *scale_mid;  /* [r] */
  const void *scale_post; /* [m] */
  int32_t scale_dtype;    /* F32 / F16 / BF16 */

  const void *bias; /* [m] or NULL */
  int32_t bias_dtype;

  /* salient (outlier) input columns, reference packed.py:230-352 */
  int64_t outlier_count;          /* k */
  const int32_t *outlier_indices; /* [k], strictly increasing, pre[idx]==0 */
  const void *outlier_values;     /* [m, k] */
  int32_t outlier_value_dtype;    /* F32 / F16 / BF16 / I8 */
  const void *outlier_scales;     /* [k] in scale_dtype, only for I8 values */

  /* int8 residual output rows (row form of the outlier overlay) */
  int64_t overlay_rows;          /* R */
  const int32_t *overlay_row_ids; /* [R], strictly increasing, < m          */
  const int8_t *overlay_values;  /* [R, n]                                  */
  const void *overlay_scales;    /* [R] in overlay_scale_dtype              */
  int32_t overlay_scale_dtype;

  /* product-codebook right factor (product-codebook-free-k16-v1, canonical
   * orientation): rows < free_rows are plain words, the rest one 16-bit record
   * per word indexing two 256-entry half-word tables.                        */
  int64_t codebook_free_rows;
  const int32_t *codebook_free_words; /* [free_rows, ceil(n/32)]            */
  const int32_t *codebook_payload;    /* 16-bit records, two per word       */
  const int16_t *codebook_first;      /* [256] bits 0..15 of a coded word   */
  const int16_t *codebook_second;     /* [256] bits 16..31 of a coded word  */

  /* Optional kernel-native copies of U and V made by nqb_repack_signs
   * (16-byte aligned).  When both are present, 1..16 tokens run on the
   * tensor-core decode path (exact integer products of 22-bit fixed-point
   * activations) and more tokens on the tensor-core prefill path (fp16
   * activations, fp32 accumulation); without them every call runs on the
   * generic CUDA-core path (fp32).                                          */
  const void *left_tiles;  /* nqb_repack_signs(left_words,  m, r) */
  const void *right_tiles; /* nqb_repack_signs(right_words, r, n) */

  /* Dense low-rank patch, y += L (R x) (reference cuda_backend.py:275-277,
   * reference.py:224-232).  nqb_linear applies it itself: on the tensor-core
   * decode path and in programs fused into the two stages (stage 1 also forms
   * the patch latent R x, stage 2's epilogue adds L times it); on the other
   * paths as two small kernels after stage 2.  patch_rank 0 = no patch.     */
  int64_t patch_rank;      /* p */
  const void *patch_left;  /* [m, p] in patch_dtype */
  const void *patch_right; /* [p, n] in patch_dtype */
  int32_t patch_dtype;     /* F32 / F16 / BF16 */

  /* Right factor kept coded for decode programs (optional; NULL
   * coded_right_tiles = none).  Programs stream the coded tiles of V and
   * decode their records in stage 1; the 128-row tiles below
   * ceil(coded_free_rows / 128) * 128 still come from right_tiles, which the
   * per-call paths keep using for every row.  coded_format says which
   * records the tiles hold:
   *   NQB_CODED_MIXED_V          nqb_repack_mixed_v tiles, coded_codebook the
   *                              layer's 1024 full sign words;
   *   NQB_CODED_PRODUCT_CODEBOOK nqb_repack_product_codebook tiles and table. */
  const void *coded_right_tiles;
  const int32_t *coded_codebook;  /* [1024] words, 16-byte aligned                 */
  int64_t coded_free_rows;        /* the layer's plain (free) rows                 */
  int32_t coded_format;           /* NQB_CODED_*                                   */
} nqb_linear_desc;

#define NQB_CODED_MIXED_V 0
#define NQB_CODED_PRODUCT_CODEBOOK 1

/*
 * Coded tiles of a mixed-V right factor (mixed-v-free-k10-pair9-v1: rows
 * below free_rows plain, every later word one 19-bit record, packed back to
 * back from bit 0 of `payload`).  The tiles of 128 rows from
 * ceil(free_rows / 128) on keep one record per word, widened to 20 bits with
 * the pair id resolved (codebook index | a << 10 | b << 15, a < b the two
 * flipped bits): per tile and per 256-column slice, row r's 8 records (words
 * 8s .. 8s+7, zero past the row) sit back to back from bit 160 r, so one
 * tile slice is 2560 bytes against 4096 for sign words.  No counterpart in the reference, whose backend expands the
 * records before its kernels run (cuda_backend.py:209-224); this layout feeds
 * the decode programs' stage-1 record decode.
 */
int nqb_mixed_v_tiles_bytes(int64_t rank, int64_t in_features, int64_t free_rows, size_t *bytes);
int nqb_repack_mixed_v(const int32_t *payload, int64_t rank, int64_t in_features, int64_t free_rows,
                       void *out, void *stream);

/*
 * Coded tiles of a product-codebook right factor (product-codebook-free-k16-v1,
 * canonical orientation: rows below free_rows plain, every later word one
 * 16-bit record, low byte indexing `first` for bits 0..15 and high byte
 * indexing `second` for bits 16..31).  The tiles of 128 rows from
 * ceil(free_rows / 128) on keep the records: per tile and per 256-column
 * slice, row r's 8 records (words 8s .. 8s+7, zero past the row) are the
 * 16-byte block at byte 16 r, so one tile slice is 2048 bytes against 4096
 * for sign words.  `table_out` receives the 1024-word decode table of the
 * programs' record decode (word = table[rec & 255] | table[256 + (rec >> 8)]):
 * entries 0..255 the first half words, 256..511 the second half words
 * shifted to bits 16..31, the rest zero.  No counterpart in the reference,
 * whose runtime expands the records to sign words before its kernels run
 * (product_codebook.py:110-143, :229-237); this layout feeds the decode
 * programs' stage-1 record decode.  0 < free_rows < rank, as in
 * nqb_decode_product_codebook.
 */
int nqb_product_codebook_tiles_bytes(int64_t rank, int64_t in_features, int64_t free_rows, size_t *bytes);
int nqb_repack_product_codebook(const int32_t *payload, const int16_t *first, const int16_t *second,
                                int64_t rank, int64_t in_features, int64_t free_rows, void *tiles_out,
                                int32_t *table_out, void *stream);

/* Library identity: NQB_ABI_VERSION of the loaded build. */
int nqb_abi_version(void);

/* Last error message of the calling thread ("" after a successful call). */
const char *nqb_last_error(void);

/*
 * Bytes of device workspace nqb_linear needs for `tokens` tokens.
 * The workspace is scratch owned by the caller (256-byte aligned).  Its first
 * 16 KiB hold completion counters: zero-fill the workspace once before its
 * first use; every call leaves that region zero again, so one workspace
 * serves any sequence of calls (of any layer and token count) on one stream.
 * It must not be shared by calls that may run concurrently; after a call that
 * overlapped another on the same workspace, or after nqb_device_status
 * reported NQB_ERR_TIMEOUT, zero the counters again (nqb_workspace_reset).
 */
int nqb_linear_workspace_bytes(const nqb_linear_desc *layer, int64_t tokens, size_t *bytes);

/*
 * Zeroes the 16 KiB counter region at the start of a workspace (of nqb_linear,
 * nqb_grouped_linear or a program run) on `stream`, with cudaMemsetAsync; no
 * allocation.  No counterpart in the reference, which allocates its scratch
 * per call (cuda_kernels.py:816-874).
 */
int nqb_workspace_reset(void *workspace, size_t workspace_bytes, void *stream);

/*
 * y[tokens, m] (fp32, row-major) = layer(x[tokens, n]).
 * x_dtype: F32 / F16 / BF16, row-major contiguous.  Deterministic: the same
 * inputs give bitwise-identical y on every call.
 * Replaces launch_packed_linear (reference cuda_kernels.py:816-874), the
 * launcher behind CudaPackedBackend.linear (reference cuda_backend.py:243-278).
 */
int nqb_linear(const nqb_linear_desc *layer, const void *x, int32_t x_dtype, int64_t tokens,
               float *y, void *workspace, size_t workspace_bytes, void *stream);

/*
 * nqb_linear without a workspace argument, for callers that cannot allocate
 * device memory: plugins running inside another engine's executor or
 * processes with a fixed device-memory plan, where a cudaMalloc would bypass
 * the host's accounting or break its stream capture.  No counterpart in the
 * reference.
 *
 * Scratch comes from a static 8 MiB array in the library's device image (held
 * on every GPU that loads the library until exit).  Calls whose workspace
 * (nqb_linear_workspace_bytes) exceeds 8 MiB are rejected with
 * NQB_ERR_WORKSPACE and launch nothing.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress, with that device current);
 * make that first call before any stream capture.  Every call first zeroes the
 * array's counter region on its stream (cudaMemsetAsync), so a call that gave
 * up a bounded wait does not spoil later ones.  All calls on a device share
 * the one array, so calls that may overlap on the GPU (for example calls on
 * different streams) race: serialise them.  Allocates nothing.
 */
int nqb_linear_noalloc(const nqb_linear_desc *layer, const void *x, int32_t x_dtype, int64_t tokens,
                       float *y, void *stream);

/*
 * Two or three layers that share one input x, executed as one stage-1 and
 * one stage-2 launch.  y_out[i] is [tokens, layers[i].out_features] fp32.
 * Replaces launch_grouped_packed_linears (reference cuda_kernels.py:301-374);
 * unlike the reference it accepts any rank / width alignment, bias and int8
 * outlier scales.
 */
int nqb_grouped_workspace_bytes(const nqb_linear_desc *layers, int32_t count, int64_t tokens,
                                size_t *bytes);
int nqb_grouped_linear(const nqb_linear_desc *layers, int32_t count, const void *x,
                       int32_t x_dtype, int64_t tokens, float *const *y_out, void *workspace,
                       size_t workspace_bytes, void *stream);

/*
 * Dense low-rank patch epilogue: y[t,o] += sum_p L[o,p] * sum_i R[p,i] x[t,i].
 * L [m, p], R [p, n] in patch_dtype.  Workspace: tokens*p fp32.  A layer
 * whose descriptor carries the patch needs no separate call: nqb_linear
 * applies it (fused on the decode paths); this entry point stays for callers
 * that keep the patch outside the descriptor.
 * Replaces the F.linear pair of CudaPackedBackend.linear (reference
 * cuda_backend.py:275-277).
 */
int nqb_patch_accumulate(const void *x, int32_t x_dtype, int64_t tokens, int64_t in_features,
                         int64_t out_features, int64_t patch_rank, const void *patch_left,
                         const void *patch_right, int32_t patch_dtype, float *y, void *workspace,
                         size_t workspace_bytes, void *stream);

/*
 * Layout-v1 packing on the device.
 * nqb_pack_signs: signs [rows, cols] (+1/-1, F32/F16/BF16) -> words [rows, ceil(cols/32)].
 *   Replaces pack_sign_matrix (reference packed.py:170-188).
 * nqb_unpack_signs: words -> signs fp32 [rows, cols].  Replaces
 *   unpack_sign_matrix (reference packed.py:204-218).  Non-zero padding bits
 *   are reported through *bad_padding_rows (device int32, count of offending
 *   rows; may be NULL).
 */
int nqb_pack_signs(const void *signs, int32_t signs_dtype, int64_t rows, int64_t cols,
                   int32_t *words, void *stream);
int nqb_unpack_signs(const int32_t *words, int64_t rows, int64_t cols, float *signs,
                     int32_t *bad_padding_rows, void *stream);

/*
 * Expand a product-codebook right factor to layout-v1 words on the device.
 * Replaces decode_product_codebook_right_words (reference
 * product_codebook.py:110-143).
 */
int nqb_decode_product_codebook(const int32_t *free_words, int64_t free_rows, int64_t rank,
                                int64_t columns, const int32_t *payload, const int16_t *first,
                                const int16_t *second, int32_t *words_out, void *stream);

/*
 * Expand a mixed-V right factor (format mixed-v-free-k10-pair9-v1) to
 * layout-v1 words on the device: rows [0, free_rows) are copied from
 * free_words [free_rows, ceil(columns/32)]; every later word is
 * codebook[index] with the bit pair `pair` flipped, read from one 19-bit
 * record (index = bits 0..9, pair = bits 10..18, LSB-first across the
 * payload words; pairs (a, b), a < b < 32, numbered lexicographically).
 * codebook holds 1024 words.  Pair ids above 495 are the caller's to reject
 * (the kernel stays in bounds for any payload).  Replaces
 * launch_decode_mixed_v_right_words (reference cuda_kernels.py:877-910, the
 * Triton kernel at :11-62).
 */
int nqb_decode_mixed_v(const int32_t *free_words, int64_t free_rows, int64_t rank, int64_t columns,
                       const int32_t *payload, const int32_t *codebook, int32_t *words_out, void *stream);

/*
 * Decode-step shell (batch 1..16): the non-packed work of a decoder step
 * around its packed linears.  The reference runs these in its model shell
 * (runtime/torch_model.py:185-421) with Triton kernels pinned to one geometry
 * (cuda_kernels.py:401-812: RoPE, decode attention, cache update, bf16
 * output projection); these take any head count and cache length.
 * Asynchronous on `stream`; no allocation, no synchronisation.
 *
 * nqb_rmsnorm: per token, h += delta (when delta is not NULL, h written
 *   back), out = h * rsqrt(mean(h^2) + eps) * weight.  h, delta fp32
 *   [tokens, hidden]; weight [hidden]; out [tokens, hidden] in out_dtype.
 * nqb_qk_norm_rope: q fp32 [tokens, q_heads, head_dim], k and v fp32
 *   [tokens, kv_heads, head_dim].  q and k heads: RMSNorm over the head with
 *   q_weight / k_weight (either may be NULL: no norm), then rotate-half RoPE
 *   with cos_table / sin_table rows [tokens, head_dim]; q to q_out (bf16,
 *   shaped like q), k and v to the bf16 caches [kv_heads, cache_len, head_dim]
 *   at row position + t.  head_dim is 64, 128 or 256.
 * nqb_decode_attention: q bf16 [tokens, q_heads, head_dim]; token t attends
 *   to cache rows [0, keys + t) of kv head (q head / (q_heads / kv_heads))
 *   with scale head_dim^-1/2; out bf16 [tokens, q_heads * head_dim].
 *   Split-K partials go to the workspace (nqb_decode_attention_workspace_bytes).
 *   Alignment (else NQB_ERR_ALIGNMENT): k_cache, v_cache and workspace 16
 *   bytes; q and out head_dim / 16 bytes (8 for head_dim 128).
 * nqb_rmsnorm_residual: nqb_rmsnorm whose delta is normalised first when
 *   delta_weight is given: h += delta * rsqrt(mean(delta^2) + eps) *
 *   delta_weight, then out = h * rsqrt(mean(h^2) + eps) * weight (both
 *   weights in weight_dtype).  Gemma-3's sandwich norms: the post-attention
 *   (or post-feedforward) norm of the delta, the residual add and the next
 *   pre-norm in one pass (reference runtime/torch_model.py:637-653).
 * nqb_decode_attention_window: nqb_decode_attention where token t sees only
 *   the last `window` rows [keys + t - window, keys + t) (window 0: all);
 *   Gemma-3's sliding-window layers (torch_model.py:573-614).
 * nqb_embedding_bf16: out[t, :] = float(weight[ids[t], :]) * scale; weight
 *   bf16 [rows, dim], ids int64 [tokens], out fp32 [tokens, dim]; an id
 *   outside [0, rows) gives a zero row.  Replaces launch_bfloat16_embedding
 *   (reference cuda_kernels.py:620-668).
 * nqb_silu_mul: out[i] = silu(gate[i]) * up[i] over `count` fp32 values.
 * nqb_gemv_bf16: out[t, r] = sum_c weight[r, c] * x[t, c]; weight bf16
 *   [rows, cols] (cols a multiple of 8, at most 51200, 16-byte aligned),
 *   x bf16 [tokens, cols], out fp32 [tokens, rows].
 */
int nqb_rmsnorm(float *h, const float *delta, const void *weight, int32_t weight_dtype, int64_t tokens,
                int64_t hidden, float eps, void *out, int32_t out_dtype, void *stream);
int nqb_qk_norm_rope(const float *q, const float *k, const float *v, const void *q_weight, const void *k_weight,
                     int32_t weight_dtype, const float *cos_table, const float *sin_table, int64_t tokens,
                     int32_t q_heads, int32_t kv_heads, int32_t head_dim, float eps, void *q_out, void *k_cache,
                     void *v_cache, int64_t cache_len, int64_t position, void *stream);
int nqb_decode_attention_workspace_bytes(int64_t keys, int64_t tokens, int32_t q_heads, int32_t head_dim,
                                         size_t *bytes);
int nqb_decode_attention(const void *q, const void *k_cache, const void *v_cache, int64_t cache_len, int64_t keys,
                         int64_t tokens, int32_t q_heads, int32_t kv_heads, int32_t head_dim, void *out,
                         void *workspace, size_t workspace_bytes, void *stream);
int nqb_rmsnorm_residual(float *h, const float *delta, const void *delta_weight, const void *weight,
                         int32_t weight_dtype, int64_t tokens, int64_t hidden, float eps, void *out, int32_t out_dtype,
                         void *stream);
int nqb_decode_attention_window(const void *q, const void *k_cache, const void *v_cache, int64_t cache_len,
                                int64_t keys, int64_t tokens, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                                int64_t window, void *out, void *workspace, size_t workspace_bytes, void *stream);
int nqb_embedding_bf16(const int64_t *ids, int64_t tokens, const void *weight, int64_t rows, int64_t dim, float scale,
                       float *out, void *stream);
int nqb_silu_mul(const float *gate, const float *up, int64_t count, void *out, int32_t out_dtype, void *stream);
int nqb_gemv_bf16(const void *weight, int64_t rows, int64_t cols, const void *x, int64_t tokens, float *out,
                  void *stream);

/*
 * Kernel-native copy of a layout-v1 sign matrix for the tensor-core path:
 * rows are grouped in tiles of 128; within a tile, for every 4-word chunk of a
 * row, the 128 rows' 16-byte chunks are stored consecutively; rows and chunks
 * are zero-padded (to a multiple of 128 rows and of 8 words per row).
 * The reference has no counterpart: it re-reads layout v1 in every kernel
 * (cuda_kernels.py:65-162); preparing a device layout at load time follows its
 * own prepare-time transform for mixed-V (cuda_backend.py:209-224).
 */
int nqb_repack_bytes(int64_t rows, int64_t cols, size_t *bytes);
int nqb_repack_signs(const int32_t *words, int64_t rows, int64_t cols, void *tiles, void *stream);

/*
 * Which kernels a call with these arguments would run: *path is
 * NQB_PATH_GENERIC (CUDA-core kernels), NQB_PATH_TENSOR_CORE (tcgen05 decode
 * kernels) or NQB_PATH_PREFILL (tcgen05 prefill kernels).  Host-only;
 * launches nothing.
 */
#define NQB_PATH_GENERIC 0
#define NQB_PATH_TENSOR_CORE 1 /* tcgen05 int8 decode kernels, 1..16 tokens */
#define NQB_PATH_PREFILL 2     /* tcgen05 fp16 prefill kernels, more than 16 tokens */
int nqb_linear_path(const nqb_linear_desc *layers, int32_t count, int32_t x_dtype, int64_t tokens,
                    int32_t *path);

/*
 * Reads and clears the device-side status word of the tensor-core kernels
 * (NQB_ERR_TIMEOUT when a bounded wait gave up, else NQB_OK).  Synchronous.
 */
int nqb_device_status(int32_t *status);

/*
 * Persistent decode program: a fixed, ordered sequence of packed-linear calls
 * ("ops", each 1..3 layers sharing one input, 1..16 tokens) run by ONE
 * cooperative launch with one CTA per SM.  Ops and their two stages execute
 * strictly in order (a grid-wide barrier after every stage, so an op may read
 * an earlier op's output); only the sign-word streaming runs ahead of the
 * barriers.  It replaces the reference's CUDA-graph replay of per-linear
 * kernels for a decode step (runtime/torch_model.py:300-340 captures the
 * per-projection Triton launches; cuda_backend.py:286-330 is the per-call
 * launcher): results equal the per-call nqb_linear / nqb_grouped_linear
 * tensor-core path within fp32 reduction-order rounding.
 *
 * Every op must take the tensor-core decode path (nqb_linear_path ==
 * NQB_PATH_TENSOR_CORE).  The x and y device pointers, the descriptors and
 * the device arrays they point to are captured at create time and must stay
 * valid while the program exists.  Run needs a workspace of
 * nqb_program_workspace_bytes (256-byte aligned) whose first 16 KiB are zero
 * before the first run (every run leaves them zero).
 */
/* Program op input code: x is the gate and x2 the up projection, both fp32
 * [tokens, in_features]; the op reads silu(gate) * up (a SwiGLU product) as
 * its input, so a gate/up op and the down op that consumes it share one
 * program.  Members of such an op carry no salient columns or overlay rows. */
#define NQB_X_SWIGLU 16
/* Program op input code: like NQB_X_SWIGLU with gelu_tanh(gate) * up, the
 * tanh form of GELU (Gemma-3's gated-GELU MLP, reference
 * runtime/torch_model.py:460-505).                                          */
#define NQB_X_GEGLU 17

/*
 * Decoder-step extensions of a program op (nqb_program_op.ext; NULL = a plain
 * linear op).  With them one program runs a whole Qwen3-style decode step
 * (reference runtime/torch_model.py:185-421 runs it as separate modules):
 *
 * - Residual-stream input (norm_stats != NULL, linear ops): x is the fp32
 *   residual stream h [tokens, in_features]; the op's input is
 *   h * rsqrt(sum(h^2) / in_features + eps) * norm_weight, with sum(h^2) per
 *   token added up (in tile order) from norm_stats [ceil(in_features/128)]
 *   [tokens]: per-128-row partial sums written by nqb_residual_stats or by a
 *   NQB_EPI_RESIDUAL epilogue.  The weight is folded into the input scale and
 *   the norm factor applied to the latent, so h is read once.
 * - Epilogue (stage 2 of linear ops):
 *   NQB_EPI_STORE    y = out (plain);
 *   NQB_EPI_RESIDUAL y[0] is h: h += out, and out_stats [ceil(m/128)][tokens]
 *                    receives the new h's per-tile sums of squares;
 *   NQB_EPI_QK_ROPE  members q, k, v with head_dim 128 (one 128-row tile per
 *                    head): per-head RMSNorm of q and k with q_norm_weight /
 *                    k_norm_weight (NULL: none), rotate-half RoPE with the
 *                    cos/sin rows [tokens][128], then q -> `q` (bf16
 *                    [tokens, q_heads * 128]) and k, v -> the bf16 caches
 *                    [kv_heads, cache_len, 128] at row position + t.  y is
 *                    not written.
 *   Members of these epilogues carry no int8 overlay rows.
 * - NQB_OP_ATTENTION (layers NULL, count 0, x / y NULL): grouped-query
 *   attention of `q` over the caches, token t seeing rows [0, position + 1 + t),
 *   scale head_dim^-1/2, bf16 result to attn_out [tokens, q_heads * 128];
 *   head_dim 128 and q_heads == 4 * kv_heads.  It takes two stages of the
 *   program (split-K partials over all CTAs, then their fixed-order join).
 */
#define NQB_OP_LINEAR 0
#define NQB_OP_ATTENTION 1
#define NQB_EPI_STORE 0
#define NQB_EPI_RESIDUAL 1
#define NQB_EPI_QK_ROPE 2

typedef struct nqb_program_op_ext {
  int32_t kind;              /* NQB_OP_LINEAR / NQB_OP_ATTENTION */
  int32_t epilogue;          /* NQB_EPI_* (linear ops) */
  const float *norm_stats;   /* residual-stream input: per-tile sums of h^2, or NULL */
  const void *norm_weight;   /* [in_features] */
  int32_t norm_weight_dtype; /* F32 / F16 / BF16 */
  float eps;                 /* of the input norm and of the q/k head norms */
  float *out_stats;          /* NQB_EPI_RESIDUAL: per-tile sums of the new h^2 */
  int32_t q_heads, kv_heads, head_dim;
  const void *q_norm_weight; /* [head_dim] or NULL */
  const void *k_norm_weight; /* [head_dim] or NULL */
  int32_t qk_norm_dtype;
  const float *cos_table;    /* [tokens][head_dim] */
  const float *sin_table;
  void *q;                   /* bf16 [tokens, q_heads * head_dim] */
  void *k_cache;             /* bf16 [kv_heads, cache_len, head_dim] */
  void *v_cache;
  int64_t cache_len;
  int64_t position;          /* first row of this step's tokens in the caches */
  void *attn_out;            /* NQB_OP_ATTENTION: bf16 [tokens, q_heads * head_dim] */
  /* 0: the tokens are consecutive positions of one sequence (token t at
   * cache row position + t, attending to rows [0, position + t]).  > 0: a
   * batch of independent sequences, token t the next token of sequence t,
   * whose caches start sequence_stride elements after sequence t - 1's
   * (k_cache / v_cache then hold [tokens][kv_heads, cache_len, head_dim]):
   * token t at row `position` of its own caches, attending to rows
   * [0, position].  A multiple of 8, at least kv_heads * cache_len *
   * head_dim; the same on an op's QK_ROPE epilogue and its attention op.   */
  int64_t sequence_stride;
} nqb_program_op_ext;

typedef struct nqb_program_op {
  const nqb_linear_desc *layers; /* count members sharing x */
  int32_t count;                 /* 1..3 */
  const void *x;                 /* [tokens, in_features], x_dtype */
  int32_t x_dtype;               /* NQB_F32 / NQB_F16 / NQB_BF16, NQB_X_SWIGLU or NQB_X_GEGLU */
  float *const *y;               /* count outputs [tokens, out_features] fp32 */
  const void *x2;                /* NQB_X_SWIGLU / NQB_X_GEGLU: the up projection; else NULL */
  const nqb_program_op_ext *ext; /* decoder-step extensions, or NULL */
} nqb_program_op;

typedef struct nqb_program nqb_program;

int nqb_program_create(const nqb_program_op *ops, int32_t op_count, int64_t tokens, nqb_program **program);
/*
 * Per-128-row partial sums of squares of the fp32 residual stream h [tokens,
 * hidden]: stats[i][t] = sum of h[t][128 i .. 128 i + 127]^2 (fixed order), the
 * norm_stats a program's first residual-stream op reads.  No counterpart in
 * the reference (its RMSNorm module reduces the row itself).
 */
int nqb_residual_stats(const float *h, int64_t tokens, int64_t hidden, float *stats, void *stream);
int nqb_program_workspace_bytes(const nqb_program *program, size_t *bytes);
int nqb_program_run(const nqb_program *program, void *workspace, size_t workspace_bytes, void *stream);
/*
 * nqb_program_run as a programmatic dependent launch of the preceding kernel
 * on the stream: the program's producer warps start streaming sign words while
 * that kernel finishes; everything that reads activations or the workspace
 * waits for its completion.  For a program that follows other kernels (a
 * decoder step's norm and attention kernels); a run right after a run of a
 * program measured slower than nqb_program_run.
 */
int nqb_program_run_dependent(const nqb_program *program, void *workspace, size_t workspace_bytes,
                              void *stream);
int nqb_program_destroy(nqb_program *program);
/* Launch shape of a created program: CTAs (one per SM used) and cluster size. */
int nqb_program_shape(const nqb_program *program, int32_t *ctas, int32_t *cluster_size);
/*
 * Failure-path tests.  nqb_debug_set_barrier_limit sets how many polls a
 * program's grid barrier makes before it gives up (0 restores the default of
 * 2^22) for later launches; nqb_program_debug_barrier_skew makes every grid
 * barrier of later runs of `program` wait for `skew` arrivals that never come
 * (0 turns it off).  A run with a skew gives up each barrier after the limit,
 * reports NQB_ERR_TIMEOUT through nqb_device_status, leaves its outputs
 * undefined and its workspace counters zero, and a later run without the skew
 * is correct again.  No counterpart in the reference (its kernels wait on
 * nothing).
 */
int nqb_debug_set_barrier_limit(uint32_t polls);
int nqb_program_debug_barrier_skew(nqb_program *program, uint32_t skew);
/*
 * Phase trace of the last run (trace build only, libnqb_trace.so; the normal
 * build returns NQB_ERR_UNSUPPORTED): SM cycles per [cta][stage][phase] spent
 * by the CTA's first consumer thread; count >= ctas * 2 * ops * 11.  Phases:
 * tables, quantise, wait-signs, mma, drain, send, wait-quarters, sum,
 * release, epilogue, grid-barrier.  Synchronous.
 */
int nqb_program_trace(const nqb_program *program, int64_t *cycles, size_t count);

#ifdef __cplusplus
}
#endif

#endif /* NQB_H */
