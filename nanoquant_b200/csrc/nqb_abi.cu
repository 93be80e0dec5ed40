// C ABI of libnqb (declared in include/nqb.h): argument validation,
// workspace accounting and dispatch to the kernels.
#include <cstring>
#include <mutex>
#include <vector>

#include "nqb_decode_tc.cuh"
#include "nqb_generic.cuh"
#include "nqb_prefill_tc.cuh"
#include "nqb_program.cuh"

namespace nqb {

static thread_local char g_last_error[1024] = "";

int fail(int code, const char *fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return code;
}

int ok() {
  g_last_error[0] = '\0';
  return NQB_OK;
}

int cuda_status(cudaError_t err, const char *what) {
  return fail(NQB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

static bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int ensure_dynamic_smem(const void *kernel, size_t bytes) {
  struct Entry {
    const void *kernel;
    int device;
    size_t bytes;
  };
  static std::mutex lock;
  static std::vector<Entry> entries;
  // static shared memory counts against the same 48 KB default, so any
  // non-zero dynamic size gets the attribute
  if (bytes == 0) return NQB_OK;
  int device = 0;
  NQB_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  std::lock_guard<std::mutex> guard(lock);
  for (Entry &e : entries) {
    if (e.kernel == kernel && e.device == device) {
      if (e.bytes >= bytes) return NQB_OK;
      NQB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
               "cudaFuncSetAttribute");
      e.bytes = bytes;
      return NQB_OK;
    }
  }
  int optin = 0;
  NQB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device), "cudaDeviceGetAttribute");
  if (bytes > static_cast<size_t>(optin))
    return fail(NQB_ERR_UNSUPPORTED, "kernel needs %zu B of shared memory, device allows %d", bytes, optin);
  NQB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
           "cudaFuncSetAttribute");
  entries.push_back({kernel, device, bytes});
  return NQB_OK;
}

// Checks one layer descriptor; `name` prefixes messages for grouped calls.
static int validate_layer(const nqb_linear_desc *d, const char *name) {
  if (d == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "%s: layer descriptor is NULL", name);
  if (d->in_features <= 0 || d->out_features <= 0 || d->rank <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: in_features, out_features and rank must be positive", name);
  if (d->in_features > (1ll << 31) || d->out_features > (1ll << 31) || d->rank > (1ll << 31))
    return fail(NQB_ERR_UNSUPPORTED, "%s: dimensions above 2^31 are not supported", name);
  // A tiles-only layer (no layout-v1 words, no compact V) runs on the
  // tensor-core decode, prefill and program paths, which read the tiles only.
  const bool tiles_only = d->left_words == nullptr && d->right_words == nullptr && d->codebook_payload == nullptr;
  if (tiles_only) {
    if (d->left_tiles == nullptr || d->right_tiles == nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: left_words is NULL (a layer without words needs both tile copies)",
                  name);
  } else if (d->left_words == nullptr) {
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: left_words is NULL", name);
  }
  const bool codebook = d->codebook_payload != nullptr;
  if (codebook) {
    if (d->right_words != nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: give either right_words or a product codebook, not both", name);
    if (d->codebook_free_rows <= 0 || d->codebook_free_rows >= d->rank)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: product-codebook free rows must be between zero and rank", name);
    if (d->codebook_free_words == nullptr || d->codebook_first == nullptr || d->codebook_second == nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: product-codebook tables or free words are NULL", name);
    if (!aligned(d->codebook_free_words, 4) || !aligned(d->codebook_payload, 4) ||
        !aligned(d->codebook_first, 2) || !aligned(d->codebook_second, 2))
      return fail(NQB_ERR_ALIGNMENT, "%s: product-codebook operands are misaligned", name);
  } else if (d->right_words == nullptr && !tiles_only) {
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: right_words is NULL", name);
  }
  if ((d->left_words && !aligned(d->left_words, 4)) || (d->right_words && !aligned(d->right_words, 4)))
    return fail(NQB_ERR_ALIGNMENT, "%s: sign words must be 4-byte aligned", name);
  if (!is_float_dtype(d->scale_dtype))
    return fail(NQB_ERR_DTYPE, "%s: scale dtype %d is not F32/F16/BF16", name, d->scale_dtype);
  if (d->scale_pre == nullptr || d->scale_mid == nullptr || d->scale_post == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: a scale vector is NULL", name);
  if (d->bias != nullptr && !is_float_dtype(d->bias_dtype))
    return fail(NQB_ERR_DTYPE, "%s: bias dtype %d is not F32/F16/BF16", name, d->bias_dtype);
  if (d->outlier_count < 0 || d->outlier_count > d->in_features)
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: outlier count is outside the input dimension", name);
  if (d->outlier_count > 0) {
    if (d->outlier_indices == nullptr || d->outlier_values == nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: outlier indices or values are NULL", name);
    const int32_t vd = d->outlier_value_dtype;
    if (!(is_float_dtype(vd) || vd == NQB_I8))
      return fail(NQB_ERR_DTYPE, "%s: outlier value dtype %d is not F32/F16/BF16/I8", name, vd);
    if ((vd == NQB_I8) != (d->outlier_scales != nullptr))
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: outlier scales are required for, and only for, int8 values",
                  name);
  }
  if (d->overlay_rows < 0 || d->overlay_rows > d->out_features)
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: overlay row count is outside the output dimension", name);
  if (d->overlay_rows > 0) {
    if (d->overlay_row_ids == nullptr || d->overlay_values == nullptr || d->overlay_scales == nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: overlay operands are NULL", name);
    if (!is_float_dtype(d->overlay_scale_dtype))
      return fail(NQB_ERR_DTYPE, "%s: overlay scale dtype %d is not F32/F16/BF16", name, d->overlay_scale_dtype);
  }
  if (d->coded_right_tiles != nullptr) {
    if (d->coded_codebook == nullptr || d->right_tiles == nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: coded tiles need the codebook and the plain right tiles", name);
    if (d->coded_free_rows <= 0 || d->coded_free_rows >= d->rank)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: coded free rows must be between zero and rank", name);
    if (d->coded_format != NQB_CODED_MIXED_V && d->coded_format != NQB_CODED_PRODUCT_CODEBOOK)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: coded format %d is not NQB_CODED_*", name, d->coded_format);
    if (!aligned(d->coded_right_tiles, 16) || !aligned(d->coded_codebook, 16))
      return fail(NQB_ERR_ALIGNMENT, "%s: coded tiles and codebook must be 16-byte aligned", name);
  }
  if (d->patch_rank < 0 || d->patch_rank > (1ll << 20))
    return fail(NQB_ERR_INVALID_ARGUMENT, "%s: patch rank must be between 0 and 2^20", name);
  if (d->patch_rank > 0) {
    if (d->patch_left == nullptr || d->patch_right == nullptr)
      return fail(NQB_ERR_INVALID_ARGUMENT, "%s: patch factors are NULL", name);
    if (!is_float_dtype(d->patch_dtype))
      return fail(NQB_ERR_DTYPE, "%s: patch dtype %d is not F32/F16/BF16", name, d->patch_dtype);
  }
  return NQB_OK;
}

static int validate_input(const void *x, int32_t x_dtype, int64_t tokens) {
  if (x == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "input x is NULL");
  if (!is_float_dtype(x_dtype)) return fail(NQB_ERR_DTYPE, "input dtype %d is not F32/F16/BF16", x_dtype);
  if (tokens <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "token count must be positive");
  if (tokens > (1ll << 24)) return fail(NQB_ERR_UNSUPPORTED, "token count above 2^24 is not supported");
  return NQB_OK;
}

// Latent columns reserved for a member: its rank rounded up to 4 floats, so
// the prefill path can place every member on a 16-byte boundary.
static int64_t latent_columns(int64_t rank) { return (rank + 3) & ~int64_t(3); }

static size_t latent_bytes(int64_t tokens, int64_t total_columns) {
  return align_up(static_cast<size_t>(tokens) * total_columns * sizeof(float), 256);
}

// Latent region of a call: the members' latents, then their patch latents
// (member i's [tokens][patch_rank_i] block after those of members < i).
static size_t latent_region_bytes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  int64_t columns = 0, patch = 0;
  for (int i = 0; i < count; ++i) {
    columns += latent_columns(layers[i].rank);
    patch += layers[i].patch_rank;
  }
  return latent_bytes(tokens, columns) + latent_bytes(tokens, patch);
}

// Workspace layout shared by every call: [completion counters][latent][tensor-core partials].
// The counter region has a fixed size and offset, so one workspace can serve
// calls of any shape in sequence; it must be zero before its first use and
// every call leaves it zero.
static size_t workspace_bytes(size_t latent, size_t tc_partials) { return kCounterRegionBytes + latent + tc_partials; }

// Path-specific workspace after the latent: tensor-core decode partials or
// prefill fp16 activations (at most one of the two is non-zero for a call).
static size_t path_extra_bytes(const nqb_linear_desc *layers, int count, int64_t tokens) {
  return tc_extra_workspace_bytes(layers, count, tokens) + prefill_workspace_bytes(layers, count, tokens);
}

static void fill_stage1_member(Stage1Member &m, const nqb_linear_desc &d, int64_t latent_offset,
                               int32_t block_begin) {
  m.words = reinterpret_cast<const uint32_t *>(d.right_words);
  m.cb_free = reinterpret_cast<const uint32_t *>(d.codebook_free_words);
  m.cb_payload = reinterpret_cast<const uint16_t *>(d.codebook_payload);
  m.cb_first = reinterpret_cast<const uint16_t *>(d.codebook_first);
  m.cb_second = reinterpret_cast<const uint16_t *>(d.codebook_second);
  m.cb_free_rows = d.codebook_payload != nullptr ? d.codebook_free_rows : 0;
  m.pre = d.scale_pre;
  m.mid = d.scale_mid;
  m.rank = d.rank;
  m.latent_offset = latent_offset;
  m.block_begin = block_begin;
}

static void fill_stage2_member(Stage2Member &m, const nqb_linear_desc &d, int64_t latent_offset,
                               float *y, int32_t block_begin) {
  m.words = reinterpret_cast<const uint32_t *>(d.left_words);
  m.out_features = d.out_features;
  m.rank = d.rank;
  m.wpr = words_for(d.rank);
  m.latent_offset = latent_offset;
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
  m.y = y;
  m.block_begin = block_begin;
}

// Generic two-launch execution of 1..3 layers sharing x.
static int run_generic(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype,
                       int64_t tokens, float *const *ys, float *latent, cudaStream_t stream) {
  const int64_t n = layers[0].in_features;
  int64_t total_rank = 0, max_rank = 0;
  for (int i = 0; i < count; ++i) {
    total_rank += layers[i].rank;
    if (layers[i].rank > max_rank) max_rank = layers[i].rank;
  }

  Stage1Params p1;
  std::memset(&p1, 0, sizeof(p1));
  p1.count = count;
  p1.x = x;
  p1.x_dtype = x_dtype;
  p1.scale_dtype = layers[0].scale_dtype;
  p1.in_features = n;
  p1.wpr = words_for(n);
  p1.tokens = tokens;
  p1.total_rank = total_rank;
  p1.latent = latent;
  p1.tok_tile = choose_tok_tile(tokens, n);
  int64_t blocks = 0, offset = 0;
  for (int i = 0; i < count; ++i) {
    fill_stage1_member(p1.m[i], layers[i], offset, static_cast<int32_t>(blocks));
    offset += layers[i].rank;
    blocks += (layers[i].rank + kGenericWarps - 1) / kGenericWarps;
  }
  if ((tokens + p1.tok_tile - 1) / p1.tok_tile > 65535)
    return fail(NQB_ERR_UNSUPPORTED, "too many tokens for the generic path: %lld", (long long)tokens);
  NQB_CHECK(launch_stage1_generic(p1, static_cast<int32_t>(blocks), stream));

  Stage2Params p2;
  std::memset(&p2, 0, sizeof(p2));
  p2.count = count;
  p2.x = x;
  p2.x_dtype = x_dtype;
  p2.scale_dtype = layers[0].scale_dtype;
  p2.in_features = n;
  p2.tokens = tokens;
  p2.total_rank = total_rank;
  p2.latent = latent;
  p2.tok_tile = choose_tok_tile(tokens, max_rank);
  blocks = 0;
  offset = 0;
  for (int i = 0; i < count; ++i) {
    fill_stage2_member(p2.m[i], layers[i], offset, ys[i], static_cast<int32_t>(blocks));
    offset += layers[i].rank;
    blocks += (layers[i].out_features + kGenericWarps - 1) / kGenericWarps;
  }
  if ((tokens + p2.tok_tile - 1) / p2.tok_tile > 65535)
    return fail(NQB_ERR_UNSUPPORTED, "too many tokens for the generic path: %lld", (long long)tokens);
  NQB_CHECK(launch_stage2_generic(p2, static_cast<int32_t>(blocks), max_rank, stream));
  return NQB_OK;
}

}  // namespace nqb

using namespace nqb;

extern "C" {

int nqb_abi_version(void) { return NQB_ABI_VERSION; }

const char *nqb_last_error(void) { return g_last_error; }

int nqb_workspace_reset(void *workspace, size_t workspace_bytes, void *stream) {
  if (workspace == nullptr || workspace_bytes < kCounterRegionBytes)
    return fail(NQB_ERR_WORKSPACE, "workspace must hold at least the %zu-byte counter region", kCounterRegionBytes);
  NQB_CUDA(cudaMemsetAsync(workspace, 0, kCounterRegionBytes, static_cast<cudaStream_t>(stream)),
           "zeroing the workspace counters");
  return ok();
}

int nqb_linear_workspace_bytes(const nqb_linear_desc *layer, int64_t tokens, size_t *bytes) {
  NQB_CHECK(validate_layer(layer, "layer"));
  if (bytes == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (tokens <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "token count must be positive");
  *bytes = workspace_bytes(latent_region_bytes(layer, 1, tokens), path_extra_bytes(layer, 1, tokens));
  return ok();
}

}  // extern "C"

namespace nqb {

// Runs 1..3 validated layers sharing x on the path their shapes take.  The
// tensor-core decode path applies each member's patch inside its stages; the
// prefill and generic paths add it with two small kernels per patched member.
static int run_layers(const nqb_linear_desc *layers, int count, const void *x, int32_t x_dtype, int64_t tokens,
                      float *const *ys, void *workspace, size_t workspace_bytes_given, void *stream) {
  const size_t need = latent_region_bytes(layers, count, tokens);
  const size_t tc_need = path_extra_bytes(layers, count, tokens);
  if (workspace == nullptr || workspace_bytes_given < workspace_bytes(need, tc_need) || !aligned(workspace, 256))
    return fail(NQB_ERR_WORKSPACE, "workspace needs %zu bytes aligned to 256, got %zu",
                workspace_bytes(need, tc_need), workspace_bytes_given);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char *base = static_cast<char *>(workspace);
  int32_t *counters = reinterpret_cast<int32_t *>(base);
  float *latent = reinterpret_cast<float *>(base + kCounterRegionBytes);
  int64_t columns = 0;
  for (int i = 0; i < count; ++i) columns += latent_columns(layers[i].rank);
  float *patch = reinterpret_cast<float *>(base + kCounterRegionBytes + latent_bytes(tokens, columns));
  char *extra = base + kCounterRegionBytes + need;
  if (tc_eligible(layers, count, x_dtype, tokens))
    return run_tc(layers, count, x, x_dtype, tokens, ys, counters, extra, tc_need, latent, patch, s);
  if (prefill_eligible(layers, count, x_dtype, tokens)) {
    NQB_CHECK(run_prefill(layers, count, x, x_dtype, tokens, ys, latent, extra, tc_need, s));
  } else {
    for (int i = 0; i < count; ++i)
      if (layers[i].left_words == nullptr)
        return fail(NQB_ERR_UNSUPPORTED,
                    "layer %d keeps only its kernel-native tiles, and %lld token(s) of this input take the generic "
                    "path, which reads the layout-v1 words",
                    i, static_cast<long long>(tokens));
    NQB_CHECK(run_generic(layers, count, x, x_dtype, tokens, ys, latent, s));
  }
  int64_t patch_offset = 0;
  for (int i = 0; i < count; ++i) {
    const nqb_linear_desc &d = layers[i];
    if (d.patch_rank == 0) continue;
    NQB_CHECK(launch_patch(x, x_dtype, tokens, d.in_features, d.out_features, d.patch_rank, d.patch_left,
                           d.patch_right, d.patch_dtype, ys[i], patch + tokens * patch_offset, s));
    patch_offset += d.patch_rank;
  }
  return NQB_OK;
}

}  // namespace nqb

extern "C" {

int nqb_linear(const nqb_linear_desc *layer, const void *x, int32_t x_dtype, int64_t tokens, float *y,
               void *workspace, size_t workspace_bytes, void *stream) {
  NQB_CHECK(validate_layer(layer, "layer"));
  NQB_CHECK(validate_input(x, x_dtype, tokens));
  if (y == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "output y is NULL");
  float *ys[1] = {y};
  NQB_CHECK(run_layers(layer, 1, x, x_dtype, tokens, ys, workspace, workspace_bytes, stream));
  return ok();
}

int nqb_grouped_workspace_bytes(const nqb_linear_desc *layers, int32_t count, int64_t tokens, size_t *bytes) {
  if (layers == nullptr || count < 1 || count > kMaxMembers)
    return fail(NQB_ERR_INVALID_ARGUMENT, "grouped call takes 1 to %d layers", kMaxMembers);
  if (bytes == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (tokens <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "token count must be positive");
  for (int i = 0; i < count; ++i) NQB_CHECK(validate_layer(layers + i, "grouped member"));
  *bytes = workspace_bytes(latent_region_bytes(layers, count, tokens), path_extra_bytes(layers, count, tokens));
  return ok();
}

int nqb_grouped_linear(const nqb_linear_desc *layers, int32_t count, const void *x, int32_t x_dtype,
                       int64_t tokens, float *const *y_out, void *workspace, size_t workspace_bytes,
                       void *stream) {
  if (layers == nullptr || count < 1 || count > kMaxMembers)
    return fail(NQB_ERR_INVALID_ARGUMENT, "grouped call takes 1 to %d layers", kMaxMembers);
  if (y_out == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "output list is NULL");
  for (int i = 0; i < count; ++i) {
    NQB_CHECK(validate_layer(layers + i, "grouped member"));
    if (layers[i].in_features != layers[0].in_features)
      return fail(NQB_ERR_INVALID_ARGUMENT, "grouped members must share in_features");
    if (layers[i].scale_dtype != layers[0].scale_dtype)
      return fail(NQB_ERR_DTYPE, "grouped members must share the scale dtype");
    if (y_out[i] == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "output %d is NULL", i);
  }
  NQB_CHECK(validate_input(x, x_dtype, tokens));
  NQB_CHECK(run_layers(layers, count, x, x_dtype, tokens, y_out, workspace, workspace_bytes, stream));
  return ok();
}

int nqb_patch_accumulate(const void *x, int32_t x_dtype, int64_t tokens, int64_t in_features,
                         int64_t out_features, int64_t patch_rank, const void *patch_left,
                         const void *patch_right, int32_t patch_dtype, float *y, void *workspace,
                         size_t workspace_bytes, void *stream) {
  NQB_CHECK(validate_input(x, x_dtype, tokens));
  if (in_features <= 0 || out_features <= 0 || patch_rank <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "patch dimensions must be positive");
  if (patch_left == nullptr || patch_right == nullptr || y == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "patch operand is NULL");
  if (!is_float_dtype(patch_dtype)) return fail(NQB_ERR_DTYPE, "patch dtype %d is not F32/F16/BF16", patch_dtype);
  const size_t need = static_cast<size_t>(tokens) * patch_rank * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(NQB_ERR_WORKSPACE, "patch workspace needs %zu bytes, got %zu", need, workspace_bytes);
  NQB_CHECK(launch_patch(x, x_dtype, tokens, in_features, out_features, patch_rank, patch_left, patch_right,
                         patch_dtype, y, static_cast<float *>(workspace), reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_pack_signs(const void *signs, int32_t signs_dtype, int64_t rows, int64_t cols, int32_t *words,
                   void *stream) {
  if (signs == nullptr || words == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "pack operand is NULL");
  if (rows <= 0 || cols <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "sign matrix dimensions must be positive");
  if (!is_float_dtype(signs_dtype)) return fail(NQB_ERR_DTYPE, "sign dtype %d is not F32/F16/BF16", signs_dtype);
  NQB_CHECK(launch_pack(signs, signs_dtype, rows, cols, reinterpret_cast<uint32_t *>(words),
                        reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_unpack_signs(const int32_t *words, int64_t rows, int64_t cols, float *signs, int32_t *bad_padding_rows,
                     void *stream) {
  if (words == nullptr || signs == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "unpack operand is NULL");
  if (rows <= 0 || cols <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "sign matrix dimensions must be positive");
  NQB_CHECK(launch_unpack(reinterpret_cast<const uint32_t *>(words), rows, cols, signs, bad_padding_rows,
                          reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_repack_bytes(int64_t rows, int64_t cols, size_t *bytes) {
  if (rows <= 0 || cols <= 0 || bytes == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "repack needs positive dimensions and an output pointer");
  *bytes = repack_bytes(rows, cols);
  return ok();
}

int nqb_repack_signs(const int32_t *words, int64_t rows, int64_t cols, void *tiles, void *stream) {
  if (words == nullptr || tiles == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "repack operand is NULL");
  if (rows <= 0 || cols <= 0) return fail(NQB_ERR_INVALID_ARGUMENT, "sign matrix dimensions must be positive");
  if (!aligned(tiles, 16) || !aligned(words, 4)) return fail(NQB_ERR_ALIGNMENT, "repack buffers are misaligned");
  NQB_CHECK(launch_repack(reinterpret_cast<const uint32_t *>(words), rows, cols, static_cast<uint32_t *>(tiles),
                          reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_linear_path(const nqb_linear_desc *layers, int32_t count, int32_t x_dtype, int64_t tokens, int32_t *path) {
  if (layers == nullptr || count < 1 || count > kMaxMembers || path == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "path query takes 1 to %d layers and an output pointer", kMaxMembers);
  for (int i = 0; i < count; ++i) NQB_CHECK(validate_layer(layers + i, "layer"));
  *path = tc_eligible(layers, count, x_dtype, tokens)        ? NQB_PATH_TENSOR_CORE
          : prefill_eligible(layers, count, x_dtype, tokens) ? NQB_PATH_PREFILL
                                                              : NQB_PATH_GENERIC;
  return ok();
}

int nqb_device_status(int32_t *status) {
  if (status == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "status is NULL");
  NQB_CHECK(tc_device_error(status));
  int32_t prefill_status = 0, program_status = 0;
  NQB_CHECK(prefill_device_error(&prefill_status));
  NQB_CHECK(program_device_error(&program_status));
  if (*status == NQB_OK) *status = prefill_status;
  if (*status == NQB_OK) *status = program_status;
  return ok();
}

int nqb_decode_product_codebook(const int32_t *free_words, int64_t free_rows, int64_t rank, int64_t columns,
                                const int32_t *payload, const int16_t *first, const int16_t *second,
                                int32_t *words_out, void *stream) {
  if (free_words == nullptr || payload == nullptr || first == nullptr || second == nullptr || words_out == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "product-codebook operand is NULL");
  if (free_rows <= 0 || free_rows >= rank || columns <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "product-codebook free rows must be between zero and rank");
  NQB_CHECK(launch_decode_codebook(reinterpret_cast<const uint32_t *>(free_words), free_rows, rank, columns,
                                   reinterpret_cast<const uint16_t *>(payload),
                                   reinterpret_cast<const uint16_t *>(first),
                                   reinterpret_cast<const uint16_t *>(second),
                                   reinterpret_cast<uint32_t *>(words_out), reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_decode_mixed_v(const int32_t *free_words, int64_t free_rows, int64_t rank, int64_t columns,
                       const int32_t *payload, const int32_t *codebook, int32_t *words_out, void *stream) {
  if (free_words == nullptr || payload == nullptr || codebook == nullptr || words_out == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "mixed-V operand is NULL");
  if (free_rows <= 0 || free_rows >= rank || columns <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "mixed-V free rows must be between zero and rank");
  NQB_CHECK(launch_decode_mixed_v(reinterpret_cast<const uint32_t *>(free_words), free_rows, rank, columns,
                                  reinterpret_cast<const uint32_t *>(payload),
                                  reinterpret_cast<const uint32_t *>(codebook),
                                  reinterpret_cast<uint32_t *>(words_out), reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_mixed_v_tiles_bytes(int64_t rank, int64_t in_features, int64_t free_rows, size_t *bytes) {
  if (bytes == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (free_rows <= 0 || free_rows >= rank || in_features <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "mixed-V free rows must be between zero and rank");
  *bytes = mixed_v_tiles_bytes(rank, in_features, free_rows);
  return ok();
}

int nqb_repack_mixed_v(const int32_t *payload, int64_t rank, int64_t in_features, int64_t free_rows, void *out,
                       void *stream) {
  if (payload == nullptr || out == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "mixed-V operand is NULL");
  if (free_rows <= 0 || free_rows >= rank || in_features <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "mixed-V free rows must be between zero and rank");
  if (!aligned(out, 16)) return fail(NQB_ERR_ALIGNMENT, "coded tiles must be 16-byte aligned");
  NQB_CHECK(launch_repack_mixed_v(reinterpret_cast<const uint32_t *>(payload), rank, in_features, free_rows,
                                  static_cast<uint8_t *>(out), reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

int nqb_product_codebook_tiles_bytes(int64_t rank, int64_t in_features, int64_t free_rows, size_t *bytes) {
  if (bytes == nullptr) return fail(NQB_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (free_rows <= 0 || free_rows >= rank || in_features <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "product-codebook free rows must be between zero and rank");
  *bytes = product_codebook_tiles_bytes(rank, in_features, free_rows);
  return ok();
}

int nqb_repack_product_codebook(const int32_t *payload, const int16_t *first, const int16_t *second,
                                int64_t rank, int64_t in_features, int64_t free_rows, void *tiles_out,
                                int32_t *table_out, void *stream) {
  if (payload == nullptr || first == nullptr || second == nullptr || tiles_out == nullptr || table_out == nullptr)
    return fail(NQB_ERR_INVALID_ARGUMENT, "product-codebook operand is NULL");
  if (free_rows <= 0 || free_rows >= rank || in_features <= 0)
    return fail(NQB_ERR_INVALID_ARGUMENT, "product-codebook free rows must be between zero and rank");
  if (!aligned(tiles_out, 16) || !aligned(table_out, 16))
    return fail(NQB_ERR_ALIGNMENT, "coded tiles and table must be 16-byte aligned");
  NQB_CHECK(launch_repack_product_codebook(
      reinterpret_cast<const uint16_t *>(payload), reinterpret_cast<const uint16_t *>(first),
      reinterpret_cast<const uint16_t *>(second), rank, in_features, free_rows, static_cast<uint8_t *>(tiles_out),
      reinterpret_cast<uint32_t *>(table_out), reinterpret_cast<cudaStream_t>(stream)));
  return ok();
}

}  // extern "C"
