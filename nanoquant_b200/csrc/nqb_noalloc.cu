// nqb_linear_noalloc: nqb_linear for callers that may not allocate device memory.
//
// Some hosts own every byte of device memory themselves: an inference engine
// that runs this operator as a plugin inside its own graph executor, or a
// serving process with a fixed, pre-planned memory budget.  Such a caller
// cannot call cudaMalloc (it would bypass the host's accounting, and a
// synchronising allocation would stall or break its stream capture), and it
// may have no workspace of its own to lend.  For them this entry point takes
// its scratch from a fixed array in the library's own device image, so a call
// needs only the inputs and the output.
#include <mutex>

#include "nqb_common.cuh"
#include "nqb_decode_tc.cuh"

namespace {

// Scratch size: enough for nqb_linear's workspace at decode sizes (e.g. a
// 12288 -> 4096 layer at rank 3072 needs 0.25 MiB for one token and about
// 4 MiB for 16).
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(8) << 20;  // 8 MiB per device

// In host code this name is only a host-side stand-in for the device array;
// its device address comes from cudaGetSymbolAddress below.  Every GPU that
// loads the library keeps these 8 MiB until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_lock;
void *g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached.
int scratch_address(void **out) {
  int device = 0;
  NQB_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices)
    return nqb::fail(NQB_ERR_UNSUPPORTED, "nqb_linear_noalloc supports device ordinals below %d", kMaxDevices);
  std::lock_guard<std::mutex> guard(g_scratch_lock);
  if (g_scratch_address[device] == nullptr) {
    void *address = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (err != cudaSuccess) return nqb::cuda_status(err, "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch_address[device] = address;
  }
  *out = g_scratch_address[device];
  return NQB_OK;
}

}  // namespace

extern "C" int nqb_linear_noalloc(const nqb_linear_desc *layer, const void *x, int32_t x_dtype, int64_t tokens,
                                  float *y, void *stream) {
  size_t needed = 0;
  NQB_CHECK(nqb_linear_workspace_bytes(layer, tokens, &needed));
  if (needed > kNoAllocScratchBytes)
    return nqb::fail(NQB_ERR_WORKSPACE,
                     "nqb_linear_noalloc: this call needs %zu bytes of scratch but the static scratch holds %zu; "
                     "use nqb_linear with a caller-provided workspace",
                     needed, kNoAllocScratchBytes);
  void *scratch = nullptr;
  NQB_CHECK(scratch_address(&scratch));
  // The shared array is handed over as nqb_linear's workspace.  Its first
  // kCounterRegionBytes hold completion counters that must be zero when a call
  // starts; nqb_linear leaves them zero, but a call that overlapped another one
  // on the GPU or gave up a bounded wait may not have, and no caller can reach
  // this array to repair it.  So every call zeroes them first, on its stream
  // (a memset, no allocation); the rest of the array is written before it is read.
  NQB_CUDA(cudaMemsetAsync(scratch, 0, nqb::kCounterRegionBytes, static_cast<cudaStream_t>(stream)),
           "zeroing the no-alloc scratch counters");
  return nqb_linear(layer, x, x_dtype, tokens, y, scratch, kNoAllocScratchBytes, stream);
}
