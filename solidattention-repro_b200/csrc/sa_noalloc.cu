// sa_noalloc.cu -- packed GQA decode attention for callers that cannot
// allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at the point where they
// need attention: a serving process that reserved all free HBM for its KV
// pool up front, a decode loop where an allocation's implicit device
// synchronisation is not acceptable, or a foreign-language host (cgo, JNI,
// ctypes) that has no device allocator to hand. sa_attention_packed needs a
// caller-provided workspace for its split-K partials and arrival counters;
// sa_attention_packed_noalloc instead uses the fixed array below, which every
// GPU that loads the library holds until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "sa_internal.h"

namespace {

// Split-K scratch of sa_attention_packed_noalloc: 2 MiB per device. Calls
// whose workspace (sa_attention_workspace_size) would exceed it are refused.
constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device (host code cannot use the
// symbol itself as a device pointer).
void* g_scratch_address[sa::kMaxDevices];
std::mutex g_scratch_mutex;

// The array's device address on the current device. Outside a stream
// capture it is looked up on every call (cheap once the module is loaded),
// so a device reset or a new primary context never leaves a stale address
// behind; while `stream` is capturing, the address of the last uncaptured
// call on this device is used, and a device that has had none is refused.
sa_status scratch_address_for_current_device(cudaStream_t stream, void** out) {
  int device = 0;
  SA_CUDA_TRY(cudaGetDevice(&device));
  if (device < 0 || device >= sa::kMaxDevices)
    return sa::fail(SA_ERR_UNSUPPORTED, "attention_noalloc: device index above 63");
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  SA_CUDA_TRY(cudaStreamIsCapturing(stream, &capture));
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (capture == cudaStreamCaptureStatusNone) {
    void* address = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (err != cudaSuccess)
      return sa::cuda_status(err, "cudaGetSymbolAddress(no-alloc attention scratch)");
    g_scratch_address[device] = address;
  } else if (!g_scratch_address[device]) {
    return sa::fail(SA_ERR_INVALID_ARG,
                    "attention_noalloc: make a first call on this device before stream capture");
  }
  *out = g_scratch_address[device];
  return SA_OK;
}

}  // namespace

extern "C" SA_API sa_status sa_attention_packed_noalloc(const uint16_t* kv, const float* query,
                                                        size_t tokens, size_t query_heads,
                                                        size_t kv_heads, size_t head_dim,
                                                        float scale, void* out, int out_fp16,
                                                        void* stream) {
  if (!kv || !query || !out) return sa::fail(SA_ERR_INVALID_ARG, "attention_noalloc: null pointer");
  if (kv_heads == 0 || query_heads % kv_heads != 0 || tokens == 0)
    return sa::fail(SA_ERR_INVALID_ARG, "invalid GQA attention dimensions");
  const size_t need = sa_attention_workspace_size(tokens, query_heads, kv_heads);
  if (need > kNoAllocScratchBytes)
    return sa::fail(SA_ERR_CAPACITY,
                    "attention_noalloc: this problem needs " + std::to_string(need) +
                        " bytes of scratch, above the 2 MiB static array; use "
                        "sa_attention_packed with a caller workspace");
  void* scratch = nullptr;
  const sa_status st =
      scratch_address_for_current_device(static_cast<cudaStream_t>(stream), &scratch);
  if (st != SA_OK) return st;
  // The same kernel as sa_attention_packed, with the static array as its
  // workspace; that call clears the arrival counters before launching.
  return sa_attention_packed(kv, query, tokens, query_heads, kv_heads, head_dim, scale, out,
                             out_fp16, scratch, kNoAllocScratchBytes, stream);
}
