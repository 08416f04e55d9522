// qg_noalloc.cu -- qg_layer_slice_forward_static: the mixed-format layer slice with its
// intermediates in a fixed, file-scope device array instead of a caller workspace.
//
// Some callers cannot hand the slice a workspace:
//  * a plugin host that passes only weights, activations and a stream, with no hook
//    for device memory, so the plugin would have to allocate behind the host's back;
//  * a serving process whose allocator has already reserved nearly all of HBM for
//    weights and KV pages, where one more cudaMalloc fails or fragments the pool;
//  * a latency-critical decode loop, where cudaMalloc/cudaFree can synchronise the
//    device and stall the stream the step runs on.
// For them the scratch is linked into the library: QG_SLICE_STATIC_SCRATCH_BYTES per
// device, reserved when the module loads, never allocated or freed by this code.
//
// Set-up: the first call on each device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and caches it.  That lookup may
// load the module, so the first call on a device should come before any stream
// capture.  Later calls do no CUDA API work besides the slice's own launches.
//
// Nothing in the scratch needs to start at zero: every intermediate vector and every
// activation plane buffer is fully written by one launch before a later launch reads it.
//
// There is one scratch per device: calls whose launches overlap on the device (two
// streams, two host threads, or a second call enqueued on another stream before the
// first finishes) race on it.  Serialise them on one stream, or use
// qg_layer_slice_forward with a workspace per concurrent caller.
#include <atomic>
#include <mutex>

#include "qg_host.h"

namespace {

constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_slice_scratch[QG_SLICE_STATIC_SCRATCH_BYTES];

std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mutex;

// Device address of g_slice_scratch on the current device (looked up once per device).
cudaError_t scratch_for_current_device(void** ptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      e = cudaGetSymbolAddress(&p, g_slice_scratch);
      if (e != cudaSuccess) return e;
      if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255u) != 0u) return cudaErrorInvalidSymbol;
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *ptr = p;
  return cudaSuccess;
}

}  // namespace

extern "C" cudaError_t qg_layer_slice_forward_static(const qg_layer_slice* s, const float* x,
                                                     float* out, cudaStream_t stream) {
  size_t need = 0;
  // validates s (dims, formats, pointers) exactly as qg_layer_slice_forward does
  cudaError_t e = qg_layer_slice_workspace_bytes(s, &need);
  if (e != cudaSuccess) return e;
  if (need > QG_SLICE_STATIC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  if (x == nullptr || out == nullptr) return cudaErrorInvalidValue;
  void* scratch = nullptr;
  e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return e;
  return qg_layer_slice_forward(s, x, out, scratch, stream);
}
