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
// Set-up: a device address of the array is only valid in the CUDA context that was
// current when it was looked up.  Each call reads the current context's process-unique
// id (cuCtxGetCurrent + cuCtxGetId, through the runtime's driver entry points, so the
// library does not link libcuda itself); the first call in a context (the first on
// each device, and the first after cudaDeviceReset or under a different driver-API
// context) looks the address up with cudaGetSymbolAddress and caches it beside that id.
// That lookup may load the module, so the first call in a context should come before
// any stream capture.  Later calls in the same context do no CUDA API work besides the
// id query and the slice's own launches.
//
// Nothing in the scratch needs to start at zero: every intermediate vector and every
// activation plane buffer is fully written by one launch before a later launch reads it.
//
// There is one scratch per device: calls whose launches overlap on the device (two
// streams, two host threads, or a second call enqueued on another stream before the
// first finishes) race on it.  Serialise them on one stream, or use
// qg_layer_slice_forward with a workspace per concurrent caller.
#include <mutex>

#include "qg_ctx_cache.h"
#include "qg_host.h"

namespace {

constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_slice_scratch[QG_SLICE_STATIC_SCRATCH_BYTES];

// Driver-API calls resolved once through cudaGetDriverEntryPoint (signatures of
// cuCtxGetCurrent and cuCtxGetId; CUcontext is an opaque pointer).
using CtxGetCurrentFn = int (*)(void** ctx);
using CtxGetIdFn = int (*)(void* ctx, unsigned long long* id);

std::mutex g_setup_mutex;
qg::CtxAddressCache<kMaxDevices> g_scratch;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

cudaError_t resolve_driver_calls() {
  if (g_ctx_get_current != nullptr && g_ctx_get_id != nullptr) return cudaSuccess;
  void* f0 = nullptr;
  void* f1 = nullptr;
  cudaDriverEntryPointQueryResult q0 = cudaDriverEntryPointSymbolNotFound, q1 = q0;
  cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f0, cudaEnableDefault, &q0);
  if (e != cudaSuccess) return e;
  e = cudaGetDriverEntryPoint("cuCtxGetId", &f1, cudaEnableDefault, &q1);
  if (e != cudaSuccess) return e;
  if (q0 != cudaDriverEntryPointSuccess || q1 != cudaDriverEntryPointSuccess || f0 == nullptr ||
      f1 == nullptr) {
    return cudaErrorNotSupported;
  }
  g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f0);
  g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f1);
  return cudaSuccess;
}

// Device address of g_slice_scratch in the current context (looked up once per context).
cudaError_t scratch_for_current_context(void** ptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  e = resolve_driver_calls();
  if (e != cudaSuccess) return e;
  void* ctx = nullptr;
  if (g_ctx_get_current(&ctx) != 0) return cudaErrorDeviceUninitialized;
  unsigned long long id = 0;
  if (ctx != nullptr && g_ctx_get_id(ctx, &id) != 0) return cudaErrorDeviceUninitialized;
  auto lookup = [](void** p) -> int {
    const cudaError_t le = cudaGetSymbolAddress(p, g_slice_scratch);
    if (le != cudaSuccess) return static_cast<int>(le);
    if (*p == nullptr || (reinterpret_cast<uintptr_t>(*p) & 255u) != 0u) {
      return static_cast<int>(cudaErrorInvalidSymbol);
    }
    return 0;
  };
  if (ctx == nullptr) {
    // No context yet: the lookup makes the device's primary context current; cache the
    // address under that context's id.
    void* p = nullptr;
    const int rc = lookup(&p);
    if (rc != 0) return static_cast<cudaError_t>(rc);
    if (g_ctx_get_current(&ctx) != 0 || ctx == nullptr || g_ctx_get_id(ctx, &id) != 0) {
      return cudaErrorDeviceUninitialized;
    }
  }
  const int rc = g_scratch.get(dev, id, lookup, ptr);
  if (rc < 0) return cudaErrorInvalidDevice;
  return static_cast<cudaError_t>(rc);
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
  e = scratch_for_current_context(&scratch);
  if (e != cudaSuccess) return e;
  return qg_layer_slice_forward(s, x, out, scratch, stream);
}
