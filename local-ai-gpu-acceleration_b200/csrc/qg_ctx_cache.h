// qg_ctx_cache.h -- per-device cache of an address that is valid in one CUDA context.
//
// A device address returned by cudaGetSymbolAddress belongs to the context that was
// current when it was looked up; after cudaDeviceReset, or under another driver-API
// context on the same device, it must be looked up again.  The cache keeps the
// process-unique id of that context (cuCtxGetId) beside the address and calls the
// lookup again whenever the current context's id differs.  Plain host C++ (no CUDA
// headers), so its logic is tested on machines without a GPU.
#pragma once

#include <cstdint>

namespace qg {

template <int kMaxDevices>
struct CtxAddressCache {
  struct Entry {
    unsigned long long ctx_id = 0;
    void* ptr = nullptr;
  };
  Entry entry[kMaxDevices];

  // The address for device `dev` in the context with id `ctx_id`: the cached one when the
  // context is unchanged, else lookup(&ptr) (returns 0 on success).  Returns lookup's
  // error, -1 for a device index out of range, 0 on success.
  template <typename Lookup>
  int get(int dev, unsigned long long ctx_id, Lookup&& lookup, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return -1;
    Entry& e = entry[dev];
    if (e.ptr == nullptr || e.ctx_id != ctx_id) {
      void* p = nullptr;
      const int rc = lookup(&p);
      if (rc != 0) return rc;
      e.ptr = p;
      e.ctx_id = ctx_id;
    }
    *out = e.ptr;
    return 0;
  }
};

}  // namespace qg
