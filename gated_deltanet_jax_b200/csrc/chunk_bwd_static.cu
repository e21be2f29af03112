// Fixed scratch for the allocation-free backward (gdn_chunk_bwd_noalloc).
//
// The backward needs device scratch (gdn_chunk_bwd_workspace_bytes): the
// state entering and the state gradient leaving every chunk, four per-chunk
// products, and per-value-head dq / dk for grouped heads.  gdn_chunk_bwd takes
// that scratch from the caller.  Some callers cannot hand it over or allocate
// it: a host framework that owns the device memory and gives the call no
// scratch (XLA reserves most of HBM for its own pool, so a cudaMalloc inside
// one of its custom calls can fail or fragment memory), or a loop that must
// not stop for cudaMalloc, which can synchronise the device.
// For them the scratch lives here, in one array of this library's own device
// memory, reserved when the CUDA driver loads this file's code on a GPU and
// held until the process exits.  This file must stay a module of its own (no
// relocatable device code): under CUDA's default lazy loading the array is
// then reserved only on GPUs where this entry point is called.
//
// This file only holds the array and finds its device address; the kernels
// are gdn_chunk_bwd's own, given that address as their workspace.
#include <atomic>
#include <cstddef>

#include <cuda_runtime.h>

#include "gdn.h"

namespace gdn {

namespace {

// Device memory, one copy per GPU.  In host code this name is a host-side
// stand-in for the array, not a device address: only the pointer that
// cudaGetSymbolAddress returns may be given to a kernel.
static __device__ __align__(256) unsigned char g_bwd_scratch[GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES];

constexpr int kCachedDevices = 64;
std::atomic<void*> g_scratch_addr[kCachedDevices] = {};

}  // namespace

// Device address of the scratch array on the current device.  The first call
// on a device looks it up (cudaGetSymbolAddress, which also makes the driver
// load this file's code on that device if it has not yet) and keeps it;
// later calls on that device read the kept value.
cudaError_t chunk_bwd_static_scratch(void** out) {
  *out = nullptr;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool cached = dev >= 0 && dev < kCachedDevices;
  if (cached) {
    void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (p) {
      *out = p;
      return cudaSuccess;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_bwd_scratch);
  if (e != cudaSuccess) return e;
  if (!p) return cudaErrorInvalidSymbol;
  if (cached) g_scratch_addr[dev].store(p, std::memory_order_release);
  *out = p;
  return cudaSuccess;
}

}  // namespace gdn
