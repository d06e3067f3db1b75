// The fixed device scratch of pesti_sample_batch_noalloc and its per-device
// set-up.  The array sits in a translation unit of its own, so it belongs to a
// device module apart from the sampler kernels: with CUDA's lazy module
// loading, a device reserves it only once the no-allocation entry point has
// run there, and callers of the other entry points never do.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "../../include/pesti_sampler.h"
#include "pesti_noalloc.h"

// Every call on a device shares this array and finds the previous call's
// contents in it; the entry point clears what must start at zero.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PESTI_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

struct DeviceSlot {
  std::atomic<bool> ready{false};
  pesti_noalloc_device dev{};
};

DeviceSlot g_slots[kMaxDevices];
std::mutex g_setup_mu;

}  // namespace

cudaError_t pesti_noalloc_setup(int device, pesti_noalloc_device* out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  DeviceSlot& slot = g_slots[device];
  if (!slot.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!slot.ready.load(std::memory_order_relaxed)) {
      pesti_noalloc_device d{};
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, device);
      if (e != cudaSuccess) return e;
      d.scratch = static_cast<char*>(p);
      slot.dev = d;
      slot.ready.store(true, std::memory_order_release);
    }
  }
  *out = slot.dev;
  return cudaSuccess;
}
