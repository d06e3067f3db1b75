// Per-device set-up of the static scratch that pesti_sample_batch_noalloc
// (include/pesti_sampler.h) runs in.  Internal to the library.
#pragma once
#include <cuda_runtime.h>

struct pesti_noalloc_device {
  char* scratch;  // device address of the static scratch array on this device
  int num_sms;
  int cc_major;
};

// Returns the scratch address and device properties of `device`, which must be
// the calling thread's current device.  The first call for a device looks the
// array up with cudaGetSymbolAddress (which loads the array's module there);
// later calls return the cached values.
__attribute__((visibility("hidden"))) cudaError_t pesti_noalloc_setup(int device,
                                                                      pesti_noalloc_device* out);
