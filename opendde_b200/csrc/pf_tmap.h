// pf_tmap.h -- host-side TMA tensor-map encoding (driver entry point fetched at run time,
// so the library has no link-time dependency on libcuda) and the device status word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace pf {

// Encode a tiled tensor map. dims[0] is the contiguous dim; strides_bytes has rank-1
// entries (byte stride of dims 1..rank-1). Out-of-bounds elements read as zero.
int make_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swz);

// Process-wide device status word (bit 0: a bounded device-side wait timed out). Lives
// in a static __device__ variable of the current device; returns its device address.
int device_status_ptr(unsigned int** out);

// Number of SMs of the current device (persistent grids are sized by it).
int64_t sm_count();         // SMs for persistent grids (less the reserve of the calling thread)
int64_t device_sm_count();  // all SMs of the current device
void set_sm_reserve(int r);
int sm_reserve();

// Ordinal of the current device, checked against the per-device tables (< 64).
int current_device(int* dev);

// Runs `fn` (returning a pf_status) once per device, with that device current. Kernel
// attributes such as the dynamic shared-memory limit are per device, so a process that drives
// several GPUs needs them set on each. Thread-safe: racing first calls may both run `fn`,
// which only repeats idempotent attribute settings.
template <class F>
int once_per_device(std::atomic<unsigned long long>& done, F&& fn) {
  int dev = 0;
  int st = current_device(&dev);
  if (st != 0) return st;
  const unsigned long long bit = 1ull << dev;
  if (done.load(std::memory_order_acquire) & bit) return 0;
  st = fn();
  if (st != 0) return st;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return 0;
}

}  // namespace pf
