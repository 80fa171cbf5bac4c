// pf_tmap.h -- host-side TMA tensor-map encoding (driver entry point fetched at run time,
// so the library has no link-time dependency on libcuda) and the device status word.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

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
int64_t sm_count();

}  // namespace pf
