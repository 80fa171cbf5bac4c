// pf_noalloc.cu -- pf_trimul_fwd_static_scratch: the triangle multiplicative update for
// callers that cannot allocate device memory.
//
// Some hosts of this library cannot hand it a workspace: a plugin running inside another
// runtime that owns every device allocation (and forbids cudaMalloc/cudaFree between its
// steps because they synchronise the device and fragment its pool), or a thin foreign-language
// binding that only receives the pointers of its inputs and outputs. For them this entry point
// takes its scratch from a fixed array compiled into the library instead of from the caller.
//
// The array is a file-scope __device__ variable, so every GPU that loads the library reserves
// PF_STATIC_SCRATCH_BYTES for the life of the process. Its symbol is a host-side stand-in:
// the device address is obtained once per device with cudaGetSymbolAddress (the first call on
// each device does this, with that device current, so make that first call before any stream
// capture begins). All calls share the one array and it keeps whatever the previous call left
// in it; the trimul kernels overwrite every scratch element they read, so nothing needs to be
// cleared. Calls whose GPU work overlaps (different streams, or concurrent host threads on
// one device) race on the array and must be serialised by the caller.

#include <mutex>

#include "pf_common.cuh"

namespace pf {
namespace {

constexpr size_t kScratchBytes = PF_STATIC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_static_scratch[PF_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once per device).
int scratch_ptr(void** out) {
  int dev = 0;
  PF_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(PF_EUNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess)
      return fail(PF_ECUDA, "cudaGetSymbolAddress(static scratch) failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PF_OK;
}

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" PF_API size_t pf_static_scratch_bytes(void) { return kScratchBytes; }

extern "C" PF_API int pf_trimul_fwd_static_scratch(const pf_trimul_params* w, pf_pair_view za,
                                                   pf_pair_view zb, pf_mask_view ma, pf_mask_view mb,
                                                   pf_pair_view zg, pf_pair_view zo, int64_t n_i,
                                                   int64_t n_j, int64_t n_k, int32_t c_z, int32_t c_h,
                                                   int32_t accumulate, int32_t dtype, void* stream) {
  size_t need = 0;
  PF_TRY(pf_trimul_workspace_size(n_i, n_j, n_k, c_z, c_h, dtype, &need));
  if (need > kScratchBytes)
    return fail(PF_EINVAL_SHAPE,
                "pf_trimul_fwd_static_scratch: this problem needs %zu bytes of scratch, more than the "
                "library's fixed %zu-byte array (n_i=%lld n_j=%lld n_k=%lld c_z=%d c_h=%d); use "
                "pf_trimul_fwd with a caller-provided workspace",
                need, kScratchBytes, (long long)n_i, (long long)n_j, (long long)n_k, c_z, c_h);
  void* scratch = nullptr;
  PF_TRY(scratch_ptr(&scratch));
  return pf_trimul_fwd(w, za, zb, ma, mb, zg, zo, n_i, n_j, n_k, c_z, c_h, accumulate, dtype, scratch,
                       kScratchBytes, stream);
}
