// pf_tmap.cu -- tensor-map encoding and the device status word (see pf_tmap.h).
#include <cudaTypedefs.h>

#include <mutex>

#include "pf_common.cuh"
#include "pf_tmap.h"

namespace pf {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;
static cudaError_t g_encode_err = cudaSuccess;

static void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
}

int make_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swz) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode)
    return fail(PF_ECUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(g_encode_err));
  if (((uintptr_t)base) % 16 != 0) return fail(PF_EINVAL_SHAPE, "TMA base address not 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] % 16 != 0)
      return fail(PF_EINVAL_SHAPE, "TMA stride %d (%llu bytes) not a multiple of 16", i,
                  (unsigned long long)strides_bytes[i]);
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), (const cuuint64_t*)dims,
                        (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PF_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return PF_OK;
}

static __device__ unsigned int g_device_status;

int device_status_ptr(unsigned int** out) {
  void* p = nullptr;
  PF_CUDA_TRY(cudaGetSymbolAddress(&p, g_device_status));
  *out = (unsigned int*)p;
  return PF_OK;
}

static thread_local int g_sm_reserve = 0;

void set_sm_reserve(int r) { g_sm_reserve = r < 0 ? 0 : r; }
int sm_reserve() { return g_sm_reserve; }

int64_t device_sm_count() {
  static std::atomic<int> n[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int v = n[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (v <= 0) v = 148;
    n[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// The persistent kernels' grid: every SM, less the ones this thread reserved for a band copy
// that runs beside them (pf_set_option(PF_OPT_SM_RESERVE, r)).
int64_t sm_count() {
  const int64_t v = device_sm_count() - g_sm_reserve;
  return v < 1 ? 1 : v;
}

int current_device(int* dev) {
  PF_CUDA_TRY(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= 64) return fail(PF_EUNSUPPORTED, "device ordinal %d out of range (< 64)", *dev);
  return PF_OK;
}

}  // namespace pf

extern "C" PF_API int pf_device_status(int* status_out, int clear) {
  using namespace pf;
  if (!status_out) return fail(PF_EINVAL_ARG, "status_out is NULL");
  unsigned int v = 0;
  PF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)));
  if (clear) {
    unsigned int z = 0;
    PF_CUDA_TRY(cudaMemcpyToSymbol(g_device_status, &z, sizeof(z)));
  }
  *status_out = (int)v;
  return PF_OK;
}

extern "C" PF_API int pf_device_status_async(unsigned int* dst, void* stream) {
  using namespace pf;
  if (!dst) return fail(PF_EINVAL_ARG, "dst is NULL");
  PF_CUDA_TRY(cudaMemcpyFromSymbolAsync(dst, g_device_status, sizeof(unsigned int), 0, cudaMemcpyDefault,
                                        (cudaStream_t)stream));
  return PF_OK;
}
