// pf_common.cuh -- shared host/device helpers for the pairformer_b200 library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>

#include "../../include/pairformer_b200.h"

namespace pf {

// ---------------------------------------------------------------- host error plumbing
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
void set_path(const char* p);
bool force_simt();

#define PF_CUDA_TRY(expr)                                                            \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess)                                                           \
      return ::pf::fail(PF_ECUDA, "%s failed: %s (%s:%d)", #expr,                    \
                        cudaGetErrorString(_e), __FILE__, __LINE__);                 \
  } while (0)

#define PF_CHECK_LAUNCH()                                                            \
  do {                                                                               \
    cudaError_t _e = cudaGetLastError();                                             \
    if (_e != cudaSuccess)                                                           \
      return ::pf::fail(PF_ECUDA, "kernel launch failed: %s (%s:%d)",                \
                        cudaGetErrorString(_e), __FILE__, __LINE__);                 \
  } while (0)

#define PF_TRY(expr)                                                                 \
  do {                                                                               \
    int _s = (expr);                                                                 \
    if (_s != PF_OK) return _s;                                                      \
  } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// A bump allocator over the caller's workspace (no device allocation).
struct Arena {
  char* base;
  size_t cap;
  size_t used = 0;
  bool counting;  // true => only measure
  Arena(void* b, size_t c) : base((char*)b), cap(c), counting(b == nullptr) {}
  template <class T>
  T* take(size_t n) {
    size_t off = align_up(used, 256);
    used = off + n * sizeof(T);
    if (counting) return nullptr;
    return (T*)(base + off);
  }
  bool ok() const { return counting || used <= cap; }
};

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
template <class T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
// accurate variants for the fp32 mode
__device__ __forceinline__ float sigmoid_acc(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_acc(float x) { return x / (1.0f + expf(-x)); }

}  // namespace pf
