// pf_peer.cu -- peer-memory windows and the region gather of the Fold-CP band exchange.
//
// On one NVLink / NVSwitch node every GPU can load from every other GPU's memory. A Fold-CP
// rank publishes a snapshot of its pair tile into a window (a cudaMalloc'd buffer exported
// with a CUDA IPC handle); after a stream-ordered barrier every rank copies the parts of the
// peers' tiles that its bands need straight out of their windows with one kernel launch
// (pf_copy_regions), instead of point-to-point send/receive pairs plus packing and unpacking
// copies on both sides. The loads are plain vectorised global loads; nothing here uses TMA.
//
// Regions are 2D byte rectangles (rows x row_bytes with independent source / destination
// pitches): the intersection of a band with a tile is one such rectangle because a tile row is
// contiguous over its columns and channels.

#include <string.h>

#include "pf_common.cuh"
#include "pf_prof.h"

namespace pf {
namespace {

struct RegionSet {
  pf_copy_region r[PF_MAX_COPY_REGIONS];
  int64_t row_start[PF_MAX_COPY_REGIONS + 1];  // prefix sums of rows (work items)
  int32_t n;
};

// One work item = one row of one region; the CTA's threads stride over that row's vectors,
// each thread keeping kUnroll loads in flight before it stores (peer loads cross NVLink and
// need many bytes in flight per SM to reach link bandwidth).
template <class V>
__global__ void __launch_bounds__(256) k_copy_regions(const __grid_constant__ RegionSet rs) {
  constexpr int kUnroll = 4;
  const int64_t items = rs.row_start[rs.n];
  int reg = 0;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    while (it >= rs.row_start[reg + 1]) ++reg;  // items are visited in increasing order
    const pf_copy_region& R = rs.r[reg];
    const int64_t row = it - rs.row_start[reg];
    const V* __restrict__ src = reinterpret_cast<const V*>((const char*)R.src + row * R.src_pitch);
    V* __restrict__ dst = reinterpret_cast<V*>((char*)R.dst + row * R.dst_pitch);
    const int64_t nv = R.row_bytes / (int64_t)sizeof(V);
    int64_t v = threadIdx.x;
    for (; v + (kUnroll - 1) * (int64_t)blockDim.x < nv; v += kUnroll * (int64_t)blockDim.x) {
      V t[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) t[u] = src[v + u * blockDim.x];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) dst[v + u * blockDim.x] = t[u];
    }
    for (; v < nv; v += blockDim.x) dst[v] = src[v];
  }
}

int widest_unit(const pf_copy_region* r, int n) {
  uintptr_t acc = 0;
  for (int i = 0; i < n; ++i)
    acc |= (uintptr_t)r[i].src | (uintptr_t)r[i].dst | (uintptr_t)r[i].row_bytes |
           (uintptr_t)r[i].src_pitch | (uintptr_t)r[i].dst_pitch;
  if ((acc & 15) == 0) return 16;
  if ((acc & 7) == 0) return 8;
  if ((acc & 3) == 0) return 4;
  return 1;
}

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" PF_API size_t pf_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" PF_API int pf_peer_window_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  if (ptr_out == nullptr || handle_out == nullptr) return fail(PF_EINVAL_ARG, "null output pointer");
  if (bytes == 0) return fail(PF_EINVAL_ARG, "window of 0 bytes");
  void* p = nullptr;
  PF_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(PF_ECUDA, "cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return PF_OK;
}

extern "C" PF_API int pf_peer_window_free(void* ptr) {
  if (ptr == nullptr) return fail(PF_EINVAL_ARG, "null window");
  PF_CUDA_TRY(cudaFree(ptr));
  return PF_OK;
}

extern "C" PF_API int pf_peer_window_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return fail(PF_EINVAL_ARG, "null handle or output pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  PF_CUDA_TRY(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return PF_OK;
}

extern "C" PF_API int pf_peer_window_close(void* ptr) {
  if (ptr == nullptr) return fail(PF_EINVAL_ARG, "null window");
  PF_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return PF_OK;
}

extern "C" PF_API int pf_copy_regions(const pf_copy_region* regions, int32_t n_regions, void* stream) {
  if (n_regions < 0 || n_regions > PF_MAX_COPY_REGIONS)
    return fail(PF_EINVAL_ARG, "n_regions %d outside [0, %d]", n_regions, PF_MAX_COPY_REGIONS);
  if (n_regions > 0 && regions == nullptr) return fail(PF_EINVAL_ARG, "null region list");
  RegionSet rs;
  memset(&rs, 0, sizeof(rs));
  int n = 0;
  rs.row_start[0] = 0;
  for (int i = 0; i < n_regions; ++i) {
    const pf_copy_region& r = regions[i];
    if (r.rows < 0 || r.row_bytes < 0) return fail(PF_EINVAL_SHAPE, "region %d: negative size", i);
    if (r.rows == 0 || r.row_bytes == 0) continue;
    if (r.src == nullptr || r.dst == nullptr) return fail(PF_EINVAL_ARG, "region %d: null pointer", i);
    if (r.rows > 1 && (r.src_pitch < r.row_bytes || r.dst_pitch < r.row_bytes))
      return fail(PF_EINVAL_SHAPE, "region %d: pitch smaller than the row", i);
    rs.r[n] = r;
    rs.row_start[n + 1] = rs.row_start[n] + r.rows;
    ++n;
  }
  rs.n = n;
  if (n == 0) return PF_OK;
  for (int i = n + 1; i <= PF_MAX_COPY_REGIONS; ++i) rs.row_start[i] = rs.row_start[n];
  int dev = 0, sms = 0;
  PF_CUDA_TRY(cudaGetDevice(&dev));
  PF_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t items = rs.row_start[n];
  const int grid = (int)(items < (int64_t)sms * 4 ? items : (int64_t)sms * 4);
  cudaStream_t st = (cudaStream_t)stream;
  PF_LAUNCH_SCOPE(st, "k_copy_regions");
  switch (widest_unit(rs.r, n)) {
    case 16: k_copy_regions<uint4><<<grid, 256, 0, st>>>(rs); break;
    case 8: k_copy_regions<uint2><<<grid, 256, 0, st>>>(rs); break;
    case 4: k_copy_regions<uint32_t><<<grid, 256, 0, st>>>(rs); break;
    default: k_copy_regions<unsigned char><<<grid, 256, 0, st>>>(rs); break;
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}
