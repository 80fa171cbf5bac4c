// pf_peer.cu -- peer-memory windows and the region gather of the Fold-CP band exchange.
//
// On one NVLink / NVSwitch node every GPU can load from every other GPU's memory. A Fold-CP
// rank publishes a snapshot of its pair tile into a window (a cudaMalloc'd buffer exported
// with a CUDA IPC handle); after a stream-ordered barrier every rank copies the parts of the
// peers' tiles that its bands need straight out of their windows with one kernel launch
// (pf_copy_regions), instead of point-to-point send/receive pairs plus packing and unpacking
// copies on both sides. The loads are plain vectorised global loads; nothing here uses TMA.
//
// Regions are byte boxes (planes x rows x row_bytes with independent source / destination
// pitches): the intersection of a band with a pair tile is one plane because a tile row is
// contiguous over its columns and channels; a band of a channel-major projection has one plane
// per channel.

#include <string.h>

#include "pf_common.cuh"
#include "pf_prof.h"
#include "pf_tmap.h"

namespace pf {
namespace {

struct Box {
  const char* src;
  char* dst;
  int64_t src_pitch, dst_pitch, src_plane_pitch, dst_plane_pitch;
  uint32_t rows;   // rows per plane
  uint32_t nv;     // vectors per row
  uint32_t lines;  // planes * rows
  uint32_t lpi;    // lines per work item
};

struct BoxSet {
  Box b[PF_MAX_COPY_REGIONS];
  int64_t item_start[PF_MAX_COPY_REGIONS + 1];  // prefix sums of work items
  int32_t n;
};

// A work item is a run of consecutive lines (plane-major rows) of one box, about 2048 vectors;
// the CTA's threads stride over the run's (line, vector) pairs, each thread keeping kUnroll
// loads in flight before it stores (peer loads cross NVLink and need many bytes in flight per
// SM to reach link bandwidth).
template <class V>
__global__ void __launch_bounds__(256) k_copy_regions(const __grid_constant__ BoxSet bs) {
  constexpr int kUnroll = 4;
  const int64_t items = bs.item_start[bs.n];
  int reg = 0;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    while (it >= bs.item_start[reg + 1]) ++reg;  // items are visited in increasing order
    const Box& B = bs.b[reg];
    const uint32_t line0 = (uint32_t)(it - bs.item_start[reg]) * B.lpi;
    const uint32_t nl = min(B.lpi, B.lines - line0);
    const uint32_t total = nl * B.nv;
    for (uint32_t base = threadIdx.x; base < total; base += kUnroll * blockDim.x) {
      V t[kUnroll];
      V* dst[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const uint32_t e = base + u * blockDim.x;
        dst[u] = nullptr;
        if (e < total) {
          const uint32_t l = e / B.nv, v = e - l * B.nv;
          const uint32_t line = line0 + l;
          const uint32_t plane = line / B.rows, row = line - plane * B.rows;
          const V* src = reinterpret_cast<const V*>(B.src + plane * B.src_plane_pitch + row * B.src_pitch) + v;
          dst[u] = reinterpret_cast<V*>(B.dst + plane * B.dst_plane_pitch + row * B.dst_pitch) + v;
          t[u] = *src;
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (dst[u]) *dst[u] = t[u];
    }
  }
}

int widest_unit(const pf_copy_region* r, int n) {
  uintptr_t acc = 0;
  for (int i = 0; i < n; ++i)
    acc |= (uintptr_t)r[i].src | (uintptr_t)r[i].dst | (uintptr_t)r[i].row_bytes | (uintptr_t)r[i].src_pitch |
           (uintptr_t)r[i].dst_pitch | (uintptr_t)r[i].src_plane_pitch | (uintptr_t)r[i].dst_plane_pitch;
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
  pf_copy_region live[PF_MAX_COPY_REGIONS];
  int n = 0;
  for (int i = 0; i < n_regions; ++i) {
    const pf_copy_region& r = regions[i];
    if (r.planes < 0 || r.rows < 0 || r.row_bytes < 0) return fail(PF_EINVAL_SHAPE, "region %d: negative size", i);
    if (r.planes == 0 || r.rows == 0 || r.row_bytes == 0) continue;
    if (r.src == nullptr || r.dst == nullptr) return fail(PF_EINVAL_ARG, "region %d: null pointer", i);
    if (r.rows > 1 && (r.src_pitch < r.row_bytes || r.dst_pitch < r.row_bytes))
      return fail(PF_EINVAL_SHAPE, "region %d: row pitch smaller than the row", i);
    if (r.planes > 1 && (r.src_plane_pitch < r.rows * r.src_pitch || r.dst_plane_pitch < r.rows * r.dst_pitch))
      return fail(PF_EINVAL_SHAPE, "region %d: plane pitch smaller than the plane", i);
    if (r.planes * r.rows >= (1ll << 31)) return fail(PF_EINVAL_SHAPE, "region %d: more than 2^31 rows", i);
    live[n++] = r;
  }
  if (n == 0) return PF_OK;
  const int unit = widest_unit(live, n);
  BoxSet bs;
  memset(&bs, 0, sizeof(bs));
  bs.n = n;
  bs.item_start[0] = 0;
  for (int i = 0; i < n; ++i) {
    const pf_copy_region& r = live[i];
    const int64_t nv = r.row_bytes / unit;
    if (nv >= (1ll << 31)) return fail(PF_EINVAL_SHAPE, "region %d: row of 2^31 vectors or more", i);
    Box& B = bs.b[i];
    B.src = (const char*)r.src;
    B.dst = (char*)r.dst;
    B.src_pitch = r.src_pitch;
    B.dst_pitch = r.dst_pitch;
    B.src_plane_pitch = r.src_plane_pitch;
    B.dst_plane_pitch = r.dst_plane_pitch;
    B.rows = (uint32_t)r.rows;
    B.nv = (uint32_t)nv;
    B.lines = (uint32_t)(r.planes * r.rows);
    B.lpi = (uint32_t)(nv >= 2048 ? 1 : (2048 + nv - 1) / nv);
    if ((uint64_t)B.lpi * B.nv >= (1ull << 31)) return fail(PF_EINVAL_SHAPE, "region %d: work item too large", i);
    bs.item_start[i + 1] = bs.item_start[i] + (B.lines + B.lpi - 1) / B.lpi;
  }
  for (int i = n + 1; i <= PF_MAX_COPY_REGIONS; ++i) bs.item_start[i] = bs.item_start[n];
  int dev = 0, sms = 0;
  PF_CUDA_TRY(cudaGetDevice(&dev));
  PF_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t items = bs.item_start[n];
  // with an SM reserve set, at most 8 CTAs per reserved SM, so that the copy fits beside the
  // persistent kernels that leave those SMs free
  const int64_t cap = sm_reserve() > 0 ? (int64_t)sm_reserve() * 8 : (int64_t)sms * 4;
  const int grid = (int)(items < cap ? items : cap);
  cudaStream_t st = (cudaStream_t)stream;
  double copied = 0.0;  // bytes copied (each read once from its source, written once)
  for (int i = 0; i < n; ++i) copied += (double)live[i].planes * live[i].rows * live[i].row_bytes;
  PF_LAUNCH_SCOPE_WORK(st, "k_copy_regions", copied, 'b');
  switch (unit) {
    case 16: k_copy_regions<uint4><<<grid, 256, 0, st>>>(bs); break;
    case 8: k_copy_regions<uint2><<<grid, 256, 0, st>>>(bs); break;
    case 4: k_copy_regions<uint32_t><<<grid, 256, 0, st>>>(bs); break;
    default: k_copy_regions<unsigned char><<<grid, 256, 0, st>>>(bs); break;
  }
  PF_CHECK_LAUNCH();
  return PF_OK;
}

// The same regions moved by the copy engines instead of SMs: one 2-D copy per region whose
// planes are evenly spaced rows of one pitch, one 3-D copy when each side's plane pitch is a
// whole number of its row pitches, else one 2-D copy per plane. DMA copies run beside the
// persistent kernels, which hold every SM's shared memory and would otherwise keep an SM copy
// kernel waiting until they finish; so a band copied on a side stream overlaps the compute on
// the main stream. Each copy is one call (no batched copy API).
extern "C" PF_API int pf_copy_regions_dma(const pf_copy_region* regions, int32_t n_regions, void* stream) {
  if (n_regions < 0) return fail(PF_EINVAL_ARG, "n_regions %d < 0", n_regions);
  if (n_regions > 0 && regions == nullptr) return fail(PF_EINVAL_ARG, "null region list");
  cudaStream_t st = (cudaStream_t)stream;
  for (int i = 0; i < n_regions; ++i) {
    const pf_copy_region& r = regions[i];
    if (r.planes < 0 || r.rows < 0 || r.row_bytes < 0) return fail(PF_EINVAL_SHAPE, "region %d: negative size", i);
    if (r.planes == 0 || r.rows == 0 || r.row_bytes == 0) continue;
    if (r.src == nullptr || r.dst == nullptr) return fail(PF_EINVAL_ARG, "region %d: null pointer", i);
    const int64_t sp = r.rows > 1 ? r.src_pitch : r.row_bytes, dp = r.rows > 1 ? r.dst_pitch : r.row_bytes;
    if (sp < r.row_bytes || dp < r.row_bytes) return fail(PF_EINVAL_SHAPE, "region %d: row pitch smaller than the row", i);
    if (r.planes > 1 && (r.src_plane_pitch < r.rows * sp || r.dst_plane_pitch < r.rows * dp))
      return fail(PF_EINVAL_SHAPE, "region %d: plane pitch smaller than the plane", i);
    PF_LAUNCH_SCOPE_WORK(st, "dma_copy_regions", (double)r.planes * r.rows * r.row_bytes, 'b');
    if (r.planes == 1 || (r.src_plane_pitch == r.rows * sp && r.dst_plane_pitch == r.rows * dp)) {
      // the planes are consecutive rows of one 2-D box
      PF_CUDA_TRY(cudaMemcpy2DAsync(r.dst, (size_t)dp, r.src, (size_t)sp, (size_t)r.row_bytes,
                                    (size_t)(r.rows * r.planes), cudaMemcpyDefault, st));
    } else if (r.src_plane_pitch % sp == 0 && r.dst_plane_pitch % dp == 0) {
      cudaMemcpy3DParms p;
      memset(&p, 0, sizeof(p));
      p.srcPtr = make_cudaPitchedPtr(const_cast<void*>(r.src), (size_t)sp, (size_t)r.row_bytes,
                                     (size_t)(r.src_plane_pitch / sp));
      p.dstPtr = make_cudaPitchedPtr(r.dst, (size_t)dp, (size_t)r.row_bytes, (size_t)(r.dst_plane_pitch / dp));
      p.extent = make_cudaExtent((size_t)r.row_bytes, (size_t)r.rows, (size_t)r.planes);
      p.kind = cudaMemcpyDefault;
      PF_CUDA_TRY(cudaMemcpy3DAsync(&p, st));
    } else {
      for (int64_t pl = 0; pl < r.planes; ++pl)
        PF_CUDA_TRY(cudaMemcpy2DAsync((char*)r.dst + pl * r.dst_plane_pitch, (size_t)dp,
                                      (const char*)r.src + pl * r.src_plane_pitch, (size_t)sp, (size_t)r.row_bytes,
                                      (size_t)r.rows, cudaMemcpyDefault, st));
    }
  }
  return PF_OK;
}
