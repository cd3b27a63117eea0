// NVFP4 export that allocates nothing: pq_nvfp4_pack_noalloc.
//
// pq_nvfp4_pack needs two scratch buffers from its caller (the bf16 amax of
// every 16-group and one running max per slice).  Some callers cannot provide
// them: programs whose device memory is already handed out to another
// allocator's pool, plug-in hosts whose contract forbids device allocations,
// and code that must not risk the device-wide synchronisation a cudaMalloc can
// cause.  For them this variant keeps its scratch in a file-scope device array
// of fixed size, reserved once per GPU when the library's device code is
// loaded and held until the process exits.
//
// Limits and sharing:
//  * at most NOALLOC_MAX_GROUPS 16-element groups per call
//    (batch * rows * cols <= 134,217,728 elements) and at most 256 slices;
//  * every call on a device uses the same array, which keeps the previous
//    call's contents: the per-slice maxima are cleared at the start of each
//    call (the group amax is fully rewritten), and calls that overlap on the
//    GPU (different streams, or several host threads) race on the array.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture on that device.  The address is kept for the
//    life of the process: do not call this entry point on a device after a
//    cudaDeviceReset (or any re-creation of its primary context) in the same
//    process, since the kept address would then be stale.
//
// This file is part of the single translation unit pq_lib.cu and uses the
// launchers and helpers of pq_pack.cu / pq_capi.cu unchanged.
#include <mutex>

#include "pq_common.cuh"
#include "pq_internal.h"

namespace pq {

constexpr int64_t NOALLOC_MAX_GROUPS = 8 * 1024 * 1024;   // 16 MiB of bf16 group amax
constexpr int NOALLOC_MAX_SLICES = MAX_SCALE_SLICES;      // 256 per-slice maxima (1 KiB)

static __device__ __align__(256) uint16_t g_noalloc_amax[NOALLOC_MAX_GROUPS];
static __device__ __align__(256) uint32_t g_noalloc_tmax[NOALLOC_MAX_SLICES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
uint16_t* g_noalloc_amax_ptr[kMaxDevices] = {};
uint32_t* g_noalloc_tmax_ptr[kMaxDevices] = {};

// Device addresses of the two arrays on the current device (looked up once per
// device; the host-side names are only stand-ins and never go to a kernel).
int noalloc_scratch(uint16_t** amax, uint32_t** tmax) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return PQ_ERR_LIMIT;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_amax_ptr[dev] == nullptr) {
    void* a = nullptr;
    void* t = nullptr;
    e = cudaGetSymbolAddress(&a, g_noalloc_amax);
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaGetSymbolAddress(&t, g_noalloc_tmax);
    if (e != cudaSuccess) return cuda_status(e);
    g_noalloc_amax_ptr[dev] = static_cast<uint16_t*>(a);
    g_noalloc_tmax_ptr[dev] = static_cast<uint32_t*>(t);
  }
  *amax = g_noalloc_amax_ptr[dev];
  *tmax = g_noalloc_tmax_ptr[dev];
  return PQ_OK;
}

}  // namespace
}  // namespace pq

extern "C" int pq_nvfp4_pack_noalloc(const uint16_t* w, int64_t batch, int64_t rows, int64_t cols,
                                     const float* override_dev, uint8_t* codes, uint8_t* scales, float* global_div,
                                     void* stream_) {
  if (batch < 0 || rows < 0 || cols < 1) return PQ_ERR_SHAPE;
  if (cols % 16) return PQ_ERR_SHAPE;
  if (batch == 0) return PQ_OK;
  if (batch > pq::NOALLOC_MAX_SLICES) return PQ_ERR_LIMIT;
  const int64_t groups_per_row = cols / 16;
  // compared by division, so that no product of the caller's sizes can overflow
  if (rows > pq::NOALLOC_MAX_GROUPS / groups_per_row / batch) return PQ_ERR_LIMIT;
  const int64_t per_slice = rows * groups_per_row;
  if (!global_div) return PQ_ERR_NULL;
  if (rows > 0 && (!w || !codes || !scales)) return PQ_ERR_NULL;
  uint16_t* amax = nullptr;
  uint32_t* tmax = nullptr;
  int st = pq::noalloc_scratch(&amax, &tmax);
  if (st) return st;
  cudaStream_t stream = (cudaStream_t)stream_;
  // the per-slice maxima must start at zero; the group amax is rewritten in full
  st = cuda_status(cudaMemsetAsync(tmax, 0, (size_t)batch * sizeof(uint32_t), stream));
  if (st) return st;
  // the codes pass of pq_nvfp4_pack, unchanged (the fast sweep kernel's codes-only form where the
  // shape and alignment allow it); with rows == 0 it does nothing and the scale pass still writes
  // each slice's global, as pq_nvfp4_pack does
  st = pq_nvfp4_codes(w, batch, rows, cols, codes, amax, tmax, stream_);
  if (st) return st;
  const uint16_t* am[pq::NOALLOC_MAX_SLICES];
  int64_t ngs[pq::NOALLOC_MAX_SLICES];
  uint8_t* sc[pq::NOALLOC_MAX_SLICES];
  for (int b = 0; b < (int)batch; ++b) {
    am[b] = amax + b * per_slice;
    ngs[b] = per_slice;
    sc[b] = scales ? scales + b * per_slice : nullptr;
  }
  return pq_nvfp4_scales((int)batch, am, ngs, tmax, nullptr, override_dev, sc, global_div, stream_);
}
