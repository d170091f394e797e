// sqb_bwd_noalloc: the backward entry point for callers that cannot allocate.
//
// Some callers of this library cannot call cudaMalloc at the point where they run
// the attention backward: their device memory is owned by another component (a
// serving runtime's fixed arena, or a framework allocator that is not reachable
// through a C ABI), or they must not grow the device footprint after start-up.
// They still own their inputs and outputs, but cannot provide the scratch
// workspace sqb_bwd asks for.  This entry point takes the same arguments as
// sqb_bwd minus the workspace and uses scratch that the library itself holds:
// one file-scope __device__ array of kNoAllocScratchBytes, created when the
// library is loaded on a GPU and held until the process exits.
//
// Behaviour:
//  * Problems whose workspace (sqb_workspace_bytes) exceeds the array are
//    rejected with SQB_ERR_WORKSPACE before anything is launched.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (the host-side symbol is only a stand-in, not a
//    device pointer).  Make that first call before any stream capture.
//  * Every call clears the part of the array it uses (cudaMemsetAsync, no
//    allocation) and then runs the regular backward on it - all but the two
//    status words: a device-side failure (a bounded wait that gave up) stays
//    recorded until sqb_read_status_noalloc reads and clears it, so the next
//    call does not wipe it.  Until then later calls give up their waits on
//    other work tiles at once, and their results are wrong too.
//  * All calls on a device share the array, so calls that overlap on the GPU
//    (different streams, or host threads without ordering) race on it and
//    must not be issued; calls ordered on one stream are fine.
//  * It calls no cudaMalloc, cudaFree or allocating library routine.

#include <mutex>

#include "sqb_internal.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per GPU
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// CUDA errors of the address lookup that mean the library has no code for
// this GPU (no sm_100a image), reported like sqb_bwd reports such a device.
int lookup_error(cudaError_t e) {
  cudaGetLastError();  // the lookup's error is not left behind for the caller
  return (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction ||
          e == cudaErrorInvalidDevice)
             ? SQB_ERR_DEVICE
             : SQB_ERR_CUDA;
}

// Device address of the scratch array on the current device (set up once).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return lookup_error(e);
  if (dev < 0 || dev >= kMaxDevices) return SQB_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch)) return lookup_error(e);
    if (!p) return SQB_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SQB_OK;
}

}  // namespace

extern "C" int sqb_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                               const void* dout, const float* lse, const void* kbar,
                               const void* vbar, void* dq, void* dk, void* dv, int64_t B,
                               int64_t T, int64_t H, int64_t D, int64_t block,
                               const int64_t* strides, int dtype, float scale, int impl,
                               void* stream) {
  const size_t need = sqb_workspace_bytes(B, T, H, D, block);
  if (need == 0) return SQB_ERR_ARG;
  if (need > kNoAllocScratchBytes) return SQB_ERR_WORKSPACE;
  void* scratch = nullptr;
  if (int e = scratch_address(&scratch)) return e;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // clear everything but the status and its detail (control words kStatus and
  // kStatusDetail), which stay until sqb_read_status_noalloc clears them
  uint8_t* base = static_cast<uint8_t*>(scratch);
  const size_t keep_lo = (size_t)sqb::kStatus * 4, keep_hi = (size_t)(sqb::kStatusDetail + 1) * 4;
  if (cudaMemsetAsync(base, 0, keep_lo, s) != cudaSuccess ||
      cudaMemsetAsync(base + keep_hi, 0, need - keep_hi, s) != cudaSuccess)
    return SQB_ERR_CUDA;
  return sqb_bwd(q, k, v, o, dout, lse, kbar, vbar, dq, dk, dv, B, T, H, D, block, strides, dtype,
                 scale, impl, scratch, need, stream);
}

extern "C" int sqb_read_status_noalloc(void* stream, int64_t* detail) {
  void* scratch = nullptr;
  if (int e = scratch_address(&scratch)) return e;
  return sqb_read_status(scratch, stream, detail);
}
