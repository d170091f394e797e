// extern "C" entry points of the sqrt-block attention library (include/sqrtblock.h):
// argument checks, geometry, workspace layout and kernel-family dispatch.

#include <math.h>
#include <string.h>

#include "sqb_internal.cuh"
#include "sqb_sm100.cuh"

namespace sqb {
namespace {

// b = round_up(ceil(sqrt(T)), 16), with ceil(sqrt(T)) = isqrt(T - 1) + 1.
int64_t default_block(int64_t T) {
  int64_t r = (int64_t)sqrt((double)(T - 1));
  while (r > 0 && r * r > T - 1) --r;
  while ((r + 1) * (r + 1) <= T - 1) ++r;
  return (r + 1 + 15) / 16 * 16;
}

bool elt_size(int dtype, int* sz) {
  if (dtype == SQB_F32) {
    *sz = 4;
    return true;
  }
  if (dtype == SQB_BF16) {
    *sz = 2;
    return true;
  }
  return false;
}

int check_dims(int64_t B, int64_t T, int64_t H, int64_t D, int64_t block) {
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0 || block <= 0) return SQB_ERR_ARG;
  if (B * H > (int64_t)1 << 30 || T > (int64_t)1 << 30 || D > 1024) return SQB_ERR_ARG;
  return SQB_OK;
}

TensorView view(const void* p, const int64_t* s) {
  return TensorView{const_cast<void*>(p), s[0], s[1], s[2]};
}

Problem make_problem(int64_t B, int64_t T, int64_t H, int64_t D, int64_t b, float scale,
                     int dtype) {
  Problem p;
  p.B = (int)B;
  p.T = (int)T;
  p.H = (int)H;
  p.D = (int)D;
  p.b = (int)b;
  p.G = (int)((T + b - 1) / b);
  p.Gc = (int)(T / b);
  p.scale = scale;
  p.dtype = dtype;
  return p;
}

}  // namespace
}  // namespace sqb

using namespace sqb;

extern "C" {

int sqb_version(void) { return 101; }

const char* sqb_strerror(int code) {
  switch (code) {
    case SQB_OK: return "ok";
    case SQB_ERR_ARG: return "invalid argument (null pointer, non-positive size or bad block)";
    case SQB_ERR_DTYPE: return "unknown dtype";
    case SQB_ERR_ALIGN: return "pointer or stride breaks the 16-byte alignment rule";
    case SQB_ERR_UNSUPPORTED: return "shape or dtype not supported by the requested kernels";
    case SQB_ERR_WORKSPACE: return "workspace missing or too small";
    case SQB_ERR_LAUNCH: return "kernel launch failed";
    case SQB_ERR_TIMEOUT: return "a device-side bounded wait gave up";
    case SQB_ERR_CUDA: return "CUDA runtime error";
    case SQB_ERR_DEVICE: return "device is not an sm_100 (B200-class) GPU";
    default: return "unknown error code";
  }
}

int sqb_geometry(int64_t T, int64_t block_req, int64_t* block, int64_t* n_blocks,
                 int64_t* n_complete) {
  if (T <= 0 || !block || !n_blocks || !n_complete) return SQB_ERR_ARG;
  int64_t b = block_req > 0 ? block_req : default_block(T);
  *block = b;
  *n_blocks = (T + b - 1) / b;
  *n_complete = T / b;
  return SQB_OK;
}

size_t sqb_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D, int64_t block) {
  if (check_dims(B, T, H, D, block)) return 0;
  return workspace_layout(B, T, H, D, block).total;
}

int sqb_fwd(const void* q, const void* k, const void* v, void* o, float* lse, void* kbar,
            void* vbar, int64_t B, int64_t T, int64_t H, int64_t D, int64_t block,
            const int64_t* strides, int dtype, float scale, int impl, void* workspace,
            size_t workspace_bytes, void* stream) {
  if (int e = check_dims(B, T, H, D, block)) return e;
  int esz;
  if (!elt_size(dtype, &esz)) return SQB_ERR_DTYPE;
  if (!q || !k || !v || !o || !lse || !strides) return SQB_ERR_ARG;
  const bool has_summaries = T / block > 0;
  if (has_summaries && (!kbar || !vbar)) return SQB_ERR_ARG;
  WorkspaceLayout wl = workspace_layout(B, T, H, D, block);
  if (!workspace || workspace_bytes < wl.total) return SQB_ERR_WORKSPACE;
  if (!(scale > 0.f) || !isfinite(scale)) return SQB_ERR_ARG;
  Problem p = make_problem(B, T, H, D, block, scale, dtype);
  TensorView tq = view(q, strides), tk = view(k, strides + 3), tv = view(v, strides + 6),
             to = view(o, strides + 9);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();  // clear a stale error so launch checks see only ours
  const bool tc_ok = sm100_fwd_supported(p, {tq, tk, tv, to}, lse, kbar, vbar);
  if (impl == SQB_IMPL_TCGEN05 && !tc_ok) return SQB_ERR_UNSUPPORTED;
  if (impl == SQB_IMPL_TCGEN05 || (impl == SQB_IMPL_AUTO && tc_ok))
    return sm100_forward(p, tq, tk, tv, to, lse, kbar, vbar, (uint8_t*)workspace, wl, s);
  if (impl != SQB_IMPL_SIMT && impl != SQB_IMPL_AUTO) return SQB_ERR_ARG;
  return simt_forward(p, tq, tk, tv, to, lse, kbar, vbar, s);
}

int sqb_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
            const float* lse, const void* kbar, const void* vbar, void* dq, void* dk, void* dv,
            int64_t B, int64_t T, int64_t H, int64_t D, int64_t block, const int64_t* strides,
            int dtype, float scale, int impl, void* workspace, size_t workspace_bytes,
            void* stream) {
  if (int e = check_dims(B, T, H, D, block)) return e;
  int esz;
  if (!elt_size(dtype, &esz)) return SQB_ERR_DTYPE;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv || !strides) return SQB_ERR_ARG;
  const bool has_summaries = T / block > 0;
  if (has_summaries && (!kbar || !vbar)) return SQB_ERR_ARG;
  WorkspaceLayout wl = workspace_layout(B, T, H, D, block);
  if (!workspace || workspace_bytes < wl.total) return SQB_ERR_WORKSPACE;
  if (!(scale > 0.f) || !isfinite(scale)) return SQB_ERR_ARG;
  Problem p = make_problem(B, T, H, D, block, scale, dtype);
  TensorView tq = view(q, strides), tk = view(k, strides + 3), tv = view(v, strides + 6),
             to = view(o, strides + 9), tdo = view(dout, strides + 12),
             tdq = view(dq, strides + 15), tdk = view(dk, strides + 18),
             tdv = view(dv, strides + 21);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();
  const bool tc_ok =
      sm100_bwd_supported(p, {tq, tk, tv, to, tdo, tdq, tdk, tdv}, lse, kbar, vbar);
  if (impl == SQB_IMPL_TCGEN05 && !tc_ok) return SQB_ERR_UNSUPPORTED;
  if (impl == SQB_IMPL_TCGEN05 || (impl == SQB_IMPL_AUTO && tc_ok))
    return sm100_backward(p, tq, tk, tv, to, tdo, lse, kbar, vbar, tdq, tdk, tdv,
                          (uint8_t*)workspace, wl, s);
  if (impl != SQB_IMPL_SIMT && impl != SQB_IMPL_AUTO) return SQB_ERR_ARG;
  return simt_backward(p, tq, tk, tv, to, tdo, lse, kbar, vbar, tdq, tdk, tdv,
                       (uint8_t*)workspace, wl, s);
}

int sqb_read_status(void* workspace, void* stream, int64_t* detail) {
  if (!workspace) return SQB_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t words[3] = {0, 0, 0};
  if (cudaStreamSynchronize(s) != cudaSuccess) return SQB_ERR_CUDA;
  uint8_t* base = (uint8_t*)workspace + kStatus * 4;
  if (cudaMemcpy(words, base, sizeof(words), cudaMemcpyDeviceToHost) != cudaSuccess)
    return SQB_ERR_CUDA;
  // status, detail and the abort word (normally already cleared by the launch)
  if ((words[0] | words[2]) != 0 && cudaMemset(base, 0, sizeof(words)) != cudaSuccess)
    return SQB_ERR_CUDA;
  if (detail) *detail = (int64_t)words[1];
  return (int)words[0];
}

int sqb_attach_status(void* workspace, uint32_t* mailbox, uint32_t wait_budget_us,
                      void* stream) {
  if (!workspace) return SQB_ERR_ARG;
  uint64_t mb = 0;
  if (mailbox) {
    // the device's address of the caller's page-locked pair (equal to the host
    // address under unified addressing)
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, mailbox) != cudaSuccess) {
      cudaGetLastError();
      return SQB_ERR_ARG;
    }
    void* dptr = attr.devicePointer;
    if (attr.type != cudaMemoryTypeHost || !dptr) return SQB_ERR_ARG;  // not page-locked
    if ((reinterpret_cast<uintptr_t>(dptr) & 7) != 0) return SQB_ERR_ALIGN;
    mb = (uint64_t)reinterpret_cast<uintptr_t>(dptr);
  }
  const uint32_t words[3] = {wait_budget_us, (uint32_t)(mb & 0xFFFFFFFFull),
                             (uint32_t)(mb >> 32)};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* dst = (uint8_t*)workspace + kWaitBudgetUs * 4;
  if (cudaMemcpyAsync(dst, words, sizeof(words), cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return SQB_ERR_CUDA;
  return SQB_OK;
}

}  // extern "C"
