// Host side of the sm_100a path: support checks, TMA tensor-map encoding and
// launch dispatch.  cuTensorMapEncodeTiled is fetched through the runtime's
// driver entry-point query, so the library does not link libcuda directly.

#include <mutex>

#include "sqb_sm100.cuh"

namespace sqb {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool view_ok(const TensorView& t) {
  // bf16: every stride in bytes must be a multiple of 16 (TMA global strides)
  return t.ptr && aligned16(t.ptr) && t.sb % 8 == 0 && t.st % 8 == 0 && t.sh % 8 == 0 &&
         t.sb > 0 && t.st > 0 && t.sh > 0;
}

bool device_ok(int* num_sms) {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return false;
  if (num_sms && cudaDeviceGetAttribute(num_sms, cudaDevAttrMultiProcessorCount, dev) !=
                     cudaSuccess)
    return false;
  return major == 10;
}

bool common_ok(const Problem& p, std::initializer_list<TensorView> views, const float* lse,
               const void* kbar, const void* vbar) {
  if (p.dtype != SQB_BF16) return false;
  if (p.D != 64 && p.D != 128) return false;
  if (p.b % 16 != 0 || p.b < 32) return false;
  if (!lse || !aligned16(lse)) return false;
  if (p.Gc > 0 && (!aligned16(kbar) || !aligned16(vbar))) return false;
  for (const TensorView& t : views)
    if (!view_ok(t)) return false;
  if (!encode_fn()) return false;
  return device_ok(nullptr);
}

// (B, T, H, D) bf16 view as a 4-D tensor map {D, H, T, B}, box {64, 1, rows, 1}.
bool encode_bthd(CUtensorMap* m, const Problem& p, const TensorView& t, int rows) {
  const cuuint64_t dims[4] = {(cuuint64_t)p.D, (cuuint64_t)p.H, (cuuint64_t)p.T, (cuuint64_t)p.B};
  const cuuint64_t strides[3] = {(cuuint64_t)t.sh * 2, (cuuint64_t)t.st * 2,
                                 (cuuint64_t)t.sb * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.ptr, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// (B, T, H, D) bf16 view as a store map with box {32, 1, 16, 1} (64 bytes x 16
// rows) and the 64-byte swizzle: the forward's per-warp O store units.
bool encode_bthd_store16(CUtensorMap* m, const Problem& p, const TensorView& t) {
  const cuuint64_t dims[4] = {(cuuint64_t)p.D, (cuuint64_t)p.H, (cuuint64_t)p.T, (cuuint64_t)p.B};
  const cuuint64_t strides[3] = {(cuuint64_t)t.sh * 2, (cuuint64_t)t.st * 2,
                                 (cuuint64_t)t.sb * 2};
  const cuuint32_t box[4] = {32, 1, 16, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.ptr, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// (B*H, Gc, D) contiguous bf16 summaries as {D, Gc, BH}, box {64, 128, 1}.
bool encode_summaries(CUtensorMap* m, const Problem& p, const void* ptr) {
  const cuuint64_t dims[3] = {(cuuint64_t)p.D, (cuuint64_t)p.Gc, (cuuint64_t)p.B * p.H};
  const cuuint64_t strides[2] = {(cuuint64_t)p.D * 2, (cuuint64_t)p.Gc * p.D * 2};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool sm100_device(int* num_sms) { return encode_fn() != nullptr && device_ok(num_sms); }

bool sm100_views_ok(std::initializer_list<TensorView> views) {
  for (const TensorView& t : views)
    if (!view_ok(t)) return false;
  return true;
}

bool sm100_encode_rows(CUtensorMap* m, int B, int T, int H, int D, const TensorView& t,
                       int rows) {
  Problem p{};
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  return encode_bthd(m, p, t, rows);
}

bool sm100_fwd_supported(const Problem& p, std::initializer_list<TensorView> views,
                         const float* lse, const void* kbar, const void* vbar) {
  return common_ok(p, views, lse, kbar, vbar);
}

bool sm100_bwd_supported(const Problem& p, std::initializer_list<TensorView> views,
                         const float* lse, const void* kbar, const void* vbar) {
  return common_ok(p, views, lse, kbar, vbar);
}

int sm100_forward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                  float* lse, void* kbar, void* vbar, uint8_t* ws, const WorkspaceLayout& wl,
                  cudaStream_t stream) {
  int num_sms = 0;
  if (!device_ok(&num_sms)) return SQB_ERR_DEVICE;
  const int R = sm100::tile_rows(p.b);
  sm100::TensorMaps tm;
  if (!encode_bthd(&tm.q, p, q, R) || !encode_bthd(&tm.k, p, k, R) ||
      !encode_bthd(&tm.v, p, v, R) || !encode_bthd_store16(&tm.o, p, o))
    return SQB_ERR_CUDA;
  if (p.Gc > 0) {
    if (!encode_summaries(&tm.kbar, p, kbar) || !encode_summaries(&tm.vbar, p, vbar))
      return SQB_ERR_CUDA;
  } else {
    tm.kbar = tm.k;  // never read: a sequence shorter than one block has no summaries
    tm.vbar = tm.v;
  }
  return sm100::launch_forward(p, tm, lse, kbar, vbar, ws, wl, num_sms, stream);
}

int sm100_backward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                   TensorView dout, const float* lse, const void* kbar, const void* vbar,
                   TensorView dq, TensorView dk, TensorView dv, uint8_t* ws,
                   const WorkspaceLayout& wl, cudaStream_t stream) {
  int num_sms = 0;
  if (!device_ok(&num_sms)) return SQB_ERR_DEVICE;
  const int R = sm100::tile_rows(p.b), RS = sm100::store_rows(p.b);
  sm100::BwdTensorMaps tm;
  if (!encode_bthd(&tm.q, p, q, R) || !encode_bthd(&tm.k, p, k, R) ||
      !encode_bthd(&tm.v, p, v, R) || !encode_bthd(&tm.o, p, o, R) ||
      !encode_bthd(&tm.dout, p, dout, R) ||
      !encode_bthd(&tm.dq, p, dq, RS) || !encode_bthd(&tm.dk, p, dk, RS) ||
      !encode_bthd(&tm.dv, p, dv, RS))
    return SQB_ERR_CUDA;
  if (p.Gc > 0) {
    if (!encode_summaries(&tm.kbar, p, kbar) || !encode_summaries(&tm.vbar, p, vbar))
      return SQB_ERR_CUDA;
  } else {
    tm.kbar = tm.k;  // never read: no summaries
    tm.vbar = tm.v;
  }
  return sm100::launch_backward(p, tm, lse, o, ws, wl, num_sms, stream);
}

}  // namespace sqb
