// Fused token cross-entropy for the GPT training caller (include/sqb_train.h).
//
// One CTA per row of logits.  Forward: a max pass and a sum-of-exp pass over
// the row (the second re-read comes from L2; a 50K-column bf16 row is 100 KB),
// then lse and the token loss.  Backward: one pass writing
// (softmax - one-hot) * scale in the logits' dtype.  Rows are read with 16-byte
// vector loads when the base and the row stride allow it; columns at or past V
// are never read.  fp32 math throughout, like the reference's autocast
// cross-entropy (training_utils.py:8-17).

#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "sqb_train.h"

namespace sqb {
namespace xent {
namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) {
  return x;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Block-wide reduction of one float per thread (op: max or sum); every thread
// gets the result.
template <bool kMax>
__device__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < kThreads / 32 ? red[lane] : (kMax ? -INFINITY : 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, w) : v + w;
  }
  return v;
}

// Calls f(c, x) for every column c < V of `row`, with 16-byte loads where the
// whole vector lies below V.
template <typename T, bool kVec, typename F>
__device__ __forceinline__ void for_row(const T* row, int64_t V, F&& f) {
  constexpr int kN = 16 / sizeof(T);
  if constexpr (kVec) {
    const int64_t nvec = V / kN;
    for (int64_t i = threadIdx.x; i < nvec; i += kThreads) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + i * kN);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < kN; ++j) f(i * kN + j, to_f(e[j]));
    }
    for (int64_t c = nvec * kN + threadIdx.x; c < V; c += kThreads) f(c, to_f(row[c]));
  } else {
    for (int64_t c = threadIdx.x; c < V; c += kThreads) f(c, to_f(row[c]));
  }
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads) fwd_kernel(const T* logits, const int64_t* targets,
                                                       float* loss, float* lse, int64_t V,
                                                       int64_t ld) {
  __shared__ float red[kThreads / 32];
  const int64_t r = blockIdx.x;
  const T* row = logits + r * ld;
  float m = -INFINITY;
  for_row<T, kVec>(row, V, [&](int64_t, float x) { m = fmaxf(m, x); });
  m = block_reduce<true>(m, red);
  float s = 0.f;
  if (m != -INFINITY) for_row<T, kVec>(row, V, [&](int64_t, float x) { s += __expf(x - m); });
  s = block_reduce<false>(s, red);
  if (threadIdx.x == 0) {
    const float l = m + __logf(s);
    const int64_t t = targets[r];
    lse[r] = l;
    // an ignored row has loss 0; a target past the vocabulary is never read
    // (NaN marks it, as the reference's cross-entropy would fail on it)
    loss[r] = t < 0 ? 0.f : t < V ? l - to_f(row[t]) : NAN;
  }
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads) bwd_kernel(const T* logits, const int64_t* targets,
                                                       const float* lse, const float* scale,
                                                       T* dlogits, int64_t V, int64_t ld) {
  const int64_t r = blockIdx.x;
  const T* row = logits + r * ld;
  T* drow = dlogits + r * ld;
  const int64_t t = targets[r];
  const float l = lse[r];
  const float g = t >= 0 ? *scale : 0.f;
  constexpr int kN = 16 / sizeof(T);
  if constexpr (kVec) {
    const int64_t nvec = V / kN;
    for (int64_t i = threadIdx.x; i < nvec; i += kThreads) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + i * kN);
      const T* e = reinterpret_cast<const T*>(&u);
      uint4 o;
      T* d = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int j = 0; j < kN; ++j) {
        const int64_t c = i * kN + j;
        d[j] = from_f<T>((__expf(to_f(e[j]) - l) - (c == t ? 1.f : 0.f)) * g);
      }
      *reinterpret_cast<uint4*>(drow + i * kN) = o;
    }
    for (int64_t c = nvec * kN + threadIdx.x; c < ld; c += kThreads)
      drow[c] = from_f<T>(c < V ? (__expf(to_f(row[c]) - l) - (c == t ? 1.f : 0.f)) * g : 0.f);
  } else {
    for (int64_t c = threadIdx.x; c < ld; c += kThreads)
      drow[c] = from_f<T>(c < V ? (__expf(to_f(row[c]) - l) - (c == t ? 1.f : 0.f)) * g : 0.f);
  }
}

int elt_of(int dtype) { return dtype == SQB_BF16 ? 2 : dtype == SQB_F32 ? 4 : 0; }

bool vec_ok(const void* p, int64_t ld, int elt) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * elt) % 16 == 0;
}

}  // namespace
}  // namespace xent
}  // namespace sqb

using namespace sqb::xent;

extern "C" int sqb_xent_fwd(const void* logits, const int64_t* targets, float* loss, float* lse,
                            int64_t N, int64_t V, int64_t ld, int dtype, void* stream) {
  if (!logits || !targets || !loss || !lse || N <= 0 || V <= 0 || ld < V || N > INT32_MAX)
    return SQB_ERR_ARG;
  const int elt = elt_of(dtype);
  if (!elt) return SQB_ERR_DTYPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = vec_ok(logits, ld, elt);
  const dim3 grid((unsigned)N);
  if (dtype == SQB_BF16) {
    auto x = static_cast<const __nv_bfloat16*>(logits);
    if (vec)
      fwd_kernel<__nv_bfloat16, true><<<grid, kThreads, 0, s>>>(x, targets, loss, lse, V, ld);
    else
      fwd_kernel<__nv_bfloat16, false><<<grid, kThreads, 0, s>>>(x, targets, loss, lse, V, ld);
  } else {
    auto x = static_cast<const float*>(logits);
    if (vec)
      fwd_kernel<float, true><<<grid, kThreads, 0, s>>>(x, targets, loss, lse, V, ld);
    else
      fwd_kernel<float, false><<<grid, kThreads, 0, s>>>(x, targets, loss, lse, V, ld);
  }
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

extern "C" int sqb_xent_bwd(const void* logits, const int64_t* targets, const float* lse,
                            const float* scale, void* dlogits, int64_t N, int64_t V, int64_t ld,
                            int dtype, void* stream) {
  if (!logits || !targets || !lse || !scale || !dlogits || N <= 0 || V <= 0 || ld < V ||
      N > INT32_MAX)
    return SQB_ERR_ARG;
  const int elt = elt_of(dtype);
  if (!elt) return SQB_ERR_DTYPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = vec_ok(logits, ld, elt) && vec_ok(dlogits, ld, elt);
  const dim3 grid((unsigned)N);
  if (dtype == SQB_BF16) {
    auto x = static_cast<const __nv_bfloat16*>(logits);
    auto d = static_cast<__nv_bfloat16*>(dlogits);
    if (vec)
      bwd_kernel<__nv_bfloat16, true><<<grid, kThreads, 0, s>>>(x, targets, lse, scale, d, V, ld);
    else
      bwd_kernel<__nv_bfloat16, false><<<grid, kThreads, 0, s>>>(x, targets, lse, scale, d, V, ld);
  } else {
    auto x = static_cast<const float*>(logits);
    auto d = static_cast<float*>(dlogits);
    if (vec)
      bwd_kernel<float, true><<<grid, kThreads, 0, s>>>(x, targets, lse, scale, d, V, ld);
    else
      bwd_kernel<float, false><<<grid, kThreads, 0, s>>>(x, targets, lse, scale, d, V, ld);
  }
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}
