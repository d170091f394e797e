// Fused LayerNorm over the last dimension for the GPT training caller
// (include/sqb_train.h), as the reference's LayerNorm module (model/layer_norm.py:4-13,
// torch.nn.LayerNorm with an optional bias) computes it under bf16 autocast: fp32
// math on the fp32 residual stream.
//
// Forward: one warp per row, the row held in registers (C / 128 float4 per
// lane), mean and 1/std by two warp reductions, y = (x - mean) * rstd * w + b
// written as fp32 or directly as bf16 (what the next autocast Linear would cast
// it to).  Backward: one warp per row for dx; every lane keeps its columns'
// partial sums of dy * xhat (and dy) over the rows its warp visits, a CTA sums
// its warps in shared memory and writes one partial row per CTA, and a second
// kernel adds the partial rows column by column: dweight and dbias come out in a
// fixed order (bit-reproducible).
//
// Residual variants (sqb_add_layernorm_*): the forward first forms the row
// x_out = x + h (h fp32 or bf16, what a bf16 autocast Linear hands the residual
// stream) and writes it, then normalises it; the backward adds the gradient
// reaching x_out from its other uses to the LayerNorm's dx and also writes the
// sum as bf16 (the gradient of a bf16 h).  One pass each instead of an add, a
// LayerNorm, a gradient add and a cast.

#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "sqb_train.h"

namespace sqb {
namespace lnorm {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxVpl = 8;      // C <= 1024
constexpr int kPartRows = 296;  // CTAs of the backward (2 per SM on 148 SMs)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
  const __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// Column of lane `lane`'s k-th float4: the warp reads 512 contiguous bytes per k.
__device__ __forceinline__ int col(int lane, int k) { return (k * 32 + lane) * 4; }

// h (null, or fp32 / bf16 rows by h_bf16): x_out = x + h is written and normalised.
template <int VPL, typename OutT>
__global__ void __launch_bounds__(kThreads) fwd_kernel(const float* x, const void* h,
                                                       bool h_bf16, float* xo, const float* w,
                                                       const float* b, OutT* y, float* mean,
                                                       float* rstd, int64_t N, float eps) {
  constexpr int C = VPL * 128;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= N) return;
  const float* xr = x + row * C;
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int c0 = col(lane, k);
    v[k] = load4(xr + c0);
    if (h) {
      const float4 hv = h_bf16 ? load4(static_cast<const __nv_bfloat16*>(h) + row * C + c0)
                               : load4(static_cast<const float*>(h) + row * C + c0);
      v[k] = make_float4(v[k].x + hv.x, v[k].y + hv.y, v[k].z + hv.z, v[k].w + hv.w);
      store4(xo + row * C + c0, v[k]);
    }
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
  const float mu = warp_sum(s) * (1.f / C);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const float a = v[k].x - mu, c = v[k].y - mu, d = v[k].z - mu, e = v[k].w - mu;
    q += (a * a + c * c) + (d * d + e * e);
  }
  const float rs = rsqrtf(warp_sum(q) * (1.f / C) + eps);
  OutT* yr = y + row * C;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int c0 = col(lane, k);
    const float4 wk = load4(w + c0);
    const float4 bk = b ? load4(b + c0) : make_float4(0.f, 0.f, 0.f, 0.f);
    store4(yr + c0, make_float4((v[k].x - mu) * rs * wk.x + bk.x, (v[k].y - mu) * rs * wk.y + bk.y,
                                (v[k].z - mu) * rs * wk.z + bk.z, (v[k].w - mu) * rs * wk.w + bk.w));
  }
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

// Two CTAs per SM while a lane's running sums fit the register budget (C <= 768
// without a bias, C <= 512 with one), else one.
template <int VPL, typename DyT, bool kBias>
__global__ void __launch_bounds__(kThreads, VPL * (kBias ? 3 : 2) <= 12 ? 2 : 1)
    bwd_kernel(const DyT* dy, const float* x, const float* w, const float* mean,
               const float* rstd, const float* dres, float* dx, __nv_bfloat16* dh,
               float* part_w, float* part_b, int64_t N) {
  constexpr int C = VPL * 128;
  __shared__ float red[kWarps][C];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4 wk[VPL], aw[VPL], ab[kBias ? VPL : 1];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    wk[k] = load4(w + col(lane, k));
    aw[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (kBias) ab[k] = aw[k];
  }
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < N;
       row += (int64_t)gridDim.x * kWarps) {
    const float mu = mean[row], rs = rstd[row];
    float4 xh[VPL], g[VPL];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int c0 = col(lane, k);
      const float4 xv = load4(x + row * C + c0);
      const float4 d = load4(dy + row * C + c0);
      xh[k] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs, (xv.w - mu) * rs);
      g[k] = make_float4(d.x * wk[k].x, d.y * wk[k].y, d.z * wk[k].z, d.w * wk[k].w);
      s1 += (g[k].x + g[k].y) + (g[k].z + g[k].w);
      s2 += (g[k].x * xh[k].x + g[k].y * xh[k].y) + (g[k].z * xh[k].z + g[k].w * xh[k].w);
      aw[k].x += d.x * xh[k].x;
      aw[k].y += d.y * xh[k].y;
      aw[k].z += d.z * xh[k].z;
      aw[k].w += d.w * xh[k].w;
      if constexpr (kBias) {
        ab[k].x += d.x;
        ab[k].y += d.y;
        ab[k].z += d.z;
        ab[k].w += d.w;
      }
    }
    const float m1 = warp_sum(s1) * (1.f / C), m2 = warp_sum(s2) * (1.f / C);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int c0 = col(lane, k);
      float4 o = make_float4(rs * (g[k].x - m1 - xh[k].x * m2), rs * (g[k].y - m1 - xh[k].y * m2),
                             rs * (g[k].z - m1 - xh[k].z * m2), rs * (g[k].w - m1 - xh[k].w * m2));
      if (dres) {  // the gradient reaching x_out from its other uses
        const float4 r = load4(dres + row * C + c0);
        o = make_float4(o.x + r.x, o.y + r.y, o.z + r.z, o.w + r.w);
      }
      store4(dx + row * C + c0, o);
      if (dh) store4(dh + row * C + c0, o);
    }
  }
  // this CTA's column sums: dweight, then dbias (when asked for)
#pragma unroll 1
  for (int pass = 0; pass < (kBias ? 2 : 1); ++pass) {
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      if constexpr (kBias)
        store4(&red[warp][col(lane, k)], pass ? ab[k] : aw[k]);
      else
        store4(&red[warp][col(lane, k)], aw[k]);
    }
    __syncthreads();
    float* out = (pass ? part_b : part_w) + (int64_t)blockIdx.x * C;
    for (int c = threadIdx.x; c < C; c += kThreads) {
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) t += red[i][c];
      out[c] = t;
    }
    __syncthreads();
  }
}

// out[c] = sum over the `rows` partial rows of column c: a CTA of 8 x 32 threads
// takes 32 columns, thread (g, j) sums rows g, g + 8, ... of column j and the
// eight group sums are added in shared memory (a fixed order).
__global__ void __launch_bounds__(256) colsum_kernel(const float* part, float* out, int rows,
                                                     int C) {
  __shared__ float red[8][33];
  const int j = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + j;
  float t = 0.f;
  if (c < C)
    for (int r = grp; r < rows; r += 8) t += part[(int64_t)r * C + c];
  red[grp][j] = t;
  __syncthreads();
  if (grp == 0 && c < C) {
    float u = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) u += red[i][j];
    out[c] = u;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int part_rows(int64_t N) {
  const int64_t ctas = (N + kWarps - 1) / kWarps;
  return (int)(ctas < kPartRows ? ctas : kPartRows);
}

template <int VPL>
int launch_fwd(const float* x, const void* h, bool h_bf16, float* xo, const float* w,
               const float* b, void* y, int y_dtype, float* mean, float* rstd, int64_t N,
               float eps, cudaStream_t s) {
  const dim3 grid((unsigned)((N + kWarps - 1) / kWarps));
  if (y_dtype == SQB_BF16)
    fwd_kernel<VPL, __nv_bfloat16><<<grid, kThreads, 0, s>>>(
        x, h, h_bf16, xo, w, b, static_cast<__nv_bfloat16*>(y), mean, rstd, N, eps);
  else
    fwd_kernel<VPL, float><<<grid, kThreads, 0, s>>>(x, h, h_bf16, xo, w, b,
                                                     static_cast<float*>(y), mean, rstd, N, eps);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

template <int VPL>
int launch_bwd(const void* dy, int dy_dtype, const float* x, const float* w, const float* mean,
               const float* rstd, const float* dres, float* dx, __nv_bfloat16* dh, float* dw,
               float* db, float* part, int64_t N, cudaStream_t s) {
  constexpr int C = VPL * 128;
  const int rows = part_rows(N);
  float* part_w = part;
  float* part_b = db ? part + (int64_t)rows * C : nullptr;
  auto dyb = static_cast<const __nv_bfloat16*>(dy);
  auto dyf = static_cast<const float*>(dy);
  if (dy_dtype == SQB_BF16 && db)
    bwd_kernel<VPL, __nv_bfloat16, true><<<rows, kThreads, 0, s>>>(
        dyb, x, w, mean, rstd, dres, dx, dh, part_w, part_b, N);
  else if (dy_dtype == SQB_BF16)
    bwd_kernel<VPL, __nv_bfloat16, false><<<rows, kThreads, 0, s>>>(
        dyb, x, w, mean, rstd, dres, dx, dh, part_w, part_b, N);
  else if (db)
    bwd_kernel<VPL, float, true><<<rows, kThreads, 0, s>>>(dyf, x, w, mean, rstd, dres, dx, dh,
                                                            part_w, part_b, N);
  else
    bwd_kernel<VPL, float, false><<<rows, kThreads, 0, s>>>(dyf, x, w, mean, rstd, dres, dx,
                                                             dh, part_w, part_b, N);
  colsum_kernel<<<(C + 31) / 32, 256, 0, s>>>(part_w, dw, rows, C);
  if (db) colsum_kernel<<<(C + 31) / 32, 256, 0, s>>>(part_b, db, rows, C);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

}  // namespace
}  // namespace lnorm
}  // namespace sqb

using namespace sqb::lnorm;

extern "C" size_t sqb_layernorm_workspace_bytes(int64_t N, int64_t C) {
  if (N <= 0 || C <= 0) return 0;
  return (size_t)part_rows(N) * (size_t)C * 2 * sizeof(float);
}

namespace {

int fwd_dispatch(const float* x, const void* h, int h_dtype, float* x_out, const float* weight,
                 const float* bias, void* y, int y_dtype, float* mean, float* rstd, int64_t N,
                 int64_t C, float eps, void* stream) {
  if (!x || !weight || !y || !mean || !rstd || N <= 0 || N > ((int64_t)1 << 31) * kWarps)
    return SQB_ERR_ARG;
  if (h && !x_out) return SQB_ERR_ARG;
  if (y_dtype != SQB_F32 && y_dtype != SQB_BF16) return SQB_ERR_DTYPE;
  if (h && h_dtype != SQB_F32 && h_dtype != SQB_BF16) return SQB_ERR_DTYPE;
  if (C <= 0 || C % 128 != 0 || C / 128 > kMaxVpl) return SQB_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(weight) || (bias && !aligned16(bias)) || !aligned16(y) ||
      (h && (!aligned16(h) || !aligned16(x_out))))
    return SQB_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool hb = h_dtype == SQB_BF16;
#define SQB_LN_FWD(V) launch_fwd<V>(x, h, hb, x_out, weight, bias, y, y_dtype, mean, rstd, N, eps, s)
  switch (C / 128) {
    case 1: return SQB_LN_FWD(1);
    case 2: return SQB_LN_FWD(2);
    case 3: return SQB_LN_FWD(3);
    case 4: return SQB_LN_FWD(4);
    case 5: return SQB_LN_FWD(5);
    case 6: return SQB_LN_FWD(6);
    case 7: return SQB_LN_FWD(7);
    default: return SQB_LN_FWD(8);
  }
#undef SQB_LN_FWD
}

int bwd_dispatch(const void* dy, int dy_dtype, const float* x, const float* weight,
                 const float* mean, const float* rstd, const float* dres, float* dx, void* dh,
                 float* dweight, float* dbias, void* workspace, size_t ws_bytes, int64_t N,
                 int64_t C, void* stream) {
  if (!dy || !x || !weight || !mean || !rstd || !dx || !dweight || N <= 0) return SQB_ERR_ARG;
  if (dy_dtype != SQB_F32 && dy_dtype != SQB_BF16) return SQB_ERR_DTYPE;
  if (C <= 0 || C % 128 != 0 || C / 128 > kMaxVpl) return SQB_ERR_UNSUPPORTED;
  if (!workspace || ws_bytes < sqb_layernorm_workspace_bytes(N, C)) return SQB_ERR_WORKSPACE;
  if (!aligned16(dy) || !aligned16(x) || !aligned16(weight) || !aligned16(dx) ||
      !aligned16(workspace) || (dres && !aligned16(dres)) || (dh && !aligned16(dh)))
    return SQB_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  auto* dhb = static_cast<__nv_bfloat16*>(dh);
#define SQB_LN_BWD(V) \
  launch_bwd<V>(dy, dy_dtype, x, weight, mean, rstd, dres, dx, dhb, dweight, dbias, part, N, s)
  switch (C / 128) {
    case 1: return SQB_LN_BWD(1);
    case 2: return SQB_LN_BWD(2);
    case 3: return SQB_LN_BWD(3);
    case 4: return SQB_LN_BWD(4);
    case 5: return SQB_LN_BWD(5);
    case 6: return SQB_LN_BWD(6);
    case 7: return SQB_LN_BWD(7);
    default: return SQB_LN_BWD(8);
  }
#undef SQB_LN_BWD
}

}  // namespace

extern "C" int sqb_layernorm_fwd(const float* x, const float* weight, const float* bias, void* y,
                                 int y_dtype, float* mean, float* rstd, int64_t N, int64_t C,
                                 float eps, void* stream) {
  return fwd_dispatch(x, nullptr, SQB_F32, nullptr, weight, bias, y, y_dtype, mean, rstd, N, C,
                      eps, stream);
}

extern "C" int sqb_layernorm_bwd(const void* dy, int dy_dtype, const float* x,
                                 const float* weight, const float* mean, const float* rstd,
                                 float* dx, float* dweight, float* dbias, void* workspace,
                                 size_t ws_bytes, int64_t N, int64_t C, void* stream) {
  return bwd_dispatch(dy, dy_dtype, x, weight, mean, rstd, nullptr, dx, nullptr, dweight, dbias,
                      workspace, ws_bytes, N, C, stream);
}

extern "C" int sqb_add_layernorm_fwd(const float* x, const void* h, int h_dtype, float* x_out,
                                     const float* weight, const float* bias, void* y,
                                     int y_dtype, float* mean, float* rstd, int64_t N,
                                     int64_t C, float eps, void* stream) {
  if (!h) return SQB_ERR_ARG;
  return fwd_dispatch(x, h, h_dtype, x_out, weight, bias, y, y_dtype, mean, rstd, N, C, eps,
                      stream);
}

extern "C" int sqb_add_layernorm_bwd(const void* dy, int dy_dtype, const float* x_out,
                                     const float* weight, const float* mean, const float* rstd,
                                     const float* dres, float* dx, void* dh_bf16,
                                     float* dweight, float* dbias, void* workspace,
                                     size_t ws_bytes, int64_t N, int64_t C, void* stream) {
  return bwd_dispatch(dy, dy_dtype, x_out, weight, mean, rstd, dres, dx, dh_bf16, dweight,
                      dbias, workspace, ws_bytes, N, C, stream);
}
