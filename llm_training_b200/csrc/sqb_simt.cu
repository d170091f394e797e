// SIMT (CUDA-core) sqrt-block attention: forward, backward and block pooling.
//
// One warp per output row, fp32 accumulation, any head dim D <= 256.  This is
// the fp32 path (fp32 inputs need fp32 products: the tensor-core kinds that
// take fp32 operands round them to tf32) and the debugging baseline the
// tcgen05 kernels are checked against.  The math follows the operator's
// definition term by term; the reference's own core (model/custom_attention.py
// :195-225) computes a different summary, so only its conventions are shared:
// scale applied to q.k, inclusive causal diagonal (custom_attention.py:195-198).

#include <math.h>

#include "sqb_internal.cuh"

namespace sqb {
namespace {

constexpr int kMaxPerLane = 8;  // D <= 256 = 8 * 32
constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename E>
__device__ __forceinline__ E from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename E>
__device__ __forceinline__ const E* row_ptr(const TensorView& t, int n, int tok, int h) {
  return reinterpret_cast<const E*>(t.ptr) + (int64_t)n * t.sb + (int64_t)tok * t.st +
         (int64_t)h * t.sh;
}
template <typename E>
__device__ __forceinline__ E* row_ptr_w(const TensorView& t, int n, int tok, int h) {
  return reinterpret_cast<E*>(t.ptr) + (int64_t)n * t.sb + (int64_t)tok * t.st +
         (int64_t)h * t.sh;
}

template <typename E>
__device__ __forceinline__ void load_row(const E* r, int D, int lane, float (&x)[kMaxPerLane]) {
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    int d = lane + 32 * i;
    x[i] = d < D ? to_f(r[d]) : 0.f;
  }
}

template <typename E>
__device__ __forceinline__ float dot_row(const E* r, int D, int lane,
                                         const float (&x)[kMaxPerLane]) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    int d = lane + 32 * i;
    if (d < D) s += x[i] * to_f(r[d]);
  }
  return warp_sum(s);
}

// Block means of K and V over each complete block.  grid (Gc, B*H), D threads.
template <typename E>
__global__ void pool_kernel(Problem p, TensorView k, TensorView v, E* kbar, E* vbar) {
  const int j = blockIdx.x, bh = blockIdx.y;
  const int n = bh / p.H, h = bh % p.H;
  const int d = threadIdx.x;
  if (d >= p.D) return;
  float sk = 0.f, sv = 0.f;
  for (int r = 0; r < p.b; ++r) {
    int tok = j * p.b + r;
    sk += to_f(row_ptr<E>(k, n, tok, h)[d]);
    sv += to_f(row_ptr<E>(v, n, tok, h)[d]);
  }
  const float inv = 1.f / (float)p.b;
  const int64_t off = ((int64_t)bh * p.Gc + j) * p.D + d;
  kbar[off] = from_f<E>(sk * inv);
  vbar[off] = from_f<E>(sv * inv);
}

// Forward: one warp per query row, online softmax over the in-block keys
// followed by the summaries of the earlier blocks.
template <typename E>
__global__ void fwd_kernel(Problem p, TensorView q, TensorView k, TensorView v, TensorView o,
                           float* lse, const E* kbar, const E* vbar) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int bh = blockIdx.y;
  const int n = bh / p.H, h = bh % p.H;
  if (t >= p.T) return;
  float qv[kMaxPerLane];
  load_row(row_ptr<E>(q, n, t, h), p.D, lane, qv);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) qv[i] *= p.scale;
  float acc[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int blk = t / p.b;
  auto consume = [&](float s, const E* vr) {
    const float m_new = fmaxf(m, s);
    const float corr = expf(m - m_new);  // 0 on the first key (m = -inf)
    const float e = expf(s - m_new);
    l = l * corr + e;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      int d = lane + 32 * i;
      acc[i] = acc[i] * corr + (d < p.D ? e * to_f(vr[d]) : 0.f);
    }
    m = m_new;
  };
  for (int kk = blk * p.b; kk <= t; ++kk) {
    float s = dot_row(row_ptr<E>(k, n, kk, h), p.D, lane, qv);
    consume(s, row_ptr<E>(v, n, kk, h));
  }
  for (int j = 0; j < blk; ++j) {
    const int64_t off = ((int64_t)bh * p.Gc + j) * p.D;
    float s = dot_row(kbar + off, p.D, lane, qv);
    consume(s, vbar + off);
  }
  const float inv = 1.f / l;
  E* orow = row_ptr_w<E>(o, n, t, h);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    int d = lane + 32 * i;
    if (d < p.D) orow[d] = from_f<E>(acc[i] * inv);
  }
  if (lane == 0) lse[(int64_t)bh * p.T + t] = m + logf(l);
}

// delta_t = dO_t . O_t
template <typename E>
__global__ void delta_kernel(Problem p, TensorView o, TensorView dout, float* delta) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int bh = blockIdx.y;
  const int n = bh / p.H, h = bh % p.H;
  if (t >= p.T) return;
  float x[kMaxPerLane];
  load_row(row_ptr<E>(dout, n, t, h), p.D, lane, x);
  float s = dot_row(row_ptr<E>(o, n, t, h), p.D, lane, x);
  if (lane == 0) delta[(int64_t)bh * p.T + t] = s;
}

// Summary gradients: one CTA per (summary j, bh); its warps split the later
// queries (warp w takes t = first + w, first + w + 8, ...) and add their
// partial sums in shared memory in warp order, so the result does not depend on
// scheduling (one warp walking every later query made the first summaries'
// chains the kernel's length).
//   dKbar_j = scale * sum_t ds_tj q_t,  dVbar_j = sum_t p_tj dO_t.
template <typename E>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) summary_grad_kernel(
    Problem p, TensorView q, TensorView dout, const float* lse, const float* delta,
    const E* kbar, const E* vbar, float* dkbar, float* dvbar) {
  __shared__ float red[2][kWarpsPerBlock][32 * kMaxPerLane];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = blockIdx.x;
  const int bh = blockIdx.y;
  const int n = bh / p.H, h = bh % p.H;
  const int64_t soff = ((int64_t)bh * p.Gc + j) * p.D;
  float kb[kMaxPerLane], vb[kMaxPerLane], gk[kMaxPerLane], gv[kMaxPerLane];
  load_row(kbar + soff, p.D, lane, kb);
  load_row(vbar + soff, p.D, lane, vb);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) gk[i] = gv[i] = 0.f;
  for (int t = (j + 1) * p.b + warp; t < p.T; t += kWarpsPerBlock) {
    const E* qr = row_ptr<E>(q, n, t, h);
    const E* dr = row_ptr<E>(dout, n, t, h);
    const float s = dot_row(qr, p.D, lane, kb) * p.scale;
    const float pr = expf(s - lse[(int64_t)bh * p.T + t]);
    const float dp = dot_row(dr, p.D, lane, vb);
    const float ds = pr * (dp - delta[(int64_t)bh * p.T + t]);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      int d = lane + 32 * i;
      if (d < p.D) {
        gk[i] += ds * to_f(qr[d]);
        gv[i] += pr * to_f(dr[d]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    red[0][warp][lane + 32 * i] = gk[i];
    red[1][warp][lane + 32 * i] = gv[i];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < p.D; d += 32 * kWarpsPerBlock) {
    float sk = 0.f, sv = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsPerBlock; ++w) {
      sk += red[0][w][d];
      sv += red[1][w][d];
    }
    dkbar[soff + d] = sk * p.scale;
    dvbar[soff + d] = sv;
  }
}

// dQ: one warp per query row over its in-block keys and earlier summaries.
template <typename E>
__global__ void dq_kernel(Problem p, TensorView q, TensorView k, TensorView v, TensorView dout,
                          const float* lse, const float* delta, const E* kbar, const E* vbar,
                          TensorView dq) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int bh = blockIdx.y;
  const int n = bh / p.H, h = bh % p.H;
  if (t >= p.T) return;
  float qv[kMaxPerLane], dov[kMaxPerLane], acc[kMaxPerLane];
  load_row(row_ptr<E>(q, n, t, h), p.D, lane, qv);
  load_row(row_ptr<E>(dout, n, t, h), p.D, lane, dov);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.f;
  const float L = lse[(int64_t)bh * p.T + t];
  const float dl = delta[(int64_t)bh * p.T + t];
  const int blk = t / p.b;
  auto consume = [&](const E* kr, const E* vr) {
    const float s = dot_row(kr, p.D, lane, qv) * p.scale;
    const float pr = expf(s - L);
    const float dp = dot_row(vr, p.D, lane, dov);
    const float ds = pr * (dp - dl);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      int d = lane + 32 * i;
      if (d < p.D) acc[i] += ds * to_f(kr[d]);
    }
  };
  for (int kk = blk * p.b; kk <= t; ++kk) consume(row_ptr<E>(k, n, kk, h), row_ptr<E>(v, n, kk, h));
  for (int j = 0; j < blk; ++j) {
    const int64_t off = ((int64_t)bh * p.Gc + j) * p.D;
    consume(kbar + off, vbar + off);
  }
  E* out = row_ptr_w<E>(dq, n, t, h);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    int d = lane + 32 * i;
    if (d < p.D) out[d] = from_f<E>(acc[i] * p.scale);
  }
}

// dK, dV: one warp per key row over the later queries of its block, plus the
// block's summary gradient divided by b (a summary is the mean of its block).
template <typename E>
__global__ void dkdv_kernel(Problem p, TensorView q, TensorView k, TensorView v, TensorView dout,
                            const float* lse, const float* delta, const float* dkbar,
                            const float* dvbar, TensorView dk, TensorView dv) {
  const int lane = threadIdx.x & 31;
  const int kk = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int bh = blockIdx.y;
  const int n = bh / p.H, h = bh % p.H;
  if (kk >= p.T) return;
  float kv[kMaxPerLane], vv[kMaxPerLane], gk[kMaxPerLane], gv[kMaxPerLane];
  load_row(row_ptr<E>(k, n, kk, h), p.D, lane, kv);
  load_row(row_ptr<E>(v, n, kk, h), p.D, lane, vv);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) gk[i] = gv[i] = 0.f;
  const int blk = kk / p.b;
  const int t_end = min((blk + 1) * p.b, p.T);
  for (int t = kk; t < t_end; ++t) {
    const E* qr = row_ptr<E>(q, n, t, h);
    const E* dr = row_ptr<E>(dout, n, t, h);
    const float s = dot_row(qr, p.D, lane, kv) * p.scale;
    const float pr = expf(s - lse[(int64_t)bh * p.T + t]);
    const float dp = dot_row(dr, p.D, lane, vv);
    const float ds = pr * (dp - delta[(int64_t)bh * p.T + t]);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      int d = lane + 32 * i;
      if (d < p.D) {
        gk[i] += ds * to_f(qr[d]);
        gv[i] += pr * to_f(dr[d]);
      }
    }
  }
  const bool complete = blk < p.Gc;
  const int64_t soff = ((int64_t)bh * p.Gc + blk) * p.D;
  const float invb = 1.f / (float)p.b;
  E* outk = row_ptr_w<E>(dk, n, kk, h);
  E* outv = row_ptr_w<E>(dv, n, kk, h);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    int d = lane + 32 * i;
    if (d < p.D) {
      float a = gk[i] * p.scale, c = gv[i];
      if (complete) {
        a += dkbar[soff + d] * invb;
        c += dvbar[soff + d] * invb;
      }
      outk[d] = from_f<E>(a);
      outv[d] = from_f<E>(c);
    }
  }
}

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

template <typename E>
int forward_t(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o, float* lse,
              void* kbar, void* vbar, cudaStream_t s) {
  const int BH = p.B * p.H;
  if (p.Gc > 0) {
    pool_kernel<E><<<dim3(p.Gc, BH), p.D, 0, s>>>(p, k, v, (E*)kbar, (E*)vbar);
    if (int e = launch_status()) return e;
  }
  dim3 grid((p.T + kWarpsPerBlock - 1) / kWarpsPerBlock, BH);
  fwd_kernel<E><<<grid, 32 * kWarpsPerBlock, 0, s>>>(p, q, k, v, o, lse, (const E*)kbar,
                                                      (const E*)vbar);
  return launch_status();
}

template <typename E>
int backward_t(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
               TensorView dout, const float* lse, const void* kbar, const void* vbar,
               TensorView dq, TensorView dk, TensorView dv, uint8_t* ws,
               const WorkspaceLayout& wl, cudaStream_t s) {
  const int BH = p.B * p.H;
  float* delta = reinterpret_cast<float*>(ws + wl.delta);
  float* dkbar = reinterpret_cast<float*>(ws + wl.dkbar);
  float* dvbar = reinterpret_cast<float*>(ws + wl.dvbar);
  dim3 rows((p.T + kWarpsPerBlock - 1) / kWarpsPerBlock, BH);
  const int nt = 32 * kWarpsPerBlock;
  delta_kernel<E><<<rows, nt, 0, s>>>(p, o, dout, delta);
  if (int e = launch_status()) return e;
  if (p.Gc > 0) {
    dim3 sg(p.Gc, BH);
    summary_grad_kernel<E><<<sg, nt, 0, s>>>(p, q, dout, lse, delta, (const E*)kbar,
                                             (const E*)vbar, dkbar, dvbar);
    if (int e = launch_status()) return e;
  }
  dq_kernel<E><<<rows, nt, 0, s>>>(p, q, k, v, dout, lse, delta, (const E*)kbar, (const E*)vbar,
                                   dq);
  if (int e = launch_status()) return e;
  dkdv_kernel<E><<<rows, nt, 0, s>>>(p, q, k, v, dout, lse, delta, dkbar, dvbar, dk, dv);
  if (int e = launch_status()) return e;
  // leave the summary-gradient scratch zeroed: the tcgen05 backward
  // accumulates into the same workspace region and expects zeros
  if (p.Gc > 0 && cudaMemsetAsync(ws + wl.dkbar, 0, wl.total - wl.dkbar, s) != cudaSuccess)
    return SQB_ERR_CUDA;
  return SQB_OK;
}

}  // namespace

int simt_forward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                 float* lse, void* kbar, void* vbar, cudaStream_t stream) {
  if (p.D > 32 * kMaxPerLane) return SQB_ERR_UNSUPPORTED;
  if (p.dtype == SQB_F32) return forward_t<float>(p, q, k, v, o, lse, kbar, vbar, stream);
  return forward_t<__nv_bfloat16>(p, q, k, v, o, lse, kbar, vbar, stream);
}

int simt_backward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                  TensorView dout, const float* lse, const void* kbar, const void* vbar,
                  TensorView dq, TensorView dk, TensorView dv, uint8_t* ws,
                  const WorkspaceLayout& wl, cudaStream_t stream) {
  if (p.D > 32 * kMaxPerLane) return SQB_ERR_UNSUPPORTED;
  if (p.dtype == SQB_F32)
    return backward_t<float>(p, q, k, v, o, dout, lse, kbar, vbar, dq, dk, dv, ws, wl, stream);
  return backward_t<__nv_bfloat16>(p, q, k, v, o, dout, lse, kbar, vbar, dq, dk, dv, ws, wl,
                                   stream);
}

}  // namespace sqb
