// Reference-semantics mode: the attention core of the reference's registered
// sqrt_block / custom module (model/custom_attention.py:138), on CUDA cores.
//
// Per (batch n, head h), T = G * L tokens with G = L = sqrt(T)
// (block_geometry, custom_attention.py:68-79):
//   local_i   = causal softmax(Q_i K_i^T * scale)              :195-198
//   summary_i = column sums of local_i (length L)               :203
//   glob      = strictly-causal softmax(summary summary^T / sqrt(L)), row 0 zero
//                                                               :209-213
//   P_i       = local_i V_i,  out_i = P_i + sum_{j<i} glob[i,j] P_j
//                                                               _ScaledBlockCombine :99-109
// The backward is the analytic gradient of that composition (the combine's
// backward :111-135, then the glob and local softmax backwards, the summary's
// gradient reaching every row of its block).  fp32 arithmetic throughout for
// fp32 and bf16 inputs; L <= 64 and D <= 128 (the reference runs L = 16..32).
//
// Kernels, one CTA of 256 threads per (block i, batch*head) or per batch*head:
//   fwd: local_summary_p (local map, summary, P), glob_softmax, combine (one
//        CTA per row l of every block: each P row read once)
//   bwd: local_summary_p (P recomputed: the forward's workspace copy may have
//        been overwritten by another layer of the same shape), dp_dglob (per
//        row l like the combine; d_glob as L row shares), dglob_dsummary,
//        local_grads (dQ, dK, dV)
// For bf16 inputs with L in {16, 32, 64} and D in {64, 128} the local passes
// (local_summary_p and local_grads) run on the tensor cores instead
// (sqb_refsem_sm100.cu): 128-row tiles of whole blocks, bf16 operands, fp32
// accumulation and fp32 softmax arithmetic.

#include <math.h>

#include "sqb_internal.cuh"
#include "sqb_refsem_sm100.cuh"

namespace sqb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxL = 64;
constexpr int kMaxD = 128;

__device__ __forceinline__ float ld_f(const float* p) { return *p; }
__device__ __forceinline__ float ld_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st_f(float* p, float x) { *p = x; }
__device__ __forceinline__ void st_f(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }

struct RefsemParams {
  int H, G, L, D;
  float scale;      // on q.k
  float inv_sqrt_l; // on summary.summary
};

template <typename E>
__device__ __forceinline__ const E* at(const TensorView& t, int n, int tok, int h) {
  return reinterpret_cast<const E*>(t.ptr) + (int64_t)n * t.sb + (int64_t)tok * t.st +
         (int64_t)h * t.sh;
}
template <typename E>
__device__ __forceinline__ E* at_w(const TensorView& t, int n, int tok, int h) {
  return reinterpret_cast<E*>(t.ptr) + (int64_t)n * t.sb + (int64_t)tok * t.st +
         (int64_t)h * t.sh;
}

// Row pitch of the L x D fp32 tiles in shared memory: D + 1, so that a warp
// whose lanes read the same column d of 32 different rows (the q.k and dP.v
// products, lanes along the key index) hits 32 different banks; with a pitch
// of D (a multiple of 32) all 32 lanes hit one bank.
__host__ __device__ __forceinline__ int tile_pitch(int D) { return D + 1; }

// Block i's L x D rows of a (B, T, H, D) view into shared memory as fp32, rows
// ld floats apart (the padded pitch unless a kernel reads the tile along rows only).
template <typename E>
__device__ void load_tile(float* dst, const TensorView& t, int n, int h, int i,
                          const RefsemParams& p, int ld) {
  for (int e = threadIdx.x; e < p.L * p.D; e += kThreads) {
    const int l = e / p.D, d = e % p.D;
    dst[l * ld + d] = ld_f(at<E>(t, n, i * p.L + l, h) + d);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// local = causal softmax(q k^T * scale) of one block, L x L in shared memory
// (zero above the diagonal).  q, k: L x D fp32 tiles.
__device__ void local_map(float* local, const float* q, const float* k, const RefsemParams& p) {
  const int L = p.L, D = p.D, ld = tile_pitch(D);
  for (int e = threadIdx.x; e < L * L; e += kThreads) {
    const int l = e / L, m = e % L;
    float s = 0.f;
    if (m <= l) {
      for (int d = 0; d < D; ++d) s += q[l * ld + d] * k[m * ld + d];
      s *= p.scale;
    }
    local[e] = s;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int l = warp; l < L; l += kThreads / 32) {
    float mx = -INFINITY;
    for (int m = lane; m <= l; m += 32) mx = fmaxf(mx, local[l * L + m]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int m = lane; m < L; m += 32) {
      const float e = m <= l ? expf(local[l * L + m] - mx) : 0.f;
      local[l * L + m] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    for (int m = lane; m < L; m += 32) local[l * L + m] *= inv;
  }
  __syncthreads();
}

// Per (block i, bh): local map; summary (if requested); P_i = local V_i into P.
template <typename E>
__global__ void __launch_bounds__(kThreads) local_summary_p_kernel(
    TensorView q, TensorView k, TensorView v, float* summary, float* P, RefsemParams p) {
  extern __shared__ float sm[];
  const int i = blockIdx.x, bh = blockIdx.y, n = bh / p.H, h = bh % p.H;
  const int L = p.L, D = p.D, ld = tile_pitch(D);
  float* sq = sm;
  float* sk = sq + L * ld;
  float* sv = sk + L * ld;
  float* local = sv + L * ld;
  load_tile<E>(sq, q, n, h, i, p, ld);
  load_tile<E>(sk, k, n, h, i, p, ld);
  load_tile<E>(sv, v, n, h, i, p, ld);
  __syncthreads();
  local_map(local, sq, sk, p);
  if (summary) {
    for (int m = threadIdx.x; m < L; m += kThreads) {
      float s = 0.f;
      for (int l = m; l < L; ++l) s += local[l * L + m];
      summary[((size_t)bh * p.G + i) * L + m] = s;
    }
  }
  float* Pi = P + ((size_t)bh * p.G + i) * L * D;
  for (int e = threadIdx.x; e < L * D; e += kThreads) {
    const int l = e / D, d = e % D;
    float acc = 0.f;
    for (int m = 0; m <= l; ++m) acc += local[l * L + m] * sv[m * ld + d];
    Pi[e] = acc;
  }
}

// Per bh: glob = strictly-causal softmax of summary . summary^T / sqrt(L),
// row 0 all zero.
__global__ void __launch_bounds__(kThreads) glob_kernel(const float* summary, float* glob,
                                                        RefsemParams p) {
  extern __shared__ float sm[];
  const int bh = blockIdx.x, G = p.G, L = p.L;
  float* s = sm;            // G x L
  float* gs = s + G * L;    // G x G
  const float* sb = summary + (size_t)bh * G * L;
  for (int e = threadIdx.x; e < G * L; e += kThreads) s[e] = sb[e];
  __syncthreads();
  for (int e = threadIdx.x; e < G * G; e += kThreads) {
    const int a = e / G, c = e % G;
    float acc = 0.f;
    if (c < a)
      for (int m = 0; m < L; ++m) acc += s[a * L + m] * s[c * L + m];
    gs[e] = acc * p.inv_sqrt_l;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* gb = glob + (size_t)bh * G * G;
  for (int a = warp; a < G; a += kThreads / 32) {
    float mx = -INFINITY;
    for (int c = lane; c < a; c += 32) mx = fmaxf(mx, gs[a * G + c]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int c = lane; c < a; c += 32) sum += expf(gs[a * G + c] - mx);
    sum = warp_sum(sum);
    for (int c = lane; c < G; c += 32)
      gb[a * G + c] = c < a ? expf(gs[a * G + c] - mx) / sum : 0.f;
  }
}

// Per (row l of every block, bh): out_i[l] = P_i[l] + sum_{j<i} glob[i, j] P_j[l]
// for every block i.  Each P row is read once; the glob matrix and the G rows
// l of P sit in shared memory.
template <typename E>
__global__ void __launch_bounds__(kThreads) combine_kernel(const float* P, const float* glob,
                                                           TensorView o, RefsemParams p) {
  extern __shared__ float sm[];
  const int l = blockIdx.x, bh = blockIdx.y, n = bh / p.H, h = bh % p.H;
  const int L = p.L, D = p.D, G = p.G;
  float* sg = sm;           // G x G
  float* sp = sg + G * G;   // G x D: row l of every block
  const float* gb = glob + (size_t)bh * G * G;
  for (int e = threadIdx.x; e < G * G; e += kThreads) sg[e] = gb[e];
  for (int e = threadIdx.x; e < G * D; e += kThreads) {
    const int i = e / D, d = e % D;
    sp[e] = P[(((size_t)bh * G + i) * L + l) * D + d];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += kThreads) {
    const int i = e / D, d = e % D;
    float acc = sp[e];
    for (int j = 0; j < i; ++j) acc += sg[i * G + j] * sp[j * D + d];
    st_f(at_w<E>(o, n, i * L + l, h) + d, acc);
  }
}

// Per (row l of every block, bh): dP_j[l] = dO_j[l] + sum_{i>j} glob[i, j] dO_i[l]
// for every block j, and this row's share of d_glob:
// part[l][j, c] = <dO_j[l], P_c[l]> for c < j (zero otherwise).  d_glob is the
// sum of the L shares, added in a fixed order by dglob_dsummary_kernel.
template <typename E>
__global__ void __launch_bounds__(kThreads) dp_dglob_kernel(TensorView dout, const float* P,
                                                            const float* glob, float* dP,
                                                            float* dglob_part, RefsemParams p) {
  extern __shared__ float sm[];
  const int l = blockIdx.x, bh = blockIdx.y, n = bh / p.H, h = bh % p.H;
  const int L = p.L, D = p.D, G = p.G, ld = D + 1;
  float* sg = sm;            // G x G
  float* sdo = sg + G * G;   // G x ld: row l of every block's dO (padded pitch)
  float* sp = sdo + G * ld;  // G x ld: row l of every block's P
  const float* gb = glob + (size_t)bh * G * G;
  for (int e = threadIdx.x; e < G * G; e += kThreads) sg[e] = gb[e];
  for (int e = threadIdx.x; e < G * D; e += kThreads) {
    const int i = e / D, d = e % D;
    sdo[i * ld + d] = ld_f(at<E>(dout, n, i * L + l, h) + d);
    sp[i * ld + d] = P[(((size_t)bh * G + i) * L + l) * D + d];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += kThreads) {
    const int j = e / D, d = e % D;
    float acc = sdo[j * ld + d];
    for (int i = j + 1; i < G; ++i) acc += sg[i * G + j] * sdo[i * ld + d];
    dP[(((size_t)bh * G + j) * L + l) * D + d] = acc;
  }
  float* part = dglob_part + ((size_t)bh * L + l) * G * G;
  for (int e = threadIdx.x; e < G * G; e += kThreads) {
    const int j = e / G, c = e % G;
    float acc = 0.f;
    if (c < j)
      for (int d = 0; d < D; ++d) acc += sdo[j * ld + d] * sp[c * ld + d];
    part[e] = acc;
  }
}

// Per bh: d_glob = the sum of the L row shares (in row order); d_gs = glob *
// (d_glob - rowsum(glob * d_glob)); d_summary = (d_gs + d_gs^T) summary / sqrt(L).
__global__ void __launch_bounds__(kThreads) dglob_dsummary_kernel(const float* glob,
                                                                  const float* dglob_part,
                                                                  const float* summary,
                                                                  float* dsum, RefsemParams p) {
  extern __shared__ float sm[];
  const int bh = blockIdx.x, G = p.G, L = p.L;
  float* dgs = sm;          // G x G
  float* s = dgs + G * G;   // G x L
  float* db = s + G * L;    // G x G: d_glob
  const float* gb = glob + (size_t)bh * G * G;
  const float* pb = dglob_part + (size_t)bh * L * G * G;
  for (int e = threadIdx.x; e < G * G; e += kThreads) {
    // eight independent partial sums (rows l = u mod 8), combined in a fixed
    // order: the loads of one element overlap instead of forming one chain
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int l = 0;
    for (; l + 8 <= L; l += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] += pb[(size_t)(l + u) * G * G + e];
    }
    for (; l < L; ++l) a[0] += pb[(size_t)l * G * G + e];
    db[e] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
  }
  for (int e = threadIdx.x; e < G * L; e += kThreads) s[e] = summary[(size_t)bh * G * L + e];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int a = warp; a < G; a += kThreads / 32) {
    float r = 0.f;
    for (int c = lane; c < a; c += 32) r += gb[a * G + c] * db[a * G + c];
    r = warp_sum(r);
    for (int c = lane; c < G; c += 32)
      dgs[a * G + c] = c < a ? gb[a * G + c] * (db[a * G + c] - r) : 0.f;
  }
  __syncthreads();
  float* out = dsum + (size_t)bh * G * L;
  for (int e = threadIdx.x; e < G * L; e += kThreads) {
    const int a = e / L, m = e % L;
    float acc = 0.f;
    for (int c = 0; c < G; ++c) acc += (dgs[a * G + c] + dgs[c * G + a]) * s[c * L + m];
    out[e] = acc * p.inv_sqrt_l;
  }
}

// Per (block i, bh): local recomputed; d_local = dP_i V_i^T + d_summary_i (every
// row); dS = local * (d_local - rowsum(local * d_local)); dQ = dS K * scale,
// dK = dS^T Q * scale, dV = local^T dP_i.
template <typename E>
__global__ void __launch_bounds__(kThreads) local_grads_kernel(
    TensorView q, TensorView k, TensorView v, const float* dP, const float* dsum,
    TensorView dq, TensorView dk, TensorView dv, RefsemParams p) {
  extern __shared__ float sm[];
  const int i = blockIdx.x, bh = blockIdx.y, n = bh / p.H, h = bh % p.H;
  const int L = p.L, D = p.D, ld = tile_pitch(D);
  float* sq = sm;
  float* sk = sq + L * ld;
  float* sv = sk + L * ld;
  float* sdp = sv + L * ld;
  float* local = sdp + L * ld;
  float* ds = local + L * L;
  load_tile<E>(sq, q, n, h, i, p, ld);
  load_tile<E>(sk, k, n, h, i, p, ld);
  load_tile<E>(sv, v, n, h, i, p, ld);
  const float* dPi = dP + ((size_t)bh * p.G + i) * L * D;
  for (int e = threadIdx.x; e < L * D; e += kThreads) sdp[(e / D) * ld + e % D] = dPi[e];
  __syncthreads();
  local_map(local, sq, sk, p);
  const float* dsi = dsum + ((size_t)bh * p.G + i) * L;
  for (int e = threadIdx.x; e < L * L; e += kThreads) {
    const int l = e / L, m = e % L;
    float g = 0.f;
    if (m <= l) {
      for (int d = 0; d < D; ++d) g += sdp[l * ld + d] * sv[m * ld + d];
      g += dsi[m];
    }
    ds[e] = g;  // d_local for now
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int l = warp; l < L; l += kThreads / 32) {
    float r = 0.f;
    for (int m = lane; m <= l; m += 32) r += local[l * L + m] * ds[l * L + m];
    r = warp_sum(r);
    for (int m = lane; m < L; m += 32)
      ds[l * L + m] = m <= l ? local[l * L + m] * (ds[l * L + m] - r) : 0.f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < L * D; e += kThreads) {
    const int r = e / D, d = e % D;
    float gq = 0.f, gk = 0.f, gv = 0.f;
    for (int m = 0; m <= r; ++m) gq += ds[r * L + m] * sk[m * ld + d];  // row r as query
    for (int l = r; l < L; ++l) {                                       // row r as key
      gk += ds[l * L + r] * sq[l * ld + d];
      gv += local[l * L + r] * sdp[l * ld + d];
    }
    st_f(at_w<E>(dq, n, i * L + r, h) + d, gq * p.scale);
    st_f(at_w<E>(dk, n, i * L + r, h) + d, gk * p.scale);
    st_f(at_w<E>(dv, n, i * L + r, h) + d, gv);
  }
}

struct RefsemWorkspace {
  size_t P, dP, dglob_part, dsum, status, total;
};

RefsemWorkspace refsem_layout(int64_t B, int64_t T, int64_t H, int64_t D) {
  RefsemWorkspace w{};
  const int64_t BH = B * H;
  const int64_t L = (int64_t)llround(sqrt((double)T));
  size_t off = 0;
  w.P = off;
  off = align_up(off + (size_t)BH * T * D * 4, 256);
  w.dP = off;
  off = align_up(off + (size_t)BH * T * D * 4, 256);
  w.dglob_part = off;  // (B*H, L, G, G) row shares of d_glob (G = L)
  off = align_up(off + (size_t)BH * L * L * L * 4, 256);
  w.dsum = off;
  off = align_up(off + (size_t)BH * L * L * 4, 256);
  w.status = off;  // status words of the tensor-core kernel's waits
  off = align_up(off + 64, 256);
  w.total = off;
  return w;
}

// 0 when T is a perfect square with L <= kMaxL and the other sizes fit, else an
// error code (SQB_ERR_ARG for a T the reference itself rejects).
int refsem_check(int64_t B, int64_t T, int64_t H, int64_t D, int* L) {
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0) return SQB_ERR_ARG;
  if (B * H > 65535) return SQB_ERR_UNSUPPORTED;
  int64_t r = (int64_t)llround(sqrt((double)T));
  while (r * r > T) --r;
  while ((r + 1) * (r + 1) <= T) ++r;
  if (r * r != T) return SQB_ERR_ARG;
  if (r > kMaxL || D > kMaxD) return SQB_ERR_UNSUPPORTED;
  *L = (int)r;
  return SQB_OK;
}

TensorView tview(const void* ptr, const int64_t* s) {
  return TensorView{const_cast<void*>(ptr), s[0], s[1], s[2]};
}

bool strides_ok(const TensorView& t) { return t.ptr && t.st > 0 && t.sh > 0 && t.sb > 0; }

template <typename K>
bool set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
         cudaSuccess;
}

// The local maps, summaries (when requested) and P of every block: on the
// tensor cores where refsem_tc_supported holds (bf16, L in {16, 32, 64}, D in
// {64, 128}), else on CUDA cores.
template <typename E>
int local_pass(TensorView q, TensorView k, TensorView v, float* summary, float* P, uint8_t* ws,
               const RefsemWorkspace& wl, int B, const RefsemParams& p, int dtype,
               cudaStream_t s) {
  if (refsem_tc_supported(p.L, p.D, dtype, {q, k, v})) {
    uint32_t* status = reinterpret_cast<uint32_t*>(ws + wl.status);
    if (cudaMemsetAsync(status, 0, 3 * sizeof(uint32_t), s) != cudaSuccess) return SQB_ERR_CUDA;
    return refsem_tc_local(q, k, v, summary, P, B, p.G * p.L, p.H, p.D, p.L, p.scale, status,
                           s);
  }
  const size_t sm1 = (size_t)(3 * p.L * tile_pitch(p.D) + p.L * p.L) * 4;
  if (!set_smem(local_summary_p_kernel<E>, sm1)) return SQB_ERR_LAUNCH;
  local_summary_p_kernel<E><<<dim3(p.G, B * p.H), kThreads, sm1, s>>>(q, k, v, summary, P, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

template <typename E>
int refsem_forward(TensorView q, TensorView k, TensorView v, TensorView o, float* glob,
                   float* summary, uint8_t* ws, const RefsemWorkspace& wl, int B,
                   const RefsemParams& p, int dtype, cudaStream_t s) {
  float* P = reinterpret_cast<float*>(ws + wl.P);
  const int BH = B * p.H;
  const size_t sm2 = (size_t)(p.G * p.L + p.G * p.G) * 4;
  if (!set_smem(glob_kernel, sm2)) return SQB_ERR_LAUNCH;
  const size_t sm3 = (size_t)(p.G * p.G + p.G * p.D) * 4;
  if (!set_smem(combine_kernel<E>, sm3)) return SQB_ERR_LAUNCH;
  if (int e = local_pass<E>(q, k, v, summary, P, ws, wl, B, p, dtype, s)) return e;
  glob_kernel<<<BH, kThreads, sm2, s>>>(summary, glob, p);
  combine_kernel<E><<<dim3(p.L, BH), kThreads, sm3, s>>>(P, glob, o, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

template <typename E>
int refsem_backward(TensorView q, TensorView k, TensorView v, TensorView dout, const float* glob,
                    const float* summary, TensorView dq, TensorView dk, TensorView dv,
                    uint8_t* ws, const RefsemWorkspace& wl, int B, const RefsemParams& p,
                    int dtype, cudaStream_t s) {
  const int BH = B * p.H;
  float* P = reinterpret_cast<float*>(ws + wl.P);
  float* dP = reinterpret_cast<float*>(ws + wl.dP);
  float* dglob_part = reinterpret_cast<float*>(ws + wl.dglob_part);
  float* dsum = reinterpret_cast<float*>(ws + wl.dsum);
  const size_t sm2 = (size_t)(p.G * p.G + 2 * p.G * (p.D + 1)) * 4;
  const size_t sm3 = (size_t)(2 * p.G * p.G + p.G * p.L) * 4;
  const size_t sm4 = (size_t)(4 * p.L * tile_pitch(p.D) + 2 * p.L * p.L) * 4;
  if (!set_smem(dp_dglob_kernel<E>, sm2) || !set_smem(dglob_dsummary_kernel, sm3) ||
      !set_smem(local_grads_kernel<E>, sm4))
    return SQB_ERR_LAUNCH;
  if (int e = local_pass<E>(q, k, v, nullptr, P, ws, wl, B, p, dtype, s)) return e;
  dp_dglob_kernel<E><<<dim3(p.L, BH), kThreads, sm2, s>>>(dout, P, glob, dP, dglob_part, p);
  dglob_dsummary_kernel<<<BH, kThreads, sm3, s>>>(glob, dglob_part, summary, dsum, p);
  if (refsem_tc_supported(p.L, p.D, dtype, {q, k, v, dq, dk, dv})) {
    uint32_t* status = reinterpret_cast<uint32_t*>(ws + wl.status);
    if (int e = refsem_tc_grads(q, k, v, dP, dsum, dq, dk, dv, B, p.G * p.L, p.H, p.D, p.L,
                                p.scale, status, s))
      return e;
    return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
  }
  local_grads_kernel<E><<<dim3(p.G, BH), kThreads, sm4, s>>>(q, k, v, dP, dsum, dq, dk, dv, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

}  // namespace
}  // namespace sqb

using namespace sqb;

extern "C" {

size_t sqb_refsem_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D) {
  int L;
  if (refsem_check(B, T, H, D, &L) != SQB_OK) return 0;
  return refsem_layout(B, T, H, D).total;
}

int sqb_refsem_fwd(const void* q, const void* k, const void* v, void* o, float* glob,
                   float* summary, int64_t B, int64_t T, int64_t H, int64_t D,
                   const int64_t* strides, int dtype, float scale, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int L;
  if (int e = refsem_check(B, T, H, D, &L)) return e;
  if (dtype != SQB_F32 && dtype != SQB_BF16) return SQB_ERR_DTYPE;
  if (!q || !k || !v || !o || !glob || !summary || !strides) return SQB_ERR_ARG;
  if (!(scale > 0.f) || !isfinite(scale)) return SQB_ERR_ARG;
  const RefsemWorkspace wl = refsem_layout(B, T, H, D);
  if (!workspace || workspace_bytes < wl.total) return SQB_ERR_WORKSPACE;
  TensorView tq = tview(q, strides), tk = tview(k, strides + 3), tv = tview(v, strides + 6),
             to = tview(o, strides + 9);
  if (!strides_ok(tq) || !strides_ok(tk) || !strides_ok(tv) || !strides_ok(to))
    return SQB_ERR_ARG;
  const RefsemParams p{(int)H, L, L, (int)D, scale, 1.f / sqrtf((float)L)};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();
  if (dtype == SQB_F32)
    return refsem_forward<float>(tq, tk, tv, to, glob, summary, (uint8_t*)workspace, wl,
                                 (int)B, p, dtype, s);
  return refsem_forward<__nv_bfloat16>(tq, tk, tv, to, glob, summary, (uint8_t*)workspace, wl,
                                       (int)B, p, dtype, s);
}

int sqb_refsem_bwd(const void* q, const void* k, const void* v, const void* dout,
                   const float* glob, const float* summary, void* dq, void* dk, void* dv,
                   int64_t B, int64_t T, int64_t H, int64_t D, const int64_t* strides,
                   int dtype, float scale, void* workspace, size_t workspace_bytes,
                   void* stream) {
  int L;
  if (int e = refsem_check(B, T, H, D, &L)) return e;
  if (dtype != SQB_F32 && dtype != SQB_BF16) return SQB_ERR_DTYPE;
  if (!q || !k || !v || !dout || !glob || !summary || !dq || !dk || !dv || !strides)
    return SQB_ERR_ARG;
  if (!(scale > 0.f) || !isfinite(scale)) return SQB_ERR_ARG;
  const RefsemWorkspace wl = refsem_layout(B, T, H, D);
  if (!workspace || workspace_bytes < wl.total) return SQB_ERR_WORKSPACE;
  TensorView tq = tview(q, strides), tk = tview(k, strides + 3), tv = tview(v, strides + 6),
             tdo = tview(dout, strides + 9), tdq = tview(dq, strides + 12),
             tdk = tview(dk, strides + 15), tdv = tview(dv, strides + 18);
  for (const TensorView& t : {tq, tk, tv, tdo, tdq, tdk, tdv})
    if (!strides_ok(t)) return SQB_ERR_ARG;
  const RefsemParams p{(int)H, L, L, (int)D, scale, 1.f / sqrtf((float)L)};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaGetLastError();
  if (dtype == SQB_F32)
    return refsem_backward<float>(tq, tk, tv, tdo, glob, summary, tdq, tdk, tdv,
                                  (uint8_t*)workspace, wl, (int)B, p, dtype, s);
  return refsem_backward<__nv_bfloat16>(tq, tk, tv, tdo, glob, summary, tdq, tdk, tdv,
                                        (uint8_t*)workspace, wl, (int)B, p, dtype, s);
}

}  // extern "C"
