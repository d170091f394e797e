// sm_100a tensor-core kernel of the reference-semantics mode: every block's
// local attention map, its column sums (the block summary) and
// P_i = local_i V_i (model/custom_attention.py:195-203 and the own-block term
// of _ScaledBlockCombine, :99-109), for bf16 inputs with block length
// L in {16, 32, 64} and D in {64, 128}.
//
// One CTA of four warps per 128-row tile of one (batch, head), i.e. 128 / L
// whole blocks:
//   S = Q K^T of the tile     tcgen05.mma, Q/K staged by TMA, S in TMEM
//   local row                 one thread per row (TMEM lane): the causal
//                             softmax of its L block scores in fp32
//   summary                   the local rows staged in shared memory as fp32,
//                             summed down each block's columns
//   P = local V               the local rows written back over S as bf16 (zero
//                             outside the row's block), tcgen05.mma with A
//                             from TMEM; P leaves as fp32 rows
// Every wait is bounded (mbarrier budget) and records SQB_ERR_TIMEOUT in the
// caller's status words.

#include "sqb_refsem_sm100.cuh"
#include "sqb_sm100.cuh"
#include "sqb_sm100_common.cuh"

namespace sqb {
namespace sm100 {
namespace {

struct RsParams {
  int H, T, G;       // heads, tokens, blocks per sequence (T / L)
  float scale_log2;  // softmax scale * log2(e)
  float* summary;    // (B*H, G, L) fp32, or null
  float* P;          // (B*H, T, D) fp32
  uint32_t* status;
};

constexpr int kRsThreads = 128;
constexpr int kRsPitch = 65;  // fp32 local rows in shared memory: L <= 64, plus one
constexpr uint32_t kRsCols = 256;  // TMEM: S at 0 (128 columns), P at 128 (D columns)

template <int D>
struct RsSmem {
  static constexpr int kTileBytes = (D / 64) * kAtomBytes;
  alignas(1024) uint8_t q[kTileBytes];
  alignas(1024) uint8_t k[kTileBytes];
  alignas(1024) uint8_t v[kTileBytes];
  float loc[128 * kRsPitch];
  uint64_t ld_full, s_full, p_full, o_full;
  uint32_t tmem_base;
};

template <int D, int kL>
__global__ void __launch_bounds__(kRsThreads) refsem_local_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const RsParams p) {
  extern __shared__ uint8_t smem_raw[];
  RsSmem<D>& sm = *reinterpret_cast<RsSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, bh = blockIdx.y, n = bh / p.H, h = bh % p.H;
  const int r0 = tile * 128;
  constexpr int kAtoms = D / 64;
  uint32_t* status = p.status;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&sm.ld_full, 1);
    ptx::mbar_init(&sm.s_full, 1);
    ptx::mbar_init(&sm.p_full, 4);  // one arrive per warp
    ptx::mbar_init(&sm.o_full, 1);
    ptx::fence_mbarrier_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&sm.tmem_base, kRsCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (threadIdx.x == 0) {
    ptx::mbar_arrive_expect_tx(&sm.ld_full, 3 * kAtoms * kAtomBytes);
#pragma unroll
    for (int a = 0; a < kAtoms; ++a) {
      ptx::tma_load_4d(sm.q + a * kAtomBytes, &tm_q, &sm.ld_full, a * 64, h, r0, n);
      ptx::tma_load_4d(sm.k + a * kAtomBytes, &tm_k, &sm.ld_full, a * 64, h, r0, n);
      ptx::tma_load_4d(sm.v + a * kAtomBytes, &tm_v, &sm.ld_full, a * 64, h, r0, n);
    }
    ptx::mbar_wait(&sm.ld_full, 0, status, 0x90000000u);
    ptx::tc_fence_after();
    const uint32_t q_s = ptx::smem_u32(sm.q), k_s = ptx::smem_u32(sm.k);
    constexpr uint32_t idesc_s = ptx::idesc_bf16(128, 128, false, false);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      ptx::mma_ss(tmem, desc_kmajor(q_s, kk), desc_kmajor(k_s, kk), idesc_s, kk > 0 ? 1u : 0u);
    ptx::mma_commit(&sm.s_full);
  }
  __syncwarp();

  // ---- one row per thread: the causal softmax of its block's scores
  const int row = warp * 32 + lane;  // TMEM lane = tile row
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  constexpr int kW = kL > 32 ? kL : 32;        // key columns a warp loads (warp-uniform)
  const int wc0 = (warp * 32 / kW) * kW;       // the warp's first key column
  const int c0 = (row / kL) * kL;              // the row's block's first key column
  const int l = row - c0;                      // row within its block
  ptx::mbar_wait(&sm.s_full, 0, status, 0x91000000u);
  ptx::tc_fence_after();
  uint32_t sr[kW];
#pragma unroll
  for (int pc = 0; pc < kW / 16; ++pc)
    ptx::tmem_ld16(tmem + lane_off + wc0 + pc * 16,
                   *reinterpret_cast<uint32_t(*)[16]>(sr + pc * 16));
  ptx::tmem_wait_ld();
  ptx::reg_fence(sr);
  // the row's L scores start at column c0 - wc0 of the loaded window (16 for
  // the second block of a warp when L = 16, else 0)
  const bool upper = kL == 16 && c0 != wc0;
  float e[kL];
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < kL; ++m) {
    const uint32_t raw = (kL == 16) ? (upper ? sr[16 + (m & 15)] : sr[m & 15]) : sr[m];
    e[m] = m <= l ? __uint_as_float(raw) * p.scale_log2 : -INFINITY;
    mx = fmaxf(mx, e[m]);
  }
  float sum = 0.f;
#pragma unroll
  for (int m = 0; m < kL; ++m) {
    e[m] = m <= l ? ptx::ex2(e[m] - mx) : 0.f;
    sum += e[m];
  }
  const float inv = 1.f / sum;
  float* lrow = sm.loc + row * kRsPitch;
#pragma unroll
  for (int m = 0; m < kL; ++m) lrow[m] = e[m] * inv;

  // local as bf16 over S (keys 16q..16q+15 -> TMEM columns 8q..8q+7), zero
  // outside the row's block; every row was read above before any is written
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint32_t pk[8];
    const bool in_window = q * 16 >= wc0 && q * 16 < wc0 + kW;  // warp-uniform
    const bool mine = q * 16 >= c0 && q * 16 < c0 + kL;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      pk[j] = 0u;
      if (in_window && mine) {
        const int m = q * 16 - c0 + 2 * j;
        pk[j] = ptx::pack_bf16x2(lrow[m], lrow[m + 1]);
      }
    }
    ptx::tmem_st8(tmem + lane_off + q * 8, pk);
  }
  ptx::tmem_wait_st();
  ptx::tc_fence_before();
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(&sm.p_full);

  if (threadIdx.x == 0) {
    ptx::mbar_wait(&sm.p_full, 0, status, 0x92000000u);
    ptx::tc_fence_after();
    const uint32_t v_s = ptx::smem_u32(sm.v);
    constexpr uint32_t idesc_pv = ptx::idesc_bf16(128, D, false, true);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)  // P = local V over the tile's 128 keys
      ptx::mma_ts(tmem + 128, tmem + kk * 8, desc_mnmajor(v_s, kk), idesc_pv,
                  kk > 0 ? 1u : 0u);
    ptx::mma_commit(&sm.o_full);
  }
  __syncwarp();

  // ---- summaries: column sums of each block's local map (fp32)
  __syncthreads();
  if (p.summary) {
    const int t = threadIdx.x, blk = t / kL, m = t % kL;
    float s = 0.f;
    for (int r = m; r < kL; ++r) s += sm.loc[(blk * kL + r) * kRsPitch + m];
    p.summary[((size_t)bh * p.G + tile * (128 / kL) + blk) * kL + m] = s;
  }

  // ---- P rows out as fp32
  ptx::mbar_wait(&sm.o_full, 0, status, 0x93000000u);
  ptx::tc_fence_after();
  float* prow = p.P + ((size_t)bh * p.T + r0 + row) * D;
#pragma unroll 1
  for (int pc = 0; pc < D / 32; ++pc) {
    uint32_t r[32];
    ptx::tmem_ld32(tmem + lane_off + 128 + pc * 32, r);
    ptx::tmem_wait_ld();
    ptx::reg_fence(r);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      reinterpret_cast<float4*>(prow + pc * 32)[j] =
          make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                      __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kRsCols);
  }
}

// ---- backward: dQ, dK, dV of every block's local attention
//
// Per 128-row tile, with dP = dO_i + sum_{j>i} glob[j, i] dO_j (fp32, from the
// combine's backward) and d_summary (fp32) of its blocks:
//   S = Q K^T and G = dP V^T         tcgen05.mma (dP staged as bf16)
//   local row, g = G + d_summary     one thread per row, fp32:
//   dS = local * (g - rowsum(local * g))
//   dQ = dS K * scale, dK = dS^T Q * scale, dV = local^T dP
//                                    tcgen05.mma from local and dS staged as
//                                    bf16 (zero outside each row's block)
// The gradient rows leave through the caller's (B, T, H, D) bf16 views.

struct RgParams {
  int H, T, G;
  float scale;       // on q.k
  float scale_log2;  // scale * log2(e)
  const float* dP;   // (B*H, T, D) fp32
  const float* dsum; // (B*H, G, L) fp32
  TensorView dq, dk, dv;
  uint32_t* status;
};

template <int D>
struct RgSmem {
  static constexpr int kTileBytes = (D / 64) * kAtomBytes;
  alignas(1024) uint8_t q[kTileBytes];
  alignas(1024) uint8_t k[kTileBytes];
  alignas(1024) uint8_t v[kTileBytes];
  alignas(1024) uint8_t dp[kTileBytes];    // dP rows as bf16
  alignas(1024) uint8_t lo[2 * kAtomBytes];  // local rows as bf16 (128 keys)
  alignas(1024) uint8_t ds[2 * kAtomBytes];  // dS rows as bf16
  uint64_t ld_full, s_full, ps_full, o_full;
  uint32_t tmem_base;
};

// TMEM: S at 0 and G at 128; after both are read, dQ at 0, dK at D, dV at 2D.
template <int D>
constexpr uint32_t rg_tmem_cols() {
  return D == 64 ? 256u : 512u;
}

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const uint32_t (&r)[32],
                                               float mul) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    reinterpret_cast<uint4*>(dst)[j] = make_uint4(
        ptx::pack_bf16x2(__uint_as_float(r[8 * j]) * mul, __uint_as_float(r[8 * j + 1]) * mul),
        ptx::pack_bf16x2(__uint_as_float(r[8 * j + 2]) * mul,
                         __uint_as_float(r[8 * j + 3]) * mul),
        ptx::pack_bf16x2(__uint_as_float(r[8 * j + 4]) * mul,
                         __uint_as_float(r[8 * j + 5]) * mul),
        ptx::pack_bf16x2(__uint_as_float(r[8 * j + 6]) * mul,
                         __uint_as_float(r[8 * j + 7]) * mul));
}

template <int D, int kL>
__global__ void __launch_bounds__(kRsThreads) refsem_grads_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const RgParams p) {
  extern __shared__ uint8_t smem_raw[];
  RgSmem<D>& sm = *reinterpret_cast<RgSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, bh = blockIdx.y, n = bh / p.H, h = bh % p.H;
  const int r0 = tile * 128;
  constexpr int kAtoms = D / 64;
  constexpr uint32_t kCols = rg_tmem_cols<D>();
  uint32_t* status = p.status;
  const int row = warp * 32 + lane;  // TMEM lane = tile row (a query, then a key)
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&sm.ld_full, 1);
    ptx::mbar_init(&sm.s_full, 1);
    ptx::mbar_init(&sm.ps_full, 4);  // one arrive per warp
    ptx::mbar_init(&sm.o_full, 1);
    ptx::fence_mbarrier_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&sm.tmem_base, kCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (threadIdx.x == 0) {
    ptx::mbar_arrive_expect_tx(&sm.ld_full, 3 * kAtoms * kAtomBytes);
#pragma unroll
    for (int a = 0; a < kAtoms; ++a) {
      ptx::tma_load_4d(sm.q + a * kAtomBytes, &tm_q, &sm.ld_full, a * 64, h, r0, n);
      ptx::tma_load_4d(sm.k + a * kAtomBytes, &tm_k, &sm.ld_full, a * 64, h, r0, n);
      ptx::tma_load_4d(sm.v + a * kAtomBytes, &tm_v, &sm.ld_full, a * 64, h, r0, n);
    }
  }
  __syncwarp();
  // this row's dP as bf16 into the swizzled dP tile
  {
    const float4* src =
        reinterpret_cast<const float4*>(p.dP + ((size_t)bh * p.T + r0 + row) * D);
#pragma unroll 2
    for (int c = 0; c < D / 8; ++c) {
      const float4 a = src[2 * c], b = src[2 * c + 1];
      *reinterpret_cast<uint4*>(sm.dp + swz_offset(row, c * 8)) =
          make_uint4(ptx::pack_bf16x2(a.x, a.y), ptx::pack_bf16x2(a.z, a.w),
                     ptx::pack_bf16x2(b.x, b.y), ptx::pack_bf16x2(b.z, b.w));
    }
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x == 0) {
    ptx::mbar_wait(&sm.ld_full, 0, status, 0x94000000u);
    ptx::tc_fence_after();
    const uint32_t q_s = ptx::smem_u32(sm.q), k_s = ptx::smem_u32(sm.k);
    const uint32_t v_s = ptx::smem_u32(sm.v), dp_s = ptx::smem_u32(sm.dp);
    constexpr uint32_t idesc_s = ptx::idesc_bf16(128, 128, false, false);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)  // S = Q K^T
      ptx::mma_ss(tmem, desc_kmajor(q_s, kk), desc_kmajor(k_s, kk), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)  // G = dP V^T
      ptx::mma_ss(tmem + 128, desc_kmajor(dp_s, kk), desc_kmajor(v_s, kk), idesc_s,
                  kk > 0 ? 1u : 0u);
    ptx::mma_commit(&sm.s_full);
  }
  __syncwarp();

  // ---- one row per thread: local, g, dS in fp32 over the row's block
  constexpr int kW = kL > 32 ? kL : 32;
  const int wc0 = (warp * 32 / kW) * kW;
  const int c0 = (row / kL) * kL;
  const int l = row - c0;
  const bool upper = kL == 16 && c0 != wc0;
  ptx::mbar_wait(&sm.s_full, 0, status, 0x95000000u);
  ptx::tc_fence_after();
  float e[kL], g[kL];
  {
    uint32_t sr[kW];
#pragma unroll
    for (int pc = 0; pc < kW / 16; ++pc)
      ptx::tmem_ld16(tmem + lane_off + wc0 + pc * 16,
                     *reinterpret_cast<uint32_t(*)[16]>(sr + pc * 16));
    ptx::tmem_wait_ld();
    ptx::reg_fence(sr);
#pragma unroll
    for (int m = 0; m < kL; ++m) {
      const uint32_t raw = (kL == 16) ? (upper ? sr[16 + (m & 15)] : sr[m & 15]) : sr[m];
      e[m] = __uint_as_float(raw);
    }
#pragma unroll
    for (int pc = 0; pc < kW / 16; ++pc)
      ptx::tmem_ld16(tmem + lane_off + 128 + wc0 + pc * 16,
                     *reinterpret_cast<uint32_t(*)[16]>(sr + pc * 16));
    ptx::tmem_wait_ld();
    ptx::reg_fence(sr);
#pragma unroll
    for (int m = 0; m < kL; ++m) {
      const uint32_t raw = (kL == 16) ? (upper ? sr[16 + (m & 15)] : sr[m & 15]) : sr[m];
      g[m] = __uint_as_float(raw);
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < kL; ++m) {
    e[m] = m <= l ? e[m] * p.scale_log2 : -INFINITY;
    mx = fmaxf(mx, e[m]);
  }
  float sum = 0.f;
#pragma unroll
  for (int m = 0; m < kL; ++m) {
    e[m] = m <= l ? ptx::ex2(e[m] - mx) : 0.f;
    sum += e[m];
  }
  const float inv = 1.f / sum;
  const float* dsr = p.dsum + ((size_t)bh * p.G + (r0 + c0) / kL) * kL;
  float rsum = 0.f;
#pragma unroll
  for (int m = 0; m < kL; ++m) {
    e[m] *= inv;                                   // local
    g[m] = m <= l ? g[m] + __ldg(dsr + m) : 0.f;   // d_local
    rsum += e[m] * g[m];
  }
  // local and dS rows as bf16 over the tile's 128 keys: zero outside the
  // row's block, then the block's own 8-key chunks (static register indices,
  // the shared-memory address carries the block's position)
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    if (c * 8 < c0 || c * 8 >= c0 + kL) {
      *reinterpret_cast<uint4*>(sm.lo + swz_offset(row, c * 8)) = z4;
      *reinterpret_cast<uint4*>(sm.ds + swz_offset(row, c * 8)) = z4;
    }
  }
#pragma unroll
  for (int cr = 0; cr < kL / 8; ++cr) {
    uint32_t pl[4], pd[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = cr * 8 + 2 * j;
      pl[j] = ptx::pack_bf16x2(e[m], e[m + 1]);
      pd[j] = ptx::pack_bf16x2(e[m] * (g[m] - rsum), e[m + 1] * (g[m + 1] - rsum));
    }
    *reinterpret_cast<uint4*>(sm.lo + swz_offset(row, c0 + cr * 8)) =
        make_uint4(pl[0], pl[1], pl[2], pl[3]);
    *reinterpret_cast<uint4*>(sm.ds + swz_offset(row, c0 + cr * 8)) =
        make_uint4(pd[0], pd[1], pd[2], pd[3]);
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(&sm.ps_full);

  if (threadIdx.x == 0) {
    ptx::mbar_wait(&sm.ps_full, 0, status, 0x96000000u);
    ptx::tc_fence_after();
    const uint32_t q_s = ptx::smem_u32(sm.q), k_s = ptx::smem_u32(sm.k);
    const uint32_t dp_s = ptx::smem_u32(sm.dp);
    const uint32_t lo_s = ptx::smem_u32(sm.lo), ds_s = ptx::smem_u32(sm.ds);
    constexpr uint32_t idesc_dq = ptx::idesc_bf16(128, D, false, true);
    constexpr uint32_t idesc_kv = ptx::idesc_bf16(128, D, true, true);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)  // dQ = dS K (keys)
      ptx::mma_ss(tmem, desc_kmajor(ds_s, kk), desc_mnmajor(k_s, kk), idesc_dq,
                  kk > 0 ? 1u : 0u);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)  // dK = dS^T Q (queries)
      ptx::mma_ss(tmem + D, desc_mnmajor(ds_s, kk), desc_mnmajor(q_s, kk), idesc_kv,
                  kk > 0 ? 1u : 0u);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)  // dV = local^T dP (queries)
      ptx::mma_ss(tmem + 2 * D, desc_mnmajor(lo_s, kk), desc_mnmajor(dp_s, kk), idesc_kv,
                  kk > 0 ? 1u : 0u);
    ptx::mma_commit(&sm.o_full);
  }
  __syncwarp();

  // ---- gradient rows out: dQ (row = query), dK and dV (row = key)
  ptx::mbar_wait(&sm.o_full, 0, status, 0x97000000u);
  ptx::tc_fence_after();
  const int tok = r0 + row;
  __nv_bfloat16* dqr = reinterpret_cast<__nv_bfloat16*>(p.dq.ptr) + (int64_t)n * p.dq.sb +
                       (int64_t)tok * p.dq.st + (int64_t)h * p.dq.sh;
  __nv_bfloat16* dkr = reinterpret_cast<__nv_bfloat16*>(p.dk.ptr) + (int64_t)n * p.dk.sb +
                       (int64_t)tok * p.dk.st + (int64_t)h * p.dk.sh;
  __nv_bfloat16* dvr = reinterpret_cast<__nv_bfloat16*>(p.dv.ptr) + (int64_t)n * p.dv.sb +
                       (int64_t)tok * p.dv.st + (int64_t)h * p.dv.sh;
#pragma unroll 1
  for (int pc = 0; pc < D / 32; ++pc) {
    uint32_t r[32];
    ptx::tmem_ld32(tmem + lane_off + pc * 32, r);
    ptx::tmem_wait_ld();
    ptx::reg_fence(r);
    store_row_bf16(dqr + pc * 32, r, p.scale);
    ptx::tmem_ld32(tmem + lane_off + D + pc * 32, r);
    ptx::tmem_wait_ld();
    ptx::reg_fence(r);
    store_row_bf16(dkr + pc * 32, r, p.scale);
    ptx::tmem_ld32(tmem + lane_off + 2 * D + pc * 32, r);
    ptx::tmem_wait_ld();
    ptx::reg_fence(r);
    store_row_bf16(dvr + pc * 32, r, 1.f);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kCols);
  }
}

template <int D, int kL>
int launch_grads(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const RgParams& p, int BH, cudaStream_t s) {
  auto kern = refsem_grads_kernel<D, kL>;
  const size_t smem = sizeof(RgSmem<D>) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return SQB_ERR_LAUNCH;
  kern<<<dim3(p.T / 128, BH), kRsThreads, smem, s>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

template <int D>
int launch_grads_l(int L, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const RgParams& p, int BH, cudaStream_t s) {
  if (L == 16) return launch_grads<D, 16>(tq, tk, tv, p, BH, s);
  if (L == 32) return launch_grads<D, 32>(tq, tk, tv, p, BH, s);
  if (L == 64) return launch_grads<D, 64>(tq, tk, tv, p, BH, s);
  return SQB_ERR_UNSUPPORTED;
}

template <int D, int kL>
int launch_local(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const RsParams& p, int BH, cudaStream_t s) {
  auto kern = refsem_local_kernel<D, kL>;
  const size_t smem = sizeof(RsSmem<D>) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return SQB_ERR_LAUNCH;
  kern<<<dim3(p.T / 128, BH), kRsThreads, smem, s>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

template <int D>
int launch_local_l(int L, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const RsParams& p, int BH, cudaStream_t s) {
  if (L == 16) return launch_local<D, 16>(tq, tk, tv, p, BH, s);
  if (L == 32) return launch_local<D, 32>(tq, tk, tv, p, BH, s);
  if (L == 64) return launch_local<D, 64>(tq, tk, tv, p, BH, s);
  return SQB_ERR_UNSUPPORTED;
}

}  // namespace
}  // namespace sm100

bool refsem_tc_supported(int L, int D, int dtype, std::initializer_list<TensorView> views) {
  if (dtype != SQB_BF16) return false;
  if (L != 16 && L != 32 && L != 64) return false;
  if (D != 64 && D != 128) return false;
  return sm100_views_ok(views) && sm100_device(nullptr);
}

int refsem_tc_local(TensorView q, TensorView k, TensorView v, float* summary, float* P, int B,
                    int T, int H, int D, int L, float scale, uint32_t* status,
                    cudaStream_t s) {
  if (T % 128 != 0 || T / L * L != T) return SQB_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  if (!sm100_encode_rows(&tq, B, T, H, D, q, 128) || !sm100_encode_rows(&tk, B, T, H, D, k, 128) ||
      !sm100_encode_rows(&tv, B, T, H, D, v, 128))
    return SQB_ERR_CUDA;
  sm100::RsParams p{H, T, T / L, scale * 1.4426950408889634f, summary, P, status};
  if (D == 64) return sm100::launch_local_l<64>(L, tq, tk, tv, p, B * H, s);
  if (D == 128) return sm100::launch_local_l<128>(L, tq, tk, tv, p, B * H, s);
  return SQB_ERR_UNSUPPORTED;
}

int refsem_tc_grads(TensorView q, TensorView k, TensorView v, const float* dP,
                    const float* dsum, TensorView dq, TensorView dk, TensorView dv, int B, int T,
                    int H, int D, int L, float scale, uint32_t* status, cudaStream_t s) {
  if (T % 128 != 0 || T / L * L != T) return SQB_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  if (!sm100_encode_rows(&tq, B, T, H, D, q, 128) || !sm100_encode_rows(&tk, B, T, H, D, k, 128) ||
      !sm100_encode_rows(&tv, B, T, H, D, v, 128))
    return SQB_ERR_CUDA;
  sm100::RgParams p{H, T, T / L, scale, scale * 1.4426950408889634f, dP, dsum, dq, dk, dv,
                    status};
  if (D == 64) return sm100::launch_grads_l<64>(L, tq, tk, tv, p, B * H, s);
  if (D == 128) return sm100::launch_grads_l<128>(L, tq, tk, tv, p, B * H, s);
  return SQB_ERR_UNSUPPORTED;
}

}  // namespace sqb
