// sm_100a forward kernel of sqrt-block attention.
//
// Persistent, warp-specialised, one CTA per SM (320 threads):
//   warp 0      TMA producer + tile scheduler (atomic tile counter)
//   warp 1      tcgen05.mma issuer (one thread) and TMEM owner
//   warps 2-5   softmax + epilogue, one query row (TMEM lane) per thread
//   warps 6-9   block pooling: Kbar/Vbar of the tile's complete blocks
//
// Per work tile (R query rows of one (batch, head), see sqb_sm100_common.cuh)
// the chunk sequence is: the tile's own keys (in-block, causal), then the
// pooled summaries of every earlier block in chunks of <= 128.  Each chunk:
//   S = Q K^T            tcgen05.mma, A/B from swizzled smem, D in TMEM
//   P = exp2(S*c - m)    softmax warps (online max; O rescaled in TMEM)
//   O += P V             tcgen05.mma, A = P from TMEM (bf16), B = V smem
// The online softmax spans both kinds of chunk, so in-block keys and
// summaries share one softmax.  LSE (natural log) and O are written at the
// end; O goes through smem and a TMA store.
//
// Summaries cross CTAs: tiles are handed out in ascending sequence order
// (tile index n -> s = n / BH), the pooling warps of tile s publish their
// blocks' means and set flag[s].  Before loading summaries with TMA the
// producer warp checks, 32 flags at a time, that every tile holding one of
// the summaries it needs has published.
// A tile only ever waits on tiles with a smaller index, and tiles are only
// claimed by running CTAs, so every wait ends; each is still bounded in time
// and records SQB_ERR_TIMEOUT if it gives up.  Flags carry an epoch token so
// the workspace needs no clearing between calls.

#include "sqb_sm100.cuh"
#include "sqb_sm100_common.cuh"

namespace sqb {
namespace sm100 {
namespace {

struct FwdParams {
  Geometry g;
  int H, BH;
  int total_tiles;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* kbar;
  __nv_bfloat16* vbar;
  float* lse;
  uint32_t* ctrl;
  uint32_t* flags;
  int flags_stride;
};

template <int D>
struct FwdSmem {
  static constexpr int kTileBytes = (D / 64) * kAtomBytes;
  alignas(1024) uint8_t q[2][kTileBytes];
  alignas(1024) uint8_t k[2][kTileBytes];
  alignas(1024) uint8_t v[2][kTileBytes];
  float red[4][2][D];
  uint64_t q_full[2], q_empty[2], kv_full[2], kv_empty[2];
  uint64_t s_full[2], p_full[2], s_free[2], o_full, o_free;
  int tile_ring[2];
  uint32_t tmem_base;
};

constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 q) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
               const __grid_constant__ CUtensorMap tm_kbar,
               const __grid_constant__ CUtensorMap tm_vbar, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  FwdSmem<D>& sm = *reinterpret_cast<FwdSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t* status = p.ctrl + kStatus;
  const uint32_t token = *reinterpret_cast<volatile uint32_t*>(p.ctrl + kFwdEpoch) + 1u;
  constexpr int kAtoms = D / 64;
  const uint32_t box_bytes = (uint32_t)p.g.R * 128u;  // one atom of an R-row box

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&sm.q_full[i], 1);
      ptx::mbar_init(&sm.q_empty[i], 2);   // epilogue store done + pooling done
      ptx::mbar_init(&sm.kv_full[i], 1);
      ptx::mbar_init(&sm.kv_empty[i], 2);  // PV mma complete + pooling done
      ptx::mbar_init(&sm.s_full[i], 1);
      ptx::mbar_init(&sm.p_full[i], 4);    // one arrive per softmax warp
      ptx::mbar_init(&sm.s_free[i], 1);
    }
    ptx::mbar_init(&sm.o_full, 1);
    ptx::mbar_init(&sm.o_free, 4);
    ptx::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::tma_prefetch_desc(&tm_q);
    ptx::tma_prefetch_desc(&tm_k);
    ptx::tma_prefetch_desc(&tm_v);
    ptx::tma_prefetch_desc(&tm_o);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&sm.tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop (the summary-flag wait is warp-parallel);
    // lane 0 claims tiles and issues every TMA and barrier operation.
    int tc = 0, kc = 0;
    while (true) {
      const int slot = tc & 1;
      int n = 0;
      if (lane == 0) {
        n = (int)atomicAdd(p.ctrl + kFwdTileCounter, 1u);
        if (n >= p.total_tiles) n = -1;
      }
      n = __shfl_sync(0xffffffffu, n, 0);
      ptx::mbar_wait(&sm.q_empty[slot], ((tc >> 1) & 1) ^ 1, status, 0x10000000u | slot);
      if (lane == 0) {
        sm.tile_ring[slot] = n;
        if (n < 0) ptx::mbar_arrive(&sm.q_full[slot]);
      }
      if (n < 0) break;
      const Tile t = make_tile(p.g, p.H, n / p.BH, n % p.BH);
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(&sm.q_full[slot], kAtoms * box_bytes);
#pragma unroll
        for (int a = 0; a < kAtoms; ++a)
          ptx::tma_load_4d(sm.q[slot] + a * kAtomBytes, &tm_q, &sm.q_full[slot], a * 64, t.h,
                           t.r0, t.n);
      }
      {
        const int st = kc & 1;
        ptx::mbar_wait(&sm.kv_empty[st], ((kc >> 1) & 1) ^ 1, status, 0x11000000u | st);
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kAtoms * box_bytes);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a) {
            ptx::tma_load_4d(sm.k[st] + a * kAtomBytes, &tm_k, &sm.kv_full[st], a * 64, t.h,
                             t.r0, t.n);
            ptx::tma_load_4d(sm.v[st] + a * kAtomBytes, &tm_v, &sm.kv_full[st], a * 64, t.h,
                             t.r0, t.n);
          }
        }
        ++kc;
      }
      if (t.nsc > 0) {
        // every tile holding one of the needed summaries has published
        const int s_need = ((t.ns - 1) * p.g.b) / p.g.R;
        ptx::flags_wait_range(p.flags + (size_t)t.bh * p.flags_stride, 0, s_need + 1, token,
                              status, (uint32_t)n);
        if (lane == 0) ptx::fence_proxy_async_global();
        for (int c = 0; c < t.nsc; ++c) {
          const SumChunk sc = sum_chunk(t, c);
          const int st = kc & 1;
          ptx::mbar_wait(&sm.kv_empty[st], ((kc >> 1) & 1) ^ 1, status, 0x12000000u | st);
          if (lane == 0) {
            ptx::mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kAtoms * kAtomBytes);
#pragma unroll
            for (int a = 0; a < kAtoms; ++a) {
              ptx::tma_load_3d(sm.k[st] + a * kAtomBytes, &tm_kbar, &sm.kv_full[st], a * 64,
                               sc.w, t.bh);
              ptx::tma_load_3d(sm.v[st] + a * kAtomBytes, &tm_vbar, &sm.kv_full[st], a * 64,
                               sc.w, t.bh);
            }
          }
          ++kc;
        }
      }
      ++tc;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t s_tmem[2] = {tmem, tmem + 128};
      const uint32_t o_tmem = tmem + 256;
      const uint32_t idesc_pv = ptx::idesc_bf16(128, D, false, true);
      int tc = 0, kc = 0, gc = 0;
      while (true) {
        const int slot = tc & 1;
        ptx::mbar_wait(&sm.q_full[slot], (tc >> 1) & 1, status, 0x20000000u | slot);
        const int n = sm.tile_ring[slot];
        if (n < 0) break;
        const Tile t = make_tile(p.g, p.H, n / p.BH, n % p.BH);
        const int nch = 1 + t.nsc;
        const uint32_t q_saddr = ptx::smem_u32(sm.q[slot]);
        auto chunk_n = [&](int c) { return c == 0 ? t.n_in : sum_chunk(t, c - 1).n16; };
        auto issue_pv = [&](int c) {
          const int g = gc + c, x = g & 1, st = (kc + c) & 1;
          ptx::mbar_wait(&sm.p_full[x], (g >> 1) & 1, status, 0x21000000u | x);
          if (c == 0 && tc > 0) ptx::mbar_wait(&sm.o_free, (tc - 1) & 1, status, 0x22000000u);
          ptx::tc_fence_after();
          const uint32_t v_saddr = ptx::smem_u32(sm.v[st]);
          const int nk = chunk_n(c) / 16;
          for (int kk = 0; kk < nk; ++kk)
            ptx::mma_ts(o_tmem, s_tmem[x] + kk * 8, desc_mnmajor(v_saddr, kk), idesc_pv,
                        (c > 0 || kk > 0) ? 1u : 0u);
          ptx::mma_commit(&sm.kv_empty[st]);
          ptx::mma_commit(&sm.s_free[x]);
          if (c == nch - 1) ptx::mma_commit(&sm.o_full);
        };
        for (int c = 0; c < nch; ++c) {
          const int g = gc + c, x = g & 1, st = (kc + c) & 1;
          ptx::mbar_wait(&sm.kv_full[st], ((kc + c) >> 1) & 1, status, 0x23000000u | st);
          if (g >= 2) ptx::mbar_wait(&sm.s_free[x], ((g - 2) >> 1) & 1, status, 0x24000000u | x);
          ptx::tc_fence_after();
          const uint32_t k_saddr = ptx::smem_u32(sm.k[st]);
          const uint32_t idesc_s = ptx::idesc_bf16(128, chunk_n(c), false, false);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            ptx::mma_ss(s_tmem[x], desc_kmajor(q_saddr, kk), desc_kmajor(k_saddr, kk), idesc_s,
                        kk > 0 ? 1u : 0u);
          ptx::mma_commit(&sm.s_full[x]);
          if (c >= 1) issue_pv(c - 1);
        }
        issue_pv(nch - 1);
        gc += nch;
        kc += nch;
        ++tc;
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + 256;
    int tc = 0, gc = 0;
    while (true) {
      const int slot = tc & 1;
      ptx::mbar_wait(&sm.q_full[slot], (tc >> 1) & 1, status, 0x30000000u | slot);
      const int n = sm.tile_ring[slot];
      if (n < 0) break;
      const Tile t = make_tile(p.g, p.H, n / p.BH, n % p.BH);
      const int nch = 1 + t.nsc;
      const int tq = t.r0 + row;
      const bool valid = row < t.rows;
      const int blk_t = valid ? tq / p.g.b : 0;
      const int lim = valid ? min(blk_t, p.g.Gc) : 0;  // visible summaries j < lim
      float m = -INFINITY, l = 0.f;
      for (int c = 0; c < nch; ++c) {
        const int g = gc + c, x = g & 1;
        int N, vlo, vhi;  // MMA width and the valid column range [vlo, vhi)
        if (c == 0) {
          N = t.n_in;
          vlo = valid ? blk_t * p.g.b - t.r0 : 0;
          vhi = valid ? row + 1 : 0;
        } else {
          const SumChunk sc = sum_chunk(t, c - 1);
          N = sc.n16;
          vlo = sc.lo - sc.w;
          vhi = min(sc.e, lim) - sc.w;
        }
        ptx::mbar_wait(&sm.s_full[x], (g >> 1) & 1, status, 0x31000000u | x);
        ptx::tc_fence_after();
        const uint32_t s_addr = tmem + lane_off + x * 128;
        const int npieces = (N + 31) >> 5;
        float mx = -INFINITY;
        for (int pc = 0; pc < npieces; ++pc) {
          uint32_t r[32];
          ptx::tmem_ld32(s_addr + pc * 32, r);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = pc * 32 + j;
            if (col >= vlo && col < vhi) mx = fmaxf(mx, __uint_as_float(r[j]));
          }
        }
        const float m_new = fmaxf(m, mx * p.scale_log2);
        if (c > 0) {
          const bool need = m_new > m;
          if (__any_sync(0xffffffffu, need)) {
            // PV of the previous chunk must have landed before O is rescaled
            ptx::mbar_wait(&sm.s_free[(g - 1) & 1], ((g - 1) >> 1) & 1, status, 0x32000000u);
            ptx::tc_fence_after();
            const float alpha = need ? (m == -INFINITY ? 0.f : ptx::ex2(m - m_new)) : 1.f;
#pragma unroll 1
            for (int pc = 0; pc < D / 32; ++pc) {
              uint32_t r[32];
              ptx::tmem_ld32(o_addr + pc * 32, r);
              ptx::tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
              ptx::tmem_st32(o_addr + pc * 32, r);
            }
            ptx::tmem_wait_st();
            l *= alpha;
          }
        }
        m = m_new;
        const float mm = (m == -INFINITY) ? 0.f : m;
        for (int pc = 0; pc < npieces; ++pc) {
          uint32_t r[32];
          ptx::tmem_ld32(s_addr + pc * 32, r);
          ptx::tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const int col = pc * 32 + j;
            const float p0 = (col >= vlo && col < vhi)
                                 ? ptx::ex2(fmaf(__uint_as_float(r[j]), p.scale_log2, -mm))
                                 : 0.f;
            const float p1 = (col + 1 >= vlo && col + 1 < vhi)
                                 ? ptx::ex2(fmaf(__uint_as_float(r[j + 1]), p.scale_log2, -mm))
                                 : 0.f;
            l += p0 + p1;
            pk[j >> 1] = ptx::pack_bf16x2(p0, p1);
          }
          ptx::tmem_st16(s_addr + pc * 16, pk);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&sm.p_full[x]);
      }
      // ---- epilogue: O / l -> bf16 -> swizzled smem (the Q slot) -> TMA store
      ptx::mbar_wait(&sm.o_full, tc & 1, status, 0x33000000u);
      ptx::tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      uint8_t* stage = sm.q[slot];
#pragma unroll 1
      for (int pc = 0; pc < D / 32; ++pc) {
        uint32_t r[32];
        ptx::tmem_ld32(o_addr + pc * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          uint4 w;
          w.x = ptx::pack_bf16x2(__uint_as_float(r[8 * j8 + 0]) * inv_l,
                                 __uint_as_float(r[8 * j8 + 1]) * inv_l);
          w.y = ptx::pack_bf16x2(__uint_as_float(r[8 * j8 + 2]) * inv_l,
                                 __uint_as_float(r[8 * j8 + 3]) * inv_l);
          w.z = ptx::pack_bf16x2(__uint_as_float(r[8 * j8 + 4]) * inv_l,
                                 __uint_as_float(r[8 * j8 + 5]) * inv_l);
          w.w = ptx::pack_bf16x2(__uint_as_float(r[8 * j8 + 6]) * inv_l,
                                 __uint_as_float(r[8 * j8 + 7]) * inv_l);
          *reinterpret_cast<uint4*>(stage + swz_offset(row, pc * 32 + j8 * 8)) = w;
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sm.o_free);
      if (valid) p.lse[(size_t)t.bh * p.g.T + tq] = (m + __log2f(l)) * kLn2;
      ptx::fence_proxy_async_smem();
      ptx::named_barrier(1, 128);
      if (warp == 2 && lane == 0) {
#pragma unroll
        for (int a = 0; a < kAtoms; ++a)
          ptx::tma_store_4d(&tm_o, stage + a * kAtomBytes, a * 64, t.h, t.r0, t.n);
        ptx::tma_store_commit();
        ptx::tma_store_wait_read_all();
        ptx::mbar_arrive(&sm.q_empty[slot]);
      }
      gc += nch;
      ++tc;
    }
    if (warp == 2 && lane == 0) ptx::tma_store_wait_all();
  } else {
    // ------------------------------------------------------------ pooling
    const int ptid = threadIdx.x - 192;  // 0..127
    const int cc = ptid & 15;            // 8-column chunk
    const int rg = ptid >> 4;            // row group: rows == rg (mod 8)
    const int pw = ptid >> 5;            // pooling warp 0..3
    const float inv_b = 1.f / (float)p.g.b;
    int tc = 0, kc = 0;
    while (true) {
      const int slot = tc & 1;
      ptx::mbar_wait(&sm.q_full[slot], (tc >> 1) & 1, status, 0x40000000u | slot);
      const int n = sm.tile_ring[slot];
      if (n < 0) break;
      const Tile t = make_tile(p.g, p.H, n / p.BH, n % p.BH);
      {
        const int st = kc & 1;
        ptx::mbar_wait(&sm.kv_full[st], (kc >> 1) & 1, status, 0x41000000u | st);
        const int nb = p.g.R / p.g.b;
        const int nfull = max(0, min(nb, p.g.Gc - t.blk0));
        for (int lb = 0; lb < nfull; ++lb) {
          float ak[8], av[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) ak[j] = av[j] = 0.f;
          if (cc < D / 8) {
            for (int i = 0; i < p.g.b / 8; ++i) {
              const int r = lb * p.g.b + rg + 8 * i;
              const uint32_t off = swz_offset(r, cc * 8);
              add_bf16x8(ak, *reinterpret_cast<const uint4*>(sm.k[st] + off));
              add_bf16x8(av, *reinterpret_cast<const uint4*>(sm.v[st] + off));
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            ak[j] += __shfl_xor_sync(0xffffffffu, ak[j], 16);
            av[j] += __shfl_xor_sync(0xffffffffu, av[j], 16);
          }
          if ((ptid & 16) == 0 && cc < D / 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              sm.red[pw][0][cc * 8 + j] = ak[j];
              sm.red[pw][1][cc * 8 + j] = av[j];
            }
          }
          ptx::named_barrier(2, 128);
          if (ptid < D) {
            const float sk = sm.red[0][0][ptid] + sm.red[1][0][ptid] + sm.red[2][0][ptid] +
                             sm.red[3][0][ptid];
            const float sv = sm.red[0][1][ptid] + sm.red[1][1][ptid] + sm.red[2][1][ptid] +
                             sm.red[3][1][ptid];
            const size_t off = ((size_t)t.bh * p.g.Gc + t.blk0 + lb) * D + ptid;
            p.kbar[off] = __float2bfloat16_rn(sk * inv_b);
            p.vbar[off] = __float2bfloat16_rn(sv * inv_b);
          }
          ptx::named_barrier(2, 128);
        }
        ptx::fence_proxy_async_global();
        ptx::named_barrier(2, 128);
        if (ptid == 0) {
          ptx::mbar_arrive(&sm.kv_empty[st]);
          __threadfence();
          ptx::st_release_gpu(p.flags + (size_t)t.bh * p.flags_stride + t.s, token);
        }
        ++kc;
      }
      for (int c = 0; c < t.nsc; ++c) {
        if (ptid == 0) {
          const int st = kc & 1;
          ptx::mbar_wait(&sm.kv_full[st], (kc >> 1) & 1, status, 0x42000000u | st);
          ptx::mbar_arrive(&sm.kv_empty[st]);
        }
        ++kc;
      }
      if (ptid == 0) ptx::mbar_arrive(&sm.q_empty[slot]);
      ++tc;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.ctrl + kFwdExitCounter, 1u);
    if (prev == gridDim.x - 1) {
      // every CTA has left its scheduling loop: reset for the next launch
      atomicExch(p.ctrl + kFwdTileCounter, 0u);
      atomicExch(p.ctrl + kFwdExitCounter, 0u);
      __threadfence();
      atomicExch(p.ctrl + kFwdEpoch, token);
    }
  }
}

template <int D>
int launch(const Problem& pr, const TensorMaps& tm, float* lse, void* kbar, void* vbar,
           uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream) {
  FwdParams p;
  p.g.T = pr.T;
  p.g.b = pr.b;
  p.g.Gc = pr.Gc;
  p.g.R = tile_rows(pr.b);
  p.g.tiles_per_seq = (pr.T + p.g.R - 1) / p.g.R;
  p.H = pr.H;
  p.BH = pr.B * pr.H;
  p.total_tiles = p.g.tiles_per_seq * p.BH;
  p.scale_log2 = pr.scale * 1.4426950408889634f;
  p.kbar = reinterpret_cast<__nv_bfloat16*>(kbar);
  p.vbar = reinterpret_cast<__nv_bfloat16*>(vbar);
  p.lse = lse;
  p.ctrl = reinterpret_cast<uint32_t*>(ws + wl.ctrl);
  p.flags = reinterpret_cast<uint32_t*>(ws + wl.flags_fwd);
  p.flags_stride = wl.tiles_per_seq;
  const size_t smem = sizeof(FwdSmem<D>) + 1024;
  if (cudaFuncSetAttribute(fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return SQB_ERR_LAUNCH;
  const int grid = p.total_tiles < num_sms ? p.total_tiles : num_sms;
  fwd_kernel<D><<<grid, kThreads, smem, stream>>>(tm.q, tm.k, tm.v, tm.o, tm.kbar, tm.vbar, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

}  // namespace

int launch_forward(const Problem& pr, const TensorMaps& tm, float* lse, void* kbar, void* vbar,
                   uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream) {
  if (pr.D == 64) return launch<64>(pr, tm, lse, kbar, vbar, ws, wl, num_sms, stream);
  if (pr.D == 128) return launch<128>(pr, tm, lse, kbar, vbar, ws, wl, num_sms, stream);
  return SQB_ERR_UNSUPPORTED;
}

}  // namespace sm100
}  // namespace sqb
