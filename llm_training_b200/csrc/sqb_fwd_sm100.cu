// sm_100a forward kernel of sqrt-block attention.
//
// Persistent, warp-specialised, two CTAs per SM (320 threads each, single
// buffered; the co-resident CTA hides each one's load and MMA latencies):
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
// end.  O leaves through a per-warp ring of three 1 KB store units (16 rows x
// 32 columns), each handed to a TMA store as soon as it is written: the
// softmax warps never wait on the global write path, and no operand buffer is
// held, so the next tile's K/V loads - and with them its pooling and the
// summary flags later tiles wait on - are never delayed by an O store.
//
// Summaries cross CTAs: tiles are handed out in ascending sequence order
// (tile index n -> s = n / BH), the pooling warps of tile s publish their
// blocks' means and set flag[s].  Before loading summaries with TMA the
// producer warp checks, 32 flags at a time, that every tile holding one of
// the summaries it needs has published.
// A tile only ever waits on tiles with a smaller index, and tiles are only
// claimed by running CTAs, so every wait ends; each is still bounded in time
// (the workspace may set the budget of the waits on other CTAs) and records
// SQB_ERR_TIMEOUT if it gives up, which the last CTA to leave posts to the
// caller's mailbox.  Flags carry an epoch token so the workspace needs no
// clearing between calls.

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
  int G;       // blocks per sequence
  float* part;  // b > 128: K / V column sums of a block's earlier sub-tiles
};

// Pipeline depths: NQ query-tile slots, NKV key/value chunk stages, NS score
// buffers in TMEM.  Depth 2 everywhere fills one SM with one CTA; depth 1
// everywhere halves shared memory and TMEM so two CTAs share an SM and hide
// each other's latencies.
template <int D, int NQ, int NKV, int NS>
struct FwdSmem {
  static constexpr int kTileBytes = (D / 64) * kAtomBytes;
  alignas(1024) uint8_t q[NQ][kTileBytes];
  alignas(1024) uint8_t k[NKV][kTileBytes];
  alignas(1024) uint8_t v[NKV][kTileBytes];
  float red[4][D];  // pooling: per-warp partial sums of one of K / V
  // per softmax warp: a ring of three O store units, 16 rows x 32 columns bf16
  // each, 16-byte chunks in the TMA 64-byte swizzle (chunk ^= (row / 2) % 4)
  alignas(1024) uint8_t ostage[4][3][1024];
  uint64_t q_full[NQ], q_empty[NQ];
  uint64_t k_full[NKV], k_empty[NKV], v_full[NKV], v_empty[NKV];
  uint64_t s_full[NS], p_full[NS], s_free[NS], o_full, o_free;
  uint64_t mma_done;  // exit: every MMA of the CTA has completed
  int tile_ring[NQ];
  uint32_t tmem_base;
};

constexpr int kThreads = 320;
constexpr float kLn2 = 0.6931471805599453f;

// TMEM columns: NS score buffers of 128 columns, then O (D columns); the
// allocation is a power of two >= 32.
__host__ __device__ constexpr uint32_t fwd_tmem_cols(int D, int NS) {
  return (NS * 128 + D) <= 256 ? 256u : 512u;
}

template <int NQ, int NKV, int NS>
constexpr int ctas_per_sm() {
  return (NQ == 1 && NKV == 1 && NS == 1) ? 2 : 1;
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 q) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <int D, int NQ, int NKV, int NS, bool kSplit>
__global__ void __launch_bounds__(kThreads, (ctas_per_sm<NQ, NKV, NS>()))
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
               const __grid_constant__ CUtensorMap tm_kbar,
               const __grid_constant__ CUtensorMap tm_vbar, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  FwdSmem<D, NQ, NKV, NS>& sm = *reinterpret_cast<FwdSmem<D, NQ, NKV, NS>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t* status = p.ctrl + kStatus;
  const uint32_t token = *reinterpret_cast<volatile uint32_t*>(p.ctrl + kFwdEpoch) + 1u;
  const uint64_t xbudget = cross_wait_budget(p.ctrl);
  constexpr int kAtoms = D / 64;
  constexpr uint32_t kTmemCols = fwd_tmem_cols(D, NS);
  const uint32_t box_bytes = (uint32_t)p.g.R * 128u;  // one atom of an R-row box

  if (threadIdx.x == 0) {
    for (int i = 0; i < NQ; ++i) {
      ptx::mbar_init(&sm.q_full[i], 1);
      ptx::mbar_init(&sm.q_empty[i], 2);   // last S mma complete + pooling done
    }
    for (int i = 0; i < NKV; ++i) {
      ptx::mbar_init(&sm.k_full[i], 1);
      ptx::mbar_init(&sm.k_empty[i], 2);  // S mma complete + pooling done
      ptx::mbar_init(&sm.v_full[i], 1);
      ptx::mbar_init(&sm.v_empty[i], 2);  // PV mma complete + pooling done
    }
    for (int i = 0; i < NS; ++i) {
      ptx::mbar_init(&sm.s_full[i], 1);
      ptx::mbar_init(&sm.p_full[i], 4);    // one arrive per softmax warp
      ptx::mbar_init(&sm.s_free[i], 1);
    }
    ptx::mbar_init(&sm.o_full, 1);
    ptx::mbar_init(&sm.o_free, 4);
    ptx::mbar_init(&sm.mma_done, 1);
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
    // Tiles are claimed only once their Q slot is free and their loads can be
    // issued: a claimed tile that waits to start would publish its summaries
    // late and stall every later tile of its sequence.  (Measured: claiming
    // before the slot wait, or prefetching the likely next tile into L2, are
    // both slower.)
    auto claim = [&]() {
      int c = 0;
      if (lane == 0) {
        c = (int)atomicAdd(p.ctrl + kFwdTileCounter, 1u);
        if (c >= p.total_tiles) c = -1;
      }
      return __shfl_sync(0xffffffffu, c, 0);
    };
    int tc = 0, kc = 0;
    while (true) {
      const int slot = tc % NQ;
      ptx::mbar_wait(&sm.q_empty[slot], ((tc / NQ) & 1) ^ 1, status, 0x10000000u | slot);
      const int n = claim();
      if (lane == 0) {
        sm.tile_ring[slot] = n;
        if (n < 0) {
          // the copies issued so far have landed (they normally have: after a
          // failed wait they may still be in flight)
          for (int i = 1; i <= NQ && i <= tc; ++i)
            ptx::mbar_drain(&sm.q_full[(tc - i) % NQ], ((tc - i) / NQ) & 1);
          for (int i = 1; i <= NKV && i <= kc; ++i) {
            ptx::mbar_drain(&sm.k_full[(kc - i) % NKV], ((kc - i) / NKV) & 1);
            ptx::mbar_drain(&sm.v_full[(kc - i) % NKV], ((kc - i) / NKV) & 1);
          }
          ptx::mbar_arrive(&sm.q_full[slot]);
        }
      }
      if (n < 0) break;
      const Tile t = make_tile<kSplit>(p.g, p.H, n / p.BH, n % p.BH);
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(&sm.q_full[slot], kAtoms * box_bytes);
#pragma unroll
        for (int a = 0; a < kAtoms; ++a)
          ptx::tma_load_4d(sm.q[slot] + a * kAtomBytes, &tm_q, &sm.q_full[slot], a * 64, t.h,
                           t.r0, t.n);
      }
      for (int u = 0; u < t.nin; ++u) {
        const InChunk ic = in_chunk<kSplit>(t, in_order<kSplit>(t, u));
        const int st = kc % NKV;
        const uint32_t par = ((kc / NKV) & 1) ^ 1;
        ptx::mbar_wait(&sm.k_empty[st], par, status, 0x11000000u | st);
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&sm.k_full[st], kAtoms * box_bytes);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            ptx::tma_load_4d(sm.k[st] + a * kAtomBytes, &tm_k, &sm.k_full[st], a * 64, t.h,
                             ic.k0, t.n);
        }
        ptx::mbar_wait(&sm.v_empty[st], par, status, 0x13000000u | st);
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(&sm.v_full[st], kAtoms * box_bytes);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            ptx::tma_load_4d(sm.v[st] + a * kAtomBytes, &tm_v, &sm.v_full[st], a * 64, t.h,
                             ic.k0, t.n);
        }
        ++kc;
      }
      if (t.nsc > 0) {
        // every tile holding one of the needed summaries has published
        const int s_need = summary_tile<kSplit>(p.g, t.ns - 1);
        ptx::flags_wait_range(p.flags + (size_t)t.bh * p.flags_stride, 0, s_need + 1, token,
                              status, (uint32_t)n, xbudget);
        if (lane == 0) ptx::fence_proxy_async_global();
        for (int c = 0; c < t.nsc; ++c) {
          const SumChunk sc = sum_chunk(t, c);
          const int st = kc % NKV;
          const uint32_t par = ((kc / NKV) & 1) ^ 1;
          ptx::mbar_wait(&sm.k_empty[st], par, status, 0x12000000u | st);
          if (lane == 0) {
            ptx::mbar_arrive_expect_tx(&sm.k_full[st], kAtoms * kAtomBytes);
#pragma unroll
            for (int a = 0; a < kAtoms; ++a)
              ptx::tma_load_3d(sm.k[st] + a * kAtomBytes, &tm_kbar, &sm.k_full[st], a * 64,
                               sc.w, t.bh);
          }
          ptx::mbar_wait(&sm.v_empty[st], par, status, 0x14000000u | st);
          if (lane == 0) {
            ptx::mbar_arrive_expect_tx(&sm.v_full[st], kAtoms * kAtomBytes);
#pragma unroll
            for (int a = 0; a < kAtoms; ++a)
              ptx::tma_load_3d(sm.v[st] + a * kAtomBytes, &tm_vbar, &sm.v_full[st], a * 64,
                               sc.w, t.bh);
          }
          ++kc;
        }
      }
      ++tc;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t o_tmem = tmem + NS * 128;
      const uint32_t idesc_pv = ptx::idesc_bf16(128, D, false, true);
      int tc = 0, kc = 0, gc = 0;
      while (true) {
        const int slot = tc % NQ;
        ptx::mbar_wait(&sm.q_full[slot], (tc / NQ) & 1, status, 0x20000000u | slot);
        const int n = sm.tile_ring[slot];
        if (n < 0) break;
        const Tile t = make_tile<kSplit>(p.g, p.H, n / p.BH, n % p.BH);
        const int nch = t.nin + t.nsc;
        const uint32_t q_saddr = ptx::smem_u32(sm.q[slot]);
        auto chunk_n = [&](int c) {
          return c < t.nin ? in_chunk<kSplit>(t, in_order<kSplit>(t, c)).n
                           : sum_chunk(t, c - t.nin).n16;
        };
        auto issue_pv = [&](int c) {
          const int g = gc + c, x = g % NS, st = (kc + c) % NKV;
          ptx::mbar_wait(&sm.p_full[x], (g / NS) & 1, status, 0x21000000u | x);
          ptx::mbar_wait(&sm.v_full[st], ((kc + c) / NKV) & 1, status, 0x25000000u | st);
          if (c == 0 && tc > 0) ptx::mbar_wait(&sm.o_free, (tc - 1) & 1, status, 0x22000000u);
          ptx::tc_fence_after();
          const uint32_t v_saddr = ptx::smem_u32(sm.v[st]);
          const int nk = chunk_n(c) / 16;
          for (int kk = 0; kk < nk; ++kk)
            ptx::mma_ts(o_tmem, tmem + x * 128 + kk * 8, desc_mnmajor(v_saddr, kk), idesc_pv,
                        (c > 0 || kk > 0) ? 1u : 0u);
          ptx::mma_commit(&sm.v_empty[st]);
          ptx::mma_commit(&sm.s_free[x]);
          if (c == nch - 1) ptx::mma_commit(&sm.o_full);
        };
        // With two score buffers and two K/V stages, S(c) is issued before
        // PV(c-1) so the QK^T of the next chunk overlaps the softmax of this
        // one; with single buffers S(c) needs both freed by PV(c-1), which
        // therefore goes first.
        constexpr bool kOverlap = NS >= 2 && NKV >= 2;
        for (int c = 0; c < nch; ++c) {
          if (!kOverlap && c >= 1) issue_pv(c - 1);
          const int g = gc + c, x = g % NS, st = (kc + c) % NKV;
          ptx::mbar_wait(&sm.k_full[st], ((kc + c) / NKV) & 1, status, 0x23000000u | st);
          if (g >= NS)
            ptx::mbar_wait(&sm.s_free[x], ((g - NS) / NS) & 1, status, 0x24000000u | x);
          ptx::tc_fence_after();
          const uint32_t k_saddr = ptx::smem_u32(sm.k[st]);
          const uint32_t idesc_s = ptx::idesc_bf16(128, chunk_n(c), false, false);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            ptx::mma_ss(tmem + x * 128, desc_kmajor(q_saddr, kk), desc_kmajor(k_saddr, kk), idesc_s,
                        kk > 0 ? 1u : 0u);
          ptx::mma_commit(&sm.s_full[x]);
          ptx::mma_commit(&sm.k_empty[st]);
          // Q is read by no later MMA of this tile: the next tile may load
          if (c == nch - 1) ptx::mma_commit(&sm.q_empty[slot]);
          if (kOverlap && c >= 1) issue_pv(c - 1);
        }
        issue_pv(nch - 1);
        gc += nch;
        kc += nch;
        ++tc;
      }
      // every MMA issued has completed before TMEM is released
      ptx::mma_commit(&sm.mma_done);
      ptx::mbar_drain(&sm.mma_done, 0);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + NS * 128;
    int tc = 0, gc = 0;
    int ucount = 0;  // O store units this warp has issued (ring position)
    while (true) {
      const int slot = tc % NQ;
      ptx::mbar_wait(&sm.q_full[slot], (tc / NQ) & 1, status, 0x30000000u | slot);
      const int n = sm.tile_ring[slot];
      if (n < 0) break;
      const Tile t = make_tile<kSplit>(p.g, p.H, n / p.BH, n % p.BH);
      const int nch = t.nin + t.nsc;
      const int tq = t.r0 + row;
      const bool valid = row < t.rows;
      const int blk_t = valid ? tq / p.g.b : 0;
      const int lim = valid ? min(blk_t, p.g.Gc) : 0;  // visible summaries j < lim
      float m = -INFINITY, l = 0.f;
      for (int c = 0; c < nch; ++c) {
        const int g = gc + c, x = g % NS;
        int N, vlo, vhi;  // MMA width and the valid column range [vlo, vhi)
        if (c < t.nin) {
          // in-block keys [k0, k0 + N): those of the row's block up to the row
          const InChunk ic = in_chunk<kSplit>(t, in_order<kSplit>(t, c));
          N = ic.n;
          vlo = valid ? max(0, blk_t * p.g.b - ic.k0) : 0;
          vhi = valid ? min(tq - ic.k0 + 1, N) : 0;
        } else {
          const SumChunk sc = sum_chunk(t, c - t.nin);
          N = sc.n16;
          vlo = sc.lo - sc.w;
          vhi = min(sc.e, lim) - sc.w;
        }
        ptx::mbar_wait(&sm.s_full[x], (g / NS) & 1, status, 0x31000000u | x);
        ptx::tc_fence_after();
        const uint32_t s_addr = tmem + lane_off + x * 128;
        // 16-column pieces no row of this warp can see are skipped (in the
        // causal in-block chunk with b = R = 128, warp q needs columns < 32q+32)
        const bool any_col = vhi > vlo;
        const int wlo = __reduce_min_sync(0xffffffffu, any_col ? vlo : 0x7fffffff);
        const int whi = __reduce_max_sync(0xffffffffu, any_col ? vhi : 0);
        const int nq = N >> 4;
        const int q_lo = whi > wlo ? (wlo >> 4) : 0;
        const int q_hi = whi > wlo ? min((whi + 15) >> 4, nq) : 0;
        const uint32_t vspan = any_col ? (uint32_t)(vhi - vlo) : 0u;
        // Both passes walk the live pieces two at a time with one 32-column
        // TMEM load (fewer load round trips than 16-column double buffering;
        // an odd last pair reads 16 columns past the live range, unused).
        // pass 1: row max over the visible columns (masked -> -inf)
        float mx = -INFINITY;
        {
          auto maxp = [&](const uint32_t (&r)[16], int q) {
            float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              m0 = fmaxf(m0, (uint32_t)(q * 16 + j - vlo) < vspan ? __uint_as_float(r[j])
                                                                  : -INFINITY);
              m1 = fmaxf(m1, (uint32_t)(q * 16 + j + 1 - vlo) < vspan ? __uint_as_float(r[j + 1])
                                                                      : -INFINITY);
            }
            mx = fmaxf(mx, fmaxf(m0, m1));
          };
          for (int q = q_lo; q < q_hi; q += 2) {
            uint32_t r[32];
            ptx::tmem_ld32(s_addr + q * 16, r);
            ptx::tmem_wait_ld();
            ptx::reg_fence(r);
            maxp(*reinterpret_cast<const uint32_t(*)[16]>(r), q);
            if (q + 1 < q_hi) maxp(*reinterpret_cast<const uint32_t(*)[16]>(r + 16), q + 1);
          }
        }
        const float m_new = fmaxf(m, mx * p.scale_log2);
        if (c > 0) {
          const bool need = m_new > m;
          if (__any_sync(0xffffffffu, need)) {
            // PV of the previous chunk must have landed before O is rescaled
            ptx::mbar_wait(&sm.s_free[(g - 1) % NS], ((g - 1) / NS) & 1, status, 0x32000000u);
            ptx::tc_fence_after();
            const float alpha = need ? (m == -INFINITY ? 0.f : ptx::ex2(m - m_new)) : 1.f;
#pragma unroll 1
            for (int pc = 0; pc < D / 32; ++pc) {
              uint32_t r[32];
              ptx::tmem_ld32(o_addr + pc * 32, r);
              ptx::tmem_wait_ld();
              ptx::reg_fence(r);
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
        // pass 2: P = exp2(S*c - m) as bf16 into TMEM over S (16 columns of S
        // -> 8 columns of packed P).  Masked columns get exponent -inf.
        {
          float ls[4] = {0.f, 0.f, 0.f, 0.f};
          auto expp = [&](const uint32_t (&r)[16], int q) {
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const float x0 = fmaf(__uint_as_float(r[j]), p.scale_log2, -mm);
              const float x1 = fmaf(__uint_as_float(r[j + 1]), p.scale_log2, -mm);
              const float e0 = ptx::ex2((uint32_t)(q * 16 + j - vlo) < vspan ? x0 : -INFINITY);
              const float e1 =
                  ptx::ex2((uint32_t)(q * 16 + j + 1 - vlo) < vspan ? x1 : -INFINITY);
              ls[(j >> 1) & 3] += e0 + e1;
              pk[j >> 1] = ptx::pack_bf16x2(e0, e1);
            }
            ptx::tmem_st8(s_addr + q * 8, pk);
          };
          const uint32_t zero8[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
          // P of piece q lands on S columns [8q, 8q+8): masked pieces below the
          // live range can be zeroed first (their P columns are below every
          // live S column); those above only after the live pieces are read
          for (int q = 0; q < q_lo; ++q) ptx::tmem_st8(s_addr + q * 8, zero8);
          for (int q = q_lo; q < q_hi; q += 2) {
            uint32_t r[32];
            ptx::tmem_ld32(s_addr + q * 16, r);
            ptx::tmem_wait_ld();
            ptx::reg_fence(r);
            expp(*reinterpret_cast<const uint32_t(*)[16]>(r), q);
            if (q + 1 < q_hi) expp(*reinterpret_cast<const uint32_t(*)[16]>(r + 16), q + 1);
          }
          for (int q = q_hi; q < nq; ++q) ptx::tmem_st8(s_addr + q * 8, zero8);
          l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&sm.p_full[x]);
      }
      // ---- epilogue: O / l -> bf16 into the warp's ring of store units, 32
      // columns (two units of 16 rows) at a time, each unit stored by TMA as
      // soon as it is written.  Each store is its own bulk group; before a
      // piece's two units are rewritten, at most the previous piece's second
      // store (in the third slot) may still be reading.
      ptx::mbar_wait(&sm.o_full, tc & 1, status, 0x33000000u);
      ptx::tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const int ug = lane >> 4, ur = lane & 15;  // this lane's unit (row group) and row in it
#pragma unroll 1
      for (int pc = 0; pc < D / 32; ++pc) {
        uint32_t r0[32];
        ptx::tmem_ld32(o_addr + pc * 32, r0);
        ptx::tmem_wait_ld();
        ptx::reg_fence(r0);
        if (lane == 0) ptx::tma_store_wait_read_1();
        __syncwarp();
        uint8_t* unit = sm.ostage[quarter][(ucount + ug) % 3];
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          uint4 w;
          w.x = ptx::pack_bf16x2(__uint_as_float(r0[8 * j8 + 0]) * inv_l,
                                 __uint_as_float(r0[8 * j8 + 1]) * inv_l);
          w.y = ptx::pack_bf16x2(__uint_as_float(r0[8 * j8 + 2]) * inv_l,
                                 __uint_as_float(r0[8 * j8 + 3]) * inv_l);
          w.z = ptx::pack_bf16x2(__uint_as_float(r0[8 * j8 + 4]) * inv_l,
                                 __uint_as_float(r0[8 * j8 + 5]) * inv_l);
          w.w = ptx::pack_bf16x2(__uint_as_float(r0[8 * j8 + 6]) * inv_l,
                                 __uint_as_float(r0[8 * j8 + 7]) * inv_l);
          *reinterpret_cast<uint4*>(unit + ur * 64 + ((j8 ^ ((ur >> 1) & 3)) << 4)) = w;
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            // a row group past the tile's rows belongs to the next tile (or
            // lies past T, where TMA clips the store)
            const int row0 = quarter * 32 + g * 16;
            if (row0 < t.rows)
              ptx::tma_store_4d(&tm_o, sm.ostage[quarter][(ucount + g) % 3], pc * 32, t.h,
                                t.r0 + row0, t.n);
            ptx::tma_store_commit();
          }
        }
        ucount += 2;
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sm.o_free);
      if (valid) p.lse[(size_t)t.bh * p.g.T + tq] = (m + __log2f(l)) * kLn2;
      gc += nch;
      ++tc;
    }
    if (lane == 0) ptx::tma_store_wait_all();  // the O stores have completed
  } else {
    // ------------------------------------------------------------ pooling
    const int ptid = threadIdx.x - 192;  // 0..127
    const int cc = ptid & 15;            // 8-column chunk
    const int rg = ptid >> 4;            // row group: rows == rg (mod 8)
    const int pw = ptid >> 5;            // pooling warp 0..3
    const float inv_b = 1.f / (float)p.g.b;
    int tc = 0, kc = 0;
    while (true) {
      const int slot = tc % NQ;
      ptx::mbar_wait(&sm.q_full[slot], (tc / NQ) & 1, status, 0x40000000u | slot);
      const int n = sm.tile_ring[slot];
      if (n < 0) break;
      const Tile t = make_tile<kSplit>(p.g, p.H, n / p.BH, n % p.BH);
      {
        // b <= 128: each complete block of the tile's single in-block chunk is
        // pooled and written on its own.  b > 128: every sub-tile of a complete
        // block sums the keys of its own rows (its diagonal chunk, processed
        // first); each but the last leaves its K / V column sums in the
        // workspace before releasing its flag, and the last adds them to its
        // own and writes the block's means.  Later chunks only pass through,
        // so no block summary waits on the softmax of a tile's earlier chunks.
        constexpr bool split = kSplit;
        const bool pool_own = split && t.blk0 < p.g.Gc;
        const int nb = split ? 0 : p.g.R / p.g.b;
        const int nfull = max(0, min(nb, p.g.Gc - t.blk0));
        float acck[8], accv[8];  // b > 128: this thread's column sums of K, V
#pragma unroll
        for (int j = 0; j < 8; ++j) acck[j] = accv[j] = 0.f;
        for (int u = 0; u < t.nin; ++u) {
          const int st = kc % NKV;
          const bool own = u == 0;  // the tile's diagonal chunk (in_order)
          // K then V: each buffer is released as soon as its own sums are read,
          // so the next chunk's K load can start while V is still pooled.
#pragma unroll 1
          for (int kv = 0; kv < 2; ++kv) {
            ptx::mbar_wait(kv == 0 ? &sm.k_full[st] : &sm.v_full[st], (kc / NKV) & 1, status,
                           (kv == 0 ? 0x41000000u : 0x43000000u) | st);
            const uint8_t* buf = kv == 0 ? sm.k[st] : sm.v[st];
            __nv_bfloat16* dst = kv == 0 ? p.kbar : p.vbar;
            for (int lb = 0; lb < nfull; ++lb) {
              float a[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] = 0.f;
              if (cc < D / 8) {
                for (int i = 0; i < p.g.b / 8; ++i) {
                  const int r = lb * p.g.b + rg + 8 * i;
                  add_bf16x8(a, *reinterpret_cast<const uint4*>(buf + swz_offset(r, cc * 8)));
                }
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] += __shfl_xor_sync(0xffffffffu, a[j], 16);
              if ((ptid & 16) == 0 && cc < D / 8) {
#pragma unroll
                for (int j = 0; j < 8; ++j) sm.red[pw][cc * 8 + j] = a[j];
              }
              ptx::named_barrier(2, 128);
              if (ptid < D) {
                const float sum =
                    sm.red[0][ptid] + sm.red[1][ptid] + sm.red[2][ptid] + sm.red[3][ptid];
                dst[((size_t)t.bh * p.g.Gc + t.blk0 + lb) * D + ptid] =
                    __float2bfloat16_rn(sum * inv_b);
              }
              ptx::named_barrier(2, 128);
            }
            if (pool_own && own && cc < D / 8) {
              for (int i = 0; i < t.rows / 8; ++i) {
                const uint4 w = *reinterpret_cast<const uint4*>(buf + swz_offset(rg + 8 * i, cc * 8));
                if (kv == 0)
                  add_bf16x8(acck, w);
                else
                  add_bf16x8(accv, w);
              }
            }
            ptx::named_barrier(2, 128);
            if (ptid == 0)
              ptx::mbar_arrive(kv == 0 ? &sm.k_empty[st] : &sm.v_empty[st]);
          }
          ++kc;
          if (!own) continue;
          if (pool_own) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acck[j] += __shfl_xor_sync(0xffffffffu, acck[j], 16);
              accv[j] += __shfl_xor_sync(0xffffffffu, accv[j], 16);
            }
            const bool last = t.sub == p.g.tpb - 1;
            float* part = p.part + ((size_t)t.bh * p.G + t.blk0) * (p.g.tpb - 1) * 2 * D;
            // the block's earlier sub-tiles have left their sums (their flags)
            if (last && pw == 0)
              ptx::flags_wait_range(p.flags + (size_t)t.bh * p.flags_stride, t.s - t.sub, t.s,
                                    token, status, (uint32_t)n, xbudget);
#pragma unroll 1
            for (int kv = 0; kv < 2; ++kv) {
              if ((ptid & 16) == 0 && cc < D / 8) {
#pragma unroll
                for (int j = 0; j < 8; ++j) sm.red[pw][cc * 8 + j] = kv == 0 ? acck[j] : accv[j];
              }
              ptx::named_barrier(2, 128);
              if (ptid < D) {
                float sum = sm.red[0][ptid] + sm.red[1][ptid] + sm.red[2][ptid] + sm.red[3][ptid];
                if (!last) {
                  part[(t.sub * 2 + kv) * D + ptid] = sum;
                } else {
                  for (int v = 0; v < t.sub; ++v) sum += __ldcg(part + (v * 2 + kv) * D + ptid);
                  (kv == 0 ? p.kbar : p.vbar)[((size_t)t.bh * p.g.Gc + t.blk0) * D + ptid] =
                      __float2bfloat16_rn(sum * inv_b);
                }
              }
              ptx::named_barrier(2, 128);
            }
          }
          // The barriers above order every pooling thread's summary (or
          // partial-sum) writes before this release store, which makes them
          // visible to any CTA that acquires the flag.
          if (ptid == 0) ptx::st_release_gpu(p.flags + (size_t)t.bh * p.flags_stride + t.s, token);
        }
      }
      for (int c = 0; c < t.nsc; ++c) {
        if (ptid == 0) {
          const int st = kc % NKV;
          ptx::mbar_wait(&sm.k_full[st], (kc / NKV) & 1, status, 0x42000000u | st);
          ptx::mbar_arrive(&sm.k_empty[st]);
          ptx::mbar_wait(&sm.v_full[st], (kc / NKV) & 1, status, 0x44000000u | st);
          ptx::mbar_arrive(&sm.v_empty[st]);
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
      post_status(p.ctrl);
    }
  }
}

template <int D, int NQ, int NKV, int NS, bool kSplit>
int launch(const Problem& pr, const TensorMaps& tm, float* lse, void* kbar, void* vbar,
           uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream) {
  FwdParams p;
  p.g.T = pr.T;
  p.g.b = pr.b;
  p.g.Gc = pr.Gc;
  p.g.R = tile_rows(pr.b);
  p.g.tiles_per_seq = tiles_per_seq(pr.T, pr.b);
  p.g.tpb = tiles_per_block(pr.b);
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
  p.G = pr.G;
  p.part = reinterpret_cast<float*>(ws + wl.pool_part);
  auto kern = fwd_kernel<D, NQ, NKV, NS, kSplit>;
  const size_t smem = sizeof(FwdSmem<D, NQ, NKV, NS>) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return SQB_ERR_LAUNCH;
  const int slots = num_sms * ctas_per_sm<NQ, NKV, NS>();
  const int grid = p.total_tiles < slots ? p.total_tiles : slots;
  kern<<<grid, kThreads, smem, stream>>>(tm.q, tm.k, tm.v, tm.o, tm.kbar, tm.vbar, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

}  // namespace

int launch_forward(const Problem& pr, const TensorMaps& tm, float* lse, void* kbar, void* vbar,
                   uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream) {
  // single-buffered, two CTAs per SM (measured faster than one double-buffered CTA)
  const bool split = pr.b > 128;
  if (pr.D == 64)
    return split ? launch<64, 1, 1, 1, true>(pr, tm, lse, kbar, vbar, ws, wl, num_sms, stream)
                 : launch<64, 1, 1, 1, false>(pr, tm, lse, kbar, vbar, ws, wl, num_sms, stream);
  if (pr.D == 128)
    return split ? launch<128, 1, 1, 1, true>(pr, tm, lse, kbar, vbar, ws, wl, num_sms, stream)
                 : launch<128, 1, 1, 1, false>(pr, tm, lse, kbar, vbar, ws, wl, num_sms, stream);
  return SQB_ERR_UNSUPPORTED;
}

}  // namespace sm100
}  // namespace sqb
