// sm_100a backward kernel of sqrt-block attention.
//
// Persistent, warp-specialised, one CTA per SM (32 * (3 + 4 * kParts) threads):
//   warp 0      TMA producer + tile scheduler
//   warp 1      tcgen05.mma issuer and TMEM owner
//   warps 2..   softmax-gradient / epilogue: kParts warps per TMEM lane quarter,
//               one TMEM lane (row) per thread, each warp 1/kParts of the columns
//   last warp   publisher of the summary-gradient counters
//
// A work tile is the same R-row tile as in the forward.  Its chunks are the
// summary chunks first, then the tile's own (in-block) keys.  Per chunk, with
// LSE and delta = rowsum(dO * O) per query row:
//   S  = Q Kc^T, dP = dO Vc^T                       (TMEM, lanes = queries)
//   P  = exp2(S*c - LSE*log2e), dS = scale * P * (dP - delta)  -> smem (bf16)
//   dVc = P^T dO, dKc = dS^T Q                       (TMEM, lanes = keys)
//   dQ += dS Kc                                      (TMEM, lanes = queries)
// For a summary chunk, dKc/dVc are summary gradients: they are added with
// fp32 atomics into per-(batch, head) accumulators in the workspace.  For
// D = 128 they are computed transposed (dVbar^T = dO^T P, dKbar^T = Q^T dS:
// TMEM lanes = feature, columns = summaries), so each warp's atomic covers
// 32 consecutive features of one summary - one 128-byte row segment - instead
// of 32 summary rows.
// For the in-block chunk they are the tile's own dK/dV, to which the epilogue
// adds (summary gradient of the key's block) / b - a summary is the mean of
// its block - before storing dK, dV and dQ through smem with TMA.
//
// The summary gradient of block j is complete once every later tile has
// added to it.  Tiles are handed out in descending sequence order.  Once
// every gradient warp of a tile has issued its additions, the publisher warp
// adds 1 to the tile's counter with release semantics, so the counter reaches
// the launch epoch; before reading its blocks' sums a tile checks (32
// counters at a time) that every later tile's counter has reached it.
// The reader re-zeroes the sums it consumed, so the accumulators are zero
// again when the kernel ends.  Waits are bounded like the forward's.

#include "sqb_sm100.cuh"
#include "sqb_sm100_common.cuh"

// Gradient warps per TMEM lane quarter (2 or 4).
#ifndef SQB_BWD_PARTS
#define SQB_BWD_PARTS 2
#endif

namespace sqb {
namespace sm100 {
namespace {

struct BwdParams {
  Geometry g;
  int H, BH;
  int total_tiles;
  float scale;       // softmax scale, folded into dS
  float scale_log2;  // scale * log2(e)
  const float* lse;
  const __nv_bfloat16* o;
  int64_t o_sb, o_st, o_sh;
  float* dkbar;  // fp32 (BH, Gc, D) accumulators, zero between launches
  float* dvbar;
  // b > 128: fp32 (BH, G, xrows, D) rows of the dK / dV that a block's later
  // sub-tiles contribute to the keys of its earlier ones (xrows = (sub-tiles
  // per block - 1) * 128): stored by the single writer with two sub-tiles per
  // block, else accumulators that are zero between launches
  float* dkx;
  float* dvx;
  uint32_t* readers;  // b > 128: per (batch*head, block) count of sub-tiles that read its sums
  int G, xrows;
  uint32_t* ctrl;
  uint32_t* flags;
  int flags_stride;
  int store_rows;  // rows per dQ/dK/dV store box
};

// At D = 64 with b <= 128 shared memory has room for the tile's own keys and
// values (its in-block chunk) in buffers of their own, so the in-block S and dP
// never wait for a K / V load behind the summary chunk's MMAs.  The epilogue
// then stages dQ and dV there (instead of in the K and dS buffers), so the
// next tile's summary Kbar / Vbar load as soon as it is claimed.
template <int D, bool kSplit>
constexpr bool in_bufs() {
  return D == 64 && !kSplit;
}
template <int D, bool kIn>
struct BwdInBufs {};
template <int D>
struct BwdInBufs<D, true> {
  alignas(1024) uint8_t kin[(D / 64) * kAtomBytes];
  alignas(1024) uint8_t vin[(D / 64) * kAtomBytes];
};

template <int D, bool kIn>
struct BwdSmem : BwdInBufs<D, kIn> {
  static constexpr int kTileBytes = (D / 64) * kAtomBytes;
  alignas(1024) uint8_t q[kTileBytes];     // Q
  alignas(1024) uint8_t dout[kTileBytes];  // dO
  alignas(1024) uint8_t k[kTileBytes];     // K chunk, then dQ staging
  alignas(1024) uint8_t v[kTileBytes];     // O (for delta), then the V chunk
  alignas(1024) uint8_t p[2 * kAtomBytes];   // P (128 query rows x 128 keys), then dK staging
  // dS (same layout), then dV staging; the first summary chunk's Vbar is
  // loaded here (the tile's O still occupies the V buffer until delta is done)
  alignas(1024) uint8_t ds[2 * kAtomBytes];
  float sgrad[2][4][D];  // summary gradient / b of the tile's blocks (dK, dV)
  float dpart[4][128];   // delta = rowsum(dO * O): the column parts' sums
  uint64_t ld_full, ld_empty, k_full, k_empty, v_full, v_empty, s_full, ps_full, g_full, g_free;
  uint64_t delta_done, stage_free;
  uint64_t red_done, pub_read, sums_ready, sgrad_free;
  // the dV half (columns 0-127) of a drained chunk has been read: the tile's
  // last chunk may compute its dP there while the dK half is still drained
  uint64_t lo_free;
  uint64_t mma_done;  // exit: every MMA of the CTA has completed
  uint64_t dq_full;   // the tile's dQ accumulation is complete
  uint64_t in_full;   // the in-block K / V buffers have landed (in_bufs)
  int tile_ring;
  uint32_t tmem_base;
};

// kParts gradient warps per TMEM lane quarter; producer, MMA and publisher warps
template <int kParts>
constexpr int bwd_threads() {
  return 32 * (3 + 4 * kParts);
}
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

// TMEM columns: S / dV chunk at 0, dP / dK chunk at 128, dQ at 256; the
// tile's last chunk takes S / dV at 384, so its S is computed while the
// previous chunk's gradients are still read out of columns 0-255.  For b > 128
// (several drained chunks per tile) the last chunk also takes dP / dK at 0,
// so its dP is computed as soon as the previous chunk's dV half (0-127) has
// been read, while the dK half (128-255) is still being drained (the drains
// then read the two halves in two passes).  Measured: T=32K 1.140 -> 1.084 ms
// backward; with b <= 128 the two-pass drain cost more than it gained
// (T=16K +1.9 %, T=8K +2.1 %).
constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256, kColSLast = 384;
template <bool kSplit>
constexpr uint32_t col_dp_last() {
  return kSplit ? 0u : kColDP;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

template <int D, bool kSplit, int kParts>
__global__ void __launch_bounds__(bwd_threads<kParts>(), 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
               const __grid_constant__ CUtensorMap tm_do,
               const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
               const __grid_constant__ CUtensorMap tm_dv,
               const __grid_constant__ CUtensorMap tm_kbar,
               const __grid_constant__ CUtensorMap tm_vbar, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  constexpr bool kIn = in_bufs<D, kSplit>();
  BwdSmem<D, kIn>& sm = *reinterpret_cast<BwdSmem<D, kIn>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t* status = p.ctrl + kStatus;
  const uint32_t token = *reinterpret_cast<volatile uint32_t*>(p.ctrl + kBwdEpoch) + 1u;
  const uint64_t xbudget = cross_wait_budget(p.ctrl);
  constexpr int kAtoms = D / 64;
  constexpr int kGradWarps = 4 * kParts;
  // summary gradients with TMEM lanes = features (needs M = D = 128)
  constexpr bool kTransposedSums = D == 128;
  const uint32_t box_bytes = (uint32_t)p.g.R * 128u;
  const int NT = p.g.tiles_per_seq;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&sm.ld_full, 1);
    ptx::mbar_init(&sm.ld_empty, 1);
    ptx::mbar_init(&sm.delta_done, 1);
    ptx::mbar_init(&sm.red_done, kGradWarps);  // one arrive per gradient warp
    ptx::mbar_init(&sm.pub_read, 1);
    ptx::mbar_init(&sm.sums_ready, 1);
    ptx::mbar_init(&sm.sgrad_free, kGradWarps);  // one arrive per gradient warp
    ptx::mbar_init(&sm.k_full, 1);
    ptx::mbar_init(&sm.k_empty, 1);  // dQ MMA of the chunk complete
    ptx::mbar_init(&sm.v_full, 1);
    ptx::mbar_init(&sm.v_empty, 1);  // dP MMA of the chunk complete
    ptx::mbar_init(&sm.stage_free, 1);
    ptx::mbar_init(&sm.s_full, 1);
    ptx::mbar_init(&sm.ps_full, kGradWarps);
    ptx::mbar_init(&sm.g_full, 1);
    ptx::mbar_init(&sm.g_free, kGradWarps);
    ptx::mbar_init(&sm.lo_free, kGradWarps);  // one arrive per gradient warp
    ptx::mbar_init(&sm.mma_done, 1);
    ptx::mbar_init(&sm.dq_full, 1);
    ptx::mbar_init(&sm.in_full, 1);
    ptx::fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::tma_prefetch_desc(&tm_q);
    ptx::tma_prefetch_desc(&tm_do);
    ptx::tma_prefetch_desc(&tm_k);
    ptx::tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&sm.tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  auto tile_of = [&](int n) {
    return make_tile<kSplit>(p.g, p.H, NT - 1 - n / p.BH, n % p.BH);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // A tile is claimed when its loads can be issued and it can start: Q, dO
    // and O of a tile load once the previous tile's last MMA has read
    // Q/dO/V (ld_empty) and its epilogue has the block sums it waits for
    // (sums_ready), i.e. during the rest of that epilogue.  A tile claimed
    // earlier would hold back every tile of its sequence that waits for its
    // summary gradients (measured: claiming one tile ahead, with or without
    // an L2 prefetch of its inputs, is slower; claiming before sums_ready
    // lets waits compound along long sequences).
    if (lane == 0) {
      auto claim = [&]() {
        const int c = (int)atomicAdd(p.ctrl + kBwdTileCounter, 1u);
        return c < p.total_tiles ? c : -1;
      };
      int tc = 0, kc = 0;  // kc: chunks loaded through the K / V buffers
      while (true) {
        if (tc > 0) {
          ptx::mbar_wait(&sm.ld_empty, (tc - 1) & 1, status, 0x50000000u);
          ptx::mbar_wait(&sm.pub_read, (tc - 1) & 1, status, 0x53000000u);
          // and only once the previous tile's epilogue has everything it
          // waits for: a tile claimed by a CTA whose gradient warps are
          // still waiting would start - and publish - late, and the tiles
          // waiting on it in turn (a convoy on long sequences)
          ptx::mbar_wait(&sm.sums_ready, (tc - 1) & 1, status, 0x56000000u);
        }
        const int n = claim();
        sm.tile_ring = n;
        if (n < 0) {
          // the copies issued so far have landed (they normally have: after a
          // failed wait they may still be in flight)
          if (tc > 0) ptx::mbar_drain(&sm.ld_full, (tc - 1) & 1);
          if constexpr (kIn) {
            if (tc > 0) ptx::mbar_drain(&sm.in_full, (tc - 1) & 1);
          }
          if (kc > 0) {
            ptx::mbar_drain(&sm.k_full, (kc - 1) & 1);
            ptx::mbar_drain(&sm.v_full, (kc - 1) & 1);
          }
          ptx::mbar_arrive(&sm.ld_full);
          break;
        }
        const Tile t = tile_of(n);
        ptx::mbar_arrive_expect_tx(&sm.ld_full, 3 * kAtoms * box_bytes);
#pragma unroll
        for (int a = 0; a < kAtoms; ++a) {
          ptx::tma_load_4d(sm.q + a * kAtomBytes, &tm_q, &sm.ld_full, a * 64, t.h, t.r0, t.n);
          ptx::tma_load_4d(sm.dout + a * kAtomBytes, &tm_do, &sm.ld_full, a * 64, t.h, t.r0,
                           t.n);
          ptx::tma_load_4d(sm.v + a * kAtomBytes, &tm_o, &sm.ld_full, a * 64, t.h, t.r0, t.n);
        }
        // K and V buffers are refilled independently: V as soon as the
        // previous chunk's dP has read it, K once its dQ has (the MMA warp
        // issues dQ last among a chunk's gradient MMAs, so the drain and the
        // epilogue of dK/dV start first).  A tile's first K
        // load also waits for the previous tile's dQ staging in the K buffer
        // to be read by its TMA store; its first V load waits for delta,
        // which reads O from the V buffer.
        const int nch = t.nsc + t.nin;  // summary chunks, then in-block chunks
        // the first chunk loaded into the V buffer waits for delta (O is there)
        const int first_v = t.nsc > 0 ? 1 : 0;
        for (int c = 0; c < nch; ++c) {
          if (kIn && c == t.nsc) continue;  // the in-block chunk, loaded above
          auto load_k = [&]() {
            ptx::mbar_wait(&sm.k_empty, (kc & 1) ^ 1, status, 0x51000000u);
            if (!kIn && c == 0 && tc > 0)
              ptx::mbar_wait(&sm.stage_free, (tc - 1) & 1, status, 0x54000000u);
            if (c < t.nsc) {
              const SumChunk sc = sum_chunk(t, c);
              ptx::mbar_arrive_expect_tx(&sm.k_full, kAtoms * kAtomBytes);
#pragma unroll
              for (int a = 0; a < kAtoms; ++a)
                ptx::tma_load_3d(sm.k + a * kAtomBytes, &tm_kbar, &sm.k_full, a * 64, sc.w, t.bh);
            } else {
              const InChunk ic = in_chunk<kSplit>(t, c - t.nsc);
              ptx::mbar_arrive_expect_tx(&sm.k_full, kAtoms * box_bytes);
#pragma unroll
              for (int a = 0; a < kAtoms; ++a)
                ptx::tma_load_4d(sm.k + a * kAtomBytes, &tm_k, &sm.k_full, a * 64, t.h, ic.k0,
                                 t.n);
            }
          };
          auto load_v = [&]() {
            ptx::mbar_wait(&sm.v_empty, (kc & 1) ^ 1, status, 0x55000000u);
            if (c == first_v) ptx::mbar_wait(&sm.delta_done, tc & 1, status, 0x52000000u);
            if (c < t.nsc) {
              // chunk 0 into the dS buffer, free since the previous tile's
              // staging was read (stage_free, waited for by load_k above), or
              // with in-block buffers (no staging there) once its last MMA
              // has read its dS
              if (kIn && c == 0 && tc > 0)
                ptx::mbar_wait(&sm.dq_full, (tc - 1) & 1, status, 0x57000000u);
              const SumChunk sc = sum_chunk(t, c);
              uint8_t* dst = c == 0 ? sm.ds : sm.v;
              ptx::mbar_arrive_expect_tx(&sm.v_full, kAtoms * kAtomBytes);
#pragma unroll
              for (int a = 0; a < kAtoms; ++a)
                ptx::tma_load_3d(dst + a * kAtomBytes, &tm_vbar, &sm.v_full, a * 64, sc.w, t.bh);
            } else {
              const InChunk ic = in_chunk<kSplit>(t, c - t.nsc);
              ptx::mbar_arrive_expect_tx(&sm.v_full, kAtoms * box_bytes);
#pragma unroll
              for (int a = 0; a < kAtoms; ++a)
                ptx::tma_load_4d(sm.v + a * kAtomBytes, &tm_v, &sm.v_full, a * 64, t.h, ic.k0,
                                 t.n);
            }
          };
          // in the order their buffers free up: for a tile's first chunk K
          // (previous tile's store read) before V (the same store read for a
          // summary chunk, else this tile's delta), for later chunks V
          // (previous dP) before K (previous dQ)
          if (c == 0) {
            load_k();
            load_v();
          } else {
            load_v();
            load_k();
          }
          ++kc;
        }
        if constexpr (kIn) {
          // the tile's own keys and values, needed last: once the previous
          // tile's dQ / dV staging there has been read by its TMA stores
          if (tc > 0) ptx::mbar_wait(&sm.stage_free, (tc - 1) & 1, status, 0x54000000u);
          ptx::mbar_arrive_expect_tx(&sm.in_full, 2 * kAtoms * box_bytes);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a) {
            ptx::tma_load_4d(sm.kin + a * kAtomBytes, &tm_k, &sm.in_full, a * 64, t.h, t.r0,
                             t.n);
            ptx::tma_load_4d(sm.vin + a * kAtomBytes, &tm_v, &sm.in_full, a * 64, t.h, t.r0,
                             t.n);
          }
        }
        ++tc;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_dvdk = ptx::idesc_bf16(128, D, true, true);
      const uint32_t idesc_dq = ptx::idesc_bf16(128, D, false, true);
      const uint32_t q_s = ptx::smem_u32(sm.q), do_s = ptx::smem_u32(sm.dout);
      const uint32_t k_s = ptx::smem_u32(sm.k), v_s = ptx::smem_u32(sm.v);
      const uint32_t p_s = ptx::smem_u32(sm.p), ds_s = ptx::smem_u32(sm.ds);
      uint32_t kin_s = 0, vin_s = 0;
      if constexpr (kIn) {
        kin_s = ptx::smem_u32(sm.kin);
        vin_s = ptx::smem_u32(sm.vin);
      }
      int tc = 0, kc = 0, kv = 0;  // kv: chunks read from the K / V buffers
      int lc = 0;                  // drained (non-last) chunks: lo_free phases
      while (true) {
        ptx::mbar_wait(&sm.ld_full, tc & 1, status, 0x60000000u);
        const int n = sm.tile_ring;
        if (n < 0) break;
        const Tile t = tile_of(n);
        const int kq = round16(t.rows) / 16;  // k-steps over query rows
        const int nch = t.nsc + t.nin;
        for (int c = 0; c < nch; ++c) {
          const int N = c < t.nsc ? sum_chunk(t, c).n16 : in_chunk<kSplit>(t, c - t.nsc).n;
          // a later last chunk's S goes to free columns, and its dP only waits
          // for the dV half of the previous chunk's gradients to be read
          // (lo_free), not for the whole drain (g_free)
          const bool last = c == nch - 1;
          const bool late_last = c > 0 && last;
          const uint32_t col_s = last ? kColSLast : kColS;
          const uint32_t col_dp = last ? col_dp_last<kSplit>() : kColDP;
          const bool inb = kIn && c == t.nsc;  // K / V in the in-block buffers
          const uint32_t kc_s = inb ? kin_s : k_s;
          if (inb)
            ptx::mbar_wait(&sm.in_full, tc & 1, status, 0x65000000u);
          else
            ptx::mbar_wait(&sm.k_full, kv & 1, status, 0x61000000u);
          if (kc > 0 && !late_last)
            ptx::mbar_wait(&sm.g_free, (kc - 1) & 1, status, 0x62000000u);
          ptx::tc_fence_after();
          const uint32_t idesc_s = ptx::idesc_bf16(128, N, false, false);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            ptx::mma_ss(tmem + col_s, desc_kmajor(q_s, kk), desc_kmajor(kc_s, kk), idesc_s,
                        kk > 0 ? 1u : 0u);
          if (!inb) ptx::mbar_wait(&sm.v_full, kv & 1, status, 0x64000000u);
          if (late_last) {
            if constexpr (kSplit)
              ptx::mbar_wait(&sm.lo_free, (lc - 1) & 1, status, 0x66000000u);
            else
              ptx::mbar_wait(&sm.g_free, (kc - 1) & 1, status, 0x62000000u);
          }
          ptx::tc_fence_after();
          // where this chunk's V is
          const uint32_t vc_s = inb ? vin_s : (c == 0 && t.nsc > 0) ? ds_s : v_s;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            ptx::mma_ss(tmem + col_dp, desc_kmajor(do_s, kk), desc_kmajor(vc_s, kk), idesc_s,
                        kk > 0 ? 1u : 0u);
          ptx::mma_commit(&sm.s_full);
          if (!inb) ptx::mma_commit(&sm.v_empty);  // the V chunk is read only by dP
          ptx::mbar_wait(&sm.ps_full, kc & 1, status, 0x63000000u);
          ptx::tc_fence_after();
          // dVc / dKc first: their drain (or the epilogue) starts while dQ runs
          if (kTransposedSums && c < t.nsc) {
            // summary gradients transposed (D = 128 = M): all 128 columns of
            // P / dS, zero outside the chunk's visible summaries
            // N = the chunk's n16 summary columns: only what the drain reads
            const uint32_t idesc_sum = ptx::idesc_bf16(128, N, true, true);
            for (int kk = 0; kk < kq; ++kk)  // dVc^T = dO^T P
              ptx::mma_ss(tmem + kColS, desc_mnmajor(do_s, kk), desc_mnmajor(p_s, kk), idesc_sum,
                          kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < kq; ++kk)  // dKc^T = Q^T dS
              ptx::mma_ss(tmem + kColDP, desc_mnmajor(q_s, kk), desc_mnmajor(ds_s, kk), idesc_sum,
                          kk > 0 ? 1u : 0u);
          } else {
            for (int kk = 0; kk < kq; ++kk)  // dVc = P^T dO
              ptx::mma_ss(tmem + col_s, desc_mnmajor(p_s, kk), desc_mnmajor(do_s, kk), idesc_dvdk,
                          kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < kq; ++kk)  // dKc = dS^T Q
              ptx::mma_ss(tmem + col_dp, desc_mnmajor(ds_s, kk), desc_mnmajor(q_s, kk), idesc_dvdk,
                          kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(&sm.g_full);
          if (c == nch - 1) ptx::mma_commit(&sm.ld_empty);  // Q, dO, V no longer read
          for (int kk = 0; kk < N / 16; ++kk)  // dQ += dS Kc
            ptx::mma_ss(tmem + kColDQ, desc_kmajor(ds_s, kk), desc_mnmajor(kc_s, kk), idesc_dq,
                        (c > 0 || kk > 0) ? 1u : 0u);
          if (!inb) ptx::mma_commit(&sm.k_empty);
          if (c == nch - 1) ptx::mma_commit(&sm.dq_full);
          ++kc;
          if (!inb) ++kv;
          if (!last) ++lc;
        }
        ++tc;
      }
      // every MMA issued has completed before TMEM is released
      ptx::mma_commit(&sm.mma_done);
      ptx::mbar_drain(&sm.mma_done, 0);
    }
  } else if (warp < 2 + kGradWarps) {
    // ------------------------------------------------------------ gradient warps
    // kParts warps per TMEM lane quarter: part h = (warp - 2) / 4 takes key
    // columns [h*128/kParts, (h+1)*128/kParts) of S/dP and columns
    // [h*D/kParts, (h+1)*D/kParts) of dK, dV and dQ, so every per-row loop is
    // 1/kParts as long as with one warp per quarter.
    const int gtid = threadIdx.x - 64;  // 0 .. 32 * kGradWarps - 1
    const int part = (warp - 2) >> 2;   // column part
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane: query row, then key row
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    constexpr int kPartD = D / kParts;        // dK / dV / dQ columns of a part
    constexpr int kPieces = 128 / kParts / 16;  // 16-column S / dP pieces of a part
    constexpr int kGradThreads = 32 * kGradWarps;
    int tc = 0, kc = 0;
    while (true) {
      ptx::mbar_wait(&sm.ld_full, tc & 1, status, 0x70000000u);
      const int n = sm.tile_ring;
      if (n < 0) break;
      const Tile t = tile_of(n);
      const bool valid = row < t.rows;
      const int tq = t.r0 + row;
      const int blk_t = valid ? tq / p.g.b : 0;
      const int lim = valid ? min(blk_t, p.g.Gc) : 0;
      // The row's LSE is loaded here and first used after the delta barrier:
      // a warp issues in order and would otherwise stall on this global load
      // (a few thousand cycles under load) before computing delta.
      float L = valid ? __ldg(p.lse + (size_t)t.bh * p.g.T + tq) : 0.f;
      // delta = rowsum(dO * O); O was loaded into the V buffer.  Each part sums
      // its D/kParts columns; the parts meet in shared memory.
      float dpart_sum = 0.f;
      if (valid) {
#pragma unroll 4
        for (int cc = part * (D / 8 / kParts); cc < (part + 1) * (D / 8 / kParts); ++cc) {
          const uint32_t off = swz_offset(row, cc * 8);
          const uint4 a = *reinterpret_cast<const uint4*>(sm.v + off);
          const uint4 g = *reinterpret_cast<const uint4*>(sm.dout + off);
          dpart_sum += bf16lo(a.x) * bf16lo(g.x) + bf16hi(a.x) * bf16hi(g.x) +
                   bf16lo(a.y) * bf16lo(g.y) + bf16hi(a.y) * bf16hi(g.y) +
                   bf16lo(a.z) * bf16lo(g.z) + bf16hi(a.z) * bf16hi(g.z) +
                   bf16lo(a.w) * bf16lo(g.w) + bf16hi(a.w) * bf16hi(g.w);
        }
      }
      sm.dpart[part][row] = dpart_sum;
      // the previous tile's dK staging (P buffer) has been read by its TMA
      // store before this tile's P/dS are written (after the barrier)
      if (gtid == 0 && tc > 0) ptx::tma_store_wait_read_all();
      // This tile's O (V buffer) has been consumed into delta: the first V
      // chunk may be loaded.
      ptx::named_barrier(1, kGradThreads);
      if (gtid == 0) ptx::mbar_arrive(&sm.delta_done);
      ptx::reg_fence1(L);  // first use of the LSE load: after delta
      L *= kLog2e;
      float delta = sm.dpart[0][row];
#pragma unroll
      for (int i = 1; i < kParts; ++i) delta += sm.dpart[i][row];

      // P and dS of one chunk into smem (this part's key columns; masked -> 0)
      auto softmax_grad = [&](int N, int vlo, int vhi, uint32_t col_s, uint32_t col_dp) {
        const bool any_col = vhi > vlo;
        const int wlo = __reduce_min_sync(0xffffffffu, any_col ? vlo : 0x7fffffff);
        const int whi = __reduce_max_sync(0xffffffffu, any_col ? vhi : 0);
        // pieces every lane of the warp sees whole need no mask
        const int lo_max = __reduce_max_sync(0xffffffffu, any_col ? vlo : 0x7fffffff);
        const int hi_min = __reduce_min_sync(0xffffffffu, any_col ? vhi : 0);
        const float delta_s = delta * p.scale;
        // this part's 16-column pieces; a piece is live (warp-uniform) when it
        // holds a column some row of this warp sees
        // pieces of the parts interleave (piece pi of part h covers columns
        // 16 * (pi * kParts + h)), so a chunk with few live columns - a summary
        // chunk of few summaries, the causal chunk's lower lane quarters -
        // still splits them between the parts
        auto col0 = [&](int pi) { return (pi * kParts + part) * 16; };
        auto live = [&](int pi) {
          const int c0 = col0(pi);
          return c0 < N && c0 < whi && c0 + 16 > wlo;
        };
        auto load = [&](int pi, uint32_t (&sv)[16], uint32_t (&dp)[16]) {
          if (live(pi)) {
            ptx::tmem_ld16(tmem + lane_off + col_s + col0(pi), sv);
            ptx::tmem_ld16(tmem + lane_off + col_dp + col0(pi), dp);
          }
        };
        // P = exp2(S*c - L), dS = P * (dP*scale - delta*scale); masked -> 0.
        // A piece no row of the warp sees only gets its zeros (warp-uniform):
        // the MMAs read every column, and its exponentials would be discarded.
        auto emit = [&](int pi, const uint32_t (&sv)[16], const uint32_t (&dp)[16]) {
          const int c0 = col0(pi);
          const bool lv = live(pi);
          if (!lv) {
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int j8 = 0; j8 < 2; ++j8) {
              const uint32_t off = swz_offset(row, c0 + j8 * 8);
              *reinterpret_cast<uint4*>(sm.p + off) = z;
              *reinterpret_cast<uint4*>(sm.ds + off) = z;
            }
            return;
          }
          const bool whole = c0 >= lo_max && c0 + 16 <= hi_min;
#pragma unroll
          for (int j8 = 0; j8 < 2; ++j8) {
            uint32_t pw[4], dw[4];
#pragma unroll
            for (int h2 = 0; h2 < 4; ++h2) {
              float pv[2], dv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int j = j8 * 8 + h2 * 2 + e;
                const float pr = ptx::ex2(fmaf(__uint_as_float(sv[j]), p.scale_log2, -L));
                const float dr = pr * fmaf(__uint_as_float(dp[j]), p.scale, -delta_s);
                if (whole) {
                  pv[e] = pr;
                  dv[e] = dr;
                } else {
                  const bool ok = (uint32_t)(c0 + j - vlo) < (uint32_t)(vhi - vlo);
                  pv[e] = ok ? pr : 0.f;
                  dv[e] = ok ? dr : 0.f;
                }
              }
              pw[h2] = ptx::pack_bf16x2(pv[0], pv[1]);
              dw[h2] = ptx::pack_bf16x2(dv[0], dv[1]);
            }
            const uint32_t off = swz_offset(row, c0 + j8 * 8);
            *reinterpret_cast<uint4*>(sm.p + off) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
            *reinterpret_cast<uint4*>(sm.ds + off) = make_uint4(dw[0], dw[1], dw[2], dw[3]);
          }
        };
        ptx::mbar_wait(&sm.s_full, kc & 1, status, 0x71000000u);
        ptx::tc_fence_after();
#pragma unroll 1
        for (int pi = 0; pi < kPieces; ++pi) {
          uint32_t sv[16], dp[16];
          load(pi, sv, dp);
          ptx::tmem_wait_ld();
          ptx::reg_fence(sv);
          ptx::reg_fence(dp);
          emit(pi, sv, dp);
        }
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&sm.ps_full);
        ptx::mbar_wait(&sm.g_full, kc & 1, status, 0x72000000u);
        ptx::tc_fence_after();
      };

      // Adds this lane's row of a chunk's dKc / dVc (TMEM, S and dP columns,
      // this warp's column part) to fp32 rows of the workspace with vector
      // atomics, then frees the columns for the next chunk's S/dP.
      // store: plain stores instead of atomic additions (a destination with a
      // single writer)
      // b > 128: two passes, dV (columns 0-127), after which lo_free lets the
      // tile's last chunk compute its dP there, then dK (columns 128-255),
      // g_free; otherwise both halves of a piece at once, then g_free.
      auto drain = [&](float* dkrow, float* dvrow, bool ok, bool store) {
        if constexpr (!kSplit) {
#pragma unroll 1
          for (int pc = 0; pc < kPartD / 16; ++pc) {
            const int col0 = part * kPartD + pc * 16;
            uint32_t gv[16], gk[16];
            ptx::tmem_ld16(tmem + lane_off + kColS + col0, gv);
            ptx::tmem_ld16(tmem + lane_off + kColDP + col0, gk);
            ptx::tmem_wait_ld();
            ptx::reg_fence(gv);
            ptx::reg_fence(gk);
            if (ok) {
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4) {
                ptx::red_add_v4(dvrow + col0 + 4 * j4, __uint_as_float(gv[4 * j4]),
                                __uint_as_float(gv[4 * j4 + 1]), __uint_as_float(gv[4 * j4 + 2]),
                                __uint_as_float(gv[4 * j4 + 3]));
                ptx::red_add_v4(dkrow + col0 + 4 * j4, __uint_as_float(gk[4 * j4]),
                                __uint_as_float(gk[4 * j4 + 1]), __uint_as_float(gk[4 * j4 + 2]),
                                __uint_as_float(gk[4 * j4 + 3]));
              }
            }
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&sm.g_free);
          ++kc;
          return;
        }
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          const uint32_t tcol = half == 0 ? kColS : kColDP;
          float* dst = half == 0 ? dvrow : dkrow;
#pragma unroll 1
          for (int pc = 0; pc < kPartD / 16; ++pc) {
            const int col0 = part * kPartD + pc * 16;
            uint32_t g[16];
            ptx::tmem_ld16(tmem + lane_off + tcol + col0, g);
            ptx::tmem_wait_ld();
            ptx::reg_fence(g);
            if (ok && store) {
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4)
                __stcg(reinterpret_cast<uint4*>(dst + col0 + 4 * j4),
                       make_uint4(g[4 * j4], g[4 * j4 + 1], g[4 * j4 + 2], g[4 * j4 + 3]));
            } else if (ok) {
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4)
                ptx::red_add_v4(dst + col0 + 4 * j4, __uint_as_float(g[4 * j4]),
                                __uint_as_float(g[4 * j4 + 1]), __uint_as_float(g[4 * j4 + 2]),
                                __uint_as_float(g[4 * j4 + 3]));
            }
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(half == 0 ? &sm.lo_free : &sm.g_free);
        }
        ++kc;
      };

      // Transposed summary chunk (D = 128): this lane holds feature d = row of
      // the chunk's summaries in columns; one scalar atomic per summary, and
      // each warp instruction covers 32 consecutive features of one summary.
      auto drain_sums_t = [&](const SumChunk& sc) {
        const int clo = sc.lo - sc.w, chi = sc.e - sc.w;  // columns of real summaries
        float* dvb = p.dvbar + (size_t)t.bh * p.g.Gc * D + row;
        float* dkb = p.dkbar + (size_t)t.bh * p.g.Gc * D + row;
        if constexpr (!kSplit) {
#pragma unroll 1
          for (int pc = 0; pc < kPieces; ++pc) {
            const int col0 = (pc * kParts + part) * 16;  // interleaved as in softmax_grad
            if (col0 + 16 <= clo || col0 >= chi) continue;  // warp-uniform
            uint32_t gv[16], gk[16];
            ptx::tmem_ld16(tmem + lane_off + kColS + col0, gv);
            ptx::tmem_ld16(tmem + lane_off + kColDP + col0, gk);
            ptx::tmem_wait_ld();
            ptx::reg_fence(gv);
            ptx::reg_fence(gk);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int col = col0 + jj;
              if (col >= clo && col < chi) {
                const size_t off = (size_t)(sc.w + col) * D;
                ptx::red_add_f32(dvb + off, __uint_as_float(gv[jj]));
                ptx::red_add_f32(dkb + off, __uint_as_float(gk[jj]));
              }
            }
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&sm.g_free);
          ++kc;
          return;
        }
        // b > 128: two passes as in drain, dVbar^T (then lo_free), dKbar^T
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          const uint32_t tcol = half == 0 ? kColS : kColDP;
          float* dst = half == 0 ? dvb : dkb;
#pragma unroll 1
          for (int pc = 0; pc < kPieces; ++pc) {
            const int col0 = (pc * kParts + part) * 16;  // interleaved as in softmax_grad
            if (col0 + 16 <= clo || col0 >= chi) continue;  // warp-uniform
            uint32_t g[16];
            ptx::tmem_ld16(tmem + lane_off + tcol + col0, g);
            ptx::tmem_wait_ld();
            ptx::reg_fence(g);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int col = col0 + jj;
              if (col >= clo && col < chi)
                ptx::red_add_f32(dst + (size_t)(sc.w + col) * D, __uint_as_float(g[jj]));
            }
          }
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(half == 0 ? &sm.lo_free : &sm.g_free);
        }
        ++kc;
      };

      // ---- summary chunks: add dKc / dVc to the summary accumulators
      for (int c = 0; c < t.nsc; ++c) {
        const SumChunk sc = sum_chunk(t, c);
        softmax_grad(sc.n16, sc.lo - sc.w, min(sc.e, lim) - sc.w, kColS, kColDP);
        if constexpr (kTransposedSums) {
          drain_sums_t(sc);
        } else {
          const int j = sc.w + row;  // this lane's summary
          const size_t jr = (size_t)t.bh * p.g.Gc + j;
          drain(p.dkbar + jr * D, p.dvbar + jr * D, row >= sc.lo - sc.w && row < sc.e - sc.w,
                false);
        }
      }

      // ---- b > 128: in-block chunks before this sub-tile's rows.  Every key is
      // visible to every row; their dKc / dVc belong to the keys of earlier
      // sub-tiles of the block and are added to the workspace accumulators
      // that those sub-tiles' epilogues read.
      for (int u = 0; u + 1 < t.nin; ++u) {
        softmax_grad(kTileRows, 0, valid ? kTileRows : 0, kColS, kColDP);
        const size_t xr = ((size_t)t.bh * p.G + t.blk0) * p.xrows + u * kTileRows + row;
        // with two sub-tiles per block (b <= 256) a key's cross contribution
        // has one writer: stored, and never re-zeroed (each launch rewrites it
        // before it is read); with more, added and re-zeroed by the reader
        drain(p.dkx + xr * D, p.dvx + xr * D, true, p.g.tpb == 2);
      }

      // ---- publish (by the publisher warp): this warp's additions are done
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sm.red_done);

      // ---- the in-block chunk of the tile's own rows (causal)
      softmax_grad(t.n_in, valid ? max(0, blk_t * p.g.b - t.r0) : 0, valid ? row + 1 : 0,
                   kColSLast, col_dp_last<kSplit>());
      // the publisher has staged sum / b of the tile's complete blocks
      ptx::mbar_wait(&sm.sums_ready, tc & 1, status, 0x73000000u);
      // dQ (the tile's last MMA) has read dS: the dS buffer may take dV staging
      ptx::mbar_wait(&sm.dq_full, tc & 1, status, 0x76000000u);
      ptx::tc_fence_after();
      {
        // staging of dQ and dV: the K and dS buffers, or the in-block K / V
        // buffers where there are some (their MMAs have completed too)
        uint8_t* stage_q = sm.k;
        uint8_t* stage_v = sm.ds;
        if constexpr (kIn) {
          stage_q = sm.kin;
          stage_v = sm.vin;
        }
        const bool complete = valid && blk_t < p.g.Gc;  // this lane's key is in a full block
        const int lb_t = valid ? blk_t - t.blk0 : 0;
        // b > 128: a sub-tile followed by others in its block adds their
        // contributions to its keys (and re-zeroes them)
        const bool cross = kSplit && valid && t.sub + 1 < block_tiles(p.g, t.blk0);
        const size_t xr = ((size_t)t.bh * p.G + t.blk0) * p.xrows + t.sub * kTileRows + row;
        // dV (kv = 1: TMEM S columns -> dV staging) or dK (kv = 0: dP columns ->
        // P buffer) of the tile's keys, plus (summary gradient of the key's
        // block) / b and, for b > 128, the later sub-tiles' contributions
        auto stage_grad = [&](int kv) {
          const uint32_t tcol = kv ? kColSLast : col_dp_last<kSplit>();
          const float* srow = sm.sgrad[kv][lb_t];
          float* xrow = (kv ? p.dvx : p.dkx) + xr * D;
          uint8_t* dst = kv ? stage_v : sm.p;
#pragma unroll 1
          for (int pc = 0; pc < kPartD / 16; ++pc) {
            const int col0 = part * kPartD + pc * 16;
            uint32_t g[16];
            ptx::tmem_ld16(tmem + lane_off + tcol + col0, g);
            ptx::tmem_wait_ld();
            ptx::reg_fence(g);
#pragma unroll
            for (int j8 = 0; j8 < 2; ++j8) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(g[8 * j8 + e]);
              const int col = col0 + j8 * 8;
              if (complete) {
                const float4 s0 = *reinterpret_cast<const float4*>(srow + col);
                const float4 s1 = *reinterpret_cast<const float4*>(srow + col + 4);
                f[0] += s0.x; f[1] += s0.y; f[2] += s0.z; f[3] += s0.w;
                f[4] += s1.x; f[5] += s1.y; f[6] += s1.z; f[7] += s1.w;
              }
              if (cross) {
                float4* x = reinterpret_cast<float4*>(xrow + col);
                const float4 x0 = __ldcg(x), x1 = __ldcg(x + 1);
                if (p.g.tpb > 2) {
                  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
                  __stcg(x, z);
                  __stcg(x + 1, z);
                }
                f[0] += x0.x; f[1] += x0.y; f[2] += x0.z; f[3] += x0.w;
                f[4] += x1.x; f[5] += x1.y; f[6] += x1.z; f[7] += x1.w;
              }
              *reinterpret_cast<uint4*>(dst + swz_offset(row, col)) =
                  make_uint4(ptx::pack_bf16x2(f[0], f[1]), ptx::pack_bf16x2(f[2], f[3]),
                             ptx::pack_bf16x2(f[4], f[5]), ptx::pack_bf16x2(f[6], f[7]));
            }
          }
        };
        auto issue_stores = [&](const CUtensorMap* tm, const uint8_t* src) {
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            for (int r = 0; r < t.rows; r += p.store_rows)
              ptx::tma_store_4d(tm, src + a * kAtomBytes + r * 128, a * 64, t.h, t.r0 + r, t.n);
        };
        // 1. dQ and dV, stored as one bulk group: once it has been read, the
        // next tile's first K and V chunks (or its in-block K and V) load there
#pragma unroll 1
        for (int pc = 0; pc < kPartD / 16; ++pc) {
          const int col0 = part * kPartD + pc * 16;
          uint32_t gq[16];
          ptx::tmem_ld16(tmem + lane_off + kColDQ + col0, gq);
          ptx::tmem_wait_ld();
          ptx::reg_fence(gq);
#pragma unroll
          for (int j8 = 0; j8 < 2; ++j8) {
            const uint32_t off = swz_offset(row, col0 + j8 * 8);
            *reinterpret_cast<uint4*>(stage_q + off) = make_uint4(
                ptx::pack_bf16x2(__uint_as_float(gq[8 * j8]), __uint_as_float(gq[8 * j8 + 1])),
                ptx::pack_bf16x2(__uint_as_float(gq[8 * j8 + 2]), __uint_as_float(gq[8 * j8 + 3])),
                ptx::pack_bf16x2(__uint_as_float(gq[8 * j8 + 4]), __uint_as_float(gq[8 * j8 + 5])),
                ptx::pack_bf16x2(__uint_as_float(gq[8 * j8 + 6]),
                                 __uint_as_float(gq[8 * j8 + 7])));
          }
        }
        stage_grad(1);
        ptx::fence_proxy_async_smem();
        ptx::named_barrier(1, kGradThreads);
        if (gtid == 0) {
          issue_stores(&tm_dq, stage_q);
          issue_stores(&tm_dv, stage_v);
          ptx::tma_store_commit();
        }
        // 2. dK (P buffer), its own bulk group
        stage_grad(0);
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          ptx::mbar_arrive(&sm.g_free);
          ptx::mbar_arrive(&sm.sgrad_free);
        }
        ptx::fence_proxy_async_smem();
        ptx::named_barrier(1, kGradThreads);
        if (gtid == 0) {
          issue_stores(&tm_dk, sm.p);
          ptx::tma_store_commit();
          // the dQ / dV group has been read: its buffers may take the next
          // tile's loads (stage_free).  The P buffer is
          // rewritten only after the barrier that follows the next tile's
          // delta, before which this thread waits for the dK read.
          ptx::tma_store_wait_read_1();
          ptx::mbar_arrive(&sm.stage_free);
        }
        ++kc;
      }
      ++tc;
    }
    if (gtid == 0) ptx::tma_store_wait_all();
  } else {
    // ------------------------------------------------------------ publisher
    // Per tile: (1) makes the tile's summary-gradient additions visible to
    // other CTAs.  The gradient warps arrive on red_done after their last
    // addition (the arrive orders them at CTA scope); lane 0's release add at
    // GPU scope then covers them for any CTA that acquires the counter, which
    // reaches token once per launch.  The release waits until every
    // outstanding addition is acknowledged, so it is kept off the gradient
    // warps.  (2) Waits until every later tile of the sequence has published,
    // stages sum / b of each of the tile's complete blocks in smem for the
    // gradient warps' epilogue (sums_ready), and re-zeroes the consumed sums.
    const float inv_b = 1.f / (float)p.g.b;
    int tc = 0;
    while (true) {
      ptx::mbar_wait(&sm.ld_full, tc & 1, status, 0x80000000u);
      const int n = sm.tile_ring;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sm.pub_read);  // the producer may rewrite tile_ring
      if (n < 0) break;
      const Tile t = tile_of(n);
      ptx::mbar_wait(&sm.red_done, tc & 1, status, 0x81000000u);
      if (lane == 0) ptx::red_release_add(p.flags + (size_t)t.bh * p.flags_stride + t.s, 1u);
      ptx::counters_wait_range(p.flags + (size_t)t.bh * p.flags_stride, t.s + 1, NT, token,
                               status, (uint32_t)n, xbudget);
      if (tc > 0) ptx::mbar_wait(&sm.sgrad_free, (tc - 1) & 1, status, 0x82000000u);
      constexpr bool split = kSplit;
      const int nb = split ? 1 : p.g.R / p.g.b;  // blocks the tile's rows cover
      const int nfull = max(0, min(nb, p.g.Gc - t.blk0));
      for (int lb = 0; lb < nfull; ++lb) {
        const size_t base = ((size_t)t.bh * p.g.Gc + t.blk0 + lb) * D;
        for (int i = lane * 4; i < D; i += 128) {
          const float4 k4 = __ldcg(reinterpret_cast<const float4*>(p.dkbar + base + i));
          const float4 v4 = __ldcg(reinterpret_cast<const float4*>(p.dvbar + base + i));
          *reinterpret_cast<float4*>(&sm.sgrad[0][lb][i]) =
              make_float4(k4.x * inv_b, k4.y * inv_b, k4.z * inv_b, k4.w * inv_b);
          *reinterpret_cast<float4*>(&sm.sgrad[1][lb][i]) =
              make_float4(v4.x * inv_b, v4.y * inv_b, v4.z * inv_b, v4.w * inv_b);
        }
        // The sums are re-zeroed by their last reader: the tile itself for
        // b <= 128; for b > 128, of the block's sub-tiles (which read in any
        // order), the one whose count increment (acq_rel, after its reads)
        // completes the count.
        bool last = true;
        if (split) {
          __syncwarp();
          uint32_t prev = 0;
          if (lane == 0)
            prev = ptx::atom_add_acq_rel_gpu(p.readers + (size_t)t.bh * p.G + t.blk0, 1u);
          prev = __shfl_sync(0xffffffffu, prev, 0);
          last = prev + 1 == (uint32_t)p.g.tpb;
          if (last && lane == 0) p.readers[(size_t)t.bh * p.G + t.blk0] = 0u;
          __syncwarp();
        }
        if (last) {
          for (int i = lane * 4; i < D; i += 128) {
            *reinterpret_cast<float4*>(p.dkbar + base + i) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(p.dvbar + base + i) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&sm.sums_ready);
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
    const uint32_t prev = atomicAdd(p.ctrl + kBwdExitCounter, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(p.ctrl + kBwdTileCounter, 0u);
      atomicExch(p.ctrl + kBwdExitCounter, 0u);
      __threadfence();
      atomicExch(p.ctrl + kBwdEpoch, token);
      post_status(p.ctrl);
    }
  }
}

template <int D, bool kSplit, int kParts>
int launch(const Problem& pr, const BwdTensorMaps& tm, const float* lse, TensorView o,
           uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream) {
  BwdParams p;
  p.g.T = pr.T;
  p.g.b = pr.b;
  p.g.Gc = pr.Gc;
  p.g.R = tile_rows(pr.b);
  p.g.tiles_per_seq = tiles_per_seq(pr.T, pr.b);
  p.g.tpb = tiles_per_block(pr.b);
  p.store_rows = store_rows(pr.b);
  p.G = pr.G;
  p.xrows = pr.b > 128 ? (tiles_per_block(pr.b) - 1) * 128 : 0;
  p.H = pr.H;
  p.BH = pr.B * pr.H;
  p.total_tiles = p.g.tiles_per_seq * p.BH;
  p.scale = pr.scale;
  p.scale_log2 = pr.scale * kLog2e;
  p.lse = lse;
  p.o = reinterpret_cast<const __nv_bfloat16*>(o.ptr);
  p.o_sb = o.sb;
  p.o_st = o.st;
  p.o_sh = o.sh;
  p.dkbar = reinterpret_cast<float*>(ws + wl.dkbar);
  p.dvbar = reinterpret_cast<float*>(ws + wl.dvbar);
  p.dkx = reinterpret_cast<float*>(ws + wl.dkx);
  p.dvx = reinterpret_cast<float*>(ws + wl.dvx);
  p.readers = reinterpret_cast<uint32_t*>(ws + wl.readers);
  p.ctrl = reinterpret_cast<uint32_t*>(ws + wl.ctrl);
  p.flags = reinterpret_cast<uint32_t*>(ws + wl.flags_bwd);
  p.flags_stride = wl.tiles_per_seq;
  const size_t smem = sizeof(BwdSmem<D, in_bufs<D, kSplit>()>) + 1024;
  static_assert(sizeof(BwdSmem<D, in_bufs<D, kSplit>()>) + 1024 <= 227 * 1024,
                "backward shared memory");
  auto kern = bwd_kernel<D, kSplit, kParts>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return SQB_ERR_LAUNCH;
  const int grid = p.total_tiles < num_sms ? p.total_tiles : num_sms;
  kern<<<grid, bwd_threads<kParts>(), smem, stream>>>(tm.q, tm.k, tm.v, tm.o, tm.dout, tm.dq,
                                                      tm.dk, tm.dv, tm.kbar, tm.vbar, p);
  return cudaGetLastError() == cudaSuccess ? SQB_OK : SQB_ERR_LAUNCH;
}

}  // namespace

int launch_backward(const Problem& pr, const BwdTensorMaps& tm, const float* lse, TensorView o,
                    uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream) {
  const bool split = pr.b > 128;
  constexpr int P = SQB_BWD_PARTS;
  if (pr.D == 64)
    return split ? launch<64, true, P>(pr, tm, lse, o, ws, wl, num_sms, stream)
                 : launch<64, false, P>(pr, tm, lse, o, ws, wl, num_sms, stream);
  if (pr.D == 128)
    return split ? launch<128, true, P>(pr, tm, lse, o, ws, wl, num_sms, stream)
                 : launch<128, false, P>(pr, tm, lse, o, ws, wl, num_sms, stream);
  return SQB_ERR_UNSUPPORTED;
}

}  // namespace sm100
}  // namespace sqb
