// Shared definitions of the sm_100a forward and backward kernels: tile geometry,
// kernel parameters and the shared-memory swizzle used by every operand tile.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "sqb_internal.cuh"
#include "sqb_ptx.cuh"

namespace sqb {
namespace sm100 {

constexpr int kTileRows = 128;    // TMEM lanes / UMMA M
constexpr int kAtomCols = 64;     // bf16 columns per 128-byte swizzle atom
constexpr int kAtomBytes = kTileRows * 128;  // one 64-column atom of a 128-row tile

// Work tile: a run of query rows that starts on a block boundary.  For
// b <= 128 a tile holds whole blocks (R = 128 when b divides 128, else R = b,
// one block per tile).  For b > 128 a block is split into tpb = ceil(b / 128)
// sub-tiles of up to 128 rows; sub-tile v of a block sees the block's keys in
// v + 1 in-block chunks of 128: chunks u < v lie wholly before its rows (every
// key visible), chunk v holds its own rows (causal).
// Tiles of one (batch, head) sequence are numbered s = 0 .. tiles_per_seq-1.
struct Geometry {
  int T, b, Gc, R, tiles_per_seq;
  int tpb;  // sub-tiles per block (b > 128), else 1
};

struct Tile {
  int s, bh, n, h;  // sequence tile, batch*head, batch, head
  int r0, rows;     // first row, valid rows (<= 128)
  int blk0;         // first block of the tile
  int sub;          // sub-tile index within its block (b > 128), else 0
  int nin;          // in-block chunks: sub + 1
  int kin0;         // first key row of in-block chunk 0
  int ns;           // summaries the last row sees: min(last block, Gc)
  int nsc;          // summary chunks of <= 128 summaries
  int n_in;         // MMA N of the diagonal in-block chunk (rows rounded up to 16)
};

__host__ __device__ inline int round16(int x) { return (x + 15) & ~15; }

// Budget of this launch's waits on other CTAs: the workspace's setting, else 2 s.
__device__ inline uint64_t cross_wait_budget(const uint32_t* ctrl) {
  const uint32_t us = *reinterpret_cast<const volatile uint32_t*>(ctrl + kWaitBudgetUs);
  return us ? (uint64_t)us * 1000ull : ptx::kWaitBudgetNs;
}

// Run by the last CTA to leave a launch.  A failure recorded by the launch is
// posted to the caller's host-mapped mailbox (detail first, then the status
// word the host polls), so the host learns of it without synchronizing; the
// abort word is cleared, since the next launch's pipelines start in step.
// The status word itself stays until sqb_read_status clears it.
__device__ inline void post_status(uint32_t* ctrl) {
  volatile uint32_t* c = ctrl;
  const uint32_t st = c[kStatus];
  if (st != 0u) {
    const uint64_t mb = ((uint64_t)c[kMailboxHi] << 32) | (uint64_t)c[kMailboxLo];
    if (mb != 0ull) {
      volatile uint32_t* m = reinterpret_cast<volatile uint32_t*>(mb);
      m[1] = c[kStatusDetail];
      __threadfence_system();
      m[0] = st;
      __threadfence_system();
    }
  }
  c[kStatusAbort] = 0u;
}

// kSplit: the geometry has b > 128 (kernels are compiled for one case or the
// other, so the b <= 128 path carries no sub-tile logic).
template <bool kSplit>
__device__ inline Tile make_tile(const Geometry& g, int H, int s, int bh) {
  Tile t;
  t.s = s;
  t.bh = bh;
  t.n = bh / H;
  t.h = bh % H;
  if constexpr (kSplit) {
    t.blk0 = s / g.tpb;
    t.sub = s % g.tpb;
    t.kin0 = t.blk0 * g.b;
    t.r0 = t.kin0 + t.sub * kTileRows;
    t.rows = min(min(kTileRows, g.b - t.sub * kTileRows), g.T - t.r0);
  } else {
    t.r0 = s * g.R;
    t.rows = min(g.R, g.T - t.r0);
    t.blk0 = t.r0 / g.b;
    t.sub = 0;
    t.kin0 = t.r0;
  }
  t.nin = kSplit ? t.sub + 1 : 1;
  const int last_blk = (t.r0 + t.rows - 1) / g.b;
  t.ns = min(last_blk, g.Gc);
  t.nsc = (t.ns + 127) / 128;
  t.n_in = round16(t.rows);
  return t;
}

// In-block chunk u of a tile: keys [k0, k0 + n) of the tile's block, MMA width n.
struct InChunk {
  int k0, n;
  bool diag;  // the tile's own rows (causal); otherwise every key is visible
};

template <bool kSplit>
__device__ inline InChunk in_chunk(const Tile& t, int u) {
  InChunk k;
  if constexpr (!kSplit) {
    k.k0 = t.r0;
    k.diag = true;
    k.n = t.n_in;
    return k;
  }
  k.k0 = t.kin0 + kTileRows * u;
  k.diag = u == t.nin - 1;
  k.n = k.diag ? t.n_in : kTileRows;
  return k;
}

// In-block chunk processed i-th.  For b > 128 a tile takes its own diagonal
// chunk (the keys of its rows) first: those are the keys it pools, so they
// load at once and the block's summary does not wait on the softmax of the
// tile's earlier chunks (whose V loads follow the previous chunk's PV).
template <bool kSplit>
__device__ inline int in_order(const Tile& t, int i) {
  if constexpr (!kSplit) return i;
  return i == 0 ? t.nin - 1 : i - 1;
}

// Tile (sequence index) whose pooling publishes summary j.
template <bool kSplit>
__device__ inline int summary_tile(const Geometry& g, int j) {
  return kSplit ? j * g.tpb + g.tpb - 1 : (j * g.b) / g.R;
}

// Number of sub-tiles of block j (the last block of a sequence may be short).
__device__ inline int block_tiles(const Geometry& g, int j) {
  const int len = min(g.b, g.T - j * g.b);
  return (len + kTileRows - 1) / kTileRows;
}

// Summary chunk c (0-based) covers summaries [128c, e); the 16-row-rounded MMA
// width N16 is loaded from window start w = e - N16 so that every row the MMA
// reads is either an earlier, already-published summary or out of bounds
// (zero-filled by TMA), never an unpublished one.
struct SumChunk {
  int lo, e, n16, w;
};

__device__ inline SumChunk sum_chunk(const Tile& t, int c) {
  SumChunk k;
  k.lo = 128 * c;
  k.e = min(128 * (c + 1), t.ns);
  k.n16 = round16(k.e - k.lo);
  k.w = k.e - k.n16;
  return k;
}

// Byte offset of element (row, col) in a 128-row tile stored as 64-column
// atoms of 128-byte rows with the 128B swizzle (16-byte chunk ^= row % 8), the
// layout TMA writes for a box of (64, rows) with CU_TENSOR_MAP_SWIZZLE_128B.
__device__ __forceinline__ uint32_t swz_offset(int row, int col) {
  const int atom = col >> 6;
  const int chunk = (col >> 3) & 7;
  return atom * kAtomBytes + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

// UMMA descriptors over such tiles.
// K-major operand (rows = M or N, K along the 64-column atoms): k-step kk of
// 16 elements starts at atom kk/4, byte 32*(kk%4) of each row; SBO = 8 rows.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile_saddr, int kk) {
  return ptx::smem_desc_sw128(tile_saddr + (kk >> 2) * kAtomBytes + (kk & 3) * 32, 16, 1024);
}
// MN-major operand (rows = K, 64-column atoms along N): k-step kk covers rows
// 16kk..16kk+15; LBO = next 64-column atom, SBO = next 8 rows.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile_saddr, int kk) {
  return ptx::smem_desc_sw128(tile_saddr + kk * 16 * 128, kAtomBytes, 1024);
}

}  // namespace sm100
}  // namespace sqb
