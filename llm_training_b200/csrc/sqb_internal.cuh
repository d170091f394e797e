// Internal declarations shared by the sqrt-block attention kernels and the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sqrtblock.h"

namespace sqb {

// A (B, T, H, D) tensor view with unit stride on D; strides in elements.
struct TensorView {
  void* ptr;
  int64_t sb, st, sh;
};

struct Problem {
  int B, T, H, D;
  int b;      // block length
  int G;      // number of blocks, ceil(T / b)
  int Gc;     // number of complete blocks, floor(T / b)
  float scale;
  int dtype;  // sqb_dtype
};

// Workspace layout (byte offsets).  Control words first, then per-tile flags,
// then fp32 scratch.  Computed identically by every entry point.
struct WorkspaceLayout {
  size_t ctrl;        // uint32 control block (see Ctrl*)
  size_t flags_fwd;   // uint32[B*H*tiles_per_seq]
  size_t flags_bwd;   // uint32[B*H*tiles_per_seq]
  size_t delta;       // fp32[B*H*T]   rowsum(dO * O)
  size_t dkbar;       // fp32[B*H*Gc*D] summary-gradient accumulators
  size_t dvbar;       // fp32[B*H*Gc*D]
  // b > 128 only: fp32[B*H*G*(tpb-1)*128*D] each, the dK / dV contributions of a
  // block's later sub-tiles to the keys of its earlier sub-tiles (stored when a
  // block has two sub-tiles, accumulated and re-zeroed when it has more)
  size_t dkx, dvx;
  // b > 128 only: uint32[B*H*G] count of a block's sub-tiles that have read
  // its summary-gradient sums (the last one re-zeroes them)
  size_t readers;
  // b > 128 only: fp32[B*H*G*(tpb-1)*2*D], the forward's K and V column sums
  // of each sub-tile but the last of a block, which adds them to its own
  size_t pool_part;
  size_t total;
  int tiles_per_seq;  // upper bound on work tiles per (batch, head)
};

// Control-block word indices (uint32).
enum CtrlWord {
  kFwdEpoch = 0,
  kFwdTileCounter = 1,
  kFwdExitCounter = 2,
  kBwdEpoch = 8,
  kBwdTileCounter = 9,
  kBwdExitCounter = 10,
  kStatus = 16,        // 0 = ok, else sqb_status (kept until sqb_read_status clears it)
  kStatusDetail = 17,  // which wait set kStatus (a wait code, or the work tile's index)
  kStatusAbort = 18,   // a wait on a CTA's own pipeline gave up (cleared at launch end)
  kWaitBudgetUs = 19,  // budget of waits on other CTAs in microseconds (0 = 2 s)
  kMailboxLo = 20,     // host-mapped (status, detail) pair a failed launch posts to,
  kMailboxHi = 21,     //   low and high halves of its device address (0 = none)
  kCtrlWords = 64
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline int tiles_per_seq_bound(int T, int b) {
  // Work tiles never hold fewer than 16 rows except at a block's or the
  // sequence's end, so ceil(T/16) + G bounds every tiling used.
  int G = (T + b - 1) / b;
  return (T + 15) / 16 + G;
}

inline WorkspaceLayout workspace_layout(int64_t B, int64_t T, int64_t H, int64_t D, int64_t b) {
  WorkspaceLayout w{};
  const int64_t BH = B * H;
  const int64_t Gc = T / b;
  w.tiles_per_seq = tiles_per_seq_bound((int)T, (int)b);
  size_t off = 0;
  w.ctrl = off;
  off += kCtrlWords * 4;
  off = align_up(off, 256);
  w.flags_fwd = off;
  off += (size_t)BH * w.tiles_per_seq * 4;
  off = align_up(off, 256);
  w.flags_bwd = off;
  off += (size_t)BH * w.tiles_per_seq * 4;
  off = align_up(off, 256);
  w.delta = off;
  off += (size_t)BH * T * 4;
  off = align_up(off, 256);
  w.dkbar = off;
  off += (size_t)BH * Gc * D * 4;
  off = align_up(off, 256);
  w.dvbar = off;
  off += (size_t)BH * Gc * D * 4;
  const int64_t G = (T + b - 1) / b;
  const int64_t xrows = b > 128 ? ((b + 127) / 128 - 1) * 128 : 0;  // per block
  off = align_up(off, 256);
  w.dkx = off;
  off += (size_t)BH * G * xrows * D * 4;
  off = align_up(off, 256);
  w.dvx = off;
  off += (size_t)BH * G * xrows * D * 4;
  off = align_up(off, 256);
  w.readers = off;
  off += b > 128 ? (size_t)BH * G * 4 : 0;
  off = align_up(off, 256);
  w.pool_part = off;
  off += b > 128 ? (size_t)BH * G * ((b + 127) / 128 - 1) * 2 * D * 4 : 0;
  w.total = align_up(off, 256);
  return w;
}

// ---- SIMT kernels (sqb_simt.cu) -------------------------------------------
// fp32-accumulating CUDA-core implementation for any D <= 256 and dtype.
int simt_forward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                 float* lse, void* kbar, void* vbar, cudaStream_t stream);
int simt_backward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                  TensorView dout, const float* lse, const void* kbar, const void* vbar,
                  TensorView dq, TensorView dk, TensorView dv, uint8_t* ws,
                  const WorkspaceLayout& wl, cudaStream_t stream);

}  // namespace sqb
