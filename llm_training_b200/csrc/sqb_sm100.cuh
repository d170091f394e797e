// sm_100a (B200) tensor-core kernels for sqrt-block attention: tcgen05.mma with
// TMEM accumulators, operands staged in shared memory by plain per-CTA TMA loads.
#pragma once

#include <cuda.h>

#include <initializer_list>

#include "sqb_internal.cuh"

namespace sqb {

// True when the tcgen05 kernels handle this problem and these tensor views
// (bf16, D in {64, 128}, block length a multiple of 16 in [32, 128], 16-byte
// aligned pointers and strides, sm_100-class device).
bool sm100_fwd_supported(const Problem& p, std::initializer_list<TensorView> views,
                         const float* lse, const void* kbar, const void* vbar);
bool sm100_bwd_supported(const Problem& p, std::initializer_list<TensorView> views,
                         const float* lse, const void* kbar, const void* vbar);

// Shared with the reference-semantics tensor-core kernels: an sm_100-class
// device (and its SM count), bf16 views the TMA maps accept (16-byte aligned,
// strides multiples of 8 elements), and a (B, T, H, D) bf16 view as a load map
// with box {64 columns, 1 head, rows, 1 batch} and the 128-byte swizzle.
bool sm100_device(int* num_sms);
bool sm100_views_ok(std::initializer_list<TensorView> views);
bool sm100_encode_rows(CUtensorMap* m, int B, int T, int H, int D, const TensorView& t,
                       int rows);

int sm100_forward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                  float* lse, void* kbar, void* vbar, uint8_t* ws, const WorkspaceLayout& wl,
                  cudaStream_t stream);

int sm100_backward(const Problem& p, TensorView q, TensorView k, TensorView v, TensorView o,
                   TensorView dout, const float* lse, const void* kbar, const void* vbar,
                   TensorView dq, TensorView dk, TensorView dv, uint8_t* ws,
                   const WorkspaceLayout& wl, cudaStream_t stream);

namespace sm100 {

// Rows per work tile: 128 when b divides 128 (whole blocks per tile), else b.
// Rows of a work tile's load box: 128 when b divides 128 or b > 128 (a block
// is then split into sub-tiles of up to 128 rows), else b.
inline int tile_rows(int b) { return (b > 128 || 128 % b == 0) ? 128 : b; }
// Rows of a store box: a sub-tile shorter than 128 rows (the last one of a
// block when b > 128) is stored 16 rows at a time, so no store writes rows of
// the next block's tile.
inline int store_rows(int b) { return b > 128 ? 16 : tile_rows(b); }
// Sub-tiles per block and work tiles per (batch, head).
inline int tiles_per_block(int b) { return b > 128 ? (b + 127) / 128 : 1; }
inline int tiles_per_seq(int T, int b) {
  if (b <= 128) return (T + tile_rows(b) - 1) / tile_rows(b);
  const int G = (T + b - 1) / b;
  return (G - 1) * tiles_per_block(b) + (T - (G - 1) * b + 127) / 128;
}

struct TensorMaps {
  CUtensorMap q, k, v, kbar, vbar;
  CUtensorMap o;  // store map: box of 32 columns x 16 rows, 64-byte swizzle
};

int launch_forward(const Problem& pr, const TensorMaps& tm, float* lse, void* kbar, void* vbar,
                   uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream);

struct BwdTensorMaps {
  CUtensorMap q, k, v, o, dout, dq, dk, dv, kbar, vbar;
};

int launch_backward(const Problem& pr, const BwdTensorMaps& tm, const float* lse, TensorView o,
                    uint8_t* ws, const WorkspaceLayout& wl, int num_sms, cudaStream_t stream);

}  // namespace sm100
}  // namespace sqb
