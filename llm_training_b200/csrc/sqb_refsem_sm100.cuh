// Tensor-core (sm_100a) kernels of the reference-semantics mode: the local
// attention maps, block summaries and P = local V of every block, and the
// gradients of the local attention.
#pragma once

#include <initializer_list>

#include "sqb_internal.cuh"

namespace sqb {

// True when refsem_tc_local handles a problem: bf16 views the TMA maps accept,
// block length L in {16, 32, 64} (so that 128-row tiles hold whole blocks),
// D in {64, 128}, and an sm_100-class device.
bool refsem_tc_supported(int L, int D, int dtype, std::initializer_list<TensorView> views);

// Per block i of every (batch, head): summary (B*H, G, L) fp32 (skipped when
// null) and P (B*H, T, D) fp32, with T = G * L.  status: three zeroed words
// where a wait that gave up records SQB_ERR_TIMEOUT.
int refsem_tc_local(TensorView q, TensorView k, TensorView v, float* summary, float* P, int B,
                    int T, int H, int D, int L, float scale, uint32_t* status, cudaStream_t s);

// dQ, dK, dV of every block's local attention from dP (B*H, T, D) fp32 and
// d_summary (B*H, G, L) fp32, written through the bf16 (B, T, H, D) views.
int refsem_tc_grads(TensorView q, TensorView k, TensorView v, const float* dP,
                    const float* dsum, TensorView dq, TensorView dk, TensorView dv, int B, int T,
                    int H, int D, int L, float scale, uint32_t* status, cudaStream_t s);

}  // namespace sqb
