/*
 * sqb_train.h - helpers of the GPT training caller (not part of the attention
 * operator's drop-in boundary, which is sqrtblock.h).
 *
 * Token cross-entropy over a (N, V) block of logits, fused: the forward reads
 * each row once (fp32 max / sum-of-exp), the backward writes each row's
 * gradient once in the logits' dtype.  It computes what the reference's
 * calculate_loss (training_utils.py:8-17: F.cross_entropy over the flattened
 * logits under bf16 autocast, fp32 softmax math) computes, per token; the mean
 * over the non-ignored tokens is taken by the caller.  And a LayerNorm (last
 * entry points) with one warp per row and a fixed-order weight gradient.
 *
 * Conventions as in sqrtblock.h: caller-owned device pointers, asynchronous on
 * `stream` (a cudaStream_t; NULL = legacy default stream), return SQB_OK or an
 * SQB_ERR_* code.  logits / dlogits are (N, ld) row-major with ld >= V,
 * dtype SQB_BF16 or SQB_F32; columns [V, ld) of logits are not read.  A column
 * holding -inf takes no probability and gets a zero gradient.
 */
#ifndef SQB_TRAIN_H_
#define SQB_TRAIN_H_

#include <stddef.h>
#include <stdint.h>

#include "sqrtblock.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Forward, per row r: lse[r] = log sum_{c < V} exp(logits[r, c]) and
 * loss[r] = lse[r] - logits[r, targets[r]]; a row with targets[r] < 0 is
 * ignored (loss[r] = 0).  targets are int64 in [0, V) or negative.  loss and
 * lse are fp32 arrays of N. */
int sqb_xent_fwd(const void* logits, const int64_t* targets, float* loss, float* lse, int64_t N,
                 int64_t V, int64_t ld, int dtype, void* stream);

/* Backward: dlogits[r, c] = (exp(logits[r, c] - lse[r]) - [c == targets[r]]) * scale[0]
 * for c < V and 0 for V <= c < ld; an ignored row is all zero.  `scale` points
 * to one fp32 on the device (d loss / d loss[r]: the upstream gradient over
 * the number of counted tokens), read there so the host never waits. */
int sqb_xent_bwd(const void* logits, const int64_t* targets, const float* lse, const float* scale,
                 void* dlogits, int64_t N, int64_t V, int64_t ld, int dtype, void* stream);

/* LayerNorm over the last dimension of N contiguous fp32 rows of C (C a
 * multiple of 128, at most 1024; else SQB_ERR_UNSUPPORTED):
 *   y = (x - mean) / sqrt(var + eps) * weight + bias   (var biased; bias may be NULL),
 * as torch.nn.LayerNorm computes it (the reference's LayerNorm module,
 * model/layer_norm.py:4-13).  y has y_dtype: fp32, or bf16 - what a bf16
 * autocast consumer of an fp32 LayerNorm would cast it to.  mean and rstd
 * (1 / sqrt(var + eps)) are fp32 arrays of N for the backward.  x, weight,
 * bias and y 16-byte aligned (else SQB_ERR_ALIGN). */
int sqb_layernorm_fwd(const float* x, const float* weight, const float* bias, void* y, int y_dtype,
                      float* mean, float* rstd, int64_t N, int64_t C, float eps, void* stream);

/* Scratch bytes sqb_layernorm_bwd needs for N rows of C. */
size_t sqb_layernorm_workspace_bytes(int64_t N, int64_t C);

/* Backward: dx (fp32, N x C) from dy (dy_dtype) and the forward's x, mean and
 * rstd; dweight and, unless dbias is NULL, dbias (fp32, C) are overwritten with
 * their column sums, added in a fixed order (bit-reproducible). */
int sqb_layernorm_bwd(const void* dy, int dy_dtype, const float* x, const float* weight,
                      const float* mean, const float* rstd, float* dx, float* dweight,
                      float* dbias, void* workspace, size_t ws_bytes, int64_t N, int64_t C,
                      void* stream);

/* Residual add fused into the LayerNorm that reads its sum (the GPT caller's
 * x = x + block(...) followed by the next LayerNorm):
 *   x_out = x + h   (h: fp32 or bf16 rows by h_dtype, e.g. a bf16 autocast
 *                    Linear's output; the sum in fp32 as torch adds them),
 *   y     = LayerNorm(x_out) as sqb_layernorm_fwd, mean and rstd of x_out.
 * x_out and h 16-byte aligned like the other rows. */
int sqb_add_layernorm_fwd(const float* x, const void* h, int h_dtype, float* x_out,
                          const float* weight, const float* bias, void* y, int y_dtype,
                          float* mean, float* rstd, int64_t N, int64_t C, float eps,
                          void* stream);

/* Its backward: dx = (LayerNorm's input gradient from dy) + dres, where dres
 * (fp32, N x C, may be NULL) is the gradient reaching x_out from its other
 * uses; dx is the gradient of both x and h, written as fp32 and, unless dh_bf16
 * is NULL, also as bf16 (for a bf16 h).  dweight / dbias and the workspace as
 * sqb_layernorm_bwd (x_out is the LayerNorm's input). */
int sqb_add_layernorm_bwd(const void* dy, int dy_dtype, const float* x_out, const float* weight,
                          const float* mean, const float* rstd, const float* dres, float* dx,
                          void* dh_bf16, float* dweight, float* dbias, void* workspace,
                          size_t ws_bytes, int64_t N, int64_t C, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SQB_TRAIN_H_ */
