/*
 * sqb_train.h - helpers of the GPT training caller (not part of the attention
 * operator's drop-in boundary, which is sqrtblock.h).
 *
 * Token cross-entropy over a (N, V) block of logits, fused: the forward reads
 * each row once (fp32 max / sum-of-exp), the backward writes each row's
 * gradient once in the logits' dtype.  It computes what the reference's
 * calculate_loss (training_utils.py:8-17: F.cross_entropy over the flattened
 * logits under bf16 autocast, fp32 softmax math) computes, per token; the mean
 * over the non-ignored tokens is taken by the caller.
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

#ifdef __cplusplus
}
#endif

#endif /* SQB_TRAIN_H_ */
