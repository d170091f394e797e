/*
 * sqrtblock.h - C ABI of the B200 (sm_100a) two-level sqrt-block attention.
 *
 * Operator, per (batch n, head h), T tokens, head dim D, block length b:
 *   G = ceil(T/b) blocks, Gc = floor(T/b) complete blocks;
 *   Kbar_j = mean of K over block j, Vbar_j likewise (j < Gc);
 *   query t in block i = t/b attends, in ONE softmax with the given scale, to
 *   the keys i*b <= k <= t of its own block and to Kbar_j for every j < i;
 *   O_t = sum_k p_tk V_k + sum_j p_tj Vbar_j.
 *
 * Boundary.  In the reference (aorko01/LLM_training) the attention core runs
 * inside the BaseAttention plugin's forward (model/custom_attention.py:175-230:
 * blocked view :188-191, in-block causal softmax :195-198, summaries and the
 * G x G global softmax :200-213, _ScaledBlockCombine :82-135), and the
 * experimental Triton path runs it as _LocalCausalAttentionFn.forward/backward
 * (Experiment/flash_attention_integrated.py:219-291) plus an SDPA cross pass
 * (:455-462).  sqb_fwd replaces the forward core (everything between the Q/K/V
 * projections and c_proj, :183-227), sqb_bwd its autograd backward.  The
 * Python plugin (llm_training_b200/model/sqrt_block_attention.py) keeps the
 * reference's module API and calls these entry points through ctypes.
 *
 * Conventions.
 *   - Q, K, V, O, dO, dQ, dK, dV are (B, T, H, D) views with unit stride on D
 *     and arbitrary (batch, token, head) strides given in ELEMENTS, so the
 *     (B, T, H*D) output of a Linear layer is consumed without a permute copy.
 *   - lse is (B, H, T) fp32, natural-log log-sum-exp of the scaled scores.
 *   - kbar, vbar are (B, H, Gc, D) contiguous, same dtype as Q.
 *   - All pointers are caller-owned device memory; the library allocates
 *     nothing.  Calls are asynchronous on `stream` (a cudaStream_t; NULL = the
 *     legacy default stream) and never synchronize the host.
 *   - Return value: SQB_OK, or an SQB_ERR_* code for a rejected argument or a
 *     failed launch.  Device-side failures (a bounded wait that gave up) are
 *     recorded in the workspace, read back (synchronizing) by sqb_read_status,
 *     and also posted, without any synchronization, to a host-mapped mailbox
 *     that sqb_attach_status registers with the workspace.
 *   - The workspace belongs to one problem shape (B, T, H, D, block): it
 *     must be zero-filled once before its first use and then passed
 *     unchanged to later calls with that shape (its regions are laid out per
 *     shape and the kernels leave them clean for the next call).  Calls
 *     sharing a workspace must be ordered on one stream.  After any
 *     device-side error, zero it again.
 */
#ifndef SQRTBLOCK_H_
#define SQRTBLOCK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum sqb_dtype { SQB_F32 = 0, SQB_BF16 = 1 };

/* Kernel family selection (the `impl` argument). */
enum sqb_impl {
  SQB_IMPL_AUTO = 0,    /* tcgen05/TMA kernels where supported, else SIMT */
  SQB_IMPL_SIMT = 1,    /* fp32-accumulating CUDA-core kernels, any D <= 256 */
  SQB_IMPL_TCGEN05 = 2  /* sm_100a tensor-core kernels; SQB_ERR_UNSUPPORTED if not */
};

enum sqb_status {
  SQB_OK = 0,
  SQB_ERR_ARG = 1,          /* null pointer, non-positive size, bad block length */
  SQB_ERR_DTYPE = 2,        /* unknown dtype */
  SQB_ERR_ALIGN = 3,        /* a pointer or stride breaks the 16-byte rule */
  SQB_ERR_UNSUPPORTED = 4,  /* shape/dtype not handled by the requested impl */
  SQB_ERR_WORKSPACE = 5,    /* workspace null or smaller than sqb_workspace_bytes */
  SQB_ERR_LAUNCH = 6,       /* a kernel launch failed */
  SQB_ERR_TIMEOUT = 7,      /* a device-side bounded wait gave up */
  SQB_ERR_CUDA = 8,         /* another CUDA runtime error */
  SQB_ERR_DEVICE = 9        /* device is not sm_100 class */
};

/* Library ABI version (major*100 + minor). */
int sqb_version(void);

/* Human-readable text for an sqb_status code (static storage). */
const char* sqb_strerror(int code);

/* Block geometry.  block_req <= 0 selects b = round_up(ceil(sqrt(T)), 16),
 * the ceil geometry of Experiment/improvement.py:10-14 (the reference's own
 * model/custom_attention.py:68-79 needs a perfect-square T). */
int sqb_geometry(int64_t T, int64_t block_req, int64_t* block, int64_t* n_blocks,
                 int64_t* n_complete);

/* Bytes of scratch workspace a (B, T, H, D, block) problem needs. */
size_t sqb_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D, int64_t block);

/* Forward.  strides: 12 int64 = (batch, token, head) for q, k, v, o.
 * Writes o, lse, kbar, vbar.  Replaces model/custom_attention.py:183-227. */
int sqb_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
            void* kbar, void* vbar, int64_t B, int64_t T, int64_t H, int64_t D,
            int64_t block, const int64_t* strides, int dtype, float scale, int impl,
            void* workspace, size_t workspace_bytes, void* stream);

/* Backward from the saved forward outputs.  strides: 24 int64 =
 * (batch, token, head) for q, k, v, o, dout, dq, dk, dv.  Writes dq, dk, dv
 * (overwritten, not accumulated).  Replaces the autograd backward of
 * model/custom_attention.py:195-225 (_ScaledBlockCombine.backward :111-135
 * and the softmax/matmul backward around it). */
int sqb_bwd(const void* q, const void* k, const void* v, const void* o,
            const void* dout, const float* lse, const void* kbar, const void* vbar,
            void* dq, void* dk, void* dv, int64_t B, int64_t T, int64_t H, int64_t D,
            int64_t block, const int64_t* strides, int dtype, float scale, int impl,
            void* workspace, size_t workspace_bytes, void* stream);

/* ---- Reference-semantics mode ---------------------------------------------
 * The attention core of the reference's registered sqrt_block / custom module
 * itself (model/custom_attention.py:138): T = G * L tokens with G = L = sqrt(T)
 * (block_geometry, custom_attention.py:68-79, T must be a perfect square);
 * local_i = causal softmax of Q_i K_i^T * scale inside block i (:195-198);
 * summary_i = column sums of local_i (:203); glob = softmax over strictly
 * earlier blocks of summary_i . summary_j / sqrt(L), row 0 zero (:209-213);
 * out_i = local_i V_i + sum_{j<i} glob[i, j] local_j V_j (_ScaledBlockCombine,
 * :82-135).  CUDA-core kernels, fp32 arithmetic for fp32 and bf16 inputs,
 * L <= 64 and D <= 128.  Layout conventions as above.  A T that is not a
 * perfect square returns SQB_ERR_ARG (the reference raises ValueError). */

/* Bytes of scratch workspace a (B, T, H, D) reference-semantics problem needs
 * (0 when unsupported).  Its contents need no initialisation. */
size_t sqb_refsem_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D);

/* Forward.  strides: 12 int64 = (batch, token, head) for q, k, v, o.  Writes o,
 * glob (B, H, G, G) fp32 and summary (B, H, G, L) fp32, both contiguous and
 * saved for the backward.  Replaces model/custom_attention.py:183-227. */
int sqb_refsem_fwd(const void* q, const void* k, const void* v, void* o, float* glob,
                   float* summary, int64_t B, int64_t T, int64_t H, int64_t D,
                   const int64_t* strides, int dtype, float scale, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Backward.  strides: 21 int64 = (batch, token, head) for q, k, v, dout, dq,
 * dk, dv.  Writes dq, dk, dv (overwritten).  Replaces the autograd backward of
 * model/custom_attention.py:195-225 (_ScaledBlockCombine.backward :111-135 and
 * the softmax / summary backward around it). */
int sqb_refsem_bwd(const void* q, const void* k, const void* v, const void* dout,
                   const float* glob, const float* summary, void* dq, void* dk, void* dv,
                   int64_t B, int64_t T, int64_t H, int64_t D, const int64_t* strides,
                   int dtype, float scale, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Backward without a caller-supplied workspace.  This entry point has no
 * counterpart in the reference.  It is for callers that cannot allocate device
 * memory where they run the backward (their memory is owned by another
 * component, or their footprint is fixed after start-up): the scratch lives in
 * one 8 MiB array the library holds on every GPU it is loaded on.  Arguments
 * are those of sqb_bwd without the workspace.  Problems whose
 * sqb_workspace_bytes exceeds 8 MiB return SQB_ERR_WORKSPACE.  The first call on
 * a device looks up the array's address; make it before any stream capture.
 * Each call clears the scratch it uses, except a recorded device-side failure,
 * which stays until sqb_read_status_noalloc reads and clears it; all calls on a
 * device share the scratch, so calls that overlap on the GPU race and must not
 * be issued.  Allocates nothing. */
int sqb_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                    const void* dout, const float* lse, const void* kbar, const void* vbar,
                    void* dq, void* dk, void* dv, int64_t B, int64_t T, int64_t H, int64_t D,
                    int64_t block, const int64_t* strides, int dtype, float scale, int impl,
                    void* stream);

/* Reads back (after synchronizing `stream`) the device-side status recorded
 * in the no-allocation scratch of the current device, as sqb_read_status does
 * for a workspace, and clears it.  sqb_bwd_noalloc keeps a recorded failure
 * across calls until this call clears it.  No counterpart in the reference. */
int sqb_read_status_noalloc(void* stream, int64_t* detail);

/* Synchronizes `stream`, returns the device-side status recorded in the
 * workspace (SQB_OK or SQB_ERR_TIMEOUT) and clears it.  `detail`, if not
 * NULL, receives the work tile index (or wait code) that reported the failure.
 * A recorded status stays until this call clears it; while it is set, the
 * kernels' waits on other work tiles give up at once, so the results of later
 * calls are wrong too: after a failure, zero the workspace again (and attach
 * the mailbox again).  The reference's kernels have no device-side waits. */
int sqb_read_status(void* workspace, void* stream, int64_t* detail);

/* Configures a zero-filled workspace before its first use (synchronizes
 * `stream`; the settings live in the workspace, so zeroing it clears them).
 * mailbox: NULL, or two uint32 words of page-locked host memory (cudaHostAlloc
 *   / cudaMallocHost, 8-byte aligned) that the device can write; when a launch
 *   on this workspace records a failure, its last CTA writes {status, detail}
 *   there (detail first).  The host polls mailbox[0] without synchronizing
 *   and, finding it non-zero, knows an earlier call's results are invalid.
 * wait_budget_us: budget of each kernel wait on another work tile's flag or
 *   counter, in microseconds (0 = the default of 2 s).  A shorter budget makes
 *   a lost flag surface sooner; every wait on a CTA's own pipeline keeps its
 *   own fixed budget.
 * Has no counterpart in the reference, whose trainer runs the attention as
 * eager PyTorch ops (model/custom_attention.py:175-230) with nothing to wait on. */
int sqb_attach_status(void* workspace, uint32_t* mailbox, uint32_t wait_budget_us,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SQRTBLOCK_H_ */
