/*
 * nimbleml_tied_ce.h — C ABI of the B200 fused tied LM-head cross-entropy.
 *
 * Plain pointers and sizes only: every pointer argument is a device address on
 * the current CUDA device unless stated otherwise, `stream` is a cudaStream_t
 * passed as void* (NULL = legacy default stream), and every entry point
 * returns 0 on success or a negative NIMBLE_ERR_* code. The message for the
 * last failure on the calling thread is available from
 * nimble_tied_ce_last_error().
 *
 * Ownership: the caller allocates every output and the workspace; no entry
 * point allocates or frees device memory. Inputs are read-only and must be
 * C-contiguous row-major. Launches are asynchronous on `stream`; nothing
 * synchronises the device.
 *
 * Layout of the path (N tokens, d hidden, V vocabulary, P vocab shards):
 *   hidden  (N, d)        compute dtype
 *   weights (V_local, d)  compute dtype, rows [v_offset, v_offset + V_local)
 *                         of the tied embedding matrix E
 *   labels  (N,)          int64 global class ids, or ignore_index
 *
 * Reference interface this library replaces (NimbleML, Python/NumPy/CuPy):
 *   NimbleML/kernels/fused_tied_crossentropy.py:8-24   forward  (h @ E^T, CE)
 *   NimbleML/kernels/fused_tied_crossentropy.py:27-48  backward (G @ E, G^T @ h)
 *   NimbleML/kernels/fused_crossentropy.py:14-30       row max / sum-exp / lse
 *   NimbleML/kernels/fused_crossentropy.py:33-50       softmax - onehot
 *   NimbleML/losses/_ce_prepare.py:46-69               ignore_index filtering
 * The reference's pybind11 device-pointer entry points follow the same
 * convention of raw addresses plus sizes (native/src/module.cpp:231-284).
 */
#ifndef NIMBLEML_TIED_CE_H
#define NIMBLEML_TIED_CE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NIMBLE_API __attribute__((visibility("default")))
#else
#define NIMBLE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of hidden / weights (the compute dtype) and of outputs. */
enum {
  NIMBLE_DTYPE_F32 = 0,  /* fp32 storage, tcgen05 kind::tf32 with RN rounding */
  NIMBLE_DTYPE_F16 = 1,  /* fp16, tcgen05 kind::f16, fp32 accumulate        */
  NIMBLE_DTYPE_BF16 = 2, /* bf16, tcgen05 kind::f16, fp32 accumulate        */
  /* fp32 storage whose values are already TF32 (rounded by nimble_round_tf32).
   * Accepted as the compute dtype of the tied-CE forward / backward only:
   * they then read hidden / weights in place instead of making rounded
   * copies, so a caller rounds once per forward + backward pair. */
  NIMBLE_DTYPE_TF32 = 3
};

/* Return codes. Device-side conditions are reported through `status`. */
enum {
  NIMBLE_OK = 0,
  NIMBLE_ERR_INVALID_ARG = -1,  /* bad shape, dtype, alignment or null pointer */
  NIMBLE_ERR_WORKSPACE = -2,    /* workspace smaller than the size query      */
  NIMBLE_ERR_CUDA = -3,         /* a CUDA runtime / driver call failed          */
  NIMBLE_ERR_UNSUPPORTED = -4   /* no sm_100 device or no driver entry point    */
};

/* Bits OR-ed into the device status word by the kernels. */
enum {
  NIMBLE_STATUS_BAD_LABEL = 1,     /* a label outside [0, V) that is not ignore_index */
  NIMBLE_STATUS_WAIT_TIMEOUT = 2   /* a bounded device wait gave up (kernel aborted)  */
};

/* nimble_tied_ce_backward for vocab-sharded ranks that overlap the grad_hidden
 * reduction with compute (no counterpart in the reference, which has no
 * multi-GPU path). Same arguments and results, plus: the last slab computes
 * grad_hidden before its grad_weights rows and records
 * grad_hidden_ready_event (a cudaEvent_t) on `stream` right after it; the
 * first capped_fraction of that slab's grad_weights rows (rounded up to
 * 256-row tiles; >= 1: all of them) then run on at most last_de_max_ctas SMs
 * (0 = all), leaving SMs for a collective the caller enqueues on another
 * stream after waiting on the event, and the remaining rows run on all SMs.
 * Slabs follow the slab_bytes budget alone (the shard is at most half of a
 * split vocabulary): size the workspace with
 * nimble_tied_ce_backward_overlap_workspace_size. */
NIMBLE_API int nimble_tied_ce_backward_overlap(const float* grad_scale, const void* hidden,
                                               const void* weights, const int64_t* labels,
                                               const float* lse, const float* valid_count,
                                               int64_t n_tokens, int64_t d_model, int64_t v_local,
                                               int64_t v_offset, int64_t ignore_index, int dtype,
                                               void* grad_hidden, int grad_hidden_dtype,
                                               void* grad_weights, int grad_weights_dtype,
                                               int accumulate_grad_weights, size_t slab_bytes,
                                               void* workspace, size_t workspace_bytes, int* status,
                                               void* stream, void* grad_hidden_ready_event,
                                               int last_de_max_ctas, float capped_fraction);

/* 1 when a compute-capability 10.x device is visible, else 0. Mirrors the
 * reference's availability flags (native/src/module.cpp:13-17,221-227). */
NIMBLE_API int nimble_tied_ce_available(void);

/* Message of the last failing call on this thread ("" if none). */
NIMBLE_API const char* nimble_tied_ce_last_error(void);

/* Bytes of workspace nimble_tied_ce_forward needs for these sizes. */
NIMBLE_API int nimble_tied_ce_forward_workspace_size(int64_t n_tokens, int64_t d_model, int64_t v_local,
                                          int dtype, size_t* bytes);

/* Forward on one vocab shard (P = 1: the whole vocabulary, v_offset = 0).
 * Replaces the logits GEMM + row statistics of
 * NimbleML/kernels/fused_tied_crossentropy.py:8-24 and
 * NimbleML/kernels/fused_crossentropy.py:14-30, without an N x V buffer.
 * Writes per token, over this shard's columns only:
 *   shard_max[i]    = max_j  s_ij            (s = h . E^T, fp32 accumulate)
 *   shard_sumexp[i] = sum_j exp(s_ij - shard_max[i])
 *   shard_target[i] = s_i,label  if label lies in this shard, else 0
 * Rows whose label equals ignore_index still get max / sumexp. */
NIMBLE_API int nimble_tied_ce_forward(const void* hidden, const void* weights, const int64_t* labels,
                           int64_t n_tokens, int64_t d_model, int64_t v_local, int64_t v_offset,
                           int dtype, float* shard_max, float* shard_sumexp, float* shard_target,
                           void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Merges n_shards shard statistics (each array laid out [n_shards][n_tokens])
 * into the global per-token statistics and the mean loss over valid rows —
 * the lse / gather / mean of NimbleML/kernels/fused_crossentropy.py:23-29
 * with the valid-row mean of NimbleML/losses/cross_entropy.py:124-148.
 *   out_max[i], out_sumexp[i]: global row max and sum-exp (fp32)
 *   out_lse[i]  = out_max[i] + log(out_sumexp[i])
 *   out_loss[0] = sum_{valid i} (lse_i - s_i,label) / n_valid   (0 if none)
 *   out_valid_count[0] = n_valid as float
 * The loss sum is a fixed-order reduction: identical inputs give identical
 * bits on every rank. Labels outside [0, vocab_size) that are not
 * ignore_index set NIMBLE_STATUS_BAD_LABEL in *status and count as ignored. */
NIMBLE_API int nimble_tied_ce_combine(const float* shard_max, const float* shard_sumexp,
                           const float* shard_target, int n_shards, const int64_t* labels,
                           int64_t n_tokens, int64_t vocab_size, int64_t ignore_index,
                           float* out_max, float* out_sumexp, float* out_lse, float* out_loss,
                           float* out_valid_count, int* status, void* stream);

/* Bytes of workspace nimble_tied_ce_backward needs. `slab_bytes` bounds the
 * per-slab gradient tiles (0 = library default, 2 GiB); the backward walks
 * the shard in vocab slabs whose G buffers fit that budget, and in at least
 * two slabs, so no buffer holds more than half of the shard's logits. */
NIMBLE_API int nimble_tied_ce_backward_workspace_size(int64_t n_tokens, int64_t d_model, int64_t v_local,
                                           int dtype, size_t slab_bytes, size_t* bytes);

/* Backward on one vocab shard. Replaces
 * NimbleML/kernels/fused_tied_crossentropy.py:27-48 and
 * NimbleML/kernels/fused_crossentropy.py:33-50: recomputes the logits of
 * this shard, forms G = (softmax - onehot) * grad_scale / n_valid with the
 * global lse, and computes
 *   grad_hidden  (N, d)        = G . E_shard   (this shard's partial sum)
 *   grad_weights (V_local, d)  = G^T . h       (complete for the shard)
 * grad_scale and valid_count are DEVICE fp32 scalars (no host sync).
 * Rows with label == ignore_index get G = 0, hence an exactly-zero
 * grad_hidden row (NimbleML/losses/cross_entropy.py:181-184).
 * grad_*_dtype selects the output element type (NIMBLE_DTYPE_*); with
 * accumulate_grad_weights != 0 the result is added to grad_weights
 * (NimbleML/utils/tensor.py:334-350 accumulation of the tied grad). */
NIMBLE_API int nimble_tied_ce_backward(const float* grad_scale, const void* hidden, const void* weights,
                            const int64_t* labels, const float* lse, const float* valid_count,
                            int64_t n_tokens, int64_t d_model, int64_t v_local, int64_t v_offset,
                            int64_t ignore_index, int dtype, void* grad_hidden,
                            int grad_hidden_dtype, void* grad_weights, int grad_weights_dtype,
                            int accumulate_grad_weights, size_t slab_bytes, void* workspace,
                            size_t workspace_bytes, int* status, void* stream);

/* Bytes of workspace nimble_tied_ce_backward_overlap needs. That entry point
 * serves a shard of a vocabulary split over P >= 2 ranks (at most half of
 * the vocabulary), so its slabs follow the slab_bytes budget alone: a shard
 * whose G fits the budget is walked in one slab, with no fp32 grad_hidden
 * accumulator. No counterpart in the reference (no multi-GPU path). */
NIMBLE_API int nimble_tied_ce_backward_overlap_workspace_size(int64_t n_tokens, int64_t d_model,
                                                              int64_t v_local, int dtype,
                                                              size_t slab_bytes, size_t* bytes);

/* dst[i] = src[i] rounded to the nearest TF32 value (ties away from zero,
 * cvt.rna.tf32.f32), in fp32 storage. A caller that passes the rounded
 * copies of hidden and weights with dtype NIMBLE_DTYPE_TF32 to the tied-CE
 * forward and backward rounds once per pair instead of once per call. Plays
 * the part of the reference's fp32 on_device copy
 * (NimbleML/utils/np_backend.py:184-190) for the TF32 tensor cores. */
NIMBLE_API int nimble_round_tf32(const float* src, float* dst, int64_t n, void* stream);

/* Diagnostic for the failure path (no counterpart in the reference, which has
 * no device-side waits): launches one block whose bounded mbarrier wait —
 * the same wait every pipeline stage of the GEMMs uses — has nothing to wait
 * for. After limit_ns (at most 2 s) it gives up, ORs
 * NIMBLE_STATUS_WAIT_TIMEOUT into *status and returns; no fault, no hang. */
NIMBLE_API int nimble_tied_ce_probe_wait_timeout(uint64_t limit_ns, int* status, void* stream);

/* Materialised tied-head logits for evaluation / generation:
 *   logits[i, :] = hidden_row_i . E^T   (fp32 accumulate, f16 / bf16 inputs)
 * where hidden_row_i starts hidden_row_pitch elements after row i-1, so
 * passing (base + (S-1)*d, pitch S*d, n_rows = B) gives the last-position
 * logits of each of B sequences of length S without a gather copy.
 * Row i of logits starts logits_row_pitch elements after row i-1 (pitch x
 * element size a multiple of 16 bytes; pad odd vocabularies). Only f16 / bf16
 * compute. Replaces the GEMM of GPT._tied_logits
 * (NimbleML/models/gpt.py:139-181) used by GPT.forward and generate
 * (NimbleML/models/generate.py:62-119). */
NIMBLE_API int nimble_tied_logits_forward(const void* hidden, int64_t hidden_row_pitch,
                                          const void* weights, int64_t n_rows, int64_t d_model,
                                          int64_t vocab, int dtype, void* logits,
                                          int64_t logits_row_pitch, int logits_dtype, void* stream);

/* Backward of the tied-head logits (NimbleML/models/gpt.py:165-178):
 *   grad_hidden  = grad_logits . E          (skipped if grad_hidden is NULL)
 *   grad_weights = grad_logits^T . hidden   (added to grad_weights when
 *                                            accumulate_grad_weights != 0;
 *                                            skipped if NULL)
 * grad_logits (n_rows x vocab, rows grad_logits_row_pitch elements apart,
 * pitch x element size a multiple of 16 bytes) and hidden (n_rows x d,
 * contiguous) are in the compute dtype. */
NIMBLE_API int nimble_tied_logits_backward(const void* grad_logits, int64_t grad_logits_row_pitch,
                                           const void* hidden,
                                           const void* weights, int64_t n_rows, int64_t d_model,
                                           int64_t vocab, int dtype, void* grad_hidden,
                                           int grad_hidden_dtype, void* grad_weights,
                                           int grad_weights_dtype, int accumulate_grad_weights,
                                           void* stream);

/* ---------------------------------------------------------------------------
 * Row kernels around the head (HBM-bound, one read / write per element).
 * ------------------------------------------------------------------------- */

/* Cross-entropy over logits that already exist: the untied
 * CrossEntropyLoss.forward (NimbleML/losses/cross_entropy.py:31-107) with
 * fused_crossentropy_forward (NimbleML/kernels/fused_crossentropy.py:14-30).
 * logits: n_rows x n_classes, rows row_pitch elements apart. Writes the row
 * max, sum-exp and label logit (n_rows each), then lse, the mean loss over
 * rows whose label != ignore_index, and that row count, exactly as
 * nimble_tied_ce_combine does for one shard. */
NIMBLE_API int nimble_ce_logits_forward(const void* logits, int64_t row_pitch, const int64_t* labels,
                                        int64_t n_rows, int64_t n_classes, int dtype,
                                        int64_t ignore_index, float* out_max, float* out_sumexp,
                                        float* out_target, float* out_lse, float* out_loss,
                                        float* out_valid_count, int* status, void* stream);

/* grad_logits = (softmax - onehot) * grad_scale / n_valid, ignored rows zero
 * (NimbleML/kernels/fused_crossentropy.py:33-50 and the row scatter of
 * NimbleML/losses/_ce_prepare.py:72-78). grad_scale / valid_count are device
 * scalars; lse comes from nimble_ce_logits_forward. */
NIMBLE_API int nimble_ce_logits_backward(const float* grad_scale, const float* valid_count,
                                         const void* logits, int64_t row_pitch, const int64_t* labels,
                                         const float* lse, int64_t n_rows, int64_t n_classes, int dtype,
                                         int64_t ignore_index, void* grad_logits,
                                         int64_t grad_row_pitch, void* stream);

/* Sampled softmax cross-entropy (NimbleML/kernels/sampled_softmax.py:66-98,
 * NimbleML/losses/sampled_cross_entropy.py:21-119): softmax over the
 * n_candidates classes of each row, candidates[i, 0] being the true class;
 * rows whose label equals ignore_index are left out of the mean. */
NIMBLE_API int nimble_sampled_ce_forward(const void* logits, int64_t row_pitch, const int64_t* candidates,
                                         const int64_t* labels, int64_t n_rows, int64_t n_classes,
                                         int64_t n_candidates, int dtype, int64_t ignore_index,
                                         float* out_max, float* out_sumexp, float* out_target,
                                         float* out_lse, float* out_loss, float* out_valid_count,
                                         int* status, void* stream);

/* Gradient of the sampled loss w.r.t. the full logits: zero everywhere except
 * the candidate columns, where repeated candidates add up in order. */
NIMBLE_API int nimble_sampled_ce_backward(const float* grad_scale, const float* valid_count,
                                          const void* logits, int64_t row_pitch,
                                          const int64_t* candidates, const int64_t* labels,
                                          const float* lse, int64_t n_rows, int64_t n_classes,
                                          int64_t n_candidates, int dtype, int64_t ignore_index,
                                          void* grad_logits, int64_t grad_row_pitch, void* stream);

/* RMSNorm over the last dimension (d_model <= 8192), the norm that produces
 * the head's input: y = x / sqrt(mean(x^2) + eps) * gamma, with per-row
 * mean(x^2) and rms saved for backward (NimbleML/layers/rms_norm.py:25-90,
 * NimbleML/kernels/fused_rmsnorm.py:130-158). fp32 statistics. */
NIMBLE_API int nimble_rmsnorm_forward(const void* x, const void* gamma, int64_t n_rows, int64_t d_model,
                                      float eps, int dtype, void* y, float* out_ms, float* out_rms,
                                      void* stream);

/* Bytes of workspace nimble_rmsnorm_backward needs (per-block grad_gamma
 * partial sums, reduced in a fixed order so the result is deterministic). */
NIMBLE_API int nimble_rmsnorm_backward_workspace_size(int64_t n_rows, int64_t d_model, size_t* bytes);

/* RMSNorm backward (NimbleML/kernels/fused_rmsnorm.py:161-217): grad_x in the
 * compute dtype and grad_gamma in fp32 (added to grad_gamma when
 * accumulate_grad_gamma != 0). grad_dtype is the compute dtype or
 * NIMBLE_DTYPE_F32: the final norm before the tied head reads the head's
 * fp32 grad_hidden directly, with no 16-bit copy in between. */
NIMBLE_API int nimble_rmsnorm_backward(const void* grad, const void* x, const void* gamma, const float* ms,
                                       const float* rms, int64_t n_rows, int64_t d_model, float eps,
                                       int dtype, int grad_dtype, void* grad_x, float* grad_gamma,
                                       int accumulate_grad_gamma, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* Bytes of workspace nimble_embedding_scatter_add needs for n_rows ids and
 * a shard of vocab_rows rows (keys and row indices of a device radix sort
 * and its temporary storage). Queries the CUDA device. */
NIMBLE_API int nimble_embedding_scatter_add_workspace_size(int64_t n_rows, int64_t vocab_rows, size_t* bytes);

/* grad_weights[ids[i] - vocab_offset, :] += grad_out[i, :] into the fp32
 * (vocab_rows x d) grad of the tied matrix's rows [vocab_offset,
 * vocab_offset + vocab_rows) — the input embedding's share of the tied grad
 * (NimbleML/kernels/embedding_scatter.py:39-81, NimbleML/layers/embedding.py:138-148).
 * Deterministic: the rows of each id are added in ascending row order onto
 * the existing grad row, the loop order of the reference's CPU scatter
 * (native/src/scatter.cpp:6-15). Ids of other shards are skipped; ids
 * outside [0, vocab_size) are skipped and set NIMBLE_STATUS_BAD_LABEL. */
NIMBLE_API int nimble_embedding_scatter_add(float* grad_weights, const int64_t* ids, const void* grad_out,
                                            int64_t n_rows, int64_t vocab_offset, int64_t vocab_rows,
                                            int64_t vocab_size, int64_t d_model, int grad_out_dtype,
                                            void* workspace, size_t workspace_bytes, int* status,
                                            void* stream);

/* One AdamW step over n fp32 master weights (NimbleML/optimizers/adam.py:20-43,
 * the fused update used for each parameter, e.g. a vocab shard of E):
 *   m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
 *   w = w (1 - lr wd) - lr (m / bc1) / (sqrt(v / bc2) + eps)
 * optionally also writing w to weights_copy in weights_copy_dtype. */
NIMBLE_API int nimble_adamw_step(float* weights, const void* grad, int grad_dtype, float* exp_avg,
                                 float* exp_avg_sq, int64_t n, float lr, float beta1, float beta2,
                                 float bias_correction1, float bias_correction2, float eps,
                                 float weight_decay, void* weights_copy, int weights_copy_dtype,
                                 void* stream);

/* Allocation-free variant of nimble_tied_ce_forward; no counterpart in the
 * reference. For callers that cannot allocate device memory (a runtime whose
 * GPU memory belongs to another framework's pool, or a binding that may only
 * pass tensors it already holds): the per-tile scratch lives in a fixed
 * 64 MiB array inside this library, resident on every GPU that loads it until
 * the process exits. Sizes whose forward workspace
 * (nimble_tied_ce_forward_workspace_size) exceeds 64 MiB are rejected with
 * NIMBLE_ERR_INVALID_ARG. Calls no cudaMalloc / cudaFree. Every call looks
 * up the array's device address on the current device (cudaGetSymbolAddress,
 * no allocation), so the address stays valid after cudaDeviceReset; the
 * first call on a device may load the module there, so make it before any
 * stream capture. All calls share the one array: calls that overlap on the
 * GPU (different streams, or different host threads on one device) race and
 * must be serialised by the caller. Results equal nimble_tied_ce_forward's. */
NIMBLE_API int nimble_tied_ce_forward_noalloc(const void* hidden, const void* weights,
                                              const int64_t* labels, int64_t n_tokens,
                                              int64_t d_model, int64_t v_local, int64_t v_offset,
                                              int dtype, float* shard_max, float* shard_sumexp,
                                              float* shard_target, int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NIMBLEML_TIED_CE_H */
