/* SPDX-License-Identifier: MIT
 *
 * dbs_cuda_b200.h -- entry points this engine adds beside the reference ABI
 * (include/dbs_cuda.h). The reference has no counterpart for them; they are
 * additive and leave the 17 reference symbols untouched.
 */
#ifndef DBS_CUDA_B200_H
#define DBS_CUDA_B200_H

#include "dbs_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define DBS_CUDA_B200_ABI_VERSION 1

DBS_CUDA_EXPORT int dbs_cuda_b200_abi_version(void);

/* Token sequences of the final beams of a decode: int64 sequences [B, K, T],
 * entry (b, k, t) the token final beam k holds at step t, following parents
 * back from the last step; -1 for dead beams and for steps past the example's
 * step count (args->steps_per_example). One kernel; replaces the T-step loop
 * of torch gathers of beamgrad.backtrack (python/beamgrad/_torch.py:582-606 of
 * beamgrad 2.3.0), with the same result. tokens / parents are the decode's
 * [B, T, K] int32 outputs. */
DBS_CUDA_EXPORT int dbs_cuda_backtrack(const DBSCudaDecodeArgs* args, const int32_t* tokens, const int32_t* parents,
                                       int64_t* sequences, void* stream);

/* The dense input gradient of a decode in one pass, overwriting grad_inputs
 * [B, T, K, V] (element type grad_type: DBS_CUDA_DTYPE_F32 / F16 / BF16). Its
 * value is what beamgrad's autograd produces from dbs_cuda_backward_ex into a
 * zero-filled float32 buffer followed by a cast to grad_type
 * (python/beamgrad/_torch.py:270-289 of beamgrad 2.3.0: decode_backward(...)
 * .to(input_dtype); python/csrc/cuda_ops.cpp:455 zero-fills), bit for bit:
 * rows of log-probabilities get their slots' path gradients at the chosen
 * tokens and zeros elsewhere; rows decoded from logits (in->logits and
 * in->row_lse set) get g_v - softmax(x_v) * S where a path gradient reaches
 * them, zeros elsewhere; rows past an example's steps or beams are zero.
 * Arguments and errors as dbs_cuda_backward_ex, plus grad_type; workspace as
 * dbs_cuda_backward_workspace_size(args) (NULL: stream-ordered allocation).
 * Every element is written once: no caller zero-fill, no accumulation. */
DBS_CUDA_EXPORT int dbs_cuda_backward_dense(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                            void* grad_inputs, int grad_type, void* workspace, int64_t workspace_bytes,
                                            void* stream);

/* Selected-beam weights of a decode: for every step, softmax_selected over the K selected
 * beams' scores (python/beamgrad estimators' "selected" surrogate; the reference computes them
 * on the CPU only, src/decoder.cpp:344 and src/kernels_scalar.cpp:277-302): scores above -1e30
 * take part, w = exp(score / T - max) / sum in slot order, all zero for a step without a
 * finite score. scores / weights are [B, T, K] float32 (the decode's scores output); the
 * temperature must be finite and positive. Bit-identical to the reference. */
DBS_CUDA_EXPORT int dbs_cuda_selected_weights(const DBSCudaDecodeArgs* args, const float* scores, float temperature,
                                              float* weights, void* stream);

/* dbs_cuda_backward_dense plus the gradient that flows through the selected-beam weights:
 * each slot with a parent adds (w_k * (gw_k - dot(w, gw))) / temperature to its score
 * gradient before the other terms (src/decoder.cpp:599-604 of beamgrad 2.3.0, the
 * grad_selected_weights of dbs_backward / dbs_backward_dense in include/dbs.h:440-455).
 * selected_weights are dbs_cuda_selected_weights' output and grad_selected_weights their
 * gradient, both [B, T, K] float32. */
DBS_CUDA_EXPORT int dbs_cuda_backward_selected(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                               const float* selected_weights, const float* grad_selected_weights,
                                               float temperature, void* grad_inputs, int grad_type, void* workspace,
                                               int64_t workspace_bytes, void* stream);

/* One step of the token prefixes of a caller-driven search, on the device.
 * After dbs_cuda_decode_step* wrote step `step`'s [B, K] parents, tokens and
 * from_logprob, writes prefixes_out [B, K, prefix_stride] int32:
 *   entries j < step: prefixes_in[b, parents[b, k], j]; entry step: the
 *   token when from_logprob[b, k], else -1; the row is -1 for parent < 0
 *   (or >= K). Entries past `step` are left as they are.
 * This is beamgrad's per-step torch gather + cat + where of the sequences
 * (python/beamgrad/_search.py:450-455 of beamgrad 2.3.0) as one kernel, so the
 * prefixes the next step reads (DBSCudaBeamState.prefixes) never leave the
 * device. prefixes_in and prefixes_out must not overlap (ping-pong two
 * buffers); prefixes_in may be NULL at step 0. When any_live is set, the
 * kernel also stores 1 there if some beam of the state after the step
 * (raw_scores, finished: the DBSCudaBeamState arrays) has a finite raw score
 * and is not finished (python/beamgrad/_search.py:366-368); it never stores 0,
 * so the caller zeroes the byte beforehand. No host synchronisation. */
DBS_CUDA_EXPORT int dbs_cuda_advance_prefixes(int batch_size, int beam_size, int step, int prefix_stride,
                                              const int32_t* parents, const int32_t* tokens,
                                              const uint8_t* from_logprob, const int32_t* prefixes_in,
                                              int32_t* prefixes_out, const float* raw_scores, const uint8_t* finished,
                                              uint8_t* any_live, void* stream);

/* Self-test of the engine's failure detection, without a GPU fault. Every inter-CTA wait
 * of the decode kernels (a flag spin, an mbarrier wait) is bounded: past its limit it
 * records a timeout in the decode's error word and returns, and the host reports
 * DBS_CUDA_STATUS_LAUNCH_FAILED when synchronization is on. This runs the same two waits,
 * one on a flag nothing sets and one on an mbarrier nothing arrives at (no copy in flight),
 * with a limit of timeout_ns (1e5 .. 1e9); words is a device buffer of 4 int32 (0, 1: the
 * waits' results; 2: the error word; 3: the unset flag). It synchronizes the stream and
 * returns DBS_CUDA_STATUS_LAUNCH_FAILED when the error word holds the timeout (the expected
 * outcome), DBS_CUDA_STATUS_OK otherwise. The context stays usable. No counterpart in the
 * reference. */
DBS_CUDA_EXPORT int dbs_cuda_b200_wait_selftest(int64_t timeout_ns, int32_t* words, void* stream);

/* ------------------------------------------------------------------------
 * Relaxed pool (beamgrad 2.3.0 src/decoder.cpp:294-312 record_pool and the
 * pool terms of run_backward, :621-657; include/dbs.h:64-79, 337-349, 373-397;
 * the CPU library's relaxed_pool_multiplier). The reference computes the pool
 * only on the CPU; these run it on the GPU with identical results.
 *
 * dbs_cuda_relaxed_pool: after a decode, the P = pool_size (K <= P <= 1024) best candidates of
 * every step under the full candidate order (the first K of them are the
 * step's selected beams), written [B, T, P] in that order (fewer than P
 * candidates: parent/token -1, length 0, scores -inf, from_logprob 0; steps
 * past an example's length are empty), and, when relaxed_weights is set, each
 * step's relaxed top-K membership sigmoid((score - theta) / temperature) with
 * theta bisected so that the weights sum to K (src/kernels_scalar.cpp:304-366).
 * inputs / data_type / from_logits / args are the decode's; trace is its
 * output (parents, tokens, lengths, raw_scores and from_logprob are read);
 * row_lse its row logsumexp (needed from logits). Not supported (as by
 * beamgrad's relaxed_topk): n-gram blocking, a repetition penalty, per-example
 * beam sizes / EOS tokens / minimum lengths, extra EOS tokens.
 * ------------------------------------------------------------------------ */
#define DBS_CUDA_B200_MAX_POOL 1024

typedef struct DBSCudaPoolOutputs {
    int32_t* parents;         /* [B, T, P] */
    int32_t* tokens;          /* [B, T, P] */
    int32_t* lengths;         /* [B, T, P] */
    float* scores;            /* [B, T, P] length-penalised ranking scores */
    float* raw_scores;        /* [B, T, P] cumulative log-probabilities */
    uint8_t* from_logprob;    /* [B, T, P] */
    float* relaxed_weights;   /* [B, T, P] relaxed top-K membership, or NULL */
    void* reserved[4];        /* must be NULL */
} DBSCudaPoolOutputs;

DBS_CUDA_EXPORT int dbs_cuda_relaxed_pool(const void* inputs, int data_type, int from_logits,
                                          const DBSCudaDecodeArgs* args, const DBSCudaDecodeOutputs* trace,
                                          const float* row_lse, int pool_size, float soft_topk_temperature,
                                          float soft_topk_tolerance, int soft_topk_max_iters,
                                          const DBSCudaPoolOutputs* pool, void* stream);

/* The pool of a decode and the gradients of its outputs, for
 * dbs_cuda_backward_pool. grad_relaxed_weights needs relaxed_weights. */
typedef struct DBSCudaPoolGradients {
    int pool_size;                        /* P */
    int reserved0;                        /* must be 0 */
    const int32_t* parents;               /* [B, T, P] as dbs_cuda_relaxed_pool wrote them */
    const int32_t* tokens;
    const int32_t* lengths;
    const uint8_t* from_logprob;
    const float* relaxed_weights;         /* [B, T, P], with grad_relaxed_weights */
    const float* grad_relaxed_weights;    /* [B, T, P] or NULL */
    const float* grad_pool_scores;        /* [B, T, P] or NULL */
    const float* grad_pool_raw_scores;    /* [B, T, P] or NULL */
    float soft_topk_temperature;          /* the relaxed weights' temperature (> 0) */
    void* reserved[4];                    /* must be NULL */
} DBSCudaPoolGradients;

/* dbs_cuda_backward_ex plus the pool terms (src/decoder.cpp:621-657): per step the
 * selected beams' raw-score gradients, then each pool candidate's
 *   d = (relaxed term + grad_pool_scores) / penalty(length) + grad_pool_raw_scores,
 * with parents summing their selected children in slot order and then their pool
 * candidates in pool order; accumulated (+=) into the caller-zeroed float32
 * [B, T, K, V] grad_inputs. Log-probability inputs only (in->logits must be NULL). */
DBS_CUDA_EXPORT int dbs_cuda_backward_pool(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                           const DBSCudaPoolGradients* pool, float* grad_inputs, void* stream);

/* Bytes of the fixed device array behind dbs_cuda_decode_no_alloc (4 MiB). */
#define DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES (4 * 1024 * 1024)

/* dbs_cuda_decode_ex2 without a workspace and without allocating. No
 * counterpart in the reference: it is for callers that may not allocate device
 * memory while they run -- an inference runtime's plugin enqueue or a serving
 * loop with a fixed, preplanned memory budget, where a cudaMalloc (or a pool
 * growing) would break the budget or stall other streams -- and that have no
 * buffer of their own to pass as workspace. Inputs and outputs are the
 * caller's, as for dbs_cuda_decode_ex2, and the results are identical.
 *
 * The scratch is one device array of DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES that
 * every GPU which loads the library keeps until the process exits. A decode
 * whose dbs_cuda_decode_workspace_size(args) exceeds it is rejected with
 * DBS_CUDA_STATUS_INVALID_ARGUMENT before anything runs. The first call on a
 * device looks up the array's device address (with that device current) and
 * caches it; make that first call before any stream capture. Every call on a
 * device uses the same array, and each decode starts by resetting what it
 * reads: calls whose work overlaps on the GPU (other streams, other threads)
 * race on the array, so order them on one stream or otherwise serialize them.
 * The cached address belongs to the device's context at the first call: after
 * cudaDeviceReset on that device it is stale, so do not call this entry point
 * on that device again in the process. 4 MiB covers small and medium decodes
 * (the chained decode needs about 130 bytes per row of B x T x K); the
 * BASELINE C2 decode [64, 128, 8, 32000] needs 8.4 MB and is refused. */
DBS_CUDA_EXPORT int dbs_cuda_decode_no_alloc(const void* inputs, int data_type, int from_logits,
                                             const DBSCudaDecodeArgs* args, const DBSCudaSearchOptions* options,
                                             const DBSCudaDecodeOutputs* outputs, float* row_lse, void* stream);

/* ------------------------------------------------------------------------
 * Vocabulary-sharded decode (no counterpart in the reference, which decodes
 * a whole vocabulary on one device). One process per GPU, world_size ranks
 * (1, 2, 4 or 8); the decode has the semantics of dbs_cuda_decode_ex2 over
 * the full [B, T, K, V] input and gives identical outputs on every rank.
 *
 * Rank r holds the tokens v with (v mod 256) in [r * 256 / W, (r + 1) * 256 / W)
 * (W = world_size), in increasing v: its shard is [B, T, K, shard_vocab] with
 * shard entry i the token (i / L) * 256 + r * L + i mod L, L = 256 / W. A
 * vocabulary-parallel output projection produces this layout directly when its
 * weight rows are ordered the same way. Interleaving by lane keeps each of the
 * reference's 256 logsumexp lanes (src/kernels_scalar.cpp:48-66 of beamgrad
 * 2.3.0) whole on one rank, so the logsumexp is bit-identical.
 *
 * Stages, each asynchronous on `stream`, with the caller's collectives between
 * them (the same on every rank, in this order):
 *   dbs_cuda_vshard_scan      row maxima, NaN/+inf flags and row records
 *   caller:                   all-reduce MAX of buffers.row_max (from logits)
 *   dbs_cuda_vshard_lanes     this rank's logsumexp lane sums (from logits)
 *   caller:                   all-gather buffers.exchange into buffers.exchange_all
 *   dbs_cuda_vshard_merge     logsumexp and merged records of every row
 *   loop:
 *     dbs_cuda_vshard_select  the selections of every example from resume[b] on;
 *                             an example stops at a step whose rows need a rescan
 *     caller:                 read resume / stalled; done when resume[b] == steps
 *                             for every b; else list the stalled rows (b * K + k,
 *                             examples ascending, then k) in rescan_rows, their
 *                             positions in rescan_slot, and
 *     dbs_cuda_vshard_rescan  this rank's best K candidates of those rows
 *     caller:                 all-gather buffers.rescan into buffers.rescan_all
 * The caller passes the same call (inputs, arguments, buffers, outputs) to
 * every stage; only the rescan fields change between rounds.
 * ------------------------------------------------------------------------ */
#define DBS_CUDA_VSHARD_MAX_WORLD 8

typedef struct DBSCudaVocabShardPlan {
    int32_t world_size;
    int32_t rank;
    int32_t shard_vocab;    /* tokens held by this rank */
    int32_t lanes;          /* 256 / world_size */
    int32_t list_len;       /* entries of a merged row record */
    int32_t shard_list_len; /* entries of a row record per rank */
    int32_t row_words;      /* 64-bit words per row of the exchange buffer */
    int32_t reserved0;
    int64_t rows;           /* batch * steps * beam */
    int64_t workspace_bytes;
} DBSCudaVocabShardPlan;

typedef struct DBSCudaVocabShardBuffers {
    float* row_max;               /* [rows] */
    float* row_min;               /* [rows] */
    uint64_t* exchange;           /* [rows, row_words] */
    const uint64_t* exchange_all; /* [world_size, rows, row_words] */
    int32_t* resume;              /* [batch]: first step not yet selected, steps when done */
    uint32_t* stalled;            /* [batch, ceil(beam / 32)]: rows of step resume[b] to rescan */
    const int32_t* rescan_rows;   /* [n_rescan] */
    const int32_t* rescan_slot;   /* [batch * beam]: position in rescan_rows, or -1 */
    uint64_t* rescan;             /* [n_rescan, beam] */
    const uint64_t* rescan_all;   /* [world_size, n_rescan, beam] */
    int64_t n_rescan;
    void* workspace;              /* plan.workspace_bytes; kept by the caller for the whole decode */
    int64_t workspace_bytes;
} DBSCudaVocabShardBuffers;

typedef struct DBSCudaVocabShardCall {
    const void* shard_inputs;     /* [batch, steps, beam, shard_vocab] of data_type */
    int32_t data_type;
    int32_t from_logits;
    int32_t world_size;
    int32_t rank;
    int32_t shard_list_len;       /* 0: the default (half the merged record) */
    int32_t reserved0;
    const DBSCudaDecodeArgs* args;        /* vocab_size is the full vocabulary */
    const DBSCudaSearchOptions* options;  /* may be NULL */
    DBSCudaVocabShardBuffers buffers;
    DBSCudaDecodeOutputs outputs;         /* as dbs_cuda_decode_ex2; every rank writes all of them */
    float* row_lse;                       /* [B, T, K] or NULL */
} DBSCudaVocabShardCall;

DBS_CUDA_EXPORT int dbs_cuda_vshard_plan(const DBSCudaDecodeArgs* args, int from_logits, int world_size, int rank,
                                         int shard_list_len, DBSCudaVocabShardPlan* plan);
/* scan also resets the decode state and resume / stalled, and (with
 * per-example arrays) checks their ranges, waiting for the stream once. */
DBS_CUDA_EXPORT int dbs_cuda_vshard_scan(const DBSCudaVocabShardCall* call, void* stream);
DBS_CUDA_EXPORT int dbs_cuda_vshard_lanes(const DBSCudaVocabShardCall* call, void* stream);
DBS_CUDA_EXPORT int dbs_cuda_vshard_merge(const DBSCudaVocabShardCall* call, void* stream);
DBS_CUDA_EXPORT int dbs_cuda_vshard_select(const DBSCudaVocabShardCall* call, void* stream);
DBS_CUDA_EXPORT int dbs_cuda_vshard_rescan(const DBSCudaVocabShardCall* call, void* stream);

#ifdef __cplusplus
}
#endif

#endif
