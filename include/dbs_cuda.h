/* SPDX-License-Identifier: MIT
 *
 * dbs_cuda.h -- C ABI of the B200 beam-search engine (libdbs_cuda.so, SOVERSION 10).
 *
 * This header is the drop-in boundary for beamgrad's CUDA engine: every type,
 * constant and function below has the name, field order, field types and
 * meaning of the reference contract in beamgrad 2.3.0, include/dbs_cuda.h
 * (cited per item as "ref: include/dbs_cuda.h:<line>"), so a program or a
 * binding built against the reference header links against this library
 * unchanged. The implementation behind it is new: sm_100a kernels that stream
 * each live [K, V] candidate slab once (see beamgrad_b200/csrc).
 *
 * Conventions (ref: include/dbs_cuda.h:26-35):
 *   - every tensor argument is a device pointer to dense row-major memory;
 *   - inputs are [B, T, K, V]; per-step outputs [B, T, K]; per-beam outputs [B, K];
 *   - slots an example does not use (steps past its step count, beams past its
 *     beam size, or fewer candidates than beams) read token = parent = -1,
 *     length = 0, scores = -inf, from_logprob = 0;
 *   - work is queued on `stream` (a cudaStream_t; NULL = legacy default stream)
 *     and the call returns without waiting, except where a function says it
 *     synchronizes; launch errors come back as a status code;
 *   - DBS_CUDA_SYNC_CHECK=1 in the environment, or dbs_cuda_set_synchronization(1),
 *     makes every call wait for its stream so device faults surface at the call.
 */
#ifndef DBS_CUDA_H
#define DBS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define DBS_CUDA_EXPORT __attribute__((visibility("default")))
#else
#define DBS_CUDA_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (ref: include/dbs_cuda.h:60-64). */
#define DBS_CUDA_STATUS_OK 0
#define DBS_CUDA_STATUS_UNAVAILABLE 1      /* no CUDA device, or a build without CUDA */
#define DBS_CUDA_STATUS_INVALID_ARGUMENT 2
#define DBS_CUDA_STATUS_LAUNCH_FAILED 3
#define DBS_CUDA_STATUS_OUT_OF_MEMORY 4

/* Largest beam size (ref: include/dbs_cuda.h:67). */
#define DBS_CUDA_MAX_BEAM 1024

/* Problem description shared by every call (ref: include/dbs_cuda.h:69-87).
 * Layout: 10 ints/floats, then 5 pointers (88 bytes on LP64). */
typedef struct DBSCudaDecodeArgs {
    int batch_size;               /* B */
    int steps;                    /* T (the largest per-example step count when steps_per_example is set) */
    int beam_size;                /* K, also the stride of every beam dimension */
    int vocab_size;               /* V */
    int eos_token;                /* end-of-sequence token, or -1 for no EOS handling */
    int min_length;               /* EOS tokens are excluded until a hypothesis would reach this length */
    float length_penalty_alpha;   /* GNMT exponent: scores are raw / ((5 + len) / 6)^alpha; 0 = off */
    int no_repeat_ngram_size;     /* n > 0: block tokens that would repeat an n-gram of the beam's own prefix */
    float repetition_penalty;     /* > 1: tokens already in the prefix lose log(penalty); <= 1 = off */
    int reserved0;                /* must be 0 */
    /* Optional int32 [B] device arrays overriding the scalars per example, or NULL:
     * steps in [1, T], beams in [1, K], EOS in [-1, V), min lengths >= 0. */
    const int32_t* steps_per_example;
    const int32_t* beam_sizes_per_example;
    const int32_t* eos_tokens_per_example;
    const int32_t* min_lengths_per_example;
    const uint8_t* banned_tokens; /* optional uint8 [V]: a non-zero entry bans the token everywhere */
} DBSCudaDecodeArgs;

/* Where a decode writes its results (ref: include/dbs_cuda.h:89-100).
 * final_scores is required; every other pointer may be NULL. */
typedef struct DBSCudaDecodeOutputs {
    float* final_scores;          /* [B, K] final length-penalised scores, best first */
    float* final_raw_scores;      /* [B, K] final cumulative log-probabilities */
    int32_t* final_lengths;       /* [B, K] */
    int32_t* tokens;              /* [B, T, K] token of each slot after each step */
    int32_t* parents;             /* [B, T, K] slot of the previous step each slot extends */
    int32_t* lengths;             /* [B, T, K] hypothesis length after each step */
    float* scores;                /* [B, T, K] length-penalised ranking scores */
    float* raw_scores;            /* [B, T, K] cumulative log-probabilities */
    uint8_t* from_logprob;        /* [B, T, K] 1 when the slot consumed an input entry, 0 for carried/empty slots */
    uint8_t* invalid_input;       /* [B] 1 when a row the search read for the example held NaN or +inf */
} DBSCudaDecodeOutputs;

/* 1 when the CUDA runtime reports at least one device (ref: include/dbs_cuda.h:102). */
DBS_CUDA_EXPORT int dbs_cuda_available(void);
/* Static English text of a status code (ref: include/dbs_cuda.h:103). */
DBS_CUDA_EXPORT const char* dbs_cuda_status_string(int status);

/* Process-wide debug switch: 1 waits for the stream at the end of every call,
 * 0 (default) does not. Other values are rejected (ref: include/dbs_cuda.h:106-107). */
DBS_CUDA_EXPORT int dbs_cuda_set_synchronization(int synchronize);
DBS_CUDA_EXPORT int dbs_cuda_get_synchronization(void);

/* Bytes of scratch a decode / backward with these arguments needs, or a
 * negative value when the arguments are rejected (ref: include/dbs_cuda.h:111-112). */
DBS_CUDA_EXPORT int64_t dbs_cuda_decode_workspace_size(const DBSCudaDecodeArgs* args);
DBS_CUDA_EXPORT int64_t dbs_cuda_backward_workspace_size(const DBSCudaDecodeArgs* args);

/* Exact hard beam search over float32 log-probabilities [B, T, K, V]
 * (ref: include/dbs_cuda.h:114-128). With workspace == NULL the scratch is
 * taken from the stream-ordered allocator and returned at the end of the call.
 * NaN and +inf entries are never candidates; every element of every row the
 * search reads is checked for them and outputs->invalid_input flags the
 * examples that had one. Per-example arrays are range-checked on the device,
 * which waits for the stream once. */
DBS_CUDA_EXPORT int dbs_cuda_decode(
    const float* log_probs,
    const DBSCudaDecodeArgs* args,
    const DBSCudaDecodeOutputs* outputs,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* Beam state between steps of a caller-driven search (ref: include/dbs_cuda.h:130-154).
 * Initial state: raw_scores = {0, -inf, ...} per example, lengths = finished = 0.
 * The step ranks the candidates of live, unfinished beams by raw score; this
 * equals the CPU ranking by penalised score when, within each example, those
 * beams share one length (true of the initial state and of every state a step
 * produces). The precondition is not checked on the device. */
typedef struct DBSCudaBeamState {
    float* raw_scores;          /* [B, K], advanced in place */
    int32_t* lengths;           /* [B, K], advanced in place */
    uint8_t* finished;          /* [B, K], advanced in place; non-zero after EOS */
    const int32_t* prefixes;    /* [B, K, prefix_stride]: the first lengths[b, k] tokens of beam k.
                                   Read only for n-gram blocking, the repetition penalty, or the
                                   carried token of extra EOS; entries outside [0, V) are ignored. */
    int prefix_stride;          /* capacity of a prefix row, >= every live beam's length */
    int reserved0;              /* must be 0 */
} DBSCudaBeamState;

/* Scratch bytes of one step, or negative for rejected arguments (ref: include/dbs_cuda.h:158). */
DBS_CUDA_EXPORT int64_t dbs_cuda_decode_step_workspace_size(const DBSCudaDecodeArgs* args, int prefix_stride);

/* One search step over the step's float32 rows [B, K, V] (row k extends beam k);
 * args->steps must be 1 and steps_per_example NULL (ref: include/dbs_cuda.h:160-177).
 * Advances `state` and writes the step's [B, K] trace (tokens, parents, lengths,
 * scores, raw_scores, from_logprob), the invalid flags, and, when final_scores
 * is set, the final_* values of the beams after the step. */
DBS_CUDA_EXPORT int dbs_cuda_decode_step(
    const float* log_probs,
    const DBSCudaDecodeArgs* args,
    const DBSCudaBeamState* state,
    const DBSCudaDecodeOutputs* outputs,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* Surrogate gradient of the final scores of a decode with the same args,
 * accumulated (+=) into float32 grad_log_probs [B, T, K, V]
 * (ref: include/dbs_cuda.h:179-196). Deterministic: no atomics, parents sum
 * their children in slot order, as the CPU backward does. */
DBS_CUDA_EXPORT int dbs_cuda_backward(
    const DBSCudaDecodeArgs* args,
    const int32_t* parents,
    const int32_t* tokens,
    const int32_t* lengths,
    const uint8_t* from_logprob,
    const float* grad_final_scores,
    float* grad_log_probs,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* Input element types (ref: include/dbs_cuda.h:197-199; the values of DBSDataTypeC in dbs.h). */
#define DBS_CUDA_DTYPE_F32 0
#define DBS_CUDA_DTYPE_F16 1
#define DBS_CUDA_DTYPE_BF16 2

/* dbs_cuda_decode over inputs of data_type (ref: include/dbs_cuda.h:201-221).
 * 16-bit inputs are widened exactly. With from_logits != 0 the inputs are
 * logits and each row the search reads is normalised on the fly with the CPU
 * decoder's deterministic logsumexp, so results equal the CPU decoder's bit
 * for bit. row_lse (optional float32 [B, T, K]) receives that logsumexp for
 * every row read (-inf for a row without a finite logit) and 0 elsewhere. */
DBS_CUDA_EXPORT int dbs_cuda_decode_ex(
    const void* inputs,
    int data_type,
    int from_logits,
    const DBSCudaDecodeArgs* args,
    const DBSCudaDecodeOutputs* outputs,
    float* row_lse,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* dbs_cuda_decode_step over a step's [B, K, V] inputs of data_type; row_lse is [B, K]
 * (ref: include/dbs_cuda.h:223-236). */
DBS_CUDA_EXPORT int dbs_cuda_decode_step_ex(
    const void* inputs,
    int data_type,
    int from_logits,
    const DBSCudaDecodeArgs* args,
    const DBSCudaBeamState* state,
    const DBSCudaDecodeOutputs* outputs,
    float* row_lse,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* Inputs of dbs_cuda_backward_ex (ref: include/dbs_cuda.h:238-253). Gradient
 * pointers may be NULL (a zero gradient). */
typedef struct DBSCudaBackwardInputs {
    const int32_t* parents;              /* [B, T, K] */
    const int32_t* tokens;               /* [B, T, K] */
    const int32_t* lengths;              /* [B, T, K] */
    const uint8_t* from_logprob;         /* [B, T, K] */
    const float* grad_final_scores;      /* [B, K] or NULL */
    const float* grad_final_raw_scores;  /* [B, K] or NULL */
    const float* grad_scores;            /* [B, T, K] or NULL */
    const float* grad_raw_scores;        /* [B, T, K] or NULL */
    const void* logits;                  /* [B, T, K, V] of logits_type when decoded from logits, else NULL */
    int logits_type;                     /* DBS_CUDA_DTYPE_* */
    int reserved0;                       /* must be 0 */
    const float* row_lse;                /* [B, T, K] row_lse of the decode; required with logits */
    void* reserved[4];                   /* must be NULL */
} DBSCudaBackwardInputs;

/* Surrogate gradient of any of the decode's score outputs, accumulated (+=)
 * into float32 grad_inputs [B, T, K, V] (ref: include/dbs_cuda.h:255-268).
 * From logits, each row carrying a path gradient g also receives
 * -softmax(row) * sum(g) over the whole row. */
DBS_CUDA_EXPORT int dbs_cuda_backward_ex(
    const DBSCudaDecodeArgs* args,
    const DBSCudaBackwardInputs* inputs,
    float* grad_inputs,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* Capacity of DBSCudaSearchOptions.extra_eos_tokens (ref: include/dbs_cuda.h:271). */
#define DBS_CUDA_MAX_EXTRA_EOS 16

/* Options of the _ex2 functions; zero-initialise it (ref: include/dbs_cuda.h:273-284).
 * extra_eos_tokens are additional end-of-sequence ids in [0, V): emitting any
 * of them finishes a hypothesis, min_length masks them, and a finished beam is
 * carried forward with the token it ended on. They need EOS handling on. */
typedef struct DBSCudaSearchOptions {
    int extra_eos_count;
    int32_t extra_eos_tokens[DBS_CUDA_MAX_EXTRA_EOS];
    int reserved0;        /* must be 0 */
    void* reserved[4];    /* must be NULL */
} DBSCudaSearchOptions;

/* dbs_cuda_decode_ex with search options (NULL allowed) (ref: include/dbs_cuda.h:286-298). */
DBS_CUDA_EXPORT int dbs_cuda_decode_ex2(
    const void* inputs,
    int data_type,
    int from_logits,
    const DBSCudaDecodeArgs* args,
    const DBSCudaSearchOptions* options,
    const DBSCudaDecodeOutputs* outputs,
    float* row_lse,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* dbs_cuda_decode_step_ex with search options (ref: include/dbs_cuda.h:300-316).
 * With extra EOS tokens a finished beam carries the last token of its prefix
 * (or eos_token when the prefix does not reach it). */
DBS_CUDA_EXPORT int dbs_cuda_decode_step_ex2(
    const void* inputs,
    int data_type,
    int from_logits,
    const DBSCudaDecodeArgs* args,
    const DBSCudaSearchOptions* options,
    const DBSCudaBeamState* state,
    const DBSCudaDecodeOutputs* outputs,
    float* row_lse,
    void* workspace,
    int64_t workspace_bytes,
    void* stream);

/* out[i] = GNMT penalty ((5 + max(lengths[i], 1)) / 6)^alpha, the exact
 * value the search uses (ref: include/dbs_cuda.h:318-320). */
DBS_CUDA_EXPORT int dbs_cuda_length_penalty(const int32_t* lengths, int64_t count, float alpha, float* out, void* stream);

/* Per-slot path gradient of the final scores (ref: include/dbs_cuda.h:322-334):
 * draws[b, t, k] is the gradient of the input entry slot k of step t consumed
 * (0 for carried and empty slots). Scattering it to (b, t, parents, tokens) of
 * a zero [B, T, K, V] tensor reproduces dbs_cuda_backward exactly. */
DBS_CUDA_EXPORT int dbs_cuda_path_gradient(
    const DBSCudaDecodeArgs* args,
    const int32_t* parents,
    const int32_t* tokens,
    const int32_t* lengths,
    const uint8_t* from_logprob,
    const float* grad_final_scores,
    float* draws,
    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DBS_CUDA_H */
