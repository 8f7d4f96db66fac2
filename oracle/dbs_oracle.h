/* SPDX-License-Identifier: MIT
 *
 * dbs_oracle.h -- TEST INFRASTRUCTURE ONLY. A plain-C, single-threaded CPU
 * restatement of beamgrad's reference CPU decoder (src/decoder.cpp,
 * src/kernels.hpp, src/kernels_scalar.cpp, src/logits.hpp, src/penalty.hpp,
 * src/half.hpp, src/common.hpp of beamgrad 2.3.0), used by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU baseline as the checker of the
 * CUDA engine. Nothing in the product links or calls it.
 *
 * The functions take the engine's own argument structs (include/dbs_cuda.h)
 * with HOST pointers everywhere, so a test hands the same arguments to the
 * oracle and to the device engine.
 *
 * Parity pin: tests/test_oracle.py checks this restatement bit for bit against
 * the reference library compiled from its own sources (oracle/Makefile ->
 * oracle/_ref/libdbs.so) on seeded cases, and against the committed golden
 * vectors in tests/golden/ generated from that library.
 */
#ifndef DBS_ORACLE_H
#define DBS_ORACLE_H

#include "../include/dbs_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* 0 on success, DBS_CUDA_STATUS_INVALID_ARGUMENT otherwise. */
int oracle_decode(const void* inputs, int data_type, int from_logits, const DBSCudaDecodeArgs* args,
                  const DBSCudaSearchOptions* options, const DBSCudaDecodeOutputs* outputs, float* row_lse);

int oracle_decode_step(const void* inputs, int data_type, int from_logits, const DBSCudaDecodeArgs* args,
                       const DBSCudaSearchOptions* options, const DBSCudaBeamState* state,
                       const DBSCudaDecodeOutputs* outputs, float* row_lse);

int oracle_backward(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* inputs, float* grad_inputs);
/* oracle_backward plus the selected-beam weights term (src/decoder.cpp:599-604). */
int oracle_backward_selected(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* inputs, const float* weights,
                             const float* grad_weights, float temperature, float* grad_inputs);
/* softmax_selected (src/kernels_scalar.cpp:277-302) per step over the decode's scores [B, T, K]. */
void oracle_selected_weights(const DBSCudaDecodeArgs* args, const float* scores, float temperature, float* weights);

int oracle_path_gradient(const DBSCudaDecodeArgs* args, const int32_t* parents, const int32_t* tokens,
                         const int32_t* lengths, const uint8_t* from_logprob, const float* grad_final_scores,
                         float* draws);

void oracle_length_penalty(const int32_t* lengths, int64_t count, float alpha, float* out);

/* Building blocks, exported for unit tests. */
float oracle_gnmt_penalty(int length, float alpha);
float oracle_exp_nonpositive(float x);
float oracle_row_lse(const float* row, int vocab_size, int* invalid);
/* Vocabulary shards (lane-interleaved, world = 1, 2, 4 or 8): the shard's lane sums of
 * a row with maximum mx, and the lse from all 256 lanes. */
void oracle_shard_lanes(const float* shard_row, int shard_vocab, int world, float mx, float* lanes_out);
float oracle_lse_from_lanes(const float* lanes256, float mx);
float oracle_half_to_float(uint16_t bits, int data_type);

#ifdef __cplusplus
}
#endif

#endif
