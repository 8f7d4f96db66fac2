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
 * race on the array, so order them on one stream or otherwise serialize them. */
DBS_CUDA_EXPORT int dbs_cuda_decode_no_alloc(const void* inputs, int data_type, int from_logits,
                                             const DBSCudaDecodeArgs* args, const DBSCudaSearchOptions* options,
                                             const DBSCudaDecodeOutputs* outputs, float* row_lse, void* stream);

#ifdef __cplusplus
}
#endif

#endif
