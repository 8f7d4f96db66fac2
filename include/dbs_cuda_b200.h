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

#ifdef __cplusplus
}
#endif

#endif
