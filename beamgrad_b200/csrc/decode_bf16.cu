// SPDX-License-Identifier: MIT
//
// Decode kernels for bf16 inputs (one translation unit per input type so
// the library builds in parallel).
#include "decode_impl.cuh"

namespace dbsb {

cudaError_t launch_decode_bf16(const DecodeParams& p, bool logits, cudaStream_t stream, int sm_count) {
    return logits ? launch_decode_k<2, true>(p, stream, sm_count) : launch_decode_k<2, false>(p, stream, sm_count);
}

}  // namespace dbsb
