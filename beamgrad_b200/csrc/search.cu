// SPDX-License-Identifier: MIT
//
// Device side of a caller-driven search loop (one model call per step): the
// token prefixes of the beams stay in device memory and advance with one
// kernel per step, and whether any beam is still live is recorded on the
// device, so a loop needs no host synchronisation per step.
//
// Prefix update (python/beamgrad/_search.py:450-455 of beamgrad 2.3.0, where
// it is a torch gather + cat + where per step): after step t,
//     out[b, k, j] = in[b, parents[b, k], j]   for j < t   (parent >= 0)
//     out[b, k, t] = tokens[b, k] if from_logprob[b, k] else -1
// and the whole row is -1 for a dead slot (parent < 0).
// Live flag (python/beamgrad/_search.py:366-368): some beam has a finite raw
// score and is not finished.
#include "engine.cuh"

namespace dbsb {

__global__ void advance_prefixes_kernel(int B, int K, int step, int stride, const int32_t* __restrict__ parents,
                                        const int32_t* __restrict__ tokens, const uint8_t* __restrict__ from_logprob,
                                        const int32_t* __restrict__ in, int32_t* __restrict__ out,
                                        const float* __restrict__ raw, const uint8_t* __restrict__ finished,
                                        uint8_t* __restrict__ any_live) {
    const int64_t width = static_cast<int64_t>(step) + 1;
    const int64_t n = static_cast<int64_t>(B) * K * width;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t bk = i / width;
        const int j = static_cast<int>(i - bk * width);
        const int64_t b = bk / K;
        const int q = parents[bk];
        int32_t v = -1;
        if (q >= 0 && q < K) {
            if (j < step) v = in[(b * K + q) * stride + j];
            else v = from_logprob[bk] ? tokens[bk] : -1;
        }
        out[bk * stride + j] = v;
        if (j == 0 && any_live) {
            const float r = raw[bk];
            if (r > f_ninf() && r < f_inf() && finished[bk] == 0) *any_live = 1;  // benign race: all store 1
        }
    }
}

cudaError_t launch_advance_prefixes(int B, int K, int step, int stride, const int32_t* parents, const int32_t* tokens,
                                    const uint8_t* from_logprob, const int32_t* in, int32_t* out, const float* raw,
                                    const uint8_t* finished, uint8_t* any_live, int sm_count, cudaStream_t stream) {
    const int64_t n = static_cast<int64_t>(B) * K * (static_cast<int64_t>(step) + 1);
    const int64_t want = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count) * 8;
    const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
    advance_prefixes_kernel<<<grid > 0 ? grid : 1, 256, 0, stream>>>(B, K, step, stride, parents, tokens, from_logprob,
                                                                     in, out, raw, finished, any_live);
    return cudaGetLastError();
}

}  // namespace dbsb
