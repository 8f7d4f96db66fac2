// SPDX-License-Identifier: MIT
//
// Host-side dispatch of the decode kernels (decode_impl.cuh): the kernel family by data
// type and input kind, the chained or waiting decode, and the small helper kernels that
// every decode shares (workspace initialisation, per-example argument validation, the
// bounded-wait self test). The per-dtype kernel instantiations live in decode_f32.cu,
// decode_f16.cu and decode_bf16.cu so that they compile in parallel.
#include "decode_impl.cuh"

namespace dbsb {

cudaError_t launch_decode_f32(const DecodeParams& p, bool logits, cudaStream_t stream, int sm_count);
cudaError_t launch_decode_f16(const DecodeParams& p, bool logits, cudaStream_t stream, int sm_count);
cudaError_t launch_decode_bf16(const DecodeParams& p, bool logits, cudaStream_t stream, int sm_count);

// ---------------------------------------------------------------------------
// Set-up kernels
// ---------------------------------------------------------------------------
__global__ void init_decode_kernel(DecodeParams p) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t beams = static_cast<int64_t>(p.B) * p.K;
    if (i < beams) {
        const int b = static_cast<int>(i / p.K);
        const int k = static_cast<int>(i - static_cast<int64_t>(b) * p.K);
        if (!p.step_api) {
            const Meta m = load_meta(p, b);
            p.raw[i] = (k == 0 && k < m.beam) ? 0.0f : f_ninf();
            p.len[i] = 0;
            p.ended[i] = 0;
            p.last[i] = -1;
            if (p.prefix_len[0]) p.prefix_len[0][i] = 0;
        }
        if (k == 0) {
            p.flag[b] = 0;
            p.arrive[b] = 0;
            if (p.out.invalid_input) p.out.invalid_input[b] = 0;
        }
    }
    if (p.count && i < static_cast<int64_t>(p.B) * p.T) p.count[i] = 0;
    if (i == 0) {
        *p.ticket = 0;
        *p.error = kErrNone;
    }
}

// Per-example arguments in range? (status stays 0 when they all are.)
__global__ void validate_meta_kernel(DecodeParams p, int* status) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= p.B) return;
    const int steps = p.steps_pe ? p.steps_pe[b] : p.T;
    const int beam = p.beams_pe ? p.beams_pe[b] : p.K;
    const int eos = p.eos_pe ? p.eos_pe[b] : p.eos;
    const int ml = p.minlen_pe ? p.minlen_pe[b] : p.min_length;
    const bool ok = steps >= 1 && steps <= p.T && beam >= 1 && beam <= p.K && eos >= -1 && eos < p.V && ml >= 0;
    if (!ok) atomicExch(status, 1);
}

// ---------------------------------------------------------------------------
// Host-side launch
// ---------------------------------------------------------------------------

// Keys kept per row list.
int decode_list_len(int K) {
    if (K <= 1) return 1;
    if (K <= 2) return 2;
    if (K <= 4) return 4;
    if (K <= 8) return 8;
    if (K <= 16) return 16;
    return K;
}

// Entries kept per row record of the chained decode.
int decode_chain_list_len(int K) {
    if (K <= 4) return chain_list_len<4>();
    if (K <= 8) return chain_list_len<8>();
    if (K <= 16) return chain_list_len<16>();
    return 2 * K;
}

// Dynamic shared memory of the chained decode's selection scratch (beams above 16).
size_t decode_chain_wide_smem(int K) {
    if (K <= 64) return wide_dyn_smem<64>();
    if (K <= 256) return wide_dyn_smem<256>();
    return wide_dyn_smem<kSelectCap>();
}

size_t decode_select_smem(int K) {
    return K <= kFastBeam ? sizeof(SelectShared<kFastBeam>) : sizeof(SelectShared<kSelectCap>);
}

cudaError_t launch_decode(const DecodeParams& p, int dtype, bool logits, cudaStream_t stream, int sm_count) {
    switch (dtype) {
        case DBS_CUDA_DTYPE_F16: return launch_decode_f16(p, logits, stream, sm_count);
        case DBS_CUDA_DTYPE_BF16: return launch_decode_bf16(p, logits, stream, sm_count);
        default: return launch_decode_f32(p, logits, stream, sm_count);
    }
}

cudaError_t launch_init(const DecodeParams& p, cudaStream_t stream) {
    int64_t n = static_cast<int64_t>(p.B) * p.K;
    if (p.count && static_cast<int64_t>(p.B) * p.T > n) n = static_cast<int64_t>(p.B) * p.T;
    const int64_t blocks = (n + 255) / 256;
    init_decode_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
    return cudaGetLastError();
}

// Self-test of the bounded waits: warp 0 waits on a flag that nothing sets, warp 1 on
// an mbarrier that nothing arrives at (no copy is in flight). Both give up after
// p.timeout_ns, record kErrTimeout in p.error and return false; words[0..1] receive
// their results (1 = the wait succeeded).
__global__ void wait_selftest_kernel(DecodeParams p, const int32_t* flag, int32_t* words) {
    __shared__ unsigned long long mbar;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) mbar_init(&mbar);
    __syncthreads();
    if (warp == 0) {
        const bool ok = wait_flag_warp(p, flag, 1);
        if (lane == 0) words[0] = ok ? 1 : 0;
    } else if (warp == 1 && lane == 0) {
        words[1] = mbar_wait(p, &mbar, 0) ? 1 : 0;
    }
}

cudaError_t launch_wait_selftest(const DecodeParams& p, const int32_t* flag, int32_t* words, cudaStream_t stream) {
    wait_selftest_kernel<<<1, 64, 0, stream>>>(p, flag, words);
    return cudaGetLastError();
}

cudaError_t launch_validate(const DecodeParams& p, int* status, cudaStream_t stream) {
    validate_meta_kernel<<<static_cast<unsigned>((p.B + 255) / 256), 256, 0, stream>>>(p, status);
    return cudaGetLastError();
}

}  // namespace dbsb
