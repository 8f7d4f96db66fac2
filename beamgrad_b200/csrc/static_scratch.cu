// SPDX-License-Identifier: MIT
//
// dbs_cuda_decode_no_alloc: the decode of dbs_cuda_decode_ex2 for callers that
// can neither allocate device memory nor hand the engine a workspace.
//
// Its scratch (beam state, per-row candidate lists, arrival counters, published
// steps, the work ticket, the error word, n-gram prefixes) lives in one
// file-scope device array of DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES, which every
// GPU that loads this library holds until the process exits. Host code cannot
// pass the array's name to a kernel (on the host that name is only a stand-in
// for the device symbol), so the device address is looked up once per device
// with cudaGetSymbolAddress and cached. The decode's init kernel resets every
// counter, flag and state slot the decode reads before writing it, so the
// array needs no clearing between calls.
#include <mutex>

#include "dbs_cuda.h"
#include "dbs_cuda_b200.h"

namespace {

static __device__ __align__(256) unsigned char g_no_alloc_scratch[DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

// Device address of g_no_alloc_scratch on the current device, looked up on the
// first call made with that device current. Returns nullptr when the lookup fails.
void* scratch_address_of_current_device() {
    static std::mutex mu;
    static void* cache[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < kMaxDevices && cache[dev]) return cache[dev];
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_no_alloc_scratch) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (dev >= 0 && dev < kMaxDevices) cache[dev] = ptr;
    return ptr;
}

}  // namespace

extern "C" {

DBS_CUDA_EXPORT int dbs_cuda_decode_no_alloc(const void* inputs, int data_type, int from_logits,
                                             const DBSCudaDecodeArgs* args, const DBSCudaSearchOptions* options,
                                             const DBSCudaDecodeOutputs* outputs, float* row_lse, void* stream) {
    const int64_t need = dbs_cuda_decode_workspace_size(args);
    if (need < 0) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (need > static_cast<int64_t>(DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    void* scratch = scratch_address_of_current_device();
    if (!scratch) return DBS_CUDA_STATUS_UNAVAILABLE;
    return dbs_cuda_decode_ex2(inputs, data_type, from_logits, args, options, outputs, row_lse, scratch,
                               static_cast<int64_t>(DBS_CUDA_B200_NO_ALLOC_SCRATCH_BYTES), stream);
}

}  // extern "C"
