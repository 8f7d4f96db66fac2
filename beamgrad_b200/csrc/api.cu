// SPDX-License-Identifier: MIT
//
// The C ABI of libdbs_cuda (include/dbs_cuda.h): argument checks, workspace
// layout, launches. Every entry point is asynchronous on the caller's stream
// except where the header says it synchronizes.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <iterator>
#include <limits>
#include <memory>
#include <mutex>

#include "dbs_cuda.h"
#include "dbs_cuda_b200.h"
#include "engine.cuh"

namespace dbsb {

// decode.cu / backward.cu
cudaError_t launch_decode(const DecodeParams& p, int dtype, bool logits, cudaStream_t stream, int sm_count);
cudaError_t launch_init(const DecodeParams& p, cudaStream_t stream);
cudaError_t launch_validate(const DecodeParams& p, int* status, cudaStream_t stream);
cudaError_t launch_wait_selftest(const DecodeParams& p, const int32_t* flag, int32_t* words, cudaStream_t stream);
int decode_list_len(int K);
int decode_chain_list_len(int K);
size_t decode_chain_wide_smem(int K);
size_t decode_select_smem(int K);


cudaError_t launch_backward(const BackwardParams& p, cudaStream_t stream);
// pool.cu
cudaError_t launch_relaxed_pool(const DecodeParams& d, int dtype, bool logits, int P, const float* row_lse,
                                const int32_t* parents, const int32_t* tokens, const int32_t* lengths, const float* raw,
                                const uint8_t* from_logprob, int32_t* pool_parents, int32_t* pool_tokens,
                                int32_t* pool_lengths, float* pool_scores, float* pool_raw, uint8_t* pool_from,
                                float* relaxed, float temperature, float tolerance, int max_iters, cudaStream_t stream);
cudaError_t launch_logit_correction(const BackwardParams& p, int dtype, const void* logits, const float* row_lse,
                                    cudaStream_t stream);
cudaError_t launch_dense_grad(const BackwardParams& p, int in_type, const void* logits, const float* row_lse,
                              int out_type, void* grad, int vec, int sm_count, cudaStream_t stream);
cudaError_t launch_length_penalty(const int32_t* lengths, int64_t count, float alpha, float* out, cudaStream_t stream);
cudaError_t launch_selected_weights(int64_t rows, int K, const float* scores, float temperature, float* out,
                                    cudaStream_t stream);
// search.cu
cudaError_t launch_advance_prefixes(int B, int K, int step, int stride, const int32_t* parents, const int32_t* tokens,
                                    const uint8_t* from_logprob, const int32_t* in, int32_t* out, const float* raw,
                                    const uint8_t* finished, uint8_t* any_live, int sm_count, cudaStream_t stream);
cudaError_t launch_backtrack(int B, int T, int K, const int32_t* tokens, const int32_t* parents,
                             const int32_t* steps_pe, int64_t* out, cudaStream_t stream);

// vshard.cu
cudaError_t launch_vshard_scan(const VShardParams& q, int dtype, cudaStream_t stream, int sm_count);
cudaError_t launch_vshard_lanes(const VShardParams& q, int dtype, cudaStream_t stream, int sm_count);
cudaError_t launch_vshard_merge(const VShardParams& q, bool logits, cudaStream_t stream, int sm_count);
cudaError_t launch_vshard_select(const VShardParams& q, bool logits, cudaStream_t stream);
cudaError_t launch_vshard_rescan(const VShardParams& q, int dtype, bool logits, cudaStream_t stream, int sm_count);

namespace {

constexpr int64_t kAlign = 256;
constexpr unsigned long long kTimeoutNs = 20ull * 1000ull * 1000ull * 1000ull;  // bounded inter-CTA waits
constexpr int kMaxRowSmem = 160 * 1024;  // largest row staged in shared memory
constexpr int64_t kLanesPerRow = 256;     // logsumexp lanes of a row (the reference's fixed order)

// Synchronous checking: dbs_cuda_set_synchronization(1), or either environment variable set
// to 1 (include/dbs_cuda.h). The process-wide flag is the only state the library keeps.
std::atomic<int> g_sync{0};
constexpr const char* kSyncVariables[] = {"DBS_CUDA_SYNC_CHECK", "DBS_CUDA_DEBUG_SYNC"};

int64_t align_up(int64_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

bool sync_requested() {
    if (g_sync.load(std::memory_order_relaxed) != 0) return true;
    return std::any_of(std::begin(kSyncVariables), std::end(kSyncVariables), [](const char* name) {
        const char* v = std::getenv(name);
        return v != nullptr && v[0] == '1';
    });
}

// Element types of inputs and gradients: the header's code and the bytes per element.
struct DtypeInfo {
    int code;
    int bytes;
};
constexpr DtypeInfo kDtypes[] = {{DBS_CUDA_DTYPE_F32, 4}, {DBS_CUDA_DTYPE_F16, 2}, {DBS_CUDA_DTYPE_BF16, 2}};

int elem_bytes(int code) {
    for (const DtypeInfo& d : kDtypes)
        if (d.code == code) return d.bytes;
    return 0;
}
bool valid_dtype(int code) { return elem_bytes(code) > 0; }

bool has_per_example(const DBSCudaDecodeArgs& a) {
    const void* arrays[] = {a.steps_per_example, a.beam_sizes_per_example, a.eos_tokens_per_example,
                            a.min_lengths_per_example};
    return std::any_of(std::begin(arrays), std::end(arrays), [](const void* q) { return q != nullptr; });
}
bool constrained(const DBSCudaDecodeArgs& a) { return a.no_repeat_ngram_size > 0 || a.repetition_penalty > 1.0f; }

// The problems the engine accepts (include/dbs_cuda.h), one predicate per rule.
using ArgRule = bool (*)(const DBSCudaDecodeArgs&);
constexpr ArgRule kArgRules[] = {
    [](const DBSCudaDecodeArgs& a) { return a.batch_size > 0 && a.steps > 0 && a.beam_size > 0 && a.vocab_size > 0; },
    [](const DBSCudaDecodeArgs& a) { return a.beam_size <= DBS_CUDA_MAX_BEAM; },
    [](const DBSCudaDecodeArgs& a) { return a.eos_token >= -1 && a.eos_token < a.vocab_size; },
    [](const DBSCudaDecodeArgs& a) { return a.min_length >= 0 && a.reserved0 == 0; },
    [](const DBSCudaDecodeArgs& a) { return std::isfinite(a.length_penalty_alpha) && a.length_penalty_alpha >= 0.0f; },
    [](const DBSCudaDecodeArgs& a) { return std::isfinite(a.repetition_penalty) && a.repetition_penalty >= 0.0f; },
    // A candidate's index parent * V + token is a 32-bit key field.
    [](const DBSCudaDecodeArgs& a) {
        return static_cast<int64_t>(a.beam_size) * a.vocab_size <= std::numeric_limits<int32_t>::max();
    },
    // Row tickets (B * K * T of them) are counted in 31 bits.
    [](const DBSCudaDecodeArgs& a) {
        return static_cast<int64_t>(a.batch_size) * a.beam_size * a.steps <= (int64_t{1} << 31);
    },
    [](const DBSCudaDecodeArgs& a) {
        return static_cast<double>(a.batch_size) * a.steps * a.beam_size * a.vocab_size < 9.0e18;
    },
};

bool valid_args(const DBSCudaDecodeArgs* a) {
    return a != nullptr &&
           std::all_of(std::begin(kArgRules), std::end(kArgRules), [a](ArgRule rule) { return rule(*a); });
}

// Search options: reserved fields zero, at most DBS_CUDA_MAX_EXTRA_EOS extra EOS tokens, each
// inside the vocabulary, and only with EOS handling on.
bool valid_options(const DBSCudaSearchOptions* o, const DBSCudaDecodeArgs& a) {
    if (o == nullptr) return true;
    if (o->reserved0 != 0) return false;
    if (std::any_of(std::begin(o->reserved), std::end(o->reserved), [](const void* r) { return r != nullptr; }))
        return false;
    const int n = o->extra_eos_count;
    if (n < 0 || n > DBS_CUDA_MAX_EXTRA_EOS) return false;
    const bool inside = std::all_of(o->extra_eos_tokens, o->extra_eos_tokens + n,
                                    [&a](int32_t tok) { return tok >= 0 && tok < a.vocab_size; });
    return inside && (n == 0 || a.eos_token >= 0 || a.eos_tokens_per_example != nullptr);
}

// Largest row-record area of a chained decode; larger decodes use the waiting kernel.
constexpr int64_t kMaxChainRecordBytes = int64_t{4} << 30;

// Workspace layout of a decode or of one step.
struct DecodeLayout {
    int64_t raw, len, ended, last, keys, arrive, flag, ticket, error, status;
    int64_t prefix[2], prefix_len[2];
    int64_t rkeys, rlse, rinfo, count;  // chained decode only (else -1)
    int64_t total;
    int list_len;
    bool chain;
};

// A decode runs chained (rows keep parent-independent records, selections never wait)
// unless its record area would exceed the cap.
bool chain_eligible(const DBSCudaDecodeArgs& a) {
    const int64_t rows = static_cast<int64_t>(a.batch_size) * a.steps * a.beam_size;
    return rows * decode_chain_list_len(a.beam_size) * 8 <= kMaxChainRecordBytes;
}

DecodeLayout make_layout(const DBSCudaDecodeArgs& a, bool step_api, bool force_chain = false) {
    DecodeLayout L{};
    const int64_t B = a.batch_size, K = a.beam_size, T = a.steps;
    int64_t off = 0;
    auto take = [&off](int64_t bytes) {
        const int64_t at = off;
        off = align_up(off + (bytes > 0 ? bytes : 1));
        return at;
    };
    L.chain = !step_api && (force_chain || chain_eligible(a));
    L.list_len = L.chain ? decode_chain_list_len(a.beam_size) : decode_list_len(a.beam_size);
    if (!step_api) {
        L.raw = take(B * K * 4);
        L.len = take(B * K * 4);
        L.ended = take(B * K);
        L.last = take(B * K * 4);
    }
    L.keys = take(B * K * L.list_len * 8);
    L.arrive = take(B * 4);
    L.flag = take(B * 4);
    L.ticket = take(4);
    L.error = take(4);
    L.status = take(4);
    if (!step_api && constrained(a)) {
        for (int i = 0; i < 2; ++i) {
            L.prefix[i] = take(B * K * T * 4);
            L.prefix_len[i] = take(B * K * 4);
        }
    } else {
        L.prefix[0] = L.prefix[1] = L.prefix_len[0] = L.prefix_len[1] = -1;
    }
    L.rkeys = L.rlse = L.rinfo = L.count = -1;
    if (L.chain) {
        const int64_t rows = B * T * K;
        L.rkeys = take(rows * L.list_len * 8);
        L.rlse = take(rows * 4);
        L.rinfo = take(rows * 4);
        L.count = take(B * T * 4);
    }
    L.total = off;
    return L;
}

// The memory one call works in: the caller's workspace (rejected when smaller than the
// layout needs), or, when the caller passed none, a stream-ordered allocation on the call's
// stream that is released (also stream-ordered) when the call returns.
struct StreamOrderedFree {
    cudaStream_t stream;
    void operator()(char* p) const {
        if (p != nullptr) cudaFreeAsync(p, stream);
    }
};

struct WorkArea {
    std::unique_ptr<char, StreamOrderedFree> owned;
    char* base = nullptr;
    int status = DBS_CUDA_STATUS_OK;
    // The sub-buffer at byte offset `off` of the layout (-1: not in this layout).
    template <class T>
    T* at(int64_t off) const {
        return off < 0 ? nullptr : reinterpret_cast<T*>(base + off);
    }
};

WorkArea work_area(void* caller, int64_t caller_bytes, int64_t need, cudaStream_t stream) {
    WorkArea w{std::unique_ptr<char, StreamOrderedFree>(nullptr, StreamOrderedFree{stream})};
    if (caller != nullptr) {
        w.base = static_cast<char*>(caller);
        w.status = caller_bytes >= need ? DBS_CUDA_STATUS_OK : DBS_CUDA_STATUS_INVALID_ARGUMENT;
        return w;
    }
    void* p = nullptr;
    if (cudaMallocAsync(&p, static_cast<size_t>(std::max<int64_t>(need, 1)), stream) != cudaSuccess) {
        cudaGetLastError();  // clear the sticky-free error so later calls are not blamed for it
        w.status = DBS_CUDA_STATUS_OUT_OF_MEMORY;
        return w;
    }
    w.owned.reset(static_cast<char*>(p));
    w.base = w.owned.get();
    return w;
}

int sm_count_of_current_device() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

// The status a call returns once its work is enqueued: LAUNCH_FAILED when a launch failed;
// with synchronous checking also when the stream reports an error or a kernel recorded one
// in the engine's error word (a bounded wait that gave up).
int close_call(cudaStream_t stream, const int32_t* error_word) {
    if (cudaGetLastError() != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (!sync_requested()) return DBS_CUDA_STATUS_OK;
    int32_t recorded = 0;
    bool fine = cudaStreamSynchronize(stream) == cudaSuccess;
    if (fine && error_word != nullptr)
        fine = cudaMemcpy(&recorded, error_word, sizeof recorded, cudaMemcpyDeviceToHost) == cudaSuccess;
    fine = fine && cudaGetLastError() == cudaSuccess && recorded == 0;
    return fine ? DBS_CUDA_STATUS_OK : DBS_CUDA_STATUS_LAUNCH_FAILED;
}

void fill_params(DecodeParams& p, const DBSCudaDecodeArgs& a, const DBSCudaSearchOptions* o) {
    std::memset(&p, 0, sizeof p);
    p.B = a.batch_size;
    p.T = a.steps;
    p.K = a.beam_size;
    p.V = a.vocab_size;
    p.eos = a.eos_token;
    p.min_length = a.min_length;
    p.alpha = a.length_penalty_alpha;
    p.ngram = a.no_repeat_ngram_size > 0 ? a.no_repeat_ngram_size : 0;
    p.penalise = a.repetition_penalty > 1.0f ? 1 : 0;
    // logf of the float penalty on the host, exactly as the CPU decoder computes it.
    p.log_penalty = p.penalise ? std::log(a.repetition_penalty) : 0.0f;
    p.n_extra = o ? o->extra_eos_count : 0;
    for (int i = 0; i < p.n_extra; ++i) p.extra[i] = o->extra_eos_tokens[i];
    p.steps_pe = a.steps_per_example;
    p.beams_pe = a.beam_sizes_per_example;
    p.eos_pe = a.eos_tokens_per_example;
    p.minlen_pe = a.min_lengths_per_example;
    p.banned = a.banned_tokens;
    p.timeout_ns = kTimeoutNs;
    p.one2 = 0x3f8000003f800000ull;    // (1.0f, 1.0f)
    p.nzero2 = 0x8000000080000000ull;  // (-0.0f, -0.0f)
}

// Range check of per-example arrays on the device (one synchronization).
int validate_per_example(const DecodeParams& p, const DBSCudaDecodeArgs& a, int32_t* status, cudaStream_t stream) {
    if (!has_per_example(a)) return DBS_CUDA_STATUS_OK;
    if (cudaMemsetAsync(status, 0, sizeof(int32_t), stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (launch_validate(p, status, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    int32_t h = 1;
    if (cudaMemcpyAsync(&h, status, sizeof h, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return h == 0 ? DBS_CUDA_STATUS_OK : DBS_CUDA_STATUS_INVALID_ARGUMENT;
}

void stage_choice(DecodeParams& p, int dtype, bool from_logits) {
    const int64_t row_bytes = static_cast<int64_t>(p.V) * elem_bytes(dtype) + 16;
    const int64_t row_smem = (row_bytes + 127) / 128 * 128;
    const int64_t sel = static_cast<int64_t>(p.chain && p.K > kFastBeam ? decode_chain_wide_smem(p.K)
                                                                         : decode_select_smem(p.K));
    // From logits, rows that fit are staged in shared memory, where the three passes read
    // them. Chained log-prob rows are read from global memory (pass 1, then the record
    // scan from L2): without a row buffer more CTAs share each SM.
    p.staged = row_smem + sel <= kMaxRowSmem && (from_logits || !p.chain) ? 1 : 0;
    p.row_smem = p.staged ? static_cast<int>(row_smem) : 0;
}

int run_decode(const void* inputs, int dtype, int from_logits, const DBSCudaDecodeArgs* args,
               const DBSCudaSearchOptions* options, const DBSCudaDecodeOutputs* outputs, float* row_lse,
               void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
    if (!inputs || !valid_dtype(dtype) || !valid_args(args) || !outputs || !outputs->final_scores) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (!valid_options(options, *args)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    const DBSCudaDecodeArgs& a = *args;
    const DecodeLayout L = make_layout(a, false);
    const WorkArea ws = work_area(workspace, workspace_bytes, L.total, stream);
    if (ws.status != DBS_CUDA_STATUS_OK) return ws.status;
    DecodeParams p;
    fill_params(p, a, options);
    p.inputs = inputs;
    p.step_api = 0;
    p.raw = ws.at<float>(L.raw);
    p.len = ws.at<int32_t>(L.len);
    p.ended = ws.at<uint8_t>(L.ended);
    p.last = ws.at<int32_t>(L.last);
    for (int i = 0; i < 2; ++i) {
        p.prefix[i] = ws.at<int32_t>(L.prefix[i]);
        p.prefix_len[i] = ws.at<int32_t>(L.prefix_len[i]);
    }
    p.out = *outputs;
    p.row_lse = row_lse;
    p.keys = ws.at<uint64_t>(L.keys);
    p.list_len = L.list_len;
    p.arrive = ws.at<uint32_t>(L.arrive);
    p.flag = ws.at<int32_t>(L.flag);
    p.ticket = ws.at<uint32_t>(L.ticket);
    p.error = ws.at<int32_t>(L.error);
    p.chain = L.chain ? 1 : 0;
    p.rkeys = ws.at<uint64_t>(L.rkeys);
    p.rlse = ws.at<float>(L.rlse);
    p.rinfo = ws.at<uint32_t>(L.rinfo);
    p.count = ws.at<uint32_t>(L.count);
    stage_choice(p, dtype, from_logits != 0);
    const int rc = validate_per_example(p, a, ws.at<int32_t>(L.status), stream);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    if (launch_init(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (launch_decode(p, dtype, from_logits != 0, stream, sm_count_of_current_device()) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, p.error);
}

int run_step(const void* inputs, int dtype, int from_logits, const DBSCudaDecodeArgs* args,
             const DBSCudaSearchOptions* options, const DBSCudaBeamState* state, const DBSCudaDecodeOutputs* outputs,
             float* row_lse, void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
    if (!inputs || !valid_dtype(dtype) || !valid_args(args) || !state || !outputs) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!valid_options(options, *args)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    const DBSCudaDecodeArgs& a = *args;
    if (a.steps != 1 || a.steps_per_example) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!state->raw_scores || !state->lengths || !state->finished || state->prefix_stride < 0 || state->reserved0 != 0) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (constrained(a) && state->prefix_stride > 0 && !state->prefixes) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    const DecodeLayout L = make_layout(a, true);
    const WorkArea ws = work_area(workspace, workspace_bytes, L.total, stream);
    if (ws.status != DBS_CUDA_STATUS_OK) return ws.status;
    DecodeParams p;
    fill_params(p, a, options);
    p.inputs = inputs;
    p.step_api = 1;
    p.raw = state->raw_scores;
    p.len = state->lengths;
    p.ended = state->finished;
    p.last = nullptr;
    p.caller_prefix = state->prefixes;
    p.prefix_stride = state->prefix_stride;
    p.out = *outputs;
    p.row_lse = row_lse;
    p.keys = ws.at<uint64_t>(L.keys);
    p.list_len = L.list_len;
    p.arrive = ws.at<uint32_t>(L.arrive);
    p.flag = ws.at<int32_t>(L.flag);
    p.ticket = ws.at<uint32_t>(L.ticket);
    p.error = ws.at<int32_t>(L.error);
    p.chain = L.chain ? 1 : 0;
    p.rkeys = ws.at<uint64_t>(L.rkeys);
    p.rlse = ws.at<float>(L.rlse);
    p.rinfo = ws.at<uint32_t>(L.rinfo);
    p.count = ws.at<uint32_t>(L.count);
    stage_choice(p, dtype, from_logits != 0);
    const int rc = validate_per_example(p, a, ws.at<int32_t>(L.status), stream);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    if (launch_init(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (launch_decode(p, dtype, from_logits != 0, stream, sm_count_of_current_device()) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, p.error);
}

int64_t backward_ws_bytes(const DBSCudaDecodeArgs& a) {
    return align_up(static_cast<int64_t>(a.batch_size) * a.steps * a.beam_size * 4);
}

BackwardParams backward_params(const DBSCudaDecodeArgs& a) {
    BackwardParams p;
    std::memset(&p, 0, sizeof p);
    p.B = a.batch_size;
    p.T = a.steps;
    p.K = a.beam_size;
    p.V = a.vocab_size;
    p.alpha = a.length_penalty_alpha;
    p.steps_pe = a.steps_per_example;
    p.beams_pe = a.beam_sizes_per_example;
    return p;
}

// ---------------------------------------------------------------------------
// Vocabulary-sharded decode (vshard.cu)
// ---------------------------------------------------------------------------
int vshard_lanes_log2(int world) {
    switch (world) {
        case 1: return 8;
        case 2: return 7;
        case 4: return 6;
        case 8: return 5;
        default: return -1;
    }
}

// Tokens of rank `rank`: L of every full 256-token block, and its part of the last one.
int64_t vshard_shard_vocab(int64_t V, int world, int rank) {
    const int64_t L = kLanesPerRow / world;
    const int64_t nfull = V / kLanesPerRow;
    int64_t tail = V - nfull * kLanesPerRow - rank * L;
    tail = tail < 0 ? 0 : (tail > L ? L : tail);
    return nfull * L + tail;
}

bool vshard_plan_fill(const DBSCudaDecodeArgs* a, int from_logits, int world, int rank, int shard_list,
                      DBSCudaVocabShardPlan& pl) {
    std::memset(&pl, 0, sizeof pl);
    if (!valid_args(a) || vshard_lanes_log2(world) < 0 || rank < 0 || rank >= world || shard_list < 0) return false;
    pl.world_size = world;
    pl.rank = rank;
    pl.lanes = kLanesPerRow / world;
    pl.shard_vocab = static_cast<int32_t>(vshard_shard_vocab(a->vocab_size, world, rank));
    pl.list_len = decode_chain_list_len(a->beam_size);
    // Up to two shards keep whole records; more keep half (their union still holds far
    // more than a record, and a row short of entries is rescanned).
    const int dflt = world <= 2 ? pl.list_len : pl.list_len / 2;
    pl.shard_list_len = shard_list > 0 ? (shard_list < pl.list_len ? shard_list : pl.list_len) : dflt;
    pl.row_words = 1 + (from_logits ? pl.lanes / 2 : 0) + pl.shard_list_len;
    pl.rows = static_cast<int64_t>(a->batch_size) * a->steps * a->beam_size;
    pl.workspace_bytes = make_layout(*a, false, true).total;
    return true;
}

int vshard_setup(const DBSCudaVocabShardCall* c, VShardParams& q) {
    if (!c || !valid_dtype(c->data_type) || c->reserved0 != 0 || !valid_args(c->args)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const DBSCudaDecodeArgs& a = *c->args;
    if (!valid_options(c->options, a)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    DBSCudaVocabShardPlan pl;
    if (!vshard_plan_fill(c->args, c->from_logits, c->world_size, c->rank, c->shard_list_len, pl)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const DBSCudaVocabShardBuffers& bf = c->buffers;
    if (!bf.row_max || !bf.row_min || !bf.exchange || !bf.exchange_all || !bf.resume || !bf.stalled || !bf.workspace) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (bf.workspace_bytes < pl.workspace_bytes || (pl.shard_vocab > 0 && !c->shard_inputs)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (bf.n_rescan < 0 || bf.n_rescan > static_cast<int64_t>(a.batch_size) * a.beam_size) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (bf.n_rescan > 0 && (!bf.rescan_rows || !bf.rescan_slot || !bf.rescan || !bf.rescan_all)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const DecodeLayout L = make_layout(a, false, true);
    char* ws = static_cast<char*>(bf.workspace);
    auto at = [ws](int64_t off) { return off < 0 ? nullptr : ws + off; };
    std::memset(&q, 0, sizeof q);
    DecodeParams& p = q.d;
    fill_params(p, a, c->options);
    p.inputs = nullptr;
    p.step_api = 0;
    p.raw = reinterpret_cast<float*>(at(L.raw));
    p.len = reinterpret_cast<int32_t*>(at(L.len));
    p.ended = reinterpret_cast<uint8_t*>(at(L.ended));
    p.last = reinterpret_cast<int32_t*>(at(L.last));
    for (int i = 0; i < 2; ++i) {
        p.prefix[i] = reinterpret_cast<int32_t*>(at(L.prefix[i]));
        p.prefix_len[i] = reinterpret_cast<int32_t*>(at(L.prefix_len[i]));
    }
    p.out = c->outputs;
    p.row_lse = c->row_lse;
    p.keys = reinterpret_cast<uint64_t*>(at(L.keys));
    p.list_len = L.list_len;
    p.arrive = reinterpret_cast<uint32_t*>(at(L.arrive));
    p.flag = reinterpret_cast<int32_t*>(at(L.flag));
    p.ticket = reinterpret_cast<uint32_t*>(at(L.ticket));
    p.error = reinterpret_cast<int32_t*>(at(L.error));
    p.chain = 1;
    p.rkeys = reinterpret_cast<uint64_t*>(at(L.rkeys));
    p.rlse = reinterpret_cast<float*>(at(L.rlse));
    p.rinfo = reinterpret_cast<uint32_t*>(at(L.rinfo));
    p.count = nullptr;
    q.world = pl.world_size;
    q.rank = pl.rank;
    q.lanes = pl.lanes;
    q.lanes_log2 = vshard_lanes_log2(pl.world_size);
    q.shard_v = pl.shard_vocab;
    q.shard_list = pl.shard_list_len;
    q.row_words = pl.row_words;
    q.key_off = pl.row_words - pl.shard_list_len;
    q.shard = c->shard_inputs;
    q.row_max = bf.row_max;
    q.row_min = bf.row_min;
    q.pack = bf.exchange;
    q.pack_all = bf.exchange_all;
    q.resume = bf.resume;
    q.stalled = bf.stalled;
    q.rescan_rows = bf.rescan_rows;
    q.rescan_slot = bf.rescan_slot;
    q.n_rescan = static_cast<int>(bf.n_rescan);
    q.rescan = bf.rescan;
    q.rescan_all = bf.rescan_all;
    return DBS_CUDA_STATUS_OK;
}

}  // namespace
}  // namespace dbsb

using namespace dbsb;

extern "C" {

DBS_CUDA_EXPORT int dbs_cuda_available(void) {
    int n = 0;
    const bool ok = cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
    if (!ok) cudaGetLastError();
    return ok ? 1 : 0;
}

// Status texts (include/dbs_cuda.h: the same text for each code as beamgrad's library).
struct StatusText {
    int status;
    const char* text;
};
constexpr StatusText kStatusTexts[] = {
    {DBS_CUDA_STATUS_OK, "ok"},
    {DBS_CUDA_STATUS_UNAVAILABLE, "CUDA backend unavailable"},
    {DBS_CUDA_STATUS_INVALID_ARGUMENT, "invalid argument"},
    {DBS_CUDA_STATUS_LAUNCH_FAILED, "CUDA launch failed"},
    {DBS_CUDA_STATUS_OUT_OF_MEMORY, "CUDA out of memory"},
};

DBS_CUDA_EXPORT const char* dbs_cuda_status_string(int status) {
    for (const StatusText& e : kStatusTexts)
        if (e.status == status) return e.text;
    return "unknown CUDA status";
}

DBS_CUDA_EXPORT int dbs_cuda_set_synchronization(int synchronize) {
    if (synchronize != 0 && synchronize != 1) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    g_sync.store(synchronize, std::memory_order_relaxed);
    return DBS_CUDA_STATUS_OK;
}

DBS_CUDA_EXPORT int dbs_cuda_get_synchronization(void) { return g_sync.load(std::memory_order_relaxed); }

DBS_CUDA_EXPORT int64_t dbs_cuda_decode_workspace_size(const DBSCudaDecodeArgs* args) {
    if (!valid_args(args)) return -1;
    return make_layout(*args, false).total;
}

DBS_CUDA_EXPORT int64_t dbs_cuda_backward_workspace_size(const DBSCudaDecodeArgs* args) {
    if (!valid_args(args)) return -1;
    return backward_ws_bytes(*args);
}

DBS_CUDA_EXPORT int64_t dbs_cuda_decode_step_workspace_size(const DBSCudaDecodeArgs* args, int prefix_stride) {
    if (!valid_args(args) || args->steps != 1 || args->steps_per_example || prefix_stride < 0) return -1;
    return make_layout(*args, true).total;
}

DBS_CUDA_EXPORT int dbs_cuda_decode_ex2(const void* inputs, int data_type, int from_logits, const DBSCudaDecodeArgs* args,
                                        const DBSCudaSearchOptions* options, const DBSCudaDecodeOutputs* outputs,
                                        float* row_lse, void* workspace, int64_t workspace_bytes, void* stream) {
    return run_decode(inputs, data_type, from_logits, args, options, outputs, row_lse, workspace, workspace_bytes,
                      static_cast<cudaStream_t>(stream));
}

DBS_CUDA_EXPORT int dbs_cuda_decode_ex(const void* inputs, int data_type, int from_logits, const DBSCudaDecodeArgs* args,
                                       const DBSCudaDecodeOutputs* outputs, float* row_lse, void* workspace,
                                       int64_t workspace_bytes, void* stream) {
    return dbs_cuda_decode_ex2(inputs, data_type, from_logits, args, nullptr, outputs, row_lse, workspace,
                               workspace_bytes, stream);
}

DBS_CUDA_EXPORT int dbs_cuda_decode(const float* log_probs, const DBSCudaDecodeArgs* args,
                                    const DBSCudaDecodeOutputs* outputs, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
    return dbs_cuda_decode_ex(log_probs, DBS_CUDA_DTYPE_F32, 0, args, outputs, nullptr, workspace, workspace_bytes,
                              stream);
}

DBS_CUDA_EXPORT int dbs_cuda_decode_step_ex2(const void* inputs, int data_type, int from_logits,
                                             const DBSCudaDecodeArgs* args, const DBSCudaSearchOptions* options,
                                             const DBSCudaBeamState* state, const DBSCudaDecodeOutputs* outputs,
                                             float* row_lse, void* workspace, int64_t workspace_bytes, void* stream) {
    return run_step(inputs, data_type, from_logits, args, options, state, outputs, row_lse, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream));
}

DBS_CUDA_EXPORT int dbs_cuda_decode_step_ex(const void* inputs, int data_type, int from_logits,
                                            const DBSCudaDecodeArgs* args, const DBSCudaBeamState* state,
                                            const DBSCudaDecodeOutputs* outputs, float* row_lse, void* workspace,
                                            int64_t workspace_bytes, void* stream) {
    return dbs_cuda_decode_step_ex2(inputs, data_type, from_logits, args, nullptr, state, outputs, row_lse, workspace,
                                    workspace_bytes, stream);
}

DBS_CUDA_EXPORT int dbs_cuda_decode_step(const float* log_probs, const DBSCudaDecodeArgs* args,
                                         const DBSCudaBeamState* state, const DBSCudaDecodeOutputs* outputs,
                                         void* workspace, int64_t workspace_bytes, void* stream) {
    return dbs_cuda_decode_step_ex(log_probs, DBS_CUDA_DTYPE_F32, 0, args, state, outputs, nullptr, workspace,
                                   workspace_bytes, stream);
}

DBS_CUDA_EXPORT int dbs_cuda_backward_ex(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                         float* grad_inputs, void* workspace, int64_t workspace_bytes, void* stream_ptr) {
    if (!valid_args(args) || !in || !grad_inputs) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!in->parents || !in->tokens || !in->lengths || !in->from_logprob) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (in->reserved0 != 0 || in->reserved[0] || in->reserved[1] || in->reserved[2] || in->reserved[3]) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (in->logits && (!in->row_lse || !valid_dtype(in->logits_type))) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const DBSCudaDecodeArgs& a = *args;
    BackwardParams p = backward_params(a);
    p.parents = in->parents;
    p.tokens = in->tokens;
    p.lengths = in->lengths;
    p.from_logprob = in->from_logprob;
    p.g_final = in->grad_final_scores;
    p.g_final_raw = in->grad_final_raw_scores;
    p.g_scores = in->grad_scores;
    p.g_raw = in->grad_raw_scores;
    if (!in->logits) {
        p.grad = grad_inputs;
        if (launch_backward(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
        return close_call(stream, nullptr);
    }
    const WorkArea ws = work_area(workspace, workspace_bytes, backward_ws_bytes(a), stream);
    if (ws.status != DBS_CUDA_STATUS_OK) return ws.status;
    p.draws = ws.at<float>(0);
    const size_t slots = static_cast<size_t>(a.batch_size) * a.steps * a.beam_size;
    if (cudaMemsetAsync(p.draws, 0, slots * sizeof(float), stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (launch_backward(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    p.grad = grad_inputs;
    if (launch_logit_correction(p, in->logits_type, in->logits, in->row_lse, stream) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, nullptr);
}

// ---------------------------------------------------------------------------
// Relaxed pool (pool.cu) and its gradient terms (backward_kernel)
// ---------------------------------------------------------------------------
namespace {

bool null_reserved(void* const (&r)[4]) {
    return std::all_of(std::begin(r), std::end(r), [](const void* q) { return q == nullptr; });
}

// What the pool supports, beyond the decode's own rules: no prefix constraints, no
// per-example settings other than steps, no extra EOS tokens.
bool pool_problem_ok(const DBSCudaDecodeArgs& a) {
    return !constrained(a) && !a.beam_sizes_per_example && !a.eos_tokens_per_example && !a.min_lengths_per_example;
}

}  // namespace

DBS_CUDA_EXPORT int dbs_cuda_relaxed_pool(const void* inputs, int data_type, int from_logits,
                                          const DBSCudaDecodeArgs* args, const DBSCudaDecodeOutputs* trace,
                                          const float* row_lse, int pool_size, float soft_topk_temperature,
                                          float soft_topk_tolerance, int soft_topk_max_iters,
                                          const DBSCudaPoolOutputs* pool, void* stream_ptr) {
    if (!inputs || !valid_dtype(data_type) || !valid_args(args) || !trace || !pool) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!pool_problem_ok(*args) || !null_reserved(pool->reserved)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!trace->parents || !trace->tokens || !trace->lengths || !trace->raw_scores || !trace->from_logprob)
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (from_logits && !row_lse) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (pool_size < args->beam_size || pool_size > DBS_CUDA_B200_MAX_POOL) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (pool->relaxed_weights &&
        (!std::isfinite(soft_topk_temperature) || !(soft_topk_temperature > 0.0f) ||
         !std::isfinite(soft_topk_tolerance) || soft_topk_tolerance < 0.0f || soft_topk_max_iters < 0))
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    DecodeParams d;
    fill_params(d, *args, nullptr);
    d.inputs = inputs;
    if (launch_relaxed_pool(d, data_type, from_logits != 0, pool_size, row_lse, trace->parents, trace->tokens,
                            trace->lengths, trace->raw_scores, trace->from_logprob, pool->parents, pool->tokens,
                            pool->lengths, pool->scores, pool->raw_scores, pool->from_logprob, pool->relaxed_weights,
                            soft_topk_temperature, soft_topk_tolerance, soft_topk_max_iters, stream) != cudaSuccess)
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return close_call(stream, nullptr);
}

DBS_CUDA_EXPORT int dbs_cuda_backward_pool(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                           const DBSCudaPoolGradients* pool, float* grad_inputs, void* stream_ptr) {
    if (!valid_args(args) || !in || !pool || !grad_inputs || !pool_problem_ok(*args)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!in->parents || !in->tokens || !in->lengths || !in->from_logprob || in->logits) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (in->reserved0 != 0 || !null_reserved(in->reserved) || pool->reserved0 != 0 || !null_reserved(pool->reserved))
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (pool->pool_size < args->beam_size || pool->pool_size > DBS_CUDA_B200_MAX_POOL) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!pool->parents || !pool->tokens || !pool->lengths || !pool->from_logprob) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (pool->grad_relaxed_weights &&
        (!pool->relaxed_weights || !std::isfinite(pool->soft_topk_temperature) || !(pool->soft_topk_temperature > 0.0f)))
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    BackwardParams p = backward_params(*args);
    p.parents = in->parents;
    p.tokens = in->tokens;
    p.lengths = in->lengths;
    p.from_logprob = in->from_logprob;
    p.g_final = in->grad_final_scores;
    p.g_final_raw = in->grad_final_raw_scores;
    p.g_scores = in->grad_scores;
    p.g_raw = in->grad_raw_scores;
    p.grad = grad_inputs;
    p.P = pool->pool_size;
    p.pool_parents = pool->parents;
    p.pool_tokens = pool->tokens;
    p.pool_lengths = pool->lengths;
    p.pool_from = pool->from_logprob;
    p.relaxed = pool->relaxed_weights;
    p.g_relaxed = pool->grad_relaxed_weights;
    p.g_pool_scores = pool->grad_pool_scores;
    p.g_pool_raw = pool->grad_pool_raw_scores;
    p.soft_temp = pool->soft_topk_temperature;
    if (launch_backward(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return close_call(stream, nullptr);
}

// The dense gradient of dbs_cuda_backward_dense, with the selected-beam weights term when
// w_sel / g_wsel are given.
static int backward_dense(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in, const float* w_sel,
                          const float* g_wsel, float sel_temp, void* grad_inputs, int grad_type, void* workspace,
                          int64_t workspace_bytes, void* stream_ptr) {
    if (!valid_args(args) || !in || !grad_inputs || !valid_dtype(grad_type)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!in->parents || !in->tokens || !in->lengths || !in->from_logprob) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (in->reserved0 != 0 || in->reserved[0] || in->reserved[1] || in->reserved[2] || in->reserved[3]) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (in->logits && (!in->row_lse || !valid_dtype(in->logits_type))) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const DBSCudaDecodeArgs& a = *args;
    BackwardParams p = backward_params(a);
    p.parents = in->parents;
    p.tokens = in->tokens;
    p.lengths = in->lengths;
    p.from_logprob = in->from_logprob;
    p.g_final = in->grad_final_scores;
    p.g_final_raw = in->grad_final_raw_scores;
    p.g_scores = in->grad_scores;
    p.g_raw = in->grad_raw_scores;
    p.w_sel = w_sel;
    p.g_wsel = g_wsel;
    p.sel_temp = sel_temp;
    const WorkArea ws = work_area(workspace, workspace_bytes, backward_ws_bytes(a), stream);
    if (ws.status != DBS_CUDA_STATUS_OK) return ws.status;
    p.draws = ws.at<float>(0);
    const size_t slots = static_cast<size_t>(a.batch_size) * a.steps * a.beam_size;
    if (cudaMemsetAsync(p.draws, 0, slots * sizeof(float), stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (launch_backward(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    const int vec = (reinterpret_cast<uintptr_t>(grad_inputs) % 16 == 0) &&
                    (!in->logits || reinterpret_cast<uintptr_t>(in->logits) % 16 == 0);
    if (launch_dense_grad(p, in->logits_type, in->logits, in->row_lse, grad_type, grad_inputs, vec,
                          sm_count_of_current_device(), stream) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, nullptr);
}

DBS_CUDA_EXPORT int dbs_cuda_backward_dense(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                            void* grad_inputs, int grad_type, void* workspace, int64_t workspace_bytes,
                                            void* stream) {
    return backward_dense(args, in, nullptr, nullptr, 1.0f, grad_inputs, grad_type, workspace, workspace_bytes, stream);
}

DBS_CUDA_EXPORT int dbs_cuda_backward_selected(const DBSCudaDecodeArgs* args, const DBSCudaBackwardInputs* in,
                                               const float* selected_weights, const float* grad_selected_weights,
                                               float temperature, void* grad_inputs, int grad_type, void* workspace,
                                               int64_t workspace_bytes, void* stream) {
    if (!selected_weights || !grad_selected_weights || !std::isfinite(temperature) || !(temperature > 0.0f)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    return backward_dense(args, in, selected_weights, grad_selected_weights, temperature, grad_inputs, grad_type,
                          workspace, workspace_bytes, stream);
}

DBS_CUDA_EXPORT int dbs_cuda_selected_weights(const DBSCudaDecodeArgs* args, const float* scores, float temperature,
                                              float* weights, void* stream_ptr) {
    if (!valid_args(args) || !scores || !weights || !std::isfinite(temperature) || !(temperature > 0.0f)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const int64_t rows = static_cast<int64_t>(args->batch_size) * args->steps;
    if (launch_selected_weights(rows, args->beam_size, scores, temperature, weights, stream) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, nullptr);
}

DBS_CUDA_EXPORT int dbs_cuda_b200_wait_selftest(int64_t timeout_ns, int32_t* words, void* stream_ptr) {
    if (!words || timeout_ns < 100000 || timeout_ns > 1000000000) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    // words[0..1]: the waits' results; words[2]: the error word; words[3]: the flag nothing sets.
    if (cudaMemsetAsync(words, 0, 4 * sizeof(int32_t), stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    DecodeParams p;
    std::memset(&p, 0, sizeof p);
    p.timeout_ns = static_cast<unsigned long long>(timeout_ns);
    p.error = words + 2;
    if (launch_wait_selftest(p, words + 3, words, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    int32_t e = 0;
    if (cudaMemcpy(&e, words + 2, sizeof e, cudaMemcpyDeviceToHost) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return e == 0 ? DBS_CUDA_STATUS_OK : DBS_CUDA_STATUS_LAUNCH_FAILED;
}

DBS_CUDA_EXPORT int dbs_cuda_advance_prefixes(int batch_size, int beam_size, int step, int prefix_stride,
                                              const int32_t* parents, const int32_t* tokens,
                                              const uint8_t* from_logprob, const int32_t* prefixes_in,
                                              int32_t* prefixes_out, const float* raw_scores, const uint8_t* finished,
                                              uint8_t* any_live, void* stream_ptr) {
    if (batch_size < 1 || beam_size < 1 || beam_size > DBS_CUDA_MAX_BEAM || step < 0 || prefix_stride <= step) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (!parents || !tokens || !from_logprob || !prefixes_out || (step > 0 && !prefixes_in)) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (any_live && (!raw_scores || !finished)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (prefixes_in == prefixes_out && step > 0) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (launch_advance_prefixes(batch_size, beam_size, step, prefix_stride, parents, tokens, from_logprob, prefixes_in,
                                prefixes_out, raw_scores, finished, any_live, sm_count_of_current_device(),
                                stream) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, nullptr);
}

DBS_CUDA_EXPORT int dbs_cuda_backward(const DBSCudaDecodeArgs* args, const int32_t* parents, const int32_t* tokens,
                                      const int32_t* lengths, const uint8_t* from_logprob,
                                      const float* grad_final_scores, float* grad_log_probs, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
    if (!valid_args(args) || !parents || !tokens || !lengths || !from_logprob || !grad_final_scores || !grad_log_probs) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    DBSCudaBackwardInputs in;
    std::memset(&in, 0, sizeof in);
    in.parents = parents;
    in.tokens = tokens;
    in.lengths = lengths;
    in.from_logprob = from_logprob;
    in.grad_final_scores = grad_final_scores;
    return dbs_cuda_backward_ex(args, &in, grad_log_probs, workspace, workspace_bytes, stream);
}

DBS_CUDA_EXPORT int dbs_cuda_length_penalty(const int32_t* lengths, int64_t count, float alpha, float* out,
                                            void* stream_ptr) {
    if (count < 0 || (count > 0 && (!lengths || !out)) || !std::isfinite(alpha) || alpha < 0.0f) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (count == 0) return DBS_CUDA_STATUS_OK;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (launch_length_penalty(lengths, count, alpha, out, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return close_call(stream, nullptr);
}

DBS_CUDA_EXPORT int dbs_cuda_path_gradient(const DBSCudaDecodeArgs* args, const int32_t* parents,
                                           const int32_t* tokens, const int32_t* lengths, const uint8_t* from_logprob,
                                           const float* grad_final_scores, float* draws, void* stream_ptr) {
    if (!valid_args(args) || !parents || !tokens || !lengths || !from_logprob || !grad_final_scores || !draws) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const DBSCudaDecodeArgs& a = *args;
    const size_t slots = static_cast<size_t>(a.batch_size) * a.steps * a.beam_size;
    if (cudaMemsetAsync(draws, 0, slots * sizeof(float), stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    BackwardParams p = backward_params(a);
    p.parents = parents;
    p.tokens = tokens;
    p.lengths = lengths;
    p.from_logprob = from_logprob;
    p.g_final = grad_final_scores;
    p.draws = draws;
    if (launch_backward(p, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return close_call(stream, nullptr);
}

// ---------------------------------------------------------------------------
// Additions of this engine (include/dbs_cuda_b200.h)
// ---------------------------------------------------------------------------

DBS_CUDA_EXPORT int dbs_cuda_backtrack(const DBSCudaDecodeArgs* args, const int32_t* tokens, const int32_t* parents,
                                       int64_t* sequences, void* stream_ptr) {
    if (!valid_args(args) || !tokens || !parents || !sequences) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const DBSCudaDecodeArgs& a = *args;
    if (launch_backtrack(a.batch_size, a.steps, a.beam_size, tokens, parents, a.steps_per_example, sequences, stream) !=
        cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, nullptr);
}

DBS_CUDA_EXPORT int dbs_cuda_b200_abi_version(void) { return DBS_CUDA_B200_ABI_VERSION; }

DBS_CUDA_EXPORT int dbs_cuda_vshard_plan(const DBSCudaDecodeArgs* args, int from_logits, int world_size, int rank,
                                         int shard_list_len, DBSCudaVocabShardPlan* plan) {
    if (!plan) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    DBSCudaVocabShardPlan pl;
    if (!vshard_plan_fill(args, from_logits, world_size, rank, shard_list_len, pl)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    *plan = pl;
    return DBS_CUDA_STATUS_OK;
}

DBS_CUDA_EXPORT int dbs_cuda_vshard_scan(const DBSCudaVocabShardCall* call, void* stream_ptr) {
    VShardParams q;
    int rc = vshard_setup(call, q);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const DBSCudaDecodeArgs& a = *call->args;
    const DecodeLayout L = make_layout(a, false, true);
    rc = validate_per_example(q.d, a, reinterpret_cast<int32_t*>(static_cast<char*>(call->buffers.workspace) + L.status),
                              stream);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    const size_t kw = static_cast<size_t>((a.beam_size + 31) / 32);
    if (launch_init(q.d, stream) != cudaSuccess ||
        cudaMemsetAsync(q.resume, 0, sizeof(int32_t) * a.batch_size, stream) != cudaSuccess ||
        cudaMemsetAsync(q.stalled, 0, sizeof(uint32_t) * kw * a.batch_size, stream) != cudaSuccess ||
        launch_vshard_scan(q, call->data_type, stream, sm_count_of_current_device()) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, q.d.error);
}

DBS_CUDA_EXPORT int dbs_cuda_vshard_lanes(const DBSCudaVocabShardCall* call, void* stream_ptr) {
    VShardParams q;
    const int rc = vshard_setup(call, q);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    if (!call->from_logits) return DBS_CUDA_STATUS_OK;  // log-probs need no logsumexp
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (launch_vshard_lanes(q, call->data_type, stream, sm_count_of_current_device()) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, q.d.error);
}

DBS_CUDA_EXPORT int dbs_cuda_vshard_merge(const DBSCudaVocabShardCall* call, void* stream_ptr) {
    VShardParams q;
    const int rc = vshard_setup(call, q);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (launch_vshard_merge(q, call->from_logits != 0, stream, sm_count_of_current_device()) != cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, q.d.error);
}

DBS_CUDA_EXPORT int dbs_cuda_vshard_select(const DBSCudaVocabShardCall* call, void* stream_ptr) {
    VShardParams q;
    const int rc = vshard_setup(call, q);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    if (!call->outputs.final_scores) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (launch_vshard_select(q, call->from_logits != 0, stream) != cudaSuccess) return DBS_CUDA_STATUS_LAUNCH_FAILED;
    return close_call(stream, q.d.error);
}

DBS_CUDA_EXPORT int dbs_cuda_vshard_rescan(const DBSCudaVocabShardCall* call, void* stream_ptr) {
    VShardParams q;
    const int rc = vshard_setup(call, q);
    if (rc != DBS_CUDA_STATUS_OK) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (launch_vshard_rescan(q, call->data_type, call->from_logits != 0, stream, sm_count_of_current_device()) !=
        cudaSuccess) {
        return DBS_CUDA_STATUS_LAUNCH_FAILED;
    }
    return close_call(stream, q.d.error);
}

}  // extern "C"
