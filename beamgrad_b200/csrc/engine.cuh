// SPDX-License-Identifier: MIT
//
// Shared pieces of the B200 beam-search engine: launch parameters, bounded
// inter-CTA waits, and block-level reductions.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "dbs_cuda.h"
#include "dbs_cuda_b200.h"
#include "detmath.cuh"

namespace dbsb {

constexpr int kThreads = 256;          // threads per CTA of every row kernel (one per logsumexp lane)
constexpr int kWarps = kThreads / 32;
constexpr int kFastBeam = 16;          // largest beam of the register top-k path
constexpr int kConsCap = 512;          // constraint tokens kept in shared memory per row
constexpr int kSelectCap = 1024;       // largest beam of the generic select (DBS_CUDA_MAX_BEAM)

// Error codes written to the workspace error word (never a GPU trap).
constexpr int kErrNone = 0;
constexpr int kErrTimeout = 1;         // a bounded wait gave up

// Per-example settings (clamped into range; the host validates them first).
struct Meta {
    int steps;
    int beam;
    int eos;
    int min_length;
};

// Everything the decode kernels need. Passed by value (kernel parameter space).
struct DecodeParams {
    // problem
    int B, T, K, V;
    int eos, min_length;
    float alpha;
    int ngram;
    int penalise;
    float log_penalty;      // logf(repetition_penalty), computed on the host as the CPU decoder does
    int n_extra;            // extra EOS tokens (active for examples with EOS handling)
    int32_t extra[DBS_CUDA_MAX_EXTRA_EOS];
    const int32_t* steps_pe;
    const int32_t* beams_pe;
    const int32_t* eos_pe;
    const int32_t* minlen_pe;
    const uint8_t* banned;  // [V] or null
    // input rows
    const void* inputs;
    int step_api;           // 1: one step from a caller-owned state (T == 1)
    // beam state [B, K]
    float* raw;
    int32_t* len;
    uint8_t* ended;
    int32_t* last;          // token of each slot after the previous step (decode only)
    // prefixes for n-gram blocking / repetition penalty
    const int32_t* caller_prefix;  // step API: [B, K, prefix_stride]
    int prefix_stride;
    int32_t* prefix[2];            // decode: double-buffered [B, K, T]
    int32_t* prefix_len[2];        // decode: [B, K]
    // outputs
    DBSCudaDecodeOutputs out;
    float* row_lse;
    // scratch
    uint64_t* keys;         // [B, K, list_len] per-row candidate lists
    int list_len;
    uint32_t* arrive;       // [B] rows of the current step that finished
    int32_t* flag;          // [B] steps whose selection is published
    uint32_t* ticket;       // work-item counter
    int32_t* error;         // error word
    int staged;             // rows are staged in shared memory (from logits)
    int row_smem;           // bytes of the shared-memory row buffer
    unsigned long long timeout_ns;
    // chained decode (no inter-CTA waits): per-row records and per-step arrival counts
    int chain;              // 1: decode_chain_kernel runs this decode
    uint64_t* rkeys;        // [B, T, K, list_len] each row's best entries by x (x-keys)
    float* rlse;            // [B, T, K] each row's logsumexp (from logits)
    uint32_t* rinfo;        // [B, T, K] bit 0: NaN/+inf in the row; bits 8..: entries in rkeys
    uint32_t* count;        // [B, T] rows (and the previous step's selection) that arrived
    // packed-arithmetic constants (1.0f, 1.0f) and (-0.0f, -0.0f), supplied at run time
    uint64_t one2, nzero2;
};


// A vocabulary-sharded decode on rank `rank` of `world` (vshard.cu). Rank r holds the
// tokens v with (v mod 256) in [r * lanes, (r + 1) * lanes): shard entry i is token
// (i / lanes) * 256 + r * lanes + i mod lanes, so logsumexp lane j of the reference's
// fixed order lives whole on rank j / lanes. d describes the whole problem (V is the
// full vocabulary) and holds the decode state, the merged row records and the outputs.
struct VShardParams {
    DecodeParams d;
    int world, rank;
    int lanes, lanes_log2;     // lanes per rank (256 / world)
    int shard_v;               // tokens of this rank
    int shard_list;            // entries of a row record per rank
    int row_words;             // 64-bit words per row of the exchange buffer
    int key_off;               // word of the first record entry in an exchange row
    const void* shard;         // [B, T, K, shard_v]
    float* row_max;            // [B * T * K] this rank's row maxima, then (all-reduced) the rows'
    float* row_min;            // [B * T * K]
    uint64_t* pack;            // [rows, row_words]: info, lane sums (from logits), record
    const uint64_t* pack_all;  // [world, rows, row_words]
    int32_t* resume;           // [B] first step not yet selected (T: done)
    uint32_t* stalled;         // [B, ceil(K / 32)] rows of step resume[b] waiting for a rescan
    const int32_t* rescan_rows;  // [n_rescan] b * K + k
    const int32_t* rescan_slot;  // [B * K] position in rescan_rows or -1
    int n_rescan;
    uint64_t* rescan;            // [n_rescan, K]
    const uint64_t* rescan_all;  // [world, n_rescan, K]
    int cand_cap;                // select: candidate keys its shared-memory buffer holds (0: none)
};

// Everything the backward kernels need.
struct BackwardParams {
    int B, T, K, V;
    float alpha;
    const int32_t* steps_pe;
    const int32_t* beams_pe;
    const int32_t* parents;
    const int32_t* tokens;
    const int32_t* lengths;
    const uint8_t* from_logprob;
    const float* g_final;
    const float* g_final_raw;
    const float* g_scores;
    const float* g_raw;
    float* grad;    // dense [B, T, K, V] (+=), or null
    float* draws;   // per slot [B, T, K], or null
    const float* w_sel;   // selected-beam weights [B, T, K], or null
    const float* g_wsel;  // their gradient [B, T, K], or null
    float sel_temp;       // the weights' softmax temperature
    // Relaxed pool (P candidates per step), when pool gradients are given (P = 0: none).
    int P;
    const int32_t* pool_parents;  // [B, T, P]
    const int32_t* pool_tokens;
    const int32_t* pool_lengths;
    const uint8_t* pool_from;
    const float* relaxed;         // relaxed weights [B, T, P] (with g_relaxed)
    const float* g_relaxed;       // their gradient, or null
    const float* g_pool_scores;   // [B, T, P] or null
    const float* g_pool_raw;      // [B, T, P] or null
    float soft_temp;              // the relaxed weights' sigmoid temperature
};

__device__ __forceinline__ Meta load_meta(const DecodeParams& p, int b) {
    Meta m;
    m.steps = p.steps_pe ? p.steps_pe[b] : p.T;
    m.beam = p.beams_pe ? p.beams_pe[b] : p.K;
    m.eos = p.eos_pe ? p.eos_pe[b] : p.eos;
    m.min_length = p.minlen_pe ? p.minlen_pe[b] : p.min_length;
    m.steps = m.steps < 0 ? 0 : (m.steps > p.T ? p.T : m.steps);
    m.beam = m.beam < 0 ? 0 : (m.beam > p.K ? p.K : m.beam);
    if (m.eos < -1 || m.eos >= p.V) m.eos = -1;
    return m;
}

__device__ __forceinline__ bool is_eos(const DecodeParams& p, const Meta& m, int token) {
    if (m.eos < 0) return false;
    if (token == m.eos) return true;
    for (int i = 0; i < p.n_extra; ++i)
        if (p.extra[i] == token) return true;
    return false;
}

// ---------------------------------------------------------------------------
// Memory-model helpers for the per-example step hand-off between CTAs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ld_acquire(const int32_t* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(int32_t* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Waits until flag >= target; executed by all 32 lanes of one warp together
// (lane 0 reads, the warp follows its decision), so the warp never diverges
// around the spin. Bounded: after timeout_ns it records kErrTimeout and returns
// false; it also returns false as soon as another CTA recorded an error.
__device__ __forceinline__ bool wait_flag_warp(const DecodeParams& p, const int32_t* flag, int target) {
    const int lane = threadIdx.x & 31;
    unsigned long long start = 0;
    unsigned sleep = 32;
    for (int iter = 0;; ++iter) {
        int state = 0;  // 1 ready, 2 give up
        if (lane == 0) {
            if (ld_acquire(flag) >= target) {
                state = 1;
            } else if (ld_acquire(p.error) != kErrNone) {
                state = 2;
            } else {
                const unsigned long long now = global_ns();
                if (iter == 0) start = now;
                if (now - start > p.timeout_ns) {
                    atomicCAS(p.error, kErrNone, kErrTimeout);
                    state = 2;
                }
            }
        }
        state = __shfl_sync(0xffffffffu, state, 0);
        if (state == 1) return true;
        if (state == 2) return false;
        __nanosleep(sleep);
        if (sleep < 1024) sleep <<= 1;
    }
}

// ---------------------------------------------------------------------------
// Block-level helpers (kThreads threads).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v), m);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), m);
    return (static_cast<uint64_t>(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        const uint64_t o = shfl_xor_u64(v, m);
        v = o > v ? o : v;
    }
    return v;
}
__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// Block-wide barriers with per-thread arrival (the non-.aligned PTX forms).
// __syncthreads() is an aligned barrier, which assumes every warp arrives
// converged; a warp whose lanes diverged (one lane in a bounded spin on another
// CTA's flag, or in an atomic) can then be counted as arrived by its other
// lanes, and the block's barriers pair up across different program points.
// barrier.sync / barrier.red count threads, so every barrier of the engine
// goes through these.
__device__ __forceinline__ void block_sync() { asm volatile("barrier.sync 0;" ::: "memory"); }
__device__ __forceinline__ bool block_and(bool v) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.and.pred q, 0, p;\n selp.s32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(static_cast<unsigned>(v))
        : "memory");
    return r != 0;
}

// Global loads of data another CTA wrote during this launch: served by L2.
template <class T>
__device__ __forceinline__ T ld_cg(const T* p) {
    return __ldcg(p);
}

}  // namespace dbsb
