// SPDX-License-Identifier: MIT
//
// The relaxed pool of a decode (beamgrad 2.3.0 src/decoder.cpp:294-312, record_pool):
// for every step, the P = K * multiplier best candidates under the full candidate order,
// and optionally their relaxed top-K membership weights (soft_topk_inclusion,
// src/kernels_scalar.cpp:304-366). The pool is a function of the decode's trace: the
// state before step t is the trace at step t-1, so a separate launch after the decode
// rebuilds each step's candidates, one CTA per (example, step).
//
// Scope (as beamgrad's own torch estimator relaxed_topk, python/beamgrad/estimators.py:196):
// no n-gram blocking, no repetition penalty; banned tokens and the min-length EOS mask
// apply. Every operation is the reference's, in its order, so the pool and the weights
// are bit-identical to the CPU decoder's.
#include "decode_impl.cuh"

namespace dbsb {
namespace {

struct PoolParams {
    DecodeParams d;              // problem: B, T, K, V, eos, min_length, alpha, banned, inputs, steps_pe
    int P;                       // pool size
    const float* row_lse;        // [B, T, K] the decode's row logsumexp (from logits)
    const int32_t* parents;      // the decode's trace [B, T, K]
    const int32_t* tokens;
    const int32_t* lengths;
    const float* raw;
    const uint8_t* from_logprob;
    int32_t* pool_parents;       // [B, T, P] outputs (any may be null)
    int32_t* pool_tokens;
    int32_t* pool_lengths;
    float* pool_scores;
    float* pool_raw;
    uint8_t* pool_from;
    float* relaxed;              // [B, T, P] relaxed top-K weights, or null
    float temperature, tolerance;
    int max_iters;
};

// A candidate of the full order (src/common.hpp:269-276): score desc, raw desc, parent asc,
// token asc, length asc, expanded (from a log-prob) before carried forward.
struct PoolCand {
    float score, raw;
    int parent, token, length, from;
};

__device__ __forceinline__ bool cand_before(const PoolCand& a, const PoolCand& c) {
    if (a.score != c.score) return a.score > c.score;
    if (a.raw != c.raw) return a.raw > c.raw;
    if (a.parent != c.parent) return a.parent < c.parent;
    if (a.token != c.token) return a.token < c.token;
    if (a.length != c.length) return a.length < c.length;
    return a.from > c.from;
}

// sigmoid from the exact exponential (src/kernels_scalar.cpp:30-34).
__device__ __forceinline__ float sigmoid_exact(float x) {
    if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_nonpositive(-x)));
    const float e = exp_nonpositive(x);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

constexpr float kNegGuard = -1.0e30f;

// The weight of score x at offset theta: sigmoid((x - ref - theta) / temperature), 0 for
// empty slots.
__device__ __forceinline__ float pool_weight(float x, float ref, float offset, float temperature) {
    return x > kNegGuard ? sigmoid_exact(__fdiv_rn(__fsub_rn(__fsub_rn(x, ref), offset), temperature)) : 0.0f;
}

// Relaxed top-k membership: sigmoid((score - theta) / temperature) with theta bisected so
// that the weights sum to target_k (src/kernels_scalar.cpp:304-366, operation for operation).
// One warp: the lanes evaluate the sigmoids (into w[], P floats of shared memory), lane 0 adds
// them in index order (the reference's sequential sum; a skipped empty slot adds nothing,
// and adding +0 to a sum of non-negative terms leaves it unchanged), every lane follows the
// same bisection from the broadcast sum.
__device__ void soft_topk_inclusion_warp(const float* s, float* w, float* out, int n, int target_k, float temperature,
                                         float tolerance, int max_iters) {
    const int lane = threadIdx.x & 31;
    int active = 0;
    float min_s = f_inf(), max_s = f_ninf();
    for (int i = lane; i < n; i += 32) {
        if (s[i] > kNegGuard) {
            ++active;
            min_s = fminf(min_s, s[i]);
            max_s = fmaxf(max_s, s[i]);
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        active += __shfl_xor_sync(0xffffffffu, active, o);
        min_s = fminf(min_s, __shfl_xor_sync(0xffffffffu, min_s, o));
        max_s = fmaxf(max_s, __shfl_xor_sync(0xffffffffu, max_s, o));
    }
    if (active == 0 || target_k <= 0) {
        for (int i = lane; i < n; i += 32) out[i] = 0.0f;
        return;
    }
    if (target_k >= active) {
        for (int i = lane; i < n; i += 32) out[i] = s[i] > kNegGuard ? 1.0f : 0.0f;
        return;
    }
    const float ref = max_s;
    float lo = __fsub_rn(__fsub_rn(min_s, ref), __fmul_rn(80.0f, temperature));
    float hi = __fmul_rn(80.0f, temperature);
    const float bracket = __fmul_rn(tolerance, temperature);
    constexpr float kFourEps = 4.0f * 1.1920928955078125e-07f;  // 4 x FLT_EPSILON, exact
    for (int it = 0; it < max_iters; ++it) {
        const float mid = __fmul_rn(0.5f, __fadd_rn(lo, hi));
        for (int i = lane; i < n; i += 32) w[i] = pool_weight(s[i], ref, mid, temperature);
        __syncwarp();
        float sum = 0.0f;
        if (lane == 0)
            for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, w[i]);
        sum = __shfl_sync(0xffffffffu, sum, 0);
        __syncwarp();
        const float err = __fsub_rn(sum, static_cast<float>(target_k));
        const float ulps = __fmul_rn(kFourEps, fabsf(mid));
        if (fabsf(err) <= tolerance || __fsub_rn(hi, lo) <= fmaxf(bracket, ulps)) {
            lo = hi = mid;
            break;
        }
        if (err > 0.0f) lo = mid;
        else hi = mid;
    }
    const float offset = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    for (int i = lane; i < n; i += 32) out[i] = pool_weight(s[i], ref, offset, temperature);
}

constexpr int kPoolBuf = 2048;  // compacted candidates at or above the thread-maximum bound

// The largest entry of a row among those the calling thread owns (for_chunks' assignment),
// NaN ignored; -inf when there is none. Four 16-byte loads in flight per thread.
template <int DT>
__device__ float thread_row_max(const char* row, const RowSplit& rs) {
    using E = Elem<DT>;
    const int tid = threadIdx.x;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    auto chunk_max = [](const uint4& a) -> float {
        if constexpr (E::kBytes == 2) {
            const uint32_t m2 = h2_max<DT>(h2_max<DT>(a.x, a.y), h2_max<DT>(a.z, a.w));
            return fmaxf(h2_lo<DT>(m2), h2_hi<DT>(m2));
        } else {
            return fmaxf(fmaxf(__uint_as_float(a.x), __uint_as_float(a.y)), fmaxf(__uint_as_float(a.z), __uint_as_float(a.w)));
        }
    };
    float top = f_ninf();
    int c = tid;
    for (; c + 3 * kThreads < rs.nvec; c += 4 * kThreads) {
        uint4 a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = ld_stream_v4(body + static_cast<size_t>(c + u * kThreads) * 16);
#pragma unroll
        for (int u = 0; u < 4; ++u) top = fmaxf(top, chunk_max(a[u]));
    }
    for (; c < rs.nvec; c += kThreads) top = fmaxf(top, chunk_max(ld_stream_v4(body + static_cast<size_t>(c) * 16)));
    if (tid < rs.n_ends()) top = fmaxf(top, load_elem<DT>(row, rs.end_entry(tid)));
    return top;
}

// hit(x, v) for every entry the calling thread owns with x >= xf; a 16-byte chunk is
// unpacked only when its largest entry reaches xf. Four loads in flight per thread.
template <int DT, class Hit>
__device__ void scan_row_above(const char* row, const RowSplit& rs, float xf, Hit&& hit) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    const int tid = threadIdx.x;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    constexpr uint32_t kNegFill = E::kBytes == 2 ? h2_ninf<DT>() : 0xff800000u;
    for (int c0 = tid; c0 < rs.nvec; c0 += 4 * kThreads) {
        uint4 a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = c0 + u * kThreads;
            a[u] = c < rs.nvec ? ld_stream_v4(body + static_cast<size_t>(c) * 16)
                               : make_uint4(kNegFill, kNegFill, kNegFill, kNegFill);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float top;
            if constexpr (E::kBytes == 2) {
                const uint32_t m2 = h2_max<DT>(h2_max<DT>(a[u].x, a[u].y), h2_max<DT>(a[u].z, a[u].w));
                top = fmaxf(h2_lo<DT>(m2), h2_hi<DT>(m2));
            } else {
                top = fmaxf(fmaxf(__uint_as_float(a[u].x), __uint_as_float(a[u].y)),
                            fmaxf(__uint_as_float(a[u].z), __uint_as_float(a[u].w)));
            }
            if (top >= xf) {
                float x[PER];
                unpack16<DT>(a[u], x);
                const int v0 = rs.head + (c0 + u * kThreads) * PER;
#pragma unroll
                for (int j = 0; j < PER; ++j)
                    if (x[j] >= xf) hit(x[j], v0 + j);
            }
        }
    }
    if (tid < rs.n_ends()) {
        const int v = rs.end_entry(tid);
        const float x = load_elem<DT>(row, v);
        if (x >= xf) hit(x, v);
    }
}

template <int DT, bool LOGITS>
__global__ void __launch_bounds__(kThreads) pool_kernel(const __grid_constant__ PoolParams q) {
    __shared__ RowShared sh;
    __shared__ float s_raw[DBS_CUDA_MAX_BEAM];
    __shared__ int32_t s_len[DBS_CUDA_MAX_BEAM];
    __shared__ int32_t s_last[DBS_CUDA_MAX_BEAM];
    __shared__ uint8_t s_kind[DBS_CUDA_MAX_BEAM];  // 0 dead, 1 extends (row read), 2 carried forward
    __shared__ int n_carry;
    extern __shared__ __align__(16) unsigned char dyn[];
    const DecodeParams& p = q.d;
    const int P = q.P, K = p.K, V = p.V;
    uint64_t* keys = reinterpret_cast<uint64_t*>(dyn);        // [P] scanned candidates' keys
    uint64_t* buf = keys + P;                                  // [kPoolBuf] compacted candidates
    PoolCand* cand = reinterpret_cast<PoolCand*>(buf + kPoolBuf);  // [P + K] scanned then carried
    float* pscore = reinterpret_cast<float*>(cand + P + K);    // [P] the pool's scores, pool order
    float* wtmp = pscore + P;                                  // [P] bisection scratch
    __shared__ uint64_t tmax_s[kThreads];
    __shared__ uint64_t bound_s;
    __shared__ int n_buf;
    const int b = blockIdx.x / p.T, t = blockIdx.x - (blockIdx.x / p.T) * p.T;
    const int tid = threadIdx.x;
    const Meta m = load_meta(p, b);
    const int64_t obase = (static_cast<int64_t>(b) * p.T + t) * P;
    auto write = [&](int i, const PoolCand& c) {
        if (q.pool_parents) q.pool_parents[obase + i] = c.parent;
        if (q.pool_tokens) q.pool_tokens[obase + i] = c.token;
        if (q.pool_lengths) q.pool_lengths[obase + i] = c.length;
        if (q.pool_scores) q.pool_scores[obase + i] = c.score;
        if (q.pool_raw) q.pool_raw[obase + i] = c.raw;
        if (q.pool_from) q.pool_from[obase + i] = static_cast<uint8_t>(c.from);
    };
    const PoolCand empty{f_ninf(), f_ninf(), -1, -1, 0, 0};
    if (t >= m.steps) {  // steps past the example's length: empty slots
        for (int i = tid; i < P; i += kThreads) {
            write(i, empty);
            if (q.relaxed) q.relaxed[obase + i] = 0.0f;
        }
        return;
    }
    // The beams entering step t: the trace at step t-1 (at t = 0, beam 0 alone, empty).
    if (tid == 0) n_carry = 0;
    for (int k = tid; k < K; k += kThreads) {
        uint8_t kind = 0;
        float raw = f_ninf();
        int len = 0, last = -1;
        if (t == 0) {
            if (k == 0) kind = 1, raw = 0.0f;
        } else if (k < m.beam) {
            const int64_t s = (static_cast<int64_t>(b) * p.T + t - 1) * K + k;
            if (q.parents[s] >= 0 && f_finite(q.raw[s])) {
                raw = q.raw[s];
                len = q.lengths[s];
                last = q.tokens[s];
                const bool ended = m.eos >= 0 && (q.from_logprob[s] == 0 || last == m.eos);
                kind = ended ? 2 : 1;
            }
        }
        s_raw[k] = raw;
        s_len[k] = len;
        s_last[k] = last;
        s_kind[k] = kind;
    }
    block_sync();
    // Scanned candidates: every eligible entry of every row read at this step; the P best by
    // (raw desc, parent * V + token asc), which is the full order among them (they extend
    // beams of one length).
    const char* in = static_cast<const char*>(p.inputs);
    const bool mask_eos = m.eos >= 0;
    auto gen = [&](int i) -> uint64_t {
        const int k = i / V, v = i - k * V;
        if (s_kind[k] != 1) return 0;
        if (p.banned && p.banned[v]) return 0;
        if (mask_eos && v == m.eos && s_len[k] + 1 < m.min_length) return 0;
        const int64_t row = (static_cast<int64_t>(b) * p.T + t) * K + k;
        const float x = load_elem<DT>(in + row * static_cast<int64_t>(V) * Elem<DT>::kBytes, v);
        const float lp = LOGITS ? __fsub_rn(x, q.row_lse[row]) : x;
        if (!(lp < f_inf()) || lp == f_ninf()) return 0;
        return make_key(__fadd_rn(s_raw[k], lp), static_cast<uint32_t>(i));
    };
    // f(key) for every candidate key the calling thread owns: the rows read at this step,
    // streamed in 16-byte chunks (the same candidates and keys as gen, in another order).
    auto scan_keys = [&](auto&& f) {
        for (int k = 0; k < K; ++k) {
            if (s_kind[k] != 1) continue;
            const int64_t row = (static_cast<int64_t>(b) * p.T + t) * K + k;
            const char* src = in + row * static_cast<int64_t>(V) * Elem<DT>::kBytes;
            const RowSplit rs = RowSplit::of<Elem<DT>::kBytes>(src, V);
            const float lse = LOGITS ? q.row_lse[row] : 0.0f;
            const float base = s_raw[k];
            const bool eos_masked = mask_eos && s_len[k] + 1 < m.min_length;
            const uint32_t first = static_cast<uint32_t>(k) * static_cast<uint32_t>(V);
            for_chunks<DT>(src, rs, false, [&](float x, int v) {
                if (p.banned && p.banned[v]) return;
                if (eos_masked && v == m.eos) return;
                const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                if (!(lp < f_inf()) || lp == f_ninf()) return;
                f(make_key(__fadd_rn(base, lp), first + static_cast<uint32_t>(v)));
            });
        }
    };
    // The P best keys lie at or above the P-th largest thread maximum (P threads each own a
    // key that reaches it); when P <= 256 they are compacted first, and the select runs over
    // the compacted keys (the whole candidate set when too many reach the bound).
    const int n_all = K * V;
    auto put = [&](int pos, uint64_t key) { keys[pos] = key; };
    int n_scanned;
    bool compacted = false;
    if (P <= kThreads) {
        // Pass 1: a lower bound on each thread's best key. Without banned tokens it comes from
        // the thread's largest entry of each row read (packed maxima; no bound from a row
        // whose masked EOS the thread owns): the key of that entry's raw score with the
        // lowest index part. With banned tokens, the thread's best key itself.
        uint64_t lb = 0;
        if (!p.banned) {
            for (int k = 0; k < K; ++k) {
                if (s_kind[k] != 1) continue;
                const int64_t row = (static_cast<int64_t>(b) * p.T + t) * K + k;
                const char* src = in + row * static_cast<int64_t>(V) * Elem<DT>::kBytes;
                const RowSplit rs = RowSplit::of<Elem<DT>::kBytes>(src, V);
                if (mask_eos && s_len[k] + 1 < m.min_length && rs.owns(m.eos)) continue;
                const float top = thread_row_max<DT>(src, rs);
                if (!(top < f_inf()) || top == f_ninf()) continue;
                const float lp = LOGITS ? __fsub_rn(top, q.row_lse[row]) : top;
                if (!(lp < f_inf()) || lp == f_ninf()) continue;
                const uint64_t key = make_key(__fadd_rn(s_raw[k], lp), 0xffffffffu);
                lb = key > lb ? key : lb;
            }
        } else {
            scan_keys([&](uint64_t key) { lb = key > lb ? key : lb; });
        }
        tmax_s[tid] = lb;
        if (tid == 0) {
            bound_s = 0;
            n_buf = 0;
        }
        block_sync();
        // The P-th largest bound (ties allowed): P threads each own a key at or above it.
        int above = 0, atleast = 0;
        for (int j = 0; j < kThreads; ++j) {
            const uint64_t o = tmax_s[j];
            above += o > lb ? 1 : 0;
            atleast += o >= lb ? 1 : 0;
        }
        if (lb != 0 && above < P && atleast >= P) bound_s = lb;
        block_sync();
        const uint64_t bound = bound_s;
        if (bound != 0) {
            // Pass 2: the keys at or above the bound, i.e. raw >= rb; x >= xf is necessary for
            // that (raw is non-decreasing in x, and xf is the smallest x whose raw reaches rb).
            const float rb = key_raw(bound);
            for (int k = 0; k < K; ++k) {
                if (s_kind[k] != 1) continue;
                const int64_t row = (static_cast<int64_t>(b) * p.T + t) * K + k;
                const char* src = in + row * static_cast<int64_t>(V) * Elem<DT>::kBytes;
                const RowSplit rs = RowSplit::of<Elem<DT>::kBytes>(src, V);
                const float lse = LOGITS ? q.row_lse[row] : 0.0f;
                const float base = s_raw[k];
                const bool eos_masked = mask_eos && s_len[k] + 1 < m.min_length;
                const uint32_t first = static_cast<uint32_t>(k) * static_cast<uint32_t>(V);
                auto raw_of = [&](float x) { return __fadd_rn(base, LOGITS ? __fsub_rn(x, lse) : x); };
                const float est = LOGITS ? __fadd_rn(__fsub_rn(rb, base), lse) : __fsub_rn(rb, base);
                const float xf = smallest_x_reaching(est, rb, raw_of);
                scan_row_above<DT>(src, rs, xf, [&](float x, int v) {
                    if (p.banned && p.banned[v]) return;
                    if (eos_masked && v == m.eos) return;
                    const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                    if (!(lp < f_inf()) || lp == f_ninf()) return;
                    const uint64_t key = make_key(__fadd_rn(base, lp), first + static_cast<uint32_t>(v));
                    if (key >= bound) {
                        const int pos = atomicAdd(&n_buf, 1);
                        if (pos < kPoolBuf) buf[pos] = key;
                    }
                });
            }
            block_sync();
            const int nb = n_buf;
            if (nb <= kPoolBuf) {
                n_scanned = block_select(sh, [&](int i) { return buf[i]; }, nb, P, put);
                compacted = true;
            }
        }
    }
    if (!compacted) n_scanned = block_select(sh, gen, n_all, P, put);
    // Full candidates: the scanned ones, then the carried-forward finished beams.
    for (int i = tid; i < n_scanned; i += kThreads) {
        const uint64_t key = keys[i];
        const uint32_t idx = key_index(key);
        const int k = static_cast<int>(idx / static_cast<uint32_t>(V));
        const float raw = key_raw(key);
        const float inv = __fdiv_rn(1.0f, gnmt_penalty(s_len[k] + 1, p.alpha));
        cand[i] = PoolCand{__fmul_rn(raw, inv), raw, k, static_cast<int>(idx - static_cast<uint32_t>(k) * V), s_len[k] + 1, 1};
    }
    for (int k = tid; k < K; k += kThreads) {
        if (s_kind[k] != 2) continue;
        const int j = n_scanned + atomicAdd(&n_carry, 1);
        const int l = s_len[k] > 1 ? s_len[k] : 1;
        cand[j] = PoolCand{__fdiv_rn(s_raw[k], gnmt_penalty(l, p.alpha)), s_raw[k], k, s_last[k], s_len[k], 0};
    }
    block_sync();
    const int n = n_scanned + n_carry;
    // Rank by counting (every candidate is unique under the full order); the best P are the pool.
    for (int i = tid; i < n; i += kThreads) {
        int rank = 0;
        for (int j = 0; j < n; ++j) rank += cand_before(cand[j], cand[i]) ? 1 : 0;
        if (rank < P) {
            write(rank, cand[i]);
            pscore[rank] = cand[i].score;
        }
    }
    for (int i = n + tid; i < P; i += kThreads) {
        write(i, empty);
        pscore[i] = f_ninf();
    }
    if (q.relaxed) {
        block_sync();
        if (tid < 32) soft_topk_inclusion_warp(pscore, wtmp, q.relaxed + obase, P, K, q.temperature, q.tolerance, q.max_iters);
    }
}

template <int DT, bool LOGITS>
cudaError_t launch_pool_as(const PoolParams& q, cudaStream_t stream) {
    const size_t dyn = static_cast<size_t>(q.P) * 8 + static_cast<size_t>(kPoolBuf) * 8 +
                       static_cast<size_t>(q.P + q.d.K) * sizeof(PoolCand) + static_cast<size_t>(q.P) * 8;
    auto kernel = pool_kernel<DT, LOGITS>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e != cudaSuccess) return e;
    kernel<<<static_cast<unsigned>(static_cast<int64_t>(q.d.B) * q.d.T), kThreads, dyn, stream>>>(q);
    return cudaGetLastError();
}

}  // namespace

// Entry from the C ABI (api.cu).
cudaError_t launch_relaxed_pool(const DecodeParams& d, int dtype, bool logits, int P, const float* row_lse,
                                const int32_t* parents, const int32_t* tokens, const int32_t* lengths, const float* raw,
                                const uint8_t* from_logprob, int32_t* pool_parents, int32_t* pool_tokens,
                                int32_t* pool_lengths, float* pool_scores, float* pool_raw, uint8_t* pool_from,
                                float* relaxed, float temperature, float tolerance, int max_iters, cudaStream_t stream) {
    PoolParams q{};
    q.d = d;
    q.P = P;
    q.row_lse = row_lse;
    q.parents = parents;
    q.tokens = tokens;
    q.lengths = lengths;
    q.raw = raw;
    q.from_logprob = from_logprob;
    q.pool_parents = pool_parents;
    q.pool_tokens = pool_tokens;
    q.pool_lengths = pool_lengths;
    q.pool_scores = pool_scores;
    q.pool_raw = pool_raw;
    q.pool_from = pool_from;
    q.relaxed = relaxed;
    q.temperature = temperature;
    q.tolerance = tolerance;
    q.max_iters = max_iters;
    if (dtype == DBS_CUDA_DTYPE_F32) return logits ? launch_pool_as<0, true>(q, stream) : launch_pool_as<0, false>(q, stream);
    if (dtype == DBS_CUDA_DTYPE_F16) return logits ? launch_pool_as<1, true>(q, stream) : launch_pool_as<1, false>(q, stream);
    return logits ? launch_pool_as<2, true>(q, stream) : launch_pool_as<2, false>(q, stream);
}

}  // namespace dbsb
