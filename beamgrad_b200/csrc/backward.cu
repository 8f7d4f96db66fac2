// SPDX-License-Identifier: MIT
//
// Companion kernels of the decode: the surrogate-gradient backward (per-slot
// path gradients, optionally scattered into a dense [B, T, K, V] gradient),
// the log-softmax correction of rows decoded from logits, the GNMT length
// penalty, and backtracking of the final beams' token sequences.
//
// Backward semantics (beamgrad 2.3.0 src/decoder.cpp:186-304, run_backward
// without a relaxed pool): walking an example's steps from the last to the
// first, slot k of step t with parent q >= 0 gets
//     drank = g_scores[t, k] (+ g_final[k] at the last step)
//     draw  = next[k] + drank * (1 / penalty(max(len, 1))) + g_raw[t, k]
//             (+ g_final_raw[k] at the last step)
// and, when draw != 0, adds draw to prev[q] (children summed in slot order,
// starting from 0) and, when the slot consumed an input entry, to entry
// (t, q, token). Every slot of a step has a distinct entry, so the dense
// update needs no atomics and the result is deterministic.
#include <cuda_bf16.h>

#include <algorithm>

#include "engine.cuh"

namespace dbsb {



// Ascending bitonic sort of n (a power of two, <= DBS_CUDA_MAX_BEAM) 32-bit keys in shared
// memory by the whole CTA.
__device__ void bitonic_sort_u32(uint32_t* keys, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n; i += kThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const uint32_t a = keys[i], c = keys[j];
                    if ((a > c) == up) {
                        keys[i] = c;
                        keys[j] = a;
                    }
                }
            }
            block_sync();
        }
    }
}

constexpr int kPoolCap = DBS_CUDA_B200_MAX_POOL;  // pool candidates per step

// Beams above this many: parents find their children through one sort per step instead of
// each parent scanning every slot (without pool gradients).
constexpr int kScanParentsUpTo = 64;

// One CTA per example; its beams' running gradients live in shared memory.
__global__ void __launch_bounds__(kThreads) backward_kernel(const __grid_constant__ BackwardParams p) {
    __shared__ float next_g[DBS_CUDA_MAX_BEAM];
    __shared__ float prev_g[DBS_CUDA_MAX_BEAM];
    __shared__ float draw_s[DBS_CUDA_MAX_BEAM];
    __shared__ int32_t par_s[DBS_CUDA_MAX_BEAM];
    __shared__ uint32_t child_s[DBS_CUDA_MAX_BEAM];  // (parent << 11 | slot), sorted
    __shared__ float pdraw_s[kPoolCap];               // pool candidates' raw-score gradients
    __shared__ int32_t ppar_s[kPoolCap];              // and parents (-1: none)
    __shared__ float pool_center_s;
    __shared__ int pool_relaxed_s;
    const int b = blockIdx.x;
    const int tid = threadIdx.x;
    const int K = p.K;
    int steps = p.steps_pe ? p.steps_pe[b] : p.T;
    int Kb = p.beams_pe ? p.beams_pe[b] : K;
    steps = steps < 0 ? 0 : (steps > p.T ? p.T : steps);
    Kb = Kb < 0 ? 0 : (Kb > K ? K : Kb);
    __shared__ float wdot_s;
    for (int k = tid; k < Kb; k += kThreads) next_g[k] = 0.0f;
    block_sync();
    for (int t = steps - 1; t >= 0; --t) {
        const bool last = t == steps - 1;
        const int64_t base = (static_cast<int64_t>(b) * p.T + t) * K;
        if (p.g_wsel) {
            // dot(w, gw) over the step's K slots in slot order (src/kernels_scalar.cpp:271-275).
            if (tid == 0) {
                float s = 0.0f;
                for (int k = 0; k < K; ++k) s = __fadd_rn(s, __fmul_rn(p.w_sel[base + k], p.g_wsel[base + k]));
                wdot_s = s;
            }
            block_sync();
        }
        for (int k = tid; k < Kb; k += kThreads) {
            const int64_t slot = base + k;
            const int q = p.parents[slot];
            float d = 0.0f;
            int pq = -1;
            if (q >= 0 && q < Kb) {
                float drank = 0.0f;
                // Selected-beam weights term first (src/decoder.cpp:599-604).
                if (p.g_wsel)
                    drank = __fadd_rn(drank, __fdiv_rn(__fmul_rn(p.w_sel[slot], __fsub_rn(p.g_wsel[slot], wdot_s)),
                                                       p.sel_temp));
                if (p.g_scores) drank = __fadd_rn(drank, p.g_scores[slot]);
                if (last && p.g_final) drank = __fadd_rn(drank, p.g_final[static_cast<int64_t>(b) * K + k]);
                const float inv = __fdiv_rn(1.0f, gnmt_penalty(p.lengths[slot], p.alpha));
                d = __fadd_rn(next_g[k], __fmul_rn(drank, inv));
                if (p.g_raw) d = __fadd_rn(d, p.g_raw[slot]);
                if (last && p.g_final_raw) d = __fadd_rn(d, p.g_final_raw[static_cast<int64_t>(b) * K + k]);
                if (d != 0.0f) {
                    pq = q;
                    const int tok = p.tokens[slot];
                    if (p.from_logprob[slot] && tok >= 0 && tok < p.V) {
                        if (p.draws) p.draws[slot] = d;
                        if (p.grad) {
                            const int64_t g = (base + q) * static_cast<int64_t>(p.V) + tok;
                            p.grad[g] = __fadd_rn(p.grad[g], d);
                        }
                    }
                }
            }
            draw_s[k] = d;
            par_s[k] = pq;
        }
        block_sync();
        const bool pool = p.P > 0;
        if (pool) {
            // Pool candidates after the selected beams (src/decoder.cpp:621-657): the relaxed
            // weights' implicit gradient through the bisection threshold, and the pool scores'
            // own gradients; their sums over the pool run in pool order.
            const int64_t pbase = (static_cast<int64_t>(b) * p.T + t) * p.P;
            if (tid == 0) {
                int relaxed = 0;
                float center = 0.0f;
                if (p.g_relaxed) {
                    float denom = 0.0f, numer = 0.0f;
                    for (int i = 0; i < p.P; ++i) {
                        const float r = p.relaxed[pbase + i];
                        const float a = __fmul_rn(r, __fsub_rn(1.0f, r));
                        denom = __fadd_rn(denom, a);
                        numer = __fadd_rn(numer, __fmul_rn(p.g_relaxed[pbase + i], a));
                    }
                    if (denom > 1.0e-12f) {
                        relaxed = 1;
                        center = __fdiv_rn(numer, denom);
                    }
                }
                pool_relaxed_s = relaxed;
                pool_center_s = center;
            }
            block_sync();
            const float inv_temp = pool_relaxed_s ? __fdiv_rn(1.0f, p.soft_temp) : 0.0f;
            for (int i = tid; i < p.P; i += kThreads) {
                const int64_t slot = pbase + i;
                const int q = p.pool_parents[slot];
                float d = 0.0f;
                int pq = -1;
                if (q >= 0 && q < Kb) {
                    float drank = 0.0f;
                    if (pool_relaxed_s) {
                        const float r = p.relaxed[slot];
                        const float a = __fmul_rn(r, __fsub_rn(1.0f, r));
                        drank = __fadd_rn(drank, __fmul_rn(__fmul_rn(a, inv_temp), __fsub_rn(p.g_relaxed[slot], pool_center_s)));
                    }
                    if (p.g_pool_scores) drank = __fadd_rn(drank, p.g_pool_scores[slot]);
                    d = __fmul_rn(drank, __fdiv_rn(1.0f, gnmt_penalty(p.pool_lengths[slot], p.alpha)));
                    if (p.g_pool_raw) d = __fadd_rn(d, p.g_pool_raw[slot]);
                    if (d != 0.0f) {
                        pq = q;
                        const int tok = p.pool_tokens[slot];
                        if (p.grad && p.pool_from[slot] && tok >= 0 && tok < p.V) {
                            // After the selected beams' terms (the barrier above); pool entries are
                            // distinct candidates, so no two threads add to one element here.
                            const int64_t g = (base + q) * static_cast<int64_t>(p.V) + tok;
                            p.grad[g] = __fadd_rn(p.grad[g], d);
                        }
                    }
                }
                pdraw_s[i] = d;
                ppar_s[i] = pq;
            }
            block_sync();
        }
        // prev[q] = sum of its children's draws in slot order (then its pool candidates' in
        // pool order), from 0 (src/decoder.cpp:592-661).
        if (Kb <= kScanParentsUpTo || pool) {
            for (int q = tid; q < Kb; q += kThreads) {
                float sum = 0.0f;
                for (int k = 0; k < Kb; ++k)
                    if (par_s[k] == q) sum = __fadd_rn(sum, draw_s[k]);
                if (pool)
                    for (int i = 0; i < p.P; ++i)
                        if (ppar_s[i] == q) sum = __fadd_rn(sum, pdraw_s[i]);
                prev_g[q] = sum;
            }
        } else {
            // Children sorted by (parent, slot): each parent's children are one run, in slot
            // order; slots without a draw sort last.
            int n2 = 1;
            while (n2 < Kb) n2 <<= 1;
            for (int i = tid; i < n2; i += kThreads) {
                child_s[i] = (i < Kb && par_s[i] >= 0) ? (static_cast<uint32_t>(par_s[i]) << 11) | static_cast<uint32_t>(i)
                                                       : 0xffffffffu;
                if (i < Kb) prev_g[i] = 0.0f;
            }
            block_sync();
            bitonic_sort_u32(child_s, n2);
            for (int i = tid; i < n2; i += kThreads) {
                const uint32_t q = child_s[i] >> 11;
                if (child_s[i] == 0xffffffffu || (i > 0 && (child_s[i - 1] >> 11) == q)) continue;
                float sum = 0.0f;  // i starts parent q's run
                for (int j = i; j < n2 && (child_s[j] >> 11) == q; ++j) sum = __fadd_rn(sum, draw_s[child_s[j] & 2047u]);
                prev_g[q] = sum;
            }
        }
        block_sync();
        for (int k = tid; k < Kb; k += kThreads) next_g[k] = prev_g[k];
        block_sync();
    }
}

// Log-softmax correction, one CTA per input row (b, t, q). A row receives
// g_v - softmax(x)_v * S over every v, where g_v are the path gradients of the
// slots of step t that extend parent q (their draws, at their tokens) and S
// their sum in token order (src/decoder.hpp:212-242 apply_path_gradient).
// Rows without a path gradient are left untouched.
template <int DT>
__global__ void __launch_bounds__(kThreads) logit_correction_kernel(const __grid_constant__ BackwardParams p,
                                                                    const void* logits, const float* row_lse) {
    __shared__ int32_t tok_s[DBS_CUDA_MAX_BEAM];
    __shared__ float val_s[DBS_CUDA_MAX_BEAM];
    __shared__ int n_s;
    __shared__ float sum_s;
    const int64_t r = blockIdx.x;  // row index in [B*T*K)
    const int K = p.K;
    const int q = static_cast<int>(r % K);
    const int64_t bt = r / K;
    const int b = static_cast<int>(bt / p.T);
    const int t = static_cast<int>(bt - static_cast<int64_t>(b) * p.T);
    int steps = p.steps_pe ? p.steps_pe[b] : p.T;
    int Kb = p.beams_pe ? p.beams_pe[b] : K;
    Kb = Kb < 0 ? 0 : (Kb > K ? K : Kb);
    if (t >= steps || q >= Kb) return;
    const int64_t base = bt * K;
    const int tid = threadIdx.x;
    if (tid == 0) n_s = 0;
    block_sync();
    for (int k = tid; k < Kb; k += kThreads) {
        const float d = p.draws[base + k];
        if (d != 0.0f && p.parents[base + k] == q) {
            const int i = atomicAdd(&n_s, 1);
            tok_s[i] = p.tokens[base + k];
            val_s[i] = d;
        }
    }
    block_sync();
    const int n = n_s;
    if (n == 0) return;
    if (tid == 0) {
        // Sort by token (distinct within a row) and sum in token order.
        for (int i = 1; i < n; ++i) {
            const int32_t tk = tok_s[i];
            const float vv = val_s[i];
            int j = i;
            while (j > 0 && tok_s[j - 1] > tk) {
                tok_s[j] = tok_s[j - 1];
                val_s[j] = val_s[j - 1];
                --j;
            }
            tok_s[j] = tk;
            val_s[j] = vv;
        }
        float s = 0.0f;
        for (int i = 0; i < n; ++i) s = __fadd_rn(s, val_s[i]);
        sum_s = s;
    }
    block_sync();
    const float S = sum_s;
    const float lse = row_lse[r];
    const int64_t V = p.V;
    const int64_t off = r * V;
    float* g = p.grad + off;
    for (int64_t v = tid; v < V; v += kThreads) {
        const float x = load_elem<DT>(logits, off + v);
        float gv = 0.0f;
        int lo = 0, hi = n;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (tok_s[mid] < v) lo = mid + 1;
            else hi = mid;
        }
        if (lo < n && tok_s[lo] == v) gv = val_s[lo];
        const float d = __fsub_rn(gv, __fmul_rn(softmax_probability(x, lse), S));
        g[v] = __fadd_rn(g[v], d);
    }
}

// ---------------------------------------------------------------------------
// Dense gradient in one write pass. Every element of grad[B, T, K, V] (element
// type OT) is written exactly once with the value the reference produces by
// zero-filling a float32 gradient, accumulating the backward into it and
// casting it to the input dtype (python/beamgrad/_torch.py:270-289:
// decode_backward(...).to(input_dtype)):
//   log-prob rows: 0 + draw at the token of each child slot with a nonzero
//                  draw, 0 elsewhere (src/decoder.cpp:546-663 scatter);
//   logit rows:    0 + (g_v - softmax(x_v, lse) * S) for rows with a path
//                  gradient (src/decoder.hpp:212-242), 0 for the others;
// then rounded to nearest-even into OT. This replaces the zero-fill, the
// read-modify-write of the correction and the cast pass. Rows decoded from
// logits are written here once (16-byte stores that bypass L2 retention)
// and read once; rows of log-probabilities are almost all zero and take the
// memset + scatter_dense_kernel path instead (launch_dense_grad).
//
// A CTA takes rows r = (b*T + t)*K + q in a grid-stride loop. The children of
// row r are the slots of step t whose parent is q and whose draw is nonzero
// (draws are written only for slots that consumed an input entry); they are
// sorted by token (slot breaks ties) so the logit sum S runs in token order.
// ---------------------------------------------------------------------------
template <int OT>
struct OutElem;
template <>
struct OutElem<0> {
    using T = float;
    __device__ static __forceinline__ float cvt(float v) { return v; }
};
template <>
struct OutElem<1> {
    using T = __half;
    __device__ static __forceinline__ __half cvt(float v) { return __float2half_rn(v); }
};
template <>
struct OutElem<2> {
    using T = __nv_bfloat16;
    __device__ static __forceinline__ __nv_bfloat16 cvt(float v) { return __float2bfloat16_rn(v); }
};

template <int IT, int OT, bool LOGITS>
__global__ void __launch_bounds__(kThreads) dense_grad_kernel(const __grid_constant__ BackwardParams p,
                                                              const void* __restrict__ logits,
                                                              const float* __restrict__ row_lse, void* __restrict__ out,
                                                              int vec) {
    using OutT = typename OutElem<OT>::T;
    constexpr int kChunk = 16 / static_cast<int>(sizeof(OutT));  // elements per 16-byte store
    __shared__ int32_t tok_s[DBS_CUDA_MAX_BEAM];
    __shared__ float val_s[DBS_CUDA_MAX_BEAM];
    __shared__ int32_t slot_s[DBS_CUDA_MAX_BEAM];
    __shared__ int32_t stok_s[DBS_CUDA_MAX_BEAM];
    __shared__ float sval_s[DBS_CUDA_MAX_BEAM];
    __shared__ int n_s;
    __shared__ float sum_s;
    const int tid = threadIdx.x;
    const int K = p.K;
    const int64_t V = p.V;
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * K;
    OutT* grad = static_cast<OutT*>(out);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int q = static_cast<int>(r % K);
        const int64_t bt = r / K;
        const int b = static_cast<int>(bt / p.T);
        const int t = static_cast<int>(bt - static_cast<int64_t>(b) * p.T);
        int steps = p.steps_pe ? p.steps_pe[b] : p.T;
        int Kb = p.beams_pe ? p.beams_pe[b] : K;
        steps = steps < 0 ? 0 : (steps > p.T ? p.T : steps);
        Kb = Kb < 0 ? 0 : (Kb > K ? K : Kb);
        const bool active = t < steps && q < Kb;
        if (tid == 0) n_s = 0;
        block_sync();
        if (active) {
            const int64_t base = bt * K;
            for (int k = tid; k < Kb; k += kThreads) {
                const float d = p.draws[base + k];
                if (d != 0.0f && p.parents[base + k] == q) {
                    const int i = atomicAdd(&n_s, 1);
                    tok_s[i] = p.tokens[base + k];
                    val_s[i] = d;
                    slot_s[i] = k;
                }
            }
        }
        block_sync();
        const int n = n_s;
        if (n > 0) {
            // Rank sort by (token, slot): the keys are distinct.
            for (int i = tid; i < n; i += kThreads) {
                const int32_t ti = tok_s[i], si = slot_s[i];
                int rank = 0;
                for (int j = 0; j < n; ++j) rank += (tok_s[j] < ti) || (tok_s[j] == ti && slot_s[j] < si);
                stok_s[rank] = ti;
                sval_s[rank] = val_s[i];
            }
            block_sync();
            if (LOGITS && tid == 0) {
                float s = 0.0f;
                for (int i = 0; i < n; ++i) s = __fadd_rn(s, sval_s[i]);
                sum_s = s;
            }
            block_sync();
        }
        const float S = LOGITS && n > 0 ? sum_s : 0.0f;
        const float lse = LOGITS && n > 0 ? row_lse[r] : 0.0f;
        const int64_t off = r * V;
        // Value of element v of this row (before the cast).
        auto value = [&](int64_t v, float x, int& e) -> float {
            // e: index of the first sorted entry with token >= v (advanced by the caller's scan).
            float gv = 0.0f;
            while (e < n && stok_s[e] < v) ++e;
            bool hit = false;
            while (e < n && stok_s[e] == v) {
                gv = __fadd_rn(gv, sval_s[e]);
                hit = true;
                ++e;
            }
            if (LOGITS) {
                if (n == 0) return 0.0f;
                return __fadd_rn(0.0f, __fsub_rn(gv, __fmul_rn(softmax_probability(x, lse), S)));
            }
            return hit ? __fadd_rn(0.0f, gv) : 0.0f;
        };
        auto lower = [&](int64_t v) -> int {
            int lo = 0, hi = n;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (stok_s[mid] < v) lo = mid + 1;
                else hi = mid;
            }
            return lo;
        };
        const bool need_x = LOGITS && n > 0;
        int64_t head = V;
        if (vec) {
            const int64_t mis = off % kChunk;
            head = mis == 0 ? 0 : kChunk - mis;
            if (head > V) head = V;
        }
        const int64_t nchunks = (V - head) / kChunk;
        const int64_t body_end = head + nchunks * kChunk;
        // Scalar head [0, head) and tail [body_end, V).
        const int64_t scalar_count = head + (V - body_end);
        for (int64_t i = tid; i < scalar_count; i += kThreads) {
            const int64_t v = i < head ? i : body_end + (i - head);
            int e = n > 0 ? lower(v) : 0;
            const float x = need_x ? load_elem<IT>(logits, off + v) : 0.0f;
            grad[off + v] = OutElem<OT>::cvt(value(v, x, e));
        }
        // 16-byte body.
        for (int64_t c = tid; c < nchunks; c += kThreads) {
            const int64_t v0 = head + c * kChunk;
            float xs[kChunk];
            if (need_x) {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) xs[j] = load_elem<IT>(logits, off + v0 + j);
            }
            int e = n > 0 ? lower(v0) : 0;
            union {
                uint4 u;
                OutT h[kChunk];
            } pk;
            if (n == 0) {
                pk.u = make_uint4(0u, 0u, 0u, 0u);
            } else {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) pk.h[j] = OutElem<OT>::cvt(value(v0 + j, need_x ? xs[j] : 0.0f, e));
            }
            __stcs(reinterpret_cast<uint4*>(grad + off + v0), pk.u);
        }
        block_sync();  // the row's shared lists are rewritten by the next row
    }
}

// Rows of log-probabilities: after the gradient is zero-filled (a memset,
// the fastest way to stream zeros to HBM), each slot with a nonzero draw
// writes its entry (t, parent, token) = 0 + draw, rounded into OT. Slots of
// one step that share (parent, token) are summed in slot order by the first
// of them (from 0, as the dense kernel and the float32 accumulation do).
template <int OT>
__global__ void scatter_dense_kernel(const __grid_constant__ BackwardParams p, void* __restrict__ out) {
    using OutT = typename OutElem<OT>::T;
    OutT* grad = static_cast<OutT*>(out);
    const int K = p.K;
    const int64_t slots = static_cast<int64_t>(p.B) * p.T * K;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < slots;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float d = p.draws[i];
        if (d == 0.0f) continue;  // draws are nonzero only for valid slots that consumed an entry
        const int64_t bt = i / K;
        const int k = static_cast<int>(i - bt * K);
        const int64_t base = bt * K;
        const int q = p.parents[i];
        const int tok = p.tokens[i];
        bool first = true;
        for (int j = 0; j < k && first; ++j)
            first = !(p.draws[base + j] != 0.0f && p.parents[base + j] == q && p.tokens[base + j] == tok);
        if (!first) continue;
        float g = __fadd_rn(0.0f, d);
        for (int j = k + 1; j < K; ++j)
            if (p.draws[base + j] != 0.0f && p.parents[base + j] == q && p.tokens[base + j] == tok)
                g = __fadd_rn(g, p.draws[base + j]);
        grad[(base + q) * static_cast<int64_t>(p.V) + tok] = OutElem<OT>::cvt(__fadd_rn(0.0f, g));
    }
}

// Selected-beam weights: softmax_selected (src/kernels_scalar.cpp:277-302) over each
// step's K selected scores, one thread per (b, t) in slot order: scores above -1e30
// take part; maxv = max of score / temperature; w = exp(score / temperature - maxv)
// summed in slot order; w *= 1 / sum; all zero when no score takes part or the sum
// is not a positive finite number.
__global__ void selected_weights_kernel(int64_t rows, int K, const float* __restrict__ scores, float temperature,
                                        float* __restrict__ out) {
    const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float guard = -1.0e30f;
    const float* sc = scores + r * K;
    float* o = out + r * K;
    for (int k = 0; k < K; ++k) o[k] = 0.0f;
    float maxv = f_ninf();
    for (int k = 0; k < K; ++k) {
        if (sc[k] > guard) {
            const float q = __fdiv_rn(sc[k], temperature);
            maxv = maxv < q ? q : maxv;
        }
    }
    if (!(maxv > f_ninf() && maxv < f_inf())) return;
    float sum = 0.0f;
    for (int k = 0; k < K; ++k) {
        if (sc[k] > guard) {
            o[k] = exp_nonpositive(__fsub_rn(__fdiv_rn(sc[k], temperature), maxv));
            sum = __fadd_rn(sum, o[k]);
        }
    }
    if (!(sum > 0.0f) || !(sum < f_inf())) {
        for (int k = 0; k < K; ++k) o[k] = 0.0f;
        return;
    }
    const float inv = __fdiv_rn(1.0f, sum);
    for (int k = 0; k < K; ++k) o[k] = __fmul_rn(o[k], inv);
}

cudaError_t launch_selected_weights(int64_t rows, int K, const float* scores, float temperature, float* out,
                                    cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    selected_weights_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, stream>>>(rows, K, scores,
                                                                                            temperature, out);
    return cudaGetLastError();
}

__global__ void length_penalty_kernel(const int32_t* __restrict__ lengths, int64_t count, float alpha,
                                      float* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) out[i] = gnmt_penalty(lengths[i], alpha);
}

// Token sequences of the final beams, [B, K, T] int64: entry (b, k, t) is the
// token final beam k holds at step t, following parents back from the last
// step; -1 for dead beams and for steps past the example's length
// (python/beamgrad/_torch.py:582-606 of beamgrad 2.3.0). One thread per (b, k).
__global__ void backtrack_kernel(int B, int T, int K, const int32_t* __restrict__ tokens,
                                 const int32_t* __restrict__ parents, const int32_t* __restrict__ steps_pe,
                                 int64_t* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(B) * K) return;
    const int b = static_cast<int>(i / K);
    const int k = static_cast<int>(i - static_cast<int64_t>(b) * K);
    int steps = steps_pe ? steps_pe[b] : T;
    int beam = k;
    int64_t* o = out + i * T;
    for (int t = T - 1; t >= 0; --t) {
        const bool decoded = t < steps;
        const bool alive = beam >= 0 && decoded;
        const int64_t slot = (static_cast<int64_t>(b) * T + t) * K + (beam >= 0 ? beam : 0);
        o[t] = alive ? static_cast<int64_t>(tokens[slot]) : -1;
        if (decoded) beam = beam >= 0 ? parents[slot] : -1;
        if (beam >= K) beam = -1;
    }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
cudaError_t launch_backward(const BackwardParams& p, cudaStream_t stream) {
    backward_kernel<<<static_cast<unsigned>(p.B), kThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_logit_correction(const BackwardParams& p, int dtype, const void* logits, const float* row_lse,
                                    cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * p.K;
    const unsigned grid = static_cast<unsigned>(rows);
    switch (dtype) {
        case DBS_CUDA_DTYPE_F16: logit_correction_kernel<1><<<grid, kThreads, 0, stream>>>(p, logits, row_lse); break;
        case DBS_CUDA_DTYPE_BF16: logit_correction_kernel<2><<<grid, kThreads, 0, stream>>>(p, logits, row_lse); break;
        default: logit_correction_kernel<0><<<grid, kThreads, 0, stream>>>(p, logits, row_lse); break;
    }
    return cudaGetLastError();
}

template <int IT, bool LOGITS>
cudaError_t launch_dense_out(const BackwardParams& p, int out_type, const void* logits, const float* row_lse,
                             void* grad, int vec, unsigned grid, cudaStream_t stream) {
    switch (out_type) {
        case DBS_CUDA_DTYPE_F16:
            dense_grad_kernel<IT, 1, LOGITS><<<grid, kThreads, 0, stream>>>(p, logits, row_lse, grad, vec);
            break;
        case DBS_CUDA_DTYPE_BF16:
            dense_grad_kernel<IT, 2, LOGITS><<<grid, kThreads, 0, stream>>>(p, logits, row_lse, grad, vec);
            break;
        default: dense_grad_kernel<IT, 0, LOGITS><<<grid, kThreads, 0, stream>>>(p, logits, row_lse, grad, vec); break;
    }
    return cudaGetLastError();
}

// Log-prob rows: stream-ordered memset of the whole gradient, then the sparse
// scatter. Logit rows: dense_grad_kernel writes every element once (grid =
// 8 CTAs per SM); vec: 1 when grad and logits start on 16-byte boundaries.
cudaError_t launch_dense_grad(const BackwardParams& p, int in_type, const void* logits, const float* row_lse,
                              int out_type, void* grad, int vec, int sm_count, cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * p.K;
    if (rows == 0) return cudaSuccess;
    if (!logits) {
        const size_t elem = out_type == DBS_CUDA_DTYPE_F32 ? 4 : 2;
        const cudaError_t e = cudaMemsetAsync(grad, 0, static_cast<size_t>(rows) * static_cast<size_t>(p.V) * elem,
                                              stream);
        if (e != cudaSuccess) return e;
        const int64_t want = (rows + 255) / 256;
        const int64_t cap = static_cast<int64_t>(sm_count) * 8;
        const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
        switch (out_type) {
            case DBS_CUDA_DTYPE_F16: scatter_dense_kernel<1><<<blocks, 256, 0, stream>>>(p, grad); break;
            case DBS_CUDA_DTYPE_BF16: scatter_dense_kernel<2><<<blocks, 256, 0, stream>>>(p, grad); break;
            default: scatter_dense_kernel<0><<<blocks, 256, 0, stream>>>(p, grad); break;
        }
        return cudaGetLastError();
    }
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, static_cast<int64_t>(sm_count) * 8));
    switch (in_type) {
        case DBS_CUDA_DTYPE_F16: return launch_dense_out<1, true>(p, out_type, logits, row_lse, grad, vec, grid, stream);
        case DBS_CUDA_DTYPE_BF16: return launch_dense_out<2, true>(p, out_type, logits, row_lse, grad, vec, grid, stream);
        default: return launch_dense_out<0, true>(p, out_type, logits, row_lse, grad, vec, grid, stream);
    }
}

cudaError_t launch_length_penalty(const int32_t* lengths, int64_t count, float alpha, float* out, cudaStream_t stream) {
    const int64_t blocks = (count + 255) / 256;
    length_penalty_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(lengths, count, alpha, out);
    return cudaGetLastError();
}

cudaError_t launch_backtrack(int B, int T, int K, const int32_t* tokens, const int32_t* parents,
                             const int32_t* steps_pe, int64_t* out, cudaStream_t stream) {
    const int64_t n = static_cast<int64_t>(B) * K;
    backtrack_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, stream>>>(B, T, K, tokens, parents, steps_pe, out);
    return cudaGetLastError();
}

}  // namespace dbsb
