// SPDX-License-Identifier: MIT
//
// The decode kernels of the B200 engine (included by decode.cu and the per-dtype
// decode_*.cu units). Three kernels run a whole decode in one persistent launch each:
//
//   decode_chain_kernel       beams <= 16, rows staged in shared memory by a TMA bulk
//                             copy (or streamed when they do not fit): pass 1 (maximum,
//                             minimum, NaN/+inf flag, per-thread maxima -> a filter bound),
//                             from logits pass 2 (the reference's fixed-order logsumexp on
//                             warps 0-3, packed f32x2) beside the row record on warps 4-7;
//   decode_chain_warp_kernel  log-probability rows, beams <= 16, one warp per row straight
//                             from HBM;
//   decode_chain_wide_kernel  beams 17..1024, records of 2K entries, block selection.
//
// Chained protocol (no CTA ever waits for another): work items are beam rows (t, b, k)
// handed out by an atomic ticket in t-major order. A row needs nothing from the previous
// step: it is reduced to a parent-independent record (its best entries by x, its
// logsumexp and flags). Each (b, t) counts arrivals -- its K rows and, for t > 0, the
// selection of step t-1 -- and the CTA (or warp) that completes the count selects step t
// from the K records and the carried-forward finished beams, then arrives for t+1. A
// record that cannot prove it holds the row's best candidates (raw scores that round
// together, constraints) is rescanned by the selecting group with the parent known.
//
// decode_kernel (the waiting variant) serves the step API and decodes whose record area
// would be too large: step t of example b waits (bounded; a timeout sets the error word)
// for step t-1 to be published, then scans its row with the parent known.
//
// Candidate order: within one step every scanned candidate of an example extends a beam
// of the same length, so ranking by (raw desc, parent*V+token asc) -- a 64-bit key --
// equals the CPU decoder's ranking by (score, raw, parent, token) (src/common.hpp:269-276
// of beamgrad 2.3.0). Carried-forward candidates are merged with the full comparator.
#pragma once
#include <type_traits>

#include "engine.cuh"

namespace dbsb {
namespace {  // internal to each translation unit that includes this file

// ---------------------------------------------------------------------------
// Shared memory
// ---------------------------------------------------------------------------

// Scratch of one selecting group.
struct SelScratch {
    uint64_t wkeys[kWarps * kFastBeam];
    unsigned fallback;  // rows whose record is not enough
    int invalid;
    int next;           // broadcast of the chain's next step
};

struct RowShared {
    unsigned long long mbar;
    int ticket;
    int ready;
    int is_last;
    int invalid;
    int n_blocked;
    int n_penal;
    int count;
    int done;
    int remaining;
    unsigned long long sel_prefix;
    unsigned long long sel_mask;
    float wred[kWarps];
    float wred2[kWarps];
    int ired[kWarps];
    int nlist[kWarps];  // chained decode: nonzero keys of each warp's record list
    float row_lse;
    float lanes[kLanes];
    int hist[256];
    uint64_t wkeys[kWarps * 32];
    float wtop[kWarps * 32];  // each warp's largest per-thread bounds, sorted
    float xbound;                    // the row's filter bound (R-th largest of all thread bounds)
    int32_t blocked[kConsCap];
    int32_t penal[kConsCap];
    // select bookkeeping
    int n_scanned;
    int n_carry;
    SelScratch sel;  // chained decode: the selecting CTA's scratch
};

// Per-example select arrays of capacity KCAP, in dynamic shared memory.
template <int KCAP>
struct SelectShared {
    uint64_t keys[KCAP];
    float s_raw[KCAP];
    int32_t s_len[KCAP];
    int32_t s_last[KCAP];
    uint8_t s_ended[KCAP];
    float c_score[KCAP];
    float c_raw[KCAP];
    int32_t c_parent[KCAP];
    int32_t c_len[KCAP];
    int32_t c_token[KCAP];
    float sc_score[KCAP];
    // final assignment of slots
    int32_t o_parent[KCAP];
    int32_t o_token[KCAP];
    int32_t o_len[KCAP];
    float o_score[KCAP];
    float o_raw[KCAP];
    uint8_t o_from[KCAP];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// TMA bulk staging of one row
// ---------------------------------------------------------------------------

// Hint to bring [p, p + bytes) into L2 (p and bytes multiples of 16); no data returns.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_init(unsigned long long* mbar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(mbar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(unsigned long long* mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mbar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes, unsigned long long* mbar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(sdst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(mbar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* mbar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred P;\n mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n selp.u32 %0, 1, 0, P;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(mbar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase
// completes or about hint_ns pass, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(unsigned long long* mbar, uint32_t phase, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred P;\n mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n selp.u32 %0, 1, 0, P;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(mbar)), "r"(phase), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for the row's bulk copy. On timeout: records the error and keeps
// waiting (bounded again) so no copy is left writing into shared memory.
__device__ __forceinline__ bool mbar_wait(const DecodeParams& p, unsigned long long* mbar, uint32_t phase) {
    if (mbar_try_wait(mbar, phase)) return true;
    const unsigned long long start = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(mbar, phase, 20000u)) return true;
        if (global_ns() - start > p.timeout_ns) {
            atomicCAS(p.error, kErrNone, kErrTimeout);
            const unsigned long long again = global_ns();
            while (!mbar_try_wait(mbar, phase) && global_ns() - again < p.timeout_ns) {
            }
            return false;
        }
    }
}

// Row layout in shared memory: the row keeps its global address modulo 16,
// so the 16-byte-aligned body moves with bulk copies and the ragged head and
// tail (under 16 bytes each) with plain loads.
//
// stage_issue (one thread): the body's bulk copies, completing on mbar.
template <int EB>
__device__ __forceinline__ void stage_issue(char* sbuf, const char* g, int V, unsigned long long* mbar) {
    const uintptr_t g0 = reinterpret_cast<uintptr_t>(g);
    const uintptr_t g1 = g0 + static_cast<uintptr_t>(V) * EB;
    const uintptr_t a0 = (g0 + 15) & ~static_cast<uintptr_t>(15);
    const uintptr_t a1 = g1 & ~static_cast<uintptr_t>(15);
    if (a1 <= a0) return;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const uint32_t bytes = static_cast<uint32_t>(a1 - a0);
    mbar_expect_tx(mbar, bytes);
    constexpr uint32_t kChunk = 1u << 16;
    for (uint32_t c = 0; c < bytes; c += kChunk) {
        const uint32_t n = bytes - c < kChunk ? bytes - c : kChunk;
        bulk_g2s(sbuf + (a0 - (g0 & ~static_cast<uintptr_t>(15))) + c, reinterpret_cast<const char*>(a0) + c, n, mbar);
    }
}

// stage_finish (whole CTA): the ragged ends, then the bounded wait for the body (one
// thread waits, the CTA follows at the barrier). Returns the offset of element 0.
template <int EB>
__device__ __forceinline__ int stage_finish(const DecodeParams& p, char* sbuf, const char* g, int V,
                                            unsigned long long* mbar, uint32_t& phase, bool& ok) {
    const uintptr_t g0 = reinterpret_cast<uintptr_t>(g);
    const uintptr_t g1 = g0 + static_cast<uintptr_t>(V) * EB;
    const uintptr_t a0 = (g0 + 15) & ~static_cast<uintptr_t>(15);
    const uintptr_t a1 = g1 & ~static_cast<uintptr_t>(15);
    const int tid = threadIdx.x;
    const bool bulk = a1 > a0;
    const uintptr_t head_end = bulk ? a0 : g1;
    const int n_head = static_cast<int>((head_end - g0) / EB);
    const int n_tail = bulk ? static_cast<int>((g1 - a1) / EB) : 0;
    for (int i = tid; i < n_head + n_tail; i += kThreads) {
        const uintptr_t src = i < n_head ? g0 + static_cast<uintptr_t>(i) * EB : a1 + static_cast<uintptr_t>(i - n_head) * EB;
        char* dst = sbuf + (src - (g0 & ~static_cast<uintptr_t>(15)));
        if (EB == 4) *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
        else *reinterpret_cast<uint16_t*>(dst) = *reinterpret_cast<const uint16_t*>(src);
    }
    ok = true;
    if (bulk) {
        if (tid == 0) ok = mbar_wait(p, mbar, phase);
        phase ^= 1u;
    }
    ok = block_and(ok);
    return static_cast<int>(g0 & 15);
}

template <int EB>
__device__ __forceinline__ int stage_row(const DecodeParams& p, RowShared& sh, char* sbuf, const char* g,
                                         int V, uint32_t& phase, bool& ok) {
    if (threadIdx.x == 0) stage_issue<EB>(sbuf, g, V, &sh.mbar);
    return stage_finish<EB>(p, sbuf, g, V, &sh.mbar, phase, ok);
}

// ---------------------------------------------------------------------------
// Element iteration: 128-bit vectors for the aligned body, scalars for the
// ragged ends. f(x, v) is called for every element exactly once; each thread
// sees its elements in increasing v.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <int DT, bool kGlobal, class F>
__device__ __forceinline__ void for_row(const char* row, int V, F&& f) {
    using E = Elem<DT>;
    constexpr int EB = E::kBytes;
    constexpr int PER = 16 / EB;
    const int tid = threadIdx.x;
    const uintptr_t a = reinterpret_cast<uintptr_t>(row);
    int head = static_cast<int>(((16 - (a & 15)) & 15) / EB);
    if (head > V) head = V;
    const auto* rp = reinterpret_cast<const typename E::T*>(row);
    if (tid < head) f(E::to_f32(rp[tid]), tid);
    const int nvec = (V - head) / PER;
    const uint4* vp = reinterpret_cast<const uint4*>(row + static_cast<size_t>(head) * EB);
    auto unpack = [&](const uint4& q, int v0) {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        if constexpr (EB == 4) {
#pragma unroll
            for (int j = 0; j < 4; ++j) f(__uint_as_float(w[j]), v0 + j);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                f(E::to_f32(static_cast<uint16_t>(w[j] & 0xffffu)), v0 + 2 * j);
                f(E::to_f32(static_cast<uint16_t>(w[j] >> 16)), v0 + 2 * j + 1);
            }
        }
    };
    int c = tid;
    if constexpr (kGlobal) {
        for (; c + 3 * kThreads < nvec; c += 4 * kThreads) {
            const uint4 q0 = ld_stream_v4(vp + c);
            const uint4 q1 = ld_stream_v4(vp + c + kThreads);
            const uint4 q2 = ld_stream_v4(vp + c + 2 * kThreads);
            const uint4 q3 = ld_stream_v4(vp + c + 3 * kThreads);
            unpack(q0, head + c * PER);
            unpack(q1, head + (c + kThreads) * PER);
            unpack(q2, head + (c + 2 * kThreads) * PER);
            unpack(q3, head + (c + 3 * kThreads) * PER);
        }
        for (; c < nvec; c += kThreads) unpack(ld_stream_v4(vp + c), head + c * PER);
    } else {
        for (; c < nvec; c += kThreads) unpack(vp[c], head + c * PER);
    }
    const int tail0 = head + nvec * PER;
    if (tail0 + tid < V) f(E::to_f32(rp[tail0 + tid]), tail0 + tid);
}

// ---------------------------------------------------------------------------
// Block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_max(RowShared& sh, float v) {
    v = warp_max_f32(v);
    if ((threadIdx.x & 31) == 0) sh.wred[threadIdx.x >> 5] = v;
    block_sync();
    float r = sh.wred[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) r = fmaxf(r, sh.wred[w]);
    block_sync();
    return r;
}
__device__ __forceinline__ int block_sum(RowShared& sh, int v) {
    v = warp_sum_i32(v);
    if ((threadIdx.x & 31) == 0) sh.ired[threadIdx.x >> 5] = v;
    block_sync();
    int r = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) r += sh.ired[w];
    block_sync();
    return r;
}

// ---------------------------------------------------------------------------
// Block radix select: writes the `want` largest non-zero keys among gen(0..n)
// (keys are unique) to out[0..count) in no particular order; returns count =
// min(want, number of non-zero keys). 8-bit digits, most significant first,
// stopping as soon as the boundary bucket is taken whole.
// ---------------------------------------------------------------------------
template <class Gen, class Out>
__device__ int block_select(RowShared& sh, Gen&& gen, int n, int want, Out&& out) {
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    int c = 0;
    for (int i = tid; i < n; i += kThreads) c += gen(i) != 0 ? 1 : 0;
    const int total = block_sum(sh, c);
    uint64_t prefix = 0, mask = 0;
    const bool take_all = total <= want;
    if (!take_all) {
        if (tid == 0) {
            sh.sel_prefix = 0;
            sh.sel_mask = 0;
            sh.remaining = want;
            sh.done = 0;
        }
        for (int shift = 56; shift >= 0; shift -= 8) {
            sh.hist[tid] = 0;
            block_sync();
            prefix = sh.sel_prefix;
            mask = sh.sel_mask;
            for (int base = 0; base < n; base += kThreads) {
                const int i = base + tid;
                const uint64_t key = i < n ? gen(i) : 0;
                const bool in = key != 0 && (key & mask) == prefix;
                const int digit = in ? static_cast<int>((key >> shift) & 255u) : 256;
                const unsigned peers = __match_any_sync(0xffffffffu, digit);
                if (in && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[digit], __popc(peers));
            }
            block_sync();
            if (tid < 32) {
                // The boundary bucket: the highest digit d whose count, with every digit above
                // it, reaches `remaining`. Lane l holds digits 255 - 8l ... 248 - 8l.
                int h[8];
                int sum = 0;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    h[e] = sh.hist[255 - (lane * 8 + e)];
                    sum += h[e];
                }
                int incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                const int rem = sh.remaining;
                const int excl = incl - sum;
                const unsigned here = __ballot_sync(0xffffffffu, excl < rem && incl >= rem);
                const int owner = here ? __ffs(here) - 1 : 31;  // no lane: digit 0 (as a full scan ends)
                if (lane == owner) {
                    int c = excl, d = 0, e = 0;
                    for (; e < 8; ++e) {
                        d = 255 - (lane * 8 + e);
                        if (d == 0 || c + h[e] >= rem) break;
                        c += h[e];
                    }
                    const int left = rem - c;
                    sh.sel_prefix |= static_cast<unsigned long long>(d) << shift;
                    sh.sel_mask |= 255ull << shift;
                    sh.remaining = left;
                    sh.done = h[e] == left;
                }
            }
            block_sync();
            if (sh.done) break;
        }
        prefix = sh.sel_prefix;
        mask = sh.sel_mask;
    }
    if (tid == 0) sh.count = 0;
    block_sync();
    for (int base = 0; base < n; base += kThreads) {
        const int i = base + tid;
        const uint64_t key = i < n ? gen(i) : 0;
        const bool take = key != 0 && (take_all || (key & mask) >= prefix);
        const unsigned ballot = __ballot_sync(0xffffffffu, take);
        int pos0 = 0;
        if (lane == 0 && ballot) pos0 = atomicAdd(&sh.count, __popc(ballot));
        pos0 = __shfl_sync(0xffffffffu, pos0, 0);
        if (take) {
            const int pos = pos0 + __popc(ballot & ((1u << lane) - 1u));
            if (pos < want) out(pos, key);
        }
    }
    block_sync();
    const int count = sh.count < want ? sh.count : want;
    block_sync();
    return count;
}

// Bitonic sort (descending) of n = power of two keys in shared memory.
__device__ __forceinline__ void bitonic_desc(uint64_t* keys, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += kThreads) {
                const int partner = i ^ j;
                if (partner > i) {
                    const uint64_t a = keys[i], b = keys[partner];
                    const bool up = (i & k) == 0;
                    if (up ? (a < b) : (a > b)) {
                        keys[i] = b;
                        keys[partner] = a;
                    }
                }
            }
            block_sync();
        }
    }
}

// ---------------------------------------------------------------------------
// Constraint sets of one parent row (n-gram blocking, repetition penalty),
// src/decoder.cpp:196-258 of beamgrad 2.3.0: sorted token lists in shared
// memory. Prefixes longer than kConsCap fall back to scanning the prefix.
// ---------------------------------------------------------------------------
struct ConsView {
    const int32_t* prefix;  // the parent's prefix
    int L;
    bool in_smem;
};

__device__ __forceinline__ void sort_small(int32_t* a, int n) {
    // odd-even transposition sort, n <= kConsCap, all threads
    for (int phase = 0; phase < n; ++phase) {
        for (int i = 2 * threadIdx.x + (phase & 1); i + 1 < n; i += 2 * kThreads) {
            if (a[i] > a[i + 1]) {
                const int32_t t = a[i];
                a[i] = a[i + 1];
                a[i + 1] = t;
            }
        }
        block_sync();
    }
}

__device__ __forceinline__ bool ngram_match_at(const int32_t* pre, int L, int n, int i) {
    const int suffix = L - (n - 1);
    for (int j = 0; j < n - 1; ++j)
        if (pre[i + j] != pre[suffix + j]) return false;
    return true;
}

__device__ ConsView build_constraints(const DecodeParams& p, RowShared& sh, const int32_t* pre, int L) {
    ConsView cv{pre, L, L <= kConsCap};
    if (threadIdx.x == 0) {
        sh.n_blocked = 0;
        sh.n_penal = 0;
    }
    block_sync();
    if (!cv.in_smem) return cv;
    const int n = p.ngram;
    if (n == 1) {
        for (int i = threadIdx.x; i < L; i += kThreads) {
            const int tok = ld_cg(pre + i);
            if (tok >= 0 && tok < p.V) sh.blocked[atomicAdd(&sh.n_blocked, 1)] = tok;
        }
    } else if (n > 1 && L >= n - 1) {
        for (int i = threadIdx.x; i + n <= L; i += kThreads) {
            if (ngram_match_at(pre, L, n, i)) {
                const int tok = ld_cg(pre + i + n - 1);
                if (tok >= 0 && tok < p.V) sh.blocked[atomicAdd(&sh.n_blocked, 1)] = tok;
            }
        }
    }
    if (p.penalise) {
        for (int i = threadIdx.x; i < L; i += kThreads) {
            const int tok = ld_cg(pre + i);
            if (tok >= 0 && tok < p.V) sh.penal[atomicAdd(&sh.n_penal, 1)] = tok;
        }
    }
    block_sync();
    sort_small(sh.blocked, sh.n_blocked);
    sort_small(sh.penal, sh.n_penal);
    return cv;
}

__device__ __forceinline__ bool sorted_has(const int32_t* a, int n, int v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < v) lo = mid + 1;
        else hi = mid;
    }
    return lo < n && a[lo] == v;
}

// n-gram blocking / repetition penalty of token v after a prefix read from global memory.
__device__ __forceinline__ bool prefix_blocked(const DecodeParams& p, const ConsView& cv, int v) {
    const int n = p.ngram;
    if (n == 1) {
        for (int i = 0; i < cv.L; ++i)
            if (ld_cg(cv.prefix + i) == v) return true;
        return false;
    }
    if (n > 1 && cv.L >= n - 1) {
        for (int i = 0; i + n <= cv.L; ++i)
            if (ld_cg(cv.prefix + i + n - 1) == v && ngram_match_at(cv.prefix, cv.L, n, i)) return true;
    }
    return false;
}
__device__ __forceinline__ bool prefix_penalised(const DecodeParams& p, const ConsView& cv, int v) {
    if (!p.penalise) return false;
    for (int i = 0; i < cv.L; ++i)
        if (ld_cg(cv.prefix + i) == v) return true;
    return false;
}

__device__ __forceinline__ bool cons_blocked(const DecodeParams& p, const RowShared& sh, const ConsView& cv, int v) {
    return cv.in_smem ? sorted_has(sh.blocked, sh.n_blocked, v) : prefix_blocked(p, cv, v);
}
__device__ __forceinline__ bool cons_penalised(const DecodeParams& p, const RowShared& sh, const ConsView& cv, int v) {
    if (!p.penalise) return false;
    return cv.in_smem ? sorted_has(sh.penal, sh.n_penal, v) : prefix_penalised(p, cv, v);
}

// The parent's prefix during a chained decode (double-buffered by step parity), for the
// constraint checks at selection time; an empty view without constraints.
__device__ __forceinline__ ConsView chain_prefix(const DecodeParams& p, int t, int64_t s) {
    ConsView cv{nullptr, 0, false};
    if ((p.ngram > 0 || p.penalise) && p.prefix[0]) {
        cv.prefix = p.prefix[t & 1] + s * p.T;
        cv.L = ld_cg(p.prefix_len[t & 1] + s);
    }
    return cv;
}

// Raw score of record entry x (token v) for a parent with raw pr under the parent's
// constraints: -inf when the entry is no candidate (blocked, or the score underflows).
template <bool LOGITS>
__device__ __forceinline__ float constrained_raw(const DecodeParams& p, const ConsView& cv, float pr, float x, float lse,
                                                 int v) {
    float lp = LOGITS ? __fsub_rn(x, lse) : x;
    if (!(lp < f_inf()) || lp == f_ninf()) return f_ninf();
    if (cv.prefix) {
        if (prefix_blocked(p, cv, v)) return f_ninf();
        if (prefix_penalised(p, cv, v)) lp = __fsub_rn(lp, p.log_penalty);
    }
    return __fadd_rn(pr, lp);
}

// ---------------------------------------------------------------------------
// Candidate evaluation of one entry of a parent row.
// ---------------------------------------------------------------------------
struct RowCtx {
    float pr;        // parent raw score
    int new_len;     // parent length + 1
    int k;           // parent slot
    bool mask_eos;   // EOS tokens are masked (new_len < min_length)
    bool constrained;
    ConsView cv;
    Meta m;
};

// The full key of entry v with log-probability lp (finite), or 0 when the entry
// is not a candidate. The caller has already rejected NaN / +inf / -inf.
__device__ __forceinline__ uint64_t full_key(const DecodeParams& p, const RowShared& sh, const RowCtx& c, float lp,
                                             int v) {
    if (p.banned && p.banned[v]) return 0;
    if (c.mask_eos && is_eos(p, c.m, v)) return 0;
    float value = lp;
    if (c.constrained) {
        if (cons_blocked(p, sh, c.cv, v)) return 0;
        if (cons_penalised(p, sh, c.cv, v)) value = __fsub_rn(lp, p.log_penalty);
    }
    const float raw = __fadd_rn(c.pr, value);
    if (raw == f_ninf()) return 0;
    return make_key(raw, static_cast<uint32_t>(c.k) * static_cast<uint32_t>(p.V) + static_cast<uint32_t>(v));
}

// ---------------------------------------------------------------------------
// Selection of example b at step t (run by the CTA that finished its last row).
// ---------------------------------------------------------------------------
// cand / n_cand (optional, KMAX == 0): the step's candidate keys gathered in shared
// memory instead of the per-row lists in p.keys.
template <int KMAX, int KCAP>
__device__ void select_step(const DecodeParams& p, RowShared& sh, SelectShared<KCAP>& ss, int t, int b, const Meta& m,
                            const uint64_t* cand = nullptr, int n_cand = 0) {
    const int tid = threadIdx.x;
    const int K = p.K;
    const int V = p.V;
    const int64_t sbase = static_cast<int64_t>(b) * K;
    const int64_t obase = (static_cast<int64_t>(b) * p.T + t) * K;
    const bool active = t < m.steps;
    const bool last_step = p.step_api ? true : (t == p.T - 1);

    // Snapshot of the state before this step.
    for (int k = tid; k < m.beam; k += kThreads) {
        ss.s_raw[k] = ld_cg(p.raw + sbase + k);
        ss.s_len[k] = ld_cg(p.len + sbase + k);
        ss.s_ended[k] = ld_cg(p.ended + sbase + k);
        int last = -1;
        if (p.step_api) {
            const int L = ss.s_len[k];
            if (p.caller_prefix && L >= 1 && L <= p.prefix_stride)
                last = ld_cg(p.caller_prefix + (sbase + k) * p.prefix_stride + L - 1);
        } else {
            last = ld_cg(p.last + sbase + k);
        }
        ss.s_last[k] = last;
    }
    block_sync();

    int filled = 0;
    if (active) {
        // 1. The step's best m.beam scanned keys, sorted descending.
        int ns = 0;
        const uint64_t* lists = p.keys + sbase * p.list_len;
        if constexpr (KMAX > 0) {
            if (tid < 32) {
                constexpr int kPer = (kFastBeam * kFastBeam) / 32;
                const int n = K * KMAX;
                uint64_t mine[kPer];
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    const int i = tid + 32 * j;
                    mine[j] = i < n ? ld_cg(lists + i) : 0;
                }
                int r = 0;
                for (; r < m.beam; ++r) {
                    uint64_t best = 0;
#pragma unroll
                    for (int j = 0; j < kPer; ++j) best = mine[j] > best ? mine[j] : best;
                    const uint64_t w = warp_max_u64(best);
                    if (w == 0) break;
#pragma unroll
                    for (int j = 0; j < kPer; ++j)
                        if (mine[j] == w) mine[j] = 0;
                    if (tid == 0) ss.keys[r] = w;
                }
                if (tid == 0) sh.n_scanned = r;
            }
            block_sync();
            ns = sh.n_scanned;
        } else {
            bool ranked = false;
            if (cand && n_cand <= 512) {
                // Few candidates: each key's rank is the number of larger keys (unique keys).
                for (int i = tid; i < n_cand; i += kThreads) {
                    const uint64_t key = cand[i];
                    int rank = 0;
#pragma unroll 4
                    for (int j = 0; j < n_cand; ++j) rank += cand[j] > key ? 1 : 0;
                    if (rank < m.beam) ss.keys[rank] = key;
                }
                ns = n_cand < m.beam ? n_cand : m.beam;
                ranked = true;
            } else if (cand) {
                ns = block_select(
                    sh, [&](int i) { return cand[i]; }, n_cand, m.beam, [&](int pos, uint64_t key) { ss.keys[pos] = key; });
            } else {
                const int n = K * p.list_len;
                ns = block_select(
                    sh, [&](int i) { return ld_cg(lists + i); }, n, m.beam, [&](int pos, uint64_t key) { ss.keys[pos] = key; });
            }
            if (ranked) {
                block_sync();
            } else {
                int n2 = 1;
                while (n2 < ns) n2 <<= 1;
                for (int i = ns + tid; i < n2; i += kThreads) ss.keys[i] = 0;
                block_sync();
                bitonic_desc(ss.keys, n2);
            }
        }
        // 2. Scanned candidates' scores; carried-forward finished beams.
        for (int i = tid; i < ns; i += kThreads) {
            const uint32_t index = key_index(ss.keys[i]);
            const int parent = static_cast<int>(index / static_cast<uint32_t>(V));
            const float inv = __fdiv_rn(1.0f, gnmt_penalty(ss.s_len[parent] + 1, p.alpha));
            ss.sc_score[i] = __fmul_rn(key_raw(ss.keys[i]), inv);
        }
        if (tid == 0) sh.n_carry = 0;
        block_sync();
        if (m.eos >= 0) {
            for (int q = tid; q < m.beam; q += kThreads) {
                const float raw = ss.s_raw[q];
                if (ss.s_ended[q] && f_finite(raw)) {
                    const int l = ss.s_len[q] > 1 ? ss.s_len[q] : 1;
                    const int j = atomicAdd(&sh.n_carry, 1);
                    ss.c_score[j] = __fdiv_rn(raw, gnmt_penalty(l, p.alpha));
                    ss.c_raw[j] = raw;
                    ss.c_parent[j] = q;
                    ss.c_len[j] = l;
                    const int last = ss.s_last[q];
                    ss.c_token[j] = (last >= 0 && last < V && is_eos(p, m, last)) ? last : m.eos;
                }
            }
        }
        block_sync();
        const int nc = sh.n_carry;
        // 3. Merge by counting (every candidate is unique under the full order,
        //    src/common.hpp:269-276).
        auto better = [](float as, float ar, int ap, int at, int al, int af, float bs, float br, int bp, int bt, int bl,
                         int bf) {
            if (as != bs) return as > bs;
            if (ar != br) return ar > br;
            if (ap != bp) return ap < bp;
            if (at != bt) return at < bt;
            if (al != bl) return al < bl;
            return af > bf;
        };
        for (int i = tid; i < ns + nc; i += kThreads) {
            float cs, cr;
            int cp, ct, cl, cf;
            int pos;
            if (i < ns) {
                const uint32_t index = key_index(ss.keys[i]);
                cp = static_cast<int>(index / static_cast<uint32_t>(V));
                ct = static_cast<int>(index - static_cast<uint32_t>(cp) * static_cast<uint32_t>(V));
                cs = ss.sc_score[i];
                cr = key_raw(ss.keys[i]);
                cl = ss.s_len[cp] + 1;
                cf = 1;
                pos = i;
                for (int j = 0; j < nc; ++j)
                    pos += better(ss.c_score[j], ss.c_raw[j], ss.c_parent[j], ss.c_token[j], ss.c_len[j], 0, cs, cr, cp,
                                  ct, cl, cf);
            } else {
                const int j0 = i - ns;
                cs = ss.c_score[j0];
                cr = ss.c_raw[j0];
                cp = ss.c_parent[j0];
                ct = ss.c_token[j0];
                cl = ss.c_len[j0];
                cf = 0;
                pos = 0;
                for (int j = 0; j < nc; ++j)
                    pos += (j != j0) && better(ss.c_score[j], ss.c_raw[j], ss.c_parent[j], ss.c_token[j], ss.c_len[j], 0,
                                               cs, cr, cp, ct, cl, cf);
                for (int j = 0; j < ns; ++j) {
                    const uint32_t index = key_index(ss.keys[j]);
                    const int sp = static_cast<int>(index / static_cast<uint32_t>(V));
                    const int st = static_cast<int>(index - static_cast<uint32_t>(sp) * static_cast<uint32_t>(V));
                    pos += better(ss.sc_score[j], key_raw(ss.keys[j]), sp, st, ss.s_len[sp] + 1, 1, cs, cr, cp, ct, cl, cf);
                }
            }
            if (pos < m.beam) {
                ss.o_parent[pos] = cp;
                ss.o_token[pos] = ct;
                ss.o_len[pos] = cl;
                ss.o_score[pos] = cs;
                ss.o_raw[pos] = cr;
                ss.o_from[pos] = static_cast<uint8_t>(cf);
            }
        }
        filled = ns + nc < m.beam ? ns + nc : m.beam;
        block_sync();
    }

    // 4. Emit the step's slots and the new state.
    const int cur = t & 1, nxt = (t + 1) & 1;
    for (int k = tid; k < K; k += kThreads) {
        const int64_t o = obase + k;
        const int64_t s = sbase + k;
        if (k < filled) {
            const int par = ss.o_parent[k];
            const int tok = ss.o_token[k];
            if (p.out.tokens) p.out.tokens[o] = tok;
            if (p.out.parents) p.out.parents[o] = par;
            if (p.out.lengths) p.out.lengths[o] = ss.o_len[k];
            if (p.out.scores) p.out.scores[o] = ss.o_score[k];
            if (p.out.raw_scores) p.out.raw_scores[o] = ss.o_raw[k];
            if (p.out.from_logprob) p.out.from_logprob[o] = ss.o_from[k];
            p.raw[s] = ss.o_raw[k];
            p.len[s] = ss.o_len[k];
            p.ended[s] = static_cast<uint8_t>(ss.o_from[k] ? (ss.s_ended[par] != 0 || is_eos(p, m, tok)) : 1);
            if (!p.step_api) p.last[s] = tok;
        } else {
            if (p.out.tokens) p.out.tokens[o] = -1;
            if (p.out.parents) p.out.parents[o] = -1;
            if (p.out.lengths) p.out.lengths[o] = 0;
            if (p.out.scores) p.out.scores[o] = f_ninf();
            if (p.out.raw_scores) p.out.raw_scores[o] = f_ninf();
            if (p.out.from_logprob) p.out.from_logprob[o] = 0;
            if (active) {
                p.raw[s] = f_ninf();
                p.len[s] = 0;
                p.ended[s] = 0;
                if (!p.step_api) p.last[s] = -1;
            }
        }
    }
    // Prefixes of the new hypotheses (decode with constraints): parent's, plus the emitted token.
    if (active && p.prefix[0] && !p.step_api) {
        const int T = p.T;
        for (int k = 0; k < K; ++k) {
            int32_t* dst = p.prefix[nxt] + (sbase + k) * T;
            if (k < filled) {
                const int par = ss.o_parent[k];
                const int32_t* src = p.prefix[cur] + (sbase + par) * T;
                const int L = ld_cg(p.prefix_len[cur] + sbase + par);
                for (int i = tid; i < L; i += kThreads) dst[i] = ld_cg(src + i);
                const bool append = ss.o_from[k] && ss.o_token[k] >= 0 && L < T;
                if (tid == 0) {
                    if (append) dst[L] = ss.o_token[k];
                    p.prefix_len[nxt][sbase + k] = L + (append ? 1 : 0);
                }
            } else if (tid == 0) {
                p.prefix_len[nxt][sbase + k] = 0;
            }
        }
    } else if (!active && p.prefix[0] && !p.step_api) {
        // Inactive step: carry the prefixes over unchanged.
        const int T = p.T;
        for (int k = 0; k < K; ++k) {
            const int L = ld_cg(p.prefix_len[cur] + sbase + k);
            for (int i = tid; i < L; i += kThreads)
                p.prefix[nxt][(sbase + k) * T + i] = ld_cg(p.prefix[cur] + (sbase + k) * T + i);
            if (tid == 0) p.prefix_len[nxt][sbase + k] = L;
        }
    }
    block_sync();
    // 5. Final scores after the last step.
    if (last_step && p.out.final_scores) {
        for (int k = tid; k < K; k += kThreads) {
            const int64_t s = sbase + k;
            float raw = f_ninf(), score = f_ninf();
            int len = 0;
            if (k < m.beam) {
                raw = p.raw[s];
                len = p.len[s];
                score = __fdiv_rn(raw, gnmt_penalty(len, p.alpha));
            }
            p.out.final_scores[s] = score;
            if (p.out.final_raw_scores) p.out.final_raw_scores[s] = raw;
            if (p.out.final_lengths) p.out.final_lengths[s] = len;
        }
    }
    __threadfence();  // the new state, prefixes and trace, before the caller publishes the step
    block_sync();
}

// ---------------------------------------------------------------------------
// The persistent decode kernel.
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Warp-cooperative top-k for beams up to 16: lane j < KMAX of a warp holds the
// warp's j-th best key so far (descending; 0 = empty). Each round every lane
// offers one key; a ballot picks the offers that beat the warp's K-th key and
// they are inserted one at a time by the whole warp, so the warp never diverges
// and a rejected offer costs one compare.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t shfl_u64(uint64_t v, int src) {
    const uint32_t lo = __shfl_sync(0xffffffffu, static_cast<uint32_t>(v), src);
    const uint32_t hi = __shfl_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), src);
    return (static_cast<uint64_t>(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t shfl_up_u64(uint64_t v, int d) {
    const uint32_t lo = __shfl_up_sync(0xffffffffu, static_cast<uint32_t>(v), d);
    const uint32_t hi = __shfl_up_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), d);
    return (static_cast<uint64_t>(hi) << 32) | lo;
}

template <int KMAX>
struct WarpTopK {
    uint64_t wl;   // this lane's entry (lanes < KMAX)
    uint64_t tk;   // the KMAX-th best key of the warp (0 while the list is not full)
    float thr;     // raw-score filter: no candidate with raw < thr can enter
    float thr0;    // filter bound known before the scan (pass 1)

    __device__ __forceinline__ void init(float bound) {
        wl = 0;
        tk = 0;
        thr0 = bound;
        thr = bound;
    }
    __device__ __forceinline__ void offer(uint64_t key, int lane) {
        unsigned m = __ballot_sync(0xffffffffu, key > tk);
        while (m) {
            const int src = __ffs(m) - 1;
            const uint64_t kk = shfl_u64(key, src);
            const int pos = __popc(__ballot_sync(0xffffffffu, lane < KMAX && wl > kk));
            const uint64_t up = shfl_up_u64(wl, 1);
            if (lane < KMAX) {
                if (lane == pos) wl = kk;
                else if (lane > pos) wl = up;
            }
            tk = shfl_u64(wl, KMAX - 1);
            if (tk != 0) thr = fmaxf(thr0, key_raw(tk));
            m &= m - 1;
            m &= __ballot_sync(0xffffffffu, key > tk);
        }
    }
};

// One float per lane sorted descending across the warp (lane 0 = largest), by a bitonic network.
__device__ __forceinline__ float warp_sort_desc(float v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float o = __shfl_xor_sync(0xffffffffu, v, j);
            const bool take_max = ((lane & j) == 0) == ((lane & k) == 0);
            v = take_max ? fmaxf(v, o) : fminf(v, o);
        }
    }
    return v;
}

// The r-th largest (r in [1, 32]) of one float per lane, by a bitonic sort of the warp.
__device__ __forceinline__ float warp_rth_largest(float v, int r) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float o = __shfl_xor_sync(0xffffffffu, v, j);
            const bool lower = (lane & j) == 0;
            const bool desc = (lane & k) == 0;
            // descending blocks keep the larger value in the lower lane
            const bool take_max = (lower == desc);
            v = take_max ? fmaxf(v, o) : fminf(v, o);
        }
    }
    return __shfl_sync(0xffffffffu, v, r - 1);
}

// ---------------------------------------------------------------------------
// The smallest float x with raw(x) >= thr, for raw non-decreasing in x with
// raw(-inf) < thr <= raw(+inf): galloping from an estimate, then bisection, over
// the order-preserving integer image of the floats (about 2 log2(gap) calls).
// ---------------------------------------------------------------------------
__device__ __forceinline__ int32_t float_ord(float x) {
    const int32_t u = __float_as_int(x);
    return u >= 0 ? u : static_cast<int32_t>(0x80000000u - static_cast<uint32_t>(u));
}
__device__ __forceinline__ float ord_float(int32_t o) {
    return __int_as_float(o >= 0 ? o : static_cast<int32_t>(0x80000000u - static_cast<uint32_t>(o)));
}

template <class Raw>
__device__ __forceinline__ float smallest_x_reaching(float est, float thr, Raw&& raw) {
    const int32_t kLo = float_ord(f_ninf()), kHi = float_ord(f_inf());
    int32_t e = (est == est) ? float_ord(est) : 0;  // a NaN estimate starts from 0
    if (e < kLo) e = kLo;
    if (e > kHi) e = kHi;
    int32_t lo, hi;
    if (raw(ord_float(e)) >= thr) {
        hi = e;
        int64_t step = 1;
        lo = hi;
        do {
            lo = static_cast<int32_t>(static_cast<int64_t>(hi) - step > kLo ? static_cast<int64_t>(hi) - step : kLo);
            if (raw(ord_float(lo)) < thr) break;
            hi = lo;
            step <<= 1;
        } while (lo > kLo);
        if (lo == hi) return ord_float(hi);  // reached -inf with raw(-inf) >= thr: no filtering
    } else {
        lo = e;
        int64_t step = 1;
        hi = lo;
        do {
            hi = static_cast<int32_t>(static_cast<int64_t>(lo) + step < kHi ? static_cast<int64_t>(lo) + step : kHi);
            if (raw(ord_float(hi)) >= thr) break;
            lo = hi;
            step <<= 1;
        } while (hi < kHi);
        if (raw(ord_float(hi)) < thr) return f_inf();
    }
    // raw(lo) < thr <= raw(hi)
    while (hi - lo > 1) {
        const int32_t mid = lo + (hi - lo) / 2;
        if (raw(ord_float(mid)) >= thr) hi = mid;
        else lo = mid;
    }
    return ord_float(hi);
}

// ---------------------------------------------------------------------------
// Row split into 16-byte chunks plus ragged ends. Chunk c (c < nvec) covers
// entries [head + c*PER, head + (c+1)*PER) and belongs to thread c mod 256; the
// ragged ends (under 16 bytes before the first and after the last chunk) belong
// to threads 0..n_ends-1. Passes 1 and 3 both use this assignment, which is what
// lets pass 1's per-thread maxima bound pass 3's warp lists.
// ---------------------------------------------------------------------------
struct RowSplit {
    int V, head, nvec, tail0, per;

    template <int EB>
    __device__ __forceinline__ static RowSplit of(const char* row, int V) {
        RowSplit r;
        r.V = V;
        r.per = 16 / EB;
        const uintptr_t a = reinterpret_cast<uintptr_t>(row);
        int head = static_cast<int>(((16 - (a & 15)) & 15) / EB);
        if (head > V) head = V;
        r.head = head;
        r.nvec = (V - head) / r.per;
        r.tail0 = head + r.nvec * r.per;
        return r;
    }
    __device__ __forceinline__ int n_ends() const { return head + (V - tail0); }
    __device__ __forceinline__ int end_entry(int i) const { return i < head ? i : tail0 + (i - head); }
    // Whether the calling thread owns entry v.
    __device__ __forceinline__ bool owns(int v) const {
        if (v < 0 || v >= V) return false;
        const int tid = threadIdx.x;
        if (v < head) return tid == v;
        if (v >= tail0) return tid == head + (v - tail0);
        return ((v - head) / per) % kThreads == tid;
    }
};

template <int DT>
__device__ __forceinline__ void unpack16(const uint4& q, float (&x)[16 / Elem<DT>::kBytes]) {
    using E = Elem<DT>;
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if constexpr (E::kBytes == 4) {
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = __uint_as_float(w[j]);
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[2 * j] = E::to_f32(static_cast<uint16_t>(w[j] & 0xffffu));
            x[2 * j + 1] = E::to_f32(static_cast<uint16_t>(w[j] >> 16));
        }
    }
}

__device__ __forceinline__ uint4 ld_v4(const void* p, bool smem) {
    return smem ? *reinterpret_cast<const uint4*>(p) : ld_stream_v4(p);
}

// f(x, v) for every entry the calling thread owns (per-thread trip counts).
template <int DT, class F>
__device__ __forceinline__ void for_chunks(const char* row, const RowSplit& rs, bool smem, F&& f) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    const int tid = threadIdx.x;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    int c = tid;
    for (; c + kThreads < rs.nvec; c += 2 * kThreads) {
        const uint4 q0 = ld_v4(body + static_cast<size_t>(c) * 16, smem);
        const uint4 q1 = ld_v4(body + static_cast<size_t>(c + kThreads) * 16, smem);
        float x0[PER], x1[PER];
        unpack16<DT>(q0, x0);
        unpack16<DT>(q1, x1);
#pragma unroll
        for (int j = 0; j < PER; ++j) f(x0[j], rs.head + c * PER + j);
#pragma unroll
        for (int j = 0; j < PER; ++j) f(x1[j], rs.head + (c + kThreads) * PER + j);
    }
    for (; c < rs.nvec; c += kThreads) {
        float x0[PER];
        unpack16<DT>(ld_v4(body + static_cast<size_t>(c) * 16, smem), x0);
#pragma unroll
        for (int j = 0; j < PER; ++j) f(x0[j], rs.head + c * PER + j);
    }
    if (tid < rs.n_ends()) {
        const int v = rs.end_entry(tid);
        f(load_elem<DT>(row, v), v);
    }
}

// Warp-uniform scan by a group of NT threads (local index ltid): chunk c belongs to
// thread c mod NT, the ragged ends to threads 0..n_ends-1. test(x) on every owned
// entry; a chunk round in which any lane of the warp has a hit calls hit(x, v, valid)
// for each of its PER entries on every lane (valid = the lane owns the entry), so the
// callee may use warp collectives.
template <int DT, int NT, class Test, class Hit>
__device__ __forceinline__ void scan_chunks_ballot_n(const char* row, const RowSplit& rs, bool smem, int ltid,
                                                     Test&& test, Hit&& hit) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    const int rounds = (rs.nvec + NT - 1) / NT;
    for (int r = 0; r < rounds; ++r) {
        const int c = ltid + r * NT;
        const bool valid = c < rs.nvec;
        float x[PER];
        if (valid) {
            unpack16<DT>(ld_v4(body + static_cast<size_t>(c) * 16, smem), x);
        } else {
#pragma unroll
            for (int j = 0; j < PER; ++j) x[j] = f_ninf();
        }
        bool any = false;
#pragma unroll
        for (int j = 0; j < PER; ++j) any |= test(x[j]) && valid;
        if (__ballot_sync(0xffffffffu, any)) {
            // Rolled loop over the chunk's entries; the array shifts through registers so
            // it is never indexed dynamically.
#pragma unroll 1
            for (int j = 0; j < PER; ++j) {
                hit(x[0], rs.head + c * PER + j, valid);
#pragma unroll
                for (int q = 0; q + 1 < PER; ++q) x[q] = x[q + 1];
            }
        }
    }
    // Ragged ends: one round for every warp of the group.
    {
        const bool valid = ltid < rs.n_ends();
        const int v = valid ? rs.end_entry(ltid) : 0;
        const float x = valid ? load_elem<DT>(row, v) : f_ninf();
        const bool any = valid && test(x);
        if (__ballot_sync(0xffffffffu, any)) hit(x, v, valid);
    }
}

// The same over the whole CTA, chunk c on thread c mod 256 (the pass-1 assignment).
template <int DT, class Test, class Hit>
__device__ __forceinline__ void scan_chunks_ballot(const char* row, const RowSplit& rs, bool smem, Test&& test,
                                                   Hit&& hit) {
    scan_chunks_ballot_n<DT, kThreads>(row, rs, smem, static_cast<int>(threadIdx.x), test, hit);
}

// ---------------------------------------------------------------------------
// Row preparation, independent of the previous step's selection: stage the row
// in shared memory (optional), pass 1 (maximum, NaN/+inf flag, per-thread
// maxima for the filter bound), pass 2 (logsumexp, from logits only).
// ---------------------------------------------------------------------------
struct Prep {
    const char* src;   // the row (shared memory when staged)
    RowSplit rs;
    float lse;         // logsumexp (from logits), -inf for a row without finite entries
    float xthr;        // lower bound on the row's R-th best eligible entry (-inf: none)
    bool invalid;      // NaN/+inf in the row (valid when inv_known)
    bool inv_known;
    bool aborted;      // the staging copy timed out (error word set)
};

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
// Barrier among the 128 threads of warps 0-3 (id 2) or of warps 4-7 (id 1).
__device__ __forceinline__ void half_sync(int id) { asm volatile("barrier.sync %0, 128;" ::"r"(id) : "memory"); }

// The R-th largest (R <= RCAP) of NW warps' sorted per-thread bounds (warp w's R
// largest at wtop[w * RCAP + r], descending), written to *out by a group of NT threads
// (local index ltid): every value finds its rank in the total order (value, then warp
// index) by a binary search of each other warp's list; the value of rank R - 1 wins.
template <int NW, int RCAP, int NT>
__device__ __forceinline__ void rank_rth(const float* wtop, int R, int ltid, float* out) {
    for (int i = ltid; i < NW * R; i += NT) {
        const int w = i / R, r = i - w * R;
        const float v = wtop[w * RCAP + r];
        int rank = r;
        for (int w2 = 0; w2 < NW; ++w2) {
            if (w2 == w) continue;
            const float* list = wtop + w2 * RCAP;
            int lo = 0, hi = R;  // entries of w2 ahead of (v, w) form a prefix
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                const float e = list[mid];
                if (e > v || (e == v && w2 < w)) lo = mid + 1;
                else hi = mid;
            }
            rank += lo;
        }
        if (rank == R - 1) *out = v;
    }
}

// The R-th largest of the warps' sorted thread maxima (R <= kWarps * RCAP) into
// sh.xbound, by the 128 threads of warps 4-7: R <= RCAP ranks the R largest of each warp;
// larger R ranks every value of the RCAP-entry lists.
template <int RCAP>
__device__ __forceinline__ void bound_rank(RowShared& sh, int R, int ltid) {
    if (R <= RCAP) {
        rank_rth<kWarps, RCAP, kThreads / 2>(sh.wtop, R, ltid, &sh.xbound);
        return;
    }
    for (int i = ltid; i < kWarps * RCAP; i += kThreads / 2) {
        const int w = i / RCAP, r = i - w * RCAP;
        const float v = sh.wtop[i];
        int rank = r;
        for (int w2 = 0; w2 < kWarps; ++w2) {
            if (w2 == w) continue;
            const float* list = sh.wtop + w2 * RCAP;
            int lo = 0, hi = RCAP;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                const float e = list[mid];
                if (e > v || (e == v && w2 < w)) lo = mid + 1;
                else hi = mid;
            }
            rank += lo;
        }
        if (rank == R - 1) sh.xbound = v;
    }
}

// Rank merge of sorted warp lists: warp lw of `nl` list warps holds its LIST best keys
// in lanes 0..LIST-1 (descending, zeros last, keys unique). Each key's rank is its
// position plus the number of larger keys in the other lists (binary search); keys
// of rank < LIST go to out[rank]. Called by the nl list warps only, after their lists
// are in wkeys[w * LIST + lane].
template <int LIST>
__device__ __forceinline__ void rank_merge(const uint64_t* wkeys, int nl, int lw, uint64_t key, uint64_t* out) {
    const int lane = threadIdx.x & 31;
    if (lane < LIST && key != 0) {
        int rank = lane;
        for (int w2 = 0; w2 < nl; ++w2) {
            if (w2 == lw) continue;
            const uint64_t* list = wkeys + w2 * LIST;
            int lo = 0, hi = LIST;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (list[mid] > key) lo = mid + 1;
                else hi = mid;
            }
            rank += lo;
        }
        if (rank < LIST) out[rank] = key;
    }
}

// Entries of a staged row owned by thread ltid of an NT-thread group (chunk c on thread
// c mod NT, ragged ends on threads 0..n_ends-1), in increasing v.
template <int DT, int NT, class F>
__device__ __forceinline__ void for_chunks_n(const char* row, const RowSplit& rs, int ltid, F&& f) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    int c = ltid;
    for (; c + NT < rs.nvec; c += 2 * NT) {
        const uint4 q0 = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16);
        const uint4 q1 = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c + NT) * 16);
        float x0[PER], x1[PER];
        unpack16<DT>(q0, x0);
        unpack16<DT>(q1, x1);
#pragma unroll
        for (int j = 0; j < PER; ++j) f(x0[j], rs.head + c * PER + j);
#pragma unroll
        for (int j = 0; j < PER; ++j) f(x1[j], rs.head + (c + NT) * PER + j);
    }
    for (; c < rs.nvec; c += NT) {
        float x0[PER];
        unpack16<DT>(*reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16), x0);
#pragma unroll
        for (int j = 0; j < PER; ++j) f(x0[j], rs.head + c * PER + j);
    }
    if (ltid < rs.n_ends()) {
        const int v = rs.end_entry(ltid);
        f(load_elem<DT>(row, v), v);
    }
}
// ---------------------------------------------------------------------------
// Packed 16-bit pairs (bf16x2 / f16x2 in one 32-bit register). max and min never
// round, so pass 1 and the record scan can work on pairs: running max / min over a
// thread's chunks, and a chunk test "largest entry >= threshold" (every threshold
// is itself an input value or -inf, so the 16-bit comparison is exact).
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ uint32_t h2_max_nan(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT == 2) asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <int DT>
__device__ __forceinline__ uint32_t h2_max(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT == 2) asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <int DT>
__device__ __forceinline__ uint32_t h2_min(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT == 2) asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <int DT>
__device__ __forceinline__ float h2_lo(uint32_t w) { return Elem<DT>::to_f32(static_cast<uint16_t>(w & 0xffffu)); }
template <int DT>
__device__ __forceinline__ float h2_hi(uint32_t w) { return Elem<DT>::to_f32(static_cast<uint16_t>(w >> 16)); }
template <int DT>
constexpr uint32_t h2_ninf() { return DT == 2 ? 0xff80ff80u : 0xfc00fc00u; }
template <int DT>
constexpr uint32_t h2_inf() { return DT == 2 ? 0x7f807f80u : 0x7c007c00u; }

// Pass 1 of a staged row over one group: NaN-propagating maximum and minimum of the
// entries the thread owns (for_chunks_n's assignment).
template <int DT, int NT>
__device__ __forceinline__ void group_pass1(const char* row, const RowSplit& rs, int ltid, float& mxn, float& mn) {
    using E = Elem<DT>;
    mxn = f_ninf();
    mn = f_inf();
    if constexpr (E::kBytes == 2) {
        const char* body = row + static_cast<size_t>(rs.head) * 2;
        uint32_t mx2 = h2_ninf<DT>(), mn2 = h2_inf<DT>();
        int c = ltid;
        for (; c + NT < rs.nvec; c += 2 * NT) {
            const uint4 q0 = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16);
            const uint4 q1 = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c + NT) * 16);
            mx2 = h2_max_nan<DT>(mx2, h2_max_nan<DT>(h2_max_nan<DT>(q0.x, q0.y), h2_max_nan<DT>(q0.z, q0.w)));
            mn2 = h2_min<DT>(mn2, h2_min<DT>(h2_min<DT>(q0.x, q0.y), h2_min<DT>(q0.z, q0.w)));
            mx2 = h2_max_nan<DT>(mx2, h2_max_nan<DT>(h2_max_nan<DT>(q1.x, q1.y), h2_max_nan<DT>(q1.z, q1.w)));
            mn2 = h2_min<DT>(mn2, h2_min<DT>(h2_min<DT>(q1.x, q1.y), h2_min<DT>(q1.z, q1.w)));
        }
        for (; c < rs.nvec; c += NT) {
            const uint4 q0 = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16);
            mx2 = h2_max_nan<DT>(mx2, h2_max_nan<DT>(h2_max_nan<DT>(q0.x, q0.y), h2_max_nan<DT>(q0.z, q0.w)));
            mn2 = h2_min<DT>(mn2, h2_min<DT>(h2_min<DT>(q0.x, q0.y), h2_min<DT>(q0.z, q0.w)));
        }
        mxn = max_nan(h2_lo<DT>(mx2), h2_hi<DT>(mx2));
        mn = fminf(h2_lo<DT>(mn2), h2_hi<DT>(mn2));
        if (ltid < rs.n_ends()) {
            const float x = load_elem<DT>(row, rs.end_entry(ltid));
            mxn = max_nan(mxn, x);
            mn = fminf(mn, x);
        }
    } else {
        for_chunks_n<DT, NT>(row, rs, ltid, [&](float x, int) {
            mxn = max_nan(mxn, x);
            mn = fminf(mn, x);
        });
    }
}

// The record scan's ballot loop over one group: a chunk whose largest entry reaches
// thr() is a hit; hit(x, v, valid) is then called for each of its entries on every
// lane of the warp (valid = the lane owns the entry), so it may use warp collectives.
template <int DT, int NT, class Thr, class Hit>
__device__ __forceinline__ void group_scan(const char* row, const RowSplit& rs, int ltid, Thr&& thr, Hit&& hit) {
    using E = Elem<DT>;
    if constexpr (E::kBytes == 2) {
        const char* body = row + static_cast<size_t>(rs.head) * 2;
        const int rounds = (rs.nvec + NT - 1) / NT;
        for (int r = 0; r < rounds; ++r) {
            const int c = ltid + r * NT;
            const bool valid = c < rs.nvec;
            uint4 q = make_uint4(h2_ninf<DT>(), h2_ninf<DT>(), h2_ninf<DT>(), h2_ninf<DT>());
            if (valid) q = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16);
            const uint32_t m2 = h2_max<DT>(h2_max<DT>(q.x, q.y), h2_max<DT>(q.z, q.w));
            const float top = fmaxf(h2_lo<DT>(m2), h2_hi<DT>(m2));
            if (__ballot_sync(0xffffffffu, valid && top >= thr())) {
                uint32_t w0 = q.x, w1 = q.y, w2 = q.z, w3 = q.w;
#pragma unroll 1
                for (int j = 0; j < 8; ++j) {
                    const float x = (j & 1) ? h2_hi<DT>(w0) : h2_lo<DT>(w0);
                    hit(x, rs.head + c * 8 + j, valid);
                    if (j & 1) {
                        w0 = w1;
                        w1 = w2;
                        w2 = w3;
                    }
                }
            }
        }
        const bool valid = ltid < rs.n_ends();
        const int v = valid ? rs.end_entry(ltid) : 0;
        const float x = valid ? load_elem<DT>(row, v) : f_ninf();
        if (__ballot_sync(0xffffffffu, valid && x >= thr())) hit(x, v, valid);
    } else {
        scan_chunks_ballot_n<DT, NT>(row, rs, true, ltid, [&](float x) { return x >= thr(); }, hit);
    }
}

// Entries (v, v + 1) of a row as a packed pair (v even; the pair is aligned).
template <int DT>
__device__ __forceinline__ uint64_t load_pair(const char* row, int v) {
    if constexpr (DT == 0) {
        return *reinterpret_cast<const uint64_t*>(row + static_cast<size_t>(v) * 4);
    } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(row + static_cast<size_t>(v) * 2);
        return f2_pack(Elem<DT>::to_f32(static_cast<uint16_t>(w & 0xffffu)), Elem<DT>::to_f32(static_cast<uint16_t>(w >> 16)));
    }
}

// Pass 2 over the full 256-entry blocks for logsumexp lanes (2j, 2j + 1): thread j sums
// exp(x - max) of both lanes in increasing v, packed. MASKED: entries with x - max below
// -87 contribute +0 (adding +0 leaves a non-negative sum unchanged). stride: entries per
// block in `row` (a vocabulary shard holds stride of each block's 256 lanes).
template <int DT, bool MASKED, int UR = 4>
__device__ __forceinline__ uint64_t lane_pair_sums(const Pack2& q, const char* row, int nfull, float mx, int j,
                                                   int stride = kLanes) {
    const uint64_t mx2 = f2_splat(mx);
    uint64_t acc = f2_pack(0.0f, 0.0f);
    auto one = [&](uint64_t x2) {
        const uint64_t d = f2_sub(q, x2, mx2);
        float lo, hi;
        exp_nonpositive_fast2(q, d, lo, hi);
        if constexpr (MASKED) {
            float d_lo, d_hi;
            f2_unpack(d, d_lo, d_hi);
            uint32_t k_lo, k_hi;
            asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(k_lo) : "f"(d_lo), "f"(cephes::kMin));
            asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(k_hi) : "f"(d_hi), "f"(cephes::kMin));
            lo = __uint_as_float(__float_as_uint(lo) & k_lo);
            hi = __uint_as_float(__float_as_uint(hi) & k_hi);
        }
        return f2_pack(lo, hi);
    };
    int i = 0;
    for (; i + UR <= nfull; i += UR) {
        uint64_t x2[UR];
#pragma unroll
        for (int u = 0; u < UR; ++u) x2[u] = load_pair<DT>(row, (i + u) * stride + 2 * j);
        uint64_t e[UR];
#pragma unroll
        for (int u = 0; u < UR; ++u) e[u] = one(x2[u]);
#pragma unroll
        for (int u = 0; u < UR; ++u) acc = f2_add(q, acc, e[u]);
    }
    for (; i < nfull; ++i) acc = f2_add(q, acc, one(load_pair<DT>(row, i * stride + 2 * j)));
    return acc;
}

// One entry of a row in shared memory, widened to float.
template <int DT>
__device__ __forceinline__ float lds_elem(uint32_t a) {
    if constexpr (Elem<DT>::kBytes == 4) {
        float x;
        asm("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(a));
        return x;
    } else {
        uint16_t h;
        asm("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
        return Elem<DT>::to_f32(h);
    }
}

// One entry of a row in global memory (read-only for the kernel), widened to float.
template <int DT>
__device__ __forceinline__ float ldg_elem(const char* a) {
    if constexpr (Elem<DT>::kBytes == 4) return __ldg(reinterpret_cast<const float*>(a));
    else return Elem<DT>::to_f32(__ldg(reinterpret_cast<const unsigned short*>(a)));
}

// Logsumexp lane j of a row on one thread (all eight warps take part, one lane each):
// exp(x - max) over v = j, j + 256, ... in increasing v, the entries of two consecutive
// blocks evaluated as one packed pair and added to the lane sum in order. a: lane j's first
// entry (a shared address or a global pointer), ld(a): one entry. MASKED: entries with
// x - max below -87 contribute +0.
template <int DT, bool MASKED, int UR, class Addr, class Load>
__device__ __forceinline__ float lane_sum_loop(Addr a, int V, float mx, int j, const Pack2& q, Load&& ld) {
    constexpr uint32_t kStride = kLanes * Elem<DT>::kBytes;  // bytes between consecutive entries of a lane
    const int nfull = V / kLanes;
    const int nb = nfull + (j < V - nfull * kLanes ? 1 : 0);
    const uint64_t mx2 = f2_splat(mx);
    auto ex2 = [&](float x0, float x1, float& e0, float& e1) {
        const uint64_t d = f2_sub(q, f2_pack(x0, x1), mx2);
        exp_nonpositive_fast2(q, d, e0, e1);
        if constexpr (MASKED) {
            float d0, d1;
            f2_unpack(d, d0, d1);
            uint32_t k0, k1;
            asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(k0) : "f"(d0), "f"(cephes::kMin));
            asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(k1) : "f"(d1), "f"(cephes::kMin));
            e0 = __uint_as_float(__float_as_uint(e0) & k0);
            e1 = __uint_as_float(__float_as_uint(e1) & k1);
        }
    };
    float acc = 0.0f;
    int i = 0;
    for (; i + 2 * UR <= nb; i += 2 * UR, a += 2 * UR * kStride) {
        float ea[UR], eb[UR];
#pragma unroll
        for (int u = 0; u < UR; ++u) ex2(ld(a + 2 * u * kStride), ld(a + (2 * u + 1) * kStride), ea[u], eb[u]);
#pragma unroll
        for (int u = 0; u < UR; ++u) {
            acc = __fadd_rn(acc, ea[u]);
            acc = __fadd_rn(acc, eb[u]);
        }
    }
    for (; i + 2 <= nb; i += 2, a += 2 * kStride) {
        float ea, eb;
        ex2(ld(a), ld(a + kStride), ea, eb);
        acc = __fadd_rn(acc, ea);
        acc = __fadd_rn(acc, eb);
    }
    if (i < nb) acc = __fadd_rn(acc, exp_nonpositive_masked(__fsub_rn(ld(a), mx)));
    return acc;
}

// lane_sum_loop over a row staged at shared address `row`, and over a row in global
// memory. Functions of their own, so that the loop is scheduled with the kernel's whole
// register budget whatever state the chained kernel holds across the row (that state is
// saved once per row at the call). Measured on its own (the C2 rows, three CTAs per SM), the
// staged form runs as fast as the same loop written inline.
template <int DT, bool MASKED, int UR = 2>
__device__ __noinline__ float lane_sum_staged(uint32_t row, int V, float mx, int j, uint64_t one2, uint64_t nzero2) {
    const Pack2 q{one2, nzero2};
    return lane_sum_loop<DT, MASKED, UR>(row + static_cast<uint32_t>(j) * Elem<DT>::kBytes, V, mx, j, q,
                                         [](uint32_t a) { return lds_elem<DT>(a); });
}
template <int DT, bool MASKED, int UR = 2>
__device__ __noinline__ float lane_sum_global(const char* row, int V, float mx, int j, uint64_t one2, uint64_t nzero2) {
    const Pack2 q{one2, nzero2};
    return lane_sum_loop<DT, MASKED, UR>(row + static_cast<size_t>(j) * Elem<DT>::kBytes, V, mx, j, q,
                                         [](const char* a) { return ldg_elem<DT>(a); });
}

// Where the chained decode's from-logits record goes and which entries it may hold.
struct RecordOut {
    uint64_t* out;    // the row's LIST record keys
    int list;         // LIST
    bool mask_eos;    // EOS tokens excluded (the parent is shorter than min_length - 1)
    bool exclusions;  // banned tokens excluded
};

constexpr int kCandCap = kWarps * 32;  // record candidates collected in RowShared::wkeys

// The record candidates of a staged row: every eligible entry at or above the filter
// bound xb, as keys in sh.wkeys[0, min(count, kCandCap)) with their number in sh.count.
// Only a thread whose own maximum (pass 1's chunk assignment: chunk c on thread c mod 256,
// ragged end i on thread i) reaches xb can own such an entry. Each warp takes its own
// such threads one at a time and looks at a thread's chunks with all 32 lanes at once
// (a lane per chunk), so no warp diverges into a long per-thread loop before pass 2.
template <int DT>
__device__ __forceinline__ void collect_candidates(const DecodeParams& p, RowShared& sh, const char* row,
                                                   const RowSplit& rs, float xb, bool mine, const Meta& m,
                                                   const RecordOut& ro) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    const int lane = threadIdx.x & 31;
    const int wbase = threadIdx.x & ~31;
    auto eligible = [&](float x, int v) {
        return x >= xb && !(ro.exclusions && p.banned[v]) && !(ro.mask_eos && is_eos(p, m, v));
    };
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    unsigned owners = __ballot_sync(0xffffffffu, mine);
    while (owners) {
        const int q = wbase + __ffs(owners) - 1;  // the owning thread
        owners &= owners - 1;
        for (int i0 = 0; q + i0 * kThreads < rs.nvec; i0 += 32) {
            const int c = q + (i0 + lane) * kThreads;
            float x[PER];
            unsigned mask = 0;
            if (c < rs.nvec) {
                unpack16<DT>(*reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16), x);
                const int v0 = rs.head + c * PER;
#pragma unroll
                for (int jj = 0; jj < PER; ++jj) mask |= eligible(x[jj], v0 + jj) ? 1u << jj : 0u;
            }
            if (mask) {
                int slot = atomicAdd(&sh.count, __popc(mask));
                const int v0 = rs.head + c * PER;
#pragma unroll
                for (int jj = 0; jj < PER; ++jj) {
                    if ((mask >> jj) & 1u) {
                        if (slot < kCandCap) sh.wkeys[slot] = make_key(x[jj], static_cast<uint32_t>(v0 + jj));
                        ++slot;
                    }
                }
            }
        }
        if (lane == 0 && q < rs.n_ends()) {
            const int v = rs.end_entry(q);
            const float x = load_elem<DT>(row, v);
            if (eligible(x, v)) {
                const int slot = atomicAdd(&sh.count, 1);
                if (slot < kCandCap) sh.wkeys[slot] = make_key(x, static_cast<uint32_t>(v));
            }
        }
    }
}

// The record from the collected candidates by one warp: each key's rank is the number of
// larger keys (keys are unique); ranks below LIST are written. The list count goes to
// sh.nlist[4] (the first list warp's slot; the other list warps' slots are zero), as the
// list warps' record scan would leave it.
__device__ __forceinline__ void record_from_candidates(RowShared& sh, int n, const RecordOut& ro) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < n; i += 32) {
        const uint64_t key = sh.wkeys[i];
        int rank = 0;
        for (int k2 = 0; k2 < n; ++k2) rank += sh.wkeys[k2] > key ? 1 : 0;
        if (rank < ro.list) ro.out[rank] = key;
    }
    if (lane < kWarps / 2) sh.nlist[kWarps / 2 + lane] = lane == 0 ? (n < ro.list ? n : ro.list) : 0;
}

// Row preparation, independent of the previous step's selection: stage the row in
// shared memory (optional); pass 1: maximum, minimum, NaN/+inf flag and the per-thread
// maxima behind the filter bound; from logits, pass 2: logsumexp on warps 0-3 (two
// lanes per thread, packed) while warps 4-7 compute the bound and then run
// side(src, rs, xthr), e.g. the chained decode's record scan. RCAP: capacity of the
// bound (R <= RCAP <= 32). want_bound: the candidates are not subject to exclusions
// the per-thread maxima cannot see (banned tokens, constraints).
//
// ro (from logits, rows with a bound, staged or not): the whole CTA runs pass 2 instead, one
// logsumexp lane per thread, after the threads whose maximum reaches the bound have
// collected the record candidates; warp 4 then ranks them into ro->out while warps 0-3
// reduce the lanes, and side() runs only when the candidates overflow kCandCap or no
// bound exists.
template <int DT, bool LOGITS, int RCAP, class Side>
__device__ __forceinline__ void prepare_row(const DecodeParams& p, RowShared& sh, char* srow, const char* grow,
                                            uint32_t& phase, bool use_smem, bool want_bound, int R, const Meta& m,
                                            Prep& o, Side&& side, const RecordOut* ro = nullptr) {
    using E = Elem<DT>;
    constexpr int EB = E::kBytes;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int V = p.V;
    o.src = grow;
    o.lse = 0.0f;
    o.xthr = f_ninf();
    o.invalid = false;
    o.inv_known = false;
    o.aborted = false;
    int soff = 0;
    if (use_smem) {
        bool ok = true;
        soff = stage_row<EB>(p, sh, srow, grow, V, phase, ok);
        o.src = srow + soff;
        if (!ok) {
            o.aborted = true;
            return;
        }
    }
    const char* src = o.src;
    o.rs = RowSplit::of<EB>(src, V);
    const RowSplit& rs = o.rs;
    if (!LOGITS && !want_bound) return;
    // Pass 1 (16-byte chunks): maximum (NaN-propagating, so one test flags NaN/+inf),
    // minimum, and each thread's maximum, a lower bound on its own best entry; the R-th
    // largest of the 256 thread bounds bounds the row's R-th best entry from below.
    float mxn, mn;
    group_pass1<DT, kThreads>(src, rs, tid, mxn, mn);
    const bool bad = !(mxn < f_inf());
    if (want_bound) {
        float me = bad ? f_ninf() : mxn;
        if (m.eos >= 0) {
            // Threads owning an EOS token give no bound (a smaller bound stays valid).
            if (rs.owns(m.eos)) me = f_ninf();
            for (int i = 0; i < p.n_extra; ++i)
                if (rs.owns(p.extra[i])) me = f_ninf();
        }
        const float sorted = warp_sort_desc(me);
        if (lane < R && lane < RCAP) sh.wtop[warp * RCAP + lane] = sorted;
    }
    if (tid == 0) sh.count = 0;  // record candidates (from logits, all-warps pass 2)
    {
        const float wmx = warp_max_f32(bad ? f_ninf() : mxn);
        const float wmn = -warp_max_f32(-mn);
        const unsigned wbad = __ballot_sync(0xffffffffu, bad);
        if (lane == 0) {
            sh.wred[warp] = wmx;
            sh.wred2[warp] = wmn;
            sh.ired[warp] = wbad != 0;
        }
    }
    block_sync();
    float mx = sh.wred[0];
    mn = sh.wred2[0];
    bool any_bad = sh.ired[0] != 0;
#pragma unroll
    for (int w = 1; w < kWarps; ++w) {
        mx = fmaxf(mx, sh.wred[w]);
        mn = fminf(mn, sh.wred2[w]);
        any_bad |= sh.ired[w] != 0;
    }
    o.inv_known = true;
    o.invalid = any_bad;
    if (any_bad) {
        // Rare: the maximum over entries below +inf (NaN never raises fmaxf).
        block_sync();
        mx = f_ninf();
        for_chunks<DT>(src, rs, use_smem, [&](float x, int) {
            if (x < f_inf()) mx = fmaxf(mx, x);
        });
        mx = block_max(sh, mx);
    }
    const bool make_bound = want_bound && R > 0 && R <= kWarps * RCAP && !any_bad;
    if (!LOGITS) {
        if (make_bound && warp >= 4) bound_rank<RCAP>(sh, R, tid - kThreads / 2);
        block_sync();
        if (make_bound) o.xthr = sh.xbound;
        return;
    }
    if (ro != nullptr && make_bound && mx != f_ninf() && R <= kWarps * RCAP) {
        // The filter bound, computed by every warp on its own (no barrier): with R <= 32 and
        // at least 4 sorted maxima per warp, the R-th largest of the union of the warps'
        // top-4 thread maxima (32 values, one per lane); otherwise the smallest over the
        // warps of each warp's ceil(R / 8)-th largest. Either way at least R thread maxima
        // (each an eligible entry) reach it, so it bounds the row's R-th best eligible entry
        // from below; the first equals the R-th largest thread maximum unless a warp holds
        // more than four of the top R.
        float xb;
        if (R <= 32 && RCAP >= 4 && R >= 4) {
            xb = warp_rth_largest(sh.wtop[(lane >> 2) * RCAP + (lane & 3)], R);
        } else {
            const int per_warp = (R + kWarps - 1) / kWarps;
            xb = sh.wtop[per_warp - 1];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) xb = fminf(xb, sh.wtop[w * RCAP + per_warp - 1]);
        }
        const bool bounded = xb != f_ninf();
        collect_candidates<DT>(p, sh, src, rs, xb, bounded && mxn >= xb, m, *ro);
        const bool fast = __fsub_rn(mn, mx) >= cephes::kMin;  // every x - max >= -87
        if (use_smem) {
            const uint32_t srow_a = smem_u32(srow + soff);
            sh.lanes[tid] = fast ? lane_sum_staged<DT, false>(srow_a, V, mx, tid, p.one2, p.nzero2)
                                 : lane_sum_staged<DT, true>(srow_a, V, mx, tid, p.one2, p.nzero2);
        } else {
            // A row too large to stage: pass 2 reads it again from global memory, where
            // pass 1 has just brought it into L2.
            sh.lanes[tid] = fast ? lane_sum_global<DT, false>(src, V, mx, tid, p.one2, p.nzero2)
                                 : lane_sum_global<DT, true>(src, V, mx, tid, p.one2, p.nzero2);
        }
        block_sync();
        if (warp == 0) {
            // Pairwise tree lanes[i] += lanes[i + s], s = 128 ... 1 (src/kernels.hpp:197-202),
            // by one warp: lane i forms the s = 128, 64, 32 levels of index i from lanes
            // i, i + 32, ..., i + 224 in the tree's own order, then shuffles for s = 16 ... 1.
            const float* l = sh.lanes;
            const float a0 = __fadd_rn(l[tid], l[tid + 128]), a1 = __fadd_rn(l[tid + 32], l[tid + 160]);
            const float a2 = __fadd_rn(l[tid + 64], l[tid + 192]), a3 = __fadd_rn(l[tid + 96], l[tid + 224]);
            float x = __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
#pragma unroll
            for (int st = 16; st >= 1; st >>= 1) {
                const float y = __shfl_down_sync(0xffffffffu, x, st);
                if (tid < st) x = __fadd_rn(x, y);
            }
            if (tid == 0) sh.row_lse = logsumexp_from(mx, x);
        } else if (warp >= 4) {
            const int n = sh.count;
            if (bounded && n <= kCandCap) {
                if (warp == 4) record_from_candidates(sh, n, *ro);
            } else {
                side(src, rs, xb);
            }
        }
        block_sync();
        o.lse = sh.row_lse;
        o.xthr = xb;
        return;
    }
    if (warp >= 4) {
        if (make_bound) bound_rank<RCAP>(sh, R, tid - kThreads / 2);
        half_sync(1);
        side(src, rs, make_bound ? sh.xbound : f_ninf());
    } else {
        // Pass 2: logsumexp lanes a = 2j and b = 2j + 1 on thread j < 128.
        const int j = tid;
        float lse = f_ninf();
        if (mx != f_ninf()) {
            const auto* er = reinterpret_cast<const typename E::T*>(src);
            const int nfull = V / kLanes;
            const int a = 2 * j, b = 2 * j + 1;
            float acc_a = 0.0f, acc_b = 0.0f;
            if (!o.invalid) {
                const Pack2 q{p.one2, p.nzero2};
                const bool fast = __fsub_rn(mn, mx) >= cephes::kMin;  // every x - max >= -87
                const bool paired = (reinterpret_cast<uintptr_t>(src) & (2 * EB - 1)) == 0;
                if (paired) {
                    // A staged row is read through srow itself: the compiler then emits
                    // shared-memory loads with 32-bit addresses (measured 2.4% faster at C2
                    // than loads through the generic pointer).
                    uint64_t acc;
                    if (use_smem) {
                        acc = fast ? lane_pair_sums<DT, false>(q, srow + soff, nfull, mx, j)
                                   : lane_pair_sums<DT, true>(q, srow + soff, nfull, mx, j);
                    } else {
                        acc = fast ? lane_pair_sums<DT, false>(q, grow, nfull, mx, j)
                                   : lane_pair_sums<DT, true>(q, grow, nfull, mx, j);
                    }
                    f2_unpack(acc, acc_a, acc_b);
                } else {
                    for (int i = 0; i < nfull; ++i) {
                        acc_a = __fadd_rn(acc_a, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[i * kLanes + a]), mx)));
                        acc_b = __fadd_rn(acc_b, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[i * kLanes + b]), mx)));
                    }
                }
                // The partial last block.
                const int va = nfull * kLanes + a, vb = nfull * kLanes + b;
                if (va < V) acc_a = __fadd_rn(acc_a, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[va]), mx)));
                if (vb < V) acc_b = __fadd_rn(acc_b, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[vb]), mx)));
            } else {
                for (int v = a; v < V; v += kLanes) {
                    const float x = E::to_f32(er[v]);
                    if (x < f_inf() && x != f_ninf()) acc_a = __fadd_rn(acc_a, exp_nonpositive(__fsub_rn(x, mx)));
                }
                for (int v = b; v < V; v += kLanes) {
                    const float x = E::to_f32(er[v]);
                    if (x < f_inf() && x != f_ninf()) acc_b = __fadd_rn(acc_b, exp_nonpositive(__fsub_rn(x, mx)));
                }
            }
            sh.lanes[a] = acc_a;
            sh.lanes[b] = acc_b;
            half_sync(2);
            // Pairwise tree lanes[i] += lanes[i + s], s = 128 ... 1 (src/kernels.hpp:197-202).
#pragma unroll
            for (int st = kLanes / 2; st >= 32; st >>= 1) {
                if (tid < st) sh.lanes[tid] = __fadd_rn(sh.lanes[tid], sh.lanes[tid + st]);
                half_sync(2);
            }
            if (warp == 0) {
                float x = sh.lanes[tid];
#pragma unroll
                for (int st = 16; st >= 1; st >>= 1) {
                    const float y = __shfl_down_sync(0xffffffffu, x, st);
                    if (tid < st) x = __fadd_rn(x, y);
                }
                lse = logsumexp_from(mx, x);
            }
        }
        if (tid == 0) sh.row_lse = lse;
    }
    block_sync();
    o.lse = sh.row_lse;
    if (make_bound) o.xthr = sh.xbound;
}

// ---------------------------------------------------------------------------
// Selection of example b at step t for beams up to 16, by warp 0 alone: the
// step's best keys, the carried-forward finished beams, their merge in the
// full candidate order, and the new trace / state / prefixes / finals.
// ---------------------------------------------------------------------------
// The selection proper, from the step's row lists in registers (mine[j]: entry lane + 32j
// of the K rows' LIST-entry lists, zeros for no candidate) and the state before the step
// (lane k < beam holds slot k).
template <int KMAX, int LIST>
__device__ void select_fast_core(const DecodeParams& p, int t, int b, const Meta& m,
                                 uint64_t (&mine)[(KMAX * LIST + 31) / 32], float s_raw, int s_len, int s_end,
                                 int s_last) {
    constexpr int kPer = (KMAX * LIST + 31) / 32;
    const int lane = threadIdx.x & 31;
    const int K = p.K;
    const uint32_t V = static_cast<uint32_t>(p.V);
    const int64_t sbase = static_cast<int64_t>(b) * K;
    const int64_t obase = (static_cast<int64_t>(b) * p.T + t) * K;
    const bool active = t < m.steps;
    const bool last_step = p.step_api ? true : (t == p.T - 1);
    const int beam = m.beam;

    int filled = 0;
    // Length penalties, computed before the top-k rounds so that their latency overlaps
    // them: the reciprocal for a candidate extending a beam of length t (every scanned
    // candidate of a chained decode step), and this slot's carried score.
    const float inv_next = __fdiv_rn(1.0f, gnmt_penalty(t + 1, p.alpha));
    const int l_carry = s_len > 1 ? s_len : 1;
    const bool carry = active && m.eos >= 0 && lane < beam && s_end != 0 && f_finite(s_raw);
    const float sc = carry ? __fdiv_rn(s_raw, gnmt_penalty(l_carry, p.alpha)) : 0.0f;
    // This lane's candidate (scanned: lanes [0, ns); carried: lanes [ns, ns + nc)).
    uint64_t my_key = 0;
    float c_score = 0.0f, c_raw = 0.0f;
    int c_parent = -1, c_token = -1, c_len = 0, c_from = 0;
    int pos = 1 << 30;
    if (active) {
        int ns = 0;
        for (; ns < beam; ++ns) {
            uint64_t bst = 0;
#pragma unroll
            for (int j = 0; j < kPer; ++j) bst = mine[j] > bst ? mine[j] : bst;
            const uint64_t w = warp_max_u64(bst);
            if (w == 0) break;
#pragma unroll
            for (int j = 0; j < kPer; ++j)
                if (mine[j] == w) mine[j] = 0;
            if (lane == ns) my_key = w;
        }
        // Carried-forward candidates: finished, live beams (EOS handling on).
        const unsigned cm = __ballot_sync(0xffffffffu, carry);
        const int nc = __popc(cm);
        // Scanned candidate of lane i < ns.
        {
            const uint32_t index = key_index(my_key);
            const int par = lane < ns ? static_cast<int>(index / V) : 0;
            const int plen = __shfl_sync(0xffffffffu, s_len, par);
            if (lane < ns) {
                c_parent = par;
                c_token = static_cast<int>(index - static_cast<uint32_t>(par) * V);
                c_len = plen + 1;
                c_raw = key_raw(my_key);
                c_score = __fmul_rn(c_raw, c_len == t + 1 ? inv_next : __fdiv_rn(1.0f, gnmt_penalty(c_len, p.alpha)));
                c_from = 1;
            }
        }
        // Carried candidate j (the j-th carrying slot in slot order) moves to lane ns + j.
        {
            const int j = __popc(cm & ((1u << lane) - 1u));
            const int l = l_carry;
            const int tok = (s_last >= 0 && s_last < p.V && is_eos(p, m, s_last)) ? s_last : m.eos;
            // Source lane of carried candidate (lane - ns): the (lane - ns)-th set bit of cm.
            int srcl = 0;
            {
                const int want = lane - ns;
                unsigned mm = cm;
                for (int q = 0; q < want && mm; ++q) mm &= mm - 1;
                srcl = mm ? __ffs(mm) - 1 : 0;
            }
            const float g_sc = __shfl_sync(0xffffffffu, sc, srcl);
            const float g_raw = __shfl_sync(0xffffffffu, s_raw, srcl);
            const int g_tok = __shfl_sync(0xffffffffu, tok, srcl);
            const int g_len = __shfl_sync(0xffffffffu, l, srcl);
            (void)j;
            if (lane >= ns && lane < ns + nc) {
                c_score = g_sc;
                c_raw = g_raw;
                c_parent = srcl;
                c_token = g_tok;
                c_len = g_len;
                c_from = 0;
            }
        }
        // Positions by counting under the full order (src/common.hpp:269-276). Without
        // carried candidates, and with every scanned candidate of one length (one penalty, so
        // the score never decreases as raw grows), the extraction order by key (raw, then
        // parent and token) already is that order.
        const int total = ns + nc;
        const int len0 = __shfl_sync(0xffffffffu, c_len, 0);
        const bool one_len = __all_sync(0xffffffffu, lane >= ns || c_len == len0);
        pos = 0;
        if (nc == 0 && one_len) pos = lane;
        else for (int o = 0; o < total; ++o) {
            const float os = __shfl_sync(0xffffffffu, c_score, o);
            const float orr = __shfl_sync(0xffffffffu, c_raw, o);
            const int op = __shfl_sync(0xffffffffu, c_parent, o);
            const int ot = __shfl_sync(0xffffffffu, c_token, o);
            const int ol = __shfl_sync(0xffffffffu, c_len, o);
            const int of = __shfl_sync(0xffffffffu, c_from, o);
            bool better;
            if (os != c_score) better = os > c_score;
            else if (orr != c_raw) better = orr > c_raw;
            else if (op != c_parent) better = op < c_parent;
            else if (ot != c_token) better = ot < c_token;
            else if (ol != c_len) better = ol < c_len;
            else better = of > c_from;
            if (o != lane && better) ++pos;
        }
        if (lane >= total) pos = 1 << 30;
        filled = total < beam ? total : beam;
        // Parent-derived fields needed at the new slot.
        const int par_end = __shfl_sync(0xffffffffu, s_end, c_parent >= 0 ? c_parent : 0);
        if (pos < beam) {
            const int64_t o = obase + pos;
            if (p.out.tokens) p.out.tokens[o] = c_token;
            if (p.out.parents) p.out.parents[o] = c_parent;
            if (p.out.lengths) p.out.lengths[o] = c_len;
            if (p.out.scores) p.out.scores[o] = c_score;
            if (p.out.raw_scores) p.out.raw_scores[o] = c_raw;
            if (p.out.from_logprob) p.out.from_logprob[o] = static_cast<uint8_t>(c_from);
        }
        __syncwarp();
        // New state (every lane has its snapshot already).
        if (pos < beam) {
            const int64_t sl = sbase + pos;
            p.raw[sl] = c_raw;
            p.len[sl] = c_len;
            p.ended[sl] = static_cast<uint8_t>(c_from ? (par_end != 0 || is_eos(p, m, c_token)) : 1);
            if (!p.step_api) p.last[sl] = c_token;
        }
    }
    // Empty slots.
    if (lane < K && lane >= filled) {
        const int64_t o = obase + lane;
        if (p.out.tokens) p.out.tokens[o] = -1;
        if (p.out.parents) p.out.parents[o] = -1;
        if (p.out.lengths) p.out.lengths[o] = 0;
        if (p.out.scores) p.out.scores[o] = f_ninf();
        if (p.out.raw_scores) p.out.raw_scores[o] = f_ninf();
        if (p.out.from_logprob) p.out.from_logprob[o] = 0;
        if (active) {
            const int64_t sl = sbase + lane;
            p.raw[sl] = f_ninf();
            p.len[sl] = 0;
            p.ended[sl] = 0;
            if (!p.step_api) p.last[sl] = -1;
        }
    }
    // Prefixes of the new hypotheses (decode with n-gram blocking / repetition penalty).
    if (p.prefix[0] && !p.step_api) {
        const int T = p.T;
        const int cur = t & 1, nxt = (t + 1) & 1;
        // slot -> (parent, token, from) for the filled slots: the lane whose pos == slot.
        for (int k = 0; k < K; ++k) {
            const unsigned owner = __ballot_sync(0xffffffffu, active && pos == k);
            int32_t* dst = p.prefix[nxt] + (sbase + k) * T;
            if (owner) {
                const int ol = __ffs(owner) - 1;
                const int par = __shfl_sync(0xffffffffu, c_parent, ol);
                const int tok = __shfl_sync(0xffffffffu, c_token, ol);
                const int frm = __shfl_sync(0xffffffffu, c_from, ol);
                const int32_t* src = p.prefix[cur] + (sbase + par) * T;
                const int L = ld_cg(p.prefix_len[cur] + sbase + par);
                for (int i = lane; i < L; i += 32) dst[i] = ld_cg(src + i);
                const bool append = frm && tok >= 0 && L < T;
                if (lane == 0) {
                    if (append) dst[L] = tok;
                    p.prefix_len[nxt][sbase + k] = L + (append ? 1 : 0);
                }
            } else if (!active) {
                const int32_t* src = p.prefix[cur] + (sbase + k) * T;
                const int L = ld_cg(p.prefix_len[cur] + sbase + k);
                for (int i = lane; i < L; i += 32) dst[i] = ld_cg(src + i);
                if (lane == 0) p.prefix_len[nxt][sbase + k] = L;
            } else if (lane == 0) {
                p.prefix_len[nxt][sbase + k] = 0;
            }
        }
    }
    __syncwarp();
    // Final scores after the last step.
    if (last_step && p.out.final_scores && lane < K) {
        const int64_t sl = sbase + lane;
        float raw = f_ninf(), score = f_ninf();
        int len = 0;
        if (lane < beam) {
            raw = p.raw[sl];
            len = p.len[sl];
            score = __fdiv_rn(raw, gnmt_penalty(len, p.alpha));
        }
        p.out.final_scores[sl] = score;
        if (p.out.final_raw_scores) p.out.final_raw_scores[sl] = raw;
        if (p.out.final_lengths) p.out.final_lengths[sl] = len;
    }
    __syncwarp();  // callers order the writes for other CTAs (fence or release) before publishing
}

// select_fast_core with the state and the row lists (p.keys) read from global memory.
template <int KMAX, int LIST = KMAX>
__device__ void select_fast(const DecodeParams& p, int t, int b, const Meta& m) {
    const int lane = threadIdx.x & 31;
    const int K = p.K;
    const int64_t sbase = static_cast<int64_t>(b) * K;
    const bool active = t < m.steps;
    float s_raw = f_ninf();
    int s_len = 0, s_last = -1;
    int s_end = 0;
    if (lane < m.beam) {
        s_raw = ld_cg(p.raw + sbase + lane);
        s_len = ld_cg(p.len + sbase + lane);
        s_end = ld_cg(p.ended + sbase + lane);
        if (p.step_api) {
            if (p.caller_prefix && s_len >= 1 && s_len <= p.prefix_stride)
                s_last = ld_cg(p.caller_prefix + (sbase + lane) * p.prefix_stride + s_len - 1);
        } else {
            s_last = ld_cg(p.last + sbase + lane);
        }
    }
    constexpr int kPer = (KMAX * LIST + 31) / 32;
    const uint64_t* lists = p.keys + sbase * LIST;
    const int n = K * LIST;
    uint64_t mine[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = lane + 32 * j;
        mine[j] = (active && i < n) ? ld_cg(lists + i) : 0;
    }
    select_fast_core<KMAX, LIST>(p, t, b, m, mine, s_raw, s_len, s_end, s_last);
}

// ---------------------------------------------------------------------------
// The persistent decode kernel.
// ---------------------------------------------------------------------------
template <int DT, bool LOGITS, int KMAX>
__global__ void __launch_bounds__(kThreads, 3) decode_kernel(const __grid_constant__ DecodeParams p) {
    constexpr int KCAP = KMAX > 0 ? kFastBeam : kSelectCap;
    using E = Elem<DT>;
    constexpr int EB = E::kBytes;
    __shared__ RowShared sh;
    extern __shared__ __align__(128) unsigned char dyn[];
    auto& ss = *reinterpret_cast<SelectShared<KCAP>*>(dyn);
    char* srow = reinterpret_cast<char*>(dyn) + ((sizeof(SelectShared<KCAP>) + 127) & ~static_cast<size_t>(127));

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    if (tid == 0) mbar_init(&sh.mbar);
    block_sync();
    uint32_t phase = 0;

    const int K = p.K, V = p.V;
    const uint32_t rows_per_step = static_cast<uint32_t>(p.B) * static_cast<uint32_t>(K);
    const uint32_t total = rows_per_step * static_cast<uint32_t>(p.T);
    const bool exclusions = p.banned != nullptr;
    const bool constrained = p.ngram > 0 || p.penalise;

    for (;;) {
        if (tid == 0) {
            const uint32_t tk0 = atomicAdd(p.ticket, 1u);
            sh.ticket = static_cast<int>(tk0);
            int ready = 0;
            if (tk0 < total) ready = ld_acquire(p.flag + (tk0 - (tk0 / rows_per_step) * rows_per_step) / K) >=
                                             static_cast<int>(tk0 / rows_per_step);
            sh.ready = ready;
        }
        block_sync();
        const uint32_t tk = static_cast<uint32_t>(sh.ticket);
        if (tk >= total) break;
        const bool ready = sh.ready != 0;
        const int t = static_cast<int>(tk / rows_per_step);
        const uint32_t rem = tk - static_cast<uint32_t>(t) * rows_per_step;
        const int b = static_cast<int>(rem / static_cast<uint32_t>(K));
        const int k = static_cast<int>(rem - static_cast<uint32_t>(b) * static_cast<uint32_t>(K));
        const Meta m = load_meta(p, b);
        const int64_t s = static_cast<int64_t>(b) * K + k;
        const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + k;
        const char* grow = static_cast<const char*>(p.inputs) + rowi * static_cast<int64_t>(V) * EB;
        // Rows a step can read: an active step's beams (at t = 0 of a decode, only beam 0).
        const bool maybe = t < m.steps && k < m.beam && (p.step_api || t > 0 || k == 0);

        // Per-row results of passes 1-2.
        const char* src = grow;
        bool prepared = false;
        float lse = 0.0f;
        bool invalid = false;
        bool inv_known = false;  // invalid computed over the whole row
        float xthr = f_ninf();   // lower bound on the row's R-th best eligible entry (pass 1)
        const int R = KMAX > 0 ? (m.beam < KMAX ? m.beam : KMAX) : 0;
        bool aborted = false;
        RowSplit rs;

        // Stage the row and compute its max / logsumexp / filter bound. None of it
        // depends on the selection of the previous step.
        auto prepare = [&](bool use_smem) {
            prepared = true;
            Prep o;
            prepare_row<DT, LOGITS, kFastBeam>(p, sh, srow, grow, phase, use_smem,
                                               KMAX > 0 && !constrained && !exclusions, R, m, o,
                                               [](const char*, const RowSplit&, float) {});
            src = o.src;
            rs = o.rs;
            lse = o.lse;
            xthr = o.xthr;
            invalid = o.invalid;
            inv_known = o.inv_known;
            aborted = o.aborted;
        };

        // Speculative preparation while example b's previous step is still being selected.
        if (!ready && maybe && p.staged) {
            prepare(true);
            if (aborted) break;
        }

        if (!ready && warp == 0) {
            const bool ok = wait_flag_warp(p, p.flag + b, t);
            if (lane == 0) sh.is_last = ok ? 0 : -1;
        } else if (tid == 0) {
            sh.is_last = 0;
        }
        block_sync();
        if (sh.is_last < 0) break;  // timed out or aborted

        bool read = false;
        float pr = 0.0f;
        int plen = 0;
        if (maybe) {
            pr = ld_cg(p.raw + s);
            plen = ld_cg(p.len + s);
            const uint8_t ended = ld_cg(p.ended + s);
            read = f_finite(pr) && !(m.eos >= 0 && ended != 0);
        }
        uint64_t* list = p.keys + s * p.list_len;
        if (read) {
            if (!prepared) {
                prepare(p.staged != 0);
                if (aborted) break;
            }
            RowCtx c;
            c.pr = pr;
            c.new_len = plen + 1;
            c.k = k;
            c.m = m;
            c.mask_eos = m.eos >= 0 && c.new_len < m.min_length;
            c.constrained = constrained;
            c.cv = ConsView{nullptr, 0, true};
            if (constrained) {
                const int32_t* pre;
                int L;
                if (p.step_api) {
                    pre = p.caller_prefix ? p.caller_prefix + s * p.prefix_stride : nullptr;
                    L = plen < 0 ? 0 : (plen > p.prefix_stride ? p.prefix_stride : plen);
                    if (!pre) L = 0;
                } else {
                    pre = p.prefix[t & 1] + s * p.T;
                    L = ld_cg(p.prefix_len[t & 1] + s);
                }
                c.cv = build_constraints(p, sh, pre, L);
            }
            const bool has_cands = !LOGITS || lse != f_ninf();
            if (tid == 0 && p.row_lse) p.row_lse[rowi] = LOGITS ? lse : 0.0f;

            // Pass 3: candidate keys.
            if constexpr (KMAX > 0) {
                WarpTopK<KMAX> wt;
                float bound = f_ninf();
                if (xthr != f_ninf()) bound = __fadd_rn(pr, LOGITS ? __fsub_rn(xthr, lse) : xthr);
                wt.init(bound);
                // x-space prefilter: every entry with raw(x) >= thr has x >= xf, because raw is
                // non-decreasing in x and raw(float_below(xf)) < thr is checked exactly.
                auto raw_of = [&](float x) { return __fadd_rn(pr, LOGITS ? __fsub_rn(x, lse) : x); };
                auto prefilter = [&](float thr) {
                    if (thr == f_ninf()) return f_ninf();
                    const float est = LOGITS ? __fadd_rn(__fsub_rn(thr, pr), lse) : __fsub_rn(thr, pr);
                    return smallest_x_reaching(est, thr, raw_of);
                };
                float xf = prefilter(wt.thr);
                const bool check_inv = !inv_known;
                bool inv3 = false;
                auto exact = [&](float x, int v) -> uint64_t {
                    const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                    if (!(lp < f_inf()) || lp == f_ninf()) return 0;
                    if (__fadd_rn(pr, lp) < wt.thr) return 0;
                    return full_key(p, sh, c, lp, v);
                };
                if (has_cands) {
                    scan_chunks_ballot<DT>(src, rs, p.staged != 0 && prepared, [&](float x) {
                        if (check_inv) inv3 |= !(x < f_inf());
                        return x >= xf;
                    }, [&](float x, int v, bool valid) {
                        const uint64_t key = valid && x >= xf ? exact(x, v) : 0;
                        const float before = wt.thr;
                        wt.offer(key, lane);
                        if (wt.thr != before) xf = prefilter(wt.thr);
                    });
                }
                if (check_inv) invalid = inv3;
                if (lane < KMAX) sh.wkeys[warp * KMAX + lane] = wt.wl;
                block_sync();
                if (warp == 0) {
                    constexpr int kPer = (kWarps * KMAX + 31) / 32;
                    uint64_t mine[kPer];
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        const int i = lane + 32 * j;
                        mine[j] = i < kWarps * KMAX ? sh.wkeys[i] : 0;
                    }
                    uint64_t out = 0;
                    for (int r = 0; r < R; ++r) {
                        uint64_t bst = 0;
#pragma unroll
                        for (int j = 0; j < kPer; ++j) bst = mine[j] > bst ? mine[j] : bst;
                        const uint64_t w = warp_max_u64(bst);
#pragma unroll
                        for (int j = 0; j < kPer; ++j)
                            if (w != 0 && mine[j] == w) mine[j] = 0;
                        if (lane == r) out = w;
                    }
                    if (lane < KMAX) list[lane] = out;
                }
            } else {
                // Generic beams: block radix select of the row's best min(beam, V) keys.
                auto gen = [&](int v) -> uint64_t {
                    const float x = load_elem<DT>(src, v);
                    const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                    if (!(lp < f_inf()) || lp == f_ninf()) return 0;
                    return full_key(p, sh, c, lp, v);
                };
                if (!inv_known) {
                    bool inv = false;
                    for (int v = tid; v < V; v += kThreads) inv |= !(load_elem<DT>(src, v) < f_inf());
                    invalid = inv;
                }
                int cnt = 0;
                if (has_cands) cnt = block_select(sh, gen, V, m.beam, [&](int pos, uint64_t key) { list[pos] = key; });
                for (int i = cnt + tid; i < p.list_len; i += kThreads) list[i] = 0;
            }
        } else {
            for (int i = tid; i < p.list_len; i += kThreads) list[i] = 0;
            if (tid == 0 && p.row_lse) p.row_lse[rowi] = 0.0f;
        }

        // Arrive; the last row of (t, b) selects. Writers fence their own writes first.
        __threadfence();
        const bool all_valid = block_and(!(read && invalid));
        if (tid == 0) {
            if (!all_valid && p.out.invalid_input) p.out.invalid_input[b] = 1;
            __threadfence();
            sh.is_last = atomicAdd(p.arrive + b, 1u) == static_cast<uint32_t>(K) - 1u ? 1 : 0;
        }
        block_sync();
        if (sh.is_last) {
            __threadfence();
            if constexpr (KMAX > 0) {
                if (warp == 0) select_fast<KMAX>(p, t, b, m);
            } else {
                select_step<KMAX, KCAP>(p, sh, ss, t, b, m);
            }
            block_sync();
            if (tid == 0) {
                p.arrive[b] = 0;
                __threadfence();
                st_release(p.flag + b, t + 1);
            }
        }
        block_sync();
    }
}

// ---------------------------------------------------------------------------
// Chained decode (beams up to 16, no n-gram blocking or repetition penalty).
//
// Nothing waits. A row task (t, b, k) needs nothing from the previous step:
// it stages the row, computes its logsumexp, and keeps the row's best LIST
// entries by x (ties: lower token first) as a per-row record. Because a
// candidate's raw score fadd(parent_raw, lp(x)) never decreases as x grows,
// every entry left out of the record has raw <= raw of the record's last
// entry; so once the parent's raw score is known, the record holds the row's
// best R candidates whenever the R-th entry's raw score is strictly above the
// last entry's (or the record holds every eligible entry). Otherwise, which is
// rare, the selecting CTA rescans that row with the parent known.
//
// Each (b, t) counts arrivals: its K row tasks and, for t > 0, the selection
// of step t - 1. The CTA that completes the count selects step t of example b
// and then arrives for step t + 1, continuing the chain while it completes
// counts, so example b's selections run one after another without any CTA
// spinning on a flag.
// ---------------------------------------------------------------------------
template <int KMAX>
__host__ __device__ constexpr int chain_list_len() {
    return KMAX <= 4 ? 8 : 2 * KMAX;
}

// A group of NT threads (NT / 32 whole warps; local thread index ltid) that
// synchronizes on its own named barrier (id 0 with NT = kThreads: the whole CTA).
template <int NT>
__device__ __forceinline__ void group_sync(int id) {
    if (NT == kThreads && id == 0) block_sync();
    else asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(NT) : "memory");
}

// The best KMAX full keys of row (t, b, k), parent state known, scanned from global
// memory by the group: the fallback of the chained select, written as the row's list.
template <int DT, bool LOGITS, int KMAX, int LIST, int NT>
__device__ void rescan_row(const DecodeParams& p, SelScratch& ss, int t, int b, int k, const Meta& m, float lse,
                           int ltid, int bar) {
    using E = Elem<DT>;
    constexpr int NW = NT / 32;
    const int lane = ltid & 31;
    const int lw = ltid >> 5;
    const int K = p.K, V = p.V;
    const int64_t s = static_cast<int64_t>(b) * K + k;
    const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + k;
    const char* grow = static_cast<const char*>(p.inputs) + rowi * static_cast<int64_t>(V) * E::kBytes;
    const float pr = ld_cg(p.raw + s);
    const int new_len = ld_cg(p.len + s) + 1;
    const bool mask_eos = m.eos >= 0 && new_len < m.min_length;
    const uint32_t base = static_cast<uint32_t>(k) * static_cast<uint32_t>(V);
    const ConsView cv = chain_prefix(p, t, s);
    const RowSplit rs = RowSplit::of<E::kBytes>(grow, V);
    WarpTopK<KMAX> wt;
    wt.init(f_ninf());
    if (!LOGITS || lse != f_ninf()) {
        scan_chunks_ballot_n<DT, NT>(grow, rs, false, ltid, [&](float x) { return x < f_inf() && x != f_ninf(); },
                                     [&](float x, int v, bool valid) {
                                         uint64_t key = 0;
                                         if (valid && x < f_inf() && x != f_ninf() && !(p.banned && p.banned[v]) &&
                                             !(mask_eos && is_eos(p, m, v))) {
                                             const float raw = constrained_raw<LOGITS>(p, cv, pr, x, lse, v);
                                             if (raw != f_ninf()) key = make_key(raw, base + static_cast<uint32_t>(v));
                                         }
                                         wt.offer(key, lane);
                                     });
    }
    if (lane < KMAX) ss.wkeys[lw * KMAX + lane] = wt.wl;
    group_sync<NT>(bar);
    if (lw == 0) {
        constexpr int kPer = (NW * KMAX + 31) / 32;
        uint64_t mine[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = lane + 32 * j;
            mine[j] = i < NW * KMAX ? ss.wkeys[i] : 0;
        }
        uint64_t out = 0;
        for (int r = 0; r < KMAX; ++r) {
            uint64_t bst = 0;
#pragma unroll
            for (int j = 0; j < kPer; ++j) bst = mine[j] > bst ? mine[j] : bst;
            const uint64_t w = warp_max_u64(bst);
#pragma unroll
            for (int j = 0; j < kPer; ++j)
                if (w != 0 && mine[j] == w) mine[j] = 0;
            if (lane == r) out = w;
        }
        if (lane < LIST) p.keys[s * LIST + lane] = lane < KMAX ? out : 0;
    }
    group_sync<NT>(bar);
}

// Selection of step t of example b with n-gram blocking or a repetition penalty: warp w of
// the group takes rows w, w + NW, ..., whose constraint checks read the parent's prefix.
template <int DT, bool LOGITS, int KMAX, int LIST, int NT>
__device__ void chain_select_constrained(const DecodeParams& p, SelScratch& ss, int t, int b, const Meta& m, int ltid, int bar) {
    constexpr int NW = NT / 32;
    const int lane = ltid & 31;
    const int lw = ltid >> 5;
    const int K = p.K;
    const uint32_t V = static_cast<uint32_t>(p.V);
    const bool active = t < m.steps;
    const int R = m.beam < KMAX ? m.beam : KMAX;
    if (ltid == 0) {
        ss.fallback = 0;
        ss.invalid = 0;
    }
    group_sync<NT>(bar);
    // Warp w of the group turns the records of rows w, w + NW, ... into candidate keys.
    for (int k = lw; k < K; k += NW) {
        const int64_t s = static_cast<int64_t>(b) * K + k;
        const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + k;
        bool read = false;
        float pr = 0.0f;
        int plen = 0;
        if (active && k < m.beam && (t > 0 || k == 0)) {
            pr = ld_cg(p.raw + s);
            plen = ld_cg(p.len + s);
            const uint8_t ended = ld_cg(p.ended + s);
            read = f_finite(pr) && !(m.eos >= 0 && ended != 0);
        }
        uint64_t key = 0;
        float lse = 0.0f;
        if (read) {
            const uint32_t info = ld_cg(p.rinfo + rowi);
            lse = ld_cg(p.rlse + rowi);
            const int cnt = static_cast<int>(info >> 8);
            const uint64_t xk = lane < cnt ? ld_cg(p.rkeys + rowi * LIST + lane) : 0;
            const ConsView cv = chain_prefix(p, t, s);
            float raw_plain = f_ninf(), raw = f_ninf();
            if (xk != 0) {
                const float x = key_raw(xk);
                const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                if (lp < f_inf() && lp != f_ninf()) {
                    raw_plain = __fadd_rn(pr, lp);
                    raw = cv.prefix ? constrained_raw<LOGITS>(p, cv, pr, x, lse, static_cast<int>(key_index(xk))) : raw_plain;
                    if (raw != f_ninf()) key = make_key(raw, static_cast<uint32_t>(k) * V + key_index(xk));
                }
            }
            // Exactness of the record: every entry left out has an unconstrained raw score
            // no higher than the last entry's (raw never decreases as x grows; blocking and
            // penalties only lower it), so R entries strictly above that prove the row's
            // best R are here. The record's EOS masking assumed parent length t.
            const float raw_last = __shfl_sync(0xffffffffu, raw_plain, LIST - 1);
            const int n_above = __popc(__ballot_sync(0xffffffffu, raw > raw_last));
            const bool exact = plen == t && (cnt < LIST || n_above >= R);
            if (!exact) {
                key = 0;
                if (lane == 0) atomicOr(&ss.fallback, 1u << k);
            }
            if (lane == 0 && (info & 1u)) ss.invalid = 1;
        }
        if (lane < LIST) p.keys[s * LIST + lane] = key;
        if (lane == 0 && p.row_lse) p.row_lse[rowi] = (read && LOGITS) ? lse : 0.0f;
    }
    group_sync<NT>(bar);
    unsigned fb = ss.fallback;
    while (fb) {
        const int k = __ffs(fb) - 1;
        fb &= fb - 1;
        const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + k;
        rescan_row<DT, LOGITS, KMAX, LIST, NT>(p, ss, t, b, k, m, ld_cg(p.rlse + rowi), ltid, bar);
    }
    if (ltid == 0 && ss.invalid && p.out.invalid_input) p.out.invalid_input[b] = 1;
    group_sync<NT>(bar);
    if (lw == 0) select_fast<KMAX, LIST>(p, t, b, m);
    group_sync<NT>(bar);
}

// Selection of step t of example b from the row records (no n-gram blocking or repetition
// penalty), by a group of NT threads: warp 0 of the group loads every row's parent state, record info and record entries in one
// batch (entry f = lane + 32u of the K rows' LIST-entry lists, so each register holds whole
// rows in aligned LIST-lane segments), decides each record's exactness with segmented
// shuffles, and hands the lists and the state to the selection in registers; rows whose
// record is not enough are rescanned by the whole group first.
template <int DT, bool LOGITS, int KMAX, int LIST, int NT>
__device__ void chain_select(const DecodeParams& p, SelScratch& ss, int t, int b, const Meta& m, int ltid, int bar) {
    if (p.ngram > 0 || p.penalise) {
        chain_select_constrained<DT, LOGITS, KMAX, LIST, NT>(p, ss, t, b, m, ltid, bar);
        return;
    }
    constexpr int kPer = (KMAX * LIST + 31) / 32;
    static_assert(32 % LIST == 0 || LIST % 32 == 0, "rows must fill whole lane segments");
    const int lane = ltid & 31;
    const int lw = ltid >> 5;
    const int K = p.K;
    const uint32_t V = static_cast<uint32_t>(p.V);
    const bool active = t < m.steps;
    const int R = m.beam < KMAX ? m.beam : KMAX;
    const int64_t sbase = static_cast<int64_t>(b) * K;
    const int64_t row0 = (static_cast<int64_t>(b) * p.T + t) * K;
    float s_raw = f_ninf();
    int s_len = 0, s_end = 0, s_last = -1;
    uint64_t mine[kPer];
    if (lw == 0) {
        // One batch of loads: lane k < K the state of slot k and row k's info / lse; every
        // lane its record entries.
        float lse_l = 0.0f;
        uint32_t info_l = 0;
        if (lane < K) {
            s_raw = ld_cg(p.raw + sbase + lane);
            s_len = ld_cg(p.len + sbase + lane);
            s_end = ld_cg(p.ended + sbase + lane);
            s_last = ld_cg(p.last + sbase + lane);
            info_l = ld_cg(p.rinfo + row0 + lane);
            lse_l = ld_cg(p.rlse + row0 + lane);
        }
        uint64_t xk[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int f = lane + 32 * u;
            xk[u] = f < K * LIST ? ld_cg(p.rkeys + row0 * LIST + f) : 0;
        }
        const bool read_l = active && lane < m.beam && (t > 0 || lane == 0) && f_finite(s_raw) &&
                            !(m.eos >= 0 && s_end != 0);
        const unsigned reads = __ballot_sync(0xffffffffu, read_l);
        unsigned inexact = 0;
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int f = lane + 32 * u;
            const int k = f / LIST;       // row of this entry
            const int e = f - k * LIST;   // its position in the record
            const int src = k < K ? k : 0;
            const float pr = __shfl_sync(0xffffffffu, s_raw, src);
            const int plen = __shfl_sync(0xffffffffu, s_len, src);
            const uint32_t info = __shfl_sync(0xffffffffu, info_l, src);
            const float lse = __shfl_sync(0xffffffffu, lse_l, src);
            const bool read = k < K && ((reads >> k) & 1u);
            const int cnt = static_cast<int>(info >> 8);
            float raw_plain = f_ninf(), raw = f_ninf();
            uint64_t key = 0;
            if (read && e < cnt && xk[u] != 0) {
                const float x = key_raw(xk[u]);
                const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                if (lp < f_inf() && lp != f_ninf()) {
                    raw_plain = __fadd_rn(pr, lp);
                    raw = raw_plain;
                    key = make_key(raw, static_cast<uint32_t>(k) * V + key_index(xk[u]));
                }
            }
            // Exactness of the record: R entries whose raw is strictly above the last
            // entry's, or every eligible entry recorded. The record's EOS masking assumed
            // parent length t.
            constexpr int SEG = LIST < 32 ? LIST : 32;
            const int seg0 = lane & ~(SEG - 1);
            const float raw_last = __shfl_sync(0xffffffffu, raw_plain, seg0 + SEG - 1);
            int above = raw > raw_last ? 1 : 0;
#pragma unroll
            for (int o = SEG / 2; o >= 1; o >>= 1) above += __shfl_xor_sync(0xffffffffu, above, o);
            const bool exact = plen == t && (cnt < LIST || above >= R);
            if (read && e == 0 && !exact) inexact |= 1u << k;
            mine[u] = (read && exact) ? key : 0;
        }
        inexact = __reduce_or_sync(0xffffffffu, inexact);
        const bool any_bad = __any_sync(0xffffffffu, read_l && (info_l & 1u));
        if (lane == 0) {
            ss.fallback = inexact;
            ss.invalid = any_bad ? 1 : 0;
        }
        if (lane < K && p.row_lse) p.row_lse[row0 + lane] = (read_l && LOGITS) ? lse_l : 0.0f;
    }
    group_sync<NT>(bar);
    const unsigned fb_all = ss.fallback;
    unsigned fb = fb_all;
    while (fb) {
        const int k = __ffs(fb) - 1;
        fb &= fb - 1;
        rescan_row<DT, LOGITS, KMAX, LIST, NT>(p, ss, t, b, k, m, ld_cg(p.rlse + row0 + k), ltid, bar);
    }
    if (ltid == 0 && ss.invalid && p.out.invalid_input) p.out.invalid_input[b] = 1;
    if (fb_all) group_sync<NT>(bar);
    if (lw == 0) {
        if (fb_all) {
            // The rescanned rows' lists (p.keys) replace their entries.
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int f = lane + 32 * u;
                const int k = f / LIST;
                if (k < K && ((fb_all >> k) & 1u)) mine[u] = ld_cg(p.keys + sbase * LIST + f);
            }
        }
        select_fast_core<KMAX, LIST>(p, t, b, m, mine, lane < m.beam ? s_raw : f_ninf(), lane < m.beam ? s_len : 0,
                                     lane < m.beam ? s_end : 0, lane < m.beam ? s_last : -1);
    }
    group_sync<NT>(bar);
}

// Arrival of one finished row (or of the selection of step t - 1) on example b's step-t
// count; while the group completes counts it selects those steps (select(step)) and
// arrives for the next. Called by all NT threads of the group after their writes.
// Arrival counter increment with release (the group's writes, ordered before it by the
// group barrier, become visible first) and acquire (when this arrival completes the
// count, the other arrivals' writes are visible to the group after the next barrier).
__device__ __forceinline__ uint32_t arrive_acq_rel(uint32_t* counter) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
    return old;
}

// synced: the caller has just passed a barrier of the whole group after every write of its
// row but the calling thread's own, so the first barrier here is skipped.
template <int NT, class Select>
__device__ __forceinline__ void chain_arrive_with(const DecodeParams& p, SelScratch& ss, int t, int b, int ltid,
                                                  int bar, Select&& select, bool synced = false) {
    if (!synced) group_sync<NT>(bar);
    if (ltid == 0) {
        const uint32_t target = static_cast<uint32_t>(p.K) + (t > 0 ? 1u : 0u);
        ss.next = arrive_acq_rel(p.count + static_cast<int64_t>(b) * p.T + t) == target - 1u ? t : -1;
    }
    group_sync<NT>(bar);
    int ct = ss.next;
    while (ct >= 0) {
        select(ct);
        if (ltid == 0) {
            int nxt = -1;
            if (ct + 1 < p.T &&
                arrive_acq_rel(p.count + static_cast<int64_t>(b) * p.T + ct + 1) == static_cast<uint32_t>(p.K))
                nxt = ct + 1;
            ss.next = nxt;
        }
        group_sync<NT>(bar);
        ct = ss.next;
    }
}

template <int DT, bool LOGITS, int KMAX, int LIST, int NT>
__device__ __forceinline__ void chain_arrive(const DecodeParams& p, SelScratch& ss, int t, int b, const Meta& m,
                                             int ltid, int bar, bool synced = false) {
    chain_arrive_with<NT>(p, ss, t, b, ltid, bar,
                          [&](int ct) { chain_select<DT, LOGITS, KMAX, LIST, NT>(p, ss, ct, b, m, ltid, bar); }, synced);
}

template <int DT, bool LOGITS, int KMAX>
__global__ void __launch_bounds__(kThreads, 3) decode_chain_kernel(const __grid_constant__ DecodeParams p) {
    constexpr int LIST = chain_list_len<KMAX>();
    using E = Elem<DT>;
    __shared__ RowShared sh;
    extern __shared__ __align__(128) unsigned char dyn[];
    char* srow = reinterpret_cast<char*>(dyn);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    if (tid == 0) mbar_init(&sh.mbar);
    block_sync();
    uint32_t phase = 0;

    const int K = p.K, V = p.V, T = p.T;
    const uint32_t rows_per_step = static_cast<uint32_t>(p.B) * static_cast<uint32_t>(K);
    const uint32_t total = rows_per_step * static_cast<uint32_t>(T);
    const bool exclusions = p.banned != nullptr;

    // Tickets are fetched one row ahead, so the atomic's round trip overlaps a row.
    uint32_t next_ticket = 0;
    if (tid == 0) next_ticket = atomicAdd(p.ticket, 1u);
    for (;;) {
        if (tid == 0) {
            sh.ticket = static_cast<int>(next_ticket);
            if (next_ticket < total) next_ticket = atomicAdd(p.ticket, 1u);
        }
        block_sync();
        const uint32_t tk = static_cast<uint32_t>(sh.ticket);
        if (tk >= total) break;
        const int t = static_cast<int>(tk / rows_per_step);
        const uint32_t rem = tk - static_cast<uint32_t>(t) * rows_per_step;
        const int b = static_cast<int>(rem / static_cast<uint32_t>(K));
        const int k = static_cast<int>(rem - static_cast<uint32_t>(b) * static_cast<uint32_t>(K));
        const Meta m = load_meta(p, b);
        const int64_t rowi = (static_cast<int64_t>(b) * T + t) * K + k;

        // Rows an active step can read (at t = 0, only beam 0).
        if (t < m.steps && k < m.beam && (t > 0 || k == 0)) {
            const char* grow = static_cast<const char*>(p.inputs) + rowi * static_cast<int64_t>(V) * E::kBytes;
            // Record: the row's best LIST eligible entries by x. A parent read at step t
            // has length t, so EOS tokens are masked while t + 1 < min_length.
            const bool mask_eos = m.eos >= 0 && t + 1 < m.min_length;
            WarpTopK<LIST> wt;
            bool inv3 = false;
            bool check_inv = false;
            // NT threads (local index ltid) scan the row; each of their warps keeps a list.
            auto record_scan = [&](auto nt, const char* src, const RowSplit& rs, float xthr, int ltid) {
                constexpr int NT = decltype(nt)::value;
                wt.init(xthr);
                auto hit = [&](float x, int v, bool valid) {
                    uint64_t key = 0;
                    if (valid && x >= wt.thr && x < f_inf() && x != f_ninf() && !(exclusions && p.banned[v]) &&
                        !(mask_eos && is_eos(p, m, v)))
                        key = make_key(x, static_cast<uint32_t>(v));
                    wt.offer(key, lane);
                };
                if (check_inv) {
                    // No pass 1 ran: the NaN/+inf test needs every entry.
                    scan_chunks_ballot_n<DT, NT>(src, rs, p.staged != 0, ltid, [&](float x) {
                        inv3 |= !(x < f_inf());
                        return x >= wt.thr;
                    }, hit);
                } else {
                    // A chunk is looked at only when its largest entry reaches the threshold.
                    group_scan<DT, NT>(src, rs, ltid, [&]() { return wt.thr; }, hit);
                }
            };
            Prep o;
            // From logits, warps 4-7 scan while warps 0-3 compute the logsumexp. The bound
            // (the LIST-th largest thread maximum) is also used with banned tokens: the record
            // keeps only eligible entries at or above it, and a row with fewer than LIST such
            // entries (a banned entry took one of the top thread maxima) is redone below
            // without a bound.
            // With banned tokens the bound is ranked lower (LIST + LIST / 2 thread maxima), so
            // that a few banned entries among them still leave LIST eligible ones above it.
            const RecordOut ro{p.rkeys + rowi * LIST, LIST, mask_eos, exclusions};
            prepare_row<DT, LOGITS, LIST>(p, sh, srow, grow, phase, p.staged != 0, true,
                                          exclusions ? LIST + LIST / 2 : LIST, m, o,
                                          [&](const char* src, const RowSplit& rs, float xthr) {
                                              record_scan(std::integral_constant<int, kThreads / 2>{}, src, rs, xthr,
                                                          tid - kThreads / 2);
                                              const int lw = warp - kWarps / 2;
                                              if (lane < LIST) sh.wkeys[lw * LIST + lane] = wt.wl;
                                              const unsigned nz = __ballot_sync(0xffffffffu, lane < LIST && wt.wl != 0);
                                              if (lane == 0) sh.nlist[warp] = __popc(nz);
                                              half_sync(1);
                                              rank_merge<LIST>(sh.wkeys, kWarps / 2, lw, wt.wl, p.rkeys + rowi * LIST);
                                          },
                                          LOGITS ? &ro : nullptr);
            if (o.aborted) break;
            constexpr int kLists = LOGITS ? kWarps / 2 : kWarps;
            if constexpr (!LOGITS) {
                check_inv = !o.inv_known;
                record_scan(std::integral_constant<int, kThreads>{}, o.src, o.rs, o.xthr, tid);
            }
            const bool invalid = check_inv ? !block_and(!inv3) : o.invalid;
            // The record: rank merge of the list warps' lists (from logits, warps 4-7 already
            // did it while warps 0-3 finished the logsumexp).
            if constexpr (!LOGITS) {
                if (lane < LIST) sh.wkeys[warp * LIST + lane] = wt.wl;
                const unsigned nz = __ballot_sync(0xffffffffu, lane < LIST && wt.wl != 0);
                if (lane == 0) sh.nlist[warp] = __popc(nz);
                block_sync();
                rank_merge<LIST>(sh.wkeys, kWarps, warp, wt.wl, p.rkeys + rowi * LIST);
            }
            if (exclusions && o.xthr != f_ninf()) {
                block_sync();  // the lists' counts of every list warp are visible
                int found = 0;
#pragma unroll
                for (int w = 0; w < kLists; ++w) found += sh.nlist[kWarps - kLists + w];
                block_sync();
                if (found < LIST) {
                    // Fewer than LIST eligible entries reached the bound: the record again, unbounded.
                    if constexpr (LOGITS) {
                        if (warp >= kWarps / 2) {
                            record_scan(std::integral_constant<int, kThreads / 2>{}, o.src, o.rs, f_ninf(),
                                        tid - kThreads / 2);
                            const int lw = warp - kWarps / 2;
                            if (lane < LIST) sh.wkeys[lw * LIST + lane] = wt.wl;
                            const unsigned nz = __ballot_sync(0xffffffffu, lane < LIST && wt.wl != 0);
                            if (lane == 0) sh.nlist[warp] = __popc(nz);
                            half_sync(1);
                            rank_merge<LIST>(sh.wkeys, kWarps / 2, lw, wt.wl, p.rkeys + rowi * LIST);
                        }
                    } else {
                        record_scan(std::integral_constant<int, kThreads>{}, o.src, o.rs, f_ninf(), tid);
                        if (lane < LIST) sh.wkeys[warp * LIST + lane] = wt.wl;
                        const unsigned nz = __ballot_sync(0xffffffffu, lane < LIST && wt.wl != 0);
                        if (lane == 0) sh.nlist[warp] = __popc(nz);
                        block_sync();
                        rank_merge<LIST>(sh.wkeys, kWarps, warp, wt.wl, p.rkeys + rowi * LIST);
                    }
                    block_sync();
                }
            }
            if (tid == 0) {
                int total = 0;
#pragma unroll
                for (int w = 0; w < kLists; ++w) total += sh.nlist[kWarps - kLists + w];
                p.rlse[rowi] = o.lse;
                p.rinfo[rowi] = (invalid ? 1u : 0u) | (static_cast<uint32_t>(total < LIST ? total : LIST) << 8);
            }
        }

        // Arrive: the K rows of (t, b), prepared or not, and for t > 0 the selection of t - 1.
        // From logits every thread has passed a CTA barrier since its last write of this row
        // (the end of prepare_row, or the ticket's), except thread 0's own record header above;
        // log-probability rows merge their record after their last barrier.
        chain_arrive<DT, LOGITS, KMAX, LIST, kThreads>(p, sh.sel, t, b, m, tid, 0, LOGITS);
    }
}

// ---------------------------------------------------------------------------
// Chained decode of log-probability rows by single warps (beams up to 16, no banned
// tokens). Each warp takes row tickets on its own: it streams the row once (eight
// 16-byte loads in flight per lane) keeping the lane's maximum (NaN-propagating) and
// its four largest entries; the LIST-th largest lane maximum bounds the record from
// below (LIST eligible entries reach it), so the record is the best LIST of the kept
// entries at or above it -- a lane whose fourth entry reaches the bound reads its share
// again, with the whole warp. Rows with NaN/+inf, without a bound, or with too many
// candidates fall back to a full scan with the register top-k. Arrival and selection
// are the chained protocol at group width 32; no barrier spans more than one warp.
// ---------------------------------------------------------------------------
constexpr int kWarpCand = 64;  // record candidates per warp

struct WarpRowShared {
    SelScratch sel;
    uint64_t cand[kWarpCand];
};

// Top four (value, index) of a lane, v[0] >= ... >= v[3]; strict comparisons, so NaN
// never enters.
__device__ __forceinline__ void lane_top4(float (&v)[4], int (&ix)[4], float x, int i) {
    if (!(x > v[3])) return;
    if (x > v[1]) {
        v[3] = v[2];
        ix[3] = ix[2];
        v[2] = v[1];
        ix[2] = ix[1];
        if (x > v[0]) {
            v[1] = v[0];
            ix[1] = ix[0];
            v[0] = x;
            ix[0] = i;
        } else {
            v[1] = x;
            ix[1] = i;
        }
    } else if (x > v[2]) {
        v[3] = v[2];
        ix[3] = ix[2];
        v[2] = x;
        ix[2] = i;
    } else {
        v[3] = x;
        ix[3] = i;
    }
}

// The lane owning entry v of a row split rs among 32 lanes (chunk c on lane c mod 32,
// ragged ends on lanes 0 .. n_ends - 1); -1 outside the row.
__device__ __forceinline__ int warp_owner(const RowSplit& rs, int v) {
    if (v < 0 || v >= rs.V) return -1;
    if (v < rs.head) return v;
    if (v >= rs.tail0) return rs.head + (v - rs.tail0);
    return ((v - rs.head) / rs.per) & 31;
}

// The record of one log-probability row (best LIST eligible entries by x-key), written
// to rec by the calling warp; returns the row's info word (bit 0: NaN/+inf; count << 8).
template <int DT, int LIST>
__device__ uint32_t warp_row_record(const DecodeParams& p, WarpRowShared& ws, const char* row, const Meta& m, int t,
                                    uint64_t* rec) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    constexpr int UR = 4;
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    const int V = p.V;
    const RowSplit rs = RowSplit::of<E::kBytes>(row, V);
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    const bool mask_eos = m.eos >= 0 && t + 1 < m.min_length;
    // EOS tokens of this lane: they never bound the record; a masked one is left out of the
    // four, and a lane owning two masked ones reads its share again.
    bool dirty = false;
    int skip = -1, n_masked = 0;
    if (m.eos >= 0) {
        auto own = [&](int v) {
            if (warp_owner(rs, v) != lane) return;
            dirty = true;
            if (mask_eos && v != skip) {
                skip = v;
                ++n_masked;
            }
        };
        own(m.eos);
        for (int i = 0; i < p.n_extra; ++i) own(p.extra[i]);
    }
    float mxn = f_ninf();
    float tv[4] = {f_ninf(), f_ninf(), f_ninf(), f_ninf()};
    int ti[4] = {0, 0, 0, 0};
    auto single = [&](int v) {
        const float x = load_elem<DT>(row, v);
        mxn = max_nan(mxn, x);
        if (v != skip) lane_top4(tv, ti, x, v);
    };
    if (lane < rs.head && lane < rs.n_ends()) single(rs.end_entry(lane));
    // Warp-wide insertion threshold: the LIST-th largest of the lanes' best entries so
    // far (lanes owning an EOS token excluded, as for the bound below) is LIST distinct
    // eligible entries, so it never exceeds the row's final bound; entries below it are
    // never candidates and need not enter the lane lists. Without it a warp takes the
    // insertion branch whenever any one of its 32 lanes has a new top-4 entry.
    float wthr = f_ninf();
    // Lane 0 keeps a bulk L2 prefetch PD iterations (PD * UR * 512 bytes) ahead of the
    // warp's loads: more bytes in flight per SM than the registers of UR loads allow.
    constexpr int PD = 4;
    constexpr uint32_t kIterBytes = UR * 32 * 16;
    const uint32_t body_bytes = static_cast<uint32_t>(rs.nvec) * 16u;
    if (lane == 0 && body_bytes > 0) prefetch_l2_bulk(body, body_bytes < PD * kIterBytes ? body_bytes : PD * kIterBytes);
    auto prefetch_ahead = [&](int c00) {
        const uint32_t ahead = static_cast<uint32_t>(c00) * 16u + PD * kIterBytes;
        if (lane == 0 && ahead < body_bytes) {
            const uint32_t n = body_bytes - ahead;
            prefetch_l2_bulk(body + ahead, n < kIterBytes ? n : kIterBytes);
        }
    };
    auto raise_wthr = [&](int it) {
        if (it < 2 || (it & 3) == 3)
            wthr = fmaxf(wthr, __shfl_sync(0xffffffffu, warp_sort_desc(dirty ? f_ninf() : tv[0]), LIST - 1));
    };
    if constexpr (E::kBytes == 2) {
        uint32_t mx2 = h2_ninf<DT>();
        for (int c00 = 0, it = 0; c00 < rs.nvec; c00 += UR * 32, ++it) {
            const int c0 = c00 + lane;
            prefetch_ahead(c00);
            uint4 q[UR];
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * 32;
                if (c < rs.nvec) q[u] = ld_stream_v4(body + static_cast<size_t>(c) * 16);
            }
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * 32;
                if (c < rs.nvec) {
                    // One NaN-propagating chunk maximum serves both the row maximum and
                    // the top-4 test: a row holding NaN or +inf discards the lane lists
                    // (it takes the full-scan fallback), so a chunk skipped because a NaN
                    // hid its maximum never matters.
                    const uint32_t m2 = h2_max_nan<DT>(h2_max_nan<DT>(q[u].x, q[u].y), h2_max_nan<DT>(q[u].z, q[u].w));
                    mx2 = h2_max_nan<DT>(mx2, m2);
                    const float cmax = fmaxf(h2_lo<DT>(m2), h2_hi<DT>(m2));
                    if (cmax > tv[3] && cmax >= wthr) {
                        float x[PER];
                        unpack16<DT>(q[u], x);
#pragma unroll
                        for (int e = 0; e < PER; ++e)
                            if (rs.head + c * PER + e != skip && x[e] >= wthr)
                                lane_top4(tv, ti, x[e], rs.head + c * PER + e);
                    }
                }
            }
            raise_wthr(it);
        }
        mxn = max_nan(mxn, max_nan(h2_lo<DT>(mx2), h2_hi<DT>(mx2)));
    } else {
        for (int c00 = 0, it = 0; c00 < rs.nvec; c00 += UR * 32, ++it) {
            const int c0 = c00 + lane;
            prefetch_ahead(c00);
            uint4 q[UR];
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * 32;
                if (c < rs.nvec) q[u] = ld_stream_v4(body + static_cast<size_t>(c) * 16);
            }
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * 32;
                if (c < rs.nvec) {
                    const float a = __uint_as_float(q[u].x), b = __uint_as_float(q[u].y);
                    const float d = __uint_as_float(q[u].z), e = __uint_as_float(q[u].w);
                    const float cm = max_nan(max_nan(a, b), max_nan(d, e));  // as above
                    mxn = max_nan(mxn, cm);
                    if (cm > tv[3] && cm >= wthr) {
                        const int base = rs.head + c * 4;
                        if (base != skip && a >= wthr) lane_top4(tv, ti, a, base);
                        if (base + 1 != skip && b >= wthr) lane_top4(tv, ti, b, base + 1);
                        if (base + 2 != skip && d >= wthr) lane_top4(tv, ti, d, base + 2);
                        if (base + 3 != skip && e >= wthr) lane_top4(tv, ti, e, base + 3);
                    }
                }
            }
            raise_wthr(it);
        }
    }
    if (lane >= rs.head && lane < rs.n_ends()) single(rs.end_entry(lane));
    const bool bad = !(mxn < f_inf());
    const bool any_bad = __any_sync(0xffffffffu, bad);
    auto eligible = [&](int v) { return !(mask_eos && is_eos(p, m, v)); };
    const float bound = __shfl_sync(0xffffffffu, warp_sort_desc((bad || dirty) ? f_ninf() : mxn), LIST - 1);
    int n = 0;
    if (!any_bad && bound != f_ninf()) {
        auto push = [&](bool cond, float x, int v) {
            const unsigned mask = __ballot_sync(0xffffffffu, cond);
            const int pos = n + __popc(mask & lt);
            if (cond && pos < kWarpCand) ws.cand[pos] = make_key(x, static_cast<uint32_t>(v));
            n += __popc(mask);
        };
        const bool reread = n_masked > 1 || tv[3] >= bound;
#pragma unroll
        for (int u = 0; u < 4; ++u) push(!reread && tv[u] >= bound, tv[u], ti[u]);
        unsigned todo = __ballot_sync(0xffffffffu, reread);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            if (src < rs.n_ends()) {
                const int v = rs.end_entry(src);
                const float x = lane == 0 ? load_elem<DT>(row, v) : f_ninf();
                push(lane == 0 && x >= bound && x < f_inf() && eligible(v), x, v);
            }
            const int nch = src < rs.nvec ? (rs.nvec - src + 31) / 32 : 0;
            for (int r0 = 0; r0 < nch; r0 += 32) {
                const int c = src + (r0 + lane) * 32;
                const bool have = r0 + lane < nch;
                float x[PER];
                if (have) unpack16<DT>(ld_stream_v4(body + static_cast<size_t>(c) * 16), x);
#pragma unroll
                for (int e = 0; e < PER; ++e) {
                    const int v = rs.head + c * PER + e;
                    push(have && x[e] >= bound && x[e] < f_inf() && eligible(v), x[e], v);
                }
            }
        }
        __syncwarp();
        if (n <= kWarpCand) {
            // Rank by counting (keys are unique).
            for (int i = lane; i < n; i += 32) {
                const uint64_t key = ws.cand[i];
                int rank = 0;
                for (int j = 0; j < n; ++j) rank += ws.cand[j] > key ? 1 : 0;
                if (rank < LIST) rec[rank] = key;
            }
            __syncwarp();
            return (any_bad ? 1u : 0u) | (static_cast<uint32_t>(n < LIST ? n : LIST) << 8);
        }
    }
    // Fallback: the whole row through the register top-k.
    WarpTopK<LIST> wt;
    wt.init(f_ninf());
    scan_chunks_ballot_n<DT, 32>(row, rs, false, lane, [&](float x) { return x >= wt.thr; },
                                 [&](float x, int v, bool valid) {
                                     uint64_t key = 0;
                                     if (valid && x >= wt.thr && x < f_inf() && x != f_ninf() && eligible(v))
                                         key = make_key(x, static_cast<uint32_t>(v));
                                     wt.offer(key, lane);
                                 });
    if (lane < LIST) rec[lane] = wt.wl;
    const int cnt = __popc(__ballot_sync(0xffffffffu, lane < LIST && wt.wl != 0));
    __syncwarp();
    return (any_bad ? 1u : 0u) | (static_cast<uint32_t>(cnt) << 8);
}

template <int DT, int KMAX>
__global__ void __launch_bounds__(kThreads, 3) decode_chain_warp_kernel(const __grid_constant__ DecodeParams p) {
    constexpr int LIST = chain_list_len<KMAX>();
    using E = Elem<DT>;
    __shared__ WarpRowShared wsh[kWarps];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    WarpRowShared& ws = wsh[warp];
    const int bar = 1 + warp;  // the warp's named barrier (0 is the CTA's)
    const int K = p.K, V = p.V, T = p.T;
    const uint32_t rows_per_step = static_cast<uint32_t>(p.B) * static_cast<uint32_t>(K);
    const uint32_t total = rows_per_step * static_cast<uint32_t>(T);
    // Tickets are fetched one row ahead, so the atomic's round trip overlaps a row.
    uint32_t next = 0;
    if (lane == 0) next = atomicAdd(p.ticket, 1u);
    for (;;) {
        const uint32_t tk = __shfl_sync(0xffffffffu, next, 0);
        if (tk >= total) break;
        if (lane == 0) next = atomicAdd(p.ticket, 1u);
        const int t = static_cast<int>(tk / rows_per_step);
        const uint32_t rem = tk - static_cast<uint32_t>(t) * rows_per_step;
        const int b = static_cast<int>(rem / static_cast<uint32_t>(K));
        const int k = static_cast<int>(rem - static_cast<uint32_t>(b) * static_cast<uint32_t>(K));
        const Meta m = load_meta(p, b);
        const int64_t rowi = (static_cast<int64_t>(b) * T + t) * K + k;
        if (t < m.steps && k < m.beam && (t > 0 || k == 0)) {
            const char* row = static_cast<const char*>(p.inputs) + rowi * static_cast<int64_t>(V) * E::kBytes;
            const uint32_t info = warp_row_record<DT, LIST>(p, ws, row, m, t, p.rkeys + rowi * LIST);
            if (lane == 0) p.rinfo[rowi] = info;
        }
        chain_arrive<DT, false, KMAX, LIST, 32>(p, ws.sel, t, b, m, lane, bar);
    }
}

template <int DT, int KMAX>
static cudaError_t launch_chain_warp_as(const DecodeParams& p, cudaStream_t stream, int sm_count) {
    auto kernel = decode_chain_warp_kernel<DT, KMAX>;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const int64_t warps = static_cast<int64_t>(p.B) * p.K * p.T;
    int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
    if (grid * kWarps > warps) grid = (warps + kWarps - 1) / kWarps;
    kernel<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

template <int DT, bool LOGITS, int KMAX>
static cudaError_t launch_chain_as(const DecodeParams& p, cudaStream_t stream, int sm_count) {
    const size_t dyn = p.staged ? static_cast<size_t>(p.row_smem) : 0;
    auto kernel = decode_chain_kernel<DT, LOGITS, KMAX>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, dyn);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const int64_t tickets = static_cast<int64_t>(p.B) * p.K * p.T;
    int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
    if (grid > tickets) grid = tickets;
    kernel<<<static_cast<unsigned>(grid), kThreads, dyn, stream>>>(p);
    return cudaGetLastError();
}

// Launch of one (dtype, logits) family: the beam size picks the register
// top-k width (1..16) or the generic radix-select path.
template <int DT, bool LOGITS, int KMAX>
static cudaError_t launch_decode_as(const DecodeParams& p, cudaStream_t stream, int sm_count) {
    constexpr int KCAP = KMAX > 0 ? kFastBeam : kSelectCap;
    const size_t sel = (sizeof(SelectShared<KCAP>) + 127) & ~static_cast<size_t>(127);
    const size_t dyn = sel + (p.staged ? static_cast<size_t>(p.row_smem) : 0);
    auto kernel = decode_kernel<DT, LOGITS, KMAX>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, dyn);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const int64_t tickets = static_cast<int64_t>(p.B) * p.K * p.T;
    int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
    if (grid > tickets) grid = tickets;
    kernel<<<static_cast<unsigned>(grid), kThreads, dyn, stream>>>(p);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Chained decode for beams above 16 (up to DBS_CUDA_MAX_BEAM). Row records hold
// LIST = 2K entries: the entries that reach the filter bound (the LIST-th largest of
// the 256 thread maxima, LIST <= 256) are collected into shared memory and
// bitonic-sorted; without a bound, or when more than kWideCand entries reach it, a
// block radix select over the row takes the LIST best. The selection turns the K
// records into row lists and merges them with a block radix select (select_step).
// ---------------------------------------------------------------------------
constexpr int kWideCand = 2048;  // candidate buffer of the wide record (u64 keys)

struct WideShared {
    uint64_t cand[kWideCand];
    int n_cand;
    unsigned fb[DBS_CUDA_MAX_BEAM / 32];  // rows whose record is not enough
    unsigned long long thr;               // selection: lower bound on the step's beam-th key
};

// Every eligible entry of the group's share with x >= thr, appended as an x-key to
// ws.cand (counted in ws.n_cand; entries past kWideCand are counted, not stored). Four
// chunks are tested per round, each by its largest entry.
template <int DT, int NT, class Elig>
__device__ __forceinline__ void collect_candidates(WideShared& ws, const char* row, const RowSplit& rs, int ltid,
                                                   float thr, Elig&& eligible) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    constexpr int UR = 4;
    const int lane = ltid & 31;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    auto push = [&](float x, int v, bool cond) {
        const unsigned mask = __ballot_sync(0xffffffffu, cond);
        if (!mask) return;
        int base = 0;
        if (lane == 0) base = atomicAdd(&ws.n_cand, __popc(mask));
        base = __shfl_sync(0xffffffffu, base, 0);
        const int pos = base + __popc(mask & ((1u << lane) - 1u));
        if (cond && pos < kWideCand) ws.cand[pos] = make_key(x, static_cast<uint32_t>(v));
    };
    auto chunk_top = [&](const uint4& q) -> float {
        if constexpr (E::kBytes == 2) {
            const uint32_t m2 = h2_max<DT>(h2_max<DT>(q.x, q.y), h2_max<DT>(q.z, q.w));
            return fmaxf(h2_lo<DT>(m2), h2_hi<DT>(m2));
        } else {
            return fmaxf(fmaxf(__uint_as_float(q.x), __uint_as_float(q.y)), fmaxf(__uint_as_float(q.z), __uint_as_float(q.w)));
        }
    };
    const int rounds = (rs.nvec + NT - 1) / NT;
    for (int r0 = 0; r0 < rounds; r0 += UR) {
        uint4 q[UR];
        bool hit[UR];
        bool any = false;
#pragma unroll
        for (int u = 0; u < UR; ++u) {
            const int c = ltid + (r0 + u) * NT;
            q[u] = make_uint4(0u, 0u, 0u, 0u);
            hit[u] = false;
            if (r0 + u < rounds && c < rs.nvec) {
                q[u] = *reinterpret_cast<const uint4*>(body + static_cast<size_t>(c) * 16);
                hit[u] = chunk_top(q[u]) >= thr;
            }
            any |= hit[u];
        }
        if (!__any_sync(0xffffffffu, any)) continue;
#pragma unroll
        for (int u = 0; u < UR; ++u) {
            if (!__any_sync(0xffffffffu, hit[u])) continue;
            const int c = ltid + (r0 + u) * NT;
            float x[PER];
            unpack16<DT>(q[u], x);
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                const int v = rs.head + c * PER + j;
                push(x[j], v, hit[u] && x[j] >= thr && x[j] < f_inf() && x[j] != f_ninf() && eligible(v));
            }
        }
    }
    const bool valid = ltid < rs.n_ends();
    const int v = valid ? rs.end_entry(ltid) : 0;
    const float x = valid ? load_elem<DT>(row, v) : f_ninf();
    push(x, v, valid && x >= thr && x < f_inf() && eligible(v));
}

// Sorts ws.cand[0, n) descending (n <= kWideCand) and writes the first min(n, LIST) to out.
__device__ __forceinline__ int sort_candidates(WideShared& ws, int n, int LIST, uint64_t* out) {
    if (n <= 512) {
        // Up to 512 keys: each key's rank is the number of larger keys (keys are unique),
        // one pass without a sorting network.
        for (int i = threadIdx.x; i < n; i += kThreads) {
            const uint64_t key = ws.cand[i];
            int rank = 0;
#pragma unroll 4
            for (int j = 0; j < n; ++j) rank += ws.cand[j] > key ? 1 : 0;
            if (rank < LIST) out[rank] = key;
        }
        block_sync();
        return n < LIST ? n : LIST;
    }
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    for (int i = n + static_cast<int>(threadIdx.x); i < n2; i += kThreads) ws.cand[i] = 0;
    block_sync();
    bitonic_desc(ws.cand, n2);
    const int cnt = n < LIST ? n : LIST;
    for (int i = threadIdx.x; i < cnt; i += kThreads) out[i] = ws.cand[i];
    block_sync();
    return cnt;
}

// Fallback of the wide selection: the best K full keys of row (t, b, k) with the parent
// known, by a block radix select over the row, written as the row's list.
template <int DT, bool LOGITS>
__device__ void rescan_row_wide(const DecodeParams& p, RowShared& sh, WideShared& ws, int t, int b, int k,
                                const Meta& m, float lse) {
    using E = Elem<DT>;
    const int K = p.K, V = p.V, LIST = p.list_len;
    const int64_t s = static_cast<int64_t>(b) * K + k;
    const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + k;
    const char* grow = static_cast<const char*>(p.inputs) + rowi * static_cast<int64_t>(V) * E::kBytes;
    const float pr = ld_cg(p.raw + s);
    const bool mask_eos = m.eos >= 0 && ld_cg(p.len + s) + 1 < m.min_length;
    const uint32_t base = static_cast<uint32_t>(k) * static_cast<uint32_t>(V);
    const ConsView cv = chain_prefix(p, t, s);
    auto gen = [&](int v) -> uint64_t {
        const float x = load_elem<DT>(grow, v);
        if (!(x < f_inf()) || x == f_ninf()) return 0;
        if (p.banned && p.banned[v]) return 0;
        if (mask_eos && is_eos(p, m, v)) return 0;
        const float raw = constrained_raw<LOGITS>(p, cv, pr, x, lse, v);
        return raw == f_ninf() ? 0 : make_key(raw, base + static_cast<uint32_t>(v));
    };
    uint64_t* list = p.keys + s * LIST;
    int cnt = 0;
    if (!LOGITS || lse != f_ninf()) cnt = block_select(sh, gen, V, K, [&](int pos, uint64_t key) { list[pos] = key; });
    for (int i = cnt + static_cast<int>(threadIdx.x); i < LIST; i += kThreads) list[i] = 0;
    block_sync();
}

// Candidates of step t for an unconstrained buffered selection (K <= 128), gathered into
// cbuf (count in ws.n_cand). Without constraints a record's raw scores never increase
// along it (raw = parent raw + (x - lse), x non-increasing), so a record is enough when
// no entry may be missing after it, or when its entry R - 1 is strictly above its last
// entry (R = beam): two entries decide it. The first two entries of every exact row
// sample the step; the beam-th largest sample, ws.thr, bounds the step's beam-th
// candidate from below (samples are candidates), and each exact row contributes its
// entries down to the first whose raw score is below the bound's. Rows that are not
// exact are marked in ws.fb.
template <bool LOGITS>
__device__ void gather_sampled(const DecodeParams& p, RowShared& sh, WideShared& ws, int t, int b, const Meta& m,
                               uint64_t* cbuf) {
    constexpr int kMaxRows = kWarps * 32 / 2;  // 128: two samples per row in sh.wkeys
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int K = p.K, LIST = p.list_len;
    const uint32_t V = static_cast<uint32_t>(p.V);
    const bool active = t < m.steps;
    const int R = m.beam;
    const int64_t row0 = (static_cast<int64_t>(b) * p.T + t) * K;
    float* s_pr = sh.lanes;              // parent raw score of row k
    float* s_lse = sh.lanes + kMaxRows;  // logsumexp of row k
    int* s_cnt = sh.hist;                // record entries of row k to scan (0: none)
    // Phase A: thread k takes row k.
    for (int k = tid; k < K; k += kThreads) {
        const int64_t s = static_cast<int64_t>(b) * K + k;
        const int64_t rowi = row0 + k;
        int scan = 0;
        float pr = 0.0f, lse = 0.0f;
        bool read = false;
        if (active && k < m.beam && (t > 0 || k == 0)) {
            pr = ld_cg(p.raw + s);
            const int plen = ld_cg(p.len + s);
            const uint8_t ended = ld_cg(p.ended + s);
            const uint32_t info = ld_cg(p.rinfo + rowi);
            lse = ld_cg(p.rlse + rowi);
            read = f_finite(pr) && !(m.eos >= 0 && ended != 0);
            if (read) {
                const int cnt = static_cast<int>(info >> 8);
                const bool partial = cnt >= LIST || (info & 2u) != 0;
                const uint64_t* rec = p.rkeys + rowi * LIST;
                const uint64_t x0 = cnt > 0 ? ld_cg(rec) : 0;
                const uint64_t x1 = cnt > 1 ? ld_cg(rec + 1) : 0;
                const uint64_t xr = (partial && cnt >= R) ? ld_cg(rec + R - 1) : 0;
                const uint64_t xl = (partial && cnt > 0) ? ld_cg(rec + cnt - 1) : 0;
                auto raw_of = [&](uint64_t xk) {
                    const float x = key_raw(xk);
                    const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                    return (lp < f_inf() && lp != f_ninf()) ? __fadd_rn(pr, lp) : f_ninf();
                };
                auto key_of = [&](uint64_t xk) -> uint64_t {
                    if (xk == 0) return 0;
                    const float raw = raw_of(xk);
                    return raw != f_ninf() ? make_key(raw, static_cast<uint32_t>(k) * V + key_index(xk)) : 0;
                };
                bool exact = plen == t;
                if (partial) exact = exact && cnt >= R && raw_of(xr) > raw_of(xl);
                if (exact) {
                    scan = cnt;
                    sh.wkeys[2 * k] = key_of(x0);
                    sh.wkeys[2 * k + 1] = key_of(x1);
                } else {
                    atomicOr(&ws.fb[k >> 5], 1u << (k & 31));
                }
                if (info & 1u) sh.sel.invalid = 1;
            }
        }
        s_pr[k] = pr;
        s_lse[k] = lse;
        s_cnt[k] = scan;
        if (p.row_lse) p.row_lse[rowi] = (read && LOGITS) ? lse : 0.0f;
    }
    block_sync();
    // The bound: the sample of rank R - 1 (keys are unique); 0 with fewer than R samples.
    for (int i = tid; i < 2 * K; i += kThreads) {
        const uint64_t v = sh.wkeys[i];
        if (v == 0) continue;
        int rank = 0;
#pragma unroll 8
        for (int j = 0; j < 2 * K; ++j) rank += sh.wkeys[j] > v ? 1 : 0;
        if (rank == R - 1) ws.thr = v;
    }
    block_sync();
    const uint64_t thr = ws.thr;
    const float thr_raw = thr ? key_raw(thr) : f_ninf();
    // Phase B: warp w takes rows w, w + kWarps, ...; the first 32 entries of all its rows
    // are loaded before any is used.
    constexpr int kMaxJ = kMaxRows / kWarps;
    uint64_t first[kMaxJ];
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        const int k = warp + kWarps * j;
        first[j] = (k < K && lane < s_cnt[k]) ? ld_cg(p.rkeys + (row0 + k) * LIST + lane) : 0;
    }
    const unsigned lt = (1u << lane) - 1u;
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        const int k = warp + kWarps * j;
        if (k >= K) break;
        const int sc = s_cnt[k];
        if (sc == 0) continue;
        const float pr = s_pr[k], lse = s_lse[k];
        const uint64_t* rec = p.rkeys + (row0 + k) * LIST;
        uint64_t xk = first[j];
        for (int c0 = 0; c0 < sc; c0 += 32) {
            if (c0 > 0) xk = c0 + lane < sc ? ld_cg(rec + c0 + lane) : 0;
            float raw = f_ninf();
            uint64_t key = 0;
            const bool have = c0 + lane < sc && xk != 0;
            if (have) {
                const float x = key_raw(xk);
                const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                if (lp < f_inf() && lp != f_ninf()) raw = __fadd_rn(pr, lp);
                if (raw != f_ninf()) key = make_key(raw, static_cast<uint32_t>(k) * V + key_index(xk));
            }
            const unsigned take = __ballot_sync(0xffffffffu, key != 0 && key >= thr);
            int base = 0;
            if (lane == 0 && take) base = atomicAdd(&ws.n_cand, __popc(take));
            base = __shfl_sync(0xffffffffu, base, 0);
            if ((take >> lane) & 1u) cbuf[base + __popc(take & lt)] = key;
            // Entries after one below the bound's raw score are below the bound.
            if (__any_sync(0xffffffffu, have && !(raw >= thr_raw))) break;
        }
    }
}

// Selection of step t of example b for beams above 16 (whole CTA). Rows whose record is
// not enough are marked in ws.fb and handed to fallback() (called by every thread),
// which fills their lists and returns true, or returns false to stop before the
// selection (nothing of step t is then written but the read rows' lists and row_lse).
// A record holds cnt = info >> 8 entries; when cnt reaches the list length or bit 1
// of info is set, entries may be missing after its last one.
template <bool LOGITS, int KCAP, class Fallback>
__device__ bool chain_select_wide_with(const DecodeParams& p, RowShared& sh, WideShared& ws, SelectShared<KCAP>& ss,
                                       int t, int b, const Meta& m, Fallback&& fallback, uint64_t* cbuf = nullptr,
                                       int cap = 0) {
    constexpr int kRegKeys = 8;  // record entries per lane kept in registers (LIST <= 256)
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int K = p.K, LIST = p.list_len;
    const uint32_t V = static_cast<uint32_t>(p.V);
    const bool active = t < m.steps;
    const int R = m.beam;
    // With a shared-memory buffer that holds every row's record, the candidates are
    // gathered there (non-zero keys only) and the selection reads them from it.
    const bool use_buf = cbuf != nullptr && LIST <= 32 * kRegKeys && K * LIST <= cap;
    // Buffered mode with up to 128 rows: the first two entries of every exact row are
    // kept as samples; the beam-th largest sample bounds the step's beam-th candidate
    // from below (the samples are candidates), and only candidates at or above it go on
    // to the radix select.
    const bool sample = use_buf && 2 * K <= kWarps * 32;
    const bool unconstrained = !(p.ngram > 0 || p.penalise);
    if (use_buf && tid == 0 && t + 1 < p.T) {
        // The next step's records do not depend on this step: bring them into L2 now.
        const int64_t row1 = (static_cast<int64_t>(b) * p.T + t + 1) * K;
        prefetch_l2_bulk(p.rkeys + row1 * LIST, static_cast<uint32_t>(K) * static_cast<uint32_t>(LIST) * 8u);
        const uintptr_t i0 = reinterpret_cast<uintptr_t>(p.rinfo + row1) & ~static_cast<uintptr_t>(15);
        const uintptr_t i1 = (reinterpret_cast<uintptr_t>(p.rinfo + row1 + K) + 15) & ~static_cast<uintptr_t>(15);
        prefetch_l2_bulk(reinterpret_cast<const void*>(i0), static_cast<uint32_t>(i1 - i0));
        const uintptr_t l0 = reinterpret_cast<uintptr_t>(p.rlse + row1) & ~static_cast<uintptr_t>(15);
        const uintptr_t l1 = (reinterpret_cast<uintptr_t>(p.rlse + row1 + K) + 15) & ~static_cast<uintptr_t>(15);
        prefetch_l2_bulk(reinterpret_cast<const void*>(l0), static_cast<uint32_t>(l1 - l0));
    }
    for (int i = tid; i < DBS_CUDA_MAX_BEAM / 32; i += kThreads) ws.fb[i] = 0;
    if (sample)
        for (int i = tid; i < 2 * K; i += kThreads) sh.wkeys[i] = 0;
    if (tid == 0) {
        sh.sel.invalid = 0;
        ws.n_cand = 0;
        ws.thr = 0;
    }
    block_sync();
    auto append = [&](uint64_t key) {
        const unsigned mask = __ballot_sync(0xffffffffu, key != 0);
        if (!mask) return;
        int base = 0;
        if (lane == 0) base = atomicAdd(&ws.n_cand, __popc(mask));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (key != 0) cbuf[base + __popc(mask & ((1u << lane) - 1u))] = key;
    };
    if (sample && unconstrained) gather_sampled<LOGITS>(p, sh, ws, t, b, m, cbuf);
    // Warp w takes rows w, w + kWarps, ...; their scalars are loaded 32 rows at a time (lane
    // j: the warp's row j of the batch) before the rows are processed one by one.
    for (int j0 = 0; !(sample && unconstrained) && warp + kWarps * j0 < K; j0 += 32) {
        const int kl = warp + kWarps * (j0 + lane);
        float pr_l = 0.0f, lse_l = 0.0f;
        int plen_l = 0;
        uint32_t info_l = 0;
        bool read_l = false;
        if (kl < K) {
            const int64_t s = static_cast<int64_t>(b) * K + kl;
            const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + kl;
            const float r = ld_cg(p.raw + s);
            plen_l = ld_cg(p.len + s);
            const uint8_t ended = ld_cg(p.ended + s);
            info_l = ld_cg(p.rinfo + rowi);
            lse_l = ld_cg(p.rlse + rowi);
            pr_l = r;
            read_l = active && kl < m.beam && (t > 0 || kl == 0) && f_finite(r) && !(m.eos >= 0 && ended != 0);
        }
        const unsigned reads = __ballot_sync(0xffffffffu, read_l);
        // Buffered mode: the next row's record entries are loaded while this row's are used.
        auto load_rec = [&](int j, uint64_t (&xk)[kRegKeys]) {
            const int k = warp + kWarps * (j0 + j);
            const bool rd = ((reads >> j) & 1u) && k < K;
            const int cnt = static_cast<int>(__shfl_sync(0xffffffffu, info_l, j) >> 8);
            const uint64_t* rec = p.rkeys + ((static_cast<int64_t>(b) * p.T + t) * K + k) * LIST;
#pragma unroll
            for (int u = 0; u < kRegKeys; ++u) {
                const int i = lane + 32 * u;
                xk[u] = (rd && i < cnt) ? ld_cg(rec + i) : 0;
            }
        };
        int nj = 0;  // rows of this warp in the batch
        while (nj < 32 && warp + kWarps * (j0 + nj) < K) ++nj;
        // Row j of the batch from `use`, with row j + 1's entries loaded into `load` (the two
        // register arrays swap roles from row to row, so no load is waited for early).
        auto row_step = [&](int j, const uint64_t (&use)[kRegKeys], uint64_t (&load)[kRegKeys]) {
            if (use_buf && j + 1 < nj) load_rec(j + 1, load);
            const int k = warp + kWarps * (j0 + j);
            const int64_t s = static_cast<int64_t>(b) * K + k;
            const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * K + k;
            const bool read = (reads >> j) & 1u;
            const float pr = __shfl_sync(0xffffffffu, pr_l, j);
            const int plen = __shfl_sync(0xffffffffu, plen_l, j);
            const uint32_t info = __shfl_sync(0xffffffffu, info_l, j);
            const float lse = __shfl_sync(0xffffffffu, lse_l, j);
            uint64_t* list = p.keys + s * LIST;
            if (read) {
                const int cnt = static_cast<int>(info >> 8);
                const bool partial = cnt >= LIST || (info & 2u) != 0;
                const uint64_t* rec = p.rkeys + rowi * LIST;
                const ConsView cv = chain_prefix(p, t, s);
                // Exactness of the record (as in the narrow case): R entries whose constrained
                // raw is strictly above the last entry's unconstrained raw. The record's EOS
                // masking assumed parent length t.
                auto entry_raw = [&](uint64_t xk, float& plain) {
                    const float x = key_raw(xk);
                    const float lp = LOGITS ? __fsub_rn(x, lse) : x;
                    plain = (lp < f_inf() && lp != f_ninf()) ? __fadd_rn(pr, lp) : f_ninf();
                    return cv.prefix ? constrained_raw<LOGITS>(p, cv, pr, x, lse, static_cast<int>(key_index(xk))) : plain;
                };
                if (use_buf) {
                    const uint64_t (&xk)[kRegKeys] = use;
                    uint64_t key[kRegKeys];
                    float raw[kRegKeys];
                    uint64_t last_x = 0;
#pragma unroll
                    for (int u = 0; u < kRegKeys; ++u) {
                        float plain;
                        raw[u] = xk[u] != 0 ? entry_raw(xk[u], plain) : f_ninf();
                        key[u] = raw[u] != f_ninf() ? make_key(raw[u], static_cast<uint32_t>(k) * V + key_index(xk[u])) : 0;
                        if (cnt > 0 && u == ((cnt - 1) >> 5)) last_x = xk[u];
                    }
                    float raw_last = f_ninf();
                    if (partial && cnt > 0) {
                        const uint64_t lx = __shfl_sync(0xffffffffu, last_x, (cnt - 1) & 31);
                        entry_raw(lx, raw_last);
                    }
                    int above = 0;
#pragma unroll
                    for (int u = 0; u < kRegKeys; ++u) above += raw[u] > raw_last ? 1 : 0;
                    above = warp_sum_i32(above);
                    const bool exact = plen == t && (!partial || above >= R);
                    if (exact) {
                        // All of the row's keys with one shared-memory atomic.
                        unsigned masks[kRegKeys];
                        int tot = 0;
#pragma unroll
                        for (int u = 0; u < kRegKeys; ++u) {
                            masks[u] = __ballot_sync(0xffffffffu, 32 * u < cnt && key[u] != 0);
                            tot += __popc(masks[u]);
                        }
                        int base = 0;
                        if (lane == 0 && tot) base = atomicAdd(&ws.n_cand, tot);
                        base = __shfl_sync(0xffffffffu, base, 0);
                        const unsigned lt = (1u << lane) - 1u;
#pragma unroll
                        for (int u = 0; u < kRegKeys; ++u) {
                            if ((masks[u] >> lane) & 1u) cbuf[base + __popc(masks[u] & lt)] = key[u];
                            base += __popc(masks[u]);
                        }
                        // The row's first two entries sample the step's candidates.
                        if (sample && lane < 2) sh.wkeys[2 * k + lane] = key[0];
                    }
                    if (lane == 0) {
                        if (!exact) atomicOr(&ws.fb[k >> 5], 1u << (k & 31));
                        if (info & 1u) sh.sel.invalid = 1;
                    }
                } else {
                    float raw_last = f_ninf();
                    if (partial && cnt > 0) entry_raw(ld_cg(rec + cnt - 1), raw_last);
                    int above = 0;
                    for (int i = lane; i < LIST; i += 32) {
                        uint64_t key = 0;
                        if (i < cnt) {
                            const uint64_t xk = ld_cg(rec + i);
                            float plain;
                            const float raw = entry_raw(xk, plain);
                            if (raw != f_ninf()) key = make_key(raw, static_cast<uint32_t>(k) * V + key_index(xk));
                            above += raw > raw_last ? 1 : 0;
                        }
                        list[i] = key;
                    }
                    above = warp_sum_i32(above);
                    const bool exact = plen == t && (!partial || above >= R);
                    if (lane == 0) {
                        if (!exact) atomicOr(&ws.fb[k >> 5], 1u << (k & 31));
                        if (info & 1u) sh.sel.invalid = 1;
                    }
                }
            } else if (!use_buf) {
                for (int i = lane; i < LIST; i += 32) list[i] = 0;
            }
            if (lane == 0 && p.row_lse) p.row_lse[rowi] = (read && LOGITS) ? lse : 0.0f;
        };
        uint64_t cur[kRegKeys], nxt[kRegKeys];
        if (use_buf) load_rec(0, cur);
        for (int j = 0; j < nj; j += 2) {
            row_step(j, cur, nxt);
            if (j + 1 < nj) row_step(j + 1, nxt, cur);
        }
    }
    block_sync();
    bool any_fb = false;
    for (int w = 0; w < (K + 31) / 32; ++w) any_fb |= ws.fb[w] != 0;
    if (any_fb) {
        if (!fallback()) {
            block_sync();
            return false;
        }
        if (use_buf) {
            // The rescanned rows' lists join the buffer.
            for (int w = 0; w < (K + 31) / 32; ++w) {
                unsigned bits = ws.fb[w];
                while (bits) {
                    const int k = w * 32 + __ffs(bits) - 1;
                    bits &= bits - 1;
                    if (warp == 0) {
                        const uint64_t* list = p.keys + (static_cast<int64_t>(b) * K + k) * LIST;
                        for (int i0 = 0; i0 < LIST; i0 += 32) append(i0 + lane < LIST ? ld_cg(list + i0 + lane) : 0);
                    }
                }
            }
            block_sync();
        }
    }
    if (tid == 0 && sh.sel.invalid && p.out.invalid_input) p.out.invalid_input[b] = 1;
    int n_cand = ws.n_cand;
    if (sample && !unconstrained) {
        for (int i = tid; i < 2 * K; i += kThreads) {
            const uint64_t v = sh.wkeys[i];
            if (v == 0) continue;
            int rank = 0;
#pragma unroll 8
            for (int j = 0; j < 2 * K; ++j) rank += sh.wkeys[j] > v ? 1 : 0;
            if (rank == R - 1) ws.thr = v;  // keys are unique: one sample has rank R - 1
        }
        block_sync();
        const uint64_t thr = ws.thr;
        if (thr != 0) {
            // In-place compaction of the keys >= thr, 8 per thread per round: a round's keys
            // are all read before any is written, and writes never pass the round's end.
            if (tid == 0) ws.n_cand = 0;
            block_sync();
            for (int r0 = 0; r0 < n_cand; r0 += 8 * kThreads) {
                uint64_t v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int i = r0 + u * kThreads + tid;
                    v[u] = i < n_cand ? cbuf[i] : 0;
                }
                block_sync();
                unsigned masks[8];
                int tot = 0;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    masks[u] = __ballot_sync(0xffffffffu, v[u] != 0 && v[u] >= thr);
                    tot += __popc(masks[u]);
                }
                int base = 0;
                if (lane == 0 && tot) base = atomicAdd(&ws.n_cand, tot);
                base = __shfl_sync(0xffffffffu, base, 0);
                const unsigned lt = (1u << lane) - 1u;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if ((masks[u] >> lane) & 1u) cbuf[base + __popc(masks[u] & lt)] = v[u];
                    base += __popc(masks[u]);
                }
                block_sync();
            }
            n_cand = ws.n_cand;
        }
    }
    __threadfence_block();
    block_sync();
    if (use_buf) select_step<0, KCAP>(p, sh, ss, t, b, m, cbuf, n_cand);
    else select_step<0, KCAP>(p, sh, ss, t, b, m);
    __threadfence();
    block_sync();
    return true;
}

template <int DT, bool LOGITS, int KCAP>
__device__ void chain_select_wide(const DecodeParams& p, RowShared& sh, WideShared& ws, SelectShared<KCAP>& ss,
                                  int t, int b, const Meta& m) {
    chain_select_wide_with<LOGITS, KCAP>(p, sh, ws, ss, t, b, m, [&]() {
        for (int w = 0; w < (p.K + 31) / 32; ++w) {
            unsigned bits = ws.fb[w];
            while (bits) {
                const int k = w * 32 + __ffs(bits) - 1;
                bits &= bits - 1;
                const int64_t rowi = (static_cast<int64_t>(b) * p.T + t) * p.K + k;
                rescan_row_wide<DT, LOGITS>(p, sh, ws, t, b, k, m, ld_cg(p.rlse + rowi));
            }
        }
        return true;
    }, ws.cand, kWideCand);
}

template <int DT, bool LOGITS, int KCAP>
__global__ void __launch_bounds__(kThreads, 2) decode_chain_wide_kernel(const __grid_constant__ DecodeParams p) {
    using E = Elem<DT>;
    __shared__ RowShared sh;
    extern __shared__ __align__(128) unsigned char dyn[];
    auto& ss = *reinterpret_cast<SelectShared<KCAP>*>(dyn);
    constexpr size_t kSelBytes = (sizeof(SelectShared<KCAP>) + 127) & ~static_cast<size_t>(127);
    auto& ws = *reinterpret_cast<WideShared*>(dyn + kSelBytes);
    char* srow = reinterpret_cast<char*>(dyn) + kSelBytes + ((sizeof(WideShared) + 127) & ~static_cast<size_t>(127));

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    if (tid == 0) mbar_init(&sh.mbar);
    block_sync();
    uint32_t phase = 0;

    const int K = p.K, V = p.V, T = p.T, LIST = p.list_len;
    const uint32_t rows_per_step = static_cast<uint32_t>(p.B) * static_cast<uint32_t>(K);
    const uint32_t total = rows_per_step * static_cast<uint32_t>(T);
    const bool exclusions = p.banned != nullptr;
    // With banned tokens the bound (from thread maxima that may be banned entries) is kept;
    // a row where fewer than LIST eligible entries reach it takes the block select below.
    const bool want_bound = LIST <= kWarps * 32;

    uint32_t next_ticket = 0;
    if (tid == 0) next_ticket = atomicAdd(p.ticket, 1u);
    for (;;) {
        if (tid == 0) {
            sh.ticket = static_cast<int>(next_ticket);
            if (next_ticket < total) next_ticket = atomicAdd(p.ticket, 1u);
        }
        block_sync();
        const uint32_t tk = static_cast<uint32_t>(sh.ticket);
        if (tk >= total) break;
        const int t = static_cast<int>(tk / rows_per_step);
        const uint32_t rem = tk - static_cast<uint32_t>(t) * rows_per_step;
        const int b = static_cast<int>(rem / static_cast<uint32_t>(K));
        const int k = static_cast<int>(rem - static_cast<uint32_t>(b) * static_cast<uint32_t>(K));
        const Meta m = load_meta(p, b);
        const int64_t rowi = (static_cast<int64_t>(b) * T + t) * K + k;

        if (t < m.steps && k < m.beam && (t > 0 || k == 0)) {
            const char* grow = static_cast<const char*>(p.inputs) + rowi * static_cast<int64_t>(V) * E::kBytes;
            const bool mask_eos = m.eos >= 0 && t + 1 < m.min_length;
            auto eligible = [&](int v) { return !(exclusions && p.banned[v]) && !(mask_eos && is_eos(p, m, v)); };
            if (tid == 0) ws.n_cand = 0;
            Prep o;
            // From logits, warps 4-7 collect the entries at or above the bound during pass 2.
            prepare_row<DT, LOGITS, 32>(p, sh, srow, grow, phase, p.staged != 0, want_bound,
                                        exclusions ? (LIST + LIST / 2 < kWarps * 32 ? LIST + LIST / 2 : kWarps * 32)
                                                   : LIST,
                                        m, o,
                                        [&](const char* src, const RowSplit& rs, float xthr) {
                                            if (xthr != f_ninf())
                                                collect_candidates<DT, kThreads / 2>(ws, src, rs, tid - kThreads / 2,
                                                                                     xthr, eligible);
                                        });
            if (o.aborted) break;
            bool invalid = o.invalid;
            if constexpr (!LOGITS) {
                if (o.xthr != f_ninf()) collect_candidates<DT, kThreads>(ws, o.src, o.rs, tid, o.xthr, eligible);
                if (!o.inv_known) {
                    bool bad = false;
                    for (int v = tid; v < V; v += kThreads) bad |= !(load_elem<DT>(o.src, v) < f_inf());
                    invalid = !block_and(!bad);
                }
            }
            block_sync();
            uint64_t* rec = p.rkeys + rowi * LIST;
            const int n = ws.n_cand;
            int cnt;
            if (o.xthr != f_ninf() && n <= kWideCand && (!exclusions || n >= LIST)) {
                cnt = sort_candidates(ws, n, LIST, rec);
            } else {
                auto gen = [&](int v) -> uint64_t {
                    const float x = load_elem<DT>(o.src, v);
                    return (x < f_inf() && x != f_ninf() && eligible(v)) ? make_key(x, static_cast<uint32_t>(v)) : 0;
                };
                int got = 0;
                if (!LOGITS || o.lse != f_ninf())
                    got = block_select(sh, gen, V, LIST, [&](int pos, uint64_t key) { ws.cand[pos] = key; });
                cnt = sort_candidates(ws, got, LIST, rec);
            }
            if (tid == 0) {
                p.rlse[rowi] = o.lse;
                p.rinfo[rowi] = (invalid ? 1u : 0u) | (static_cast<uint32_t>(cnt) << 8);
            }
        }
        chain_arrive_with<kThreads>(p, sh.sel, t, b, tid, 0,
                                    [&](int ct) { chain_select_wide<DT, LOGITS, KCAP>(p, sh, ws, ss, ct, b, m); });
        (void)warp;
    }
}

template <int KCAP>
constexpr size_t wide_dyn_smem() {
    return ((sizeof(SelectShared<KCAP>) + 127) & ~static_cast<size_t>(127)) + ((sizeof(WideShared) + 127) & ~static_cast<size_t>(127));
}

template <int DT, bool LOGITS, int KCAP>
static cudaError_t launch_chain_wide_as(const DecodeParams& p, cudaStream_t stream, int sm_count) {
    const size_t dyn = wide_dyn_smem<KCAP>() + (p.staged ? static_cast<size_t>(p.row_smem) : 0);
    auto kernel = decode_chain_wide_kernel<DT, LOGITS, KCAP>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, dyn);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const int64_t tickets = static_cast<int64_t>(p.B) * p.K * p.T;
    int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
    if (grid > tickets) grid = tickets;
    kernel<<<static_cast<unsigned>(grid), kThreads, dyn, stream>>>(p);
    return cudaGetLastError();
}

// Launch of one (dtype, logits) family: the beam size picks the register top-k width
// (1..16) or the generic radix-select path; decodes without n-gram blocking or
// repetition penalty and beams up to 16 run chained.
template <int DT, bool LOGITS>
static cudaError_t launch_decode_k(const DecodeParams& p, cudaStream_t stream, int sm_count) {
    const int K = p.K;
    if (p.chain && !LOGITS && !p.banned && K <= kFastBeam) {
        if (K <= 1) return launch_chain_warp_as<DT, 1>(p, stream, sm_count);
        if (K <= 2) return launch_chain_warp_as<DT, 2>(p, stream, sm_count);
        if (K <= 4) return launch_chain_warp_as<DT, 4>(p, stream, sm_count);
        if (K <= 8) return launch_chain_warp_as<DT, 8>(p, stream, sm_count);
        return launch_chain_warp_as<DT, 16>(p, stream, sm_count);
    }
    if (p.chain) {
        if (K <= 1) return launch_chain_as<DT, LOGITS, 1>(p, stream, sm_count);
        if (K <= 2) return launch_chain_as<DT, LOGITS, 2>(p, stream, sm_count);
        if (K <= 4) return launch_chain_as<DT, LOGITS, 4>(p, stream, sm_count);
        if (K <= 8) return launch_chain_as<DT, LOGITS, 8>(p, stream, sm_count);
        if (K <= 16) return launch_chain_as<DT, LOGITS, 16>(p, stream, sm_count);
        if (K <= 64) return launch_chain_wide_as<DT, LOGITS, 64>(p, stream, sm_count);
        if (K <= 256) return launch_chain_wide_as<DT, LOGITS, 256>(p, stream, sm_count);
        return launch_chain_wide_as<DT, LOGITS, kSelectCap>(p, stream, sm_count);
    }
    if (K <= 1) return launch_decode_as<DT, LOGITS, 1>(p, stream, sm_count);
    if (K <= 2) return launch_decode_as<DT, LOGITS, 2>(p, stream, sm_count);
    if (K <= 4) return launch_decode_as<DT, LOGITS, 4>(p, stream, sm_count);
    if (K <= 8) return launch_decode_as<DT, LOGITS, 8>(p, stream, sm_count);
    if (K <= 16) return launch_decode_as<DT, LOGITS, 16>(p, stream, sm_count);
    return launch_decode_as<DT, LOGITS, 0>(p, stream, sm_count);
}

}  // namespace
}  // namespace dbsb
