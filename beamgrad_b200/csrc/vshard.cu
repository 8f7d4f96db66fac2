// SPDX-License-Identifier: MIT
//
// Vocabulary-sharded decode: each row's vocabulary is split over W ranks (W = 1, 2, 4
// or 8), one GPU per rank. The reference's logsumexp sums lane j = v mod 256 of a row
// in increasing v and then reduces the 256 lanes in a fixed tree
// (src/kernels_scalar.cpp:48-66, src/kernels.hpp:197-202 of beamgrad 2.3.0), so the
// shards are lane-interleaved: rank r holds the tokens whose lane falls in
// [r * 256 / W, (r + 1) * 256 / W), and every lane sum is computed whole on one rank.
//
// A decode runs in stages, the collectives between them issued by the caller:
//   scan    every row of the shard: maximum and minimum of the entries below +inf,
//           the NaN/+inf flag, and the row record -- the shard's best entries by x
//           (ties: lower token first) under the record's eligibility (banned tokens,
//           EOS masked before min_length at parent length t), keyed by global token;
//   (caller) all-reduce MAX of the row maxima;
//   lanes   from logits: the shard's lane sums of exp(x - max) with the row maximum;
//   (caller) all-gather of the exchange rows (info, lane sums, record);
//   merge   every row: the 256 lanes in the reference's tree -> logsumexp, and the
//           shards' records -> one record. Each shard record holds the shard's best
//           entries, so the union holds every entry at or above the largest last entry
//           of the shards whose record is full; those entries, sorted, make the merged
//           record, and entries left out lie below its last one;
//   select  the chained selection of every example on every rank (replicated), from
//           the merged records; a row whose record is not enough for an exact
//           selection stops its example before the step (resume / stalled);
//   rescan  (only when an example stopped) each shard's best K candidates of the
//           stopped rows with the parent known; the caller all-gathers them and runs
//           select again, which takes the best K of the shards' lists for those rows.
// Every rank computes the same selections from the same gathered data.
#include "dbs_cuda_b200.h"
#include "decode_impl.cuh"

namespace dbsb {
namespace {

__device__ __forceinline__ int vs_global(const VShardParams& q, int i) {
    const int c = i >> q.lanes_log2;
    return c * kLanes + q.rank * q.lanes + (i - (c << q.lanes_log2));
}

// Shard entry of token v, or -1 when another rank holds it.
__device__ __forceinline__ int vs_local(const VShardParams& q, int v) {
    if (v < 0) return -1;
    const int j = v & (kLanes - 1);
    const int lo = q.rank * q.lanes;
    if (j < lo || j >= lo + q.lanes) return -1;
    return ((v >> 8) << q.lanes_log2) + (j - lo);
}

__device__ __forceinline__ void vs_row_coords(const DecodeParams& p, int64_t rowi, int& b, int& t, int& k) {
    k = static_cast<int>(rowi % p.K);
    const int64_t bt = rowi / p.K;
    t = static_cast<int>(bt % p.T);
    b = static_cast<int>(bt / p.T);
}

// Rows the search may read: active step, slot inside the beam, and only slot 0 at t = 0.
__device__ __forceinline__ bool vs_row_read(const Meta& m, int t, int k) {
    return t < m.steps && k < m.beam && (t > 0 || k == 0);
}

// A thread's four largest entries (values, shard indices), v[0] >= ... >= v[3].
__device__ __forceinline__ void top4_insert(float (&v)[4], int (&ix)[4], float x, int i) {
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

// Pass 1 over a row in global memory, eight 16-byte loads in flight per thread: the
// NaN-propagating maximum and the minimum of the entries the thread owns (chunk c on
// thread c mod kThreads, ragged ends on threads 0 .. n_ends - 1), and its four largest
// entries (NaN never enters; +inf may, and then the row takes the slow path), leaving out
// entry `skip` (a masked EOS token; -1: none).
template <int DT>
__device__ __forceinline__ void pass1_top4(const char* row, const RowSplit& rs, int tid, int skip, float& mxn,
                                           float& mn, float (&tv)[4], int (&ti)[4]) {
    using E = Elem<DT>;
    constexpr int UR = 8;
    constexpr int PER = 16 / E::kBytes;
    const char* body = row + static_cast<size_t>(rs.head) * E::kBytes;
    mxn = f_ninf();
    mn = f_inf();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        tv[u] = f_ninf();
        ti[u] = 0;
    }
    auto single = [&](int v) {
        const float x = load_elem<DT>(row, v);
        mxn = max_nan(mxn, x);
        mn = fminf(mn, x);
        if (v != skip) top4_insert(tv, ti, x, v);
    };
    if (tid < rs.head && tid < rs.n_ends()) single(rs.end_entry(tid));  // entries before the body
    if constexpr (E::kBytes == 2) {
        uint32_t mx2 = h2_ninf<DT>(), mn2 = h2_inf<DT>();
        for (int c0 = tid; c0 < rs.nvec; c0 += UR * kThreads) {
            uint4 q[UR];
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * kThreads;
                if (c < rs.nvec) q[u] = ld_stream_v4(body + static_cast<size_t>(c) * 16);
            }
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * kThreads;
                if (c < rs.nvec) {
                    mx2 = h2_max_nan<DT>(mx2, h2_max_nan<DT>(h2_max_nan<DT>(q[u].x, q[u].y), h2_max_nan<DT>(q[u].z, q[u].w)));
                    mn2 = h2_min<DT>(mn2, h2_min<DT>(h2_min<DT>(q[u].x, q[u].y), h2_min<DT>(q[u].z, q[u].w)));
                    const uint32_t m2 = h2_max<DT>(h2_max<DT>(q[u].x, q[u].y), h2_max<DT>(q[u].z, q[u].w));
                    if (fmaxf(h2_lo<DT>(m2), h2_hi<DT>(m2)) > tv[3]) {
                        float x[PER];
                        unpack16<DT>(q[u], x);
#pragma unroll
                        for (int e = 0; e < PER; ++e)
                            if (rs.head + c * PER + e != skip) top4_insert(tv, ti, x[e], rs.head + c * PER + e);
                    }
                }
            }
        }
        mxn = max_nan(mxn, max_nan(h2_lo<DT>(mx2), h2_hi<DT>(mx2)));
        mn = fminf(mn, fminf(h2_lo<DT>(mn2), h2_hi<DT>(mn2)));
    } else {
        for (int c0 = tid; c0 < rs.nvec; c0 += UR * kThreads) {
            uint4 q[UR];
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * kThreads;
                if (c < rs.nvec) q[u] = ld_stream_v4(body + static_cast<size_t>(c) * 16);
            }
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = c0 + u * kThreads;
                if (c < rs.nvec) {
                    const float a = __uint_as_float(q[u].x), b = __uint_as_float(q[u].y);
                    const float d = __uint_as_float(q[u].z), e = __uint_as_float(q[u].w);
                    mxn = max_nan(mxn, max_nan(max_nan(a, b), max_nan(d, e)));
                    mn = fminf(mn, fminf(fminf(a, b), fminf(d, e)));
                    if (fmaxf(fmaxf(a, b), fmaxf(d, e)) > tv[3]) {
                        const int base = rs.head + c * 4;
                        if (base != skip) top4_insert(tv, ti, a, base);
                        if (base + 1 != skip) top4_insert(tv, ti, b, base + 1);
                        if (base + 2 != skip) top4_insert(tv, ti, d, base + 2);
                        if (base + 3 != skip) top4_insert(tv, ti, e, base + 3);
                    }
                }
            }
        }
    }
    if (tid >= rs.head && tid < rs.n_ends()) single(rs.end_entry(tid));  // entries after the body
}

// ---------------------------------------------------------------------------
// scan: one CTA per row (grid-stride). Pass 1 streams the row once and keeps each
// thread's four largest entries; the bound B = the smallest of the warps' q-th largest
// thread maxima (8q >= LS) has at least LS eligible entries at or above it, so the
// record lies among the entries >= B. A thread whose fourth entry is below B holds all
// of its entries >= B among its four; the others (and a thread owning an EOS token)
// read their own entries again. Rows with NaN/+inf, banned tokens, or records above
// 256 entries take a block radix select over the row.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(kThreads, 3) vs_scan_kernel(const __grid_constant__ VShardParams q) {
    using E = Elem<DT>;
    constexpr int PER = 16 / E::kBytes;
    __shared__ RowShared sh;
    __shared__ WideShared ws;
    const DecodeParams& p = q.d;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int Vr = q.shard_v, LS = q.shard_list;
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * p.K;
    const bool exclusions = p.banned != nullptr;
    const bool want_bound = !exclusions && LS <= kWarps * 32;
    const int qw = (LS + kWarps - 1) / kWarps;  // thread maxima each warp contributes to the bound
    for (int64_t rowi = blockIdx.x; rowi < rows; rowi += gridDim.x) {
        int b, t, k;
        vs_row_coords(p, rowi, b, t, k);
        const Meta m = load_meta(p, b);
        uint64_t* out = q.pack + rowi * q.row_words;
        if (!vs_row_read(m, t, k) || Vr == 0) {
            if (tid == 0) {
                out[0] = 0;
                q.row_max[rowi] = f_ninf();
                q.row_min[rowi] = f_inf();
            }
            continue;
        }
        const char* row = static_cast<const char*>(q.shard) + rowi * static_cast<int64_t>(Vr) * E::kBytes;
        const RowSplit rs = RowSplit::of<E::kBytes>(row, Vr);
        const bool mask_eos = m.eos >= 0 && t + 1 < m.min_length;
        auto eligible = [&](int i) {
            const int v = vs_global(q, i);
            return !(exclusions && p.banned[v]) && !(mask_eos && is_eos(p, m, v));
        };
        auto push = [&](bool cond, float x, int i) {
            const unsigned mask = __ballot_sync(0xffffffffu, cond);
            if (!mask) return;
            int base = 0;
            if (lane == 0) base = atomicAdd(&ws.n_cand, __popc(mask));
            base = __shfl_sync(0xffffffffu, base, 0);
            const int pos = base + __popc(mask & ((1u << lane) - 1u));
            if (cond && pos < kWideCand) ws.cand[pos] = make_key(x, static_cast<uint32_t>(vs_global(q, i)));
        };
        // EOS tokens of this thread: their entries never count toward the bound; a masked one
        // is left out of the four, and a thread owning two masked ones reads its entries again.
        bool dirty = false;
        int skip = -1, n_masked = 0;
        if (m.eos >= 0) {
            auto own = [&](int v) {
                const int i = vs_local(q, v);
                if (!rs.owns(i)) return;
                dirty = true;
                if (mask_eos && i != skip) {
                    skip = i;
                    ++n_masked;
                }
            };
            own(m.eos);
            for (int i = 0; i < p.n_extra; ++i) own(p.extra[i]);
        }
        float mxn, mn;
        float tv[4];
        int ti[4];
        pass1_top4<DT>(row, rs, tid, skip, mxn, mn, tv, ti);
        const bool bad = !(mxn < f_inf());
        {
            const float srt = warp_sort_desc((bad || dirty) ? f_ninf() : mxn);
            if (lane == qw - 1) sh.wtop[warp] = srt;
            const float wmx = warp_max_f32(bad ? f_ninf() : mxn);
            const float wmn = -warp_max_f32(-mn);
            const unsigned wbad = __ballot_sync(0xffffffffu, bad);
            if (lane == 0) {
                sh.wred[warp] = wmx;
                sh.wred2[warp] = wmn;
                sh.ired[warp] = wbad != 0;
            }
        }
        if (tid == 0) ws.n_cand = 0;
        block_sync();
        float mx = sh.wred[0];
        mn = sh.wred2[0];
        bool any_bad = sh.ired[0] != 0;
        float bound = sh.wtop[0];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
            mx = fmaxf(mx, sh.wred[w]);
            mn = fminf(mn, sh.wred2[w]);
            any_bad |= sh.ired[w] != 0;
            bound = fminf(bound, sh.wtop[w]);
        }
        if (any_bad) {
            // Rare: the maximum over entries below +inf (NaN never raises fmaxf).
            block_sync();
            mx = f_ninf();
            for_chunks<DT>(row, rs, false, [&](float x, int) {
                if (x < f_inf()) mx = fmaxf(mx, x);
            });
            mx = block_max(sh, mx);
        }
        uint64_t* keys = out + q.key_off;
        int cnt = -1;
        if (want_bound && !any_bad && bound != f_ninf()) {
            const bool reread = n_masked > 1 || tv[3] >= bound;
#pragma unroll
            for (int u = 0; u < 4; ++u) push(!reread && tv[u] >= bound, tv[u], ti[u]);
            // Threads that may own more entries >= bound than they kept: their whole share,
            // read by their warp (lane r takes the thread's chunks r, r + 32, ...).
            unsigned todo = __ballot_sync(0xffffffffu, reread);
            while (todo) {
                const int src = __ffs(todo) - 1;
                todo &= todo - 1;
                const int owner = warp * 32 + src;
                if (owner < rs.n_ends()) {
                    const int i = rs.end_entry(owner);
                    const float x = lane == 0 ? load_elem<DT>(row, i) : f_ninf();
                    push(lane == 0 && x >= bound && x < f_inf() && eligible(i), x, i);
                }
                const int nch = owner < rs.nvec ? (rs.nvec - owner + kThreads - 1) / kThreads : 0;
                for (int r0 = 0; r0 < nch; r0 += 32) {
                    const int c = owner + (r0 + lane) * kThreads;
                    const bool have = r0 + lane < nch;
                    float x[PER];
                    if (have) unpack16<DT>(ld_stream_v4(row + static_cast<size_t>(rs.head) * E::kBytes +
                                                        static_cast<size_t>(c) * 16), x);
#pragma unroll
                    for (int e = 0; e < PER; ++e) {
                        const int i = rs.head + c * PER + e;
                        push(have && x[e] >= bound && x[e] < f_inf() && eligible(i), x[e], i);
                    }
                }
            }
            block_sync();
            const int n = ws.n_cand;
            if (n <= kWideCand) cnt = sort_candidates(ws, n, LS, keys);
        }
        if (cnt < 0) {
            block_sync();
            auto gen = [&](int i) -> uint64_t {
                const float x = load_elem<DT>(row, i);
                return (x < f_inf() && x != f_ninf() && eligible(i)) ? make_key(x, static_cast<uint32_t>(vs_global(q, i)))
                                                                    : 0;
            };
            const int got = block_select(sh, gen, Vr, LS, [&](int pos, uint64_t key) { ws.cand[pos] = key; });
            cnt = sort_candidates(ws, got, LS, keys);
        }
        if (tid == 0) {
            // Bit 1: the record is full, so the shard may hold more eligible entries.
            out[0] = (any_bad ? 1u : 0u) | (cnt >= LS ? 2u : 0u) | (static_cast<uint64_t>(cnt) << 8);
            q.row_max[rowi] = mx;
            q.row_min[rowi] = mn;
        }
        block_sync();
    }
}

// ---------------------------------------------------------------------------
// lanes: lanes / 2 threads per row, thread j summing lanes 2j and 2j + 1 of the shard.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(kThreads) vs_lanes_kernel(const __grid_constant__ VShardParams q) {
    using E = Elem<DT>;
    constexpr int EB = E::kBytes;
    const DecodeParams& p = q.d;
    const int L = q.lanes;
    const int tpr = L / 2;
    const int rpc = kThreads / tpr;
    const int g = threadIdx.x / tpr;
    const int j = threadIdx.x - g * tpr;
    const int Vr = q.shard_v;
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * p.K;
    const int nfull = p.V / kLanes;
    int tail = p.V - nfull * kLanes - q.rank * L;  // shard entries in the partial last block
    tail = tail < 0 ? 0 : (tail > L ? L : tail);
    const Pack2 pk{p.one2, p.nzero2};
    const int a = 2 * j, c = 2 * j + 1;
    for (int64_t rowi = static_cast<int64_t>(blockIdx.x) * rpc + g; rowi < rows;
         rowi += static_cast<int64_t>(gridDim.x) * rpc) {
        int b, t, k;
        vs_row_coords(p, rowi, b, t, k);
        const Meta m = load_meta(p, b);
        if (!vs_row_read(m, t, k)) continue;
        float* lanes_out = reinterpret_cast<float*>(q.pack + rowi * q.row_words + 1);
        const float mx = q.row_max[rowi];
        float acc_a = 0.0f, acc_c = 0.0f;
        if (mx != f_ninf() && Vr > 0) {
            const char* row = static_cast<const char*>(q.shard) + rowi * static_cast<int64_t>(Vr) * EB;
            const auto* er = reinterpret_cast<const typename E::T*>(row);
            const bool invalid = (q.pack[rowi * q.row_words] & 1u) != 0;
            if (!invalid) {
                const bool fast = __fsub_rn(q.row_min[rowi], mx) >= cephes::kMin;  // every x - max >= -87
                const bool paired = (reinterpret_cast<uintptr_t>(row) & (2 * EB - 1)) == 0;
                if (paired) {
                    const uint64_t acc = fast ? lane_pair_sums<DT, false, 8>(pk, row, nfull, mx, j, L)
                                              : lane_pair_sums<DT, true, 8>(pk, row, nfull, mx, j, L);
                    f2_unpack(acc, acc_a, acc_c);
                } else {
                    for (int i = 0; i < nfull; ++i) {
                        acc_a = __fadd_rn(acc_a, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[i * L + a]), mx)));
                        acc_c = __fadd_rn(acc_c, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[i * L + c]), mx)));
                    }
                }
                if (a < tail) acc_a = __fadd_rn(acc_a, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[nfull * L + a]), mx)));
                if (c < tail) acc_c = __fadd_rn(acc_c, exp_nonpositive_masked(__fsub_rn(E::to_f32(er[nfull * L + c]), mx)));
            } else {
                const int na = nfull + (a < tail ? 1 : 0), nc = nfull + (c < tail ? 1 : 0);
                for (int i = 0; i < na; ++i) {
                    const float x = E::to_f32(er[i * L + a]);
                    if (x < f_inf() && x != f_ninf()) acc_a = __fadd_rn(acc_a, exp_nonpositive(__fsub_rn(x, mx)));
                }
                for (int i = 0; i < nc; ++i) {
                    const float x = E::to_f32(er[i * L + c]);
                    if (x < f_inf() && x != f_ninf()) acc_c = __fadd_rn(acc_c, exp_nonpositive(__fsub_rn(x, mx)));
                }
            }
        }
        lanes_out[a] = acc_a;
        lanes_out[c] = acc_c;
    }
}

// ---------------------------------------------------------------------------
// merge: one warp per four rows. The logsumexp of each row takes the whole warp; the
// records are merged by a tournament in eight-lane groups (group g: row g, lane r of
// the group: the head of shard r's record).
// ---------------------------------------------------------------------------
constexpr int kMergeRows = 4;

__device__ __forceinline__ uint64_t group8_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) {
        const uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

template <bool LOGITS>
__global__ void __launch_bounds__(kThreads) vs_merge_kernel(const __grid_constant__ VShardParams q) {
    const DecodeParams& p = q.d;
    const int lane = threadIdx.x & 31;
    const int W = q.world, LIST = p.list_len;
    const int64_t rows = static_cast<int64_t>(p.B) * p.T * p.K;
    const int g = lane >> 3, li = lane & 7;
    const unsigned gmask = 0xffu << (8 * g);
    const int64_t step = static_cast<int64_t>(gridDim.x) * kWarps * kMergeRows;
    for (int64_t row0 = (static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5)) * kMergeRows; row0 < rows;
         row0 += step) {
        auto part = [&](int r, int64_t rowi) {
            return q.pack_all + (static_cast<int64_t>(r) * rows + rowi) * q.row_words;
        };
        auto row_read = [&](int64_t rowi) {
            if (rowi >= rows) return false;
            int b, t, k;
            vs_row_coords(p, rowi, b, t, k);
            return vs_row_read(load_meta(p, b), t, k);
        };
        if constexpr (LOGITS) {
#pragma unroll 1
            for (int j = 0; j < kMergeRows; ++j) {
                const int64_t rowi = row0 + j;
                if (!row_read(rowi)) continue;
                const float mx = q.row_max[rowi];
                float lse = f_ninf();
                if (mx != f_ninf()) {
                    // Lane i = lane + 32u; the tree lanes[i] += lanes[i + s], s = 128 ... 1
                    // (src/kernels.hpp:197-202), the first three levels in registers.
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int jg = lane + 32 * u;
                        const int r = jg >> q.lanes_log2;
                        v[u] = reinterpret_cast<const float*>(part(r, rowi) + 1)[jg - (r << q.lanes_log2)];
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) v[u] = __fadd_rn(v[u], v[u + 4]);
#pragma unroll
                    for (int u = 0; u < 2; ++u) v[u] = __fadd_rn(v[u], v[u + 2]);
                    float x = __fadd_rn(v[0], v[1]);
#pragma unroll
                    for (int st = 16; st >= 1; st >>= 1) {
                        const float y = __shfl_down_sync(0xffffffffu, x, st);
                        if (lane < st) x = __fadd_rn(x, y);
                    }
                    lse = logsumexp_from(mx, __shfl_sync(0xffffffffu, x, 0));
                }
                if (lane == 0) p.rlse[rowi] = lse;
            }
        }
        const int64_t rowi = row0 + g;
        const bool read = row_read(rowi);
        // Shard li's record of row g: count, NaN/+inf flag, full (entries may be missing).
        const uint64_t* mine = nullptr;
        uint32_t info = 0;
        if (read && li < W) {
            mine = part(li, rowi);
            info = static_cast<uint32_t>(mine[0]);
            mine += q.key_off;
        }
        const int cnt = static_cast<int>(info >> 8);
        const bool full = (info & 2u) != 0;
        // Every entry at or above the largest last entry of a full record is in the union.
        const uint64_t bound = group8_max_u64((full && cnt > 0) ? mine[cnt - 1] : 0);
        const unsigned flags = __ballot_sync(0xffffffffu, (info & 1u) != 0) & gmask;
        const unsigned fulls = __ballot_sync(0xffffffffu, full) & gmask;
        uint64_t head = cnt > 0 ? mine[0] : 0;
        uint64_t next = cnt > 1 ? mine[1] : 0;
        if (head < bound) head = 0;
        int pos = 0;
        uint64_t* rec = read ? p.rkeys + rowi * LIST : nullptr;
        uint64_t held = 0;  // entry n of the record with n mod 8 == li, stored eight at a time
        int n = 0;
        for (; n < LIST; ++n) {
            const uint64_t best = group8_max_u64(head);
            if (!__any_sync(0xffffffffu, best != 0)) break;
            if (best != 0) {
                if ((n & 7) == li) held = best;
                if ((n & 7) == 7) rec[n - 7 + li] = held;
                if (head == best) {
                    ++pos;
                    head = next < bound ? 0 : next;
                    next = pos + 1 < cnt ? mine[pos + 1] : 0;
                }
            }
        }
        // The group's count: every entry it emitted advanced one of its lanes.
        int taken = pos;
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) taken += __shfl_xor_sync(0xffffffffu, taken, o);
        if (read) {
            const int c = taken < LIST ? taken : LIST;
            if (li < (c & 7)) rec[(c & ~7) + li] = held;
            if (li == 0) {
                p.rinfo[rowi] = (flags ? 1u : 0u) | (fulls ? 2u : 0u) | (static_cast<uint32_t>(c) << 8);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// select: one CTA per example, steps resume[b] .. T - 1.
// ---------------------------------------------------------------------------
template <bool LOGITS, int KCAP>
__global__ void __launch_bounds__(kThreads, 1) vs_select_kernel(const __grid_constant__ VShardParams q) {
    __shared__ RowShared sh;
    extern __shared__ __align__(128) unsigned char dyn[];
    auto& ss = *reinterpret_cast<SelectShared<KCAP>*>(dyn);
    constexpr size_t kSelBytes = (sizeof(SelectShared<KCAP>) + 127) & ~static_cast<size_t>(127);
    auto& ws = *reinterpret_cast<WideShared*>(dyn + kSelBytes);
    uint64_t* cbuf = reinterpret_cast<uint64_t*>(dyn + wide_dyn_smem<KCAP>());
    const DecodeParams& p = q.d;
    const int b = blockIdx.x;
    const int T = p.T, K = p.K, LIST = p.list_len;
    const int kw = (K + 31) / 32;
    const Meta m = load_meta(p, b);
    const int t0 = q.resume[b];
    if (t0 >= T) return;
    for (int t = t0; t < T; ++t) {
        const bool ok = chain_select_wide_with<LOGITS, KCAP>(p, sh, ws, ss, t, b, m, [&]() -> bool {
            // Rescanned lists exist for the step the example stopped at, one per marked row.
            bool mine = true;
            for (int kk = threadIdx.x; kk < K; kk += kThreads)
                if ((ws.fb[kk >> 5] >> (kk & 31)) & 1u)
                    mine &= t == t0 && q.n_rescan > 0 && q.rescan_slot[static_cast<int64_t>(b) * K + kk] >= 0;
            if (!__syncthreads_and(mine)) {
                for (int i = threadIdx.x; i < kw; i += kThreads) q.stalled[static_cast<int64_t>(b) * kw + i] = ws.fb[i];
                return false;
            }
            for (int w = 0; w < kw; ++w) {
                unsigned bits = ws.fb[w];
                while (bits) {
                    const int kk = w * 32 + __ffs(bits) - 1;
                    bits &= bits - 1;
                    const int slot = q.rescan_slot[static_cast<int64_t>(b) * K + kk];
                    uint64_t* list = p.keys + (static_cast<int64_t>(b) * K + kk) * LIST;
                    // The best K of the shards' lists (each its shard's best K).
                    auto gen = [&](int i) -> uint64_t {
                        const int r = i / K;
                        return ld_cg(q.rescan_all + (static_cast<int64_t>(r) * q.n_rescan + slot) * K + (i - r * K));
                    };
                    const int got = block_select(sh, gen, q.world * K, K, [&](int pos, uint64_t key) { list[pos] = key; });
                    for (int i = got + static_cast<int>(threadIdx.x); i < LIST; i += kThreads) list[i] = 0;
                    block_sync();
                }
            }
            return true;
        }, q.cand_cap > 0 ? cbuf : nullptr, q.cand_cap);
        if (!ok) {
            if (threadIdx.x == 0) q.resume[b] = t;
            return;
        }
    }
    if (threadIdx.x == 0) q.resume[b] = T;
}

// ---------------------------------------------------------------------------
// rescan: one CTA per stopped row; the shard's best K full keys with the parent known.
// ---------------------------------------------------------------------------
template <int DT, bool LOGITS>
__global__ void __launch_bounds__(kThreads) vs_rescan_kernel(const __grid_constant__ VShardParams q) {
    __shared__ RowShared sh;
    const DecodeParams& p = q.d;
    const int K = p.K, T = p.T, Vr = q.shard_v;
    for (int slot = blockIdx.x; slot < q.n_rescan; slot += gridDim.x) {
        const int bk = q.rescan_rows[slot];
        const int b = bk / K, k = bk - b * K;
        const int t = q.resume[b];
        uint64_t* list = q.rescan + static_cast<int64_t>(slot) * K;
        int cnt = 0;
        if (t >= 0 && t < T && Vr > 0) {
            const Meta m = load_meta(p, b);
            const int64_t s = static_cast<int64_t>(b) * K + k;
            const int64_t rowi = (static_cast<int64_t>(b) * T + t) * K + k;
            const char* row = static_cast<const char*>(q.shard) + rowi * static_cast<int64_t>(Vr) * Elem<DT>::kBytes;
            const float pr = ld_cg(p.raw + s);
            const bool mask_eos = m.eos >= 0 && ld_cg(p.len + s) + 1 < m.min_length;
            const float lse = LOGITS ? ld_cg(p.rlse + rowi) : 0.0f;
            const ConsView cv = chain_prefix(p, t, s);
            const uint32_t base = static_cast<uint32_t>(k) * static_cast<uint32_t>(p.V);
            auto gen = [&](int i) -> uint64_t {
                const float x = load_elem<DT>(row, i);
                if (!(x < f_inf()) || x == f_ninf()) return 0;
                const int v = vs_global(q, i);
                if (p.banned && p.banned[v]) return 0;
                if (mask_eos && is_eos(p, m, v)) return 0;
                const float raw = constrained_raw<LOGITS>(p, cv, pr, x, lse, v);
                return raw == f_ninf() ? 0 : make_key(raw, base + static_cast<uint32_t>(v));
            };
            if (!LOGITS || lse != f_ninf())
                cnt = block_select(sh, gen, Vr, K, [&](int pos, uint64_t key) { list[pos] = key; });
        }
        for (int i = cnt + static_cast<int>(threadIdx.x); i < K; i += kThreads) list[i] = 0;
        block_sync();
    }
}

template <class Kernel>
int64_t resident_grid(Kernel kernel, size_t dyn, int sm_count, int64_t work) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, dyn) != cudaSuccess) {
        cudaGetLastError();
        per_sm = 1;
    }
    if (per_sm < 1) per_sm = 1;
    int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
    if (grid > work) grid = work;
    return grid < 1 ? 1 : grid;
}

template <int DT>
cudaError_t scan_as(const VShardParams& q, cudaStream_t stream, int sm_count) {
    const int64_t rows = static_cast<int64_t>(q.d.B) * q.d.T * q.d.K;
    const int64_t grid = resident_grid(vs_scan_kernel<DT>, 0, sm_count, rows);
    vs_scan_kernel<DT><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(q);
    return cudaGetLastError();
}

template <int DT>
cudaError_t lanes_as(const VShardParams& q, cudaStream_t stream, int sm_count) {
    const int64_t rows = static_cast<int64_t>(q.d.B) * q.d.T * q.d.K;
    const int rpc = kThreads / (q.lanes / 2);
    const int64_t grid = resident_grid(vs_lanes_kernel<DT>, 0, sm_count, (rows + rpc - 1) / rpc);
    vs_lanes_kernel<DT><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(q);
    return cudaGetLastError();
}

template <int DT, bool LOGITS>
cudaError_t rescan_as(const VShardParams& q, cudaStream_t stream, int sm_count) {
    const int64_t grid = resident_grid(vs_rescan_kernel<DT, LOGITS>, 0, sm_count, q.n_rescan);
    vs_rescan_kernel<DT, LOGITS><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(q);
    return cudaGetLastError();
}

// Candidate keys of one step held in the select kernel's shared memory (128 KB).
constexpr int kSelectCandCap = 16384;

template <bool LOGITS, int KCAP>
cudaError_t select_as(const VShardParams& q0, cudaStream_t stream) {
    VShardParams q = q0;
    const int64_t all = static_cast<int64_t>(q.d.K) * q.d.list_len;
    q.cand_cap = all <= kSelectCandCap ? static_cast<int>(all) : 0;
    const size_t dyn = wide_dyn_smem<KCAP>() + static_cast<size_t>(q.cand_cap) * sizeof(uint64_t);
    auto kernel = vs_select_kernel<LOGITS, KCAP>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
    if (e != cudaSuccess) return e;
    kernel<<<static_cast<unsigned>(q.d.B), kThreads, dyn, stream>>>(q);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_vshard_scan(const VShardParams& q, int dtype, cudaStream_t stream, int sm_count) {
    switch (dtype) {
        case DBS_CUDA_DTYPE_F16: return scan_as<1>(q, stream, sm_count);
        case DBS_CUDA_DTYPE_BF16: return scan_as<2>(q, stream, sm_count);
        default: return scan_as<0>(q, stream, sm_count);
    }
}

cudaError_t launch_vshard_lanes(const VShardParams& q, int dtype, cudaStream_t stream, int sm_count) {
    switch (dtype) {
        case DBS_CUDA_DTYPE_F16: return lanes_as<1>(q, stream, sm_count);
        case DBS_CUDA_DTYPE_BF16: return lanes_as<2>(q, stream, sm_count);
        default: return lanes_as<0>(q, stream, sm_count);
    }
}

cudaError_t launch_vshard_merge(const VShardParams& q, bool logits, cudaStream_t stream, int sm_count) {
    const int64_t rows = static_cast<int64_t>(q.d.B) * q.d.T * q.d.K;
    const int64_t work = (rows + kWarps - 1) / kWarps;
    if (logits) {
        const int64_t grid = resident_grid(vs_merge_kernel<true>, 0, sm_count, work);
        vs_merge_kernel<true><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(q);
    } else {
        const int64_t grid = resident_grid(vs_merge_kernel<false>, 0, sm_count, work);
        vs_merge_kernel<false><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(q);
    }
    return cudaGetLastError();
}

cudaError_t launch_vshard_select(const VShardParams& q, bool logits, cudaStream_t stream) {
    const int K = q.d.K;
    if (logits) {
        if (K <= 64) return select_as<true, 64>(q, stream);
        if (K <= 256) return select_as<true, 256>(q, stream);
        return select_as<true, kSelectCap>(q, stream);
    }
    if (K <= 64) return select_as<false, 64>(q, stream);
    if (K <= 256) return select_as<false, 256>(q, stream);
    return select_as<false, kSelectCap>(q, stream);
}

cudaError_t launch_vshard_rescan(const VShardParams& q, int dtype, bool logits, cudaStream_t stream, int sm_count) {
    if (q.n_rescan <= 0) return cudaSuccess;
    switch (dtype) {
        case DBS_CUDA_DTYPE_F16: return logits ? rescan_as<1, true>(q, stream, sm_count) : rescan_as<1, false>(q, stream, sm_count);
        case DBS_CUDA_DTYPE_BF16: return logits ? rescan_as<2, true>(q, stream, sm_count) : rescan_as<2, false>(q, stream, sm_count);
        default: return logits ? rescan_as<0, true>(q, stream, sm_count) : rescan_as<0, false>(q, stream, sm_count);
    }
}

}  // namespace dbsb
