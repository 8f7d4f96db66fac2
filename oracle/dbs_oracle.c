/* SPDX-License-Identifier: MIT
 *
 * dbs_oracle.c -- TEST INFRASTRUCTURE ONLY (see dbs_oracle.h): the CPU
 * restatement of beamgrad's reference decoder that the CUDA engine is checked
 * against. Compiled with -ffp-contract=off (oracle/Makefile): every float
 * operation below is one IEEE-754 round-to-nearest operation, in the order the
 * reference performs it, which is what makes the results bit-comparable.
 *
 * Citations are to beamgrad 2.3.0 paths.
 */
#include "dbs_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define NEG_INF (-INFINITY)
#define LANES 256 /* src/logits.hpp:27 kLogitLanes */

/* ------------------------------------------------------------------------- */
/* Deterministic math                                                         */
/* ------------------------------------------------------------------------- */

/* ln(x) for x >= 1 from basic double operations and exact frexp
 * (src/penalty.hpp:78-106): x = m 2^e, m in [sqrt(1/2), sqrt(2)),
 * ln m = 2 atanh(s), s = (m - 1)/(m + 1), atanh by its odd series to s^23. */
static double log_ge1(double x) {
    int e = 0;
    double m = frexp(x, &e);
    if (m < 0.70710678118654752440) {
        m = m * 2.0;
        e -= 1;
    }
    const double s = (m - 1.0) / (m + 1.0);
    const double s2 = s * s;
    static const double inv_odd[12] = {1.0 / 23.0, 1.0 / 21.0, 1.0 / 19.0, 1.0 / 17.0, 1.0 / 15.0, 1.0 / 13.0,
                                       1.0 / 11.0, 1.0 / 9.0,  1.0 / 7.0,  1.0 / 5.0,  1.0 / 3.0,  1.0};
    double p = inv_odd[0];
    for (int i = 1; i < 12; ++i) p = p * s2 + inv_odd[i];
    const double log_m = (2.0 * s) * p;
    const double hi = 6.93147180369123816490e-01; /* ln 2, split so e * hi is exact */
    const double lo = 1.90821492927058770002e-10;
    const double de = (double)e;
    return de * hi + (de * lo + log_m);
}

/* exp(y) for y >= 0 (src/penalty.hpp:110-135): y = k ln2 + r, Taylor series of
 * exp(r) to r^15, scaled by ldexp. */
static double exp_ge0(double y) {
    if (y > 709.0) return HUGE_VAL;
    const double inv_ln2 = 1.44269504088896338700e+00;
    const double hi = 6.93147180369123816490e-01;
    const double lo = 1.90821492927058770002e-10;
    const int k = (int)(y * inv_ln2 + 0.5);
    const double dk = (double)k;
    const double r = (y - dk * hi) - dk * lo;
    /* 1/15!, 1/14!, ..., 1/2!, 1, 1 */
    static const double c[16] = {1.0 / 1307674368000.0, 1.0 / 87178291200.0, 1.0 / 6227020800.0,
                                 1.0 / 479001600.0,     1.0 / 39916800.0,    1.0 / 3628800.0,
                                 1.0 / 362880.0,        1.0 / 40320.0,       1.0 / 5040.0,
                                 1.0 / 720.0,           1.0 / 120.0,         1.0 / 24.0,
                                 1.0 / 6.0,             0.5,                 1.0,
                                 1.0};
    double p = c[0];
    for (int i = 1; i < 16; ++i) p = p * r + c[i];
    return ldexp(p, k);
}

/* GNMT length penalty ((5 + max(l, 1)) / 6)^alpha (src/penalty.hpp:139-160):
 * integer alpha <= 64 by repeated squaring, otherwise exp(alpha ln base). */
float oracle_gnmt_penalty(int length, float alpha) {
    if (alpha == 0.0f) return 1.0f;
    const int l = length > 1 ? length : 1;
    const double base = (5.0 + (double)l) / 6.0;
    if (alpha <= 64.0f && alpha == (float)(int)alpha) {
        int n = (int)alpha;
        double result = 1.0;
        double b = base;
        while (n > 0) {
            if (n & 1) result = result * b;
            b = b * b;
            n >>= 1;
        }
        return (float)result;
    }
    const double y = (double)alpha * log_ge1(base);
    return (float)exp_ge0(y);
}

static float as_float(uint32_t u) {
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* exp(x) for x <= 0 (src/logits.hpp:204-235): the Cephes expf range reduction
 * and degree-5 polynomial (Cephes constants, as the reference uses them),
 * 0 below -87 and for -inf/NaN. */
float oracle_exp_nonpositive(float x) {
    if (!(x >= -87.0f)) return 0.0f;
    const float k = floorf(x * 1.44269504088896341f + 0.5f);
    const float r = (x - k * 0.693359375f) - k * -2.12194440e-4f;
    const float r2 = r * r;
    float p = 1.9875691500e-4f;
    p = p * r + 1.3981999507e-3f;
    p = p * r + 8.3334519073e-3f;
    p = p * r + 4.1665795894e-2f;
    p = p * r + 1.6666665459e-1f;
    p = p * r + 5.0000001201e-1f;
    p = (p * r2 + r) + 1.0f;
    const int e = (int)k + 127;
    return p * as_float((uint32_t)e << 23);
}

/* Exact fp16 / bf16 widening (src/half.hpp:16-29). */
float oracle_half_to_float(uint16_t h, int data_type) {
    if (data_type == DBS_CUDA_DTYPE_BF16) return as_float((uint32_t)h << 16);
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu;
    const uint32_t mant = h & 0x03ffu;
    if (ex == 0) {
        const float mag = (float)mant * 5.9604644775390625e-8f; /* mant * 2^-24, exact */
        return sign ? -mag : mag;
    }
    const uint32_t out = ex == 31 ? (sign | 0x7f800000u | (mant << 13)) : (sign | ((ex + 112u) << 23) | (mant << 13));
    return as_float(out);
}

static int elem_size(int data_type) { return data_type == DBS_CUDA_DTYPE_F32 ? 4 : 2; }

static void load_row(const void* base, int data_type, int64_t row, int V, float* out) {
    if (data_type == DBS_CUDA_DTYPE_F32) {
        memcpy(out, (const float*)base + row * V, (size_t)V * sizeof(float));
        return;
    }
    const uint16_t* p = (const uint16_t*)base + row * V;
    for (int v = 0; v < V; ++v) out[v] = oracle_half_to_float(p[v], data_type);
}

/* Row logsumexp (src/kernels_scalar.cpp:48-66 logit_stats_scalar, combined by
 * src/kernels.hpp:197-202 and src/logits.hpp:241-243): maximum over entries
 * below +inf; lane j sums exp(x - max) over finite x with v = j (mod 256) in
 * increasing v; lanes combined by the pairwise tree of strides 128..1;
 * lse = max + (float)log_ge1(sum). -inf when no entry is finite. */
float oracle_row_lse(const float* row, int V, int* invalid) {
    float mx = NEG_INF;
    for (int v = 0; v < V; ++v) {
        const float x = row[v];
        if (!(x < INFINITY)) *invalid = 1;
        else if (x > mx) mx = x;
    }
    if (mx == NEG_INF) return NEG_INF;
    float lanes[LANES];
    for (int j = 0; j < LANES; ++j) lanes[j] = 0.0f;
    for (int v = 0; v < V; ++v) {
        const float x = row[v];
        if (x < INFINITY && x != NEG_INF) lanes[v & (LANES - 1)] = lanes[v & (LANES - 1)] + oracle_exp_nonpositive(x - mx);
    }
    for (int s = LANES / 2; s > 0; s >>= 1)
        for (int j = 0; j < s; ++j) lanes[j] = lanes[j] + lanes[j + s];
    return mx + (float)log_ge1((double)lanes[0]);
}

/* The row lse split by lane (a vocabulary shard's view of oracle_row_lse): rank
 * `rank` of `world` holds the tokens v with (v mod 256) in [rank * L, rank * L + L),
 * L = 256 / world, shard entry i being token (i / L) * 256 + rank * L + i mod L.
 * lanes_out[l] = the reference's lane rank * L + l of the full row, given the full
 * row's maximum mx (src/kernels_scalar.cpp:48-66). */
void oracle_shard_lanes(const float* shard_row, int shard_vocab, int world, float mx, float* lanes_out) {
    const int L = LANES / world;
    for (int l = 0; l < L; ++l) lanes_out[l] = 0.0f;
    if (mx == NEG_INF) return;
    for (int i = 0; i < shard_vocab; ++i) {
        const float x = shard_row[i];
        if (x < INFINITY && x != NEG_INF) lanes_out[i % L] = lanes_out[i % L] + oracle_exp_nonpositive(x - mx);
    }
}

/* lse from the 256 lane sums (src/kernels.hpp:197-202, src/logits.hpp:241-243). */
float oracle_lse_from_lanes(const float* lanes256, float mx) {
    if (mx == NEG_INF) return NEG_INF;
    float lanes[LANES];
    for (int j = 0; j < LANES; ++j) lanes[j] = lanes256[j];
    for (int s = LANES / 2; s > 0; s >>= 1)
        for (int j = 0; j < s; ++j) lanes[j] = lanes[j] + lanes[j + s];
    return mx + (float)log_ge1((double)lanes[0]);
}

static float softmax_probability(float x, float lse) {
    const int finite = x < INFINITY && x > NEG_INF;
    return finite ? oracle_exp_nonpositive(x - lse) : 0.0f;
}

/* ------------------------------------------------------------------------- */
/* Candidates and their total order (src/common.hpp:253-302)                  */
/* ------------------------------------------------------------------------- */

typedef struct {
    float score;
    float raw;
    int32_t parent;
    int32_t token;
    int32_t length;
    uint8_t from_logprob;
} Cand;

static int better(const Cand* a, const Cand* b) {
    if (a->score != b->score) return a->score > b->score;
    if (a->raw != b->raw) return a->raw > b->raw;
    if (a->parent != b->parent) return a->parent < b->parent;
    if (a->token != b->token) return a->token < b->token;
    if (a->length != b->length) return a->length < b->length;
    return a->from_logprob > b->from_logprob;
}

/* Descending top-n buffer with binary insertion (src/common.hpp:278-302). */
static void insert_top(Cand* top, int n, const Cand* c) {
    if (!better(c, &top[n - 1])) return;
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = lo + ((hi - lo) >> 1);
        if (better(c, &top[mid])) hi = mid;
        else lo = mid + 1;
    }
    for (int i = n - 1; i > lo; --i) top[i] = top[i - 1];
    top[lo] = *c;
}

/* ------------------------------------------------------------------------- */
/* One example's search (src/decoder.cpp:27-360, class BeamSearch)            */
/* ------------------------------------------------------------------------- */

typedef struct {
    int K;          /* the example's beam size */
    int stride;     /* beam stride of the tensors (args->beam_size) */
    int V;
    int eos;
    int min_length;
    float alpha;
    int ngram;
    int penalise;
    float log_penalty;
    const uint8_t* banned;
    int n_eos;
    int32_t eos_set[1 + DBS_CUDA_MAX_EXTRA_EOS]; /* sorted, distinct */
    int constrained;
    /* state */
    float* raw;
    int32_t* len;
    uint8_t* ended;
    int32_t* last;      /* token of each slot after the previous step */
    int32_t* prefix;    /* [K, cap] */
    int32_t* prefix_len;
    int cap;
    /* scratch */
    Cand* top;
    float* row;
    uint8_t* mask;      /* [V]: 1 banned, 2 n-gram, 4 penalised */
    int invalid;
} Search;

static int is_eos(const Search* s, int token) {
    for (int i = 0; i < s->n_eos; ++i)
        if (s->eos_set[i] == token) return 1;
    return 0;
}

static int min_masked(const Search* s, int v, int new_length) {
    return new_length < s->min_length && is_eos(s, v);
}

static void mark(Search* s, int token, uint8_t bit) {
    if (token < 0 || token >= s->V) return;
    s->mask[token] |= bit;
}

/* The candidates of one live, unfinished parent row: src/decoder.cpp:139-170
 * (RowScan setup), src/kernels.hpp:113-140 (scan_token, scan_around_masked),
 * src/decoder.cpp:196-258 (scan_constrained). */
static void scan_parent(Search* s, int p, const float* row, int has_offset, float offset) {
    const float pr = s->raw[p];
    const int new_length = s->len[p] + 1;
    const float inv = 1.0f / oracle_gnmt_penalty(new_length, s->alpha);
    const int V = s->V;
    if (s->constrained) {
        for (int v = 0; v < V; ++v) s->mask[v] = s->banned && s->banned[v] ? 1 : 0;
        const int32_t* pre = s->prefix + (size_t)p * s->cap;
        const int L = s->prefix_len[p];
        const int n = s->ngram;
        if (n == 1) {
            for (int i = 0; i < L; ++i) mark(s, pre[i], 2);
        } else if (n > 1 && L >= n - 1) {
            const int suffix = L - (n - 1);
            for (int i = 0; i + n <= L; ++i) {
                int same = 1;
                for (int j = 0; j < n - 1 && same; ++j) same = pre[i + j] == pre[suffix + j];
                if (same) mark(s, pre[i + n - 1], 2);
            }
        }
        if (s->penalise)
            for (int i = 0; i < L; ++i) mark(s, pre[i], 4);
    }
    for (int v = 0; v < V; ++v) {
        const float lp = has_offset ? row[v] - offset : row[v];
        if (!(lp < INFINITY)) {
            s->invalid = 1;
            continue;
        }
        if (lp == NEG_INF) continue;
        if (min_masked(s, v, new_length)) continue;
        float value = lp;
        if (s->constrained) {
            const uint8_t m = s->mask[v];
            if (m & 3) continue;
            if (m & 4) value = lp - s->log_penalty;
        } else if (s->banned && s->banned[v]) {
            continue;
        }
        const float raw = pr + value;
        const Cand c = {raw * inv, raw, p, v, new_length, 1};
        insert_top(s->top, s->K, &c);
    }
}

/* One step (src/decoder.cpp:122-177 step, :314-350 select). `rows` points at
 * the step's [stride, V] block; outputs are written at slot base `obase`
 * (index of slot 0 of this step in the [.., K] trace) and row_lse at `lbase`. */
static void search_step(Search* s, const void* rows, int data_type, int from_logits,
                        const DBSCudaDecodeOutputs* out, int64_t obase, float* row_lse) {
    const int K = s->K;
    const Cand empty = {NEG_INF, NEG_INF, -1, -1, 0, 0};
    for (int k = 0; k < K; ++k) s->top[k] = empty;
    for (int p = 0; p < K; ++p) {
        const float pr = s->raw[p];
        if (!isfinite(pr)) continue;
        if (s->eos >= 0 && s->ended[p]) {
            const int l = s->len[p] > 1 ? s->len[p] : 1;
            const int32_t last = s->last[p];
            const Cand c = {pr / oracle_gnmt_penalty(l, s->alpha), pr, p, is_eos(s, last) ? last : s->eos, l, 0};
            insert_top(s->top, K, &c);
            continue;
        }
        load_row(rows, data_type, p, s->V, s->row);
        float offset = 0.0f;
        if (from_logits) {
            const float lse = oracle_row_lse(s->row, s->V, &s->invalid);
            if (row_lse) row_lse[obase + p] = lse;
            if (lse == NEG_INF) continue;
            offset = lse;
        }
        scan_parent(s, p, s->row, from_logits, offset);
    }
    /* select */
    float* nraw = (float*)malloc(sizeof(float) * K);
    int32_t* nlen = (int32_t*)malloc(sizeof(int32_t) * K);
    uint8_t* nend = (uint8_t*)malloc(K);
    int32_t* npre = s->constrained ? (int32_t*)malloc(sizeof(int32_t) * (size_t)K * s->cap) : NULL;
    int32_t* nplen = s->constrained ? (int32_t*)malloc(sizeof(int32_t) * K) : NULL;
    for (int k = 0; k < K; ++k) {
        const Cand* c = &s->top[k];
        const int64_t i = obase + k;
        if (out->parents) out->parents[i] = c->parent;
        if (out->tokens) out->tokens[i] = c->token;
        if (out->lengths) out->lengths[i] = c->length;
        if (out->raw_scores) out->raw_scores[i] = c->raw;
        if (out->scores) out->scores[i] = c->score;
        if (out->from_logprob) out->from_logprob[i] = c->from_logprob;
        nraw[k] = c->raw;
        nlen[k] = c->length;
        s->last[k] = c->token;
        if (c->parent >= 0) {
            nend[k] = (uint8_t)(s->ended[c->parent] != 0 || is_eos(s, c->token));
            if (npre) {
                const int L = s->prefix_len[c->parent];
                memcpy(npre + (size_t)k * s->cap, s->prefix + (size_t)c->parent * s->cap, sizeof(int32_t) * L);
                int nl = L;
                if (c->from_logprob && c->token >= 0 && nl < s->cap) npre[(size_t)k * s->cap + nl++] = c->token;
                nplen[k] = nl;
            }
        } else {
            nend[k] = 0;
            if (nplen) nplen[k] = 0;
        }
    }
    memcpy(s->raw, nraw, sizeof(float) * K);
    memcpy(s->len, nlen, sizeof(int32_t) * K);
    memcpy(s->ended, nend, K);
    if (npre) {
        memcpy(s->prefix, npre, sizeof(int32_t) * (size_t)K * s->cap);
        memcpy(s->prefix_len, nplen, sizeof(int32_t) * K);
    }
    free(nraw);
    free(nlen);
    free(nend);
    free(npre);
    free(nplen);
}

static void empty_slot(const DBSCudaDecodeOutputs* out, int64_t i) {
    if (out->parents) out->parents[i] = -1;
    if (out->tokens) out->tokens[i] = -1;
    if (out->lengths) out->lengths[i] = 0;
    if (out->raw_scores) out->raw_scores[i] = NEG_INF;
    if (out->scores) out->scores[i] = NEG_INF;
    if (out->from_logprob) out->from_logprob[i] = 0;
}

static int args_ok(const DBSCudaDecodeArgs* a) {
    if (!a || a->batch_size <= 0 || a->steps <= 0 || a->beam_size <= 0 || a->vocab_size <= 0) return 0;
    if (a->beam_size > DBS_CUDA_MAX_BEAM || a->eos_token < -1 || a->eos_token >= a->vocab_size) return 0;
    if (a->min_length < 0 || a->reserved0 != 0) return 0;
    if (!isfinite(a->length_penalty_alpha) || a->length_penalty_alpha < 0.0f) return 0;
    if (!isfinite(a->repetition_penalty) || a->repetition_penalty < 0.0f) return 0;
    return 1;
}

static int options_ok(const DBSCudaSearchOptions* o, const DBSCudaDecodeArgs* a) {
    if (!o) return 1;
    if (o->reserved0 || o->reserved[0] || o->reserved[1] || o->reserved[2] || o->reserved[3]) return 0;
    if (o->extra_eos_count < 0 || o->extra_eos_count > DBS_CUDA_MAX_EXTRA_EOS) return 0;
    for (int i = 0; i < o->extra_eos_count; ++i)
        if (o->extra_eos_tokens[i] < 0 || o->extra_eos_tokens[i] >= a->vocab_size) return 0;
    return o->extra_eos_count == 0 || a->eos_token >= 0 || a->eos_tokens_per_example;
}

/* Per-example settings; 0 when an override is out of range. */
static int example_meta(const DBSCudaDecodeArgs* a, int b, int* steps, int* beam, int* eos, int* min_length) {
    *steps = a->steps_per_example ? a->steps_per_example[b] : a->steps;
    *beam = a->beam_sizes_per_example ? a->beam_sizes_per_example[b] : a->beam_size;
    *eos = a->eos_tokens_per_example ? a->eos_tokens_per_example[b] : a->eos_token;
    *min_length = a->min_lengths_per_example ? a->min_lengths_per_example[b] : a->min_length;
    return *steps >= 1 && *steps <= a->steps && *beam >= 1 && *beam <= a->beam_size && *eos >= -1 &&
           *eos < a->vocab_size && *min_length >= 0;
}

static void search_init(Search* s, const DBSCudaDecodeArgs* a, const DBSCudaSearchOptions* o, int beam, int eos,
                        int min_length, int cap) {
    memset(s, 0, sizeof *s);
    s->K = beam;
    s->stride = a->beam_size;
    s->V = a->vocab_size;
    s->eos = eos;
    s->min_length = min_length;
    s->alpha = a->length_penalty_alpha;
    s->ngram = a->no_repeat_ngram_size;
    s->penalise = a->repetition_penalty > 1.0f;
    s->log_penalty = s->penalise ? logf(a->repetition_penalty) : 0.0f;
    s->banned = a->banned_tokens;
    s->constrained = s->penalise || s->ngram > 0;
    if (eos >= 0) {
        /* src/decoder.cpp:57-63: every EOS token, sorted and distinct */
        s->eos_set[s->n_eos++] = eos;
        for (int i = 0; o && i < o->extra_eos_count; ++i) s->eos_set[s->n_eos++] = o->extra_eos_tokens[i];
        for (int i = 1; i < s->n_eos; ++i)
            for (int j = i; j > 0 && s->eos_set[j] < s->eos_set[j - 1]; --j) {
                const int32_t t = s->eos_set[j];
                s->eos_set[j] = s->eos_set[j - 1];
                s->eos_set[j - 1] = t;
            }
        int n = 0;
        for (int i = 0; i < s->n_eos; ++i)
            if (n == 0 || s->eos_set[n - 1] != s->eos_set[i]) s->eos_set[n++] = s->eos_set[i];
        s->n_eos = n;
    }
    s->raw = (float*)malloc(sizeof(float) * beam);
    s->len = (int32_t*)calloc(beam, sizeof(int32_t));
    s->ended = (uint8_t*)calloc(beam, 1);
    s->last = (int32_t*)malloc(sizeof(int32_t) * beam);
    s->cap = cap > 0 ? cap : 1;
    s->prefix = (int32_t*)calloc((size_t)beam * s->cap, sizeof(int32_t));
    s->prefix_len = (int32_t*)calloc(beam, sizeof(int32_t));
    s->top = (Cand*)malloc(sizeof(Cand) * beam);
    s->row = (float*)malloc(sizeof(float) * s->V);
    s->mask = (uint8_t*)malloc(s->V);
    for (int k = 0; k < beam; ++k) {
        s->raw[k] = k == 0 ? 0.0f : NEG_INF;
        s->last[k] = -1;
    }
}

static void search_free(Search* s) {
    free(s->raw);
    free(s->len);
    free(s->ended);
    free(s->last);
    free(s->prefix);
    free(s->prefix_len);
    free(s->top);
    free(s->row);
    free(s->mask);
}

/* Batch decode in the engine's layout (src/c_api.cpp:703-800 decode_batch_into,
 * plus per-example beams / EOS / min lengths, which the engine supports and the
 * CPU batch API does not: example b then behaves as a decoder of beam size
 * beam_b reading rows 0..beam_b-1 of each step). */
int oracle_decode(const void* inputs, int data_type, int from_logits, const DBSCudaDecodeArgs* a,
                  const DBSCudaSearchOptions* o, const DBSCudaDecodeOutputs* out, float* row_lse) {
    if (!inputs || !args_ok(a) || !out || !out->final_scores || !options_ok(o, a)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (data_type < 0 || data_type > 2) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    const int B = a->batch_size, T = a->steps, K = a->beam_size, V = a->vocab_size;
    for (int b = 0; b < B; ++b) {
        int st, bm, eos, ml;
        if (!example_meta(a, b, &st, &bm, &eos, &ml)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const size_t es = (size_t)elem_size(data_type);
    for (int b = 0; b < B; ++b) {
        int steps, beam, eos, min_length;
        example_meta(a, b, &steps, &beam, &eos, &min_length);
        Search s;
        search_init(&s, a, o, beam, eos, min_length, T);
        const int64_t tbase = (int64_t)b * T * K;
        if (row_lse)
            for (int64_t i = 0; i < (int64_t)T * K; ++i) row_lse[tbase + i] = 0.0f;
        for (int t = 0; t < T; ++t) {
            const int64_t obase = tbase + (int64_t)t * K;
            if (t < steps) {
                const char* rows = (const char*)inputs + (size_t)obase * V * es;
                search_step(&s, rows, data_type, from_logits, out, obase, from_logits ? row_lse : NULL);
                for (int k = beam; k < K; ++k) empty_slot(out, obase + k);
            } else {
                for (int k = 0; k < K; ++k) empty_slot(out, obase + k);
            }
        }
        for (int k = 0; k < K; ++k) {
            const int64_t i = (int64_t)b * K + k;
            float raw = NEG_INF, score = NEG_INF;
            int len = 0;
            if (k < beam) {
                raw = s.raw[k];
                len = s.len[k];
                score = raw / oracle_gnmt_penalty(len > 1 ? len : 1, s.alpha);
            }
            out->final_scores[i] = score;
            if (out->final_raw_scores) out->final_raw_scores[i] = raw;
            if (out->final_lengths) out->final_lengths[i] = len;
        }
        if (out->invalid_input) out->invalid_input[b] = (uint8_t)s.invalid;
        search_free(&s);
    }
    return DBS_CUDA_STATUS_OK;
}

/* One step from a caller state (src/decoder.cpp:441-476 BeamSearchDecoder::step
 * with restore/save at :84-116). */
int oracle_decode_step(const void* inputs, int data_type, int from_logits, const DBSCudaDecodeArgs* a,
                       const DBSCudaSearchOptions* o, const DBSCudaBeamState* st, const DBSCudaDecodeOutputs* out,
                       float* row_lse) {
    if (!inputs || !args_ok(a) || !st || !out || !options_ok(o, a)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (a->steps != 1 || a->steps_per_example) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    if (!st->raw_scores || !st->lengths || !st->finished || st->prefix_stride < 0 || st->reserved0) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const int B = a->batch_size, K = a->beam_size, V = a->vocab_size;
    const size_t es = (size_t)elem_size(data_type);
    const int stride = st->prefix_stride;
    for (int b = 0; b < B; ++b) {
        int steps, beam, eos, min_length;
        if (!example_meta(a, b, &steps, &beam, &eos, &min_length)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    for (int b = 0; b < B; ++b) {
        int steps, beam, eos, min_length;
        example_meta(a, b, &steps, &beam, &eos, &min_length);
        Search s;
        search_init(&s, a, o, beam, eos, min_length, stride + 1);
        const int64_t sb = (int64_t)b * K;
        for (int k = 0; k < beam; ++k) {
            s.raw[k] = st->raw_scores[sb + k];
            s.len[k] = st->lengths[sb + k];
            s.ended[k] = st->finished[sb + k] != 0;
            const int L = s.len[k];
            s.last[k] = st->prefixes && L >= 1 && L <= stride ? st->prefixes[(sb + k) * stride + L - 1] : -1;
            if (s.constrained && st->prefixes) {
                const int n = L < 0 ? 0 : (L > stride ? stride : L);
                memcpy(s.prefix + (size_t)k * s.cap, st->prefixes + (sb + k) * stride, sizeof(int32_t) * n);
                s.prefix_len[k] = n;
            }
        }
        if (row_lse)
            for (int k = 0; k < K; ++k) row_lse[sb + k] = 0.0f;
        const char* rows = (const char*)inputs + (size_t)sb * V * es;
        search_step(&s, rows, data_type, from_logits, out, sb, from_logits ? row_lse : NULL);
        for (int k = beam; k < K; ++k) empty_slot(out, sb + k);
        for (int k = 0; k < K; ++k) {
            const int64_t i = sb + k;
            if (k < beam) {
                st->raw_scores[i] = s.raw[k];
                st->lengths[i] = s.len[k];
                st->finished[i] = s.ended[k];
            } else {
                st->raw_scores[i] = NEG_INF;
                st->lengths[i] = 0;
                st->finished[i] = 0;
            }
            if (out->final_scores) {
                float raw = NEG_INF, score = NEG_INF;
                int len = 0;
                if (k < beam) {
                    raw = s.raw[k];
                    len = s.len[k];
                    score = raw / oracle_gnmt_penalty(len > 1 ? len : 1, s.alpha);
                }
                out->final_scores[i] = score;
                if (out->final_raw_scores) out->final_raw_scores[i] = raw;
                if (out->final_lengths) out->final_lengths[i] = len;
            }
        }
        if (out->invalid_input) out->invalid_input[b] = (uint8_t)s.invalid;
        search_free(&s);
    }
    return DBS_CUDA_STATUS_OK;
}

/* ------------------------------------------------------------------------- */
/* Backward (src/decoder.cpp:186-304 run_backward without a relaxed pool;     */
/* :639-661 path_gradient / final_scores_path_gradient; src/decoder.hpp:212-242 */
/* apply_path_gradient)                                                       */
/* ------------------------------------------------------------------------- */

typedef struct {
    int64_t index; /* within the example's [T, K, V] */
    float value;
    int64_t slot;  /* t * K + k */
} Entry;

static int cmp_entry(const void* x, const void* y) {
    const Entry* a = (const Entry*)x;
    const Entry* b = (const Entry*)y;
    if (a->index != b->index) return a->index < b->index ? -1 : 1;
    return a->slot < b->slot ? -1 : (a->slot > b->slot);
}

/* The path-gradient entries of example b (unsorted); returns their count. */
/* Selected-beam weights term of drank (src/decoder.cpp:599-604): weights / grad_weights are
 * the example's [T, K] rows, or NULL. */
typedef struct {
    const float* w;
    const float* gw;
    float temperature;
} SelectedTerm;

static int example_entries_sel(const DBSCudaDecodeArgs* a, int b, int steps, int beam,
                               const DBSCudaBackwardInputs* in, const SelectedTerm* sel, Entry* entries);

static int example_entries(const DBSCudaDecodeArgs* a, int b, int steps, int beam, const DBSCudaBackwardInputs* in,
                           Entry* entries) {
    return example_entries_sel(a, b, steps, beam, in, NULL, entries);
}

static int example_entries_sel(const DBSCudaDecodeArgs* a, int b, int steps, int beam,
                               const DBSCudaBackwardInputs* in, const SelectedTerm* sel, Entry* entries) {
    const int T = a->steps, K = a->beam_size, V = a->vocab_size;
    float* next = (float*)calloc(beam, sizeof(float));
    float* prev = (float*)calloc(beam, sizeof(float));
    int n = 0;
    for (int t = steps - 1; t >= 0; --t) {
        for (int k = 0; k < beam; ++k) prev[k] = 0.0f;
        const int last = t == steps - 1;
        const float* w = NULL;
        const float* gw = NULL;
        float weighted_dot = 0.0f;
        if (sel && sel->gw) {
            /* dot(w, gw, K) in slot order (src/kernels_scalar.cpp:271-275) */
            w = sel->w + ((int64_t)b * T + t) * K;
            gw = sel->gw + ((int64_t)b * T + t) * K;
            for (int k = 0; k < K; ++k) weighted_dot += w[k] * gw[k];
        }
        for (int k = 0; k < beam; ++k) {
            const int64_t idx = ((int64_t)b * T + t) * K + k;
            const int parent = in->parents[idx];
            if (parent < 0 || parent >= beam) continue;
            float drank = 0.0f;
            if (gw) drank += (w[k] * (gw[k] - weighted_dot)) / sel->temperature;
            if (in->grad_scores) drank += in->grad_scores[idx];
            if (in->grad_final_scores && last) drank += in->grad_final_scores[(int64_t)b * K + k];
            const int l = in->lengths[idx] > 1 ? in->lengths[idx] : 1;
            const float inv = 1.0f / oracle_gnmt_penalty(l, a->length_penalty_alpha);
            float draw = next[k] + drank * inv;
            if (in->grad_raw_scores) draw += in->grad_raw_scores[idx];
            if (in->grad_final_raw_scores && last) draw += in->grad_final_raw_scores[(int64_t)b * K + k];
            if (draw == 0.0f) continue;
            prev[parent] += draw;
            const int token = in->tokens[idx];
            if (in->from_logprob[idx] && token >= 0 && token < V) {
                entries[n].index = ((int64_t)t * K + parent) * V + token;
                entries[n].value = draw;
                entries[n].slot = (int64_t)t * K + k;
                ++n;
            }
        }
        float* tmp = next;
        next = prev;
        prev = tmp;
    }
    free(next);
    free(prev);
    return n;
}

static int backward_sel(const DBSCudaDecodeArgs* a, const DBSCudaBackwardInputs* in, const SelectedTerm* sel,
                        float* grad);

int oracle_backward(const DBSCudaDecodeArgs* a, const DBSCudaBackwardInputs* in, float* grad) {
    return backward_sel(a, in, NULL, grad);
}

int oracle_backward_selected(const DBSCudaDecodeArgs* a, const DBSCudaBackwardInputs* in, const float* weights,
                             const float* grad_weights, float temperature, float* grad) {
    if (!weights != !grad_weights || !(temperature > 0.0f)) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    SelectedTerm sel = {weights, grad_weights, temperature};
    return backward_sel(a, in, &sel, grad);
}

/* softmax_selected (src/kernels_scalar.cpp:277-302) over each step's K selected scores:
 * weights [B, T, K] from the decode's scores [B, T, K]. */
void oracle_selected_weights(const DBSCudaDecodeArgs* a, const float* scores, float temperature, float* weights) {
    const float kNegGuard = -1.0e30f;
    const int64_t rows = (int64_t)a->batch_size * a->steps;
    const int K = a->beam_size;
    for (int64_t r = 0; r < rows; ++r) {
        const float* sc = scores + r * K;
        float* out = weights + r * K;
        for (int i = 0; i < K; ++i) out[i] = 0.0f;
        float maxv = -INFINITY;
        for (int i = 0; i < K; ++i) {
            if (sc[i] > kNegGuard) {
                const float q = sc[i] / temperature;
                maxv = maxv < q ? q : maxv; /* std::max */
            }
        }
        if (!isfinite(maxv)) continue;
        float sum = 0.0f;
        for (int i = 0; i < K; ++i) {
            if (sc[i] > kNegGuard) {
                out[i] = oracle_exp_nonpositive(sc[i] / temperature - maxv);
                sum += out[i];
            }
        }
        if (!(sum > 0.0f) || !isfinite(sum)) {
            for (int i = 0; i < K; ++i) out[i] = 0.0f;
            continue;
        }
        const float inv_sum = 1.0f / sum;
        for (int i = 0; i < K; ++i) out[i] *= inv_sum;
    }
}

static int backward_sel(const DBSCudaDecodeArgs* a, const DBSCudaBackwardInputs* in, const SelectedTerm* sel,
                        float* grad) {
    if (!args_ok(a) || !in || !grad || !in->parents || !in->tokens || !in->lengths || !in->from_logprob) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    if (in->logits && !in->row_lse) return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    const int B = a->batch_size, T = a->steps, K = a->beam_size, V = a->vocab_size;
    Entry* entries = (Entry*)malloc(sizeof(Entry) * (size_t)T * K);
    float* row = (float*)malloc(sizeof(float) * V);
    float* g = (float*)malloc(sizeof(float) * V);
    for (int b = 0; b < B; ++b) {
        int steps, beam, eos, ml;
        if (!example_meta(a, b, &steps, &beam, &eos, &ml)) {
            steps = steps < 0 ? 0 : (steps > T ? T : steps);
            beam = beam < 0 ? 0 : (beam > K ? K : beam);
        }
        const int n = example_entries_sel(a, b, steps, beam, in, sel, entries);
        qsort(entries, (size_t)n, sizeof(Entry), cmp_entry);
        float* out = grad + (int64_t)b * T * K * V;
        if (!in->logits) {
            for (int i = 0; i < n; ++i) out[entries[i].index] += entries[i].value;
            continue;
        }
        int i = 0;
        while (i < n) {
            const int64_t r = entries[i].index / V;
            int j = i;
            float sum = 0.0f;
            for (; j < n && entries[j].index / V == r; ++j) sum = sum + entries[j].value;
            const int64_t grow = (int64_t)b * T * K + r;
            load_row(in->logits, in->logits_type, grow, V, row);
            const float lse = in->row_lse[grow];
            for (int v = 0; v < V; ++v) g[v] = 0.0f - softmax_probability(row[v], lse) * sum;
            for (int k = i; k < j; ++k) {
                const int v = (int)(entries[k].index - r * V);
                g[v] = entries[k].value - softmax_probability(row[v], lse) * sum;
            }
            for (int v = 0; v < V; ++v) out[r * V + v] += g[v];
            i = j;
        }
    }
    free(entries);
    free(row);
    free(g);
    return DBS_CUDA_STATUS_OK;
}

int oracle_path_gradient(const DBSCudaDecodeArgs* a, const int32_t* parents, const int32_t* tokens,
                         const int32_t* lengths, const uint8_t* from_logprob, const float* grad_final,
                         float* draws) {
    if (!args_ok(a) || !parents || !tokens || !lengths || !from_logprob || !grad_final || !draws) {
        return DBS_CUDA_STATUS_INVALID_ARGUMENT;
    }
    const int B = a->batch_size, T = a->steps, K = a->beam_size;
    DBSCudaBackwardInputs in;
    memset(&in, 0, sizeof in);
    in.parents = parents;
    in.tokens = tokens;
    in.lengths = lengths;
    in.from_logprob = from_logprob;
    in.grad_final_scores = grad_final;
    Entry* entries = (Entry*)malloc(sizeof(Entry) * (size_t)T * K);
    memset(draws, 0, sizeof(float) * (size_t)B * T * K);
    for (int b = 0; b < B; ++b) {
        int steps, beam, eos, ml;
        if (!example_meta(a, b, &steps, &beam, &eos, &ml)) {
            steps = steps < 0 ? 0 : (steps > T ? T : steps);
            beam = beam < 0 ? 0 : (beam > K ? K : beam);
        }
        const int n = example_entries(a, b, steps, beam, &in, entries);
        for (int i = 0; i < n; ++i) draws[(int64_t)b * T * K + entries[i].slot] = entries[i].value;
    }
    free(entries);
    return DBS_CUDA_STATUS_OK;
}

void oracle_length_penalty(const int32_t* lengths, int64_t count, float alpha, float* out) {
    for (int64_t i = 0; i < count; ++i) out[i] = oracle_gnmt_penalty(lengths[i], alpha);
}
