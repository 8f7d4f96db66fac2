// SPDX-License-Identifier: MIT
//
// Deterministic arithmetic of the beam-search contract, on the device.
//
// Every floating-point result the engine reports must equal the reference CPU
// decoder's bit for bit (beamgrad 2.3.0, src/penalty.hpp, src/logits.hpp,
// src/half.hpp). That holds because both sides use only correctly rounded
// IEEE-754 basic operations (add, sub, mul, div, the exact frexp/ldexp and
// floor) in the same order and never fuse a multiply with an add. Here every
// operation is an explicitly rounded intrinsic (__fadd_rn, __dmul_rn, ...),
// which nvcc never contracts, and the library is also built with -fmad=false.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace dbsb {

constexpr int kLanes = 256;  // lanes of the fixed logsumexp reduction order (src/logits.hpp:27)

__device__ __forceinline__ float f_inf() { return __uint_as_float(0x7f800000u); }
__device__ __forceinline__ float f_ninf() { return __uint_as_float(0xff800000u); }
__device__ __forceinline__ bool f_finite(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

// ---------------------------------------------------------------------------
// Double-precision pieces of the GNMT length penalty (src/penalty.hpp:78-160).
// ---------------------------------------------------------------------------

// ln(x), x >= 1: x = m 2^e with m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s),
// s = (m - 1)/(m + 1), atanh(s)/s by its series in s^2 up to s^22 (Horner).
__device__ __forceinline__ double log_ge1(double x) {
    int e = 0;
    double m = frexp(x, &e);
    if (m < 0.70710678118654752440) {
        m = __dmul_rn(m, 2.0);
        e -= 1;
    }
    const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
    const double s2 = __dmul_rn(s, s);
    double p = 1.0 / 23.0;
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 21.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 19.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 17.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 15.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 13.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 11.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 9.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 7.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 5.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0 / 3.0);
    p = __dadd_rn(__dmul_rn(p, s2), 1.0);
    const double log_m = __dmul_rn(__dmul_rn(2.0, s), p);
    const double de = static_cast<double>(e);
    // ln 2 = hi + lo with hi short enough that e * hi is exact.
    return __dadd_rn(__dmul_rn(de, 6.93147180369123816490e-01), __dadd_rn(__dmul_rn(de, 1.90821492927058770002e-10), log_m));
}

// exp(y), y >= 0: y = k ln 2 + r, Taylor polynomial of exp(r) to r^15, times 2^k.
__device__ __forceinline__ double exp_ge0(double y) {
    if (y > 709.0) return __longlong_as_double(0x7ff0000000000000LL);
    const int k = static_cast<int>(__dadd_rn(__dmul_rn(y, 1.44269504088896338700e+00), 0.5));
    const double dk = static_cast<double>(k);
    const double r = __dsub_rn(__dsub_rn(y, __dmul_rn(dk, 6.93147180369123816490e-01)), __dmul_rn(dk, 1.90821492927058770002e-10));
    double p = 1.0 / 1307674368000.0;
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 87178291200.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 6227020800.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 479001600.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 39916800.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 3628800.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 362880.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 40320.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 5040.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 720.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 120.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 24.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0 / 6.0);
    p = __dadd_rn(__dmul_rn(p, r), 0.5);
    p = __dadd_rn(__dmul_rn(p, r), 1.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0);
    return ldexp(p, k);
}

// GNMT length penalty ((5 + max(length, 1)) / 6)^alpha, rounded to float once.
// Integer exponents up to 64 by repeated squaring; others through exp/log.
__device__ __forceinline__ float gnmt_penalty(int length, float alpha) {
    if (alpha == 0.0f) return 1.0f;
    const int l = length > 1 ? length : 1;
    const double base = __ddiv_rn(__dadd_rn(5.0, static_cast<double>(l)), 6.0);
    if (alpha <= 64.0f && alpha == static_cast<float>(static_cast<int>(alpha))) {
        int n = static_cast<int>(alpha);
        double result = 1.0;
        double sq = base;
        while (n > 0) {
            if (n & 1) result = __dmul_rn(result, sq);
            sq = __dmul_rn(sq, sq);
            n >>= 1;
        }
        return __double2float_rn(result);
    }
    return __double2float_rn(exp_ge0(__dmul_rn(static_cast<double>(alpha), log_ge1(base))));
}

// ---------------------------------------------------------------------------
// exp(x) for x <= 0 (src/logits.hpp:204-235): the Cephes expf reduction
// k = floor(x log2 e + 1/2), r = x - k ln2 (two-part ln 2) and its degree-5
// polynomial, then p * 2^k; 0 below -87 (and for -inf / NaN).
// ---------------------------------------------------------------------------
namespace cephes {
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693359375f;
constexpr float kLn2Lo = -2.12194440e-4f;
constexpr float kP0 = 1.9875691500e-4f;
constexpr float kP1 = 1.3981999507e-3f;
constexpr float kP2 = 8.3334519073e-3f;
constexpr float kP3 = 4.1665795894e-2f;
constexpr float kP4 = 1.6666665459e-1f;
constexpr float kP5 = 5.0000001201e-1f;
constexpr float kMin = -87.0f;
}  // namespace cephes

// The contract's form, valid for any argument (used off the hot loop, e.g. for
// softmax probabilities of caller-supplied row_lse values).
__device__ __forceinline__ float exp_nonpositive(float x) {
    using namespace cephes;
    if (!(x >= kMin)) return 0.0f;
    const float k = floorf(__fadd_rn(__fmul_rn(x, kLog2e), 0.5f));
    const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(k, kLn2Hi)), __fmul_rn(k, kLn2Lo));
    const float r2 = __fmul_rn(r, r);
    float p = kP0;
    p = __fadd_rn(__fmul_rn(p, r), kP1);
    p = __fadd_rn(__fmul_rn(p, r), kP2);
    p = __fadd_rn(__fmul_rn(p, r), kP3);
    p = __fadd_rn(__fmul_rn(p, r), kP4);
    p = __fadd_rn(__fmul_rn(p, r), kP5);
    p = __fadd_rn(__fadd_rn(__fmul_rn(p, r2), r), 1.0f);
    const int e = static_cast<int>(k) + 127;
    return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(e) << 23));
}

// The same value for d in [-87, 0] with the hot loop's instruction mix; the
// caller guarantees d <= 0 and selects 0 where !(d >= -87).
//   * floor(y) for y in [-126, 1] is one add rounded toward -inf against
//     M = 1.5 * 2^23 (ulp 1 there) and one exact subtraction of M;
//   * k = floor(y) lies in [-125, 0], so p * 2^k (p in [0.70, 1.42]) is a
//     normal float and the product is exact: adding k to p's exponent field
//     gives the same bits. The low mantissa bits of z = M + k hold k, and
//     (bits(z) << 23) mod 2^32 is exactly k << 23.
__device__ __forceinline__ float exp_nonpositive_fast(float d) {
    using namespace cephes;
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    const float y = __fadd_rn(__fmul_rn(d, kLog2e), 0.5f);
    const float z = __fadd_rd(y, kMagic);
    const float k = __fsub_rn(z, kMagic);
    const float r = __fsub_rn(__fsub_rn(d, __fmul_rn(k, kLn2Hi)), __fmul_rn(k, kLn2Lo));
    const float r2 = __fmul_rn(r, r);
    float p = kP0;
    p = __fadd_rn(__fmul_rn(p, r), kP1);
    p = __fadd_rn(__fmul_rn(p, r), kP2);
    p = __fadd_rn(__fmul_rn(p, r), kP3);
    p = __fadd_rn(__fmul_rn(p, r), kP4);
    p = __fadd_rn(__fmul_rn(p, r), kP5);
    p = __fadd_rn(__fadd_rn(__fmul_rn(p, r2), r), 1.0f);
    return __uint_as_float(__float_as_uint(p) + (__float_as_uint(z) << 23));
}

// exp_nonpositive(d) for any d <= 0 without a branch: exp_nonpositive_fast(d)
// where d >= -87, and +0 elsewhere (d < -87, -inf, NaN) through a bit mask.
__device__ __forceinline__ float exp_nonpositive_masked(float d) {
    uint32_t keep;
    asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(keep) : "f"(d), "f"(cephes::kMin));
    return __uint_as_float(__float_as_uint(exp_nonpositive_fast(d)) & keep);
}

// ---------------------------------------------------------------------------
// Pairs of floats in one 64-bit register (f32x2), for the logsumexp hot loop.
//
// Every packed operation is a packed fused multiply-add whose extra operand
// is a runtime 1.0 or -0.0 (Pack2::one / Pack2::nzero, filled by the host):
//   fma(a, b, -0) = round(a * b)     fma(1, a, b) = round(a + b)
// so each rounds exactly once, like the scalar mul.rn / add.rn. Because the
// constants are not known when the kernel is compiled, no instruction can be
// rewritten into a different rounding sequence. (Plain packed mul / add were
// measured to differ from the scalar chain on about 0.2% of exp arguments in
// some compiled contexts, so they are not used; the form below matched the
// scalar exp on every float in [-87, 0] in both halves.)
// ---------------------------------------------------------------------------
struct Pack2 {
    uint64_t one;    // (1.0f, 1.0f)
    uint64_t nzero;  // (-0.0f, -0.0f)
};

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2_splat(float c) { return f2_pack(c, c); }
constexpr uint64_t kF2Sign = 0x8000000080000000ull;
__device__ __forceinline__ uint64_t f2_mul(const Pack2& q, uint64_t a, uint64_t b) { return f2_fma(a, b, q.nzero); }
__device__ __forceinline__ uint64_t f2_add(const Pack2& q, uint64_t a, uint64_t b) { return f2_fma(q.one, a, b); }
// round(a - b) = round(a + (-b)); negation flips the sign bits exactly.
__device__ __forceinline__ uint64_t f2_sub(const Pack2& q, uint64_t a, uint64_t b) { return f2_fma(q.one, a, b ^ kF2Sign); }

// fma(a, b, c) on both halves rounded toward minus infinity.
__device__ __forceinline__ uint64_t f2_fma_rm(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rm.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// exp_nonpositive_fast on both halves of d (each in [-87, 0]), step for step, every
// step packed: the floor's add rounded toward minus infinity is fma.rm(1, y, M), which
// rounds y + M once in that direction exactly as the scalar add.rm does.
__device__ __forceinline__ void exp_nonpositive_fast2(const Pack2& q, uint64_t d, float& e_lo, float& e_hi) {
    using namespace cephes;
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    const uint64_t y = f2_add(q, f2_mul(q, d, f2_splat(kLog2e)), f2_splat(0.5f));
    const uint64_t z2 = f2_fma_rm(q.one, y, f2_splat(kMagic));
    float z_lo, z_hi;
    f2_unpack(z2, z_lo, z_hi);
    const uint64_t k = f2_sub(q, z2, f2_splat(kMagic));
    // d - round(k ln2hi) is d - k ln2hi rounded once, a single fma: k ln2hi is exact
    // (k an integer in [-126, 0], ln2hi = 355/512 needs 9 significant bits).
    const uint64_t r1 = f2_fma(k, f2_splat(-kLn2Hi), d);
    // r1 - round(k ln2lo) = r1 + round(k (-ln2lo)): rounding to nearest is sign-symmetric.
    const uint64_t r = f2_add(q, r1, f2_mul(q, k, f2_splat(-kLn2Lo)));
    const uint64_t r2 = f2_mul(q, r, r);
    uint64_t p = f2_splat(kP0);
    p = f2_add(q, f2_mul(q, p, r), f2_splat(kP1));
    p = f2_add(q, f2_mul(q, p, r), f2_splat(kP2));
    p = f2_add(q, f2_mul(q, p, r), f2_splat(kP3));
    p = f2_add(q, f2_mul(q, p, r), f2_splat(kP4));
    p = f2_add(q, f2_mul(q, p, r), f2_splat(kP5));
    p = f2_add(q, f2_add(q, f2_mul(q, p, r2), r), f2_splat(1.0f));
    float p_lo, p_hi;
    f2_unpack(p, p_lo, p_hi);
    e_lo = __uint_as_float(__float_as_uint(p_lo) + (__float_as_uint(z_lo) << 23));
    e_hi = __uint_as_float(__float_as_uint(p_hi) + (__float_as_uint(z_hi) << 23));
}

// The largest float below x (x finite or +inf; -inf stays -inf).
__device__ __forceinline__ float float_below(float x) {
    const uint32_t u = __float_as_uint(x);
    if (x == f_ninf()) return x;
    if (x == 0.0f) return __uint_as_float(0x80000001u);
    return __uint_as_float((u & 0x80000000u) ? u + 1u : u - 1u);
}

// lse = max + (float) ln(sum), sum >= 1 (src/logits.hpp:241-243).
__device__ __forceinline__ float logsumexp_from(float mx, float sum) {
    return __fadd_rn(mx, __double2float_rn(log_ge1(static_cast<double>(sum))));
}

// Softmax probability of x in a row with logsumexp lse; 0 for non-finite x
// (src/logits.hpp:246-249).
__device__ __forceinline__ float softmax_probability(float x, float lse) {
    const bool finite = x < f_inf() && x > f_ninf();
    return finite ? exp_nonpositive(__fsub_rn(x, lse)) : 0.0f;
}

// ---------------------------------------------------------------------------
// Input elements. 16-bit values widen exactly (src/half.hpp:16-29): bf16 is
// the top half of a float; fp16 -> fp32 conversion by the hardware is exact
// for every non-NaN value, subnormals included.
// ---------------------------------------------------------------------------
template <int DT>
struct Elem;
template <>
struct Elem<0> {  // DBS_CUDA_DTYPE_F32
    using T = float;
    static constexpr int kBytes = 4;
    __device__ static __forceinline__ float to_f32(float x) { return x; }
};
template <>
struct Elem<1> {  // DBS_CUDA_DTYPE_F16
    using T = uint16_t;
    static constexpr int kBytes = 2;
    __device__ static __forceinline__ float to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
};
template <>
struct Elem<2> {  // DBS_CUDA_DTYPE_BF16
    using T = uint16_t;
    static constexpr int kBytes = 2;
    __device__ static __forceinline__ float to_f32(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }
};

template <int DT>
__device__ __forceinline__ float load_elem(const void* base, int64_t i) {
    return Elem<DT>::to_f32(static_cast<const typename Elem<DT>::T*>(base)[i]);
}

__device__ __forceinline__ float load_elem_rt(const void* base, int dtype, int64_t i) {
    if (dtype == 0) return load_elem<0>(base, i);
    if (dtype == 1) return load_elem<1>(base, i);
    return load_elem<2>(base, i);
}

// ---------------------------------------------------------------------------
// Candidate keys: ordered(raw) << 32 | (0xffffffff - (parent * V + token)).
// Larger key = better candidate among candidates that share one length
// penalty (raw descending, then parent ascending, then token ascending); 0 is
// "no candidate" (no real raw maps to a zero high word). raw + 0.0f folds -0
// into +0, which compare equal in the CPU order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t make_key(float raw, uint32_t index) {
    const uint32_t u = __float_as_uint(__fadd_rn(raw, 0.0f));
    const uint32_t ordered = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<uint64_t>(ordered) << 32) | static_cast<uint64_t>(0xffffffffu - index);
}
__device__ __forceinline__ float key_raw(uint64_t key) {
    const uint32_t o = static_cast<uint32_t>(key >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}
__device__ __forceinline__ uint32_t key_index(uint64_t key) { return 0xffffffffu - static_cast<uint32_t>(key); }

}  // namespace dbsb
