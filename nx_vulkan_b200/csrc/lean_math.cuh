// lean_math.cuh -- f64 exp, expm1 and tanh for the elementwise kernels.
//
// Table-driven exponential after P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point
// arithmetic", ACM TOMS 15(2), 1989: x = (64 m + j) ln2/64 + r with
// |r| <= ln2/128, exp(x) = 2^m 2^(j/64) e^r, e^r - 1 by its Taylor series
// to r^6 (truncation below 2^-57 relative to e^r - 1 for |r| <= ln2/128).  The table
// holds 2^(j/64) as a double head and a double tail; ln2/64 is split into a 36-bit head
// (so that k * head is exact for |k| < 2^17) and a tail.  Relative error
// within a few units of 2^-53 for |x| <= 700; outside that range (and for
// inf) the library function is used.  The constants were computed from
// their definitions with 60-digit decimal arithmetic.
//
// expm1 from the same reduction: e^x - 1 = s (1 + p) - 1 = s p + (s - 1)
// with s = 2^m 2^(j/64) (s - 1 is exact for s in [1/2, 2]), accurate near 0.
// tanh(x) = -expm1(-2|x|) / (2 + expm1(-2|x|)) with the sign of x (the
// division as a product with a Newton-refined reciprocal); 1 for |x| > 20
// (where tanh rounds to 1 in double).
//
// For f32 results evaluated in f64 and rounded once (Nx.BinaryBackend's
// semantics), round_f32_checked rounds a lean result to f32 unless it lies
// within M double ulps of an f32 rounding boundary, where the caller takes
// the library's f64 function instead: both are within M double ulps of the
// true value, so away from a boundary they round to the same f32.  The
// f32-argument functions at the end (exp_f32 .. sigmoid_f32) use a shorter
// core for that purpose.
#pragma once
#include <cuda_runtime.h>

namespace nxv {
namespace lean {

__device__ const double kExp2J64[64] = {
    0x1.0000000000000p+0, 0x1.02c9a3e778061p+0, 0x1.059b0d3158574p+0, 0x1.0874518759bc8p+0,
    0x1.0b5586cf9890fp+0, 0x1.0e3ec32d3d1a2p+0, 0x1.11301d0125b51p+0, 0x1.1429aaea92de0p+0,
    0x1.172b83c7d517bp+0, 0x1.1a35beb6fcb75p+0, 0x1.1d4873168b9aap+0, 0x1.2063b88628cd6p+0,
    0x1.2387a6e756238p+0, 0x1.26b4565e27cddp+0, 0x1.29e9df51fdee1p+0, 0x1.2d285a6e4030bp+0,
    0x1.306fe0a31b715p+0, 0x1.33c08b26416ffp+0, 0x1.371a7373aa9cbp+0, 0x1.3a7db34e59ff7p+0,
    0x1.3dea64c123422p+0, 0x1.4160a21f72e2ap+0, 0x1.44e086061892dp+0, 0x1.486a2b5c13cd0p+0,
    0x1.4bfdad5362a27p+0, 0x1.4f9b2769d2ca7p+0, 0x1.5342b569d4f82p+0, 0x1.56f4736b527dap+0,
    0x1.5ab07dd485429p+0, 0x1.5e76f15ad2148p+0, 0x1.6247eb03a5585p+0, 0x1.6623882552225p+0,
    0x1.6a09e667f3bcdp+0, 0x1.6dfb23c651a2fp+0, 0x1.71f75e8ec5f74p+0, 0x1.75feb564267c9p+0,
    0x1.7a11473eb0187p+0, 0x1.7e2f336cf4e62p+0, 0x1.82589994cce13p+0, 0x1.868d99b4492edp+0,
    0x1.8ace5422aa0dbp+0, 0x1.8f1ae99157736p+0, 0x1.93737b0cdc5e5p+0, 0x1.97d829fde4e50p+0,
    0x1.9c49182a3f090p+0, 0x1.a0c667b5de565p+0, 0x1.a5503b23e255dp+0, 0x1.a9e6b5579fdbfp+0,
    0x1.ae89f995ad3adp+0, 0x1.b33a2b84f15fbp+0, 0x1.b7f76f2fb5e47p+0, 0x1.bcc1e904bc1d2p+0,
    0x1.c199bdd85529cp+0, 0x1.c67f12e57d14bp+0, 0x1.cb720dcef9069p+0, 0x1.d072d4a07897cp+0,
    0x1.d5818dcfba487p+0, 0x1.da9e603db3285p+0, 0x1.dfc97337b9b5fp+0, 0x1.e502ee78b3ff6p+0,
    0x1.ea4afa2a490dap+0, 0x1.efa1bee615a27p+0, 0x1.f50765b6e4540p+0, 0x1.fa7c1819e90d8p+0,
};

// 2^(j/64) as the head above and a tail, 2^(j/64) - head rounded to double,
// in one 16-byte entry (one load in the f64 functions)
__device__ const double2 kExp2J64HL[64] = {
    {0x1.0000000000000p+0, 0x0.0p+0}, {0x1.02c9a3e778061p+0, -0x1.19083535b085dp-56},
    {0x1.059b0d3158574p+0, 0x1.d73e2a475b465p-55}, {0x1.0874518759bc8p+0, 0x1.186be4bb284ffp-57},
    {0x1.0b5586cf9890fp+0, 0x1.8a62e4adc610bp-54}, {0x1.0e3ec32d3d1a2p+0, 0x1.03a1727c57b53p-59},
    {0x1.11301d0125b51p+0, -0x1.6c51039449b3ap-54}, {0x1.1429aaea92de0p+0, -0x1.32fbf9af1369ep-54},
    {0x1.172b83c7d517bp+0, -0x1.19041b9d78a76p-55}, {0x1.1a35beb6fcb75p+0, 0x1.e5b4c7b4968e4p-55},
    {0x1.1d4873168b9aap+0, 0x1.e016e00a2643cp-54}, {0x1.2063b88628cd6p+0, 0x1.dc775814a8495p-55},
    {0x1.2387a6e756238p+0, 0x1.9b07eb6c70573p-54}, {0x1.26b4565e27cddp+0, 0x1.2bd339940e9d9p-55},
    {0x1.29e9df51fdee1p+0, 0x1.612e8afad1255p-55}, {0x1.2d285a6e4030bp+0, 0x1.0024754db41d5p-54},
    {0x1.306fe0a31b715p+0, 0x1.6f46ad23182e4p-55}, {0x1.33c08b26416ffp+0, 0x1.32721843659a6p-54},
    {0x1.371a7373aa9cbp+0, -0x1.63aeabf42eae2p-54}, {0x1.3a7db34e59ff7p+0, -0x1.5e436d661f5e3p-56},
    {0x1.3dea64c123422p+0, 0x1.ada0911f09ebcp-55}, {0x1.4160a21f72e2ap+0, -0x1.ef3691c309278p-58},
    {0x1.44e086061892dp+0, 0x1.89b7a04ef80d0p-59}, {0x1.486a2b5c13cd0p+0, 0x1.3c1a3b69062f0p-56},
    {0x1.4bfdad5362a27p+0, 0x1.d4397afec42e2p-56}, {0x1.4f9b2769d2ca7p+0, -0x1.4b309d25957e3p-54},
    {0x1.5342b569d4f82p+0, -0x1.07abe1db13cadp-55}, {0x1.56f4736b527dap+0, 0x1.9bb2c011d93adp-54},
    {0x1.5ab07dd485429p+0, 0x1.6324c054647adp-54}, {0x1.5e76f15ad2148p+0, 0x1.ba6f93080e65ep-54},
    {0x1.6247eb03a5585p+0, -0x1.383c17e40b497p-54}, {0x1.6623882552225p+0, -0x1.bb60987591c34p-54},
    {0x1.6a09e667f3bcdp+0, -0x1.bdd3413b26456p-54}, {0x1.6dfb23c651a2fp+0, -0x1.bbe3a683c88abp-57},
    {0x1.71f75e8ec5f74p+0, -0x1.16e4786887a99p-55}, {0x1.75feb564267c9p+0, -0x1.0245957316dd3p-54},
    {0x1.7a11473eb0187p+0, -0x1.41577ee04992fp-55}, {0x1.7e2f336cf4e62p+0, 0x1.05d02ba15797ep-56},
    {0x1.82589994cce13p+0, -0x1.d4c1dd41532d8p-54}, {0x1.868d99b4492edp+0, -0x1.fc6f89bd4f6bap-54},
    {0x1.8ace5422aa0dbp+0, 0x1.6e9f156864b27p-54}, {0x1.8f1ae99157736p+0, 0x1.5cc13a2e3976cp-55},
    {0x1.93737b0cdc5e5p+0, -0x1.75fc781b57ebcp-57}, {0x1.97d829fde4e50p+0, -0x1.d185b7c1b85d1p-54},
    {0x1.9c49182a3f090p+0, 0x1.c7c46b071f2bep-56}, {0x1.a0c667b5de565p+0, -0x1.359495d1cd533p-54},
    {0x1.a5503b23e255dp+0, -0x1.d2f6edb8d41e1p-54}, {0x1.a9e6b5579fdbfp+0, 0x1.0fac90ef7fd31p-54},
    {0x1.ae89f995ad3adp+0, 0x1.7a1cd345dcc81p-54}, {0x1.b33a2b84f15fbp+0, -0x1.2805e3084d708p-57},
    {0x1.b7f76f2fb5e47p+0, -0x1.5584f7e54ac3bp-56}, {0x1.bcc1e904bc1d2p+0, 0x1.23dd07a2d9e84p-55},
    {0x1.c199bdd85529cp+0, 0x1.11065895048ddp-55}, {0x1.c67f12e57d14bp+0, 0x1.2884dff483cadp-54},
    {0x1.cb720dcef9069p+0, 0x1.503cbd1e949dbp-56}, {0x1.d072d4a07897cp+0, -0x1.cbc3743797a9cp-54},
    {0x1.d5818dcfba487p+0, 0x1.2ed02d75b3707p-55}, {0x1.da9e603db3285p+0, 0x1.c2300696db532p-54},
    {0x1.dfc97337b9b5fp+0, -0x1.1a5cd4f184b5cp-54}, {0x1.e502ee78b3ff6p+0, 0x1.39e8980a9cc8fp-55},
    {0x1.ea4afa2a490dap+0, -0x1.e9c23179c2893p-54}, {0x1.efa1bee615a27p+0, 0x1.dc7f486a4b6b0p-54},
    {0x1.f50765b6e4540p+0, 0x1.9d3e12dd8a18bp-54}, {0x1.fa7c1819e90d8p+0, 0x1.74853f3a5931ep-55},
};

constexpr double kInvLn2x64 = 0x1.71547652b82fep+6;   // 64 / ln 2
constexpr double kLn2d64Hi = 0x1.62e42fefa0000p-7;    // ln 2 / 64, 36-bit head
constexpr double kLn2d64Lo = 0x1.cf79abc9e3b3ap-46;   // ln 2 / 64 - head
constexpr double kShift = 0x1.8p52;                   // round-to-integer shifter

// Reduction of x (|x| <= 700): x = k ln2/64 + r with |r| <= ln2/128;
// returns e^r - 1 (= p) and k.
__device__ __forceinline__ double reduce(double x, int& k) {
    const double t = __fma_rn(x, kInvLn2x64, kShift);
    k = __double2loint(t);
    const double kd = __dsub_rn(t, kShift);
    double r = __fma_rn(-kd, kLn2d64Hi, x);
    r = __fma_rn(-kd, kLn2d64Lo, r);
    // e^r - 1 = r + r^2 (1/2 + r (1/6 + r (1/24 + r (1/120 + r / 720))));
    // the first omitted term, r^7 / 7!, is below 2^-57 of e^r - 1 for
    // |r| <= ln2/128 (expm1 needs that relative to r, not to 1)
    double q = __fma_rn(r, 1.0 / 720.0, 1.0 / 120.0);
    q = __fma_rn(r, q, 1.0 / 24.0);
    q = __fma_rn(r, q, 1.0 / 6.0);
    q = __fma_rn(r, q, 0.5);
    return __fma_rn(__dmul_rn(r, r), q, r);
}

// v * 2^m by adding m to the exponent field: exact when v and the result
// are normal doubles
__device__ __forceinline__ double scale_pow2(double v, int m) {
    return __hiloint2double(__double2hiint(v) + (m << 20), __double2loint(v));
}

// The C library's functions for the arguments the table-driven ones leave
// to it (overflow, underflow, inf, NaN), out of line so that their code
// holds no registers in the kernels that inline the fast paths.
static __device__ __noinline__ double lib_exp(double x) { return ::exp(x); }
static __device__ __noinline__ double lib_expm1(double x) { return ::expm1(x); }

// e^x = 2^m (t + (t p + t_lo (1 + p))) with t + t_lo = 2^(j/64), k = 64 m + j;
// the bracket lies in [0.98, 2.03], and for |x| <= 700 the result is a
// normal double, so the power of two goes into the exponent field exactly
__device__ __forceinline__ double exp(double x) {
    if (!(fabs(x) <= 700.0)) return lib_exp(x);  // overflow, underflow, inf, NaN
    int k;
    const double p = reduce(x, k);
    const double2 t = __ldg(&kExp2J64HL[k & 63]);
    return scale_pow2(__dadd_rn(t.x, __fma_rn(t.x, p, __fma_rn(t.y, p, t.y))), k >> 6);
}

// e^x - 1 = (s - 1) + (s p + s_lo (1 + p)) with s + s_lo = 2^m 2^(j/64);
// s - 1 is exact, and the table tail keeps the result accurate where s - 1
// cancels (|x| below about 1).  For |x| <= 700 (the caller checks).
__device__ __forceinline__ double expm1_core(double x) {
    int k;
    const double p = reduce(x, k);
    const int m = k >> 6;  // floor(k / 64)
    const double2 t = __ldg(&kExp2J64HL[k & 63]);
    // 2^m s is a normal double for |m| <= 1010; the tail (possibly 0) is
    // scaled by a product
    const double s = scale_pow2(t.x, m);
    const double s_lo = __dmul_rn(t.y, __longlong_as_double((long long)(m + 1023) << 52));
    return __dadd_rn(__dsub_rn(s, 1.0), __fma_rn(s, p, __fma_rn(s_lo, p, s_lo)));
}

__device__ __forceinline__ double expm1(double x) {
    if (!(fabs(x) <= 700.0)) return lib_expm1(x);
    return expm1_core(x);
}

// expm1_core for x in [-40, 0] (tanh's argument), with 2^m (m >= -58)
// applied to the bracket t p + t_lo (1 + p) through the exponent field
// instead of a product with the tail: the same value, since the bracket is
// 0 only where m = 0 and otherwise stays far above the normal range's
// bottom when scaled.
__device__ __forceinline__ double expm1_tanh(double x) {
    int k;
    const double p = reduce(x, k);
    const int m = k >> 6;
    const double2 t = __ldg(&kExp2J64HL[k & 63]);
    const double s = scale_pow2(t.x, m);
    return __dadd_rn(__dsub_rn(s, 1.0), scale_pow2(__fma_rn(t.x, p, __fma_rn(t.y, p, t.y)), m));
}

// 1 / d for d in [1, 2]: the hardware's f64 reciprocal estimate (PTX
// rcp.approx.ftz.f64, from the high word: about 20 bits) refined by two
// Newton steps r <- r (2 - d r) to within an ulp or two of double.
__device__ __forceinline__ double recip_1_2(double d) {
    double r;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(d));
    r = __fma_rn(r, __fma_rn(-d, r, 1.0), r);
    r = __fma_rn(r, __fma_rn(-d, r, 1.0), r);
    return r;
}

__device__ __forceinline__ double tanh(double x) {
    const double a = fabs(x);
    if (a > 20.0) return copysign(1.0, x);
    const double e = expm1_tanh(-2.0 * a);  // in (-1, 0]; -2a >= -40
    return copysign(__dmul_rn(-e, recip_1_2(__dadd_rn(2.0, e))), x);
}

// y rounded to f32 when that rounding is certain for a value within M
// double ulps of y; `ok` false otherwise (near an f32 rounding boundary,
// f32 subnormal or out of f32 range: the caller falls back).
template <unsigned M = 64>
__device__ __forceinline__ float round_f32_checked(double y, bool& ok) {
    const unsigned ahi = (unsigned)__double2hiint(y) & 0x7fffffffu;
    const unsigned low = (unsigned)__double2loint(y) & ((1u << 29) - 1u);  // bits below f32
    // 2^-126 <= |y| < 2^128 (false for inf and NaN), as a test of the high word
    ok = ahi - 0x38100000u < 0x47f00000u - 0x38100000u &&
         (low + M - (1u << 28)) > 2u * M;  // not within M units of the midpoint 2^28
    return __double2float_rn(y);
}

// ---------------------------------------------------------------------------
// f32-argument exp, expm1, tanh and sigmoid for results that are rounded to
// f32 at once.  Only about 2^-44 relative accuracy is needed before the
// rounding check, so the core is shorter than exp above: one ln2/64 constant
// in the reduction (|k| <= 2^13 for |x| <= 104, so k * its rounding error
// stays below 2^-47), e^r - 1 to r^5 (truncation below 2^-47 relative to
// e^r - 1), the table head alone (2^-53), the power of two added to the
// exponent field, and a reciprocal from the f32 hardware estimate with one
// Newton step (tanh: the f64 estimate, one Newton step and a quotient
// correction).  Over a sweep of 2^26 f32 arguments against 64-bit long
// double references, with the f32 estimate taken one ulp off, the largest
// errors were 27 (exp), 65 (expm1), 391 (tanh, with the f32 estimate) and
// 217 (sigmoid) double ulps; results within kMarginF32 = 2048 double ulps of
// an f32 rounding boundary (about 8 in a million) go to the caller's library
// fallback.

constexpr unsigned kMarginF32 = 2048;
constexpr double kLn2d64 = 0x1.62e42fefa39efp-7;  // ln 2 / 64 rounded to double

// d = e^r - 1 (returned) and s = 2^(k/64) with x = k ln2/64 + r, for
// |x| <= 208 (the callers clamp)
__device__ __forceinline__ double reduce_short(double x, double& s) {
    const double t = __fma_rn(x, kInvLn2x64, kShift);
    const int k = __double2loint(t);
    const double kd = __dsub_rn(t, kShift);
    const double r = __fma_rn(-kd, kLn2d64, x);
    double q = __fma_rn(r, 1.0 / 120.0, 1.0 / 24.0);
    q = __fma_rn(r, q, 1.0 / 6.0);
    q = __fma_rn(r, q, 0.5);
    const double p = __fma_rn(__dmul_rn(r, r), q, r);
    const double tj = __ldg(&kExp2J64[k & 63]);
    s = __hiloint2double(__double2hiint(tj) + ((k >> 6) << 20), __double2loint(tj));
    return p;
}

__device__ __forceinline__ double recip_f32_newton(double d) {
    float rf;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rf) : "f"(__double2float_rn(d)));
    const double r = (double)rf;
    return __fma_rn(r, __fma_rn(-d, r, 1.0), r);
}

// exp(x) rounded to f32 as (float) of a double exp would round it; `ok`
// false where the caller must fall back (near a rounding boundary, f32
// overflow or subnormal results, NaN: the clamp maps those outside the
// certified range)
__device__ __forceinline__ float exp_f32(float x, bool& ok) {
    double s;
    const double p = reduce_short((double)fminf(fmaxf(x, -104.f), 104.f), s);
    return round_f32_checked<kMarginF32>(__fma_rn(s, p, s), ok);
}

// e^x - 1 = s p + (s - 1); s - 1 is exact for s in [1/2, 2] (|x| <= ln 2)
__device__ __forceinline__ float expm1_f32(float x, bool& ok) {
    double s;
    const double p = reduce_short((double)fminf(fmaxf(x, -104.f), 104.f), s);
    const float r = round_f32_checked<kMarginF32>(__fma_rn(s, p, __dsub_rn(s, 1.0)), ok);
    ok = ok && x == x;  // NaN would be clamped to -104 (-> -1)
    return r;
}

// tanh |x| = -e / (2 + e), e = expm1(-2|x|); tanh(10) already rounds to 1
// in f32, so |x| is clamped there
__device__ __forceinline__ float tanh_f32(float x, bool& ok) {
    const float ax = fminf(fabsf(x), 10.f);
    double s;
    const double p = reduce_short(-2.0 * (double)ax, s);
    const double e = __fma_rn(s, p, __dsub_rn(s, 1.0));
    const double den = __dadd_rn(2.0, e);
    // the f64 reciprocal estimate with one Newton step, then one quotient
    // correction: the quotient's error is the square of the reciprocal's
    double r;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(den));
    r = __fma_rn(r, __fma_rn(-den, r, 1.0), r);
    const double q0 = __dmul_rn(-e, r);
    const double q = __fma_rn(r, __fma_rn(-q0, den, -e), q0);
    const float v = round_f32_checked<kMarginF32>(q, ok);
    ok = ok && x == x;
    return copysignf(v, x);
}

// 1 / (1 + e^-x) for x >= -80 (clamped above at 80, where it rounds to 1)
__device__ __forceinline__ float sigmoid_f32(float x, bool& ok) {
    double s;
    const double p = reduce_short(-(double)fminf(fmaxf(x, -81.f), 80.f), s);
    const double den = __dadd_rn(1.0, __fma_rn(s, p, s));
    const float v = round_f32_checked<kMarginF32>(recip_f32_newton(den), ok);
    ok = ok && x >= -80.f;  // false for NaN too
    return v;
}

}  // namespace lean
}  // namespace nxv
