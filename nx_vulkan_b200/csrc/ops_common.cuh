// ops_common.cuh -- scalar op semantics shared by every kernel.
//
// Binary op codes follow lib/nx_vulkan.ex:143-154 (0 add 1 mul 2 sub 3 div
// 4 pow 5 max 6 min 7 equal 8 less 9 greater); unary op codes follow
// lib/nx_vulkan.ex:183-199 (0 exp .. 14 expm1).  The four basic operations
// use the explicit round-to-nearest intrinsics so that the compiler never
// contracts a multiply and an add into one FMA: each op rounds on its own,
// which is what Nx.BinaryBackend does (one Erlang double op per Nx op,
// rounded to the tensor type).  max/min/compare/sign/relu use the same
// branch expressions as the CPU oracle, so they agree bit for bit.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "lean_math.cuh"

namespace nxv {

__device__ __forceinline__ float add_(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul_(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float div_(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double add_(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sub_(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double mul_(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double div_(double a, double b) { return __ddiv_rn(a, b); }

__device__ __forceinline__ float exp_(float x) { return expf(x); }
__device__ __forceinline__ double exp_(double x) { return exp(x); }
__device__ __forceinline__ float log_(float x) { return logf(x); }
__device__ __forceinline__ double log_(double x) { return log(x); }
__device__ __forceinline__ float log1p_(float x) { return log1pf(x); }
__device__ __forceinline__ double log1p_(double x) { return log1p(x); }
__device__ __forceinline__ float sqrt_(float x) { return __fsqrt_rn(x); }
__device__ __forceinline__ double sqrt_(double x) { return __dsqrt_rn(x); }
__device__ __forceinline__ float tanh_(float x) { return tanhf(x); }
__device__ __forceinline__ double tanh_(double x) { return tanh(x); }
__device__ __forceinline__ float erf_(float x) { return erff(x); }
__device__ __forceinline__ double erf_(double x) { return erf(x); }
__device__ __forceinline__ float expm1_(float x) { return expm1f(x); }
__device__ __forceinline__ double expm1_(double x) { return expm1(x); }
__device__ __forceinline__ float pow_(float a, float b) { return powf(a, b); }
__device__ __forceinline__ double pow_(double a, double b) { return pow(a, b); }
__device__ __forceinline__ float ceil_(float x) { return ceilf(x); }
__device__ __forceinline__ double ceil_(double x) { return ceil(x); }
__device__ __forceinline__ float floor_(float x) { return floorf(x); }
__device__ __forceinline__ double floor_(double x) { return floor(x); }
__device__ __forceinline__ float abs_(float x) { return fabsf(x); }
__device__ __forceinline__ double abs_(double x) { return fabs(x); }

template <bool EXACT>
__device__ __forceinline__ float pow_sel(float a, float b);
template <bool EXACT>
__device__ __forceinline__ double pow_sel(double a, double b) { return pow(a, b); }

template <typename T, bool EXACT = true>
__device__ __forceinline__ T bin_op(T a, T b, unsigned op) {
    switch (op) {
        case 0: return add_(a, b);
        case 1: return mul_(a, b);
        case 2: return sub_(a, b);
        case 3: return div_(a, b);
        case 4: return pow_sel<EXACT>(a, b);
        case 5: return (a >= b) ? a : b;
        case 6: return (a <= b) ? a : b;
        case 7: return (a == b) ? T(1) : T(0);
        case 8: return (a < b) ? T(1) : T(0);
        case 9: return (a > b) ? T(1) : T(0);
        default: return a;
    }
}

// f32 transcendentals.  Nx.BinaryBackend evaluates every f32 op in double
// and rounds the result to f32 once; EXACT = true does the same on the GPU
// (f64 evaluation, one rounding), which makes f32 exp/log/tanh/sigmoid/erf/
// expm1/pow agree with the CPU oracle bit for bit except where the two
// libraries' f64 results straddle an f32 rounding boundary.  EXACT = false
// uses the f32 library functions (2-4 ulp) for throughput.
//
// In the exact mode exp, sigmoid, tanh and expm1 are evaluated with the
// short f32-argument f64 cores (lean_math.cuh: about 2^-44 relative) and
// rounded once; the library f64 function is taken instead only where that
// value lies within 2048 double ulps of an f32 rounding boundary, so the
// result is the one the library path gives.
// The library f64 function rounded to f32, out of line: it runs for about
// 8 in a million elements, and inlined its code would hold registers (and
// spill) in every kernel that evaluates the short cores.
static __device__ __noinline__ float f64_rounded(float x, unsigned op) {
    const double d = (double)x;
    switch (op) {
        case 0: return (float)exp(d);
        case 5: return (float)(1.0 / (1.0 + exp(-d)));
        case 6: return (float)tanh(d);
        default: return (float)expm1(d);
    }
}

template <bool EXACT>
__device__ __forceinline__ float tr_f32(float x, unsigned op) {
    if constexpr (EXACT) {
        bool ok;
        float r;
        switch (op) {
            case 0: r = lean::exp_f32(x, ok); break;
            case 1: return (float)log((double)x);
            case 5: r = lean::sigmoid_f32(x, ok); break;
            case 6: r = lean::tanh_f32(x, ok); break;
            case 13: return (float)erf((double)x);
            default: r = lean::expm1_f32(x, ok); break;
        }
        return ok ? r : f64_rounded(x, op);
    } else {
        switch (op) {
            case 0: return expf(x);
            case 1: return logf(x);
            case 5: return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
            case 6: return tanhf(x);
            case 13: return erff(x);
            default: return expm1f(x);
        }
    }
}

template <typename T, bool EXACT = true>
__device__ __forceinline__ T un_op(T x, unsigned op) {
    switch (op) {
        case 0:
        case 1:
        case 5:
        case 6:
        case 13:
        case 14:
            if constexpr (sizeof(T) == 4) {
                return tr_f32<EXACT>(x, op);
            } else {
                // exp, sigmoid, tanh, expm1: the table-driven f64 functions
                // (a few ulp; lean_math.cuh)
                switch (op) {
                    case 0: return lean::exp(x);
                    case 1: return log(x);
                    case 5: return div_(T(1), add_(T(1), lean::exp(-x)));
                    case 6: return lean::tanh(x);
                    case 13: return erf(x);
                    default: return lean::expm1(x);
                }
            }
        case 2: return sqrt_(x);
        case 3: return abs_(x);
        case 4: return -x;
        case 7: return (x > T(0)) ? x : T(0);
        case 8: return ceil_(x);
        case 9: return floor_(x);
        case 10: return (x > T(0)) ? T(1) : ((x < T(0)) ? T(-1) : x);
        case 11: return div_(T(1), x);
        case 12: return mul_(x, x);
        default: return x;
    }
}

// f32 pow, exact (f64 evaluation) or fast.
template <bool EXACT>
__device__ __forceinline__ float pow_sel(float a, float b) {
    if constexpr (EXACT) return (float)pow((double)a, (double)b);
    else return powf(a, b);
}

// 16-byte vector of T for coalesced 128-bit loads/stores.
template <typename T> struct Vec16;
template <> struct Vec16<float> { using type = float4; static constexpr int N = 4; };
template <> struct Vec16<double> { using type = double2; static constexpr int N = 2; };

template <typename T>
__device__ __forceinline__ void vload(const T* p, T (&r)[16 / sizeof(T)]) {
    using V = typename Vec16<T>::type;
    V v = *reinterpret_cast<const V*>(p);
    const T* s = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < (int)(16 / sizeof(T)); j++) r[j] = s[j];
}

template <typename T>
__device__ __forceinline__ void vstore(T* p, const T (&r)[16 / sizeof(T)]) {
    using V = typename Vec16<T>::type;
    V v;
    T* d = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int j = 0; j < (int)(16 / sizeof(T)); j++) d[j] = r[j];
    *reinterpret_cast<V*>(p) = v;
}

// Double-double helpers (Knuth TwoSum) for deterministic, near-exact f64 sums.
struct dd { double hi, lo; };

__device__ __forceinline__ dd dd_add_d(dd a, double b) {
    double s = __dadd_rn(a.hi, b);
    double bp = __dsub_rn(s, a.hi);
    double e = __dadd_rn(__dsub_rn(a.hi, __dsub_rn(s, bp)), __dsub_rn(b, bp));
    return dd{s, __dadd_rn(a.lo, e)};
}

__device__ __forceinline__ dd dd_add(dd a, dd b) {
    dd r = dd_add_d(a, b.hi);
    r.lo = __dadd_rn(r.lo, b.lo);
    return r;
}

__device__ __forceinline__ double dd_value(dd a) { return __dadd_rn(a.hi, a.lo); }

}  // namespace nxv
