/* oracle.c -- CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg as the checker.  The product never links it.
 *
 * Compiled with -ffp-contract=off so that every a*b+c is two roundings, as
 * in Nx.BinaryBackend (Erlang floats are doubles; no fused multiply-add).
 * Each function cites the reference file:line whose behaviour it restates.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- scalar op semantics (shared by f32 and f64 paths) ----------------- */

/* Binary op table, lib/nx_vulkan.ex:143-154.  Evaluated in double. */
static double bin_d(double a, double b, unsigned op) {
    switch (op) {
        case 0: return a + b;
        case 1: return a * b;
        case 2: return a - b;
        case 3: return a / b;
        case 4: return pow(a, b);
        case 5: return (a >= b) ? a : b;
        case 6: return (a <= b) ? a : b;
        case 7: return (a == b) ? 1.0 : 0.0;
        case 8: return (a < b) ? 1.0 : 0.0;
        case 9: return (a > b) ? 1.0 : 0.0;
        default: return NAN;
    }
}

/* Unary op table, lib/nx_vulkan.ex:183-199.  sigmoid = 1/(1+e^-x)
 * (lib/nx_vulkan/fast.ex formulas are compositions of these).  sign keeps
 * the argument for 0 and NaN; relu maps NaN and -0 to +0. */
static double un_d(double x, unsigned op) {
    switch (op) {
        case 0: return exp(x);
        case 1: return log(x);
        case 2: return sqrt(x);
        case 3: return fabs(x);
        case 4: return -x;
        case 5: return 1.0 / (1.0 + exp(-x));
        case 6: return tanh(x);
        case 7: return (x > 0.0) ? x : 0.0;
        case 8: return ceil(x);
        case 9: return floor(x);
        case 10: return (x > 0.0) ? 1.0 : ((x < 0.0) ? -1.0 : x);
        case 11: return 1.0 / x;
        case 12: return x * x;
        case 13: return erf(x);
        case 14: return expm1(x);
        default: return NAN;
    }
}

/* f32 binary: the four basic ops as IEEE single ops (== double then round);
 * everything else in double, rounded once. */
static float bin_f(float a, float b, unsigned op) {
    switch (op) {
        case 0: return a + b;
        case 1: return a * b;
        case 2: return a - b;
        case 3: return a / b;
        default: return (float)bin_d((double)a, (double)b, op);
    }
}

static float un_f(float x, unsigned op) {
    switch (op) {
        case 3: return fabsf(x);
        case 4: return -x;
        case 11: return 1.0f / x;
        case 12: return x * x;
        case 2: return sqrtf(x);
        default: return (float)un_d((double)x, op);
    }
}

void orc_binary_f32(float* out, const float* a, const float* b, size_t n, unsigned op) {
    for (size_t i = 0; i < n; i++) out[i] = bin_f(a[i], b[i], op);
}

void orc_binary_f64(double* out, const double* a, const double* b, size_t n, unsigned op) {
    for (size_t i = 0; i < n; i++) out[i] = bin_d(a[i], b[i], op);
}

void orc_unary_f32(float* out, const float* a, size_t n, unsigned op) {
    for (size_t i = 0; i < n; i++) out[i] = un_f(a[i], op);
}

void orc_unary_f64(double* out, const double* a, size_t n, unsigned op) {
    for (size_t i = 0; i < n; i++) out[i] = un_d(a[i], op);
}

/* Strided broadcast, c_src/nx_vulkan_shim.cpp:491-532: out is dense
 * row-major over shape[0..ndim); operand offsets are sum(coord_d * stride_d). */
static size_t bc_count(unsigned ndim, const unsigned* shape) {
    size_t n = 1;
    for (unsigned d = 0; d < ndim; d++) n *= shape[d];
    return n;
}

void orc_broadcast_f32(float* out, const float* a, const float* b, unsigned op, unsigned ndim,
                       const unsigned* shape, const unsigned* as, const unsigned* bs) {
    size_t n = bc_count(ndim, shape);
    for (size_t idx = 0; idx < n; idx++) {
        size_t rem = idx, oa = 0, ob = 0;
        for (int d = (int)ndim - 1; d >= 0; d--) {
            size_t c = rem % shape[d];
            rem /= shape[d];
            oa += c * as[d];
            ob += c * bs[d];
        }
        out[idx] = bin_f(a[oa], b[ob], op);
    }
}

void orc_broadcast_f64(double* out, const double* a, const double* b, unsigned op, unsigned ndim,
                       const unsigned* shape, const unsigned* as, const unsigned* bs) {
    size_t n = bc_count(ndim, shape);
    for (size_t idx = 0; idx < n; idx++) {
        size_t rem = idx, oa = 0, ob = 0;
        for (int d = (int)ndim - 1; d >= 0; d--) {
            size_t c = rem % shape[d];
            rem /= shape[d];
            oa += c * as[d];
            ob += c * bs[d];
        }
        out[idx] = bin_d(a[oa], b[ob], op);
    }
}

/* Op tape, lib/nx_vulkan.ex:457-538 and c_src/nx_vulkan_shim.h:148-167:
 * the register starts at a[i]; ops apply left to right; 255 is a nop. */
static float fused_one_f32(size_t i, const float* a, const float* const* srcs, unsigned n_ops,
                           const unsigned* ops, const unsigned* src, const double* imm) {
    float r = a[i];
    for (unsigned k = 0; k < n_ops; k++) {
        unsigned op = ops[k];
        if (op == 255) continue;
        if (op < 100) {
            unsigned s = src ? src[k] : 1;
            float rhs = (s == 0) ? (float)imm[k] : srcs[s - 1][i];
            r = bin_f(r, rhs, op);
        } else {
            r = un_f(r, op - 100);
        }
    }
    return r;
}

void orc_fused_f32(float* out, const float* a, const float* b, const float* c, const float* d,
                   size_t n, unsigned n_ops, const unsigned* ops, const unsigned* src,
                   const double* imm) {
    const float* srcs[3] = {b, c, d};
    for (size_t i = 0; i < n; i++) out[i] = fused_one_f32(i, a, srcs, n_ops, ops, src, imm);
}

void orc_fused_f32_mt(float* out, const float* a, const float* b, const float* c,
                      const float* d, size_t n, unsigned n_ops, const unsigned* ops,
                      const unsigned* src, const double* imm, int nthreads) {
    const float* srcs[3] = {b, c, d};
    (void)nthreads;
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (long long i = 0; i < (long long)n; i++)
        out[i] = fused_one_f32((size_t)i, a, srcs, n_ops, ops, src, imm);
}

void orc_fused_f64(double* out, const double* a, const double* b, const double* c,
                   const double* d, size_t n, unsigned n_ops, const unsigned* ops,
                   const unsigned* src, const double* imm) {
    const double* srcs[3] = {b, c, d};
    for (size_t i = 0; i < n; i++) {
        double r = a[i];
        for (unsigned k = 0; k < n_ops; k++) {
            unsigned op = ops[k];
            if (op == 255) continue;
            if (op < 100) {
                unsigned s = src ? src[k] : 1;
                double rhs = (s == 0) ? imm[k] : srcs[s - 1][i];
                r = bin_d(r, rhs, op);
            } else {
                r = un_d(r, op - 100);
            }
        }
        out[i] = r;
    }
}

void orc_cast_f32_f64(double* out, const float* a, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = (double)a[i];
}

void orc_cast_f64_f32(float* out, const double* a, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = (float)a[i];
}

/* c_src/nx_vulkan_shim.h:116-120: C[j, i] = A[i, j]. */
void orc_transpose_f32(float* out, const float* a, unsigned m, unsigned n) {
    for (unsigned i = 0; i < m; i++)
        for (unsigned j = 0; j < n; j++) out[(size_t)j * m + i] = a[(size_t)i * n + j];
}

/* ---- reductions --------------------------------------------------------- */

/* Full reduce, op 0 sum 1 min 2 max (lib/nx_vulkan.ex:256-263).  Sequential
 * left fold in double; NaN propagates through sum and wins min/max. */
static double fold_d(double acc, double x, unsigned op) {
    if (op == 0) return acc + x;
    if (isnan(acc) || isnan(x)) return NAN;
    if (op == 1) return (x < acc) ? x : acc;
    return (x > acc) ? x : acc;
}

double orc_reduce_full_f32(const float* a, size_t n, unsigned op) {
    double acc = (op == 0) ? 0.0 : ((op == 1) ? INFINITY : -INFINITY);
    for (size_t i = 0; i < n; i++) acc = fold_d(acc, (double)a[i], op);
    return (double)(float)acc;
}

double orc_reduce_full_f64(const double* a, size_t n, unsigned op) {
    double acc = (op == 0) ? 0.0 : ((op == 1) ? INFINITY : -INFINITY);
    for (size_t i = 0; i < n; i++) acc = fold_d(acc, a[i], op);
    return acc;
}

/* Double-double accumulation (Knuth TwoSum); error ~ eps^2 * sum|x|. */
double orc_sum_exact_f64(const double* a, size_t n) {
    double s = 0.0, c = 0.0;
    for (size_t i = 0; i < n; i++) {
        double x = a[i];
        double t = s + x;
        double bp = t - s;
        double err = (s - (t - bp)) + (x - bp);
        s = t;
        c += err;
    }
    return s + c;
}

double orc_sum_abs_f64(const double* a, size_t n) {
    double s = 0.0;
    for (size_t i = 0; i < n; i++) s += fabs(a[i]);
    return s;
}

/* Per-axis reduce: op 0 sum 1 max 2 min (c_src/nx_vulkan_shim.h:129-134;
 * note the max/min order is the reverse of the full reduce). */
static unsigned axis_to_full_op(unsigned op) { return op == 0 ? 0 : (op == 1 ? 2 : 1); }

void orc_reduce_axis_f32(float* out, const float* a, size_t outer, size_t R, size_t inner,
                         unsigned op) {
    unsigned fop = axis_to_full_op(op);
    for (size_t o = 0; o < outer; o++)
        for (size_t j = 0; j < inner; j++) {
            double acc = (fop == 0) ? 0.0 : ((fop == 1) ? INFINITY : -INFINITY);
            for (size_t r = 0; r < R; r++) acc = fold_d(acc, (double)a[(o * R + r) * inner + j], fop);
            out[o * inner + j] = (float)acc;
        }
}

void orc_reduce_axis_f64(double* out, const double* a, size_t outer, size_t R, size_t inner,
                         unsigned op) {
    unsigned fop = axis_to_full_op(op);
    for (size_t o = 0; o < outer; o++)
        for (size_t j = 0; j < inner; j++) {
            double acc = (fop == 0) ? 0.0 : ((fop == 1) ? INFINITY : -INFINITY);
            for (size_t r = 0; r < R; r++) acc = fold_d(acc, a[(o * R + r) * inner + j], fop);
            out[o * inner + j] = acc;
        }
}

/* argmax/argmin with Nx's default tie_break: :low (lowest index wins).
 * A NaN beats every number; the first NaN wins. */
#define ARGMAX_BODY(T)                                                              \
    for (size_t o = 0; o < outer; o++)                                              \
        for (size_t j = 0; j < inner; j++) {                                        \
            size_t best = 0;                                                        \
            T bv = a[(o * R) * inner + j];                                          \
            for (size_t r = 1; r < R; r++) {                                        \
                T v = a[(o * R + r) * inner + j];                                   \
                if (isnan(bv)) break;                                               \
                int better = isnan(v) || (is_min ? (v < bv) : (v > bv));            \
                if (better) { bv = v; best = r; }                                   \
            }                                                                       \
            out[o * inner + j] = (int64_t)best;                                     \
        }

void orc_argmax_axis_f32(int64_t* out, const float* a, size_t outer, size_t R, size_t inner,
                         int is_min) {
    ARGMAX_BODY(float)
}

void orc_argmax_axis_f64(int64_t* out, const double* a, size_t outer, size_t R, size_t inner,
                         int is_min) {
    ARGMAX_BODY(double)
}

/* Two-pass stable logsumexp over R (lib/nx_vulkan.ex:242-250), in double. */
void orc_logsumexp_f32(float* out, const float* a, size_t outer, size_t R, size_t inner) {
    for (size_t o = 0; o < outer; o++)
        for (size_t j = 0; j < inner; j++) {
            double mx = -INFINITY;
            for (size_t r = 0; r < R; r++) {
                double v = a[(o * R + r) * inner + j];
                if (v > mx) mx = v;
            }
            double s = 0.0;
            for (size_t r = 0; r < R; r++) s += exp((double)a[(o * R + r) * inner + j] - mx);
            out[o * inner + j] = (float)(log(s) + mx);
        }
}

/* ---- dot ------------------------------------------------------------------ */

/* C = A.B row-major, double accumulation in k order (Nx.dot on BinaryBackend;
 * c_src/nx_vulkan_shim.h:94-97). */
void orc_matmul_f32(float* c, const float* a, const float* b, size_t m, size_t n, size_t k) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; i++)
        for (size_t j = 0; j < n; j++) {
            double acc = 0.0;
            for (size_t t = 0; t < k; t++) acc += (double)a[i * k + t] * (double)b[t * n + j];
            c[i * n + j] = (float)acc;
        }
}

void orc_matmul_f64(double* c, const double* a, const double* b, size_t m, size_t n, size_t k) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; i++)
        for (size_t j = 0; j < n; j++) {
            double acc = 0.0;
            for (size_t t = 0; t < k; t++) acc += a[i * k + t] * b[t * n + j];
            c[i * n + j] = acc;
        }
}

void orc_matmul_batched_f64(double* c, const double* a, const double* b, size_t batch,
                            size_t m, size_t n, size_t k) {
    for (size_t q = 0; q < batch; q++)
        orc_matmul_f64(c + q * m * n, a + q * m * k, b + q * k * n, m, n, k);
}

void orc_matmul_batched_f32(float* c, const float* a, const float* b, size_t batch,
                            size_t m, size_t n, size_t k) {
    for (size_t q = 0; q < batch; q++)
        orc_matmul_f32(c + q * m * n, a + q * m * k, b + q * k * n, m, n, k);
}

/* ---- Philox-2x32-10 -------------------------------------------------------
 * The reference states it runs canonical Random123 Philox 2x32-10
 * (PLAN_FUSED_LEAPFROG.md:27-29); its counter layout is not in source.
 * Published algorithm (Salmon, Moraes, Dror, Shaw, SC'11): per round
 * (hi, lo) = mulhilo(0xD256D193, x0); x0' = hi ^ key ^ x1; x1' = lo; the key
 * is bumped by the Weyl constant 0x9E3779B9 between rounds.
 *
 * The library's documented mapping (the contract the GPU kernel must match):
 *   f32 uniform:  element i <- word (i & 1) of philox(ctr = (i >> 1, 0), key = seed);
 *                 u = (w >> 8) * 2^-24 in [0, 1).
 *   f32 normal:   elements 2c, 2c+1 <- both words of philox((c, 0), seed):
 *                 u1 = ((w0 >> 8) + 1) * 2^-24 in (0, 1], u2 = (w1 >> 8) * 2^-24,
 *                 r = sqrt(-2 ln u1), out = (r cos 2 pi u2, r sin 2 pi u2),
 *                 evaluated in double and rounded to f32.
 *   f64 uniform:  element i <- philox((i, 1), seed): u = (((w0 << 32) | w1) >> 11) * 2^-53.
 *   f64 normal:   pair c <- u1 from philox((2c, 1)) shifted to (0, 1], u2 from
 *                 philox((2c + 1, 1)); Box-Muller in double.
 */
void orc_philox2x32(uint32_t x0, uint32_t x1, uint32_t key, uint32_t* out0, uint32_t* out1) {
    for (int r = 0; r < 10; r++) {
        uint64_t prod = (uint64_t)0xD256D193u * (uint64_t)x0;
        uint32_t hi = (uint32_t)(prod >> 32), lo = (uint32_t)prod;
        x0 = hi ^ key ^ x1;
        x1 = lo;
        key += 0x9E3779B9u;
    }
    *out0 = x0;
    *out1 = x1;
}

static const double TWO_PI = 6.283185307179586476925286766559;

void orc_random_f32(float* out, size_t n, uint32_t seed, unsigned dist) {
    for (size_t c = 0; 2 * c < n; c++) {
        uint32_t w0, w1;
        orc_philox2x32((uint32_t)c, 0u, seed, &w0, &w1);
        float v0, v1;
        if (dist == 0) {
            v0 = (float)(w0 >> 8) * 0x1.0p-24f;
            v1 = (float)(w1 >> 8) * 0x1.0p-24f;
        } else {
            double u1 = ((double)(w0 >> 8) + 1.0) * 0x1.0p-24;
            double u2 = (double)(w1 >> 8) * 0x1.0p-24;
            double r = sqrt(-2.0 * log(u1));
            v0 = (float)(r * cos(TWO_PI * u2));
            v1 = (float)(r * sin(TWO_PI * u2));
        }
        out[2 * c] = v0;
        if (2 * c + 1 < n) out[2 * c + 1] = v1;
    }
}

static double u53(uint32_t i, uint32_t seed) {
    uint32_t w0, w1;
    orc_philox2x32(i, 1u, seed, &w0, &w1);
    uint64_t v = (((uint64_t)w0 << 32) | w1) >> 11;
    return (double)v * 0x1.0p-53;
}

void orc_random_f64(double* out, size_t n, uint32_t seed, unsigned dist) {
    if (dist == 0) {
        for (size_t i = 0; i < n; i++) out[i] = u53((uint32_t)i, seed);
        return;
    }
    for (size_t c = 0; 2 * c < n; c++) {
        double u1 = u53((uint32_t)(2 * c), seed) + 0x1.0p-53;
        double u2 = u53((uint32_t)(2 * c + 1), seed);
        double r = sqrt(-2.0 * log(u1));
        out[2 * c] = r * cos(TWO_PI * u2);
        if (2 * c + 1 < n) out[2 * c + 1] = r * sin(TWO_PI * u2);
    }
}

/* ---- fused HMC helpers ----------------------------------------------------- */

/* kinetic_energy.spv: 0.5 * sum(p^2 * inv_mass) (c_src/nx_vulkan_shim.h:169-173;
 * fallback formula lib/nx_vulkan/fast.ex:117-123). */
double orc_kinetic_energy_f32(const float* p, const float* m, size_t n) {
    double s = 0.0;
    for (size_t i = 0; i < n; i++) s += (double)((p[i] * p[i]) * m[i]);
    return (double)(float)(0.5 * s);
}

/* normal_logpdf.spv: -0.5 z^2 - log sigma - 0.5 log 2pi with z = (x-mu)/sigma
 * (lib/nx_vulkan/fast.ex:147-161 gives the op order). */
void orc_normal_logpdf_f32(float* out, const float* x, const float* mu, const float* sigma,
                           size_t n) {
    const float log_sqrt_2pi = (float)0.91893853320467274178;
    for (size_t i = 0; i < n; i++) {
        float z = (x[i] - mu[i]) / sigma[i];
        float z2 = z * z;
        float ls = (float)log((double)sigma[i]);
        out[i] = ((z2 * -0.5f) - ls) - log_sqrt_2pi;
    }
}

/* leapfrog_normal.spv single step (c_src/nx_vulkan_shim.h:181-189) with the
 * corrected sign p + eps/2 * grad logp (PLAN_FUSED_LEAPFROG.md:18-24). */
void orc_leapfrog_normal_step_f32(float* q_new, float* p_new, const float* q, const float* p,
                                  const float* m, size_t n, float eps, float mu, float sigma) {
    float inv_var = 1.0f / (sigma * sigma);
    float he = 0.5f * eps;
    for (size_t i = 0; i < n; i++) {
        float g = -((q[i] - mu) * inv_var);
        float ph = p[i] + he * g;
        float qn = q[i] + (eps * m[i]) * ph;
        float gn = -((qn - mu) * inv_var);
        q_new[i] = qn;
        p_new[i] = ph + he * gn;
    }
}

/* Family gradient and per-element log-density term on the unconstrained line
 * (lib/nx_vulkan.ex:632-726; c_src/nx_vulkan_shim.h:218-270).  The logp of a
 * step is  cst + sum_i term(q_i)  summed in double and rounded to f32:
 *   normal:      g = -(q-mu)*inv_var,  term = z*z with z=(q-mu)/sigma,
 *                logp = -0.5*sum - n*(log sigma + 0.5 log 2pi)
 *   exponential: g = 1 - lambda*e^q,   term = q - lambda*e^q, cst = n log lambda
 *   studentt:    g = -(nu+1)*d/(nu*sigma^2 + d^2), d = q-mu,
 *                term = logp_const - (nu+1)/2 * log(1 + (d/sigma)^2/nu)
 *   cauchy:      g = -2 d/(scale^2 + d^2), d = q-loc,
 *                term = log_pi_scale - log(1 + (d/scale)^2)
 *   halfnormal:  g = 1 - e^{2q}/sigma^2, term = log_const + q - e^{2q}/(2 sigma^2)
 *   weibull:     g = k*(1 - (e^q/lambda)^k), term = k q - (e^q/lambda)^k,
 *                cst = logp_const (already n*(log k - k log lambda)).
 * Transcendentals are evaluated in double and rounded to f32. */
static float fam_grad(int fam, const float* prm, float q, float inv_var) {
    switch (fam) {
        case 0: return -((q - prm[0]) * inv_var);
        case 1: return 1.0f - prm[0] * (float)exp((double)q);
        case 2: {
            float d = q - prm[0];
            return -(((prm[2] + 1.0f) * d) / ((prm[2] * (prm[1] * prm[1])) + d * d));
        }
        case 3: {
            float d = q - prm[0];
            return -((2.0f * d) / ((prm[1] * prm[1]) + d * d));
        }
        case 4: return 1.0f - ((float)exp((double)(2.0f * q)) / (prm[0] * prm[0]));
        case 5: {
            float r = (float)pow((double)((float)exp((double)q) / prm[1]), (double)prm[0]);
            return prm[0] * (1.0f - r);
        }
    }
    return NAN;
}

static double fam_term(int fam, const float* prm, float q) {
    switch (fam) {
        case 0: {
            float z = (q - prm[0]) / prm[1];
            return (double)(z * z);
        }
        case 1: return (double)(q - prm[0] * (float)exp((double)q));
        case 2: {
            float z = (q - prm[0]) / prm[1];
            float l = (float)log1p((double)((z * z) / prm[2]));
            return (double)(prm[3] - ((prm[2] + 1.0f) * 0.5f) * l);
        }
        case 3: {
            float z = (q - prm[0]) / prm[1];
            return (double)(prm[2] - (float)log1p((double)(z * z)));
        }
        case 4: {
            float e2 = (float)exp((double)(2.0f * q));
            return (double)((prm[1] + q) - e2 / (2.0f * (prm[0] * prm[0])));
        }
        case 5: {
            float r = (float)pow((double)((float)exp((double)q) / prm[1]), (double)prm[0]);
            return (double)(prm[0] * q - r);
        }
    }
    return NAN;
}

static double fam_logp(int fam, const float* prm, double sum, size_t n) {
    switch (fam) {
        case 0:
            return -0.5 * sum - (double)n * (log((double)prm[1]) + 0.91893853320467274178);
        case 1: return sum + (double)n * log((double)prm[0]);
        case 5: return sum + (double)prm[2];
        default: return sum;
    }
}

void orc_leapfrog_chain_f32(int fam, const float* prm, float* q_chain, float* p_chain,
                            float* g_chain, float* logp, const float* q0, const float* p0,
                            const float* m, size_t n, size_t chains, unsigned K, float eps) {
    float inv_var = (fam == 0) ? 1.0f / (prm[1] * prm[1]) : 0.0f;
    float he = 0.5f * eps;
    float* q = (float*)malloc(n * sizeof(float));
    float* p = (float*)malloc(n * sizeof(float));
    float* g = (float*)malloc(n * sizeof(float));
    for (size_t c = 0; c < chains; c++) {
        const float* mc = m + c * n;
        for (size_t i = 0; i < n; i++) {
            q[i] = q0[c * n + i];
            p[i] = p0[c * n + i];
            g[i] = fam_grad(fam, prm, q[i], inv_var);
        }
        for (unsigned k = 0; k < K; k++) {
            size_t row = (c * K + k) * n;
            double s = 0.0;
            for (size_t i = 0; i < n; i++) {
                float ph = p[i] + he * g[i];
                q[i] = q[i] + (eps * mc[i]) * ph;
                g[i] = fam_grad(fam, prm, q[i], inv_var);
                p[i] = ph + he * g[i];
                q_chain[row + i] = q[i];
                p_chain[row + i] = p[i];
                g_chain[row + i] = g[i];
                s += fam_term(fam, prm, q[i]);
            }
            logp[c * K + k] = (float)fam_logp(fam, prm, s, n);
        }
    }
    free(q);
    free(p);
    free(g);
}

/* f64 Gaussian chain (c_src/nx_vulkan_shim.h:272-280 generalised to a
 * precision vector and a chain batch).  Op order per element and step:
 *   ph = p + he*g;  q = q + (eps*m)*ph;  g = -(prec*(q-mu));  p = ph + he*g
 * logp_k = -0.5 * sum_i prec_i (q_i-mu)^2 + 0.5 sum_i log prec_i - n/2 log 2pi. */
void orc_leapfrog_gauss_f64(double* q_chain, double* p_chain, double* g_chain, double* logp,
                            const double* q0, const double* p0, const double* m,
                            const double* prec, double mu, size_t n, size_t chains,
                            unsigned K, double eps, int nthreads) {
    double he = 0.5 * eps;
    double cst = 0.0;
    for (size_t i = 0; i < n; i++) cst += log(prec[i]);
    cst = 0.5 * cst - (double)n * 0.91893853320467274178;
    (void)nthreads;
#pragma omp parallel num_threads(nthreads)
    {
        double* q = (double*)malloc(n * sizeof(double));
        double* p = (double*)malloc(n * sizeof(double));
        double* g = (double*)malloc(n * sizeof(double));
#pragma omp for schedule(static)
        for (long long cc = 0; cc < (long long)chains; cc++) {
            size_t c = (size_t)cc;
            const double* mc = m + c * n;
            for (size_t i = 0; i < n; i++) {
                q[i] = q0[c * n + i];
                p[i] = p0[c * n + i];
                g[i] = -(prec[i] * (q[i] - mu));
            }
            for (unsigned k = 0; k < K; k++) {
                size_t row = (c * K + k) * n;
                double s = 0.0;
                for (size_t i = 0; i < n; i++) {
                    double ph = p[i] + he * g[i];
                    q[i] = q[i] + (eps * mc[i]) * ph;
                    double d = q[i] - mu;
                    g[i] = -(prec[i] * d);
                    p[i] = ph + he * g[i];
                    q_chain[row + i] = q[i];
                    p_chain[row + i] = p[i];
                    g_chain[row + i] = g[i];
                    s += (prec[i] * d) * d;
                }
                logp[c * K + k] = -0.5 * s + cst;
            }
        }
        free(q);
        free(p);
        free(g);
    }
}

/* Logistic regression chain.  z = X q (double accumulation over the n_dim
 * features in order), r_j = y_j - sigmoid(z_j), grad_i = sum_j X_ji r_j - q_i
 * (sum over observations in order), logp = sum_j [y_j z_j - log1p(e^{z_j})]
 * - 0.5 sum_i q_i^2 (log1p(e^z) evaluated as max(z,0) + log1p(e^{-|z|})). */
static void logreg_grad(double* g, double* lp, const double* q, const double* X,
                        const double* y, size_t n_obs, size_t n_dim, double* r) {
    double l = 0.0;
    for (size_t j = 0; j < n_obs; j++) {
        double z = 0.0;
        for (size_t i = 0; i < n_dim; i++) z += X[j * n_dim + i] * q[i];
        double s = 1.0 / (1.0 + exp(-z));
        r[j] = y[j] - s;
        double sp = (z > 0.0 ? z : 0.0) + log1p(exp(-fabs(z)));
        l += y[j] * z - sp;
    }
    double qq = 0.0;
    for (size_t i = 0; i < n_dim; i++) {
        double acc = 0.0;
        for (size_t j = 0; j < n_obs; j++) acc += X[j * n_dim + i] * r[j];
        g[i] = acc - q[i];
        qq += q[i] * q[i];
    }
    *lp = l - 0.5 * qq;
}

void orc_leapfrog_logreg_f64(double* q_chain, double* p_chain, double* g_chain, double* logp,
                             const double* q0, const double* p0, const double* X,
                             const double* y, size_t n_obs, size_t n_dim, size_t chains,
                             unsigned K, double eps, int nthreads) {
    double he = 0.5 * eps;
    (void)nthreads;
#pragma omp parallel num_threads(nthreads)
    {
        double* q = (double*)malloc(n_dim * sizeof(double));
        double* p = (double*)malloc(n_dim * sizeof(double));
        double* g = (double*)malloc(n_dim * sizeof(double));
        double* r = (double*)malloc(n_obs * sizeof(double));
#pragma omp for schedule(static)
        for (long long cc = 0; cc < (long long)chains; cc++) {
            size_t c = (size_t)cc;
            double lp;
            for (size_t i = 0; i < n_dim; i++) {
                q[i] = q0[c * n_dim + i];
                p[i] = p0[c * n_dim + i];
            }
            logreg_grad(g, &lp, q, X, y, n_obs, n_dim, r);
            for (unsigned k = 0; k < K; k++) {
                size_t row = (c * K + k) * n_dim;
                for (size_t i = 0; i < n_dim; i++) {
                    double ph = p[i] + he * g[i];
                    q[i] = q[i] + eps * ph;
                    p[i] = ph;
                }
                logreg_grad(g, &lp, q, X, y, n_obs, n_dim, r);
                for (size_t i = 0; i < n_dim; i++) {
                    p[i] = p[i] + he * g[i];
                    q_chain[row + i] = q[i];
                    p_chain[row + i] = p[i];
                    g_chain[row + i] = g[i];
                }
                logp[c * K + k] = lp;
            }
        }
        free(q);
        free(p);
        free(g);
        free(r);
    }
}
