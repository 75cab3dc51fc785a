/* oracle.h -- CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * library (libnxv_b200.so): only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load it.  Nothing in the product links it.
 *
 * What it restates: Nx.BinaryBackend semantics as used by the nx_vulkan
 * reference for its hot path (elementwise chains, broadcast, reductions,
 * argmax, dot, Philox, the fused HMC leapfrog chains):
 *   - f32 ops are evaluated as IEEE single operations, which equals
 *     "compute in double, round to f32 after every op" for + - * / sqrt
 *     (double has >= 2*24+2 bits, so the double rounding is innocuous);
 *     transcendentals are computed in double and rounded once.
 *   - f64 ops are plain IEEE double, no FMA contraction (-ffp-contract=off).
 *   - reductions are sequential left folds in double; f32 results are
 *     rounded once at the end.  max/min/argmax keep the lowest index on ties.
 *   - dot accumulates in double in k order and rounds to the output type.
 *
 * Parity pin: every known-answer value of the reference's test suite for
 * this path (test/nx_vulkan_test.exs) and the Weibull chain KAT from the
 * reference docs (248_TODO.md:52-53) are checked against this library by
 * tests/test_oracle_golden.py.  The Philox bit stream is "parity unpinned"
 * (the reference's counter layout lives only in a closed SPIR-V binary);
 * this library's own documented Philox-2x32-10 mapping is the contract.
 */
#ifndef NXV_ORACLE_H
#define NXV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Elementwise ---------------------------------------------------------- */
/* binary op codes (lib/nx_vulkan.ex:143-154): 0 add 1 mul 2 sub 3 div 4 pow
 * 5 max 6 min 7 equal 8 less 9 greater (comparisons give 1.0 / 0.0). */
void orc_binary_f32(float* out, const float* a, const float* b, size_t n, unsigned op);
void orc_binary_f64(double* out, const double* a, const double* b, size_t n, unsigned op);
/* unary op codes (lib/nx_vulkan.ex:183-199): 0 exp 1 log 2 sqrt 3 abs 4 neg
 * 5 sigmoid 6 tanh 7 relu 8 ceil 9 floor 10 sign 11 reciprocal 12 square
 * 13 erf 14 expm1. */
void orc_unary_f32(float* out, const float* a, size_t n, unsigned op);
void orc_unary_f64(double* out, const double* a, size_t n, unsigned op);
/* out[idx] = a[sum c_d*sa_d] op b[sum c_d*sb_d], ndim <= 4, stride 0 broadcasts
 * (c_src/nx_vulkan_shim.cpp:491-532, lib/nx_vulkan.ex:808-835). */
void orc_broadcast_f32(float* out, const float* a, const float* b, unsigned op, unsigned ndim,
                       const unsigned* shape, const unsigned* as, const unsigned* bs);
void orc_broadcast_f64(double* out, const double* a, const double* b, unsigned op, unsigned ndim,
                       const unsigned* shape, const unsigned* as, const unsigned* bs);
/* Op tape (lib/nx_vulkan.ex:457-538): r = a[i]; for k < n_ops: binary ops
 * 0..9 combine r with operand src[k]; unary 100..114 transform r; 255 nop.
 * src[k]: 0 = immediate scalar imm[k] (rounded to the chain type),
 * 1 = b, 2 = c, 3 = d.  Each op's result is rounded to the chain type. */
void orc_fused_f32(float* out, const float* a, const float* b, const float* c, const float* d,
                   size_t n, unsigned n_ops, const unsigned* ops, const unsigned* src,
                   const double* imm);
void orc_fused_f64(double* out, const double* a, const double* b, const double* c,
                   const double* d, size_t n, unsigned n_ops, const unsigned* ops,
                   const unsigned* src, const double* imm);
void orc_cast_f32_f64(double* out, const float* a, size_t n);
void orc_cast_f64_f32(float* out, const double* a, size_t n);
void orc_transpose_f32(float* out, const float* a, unsigned m, unsigned n);

/* Reductions ----------------------------------------------------------- */
/* Full reduce, nxv_reduce op codes: 0 sum 1 min 2 max
 * (lib/nx_vulkan.ex:256-263). f32: returns the f32-rounded value. */
double orc_reduce_full_f32(const float* a, size_t n, unsigned op);
double orc_reduce_full_f64(const double* a, size_t n, unsigned op);
/* Compensated (double-double) sum: the arbiter for f64 sum disagreements. */
double orc_sum_exact_f64(const double* a, size_t n);
double orc_sum_abs_f64(const double* a, size_t n);
/* Per-axis reduce (outer, R, inner) -> (outer, inner); op 0 sum 1 max 2 min
 * (c_src/nx_vulkan_shim.h:129-134). */
void orc_reduce_axis_f32(float* out, const float* a, size_t outer, size_t R, size_t inner,
                         unsigned op);
void orc_reduce_axis_f64(double* out, const double* a, size_t outer, size_t R, size_t inner,
                         unsigned op);
/* argmax (is_min = 0) / argmin (is_min = 1) over R; lowest index on ties;
 * a NaN counts as larger (argmax) / smaller (argmin) than any number and
 * the first NaN wins. */
void orc_argmax_axis_f32(int64_t* out, const float* a, size_t outer, size_t R, size_t inner,
                         int is_min);
void orc_argmax_axis_f64(int64_t* out, const double* a, size_t outer, size_t R, size_t inner,
                         int is_min);
/* log(sum(exp(x - max))) + max over R (lib/nx_vulkan.ex:242-250). */
void orc_logsumexp_f32(float* out, const float* a, size_t outer, size_t R, size_t inner);

/* Dot ------------------------------------------------------------------ */
void orc_matmul_f32(float* c, const float* a, const float* b, size_t m, size_t n, size_t k);
void orc_matmul_f64(double* c, const double* a, const double* b, size_t m, size_t n, size_t k);
void orc_matmul_batched_f64(double* c, const double* a, const double* b, size_t batch,
                            size_t m, size_t n, size_t k);
void orc_matmul_batched_f32(float* c, const float* a, const float* b, size_t batch,
                            size_t m, size_t n, size_t k);

/* Philox-2x32-10 (Salmon et al., SC'11).  Mapping: element i uses counter
 * (ctr0 = i >> 1 ... see oracle.c) -- documented in orc_philox_f32. */
void orc_philox2x32(uint32_t ctr0, uint32_t ctr1, uint32_t key, uint32_t* out0, uint32_t* out1);
void orc_random_f32(float* out, size_t n, uint32_t seed, unsigned dist);
void orc_random_f64(double* out, size_t n, uint32_t seed, unsigned dist);

/* Fused HMC helpers ----------------------------------------------------- */
/* 0.5 * sum(p^2 * inv_mass), double accumulation, f32 result. */
double orc_kinetic_energy_f32(const float* p, const float* m, size_t n);
void orc_normal_logpdf_f32(float* out, const float* x, const float* mu, const float* sigma,
                           size_t n);
void orc_leapfrog_normal_step_f32(float* q_new, float* p_new, const float* q, const float* p,
                                  const float* m, size_t n, float eps, float mu, float sigma);

/* Leapfrog chain families (f32), layout [chain][k][i], logp [chain][k].
 * family: 0 normal(mu, sigma) 1 exponential(lambda) 2 studentt(mu, sigma, nu,
 * logp_const) 3 cauchy(loc, scale, log_pi_scale) 4 halfnormal(sigma, log_const)
 * 5 weibull(k, lambda, logp_const).  prm holds the family scalars in that
 * order.  (c_src/nx_vulkan_shim.h:191-270, lib/nx_vulkan.ex:582-726.) */
void orc_leapfrog_chain_f32(int family, const float* prm, float* q_chain, float* p_chain,
                            float* g_chain, float* logp, const float* q0, const float* p0,
                            const float* m, size_t n, size_t chains, unsigned K, float eps);
/* f64 Gaussian chain: grad = -prec .* (q - mu); logp = -0.5 sum prec (q-mu)^2
 * + 0.5 sum log prec - n/2 log(2 pi).  The reference's Normal(mu, sigma) f64
 * chain is prec = 1/sigma^2 (c_src/nx_vulkan_shim.h:272-280).  m is
 * [chains][n]; prec is [n] shared by every chain. */
void orc_leapfrog_gauss_f64(double* q_chain, double* p_chain, double* g_chain, double* logp,
                            const double* q0, const double* p0, const double* m,
                            const double* prec, double mu, size_t n, size_t chains,
                            unsigned K, double eps, int nthreads);
/* Bayesian logistic regression chain, layout as above, m = 1:
 * grad(q) = X^T (y - sigmoid(X q)) - q,
 * logp(q) = sum_j [y_j z_j - log(1 + e^{z_j})] - 0.5 |q|^2,  z = X q. */
void orc_leapfrog_logreg_f64(double* q_chain, double* p_chain, double* g_chain, double* logp,
                             const double* q0, const double* p0, const double* X,
                             const double* y, size_t n_obs, size_t n_dim, size_t chains,
                             unsigned K, double eps, int nthreads);

/* Multi-threaded fused chain for the CPU baseline (same per-element math). */
void orc_fused_f32_mt(float* out, const float* a, const float* b, const float* c,
                      const float* d, size_t n, unsigned n_ops, const unsigned* ops,
                      const unsigned* src, const double* imm, int nthreads);
int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
