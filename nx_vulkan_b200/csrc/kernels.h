// kernels.h -- host launchers for the sm_100a kernels (internal API).
#pragma once
#include "runtime.h"

namespace nxv {

enum DType : int { F32 = 0, F64 = 1 };

// f32 elementwise transcendentals (exp log sigmoid tanh erf expm1 pow) use
// the f32 library functions by default (2-4 ulp, the precision class of the
// reference's f32 shaders).  NXV_EXACT_F32=1 evaluates them in f64 and
// rounds once, which reproduces Nx.BinaryBackend bit for bit at about half
// the throughput (B200 runs f64 at half the f32 rate).
bool fast_f32();

// Op tape for the fused elementwise kernel (lib/nx_vulkan.ex:457-538).
struct Tape {
    unsigned n_ops;
    unsigned ops[8];   // 0..9 binary, 100..114 unary, 255 nop
    unsigned src[8];   // binary operand: 0 imm, 1 b, 2 c, 3 d
    double imm[8];
};

// elementwise (k_elementwise.cu)
int launch_binary(Ctx& c, int dt, void* out, const void* a, const void* b, size_t n, unsigned op);
int launch_unary(Ctx& c, int dt, void* out, const void* a, size_t n, unsigned op);
int launch_cast(Ctx& c, int to_f64, void* out, const void* a, size_t n);
int launch_broadcast(Ctx& c, int dt, void* out, const void* a, const void* b, unsigned op,
                     unsigned ndim, const unsigned* shape, const unsigned* as, const unsigned* bs);
int launch_fused(Ctx& c, int dt, void* out, const void* a, const void* b, const void* cc,
                 const void* d, size_t n, const Tape& t);
int launch_transpose(Ctx& c, int dt, void* out, const void* a, unsigned m, unsigned n);
// transpose without the finish() check (for use inside multi-launch ops)
int enqueue_transpose(Ctx& c, int dt, void* out, const void* a, unsigned m, unsigned n);
int launch_normal_logpdf(Ctx& c, void* out, const void* x, const void* mu, const void* sigma,
                         size_t n);
int launch_leapfrog_step_f32(Ctx& c, void* qn, void* pn, const void* q, const void* p,
                             const void* m, size_t n, float eps, float mu, float sigma);

// reductions (k_reduce.cu)
// Full reduce to a device scalar of the input type.  op: 0 sum 1 min 2 max.
int launch_reduce_full(Ctx& c, int dt, void* out_dev, const void* a, size_t n, unsigned op);
// (outer, R, inner) -> (outer, inner); op: 0 sum 1 max 2 min.
int launch_reduce_axis(Ctx& c, int dt, void* out, const void* a, size_t outer, size_t R,
                       size_t inner, unsigned op);
int launch_argmax(Ctx& c, int dt, void* out, const void* a, size_t outer, size_t R,
                  size_t inner, int is_min, int index_bytes);
int launch_logsumexp(Ctx& c, void* out, const void* a, size_t outer, size_t R, size_t inner);
int launch_kinetic_energy(Ctx& c, void* out, const void* p, const void* m, size_t n);

// random (k_philox.cu)
int launch_random(Ctx& c, int dt, void* out, size_t n, uint32_t seed, unsigned dist);

// leapfrog chains (k_leapfrog.cu)
enum Family : int { FAM_NORMAL = 0, FAM_EXP = 1, FAM_STUDENTT = 2, FAM_CAUCHY = 3,
                    FAM_HALFNORMAL = 4, FAM_WEIBULL = 5 };
// f32 families; logp_mode 0: logp[chain][k]; 1: partial logp [k][group of 256]
int launch_chain_f32(Ctx& c, int fam, const float* prm, void* qc, void* pc, void* gc,
                     void* logp, const void* q0, const void* p0, const void* m, size_t n,
                     size_t chains, unsigned K, float eps, int logp_mode);
// f64 Gaussian: prec == nullptr means prec_i = prec_scalar for all i.
// ke: optional [chain][k] kinetic energy 0.5 * sum(p*p*inv_mass) per step.
// m_shared: m is one [n] row used by every chain (else [chain][n]).
// cst_dev: optional device double holding the log-density constant of prec
// (from launch_gauss_const), for callers that make many calls with one prec.
int launch_chain_gauss_f64(Ctx& c, void* qc, void* pc, void* gc, void* logp, const void* q0,
                           const void* p0, const void* m, const void* prec, double prec_scalar,
                           double mu, size_t n, size_t chains, unsigned K, double eps,
                           void* ke = nullptr, bool m_shared = false,
                           const void* cst_dev = nullptr);
// The f64 Gaussian chain's log-density constant for prec [n] into out[0].
int launch_gauss_const(Ctx& c, const void* prec, size_t n, void* out);
int launch_chain_logreg_f64(Ctx& c, void* qc, void* pc, void* gc, void* logp, const void* q0,
                            const void* p0, const void* X, const void* y, size_t n_obs,
                            size_t n_dim, size_t chains, unsigned K, double eps);

// matmul (k_matmul.cu): strided, batched or split-K GEMM parameters.
template <typename T>
struct GemmP {
    const T* A;
    const T* B;
    T* C;
    int M, N, K;
    int lda, ldb, ldc;
    long long sA, sB, sC;  // batch strides (elements); sC is also the split-K partial stride
    int ksplit;            // > 0: blockIdx.z indexes K slices of this length
    int vecA, vecB;        // set by the launcher
    int batch;             // grid.z: batch count or number of K slices
};
int gemm_f64(Ctx& c, const GemmP<double>& P);
int launch_matmul_f64(Ctx& c, void* C, const void* A, const void* B, size_t batch, size_t m,
                      size_t n, size_t k);
int launch_matmul_f32(Ctx& c, void* C, const void* A, const void* B, size_t batch, size_t m,
                      size_t n, size_t k);
// 3xTF32 on tcgen05 (k_matmul_tc.cu); the default f32 path.
int launch_matmul_f32_tc(Ctx& c, void* C, const void* A, const void* B, size_t batch, size_t m,
                         size_t n, size_t k);
// Reads and clears the tensor-core GEMM's timeout flag (1 = a bounded wait ran out).
int tc_gemm_error();
// Reads and clears the persistent logistic kernel's flag (1 = a grid barrier's
// bounded wait ran out).
int lr_traj_error();

// Stream-K schedule for 128 x 128 tiles (k_matmul.cu): tiles [0, dp) run
// data-parallel; the k-tile iterations of tiles [dp, dp + tail) are cut into
// G equal ranges (W = tail * KT iterations); tail == 0: no stream-K.  The
// fix-up adds each tail tile's partials (workspace slots of 128 x 128, two
// per range) in range order into C.
struct SkPlan {
    long long dp, tail, W;
    int G;
};
// min_idle: stream-K pays when the last wave's idle SMs add up to at least
// min_idle k-tile times per SM (its fix-up and extra launches cost about that).
bool gemm_sk_enabled();
SkPlan gemm_sk_plan(long long tiles, int KT, int sms, int min_idle);
// A, B, K: the original operands ([batch][M][K], [batch][K][N]), for the
// non-finite repair below.
int launch_gemm_fix_f32(Ctx& c, float* C, const float* A, const float* B, int M, int N, int K,
                        int batch, const SkPlan& pl, int KT, const float* ws);

#ifdef __CUDACC__
// One f32 product element as Nx.BinaryBackend defines it: the f32 operands
// widened to double, products (exact in double) summed in k order, rounded
// to f32 once.  The 3xTF32 GEMMs call it for elements whose tensor-core
// result is not finite: the split x = hi + lo turns an infinite input into
// hi = inf, lo = NaN, so every output that touches a non-finite input comes
// out non-finite (and so does an f32 accumulation that overflowed); the
// recomputation then gives inf, -inf or NaN exactly where IEEE arithmetic
// does, and the exact value where only the f32 accumulator overflowed.
static __device__ __noinline__ float exact_dot_f32(const float* __restrict__ a,
                                                  const float* __restrict__ b, int K,
                                                  long long ldb) {
    double s = 0.0;
    for (int t = 0; t < K; t++) s = __dadd_rn(s, __dmul_rn((double)a[t], (double)b[t * ldb]));
    return __double2float_rn(s);
}
#endif

// Grid helper: blocks for a grid-stride kernel.
inline unsigned grid_for(Ctx& c, size_t work_items, unsigned threads, unsigned per_sm) {
    size_t want = (work_items + threads - 1) / threads;
    size_t cap = (size_t)c.dev->sm_count * per_sm;
    if (want > cap) want = cap;
    if (want == 0) want = 1;
    return (unsigned)want;
}

}  // namespace nxv
