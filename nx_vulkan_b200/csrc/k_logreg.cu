// k_logreg.cu -- batched HMC leapfrog for Bayesian logistic regression (f64).
//
// Target (the second leapfrog workload; no reference kernel exists -- the
// reference would run it through the unfused evaluator with dot on the host):
//   z = X q,  r = y - sigmoid(z),  grad(q) = X^T r - q,
//   logp(q) = sum_j [y_j z_j - softplus(z_j)] - 0.5 |q|^2,
// batched over C chains: Z = Q . X^T (C x N_obs, K = D) and G = R . X - Q
// (C x D, K = N_obs).  Both products run on the f64 DMMA GEMM; the second is
// split along N_obs into S slices whose partials are folded in slice order
// (deterministic).  The leapfrog update is fused into that fold.
// Per step: drift (1 launch), GEMM Z, residual+softplus, GEMM G (split-K),
// fold+kick+write (1 launch).  X^T is materialised once per call.
#include "kernels.h"
#include "ops_common.cuh"

#include <math.h>

namespace nxv {

namespace {

constexpr int kRT = 256;  // residual kernel threads
constexpr int kRE = 4;    // observations per residual thread

// R = y - sigmoid(Z) in place; lpart[c][blk] = sum over the block's j of
// y z - softplus(z), softplus(z) = max(z, 0) + log1p(exp(-|z|)).
__global__ void __launch_bounds__(kRT)
k_lr_resid(double* __restrict__ Z, const double* __restrict__ y, size_t n_obs, double* lpart,
           unsigned nblk) {
    const unsigned c = blockIdx.y;
    double* zr = Z + (size_t)c * n_obs;
    double t = 0.0;
    size_t base = (size_t)blockIdx.x * (kRT * kRE);
#pragma unroll
    for (int e = 0; e < kRE; e++) {
        size_t j = base + (size_t)e * kRT + threadIdx.x;
        if (j < n_obs) {
            double z = zr[j];
            double yj = y[j];
            double s = div_(1.0, add_(1.0, exp(-z)));
            zr[j] = sub_(yj, s);
            double sp = add_((z > 0.0 ? z : 0.0), log1p(exp(-fabs(z))));
            t = add_(t, sub_(mul_(yj, z), sp));
        }
    }
    __shared__ double sm[kRT / 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t = add_(t, __shfl_down_sync(0xffffffffu, t, off));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = sm[0];
        for (int w = 1; w < kRT / 32; w++) s = add_(s, sm[w]);
        lpart[(size_t)c * nblk + blockIdx.x] = s;
    }
}

// p_h = p + he*g; q = q + eps*p_h; p = p_h   (inv_mass = 1)
__global__ void k_lr_drift(double* __restrict__ q, double* __restrict__ p,
                           const double* __restrict__ g, size_t total, double eps, double he) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    double ph = add_(p[i], mul_(he, g[i]));
    q[i] = add_(q[i], mul_(eps, ph));
    p[i] = ph;
}

// One CTA per chain: g = sum_s part[s] - q; then (step) p = p + he*g and
// write q/p/g rows of step k and logp[c][k] = sum lpart - 0.5 |q|^2.
__global__ void __launch_bounds__(128)
k_lr_fold(const double* __restrict__ part, int S, size_t CD, double* __restrict__ q,
          double* __restrict__ p, double* __restrict__ g, const double* __restrict__ lpart,
          unsigned nblk, size_t D, double he, int write_step, unsigned k, unsigned K,
          double* qc, double* pc, double* gc, double* logp) {
    const unsigned c = blockIdx.x;
    double qq = 0.0;
    for (size_t i = threadIdx.x; i < D; i += blockDim.x) {
        size_t o = (size_t)c * D + i;
        double s = part[o];
        for (int t = 1; t < S; t++) s = add_(s, part[(size_t)t * CD + o]);
        double qi = q[o];
        double gi = sub_(s, qi);
        g[o] = gi;
        qq = add_(qq, mul_(qi, qi));
        if (write_step) {
            double pi = add_(p[o], mul_(he, gi));
            p[o] = pi;
            size_t row = ((size_t)c * K + k) * D + i;
            qc[row] = qi;
            pc[row] = pi;
            gc[row] = gi;
        }
    }
    if (!write_step) return;
    __shared__ double sm[4];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) qq = add_(qq, __shfl_down_sync(0xffffffffu, qq, off));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = qq;
    __syncthreads();
    if (threadIdx.x == 0) {
        double sq = sm[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) sq = add_(sq, sm[w]);
        double l = lpart[(size_t)c * nblk];
        for (unsigned b = 1; b < nblk; b++) l = add_(l, lpart[(size_t)c * nblk + b]);
        logp[(size_t)c * K + k] = sub_(l, mul_(0.5, sq));
    }
}

}  // namespace

int launch_chain_logreg_f64(Ctx& c, void* qc, void* pc, void* gc, void* logp, const void* q0,
                            const void* p0, const void* X, const void* y, size_t n_obs,
                            size_t D, size_t C, unsigned K, double eps) {
    if (C == 0 || K == 0 || D == 0) return OK;
    if (n_obs == 0) {
        set_error("logistic regression needs at least one observation");
        return E_ARG;
    }
    if (n_obs > 0x7fffffff || D > 0x7fffffff || C > 65535) {
        set_error("logistic regression extents out of range");
        return E_ARG;
    }
    const size_t CD = C * D;
    // split-K slices for G = R . X: enough CTAs to cover the SMs.
    const size_t ctas_mn = ((C + 127) / 128) * ((D + 127) / 128);
    size_t S = (2 * (size_t)c.dev->sm_count + ctas_mn - 1) / ctas_mn;
    size_t L = (n_obs + S - 1) / S;
    L = (L + 15) & ~(size_t)15;  // keep slice starts 16-byte aligned, BK multiple
    S = (n_obs + L - 1) / L;
    const unsigned nblk = (unsigned)((n_obs + kRT * kRE - 1) / (kRT * kRE));
    // scratch: Xt [D][N] | q | p | g [C][D] | Z [C][N] | lpart [C][nblk] | part [S][C][D]
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    };
    size_t oXt = take(D * n_obs * 8), oq = take(CD * 8), op = take(CD * 8), og = take(CD * 8),
           oZ = take(C * n_obs * 8), oL = take(C * nblk * 8), oP = take(S * CD * 8);
    ScratchGuard guard(c);
    char* base = (char*)scratch(c, off);
    if (!base) return E_CUDA;
    double* Xt = (double*)(base + oXt);
    double* q = (double*)(base + oq);
    double* p = (double*)(base + op);
    double* g = (double*)(base + og);
    double* Z = (double*)(base + oZ);
    double* lp = (double*)(base + oL);
    double* part = (double*)(base + oP);

    int rc = enqueue_transpose(c, F64, Xt, X, (unsigned)n_obs, (unsigned)D);
    if (rc) return rc;
    NXV_CK(cudaMemcpyAsync(q, q0, CD * 8, cudaMemcpyDeviceToDevice, c.stream));
    NXV_CK(cudaMemcpyAsync(p, p0, CD * 8, cudaMemcpyDeviceToDevice, c.stream));

    GemmP<double> G1{};  // Z = Q . Xt
    G1.A = q; G1.B = Xt; G1.C = Z;
    G1.M = (int)C; G1.N = (int)n_obs; G1.K = (int)D;
    G1.lda = (int)D; G1.ldb = (int)n_obs; G1.ldc = (int)n_obs;
    G1.batch = 1;
    GemmP<double> G2{};  // part[s] = R[:, slice s] . X[slice s, :]
    G2.A = Z; G2.B = (const double*)X; G2.C = part;
    G2.M = (int)C; G2.N = (int)D; G2.K = (int)n_obs;
    G2.lda = (int)n_obs; G2.ldb = (int)D; G2.ldc = (int)D;
    G2.sC = (long long)CD; G2.ksplit = (int)L; G2.batch = (int)S;

    const double he = 0.5 * eps;
    auto gradient = [&](int write_step, unsigned k) -> int {
        int r = gemm_f64(c, G1);
        if (r) return r;
        dim3 rg(nblk, (unsigned)C);
        k_lr_resid<<<rg, kRT, 0, c.stream>>>(Z, (const double*)y, n_obs, lp, nblk);
        count_launch();
        r = gemm_f64(c, G2);
        if (r) return r;
        k_lr_fold<<<(unsigned)C, 128, 0, c.stream>>>(part, (int)S, CD, q, p, g, lp, nblk, D, he,
                                                      write_step, k, K, (double*)qc, (double*)pc,
                                                      (double*)gc, (double*)logp);
        count_launch();
        return OK;
    };
    rc = gradient(0, 0);
    if (rc) return rc;
    for (unsigned k = 0; k < K; k++) {
        unsigned blocks = (unsigned)((CD + 255) / 256);
        k_lr_drift<<<blocks, 256, 0, c.stream>>>(q, p, g, CD, eps, he);
        count_launch();
        rc = gradient(1, k);
        if (rc) return rc;
    }
    return finish(c);
}

}  // namespace nxv
