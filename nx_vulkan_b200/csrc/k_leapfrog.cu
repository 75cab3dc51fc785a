// k_leapfrog.cu -- fused K-step HMC leapfrog chains (sm_100a).
//
// One kernel template serves every chain family of the reference
// (c_src/nx_vulkan_shim.h:191-280; lib/nx_vulkan.ex:582-726) and the batched
// f64 Gaussian of the anisotropic-target workload.  Per step k and element i:
//     p_h = p + (eps/2) * g            (g = grad log p at the current q)
//     q   = q + (eps * m_i) * p_h
//     g   = grad log p(q)
//     p   = p_h + (eps/2) * g
// (the corrected sign, PLAN_FUSED_LEAPFROG.md:18-24), then q, p, g are
// written to the [chain][k][i] trajectories and the step's log density
// logp = scale * sum_i term(q_i) + cst goes to logp[chain][k].
//
// B200 design: the work is HBM-write bound (3 * sizeof(T) bytes per element
// and step; the inputs are read once).  A CTA owns one tile of NT*VPT
// consecutive elements of one chain, keeps q, p, g, m (and the per-element
// target parameter) in registers for all K steps, and streams the three
// trajectory rows out with coalesced evict-first stores.  The per-step sum
// is a warp-shuffle tree whose per-warp results wait in shared memory; one
// barrier every 32 steps folds them (fixed order, so deterministic) instead
// of a barrier per step as in the reference shader's 256-wide tree.  When a
// chain spans several tiles, tiles write partial sums to scratch and a
// small second kernel folds them in tile order.
#include "kernels.h"
#include "ops_common.cuh"

#include <math.h>
#include <stdlib.h>
#include <string.h>

namespace nxv {

namespace {

constexpr int KC = 32;  // steps per logp flush

// ---- families (per-element math matches the CPU oracle op by op) -----------

struct NoParam {};

// f32 family transcendentals are evaluated in f64 and rounded once, as
// Nx.BinaryBackend does for every f32 op.
__device__ __forceinline__ float ex(float x) { return (float)exp((double)x); }

struct FamNormal32 {
    float mu, sigma, inv_var;
    using P = NoParam;
    __device__ P load(const void*, size_t) const { return P{}; }
    __device__ float grad(float q, P) const { return -mul_(sub_(q, mu), inv_var); }
    __device__ double term(float q, P) const {
        float z = div_(sub_(q, mu), sigma);
        return (double)mul_(z, z);
    }
};
struct FamExp32 {
    float lambda;
    using P = NoParam;
    __device__ P load(const void*, size_t) const { return P{}; }
    __device__ float grad(float q, P) const { return sub_(1.0f, mul_(lambda, ex(q))); }
    __device__ double term(float q, P) const { return (double)sub_(q, mul_(lambda, ex(q))); }
};
struct FamStudentT32 {
    float mu, sigma, nu, logp_const;
    using P = NoParam;
    __device__ P load(const void*, size_t) const { return P{}; }
    __device__ float grad(float q, P) const {
        float d = sub_(q, mu);
        return -div_(mul_(add_(nu, 1.0f), d), add_(mul_(nu, mul_(sigma, sigma)), mul_(d, d)));
    }
    __device__ double term(float q, P) const {
        float z = div_(sub_(q, mu), sigma);
        float l = (float)log1p((double)div_(mul_(z, z), nu));
        return (double)sub_(logp_const, mul_(mul_(add_(nu, 1.0f), 0.5f), l));
    }
};
struct FamCauchy32 {
    float loc, scale, log_pi_scale;
    using P = NoParam;
    __device__ P load(const void*, size_t) const { return P{}; }
    __device__ float grad(float q, P) const {
        float d = sub_(q, loc);
        return -div_(mul_(2.0f, d), add_(mul_(scale, scale), mul_(d, d)));
    }
    __device__ double term(float q, P) const {
        float z = div_(sub_(q, loc), scale);
        return (double)sub_(log_pi_scale, (float)log1p((double)mul_(z, z)));
    }
};
struct FamHalfNormal32 {
    float sigma, log_const;
    using P = NoParam;
    __device__ P load(const void*, size_t) const { return P{}; }
    __device__ float grad(float q, P) const {
        return sub_(1.0f, div_(ex(mul_(2.0f, q)), mul_(sigma, sigma)));
    }
    __device__ double term(float q, P) const {
        float e2 = ex(mul_(2.0f, q));
        return (double)sub_(add_(log_const, q), div_(e2, mul_(2.0f, mul_(sigma, sigma))));
    }
};
struct FamWeibull32 {
    float k, lambda;
    using P = NoParam;
    __device__ P load(const void*, size_t) const { return P{}; }
    __device__ float r_(float q) const { return (float)pow((double)div_(ex(q), lambda), (double)k); }
    __device__ float grad(float q, P) const { return mul_(k, sub_(1.0f, r_(q))); }
    __device__ double term(float q, P) const { return (double)sub_(mul_(k, q), r_(q)); }
};
// f64 Gaussian with a per-element precision (prec == nullptr: scalar).
struct FamGauss64 {
    const double* prec;
    double prec_s, mu;
    using P = double;
    __device__ P load(const void*, size_t i) const { return prec ? __ldg(prec + i) : prec_s; }
    __device__ double grad(double q, P pr) const { return -mul_(pr, sub_(q, mu)); }
    __device__ double term(double q, P pr) const {
        double d = sub_(q, mu);
        return mul_(mul_(pr, d), d);
    }
};

template <typename T>
struct ChainArgs {
    T* qc;
    T* pc;
    T* gc;
    T* logp;          // [chain][k] (mode 0, tiles == 1) or [k][tile] (mode 1)
    double* partial;  // [chain][k][tile] when tiles > 1 in mode 0
    const T* q0;
    const T* p0;
    const T* m;
    size_t m_cs;      // chain stride of m in elements: n ([chain][i]) or 0 (one [i] row for all)
    size_t n;
    unsigned chains, tiles, K;
    T eps, he;
    double scale, cst;
    const double* cst_dev;  // added to cst when non-null
    int mode;               // 0: per-chain logp; 1: per-256-group partials (_lg)
    T* ke;                  // [chain][k] kinetic energy 0.5 * sum(p*p*m) (KE kernels only)
    double* ke_partial;     // [chain][k][tile] when tiles > 1 (KE kernels only)
};

template <typename T>
__device__ __forceinline__ void st_stream(T* p, T v) { __stcs(p, v); }

// KE: also reduce the kinetic energy 0.5 * sum_i (p_i * p_i) * m_i of every
// step, in the same fixed tree as logp, into g.ke (or g.ke_partial).
template <typename T, class Fam, int NT, int VPT, bool KE>
__global__ void __launch_bounds__(NT) k_chain(ChainArgs<T> g, Fam fam) {
    constexpr int NW = NT / 32;
    __shared__ double red[KC][NW];
    __shared__ double redk[KE ? KC : 1][NW];
    const unsigned tile = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const double cst = g.cst + (g.cst_dev ? *g.cst_dev : 0.0);
    for (unsigned chain = blockIdx.y; chain < g.chains; chain += gridDim.y) {
        const size_t cbase = (size_t)chain * g.n;
        T q[VPT], p[VPT], gr[VPT], em[VPT];
        typename Fam::P ep[VPT];
        bool ok[VPT];
#pragma unroll
        for (int v = 0; v < VPT; v++) {
            size_t i = (size_t)tile * (NT * VPT) + (size_t)v * NT + tid;
            ok[v] = i < g.n;
            size_t ii = ok[v] ? i : 0;
            q[v] = ok[v] ? g.q0[cbase + ii] : T(0);
            p[v] = ok[v] ? g.p0[cbase + ii] : T(0);
            em[v] = ok[v] ? g.m[(size_t)chain * g.m_cs + ii] : T(0);
            ep[v] = fam.load(nullptr, ii);
            gr[v] = fam.grad(q[v], ep[v]);
        }
        const T eps = g.eps, he = g.he;
        for (unsigned k0 = 0; k0 < g.K; k0 += KC) {
            const unsigned kn = (g.K - k0) < (unsigned)KC ? (g.K - k0) : (unsigned)KC;
            for (unsigned kk = 0; kk < kn; kk++) {
                const unsigned k = k0 + kk;
                const size_t row = ((size_t)chain * g.K + k) * g.n;
                double t = 0.0, tk = 0.0;
#pragma unroll
                for (int v = 0; v < VPT; v++) {
                    T ph = add_(p[v], mul_(he, gr[v]));
                    q[v] = add_(q[v], mul_(mul_(eps, em[v]), ph));
                    gr[v] = fam.grad(q[v], ep[v]);
                    p[v] = add_(ph, mul_(he, gr[v]));
                    if (ok[v]) {
                        size_t i = (size_t)tile * (NT * VPT) + (size_t)v * NT + tid;
                        st_stream(g.qc + row + i, q[v]);
                        st_stream(g.pc + row + i, p[v]);
                        st_stream(g.gc + row + i, gr[v]);
                        t = __dadd_rn(t, fam.term(q[v], ep[v]));
                        if constexpr (KE) tk = __dadd_rn(tk, (double)mul_(mul_(p[v], p[v]), em[v]));
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    t = __dadd_rn(t, __shfl_down_sync(0xffffffffu, t, off));
                if constexpr (KE) {
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)
                        tk = __dadd_rn(tk, __shfl_down_sync(0xffffffffu, tk, off));
                    if (lane == 0) redk[kk][warp] = tk;
                }
                if (lane == 0) red[kk][warp] = t;
            }
            __syncthreads();
            if (tid < (int)kn) {
                double s = red[tid][0];
#pragma unroll
                for (int w = 1; w < NW; w++) s = __dadd_rn(s, red[tid][w]);
                const unsigned k = k0 + tid;
                if (g.mode == 1) {
                    double val = g.scale * s + (tile == 0 ? cst : 0.0);
                    g.logp[(size_t)k * g.tiles + tile] = (T)val;
                } else if (g.tiles == 1) {
                    g.logp[(size_t)chain * g.K + k] = (T)(g.scale * s + cst);
                } else {
                    g.partial[((size_t)chain * g.K + k) * g.tiles + tile] = s;
                }
                if constexpr (KE) {
                    double sk = redk[tid][0];
#pragma unroll
                    for (int w = 1; w < NW; w++) sk = __dadd_rn(sk, redk[tid][w]);
                    if (g.tiles == 1) g.ke[(size_t)chain * g.K + k] = (T)(0.5 * sk);
                    else g.ke_partial[((size_t)chain * g.K + k) * g.tiles + tile] = sk;
                }
            }
            __syncthreads();
        }
    }
}

// ---- staged-store variant (TMA bulk stores) ----------------------------------
//
// One tile per chain (n <= NT*VPT).  S consecutive steps of the q/p/grad
// rows are written to shared memory and leave as three bulk copies
// (cp.async.bulk.global.shared::cta) of S*n*sizeof(T) contiguous bytes each:
// rows k0..k0+S-1 of one chain are adjacent in the [chain][k][i] layout.  Two
// staging buffers alternate; before a buffer is rewritten the issuing thread
// waits until the bulk copies that read it two blocks earlier have finished
// reading (cp.async.bulk.wait_group.read 1), which is a completion wait on
// this CTA's own copies and always ends.  Requires n*sizeof(T) % 16 == 0.

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, unsigned bytes) {
    unsigned s = (unsigned)__cvta_generic_to_shared(ssrc);
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gdst), "r"(s),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() {
    asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

template <typename T, class Fam, int NT, int VPT, int S, bool KE>
__global__ void __launch_bounds__(NT) k_chain_tma(ChainArgs<T> g, Fam fam) {
    static_assert(KC % S == 0, "S must divide KC");
    constexpr int NW = NT / 32;
    __shared__ double red[KC][NW];
    __shared__ double redk[KE ? KC : 1][NW];
    extern __shared__ __align__(128) unsigned char dsm[];
    T* sbuf = reinterpret_cast<T*>(dsm);  // [2][3][S][n]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t n = g.n, arr = (size_t)S * n, bufsz = 3 * arr;
    const double cst = g.cst + (g.cst_dev ? *g.cst_dev : 0.0);
    T* outs[3] = {g.qc, g.pc, g.gc};
    int bsel = 0;
    for (unsigned chain = blockIdx.x; chain < g.chains; chain += gridDim.x) {
        const size_t cbase = (size_t)chain * n;
        T q[VPT], p[VPT], gr[VPT], em[VPT];
        typename Fam::P ep[VPT];
        bool ok[VPT];
#pragma unroll
        for (int v = 0; v < VPT; v++) {
            size_t i = (size_t)v * NT + tid;
            ok[v] = i < n;
            size_t ii = ok[v] ? i : 0;
            q[v] = ok[v] ? g.q0[cbase + ii] : T(0);
            p[v] = ok[v] ? g.p0[cbase + ii] : T(0);
            em[v] = ok[v] ? g.m[(size_t)chain * g.m_cs + ii] : T(0);
            ep[v] = fam.load(nullptr, ii);
            gr[v] = fam.grad(q[v], ep[v]);
        }
        const T eps = g.eps, he = g.he;
        for (unsigned k0 = 0; k0 < g.K; k0 += S) {
            const unsigned kn = (g.K - k0) < (unsigned)S ? (g.K - k0) : (unsigned)S;
            if (tid == 0) bulk_wait_read1();
            __syncthreads();
            T* b = sbuf + (size_t)bsel * bufsz;
            for (unsigned kk = 0; kk < kn; kk++) {
                double t = 0.0, tk = 0.0;
#pragma unroll
                for (int v = 0; v < VPT; v++) {
                    T ph = add_(p[v], mul_(he, gr[v]));
                    q[v] = add_(q[v], mul_(mul_(eps, em[v]), ph));
                    gr[v] = fam.grad(q[v], ep[v]);
                    p[v] = add_(ph, mul_(he, gr[v]));
                    if (ok[v]) {
                        size_t i = (size_t)v * NT + tid;
                        b[kk * n + i] = q[v];
                        b[arr + kk * n + i] = p[v];
                        b[2 * arr + kk * n + i] = gr[v];
                        t = __dadd_rn(t, fam.term(q[v], ep[v]));
                        if constexpr (KE) tk = __dadd_rn(tk, (double)mul_(mul_(p[v], p[v]), em[v]));
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    t = __dadd_rn(t, __shfl_down_sync(0xffffffffu, t, off));
                if constexpr (KE) {
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)
                        tk = __dadd_rn(tk, __shfl_down_sync(0xffffffffu, tk, off));
                    if (lane == 0) redk[(k0 + kk) % KC][warp] = tk;
                }
                if (lane == 0) red[(k0 + kk) % KC][warp] = t;
            }
            fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) {
                const size_t goff = ((size_t)chain * g.K + k0) * n;
                const unsigned bytes = (unsigned)(kn * n * sizeof(T));
#pragma unroll
                for (int a = 0; a < 3; a++) bulk_store(outs[a] + goff, b + a * arr, bytes);
                bulk_commit();
            }
            bsel ^= 1;
            const unsigned kend = k0 + kn;
            if (kend % KC == 0 || kend == g.K) {
                const unsigned kbase = ((kend - 1) / KC) * KC;
                if (tid < (int)(kend - kbase)) {
                    double s = red[tid][0];
#pragma unroll
                    for (int w = 1; w < NW; w++) s = __dadd_rn(s, red[tid][w]);
                    g.logp[(size_t)chain * g.K + kbase + tid] = (T)(g.scale * s + cst);
                    if constexpr (KE) {
                        double sk = redk[tid][0];
#pragma unroll
                        for (int w = 1; w < NW; w++) sk = __dadd_rn(sk, redk[tid][w]);
                        g.ke[(size_t)chain * g.K + kbase + tid] = (T)(0.5 * sk);
                    }
                }
            }
        }
        __syncthreads();
    }
    if (tid == 0) bulk_wait_all();
}

template <typename T>
__global__ void k_chain_fold(ChainArgs<T> g) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t total = (size_t)g.chains * g.K;
    if (t >= total) return;
    const double cst = g.cst + (g.cst_dev ? *g.cst_dev : 0.0);
    const double* pp = g.partial + t * g.tiles;
    double s = pp[0];
    for (unsigned i = 1; i < g.tiles; i++) s = __dadd_rn(s, pp[i]);
    g.logp[t] = (T)(g.scale * s + cst);
    if (g.ke) {
        const double* pk = g.ke_partial + t * g.tiles;
        double sk = pk[0];
        for (unsigned i = 1; i < g.tiles; i++) sk = __dadd_rn(sk, pk[i]);
        g.ke[t] = (T)(0.5 * sk);
    }
}

// 0.5 * sum_i log prec_i - n * log sqrt(2 pi), fixed-order block tree.
__global__ void __launch_bounds__(256) k_gauss_const(const double* __restrict__ prec, size_t n,
                                                     double* out) {
    __shared__ double sm[8];
    double s = 0.0;
    for (size_t i = threadIdx.x; i < n; i += 256) s = __dadd_rn(s, log(prec[i]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s = __dadd_rn(s, __shfl_down_sync(0xffffffffu, s, off));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = sm[0];
        for (int w = 1; w < 8; w++) t = __dadd_rn(t, sm[w]);
        *out = 0.5 * t - (double)n * 0.91893853320467274178;
    }
}

// Launch configuration: NT threads x VPT elements per thread per tile.
// NXV_LF_CFG="NTxVPT" overrides the heuristic (256x1, 256x2, 256x4, 256x8, 128x8).
struct Cfg { int nt, vpt; };

Cfg pick_cfg(Ctx& c, size_t n, size_t chains, int mode) {
    if (mode == 1) return Cfg{256, 1};
    const char* env = getenv("NXV_LF_CFG");
    if (env && *env) {
        int a = 0, b = 0;
        if (sscanf(env, "%dx%d", &a, &b) == 2) {
            if ((a == 256 && (b == 1 || b == 2 || b == 4 || b == 8)) || (a == 128 && b == 8))
                return Cfg{a, b};
        }
    }
    // One tile per chain up to n = 2048 (no partial-sum pass); measured on
    // B200 for 4096 chains x d=1000 x L=32: 256x8 0.539 ms, 128x8 0.551,
    // 256x4 0.571, 256x1 (4 tiles + fold) 0.578.
    (void)c;
    (void)chains;
    if (n <= 512) return Cfg{256, 2};
    return Cfg{256, 8};
}

// NXV_LF_OCC=k caps the resident CTAs per SM at k (by reserving shared
// memory); 0 or unset leaves occupancy to the register budget.
size_t occupancy_smem(Ctx& c) {
    const char* env = getenv("NXV_LF_OCC");
    int occ = env ? atoi(env) : 0;
    if (occ <= 0) return 0;
    int dev = c.dev->id, per_sm = 0;
    if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
        return 0;
    size_t want = (size_t)per_sm / (size_t)occ;
    return want > 4096 ? want - 4096 : 0;
}

template <typename T, class Fam, int NT, int VPT, bool KE>
int launch_cfg(Ctx& c, ChainArgs<T>& g, const Fam& fam) {
    g.tiles = (unsigned)((g.n + NT * VPT - 1) / (NT * VPT));
    if (g.mode == 0 && g.tiles > 1 && !g.partial) {
        g.partial = (double*)scratch(c, (size_t)g.chains * g.K * g.tiles * sizeof(double));
        if (!g.partial) return E_CUDA;
    }
    if (g.tiles > 65535u) {
        set_error("chain dimension too large");
        return E_ARG;
    }
    unsigned gy = g.chains < 65535u ? g.chains : 65535u;
    dim3 grid(g.tiles, gy);
    size_t dyn = occupancy_smem(c);
    if (dyn > 0) {
        cudaError_t e = cudaFuncSetAttribute(k_chain<T, Fam, NT, VPT, KE>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_chain)");
    }
    if (KE && g.tiles > 1 && !g.ke_partial) {
        set_error("kinetic-energy partials need scratch");
        return E_ARG;
    }
    k_chain<T, Fam, NT, VPT, KE><<<grid, NT, dyn, c.stream>>>(g, fam);
    count_launch();
    if (g.mode == 0 && g.tiles > 1) {
        size_t total = (size_t)g.chains * g.K;
        k_chain_fold<T><<<(unsigned)((total + 255) / 256), 256, 0, c.stream>>>(g);
        count_launch();
    }
    return finish(c);
}

// The staged-store kernel is the default whenever a chain fits one tile
// (n <= 2048) and its rows are 16-byte multiples.  Measured on B200 for
// 4096 chains x d=1000 x L=32 (f64): register stores 0.538 ms (92% of the
// measured HBM copy bandwidth); staged S=1 0.521, S=2 0.503 (98.5%),
// S=4 0.509.  NXV_LF_TMA=S (1, 2, 4) picks S; NXV_LF_TMA=0 disables it.
int tma_steps() {
    const char* env = getenv("NXV_LF_TMA");
    if (!env || !*env) return 2;
    int s = atoi(env);
    return (s == 1 || s == 2 || s == 4) ? s : 0;
}

// The staged-store kernel takes a chain when its rows fit one 256-thread
// tile (n <= 2048), are 16-byte multiples, and the double-buffered stage of
// S steps plus the reduction buffers fit the opt-in shared memory.
bool tma_fits(Ctx& c, size_t n, size_t elt, int S, bool ke) {
    if (S == 0 || n > 2048 || (n * elt) % 16 != 0) return false;
    size_t smem = 2 * 3 * (size_t)S * n * elt;
    int per_block = 0;
    cudaDeviceGetAttribute(&per_block, cudaDevAttrMaxSharedMemoryPerBlockOptin, c.dev->id);
    return smem + (ke ? 2 : 1) * KC * 8 * 8 <= (size_t)per_block;
}

template <typename T, class Fam, int VPT, int S, bool KE>
int launch_tma(Ctx& c, ChainArgs<T>& g, const Fam& fam) {
    size_t smem = 2 * 3 * (size_t)S * g.n * sizeof(T);
    if (!tma_fits(c, g.n, sizeof(T), S, KE)) return E_KERNEL;  // caller falls back
    cudaError_t e = cudaFuncSetAttribute(k_chain_tma<T, Fam, 256, VPT, S, KE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_chain_tma)");
    g.tiles = 1;
    unsigned grid = g.chains < 0x7fffffffu ? g.chains : 0x7fffffffu;
    k_chain_tma<T, Fam, 256, VPT, S, KE><<<grid, 256, smem, c.stream>>>(g, fam);
    count_launch();
    return finish(c);
}

template <typename T, class Fam, int VPT, bool KE>
int launch_tma_s(Ctx& c, ChainArgs<T>& g, const Fam& fam, int s) {
    if (s == 1) return launch_tma<T, Fam, VPT, 1, KE>(c, g, fam);
    if (s == 2) return launch_tma<T, Fam, VPT, 2, KE>(c, g, fam);
    return launch_tma<T, Fam, VPT, 4, KE>(c, g, fam);
}

// KE: the kernels also write g.ke (instantiated for the f64 Gaussian only).
template <typename T, class Fam, bool KE = false>
int launch_family(Ctx& c, ChainArgs<T>& g, const Fam& fam) {
    if (g.n == 0 || g.K == 0 || g.chains == 0) return OK;
    ScratchGuard guard(c);
    int s = tma_steps();
    if (s && g.mode == 0 && g.n <= 2048 && (g.n * sizeof(T)) % 16 == 0) {
        int rc = g.n <= 1024 ? launch_tma_s<T, Fam, 4, KE>(c, g, fam, s)
                             : launch_tma_s<T, Fam, 8, KE>(c, g, fam, s);
        if (rc != E_KERNEL) return rc;
    }
    Cfg cf = pick_cfg(c, g.n, g.chains, g.mode);
    if (cf.nt == 128) return launch_cfg<T, Fam, 128, 8, KE>(c, g, fam);
    switch (cf.vpt) {
        case 1: return launch_cfg<T, Fam, 256, 1, KE>(c, g, fam);
        case 2: return launch_cfg<T, Fam, 256, 2, KE>(c, g, fam);
        case 4: return launch_cfg<T, Fam, 256, 4, KE>(c, g, fam);
        default: return launch_cfg<T, Fam, 256, 8, KE>(c, g, fam);
    }
}

// Tiles per chain of the kernel launch_family runs for an f64 chain
// (mode 0): 1 on the staged-store kernel, else pick_cfg's tile count.  The
// scratch for per-tile partial sums is sized from it.
size_t gauss_tiles(Ctx& c, size_t n, size_t chains, bool ke) {
    if (tma_fits(c, n, sizeof(double), tma_steps(), ke)) return 1;
    const Cfg cf = pick_cfg(c, n, chains, 0);
    return (n + (size_t)cf.nt * cf.vpt - 1) / ((size_t)cf.nt * cf.vpt);
}

}  // namespace

int launch_chain_f32(Ctx& c, int fam, const float* prm, void* qc, void* pc, void* gc,
                     void* logp, const void* q0, const void* p0, const void* m, size_t n,
                     size_t chains, unsigned K, float eps, int logp_mode) {
    ChainArgs<float> g{};
    g.qc = (float*)qc;
    g.pc = (float*)pc;
    g.gc = (float*)gc;
    g.logp = (float*)logp;
    g.q0 = (const float*)q0;
    g.p0 = (const float*)p0;
    g.m = (const float*)m;
    g.m_cs = n;
    g.n = n;
    g.chains = (unsigned)chains;
    g.K = K;
    g.eps = eps;
    g.he = 0.5f * eps;
    g.mode = logp_mode;
    g.scale = 1.0;
    g.cst = 0.0;
    switch (fam) {
        case FAM_NORMAL: {
            g.scale = -0.5;
            g.cst = -(double)n * (log((double)prm[1]) + 0.91893853320467274178);
            FamNormal32 f{prm[0], prm[1], 1.0f / (prm[1] * prm[1])};
            return launch_family(c, g, f);
        }
        case FAM_EXP: {
            g.cst = (double)n * log((double)prm[0]);
            return launch_family(c, g, FamExp32{prm[0]});
        }
        case FAM_STUDENTT: return launch_family(c, g, FamStudentT32{prm[0], prm[1], prm[2], prm[3]});
        case FAM_CAUCHY: return launch_family(c, g, FamCauchy32{prm[0], prm[1], prm[2]});
        case FAM_HALFNORMAL: return launch_family(c, g, FamHalfNormal32{prm[0], prm[1]});
        case FAM_WEIBULL: {
            g.cst = (double)prm[2];
            return launch_family(c, g, FamWeibull32{prm[0], prm[1]});
        }
    }
    set_error("unknown chain family %d", fam);
    return E_ARG;
}

int launch_gauss_const(Ctx& c, const void* prec, size_t n, void* out) {
    k_gauss_const<<<1, 256, 0, c.stream>>>((const double*)prec, n, (double*)out);
    count_launch();
    return OK;
}

int launch_chain_gauss_f64(Ctx& c, void* qc, void* pc, void* gc, void* logp, const void* q0,
                           const void* p0, const void* m, const void* prec, double prec_scalar,
                           double mu, size_t n, size_t chains, unsigned K, double eps, void* ke,
                           bool m_shared, const void* cst_dev) {
    ChainArgs<double> g{};
    g.qc = (double*)qc;
    g.pc = (double*)pc;
    g.gc = (double*)gc;
    g.logp = (double*)logp;
    g.q0 = (const double*)q0;
    g.p0 = (const double*)p0;
    g.m = (const double*)m;
    g.m_cs = m_shared ? 0 : n;
    g.n = n;
    g.chains = (unsigned)chains;
    g.K = K;
    g.eps = eps;
    g.he = 0.5 * eps;
    g.mode = 0;
    g.scale = -0.5;
    g.ke = (double*)ke;
    if (n == 0 || K == 0 || chains == 0) return OK;
    ScratchGuard guard(c);
    // Scratch: [256 B: the log-density constant][tile partials of logp][tile
    // partials of the kinetic energy], partials only when a chain spans
    // several tiles.
    size_t tiles = gauss_tiles(c, n, chains, ke != nullptr);
    size_t part = tiles > 1 ? chains * (size_t)K * tiles * sizeof(double) : 0;
    size_t need = 256 + part * (ke ? 2 : 1);
    char* base = (char*)scratch(c, need);
    if (!base) return E_CUDA;
    if (tiles > 1) {
        g.partial = (double*)(base + 256);
        if (ke) g.ke_partial = (double*)(base + 256 + part);
    }
    FamGauss64 fam{(const double*)prec, prec_scalar, mu};
    if (prec && cst_dev) {
        // the caller computed the constant (launch_gauss_const) for many calls
        g.cst = 0.0;
        g.cst_dev = (const double*)cst_dev;
        fam.prec_s = 0.0;
    } else if (prec) {
        // The constant needs sum(log prec): one tiny launch ahead of the
        // chain writes it to the first 256 bytes of scratch.
        k_gauss_const<<<1, 256, 0, c.stream>>>((const double*)prec, n, (double*)base);
        count_launch();
        g.cst = 0.0;
        g.cst_dev = (const double*)base;
        fam.prec_s = 0.0;
    } else {
        // scalar precision: the reference's Normal(mu, sigma) f64 chain with
        // prec = 1/sigma^2; the constant is -n (log sigma + log sqrt(2 pi)).
        g.cst = 0.5 * (double)n * log(prec_scalar) - (double)n * 0.91893853320467274178;
    }
    if (ke) return launch_family<double, FamGauss64, true>(c, g, fam);
    return launch_family(c, g, fam);
}

}  // namespace nxv

// ---- scratch-free entry point --------------------------------------------------
//
// nxv_leapfrog_chain_gauss_f64_batched_noalloc runs the same kernels as
// nxv_leapfrog_chain_gauss_f64_batched, but its scratch (the log-density
// constant and, for chains longer than one 2048-element tile, the per-tile
// partial sums) lives in a file-scope device array instead of the
// library's allocator.  Capacity: 1 MiB, i.e. 256 bytes for the constant
// plus n_chains * K * ceil(n / 2048) partial sums of 8 bytes when n > 2048;
// chains of n <= 2048 need only the constant.  Every GPU that loads the
// library holds the array until the process exits.

namespace nxv {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};

// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory: the device address comes from cudaGetSymbolAddress, looked up once
// per device with that device current, and is what the kernels receive.
int noalloc_scratch(Ctx& c, char** out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    const int id = c.dev->id;
    if (id < 0 || id >= 64) {
        set_error("device id %d out of range", id);
        return E_ARG;
    }
    if (!g_noalloc_addr[id]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_noalloc_addr[id] = p;
    }
    *out = static_cast<char*>(g_noalloc_addr[id]);
    return OK;
}

}  // namespace
}  // namespace nxv

extern "C" int nxv_leapfrog_chain_gauss_f64_batched_noalloc(
    void* q_chain, void* p_chain, void* grad_chain, void* logp_chain, const void* q_init,
    const void* p_init, const void* inv_mass, const void* prec, unsigned int n,
    unsigned int n_chains, unsigned int K, double eps, double mu) {
    using namespace nxv;
    if (!q_chain || !p_chain || !grad_chain || !logp_chain || !q_init || !p_init || !inv_mass ||
        !prec)
        return E_NULL;
    if (K == 0) {
        set_error("K must be positive");
        return E_ARG;
    }
    Ctx c;
    int rc = begin(c, {});
    if (rc) return rc;
    char* base = nullptr;
    rc = noalloc_scratch(c, &base);
    if (rc) return rc;
    if (n == 0 || n_chains == 0) return OK;
    // partial sums only when the kernel that launch_family picks splits a
    // chain into several tiles
    const size_t tiles = gauss_tiles(c, n, n_chains, false);
    const size_t need = 256 + (tiles > 1 ? (size_t)n_chains * K * tiles * sizeof(double) : 0);
    if (need > kNoAllocScratchBytes) {
        set_error("leapfrog noalloc: %u chains x %u steps x %zu tiles per chain need %zu "
                  "bytes of scratch; the static scratch holds %zu (n_chains * K * tiles "
                  "must be <= %zu)",
                  n_chains, K, tiles, need, kNoAllocScratchBytes,
                  (kNoAllocScratchBytes - 256) / sizeof(double));
        return E_ARG;
    }
    ChainArgs<double> g{};
    g.qc = (double*)q_chain;
    g.pc = (double*)p_chain;
    g.gc = (double*)grad_chain;
    g.logp = (double*)logp_chain;
    g.q0 = (const double*)q_init;
    g.p0 = (const double*)p_init;
    g.m = (const double*)inv_mass;
    g.m_cs = n;
    g.n = n;
    g.chains = n_chains;
    g.K = K;
    g.eps = eps;
    g.he = 0.5 * eps;
    g.mode = 0;
    g.scale = -0.5;
    g.cst = 0.0;
    g.cst_dev = (const double*)base;
    if (tiles > 1) g.partial = (double*)(base + 256);
    // Every slot the kernels read is written earlier in the same call (the
    // constant by k_gauss_const, each partial by its tile), so nothing in
    // the shared array needs clearing between calls.
    k_gauss_const<<<1, 256, 0, c.stream>>>((const double*)prec, n, (double*)base);
    count_launch();
    return launch_family(c, g, FamGauss64{(const double*)prec, 0.0, mu});
}
