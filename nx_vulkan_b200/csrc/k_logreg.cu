// k_logreg.cu -- batched HMC leapfrog for Bayesian logistic regression (f64).
//
// Target (the second leapfrog workload; no reference kernel exists -- the
// reference would run it through the unfused evaluator with dot on the host):
//   z = X q,  r = y - sigmoid(z),  grad(q) = X^T r - q,
//   logp(q) = sum_j [y_j z_j - softplus(z_j)] - 0.5 |q|^2,
// batched over C chains: Z = Q . X^T (C x N_obs, K = D) and G = R . X - Q
// (C x D, K = N_obs).
//
// Fused path (D <= 104): one kernel per gradient.  CTA (s, b) owns chains
// [128 b, 128 b + 128) and observations [L s, L s + L).  Its Q block stays in
// shared memory; X streams through in tiles of 32 observations (cp.async,
// double-buffered).  Two warps serve each block of 16 chains (16 warps per
// CTA, at most 128 registers each).  Per tile, each computes a 16 x 16 half
// of the block's Z with DMMA (m16n8k4 f64), turns it into R = y - sigmoid(Z)
// and the logp terms in registers and parks R in shared memory; after a
// named barrier of the pair each accumulates half of the block's 16 x D
// G += R . X_tile with DMMA.  Z never leaves the SM; each
// CTA writes one G partial and one logp partial per chain.  A fold kernel
// (one CTA per chain) sums the partials in slice order (deterministic),
// subtracts q, completes the step (final half-kick, trajectory writes,
// logp) and performs the next step's half-kick and drift.  Two launches
// per leapfrog step; X is read from L2 (8 MB at the benchmark size).
//
// General path (D > 104): Z and G on the DMMA GEMM, G split along N_obs,
// the same fold.
#include "kernels.h"
#include "ops_common.cuh"

#include <math.h>

#include <algorithm>
#include <functional>

namespace nxv {

namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with programmatic stream serialization: the kernel's CTAs may start
// while the previous kernel on the stream finishes; each kernel here calls
// griddep_wait() before it touches memory the previous one writes or reads,
// and griddep_launch() only after that wait.  NXV_LR_PDL=0 launches plainly.
bool lr_pdl() {
    const char* e = getenv("NXV_LR_PDL");
    return !(e && e[0] == '0');
}

template <typename... KArgs, typename... Args>
int launch_pdl(Ctx& c, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
               const char* what, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = lr_pdl() ? 1 : 0;
    // these kernels let their successor start right after their own wait,
    // before they write: no successor may load early
    pdl_record_all(c);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    count_launch();
    return OK;
}

// D += A(16x4) . B(4x8), f64.  A register r: (row g + 8r, col tig);
// B: (row tig, col g); D registers: (g, 2tig), (g, 2tig+1), (g+8, 2tig),
// (g+8, 2tig+1), with g = lane / 4, tig = lane % 4.
__device__ __forceinline__ void dmma4(double (&d)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%0,%1,%2,%3};\n"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

// Residual and logp term of one observation: r = y - sigmoid(z),
// t = y z - softplus(z), softplus(z) = max(z, 0) + log1p(exp(-|z|)).
__device__ __forceinline__ double lr_resid(double z, double yj, double& t) {
    double s = div_(1.0, add_(1.0, exp(-z)));
    double sp = add_((z > 0.0 ? z : 0.0), log1p(exp(-fabs(z))));
    t = sub_(mul_(yj, z), sp);
    return sub_(yj, s);
}

// ---- fused gradient ---------------------------------------------------------------

// DT: 8-wide tiles over the padded model dimension DP = 8 DT >= D.
// NW: warps per CTA, warp w owns chains [16w, 16w + 16).  BN: observations
// per X tile.
template <int DT, int NW_, int BN_> struct LrCfg {
    static constexpr int NW = NW_;
    static constexpr int NT = 32 * NW;    // threads
    static constexpr int BC = 16 * NW;    // chains per CTA
    static constexpr int BN = BN_;
    static constexpr int DP = 8 * DT;
    // Row strides (doubles) == 4 or 12 mod 16: every fragment load below hits
    // 16 distinct 8-byte bank pairs per half-warp.
    static constexpr int DS = DP + 4;
    static constexpr int RS = BN + 4;
    static constexpr int Q_OFF = 0;
    static constexpr int X_OFF = BC * DS;
    static constexpr int R_OFF = X_OFF + 2 * BN * DS;
    static constexpr int Y_OFF = R_OFF + BC * RS;  // y tiles, 2 x BN
    static constexpr int TOTAL = Y_OFF + 2 * BN;
    static constexpr size_t BYTES = (size_t)TOTAL * 8;
    static_assert(DS % 16 == 4 || DS % 16 == 12, "DS bank layout");
    static_assert(RS % 16 == 4 || RS % 16 == 12, "RS bank layout");
    static_assert((X_OFF * 8) % 16 == 0 && (DS * 8) % 16 == 0, "cp.async alignment");
};

// Z block of one warp: z[n] (16 x 8) += Q rows . X_tile rows n*8 .. n*8+7 over
// k in [0, DP).  qa: this lane's A element (row g, col tig); xb: this lane's B
// element (tile row g, col tig).  FULL: all NZ observation groups hold data
// (no per-MMA guard); otherwise only the first ntz.
// D += A(16x8) . B(8x8), f64: A registers (row g, col tig), (g + 8, tig),
// (g, tig + 4), (g + 8, tig + 4); B registers (row tig, col g), (tig + 4, g).
__device__ __forceinline__ void dmma8(double (&d)[4], double a0, double a1, double a2, double a3,
                                      double b0, double b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(a2), "d"(a3), "d"(b0), "d"(b1));
}

// Z uses the k = 8 shape when MK8: a warp's Z block has only NZ (2) chains
// of dependent MMAs, so it is bound by their latency, and the k = 8 shape
// halves the length of each chain (DP is a multiple of 8).
template <int NZ, int DP, int DS, bool FULL, bool MK8>
__device__ __forceinline__ void z_block(double (&z)[NZ][4], const double* qa, const double* xb,
                                        unsigned ntz) {
    if constexpr (MK8) {
        static_assert(DP % 8 == 0, "k8 steps");
#pragma unroll
        for (int kk = 0; kk < DP; kk += 8) {
            const double a0 = qa[kk], a1 = qa[kk + 8 * DS], a2 = qa[kk + 4],
                         a3 = qa[kk + 4 + 8 * DS];
#pragma unroll
            for (int n = 0; n < NZ; n++)
                if (FULL || n < (int)ntz)
                    dmma8(z[n], a0, a1, a2, a3, xb[n * 8 * DS + kk], xb[n * 8 * DS + kk + 4]);
        }
    } else {
#pragma unroll
        for (int kk = 0; kk < DP; kk += 4) {
            const double a0 = qa[kk], a1 = qa[kk + 8 * DS];
#pragma unroll
            for (int n = 0; n < NZ; n++)
                if (FULL || n < (int)ntz) dmma4(z[n], a0, a1, xb[n * 8 * DS + kk]);
        }
    }
}

// G block of one warp: gacc[n] (16 x 8) += R rows . X_tile columns n*8 ..
// n*8+7 over the tile's observations k in [0, kv).  rw: this lane's A element
// (row g, col tig); xr: this lane's B element (tile row tig, col g).
template <int DT, int BN, int DS, int RS, bool FULL>
__device__ __forceinline__ void g_block(double (&gacc)[DT][4], const double* rw, const double* xr,
                                        int kv, int ncnt) {
#pragma unroll
    for (int kk = 0; kk < BN; kk += 4) {
        if (FULL || kk < kv) {
            const double a0 = rw[kk], a1 = rw[8 * RS + kk];
#pragma unroll
            for (int n = 0; n < DT; n++)
                if (n < ncnt) dmma4(gacc[n], a0, a1, xr[kk * DS + n * 8]);
        }
    }
}

// part[s][c][d] = sum over j in slice s of R[c][j] X[j][d];
// lpart[c][s] = sum over j in slice s of (y_j z_cj - softplus(z_cj)).
// vecX: X rows are 16-byte aligned (D even, X aligned) and use cp.async.
// SPLIT warps share each 16-chain block: warp w serves block w % NW as part
// wh = w / NW, taking observation tiles [wh NZW, wh NZW + NZW) of Z and
// model-dimension tiles [wh DTW, ...) of G; with SPLIT = 2 a named barrier
// per block orders the two warps' R writes before either reads R.
// The gradient of slice s, chain block cb (one CTA); PDL: the kernel was
// launched with programmatic dependent launch (wait before touching q/part).
template <int DT, int NW, int BN_, int SPLIT, bool MK8, bool PDL>
__device__ __forceinline__ void lr_grad_body(
    const double* __restrict__ q, const double* __restrict__ X, const double* __restrict__ y,
    double* __restrict__ part, double* __restrict__ lpart, unsigned C, unsigned D, unsigned n_obs,
    unsigned L, unsigned S, int vecX, unsigned s, unsigned cb, double* lr_smem) {
    using G = LrCfg<DT, NW, BN_>;
    constexpr int BN = G::BN, DS = G::DS, RS = G::RS, DP = G::DP, NT = G::NT * SPLIT;
    constexpr int NZ = BN / 8;              // 8-observation tiles of Z per chain block
    constexpr int NZW = NZ / SPLIT;         // ... per warp
    constexpr int DTW = (DT + SPLIT - 1) / SPLIT;  // 8-wide tiles of G per warp
    static_assert(NZ % SPLIT == 0, "SPLIT must divide the Z tiles");
    double* Qs = lr_smem + G::Q_OFF;
    double* Xs = lr_smem + G::X_OFF;
    double* Rs = lr_smem + G::R_OFF;
    double* Ys = lr_smem + G::Y_OFF;
    const unsigned c0 = cb * G::BC;
    const unsigned j0 = s * L;
    const unsigned j1 = max(j0, min(n_obs, j0 + L));  // empty past the last observation
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;
    const int pr = warp % NW, wh = warp / NW;    // chain block, part
    const int zoff = wh * NZW;                   // first Z observation tile
    const int nbase = wh * DTW;                  // first G tile
    const int ncnt = DT - nbase < DTW ? DT - nbase : DTW;

    // Both X buffers start as zeros: the padded columns [D, DP) stay zero and
    // rows past a partial tile hold finite values (R is zero there).
    for (int i = tid; i < 2 * BN * DS; i += NT) Xs[i] = 0.0;
    // Launched with programmatic dependent launch after the previous step's
    // fold: everything above overlaps its tail; q (written by the fold) is
    // read, and part (read by the fold) written, only after this wait.
    if constexpr (PDL) {
        griddep_wait();
        griddep_launch();
    }
    // Q block: zeros outside [c0, C) x [0, D); the rest by cp.async (with the
    // first X tile) when rows are 16-byte aligned, else by plain loads.
    const bool vq = (D & 1) == 0;
    const unsigned hd = D >> 1;  // 16-byte chunks per row on the vector paths
    const unsigned crows = min((unsigned)G::BC, C - c0);
    for (int i = tid; i < G::BC * DS; i += NT) {
        const int r = i / DS, col = i - r * DS;
        if ((unsigned)r < crows && col < (int)D) {
            if (!vq) Qs[i] = q[(size_t)(c0 + r) * D + col];
        } else {
            Qs[i] = 0.0;
        }
    }
    __syncthreads();
    if (vq) {
        const unsigned total = crows * hd;
        for (unsigned ch = tid; ch < total; ch += NT) {
            const unsigned r = ch / hd, cc = (ch - r * hd) * 2;
            cp_async16(Qs + r * DS + cc, q + (size_t)(c0 + r) * D + cc);
        }
    }

    const unsigned ntile = (j1 - j0 + BN - 1) / BN;
    auto load_x = [&](unsigned t, int buf) {
        const unsigned jt = j0 + t * BN;
        const unsigned rows = min((unsigned)BN, j1 - jt);
        double* dst = Xs + buf * BN * DS;
        const double* src = X + (size_t)jt * D;
        if (tid < (int)rows) cp_async8(Ys + buf * BN + tid, y + jt + tid);
        if (vecX) {
            const unsigned total = rows * hd;
            for (unsigned ch = tid; ch < total; ch += NT) {
                const unsigned r = ch / hd, cc = (ch - r * hd) * 2;
                cp_async16(dst + r * DS + cc, src + (size_t)r * D + cc);
            }
        } else {
            const unsigned total = rows * D;
            for (unsigned i = tid; i < total; i += NT) {
                const unsigned r = i / D, col = i - r * D;
                dst[r * DS + col] = src[i];
            }
        }
    };

    double gacc[DTW][4];
#pragma unroll
    for (int t = 0; t < DTW; t++)
#pragma unroll
        for (int e = 0; e < 4; e++) gacc[t][e] = 0.0;
    // logp of rows g and g + 8: sum of y z - max(z, 0), running product of
    // den and the sum of its flushed logs
    double lsum[2] = {0.0, 0.0}, lprod[2] = {1.0, 1.0}, llog[2] = {0.0, 0.0};
    const double* qa = Qs + (pr * 16 + g) * DS + tig;
    double* rw = Rs + pr * 16 * RS;

    load_x(0, 0);
    cp_commit();
    for (unsigned t = 0; t < ntile; t++) {
        if (t + 1 < ntile) load_x(t + 1, (t + 1) & 1);
        cp_commit();
        cp_wait<1>();
        __syncthreads();
        const double* xb = Xs + (t & 1) * BN * DS;
        const unsigned jt = j0 + t * BN;
        const unsigned valid = min((unsigned)BN, j1 - jt);
        const unsigned ntz = (valid + 7) >> 3;  // 8-observation tiles holding data

        // A 16-chain block past the last chain (C below the CTA's 128) has
        // no work: its warp pair skips the MMAs, the residual and its named
        // barrier together and only meets the CTA barriers.
        if (pr * 16 < (int)crows) {
        // Z block (16 chains x this warp's observation tiles) = Q . X_tile^T.
        double z[NZW][4];
#pragma unroll
        for (int n = 0; n < NZW; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) z[n][e] = 0.0;
        const int ntzw = min(max((int)ntz - zoff, 0), NZW);
        if (ntzw == NZW)
            z_block<NZW, DP, DS, true, MK8>(z, qa, xb + (zoff * 8 + g) * DS + tig, ntzw);
        else
            z_block<NZW, DP, DS, false, MK8>(z, qa, xb + (zoff * 8 + g) * DS + tig, ntzw);

        // R = y - sigmoid(Z) into this warp's rows of Rs (zero past the slice),
        // with e = exp(-|z|), den = 1 + e in [1, 2], sigmoid(z) = (z >= 0 ? 1 : e)
        // / den.  The 8 reciprocals of a row come from one division (batch
        // inversion: prefix products, one reciprocal, back-substitution).  The
        // logp term y z - softplus(z) = y z - max(z, 0) - log(den): the first
        // part is summed, den enters a running product whose log is taken
        // once per 64 tiles.
        const double* yb = Ys + (t & 1) * BN;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            double ev[2 * NZW], dn[2 * NZW], pf[2 * NZW], rc[2 * NZW];
#pragma unroll
            for (int n = 0; n < NZW; n++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int i = 2 * n + e;
                    const bool ok = (unsigned)((zoff + n) * 8 + 2 * tig + e) < valid;
                    ev[i] = ok ? lean::exp(-fabs(z[n][2 * h + e])) : 0.0;
                    dn[i] = add_(1.0, ev[i]);
                }
            pf[0] = dn[0];
#pragma unroll
            for (int i = 1; i < 2 * NZW; i++) pf[i] = mul_(pf[i - 1], dn[i]);
            double inv = div_(1.0, pf[2 * NZW - 1]);
#pragma unroll
            for (int i = 2 * NZW - 1; i > 0; i--) {
                rc[i] = mul_(inv, pf[i - 1]);
                inv = mul_(inv, dn[i]);
            }
            rc[0] = inv;
            lprod[h] = mul_(lprod[h], pf[2 * NZW - 1]);
#pragma unroll
            for (int n = 0; n < NZW; n++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int i = 2 * n + e;
                    const unsigned col = (zoff + n) * 8 + 2 * tig + e;
                    double r = 0.0;
                    if (col < valid) {
                        const double zz = z[n][2 * h + e], yj = yb[col];
                        r = sub_(yj, mul_(zz >= 0.0 ? 1.0 : ev[i], rc[i]));
                        lsum[h] = add_(lsum[h], sub_(mul_(yj, zz), zz > 0.0 ? zz : 0.0));
                    }
                    rw[(g + 8 * h) * RS + col] = r;
                }
            if ((t & 63) == 63) {
                llog[h] = add_(llog[h], log(lprod[h]));
                lprod[h] = 1.0;
            }
        }
        if constexpr (SPLIT == 2)  // both warps of the block have written their R columns
            asm volatile("bar.sync %0, %1;" ::"r"(pr + 1), "r"(64) : "memory");
        else
            __syncwarp();

        // G block (16 chains x this warp's model tiles) += R . X_tile.
        const int kv = (int)((valid + 3) >> 2) << 2;
        const double* xr = xb + tig * DS + g + nbase * 8;
        if (kv == BN)
            g_block<DTW, BN, DS, RS, true>(gacc, rw + g * RS + tig, xr, kv, ncnt);
        else
            g_block<DTW, BN, DS, RS, false>(gacc, rw + g * RS + tig, xr, kv, ncnt);
        }  // active chain block
        __syncthreads();  // buffer t & 1 and Rs are rewritten next iteration
    }
    cp_wait<0>();

    // Partials out: the G block goes through shared memory (the Q block's
    // space, free after the last tile's barrier) as a dense [crows][D] array,
    // which is also the layout of part[s][c0 .. c0 + crows) -- one contiguous
    // range written with coalesced 16-byte stores.
    double* Gs = Qs;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int row = pr * 16 + g + 8 * h;
#pragma unroll
        for (int n = 0; n < DTW; n++) {
            if (n >= ncnt) continue;
            const unsigned d = (nbase + n) * 8 + 2 * tig;
            if (vq) {
                if (d < D)
                    *reinterpret_cast<double2*>(Gs + row * D + d) =
                        make_double2(gacc[n][2 * h], gacc[n][2 * h + 1]);
            } else {
                if (d < D) Gs[row * D + d] = gacc[n][2 * h];
                if (d + 1 < D) Gs[row * D + d + 1] = gacc[n][2 * h + 1];
            }
        }
    }
    __syncthreads();
    {
        double* dst = part + ((size_t)s * C + c0) * D;
        if (vq) {
            const unsigned total = crows * hd;
            for (unsigned k = tid; k < total; k += NT)
                reinterpret_cast<double2*>(dst)[k] = reinterpret_cast<const double2*>(Gs)[k];
        } else {
            const unsigned total = crows * D;
            for (unsigned k = tid; k < total; k += NT) dst[k] = Gs[k];
        }
    }
    // logp partial per chain: sum over the four lanes of a row (tig), a fixed
    // pairing so the result is identical on every lane.
    double lp0 = sub_(lsum[0], add_(llog[0], log(lprod[0])));
    double lp1 = sub_(lsum[1], add_(llog[1], log(lprod[1])));
    lp0 = add_(lp0, __shfl_xor_sync(0xffffffffu, lp0, 1));
    lp0 = add_(lp0, __shfl_xor_sync(0xffffffffu, lp0, 2));
    lp1 = add_(lp1, __shfl_xor_sync(0xffffffffu, lp1, 1));
    lp1 = add_(lp1, __shfl_xor_sync(0xffffffffu, lp1, 2));
    if constexpr (SPLIT == 2) {  // part 0 + part 1, in that order
        __shared__ double lpx[NW][16];
        if (wh == 1 && tig == 0) {
            lpx[pr][g] = lp0;
            lpx[pr][g + 8] = lp1;
        }
        __syncthreads();
        if (wh == 1) return;
        lp0 = add_(lp0, lpx[pr][g]);
        lp1 = add_(lp1, lpx[pr][g + 8]);
    }
    if (tig == 0) {
        const unsigned ca = c0 + pr * 16 + g, cb = ca + 8;
        if (ca < C) lpart[(size_t)ca * S + s] = lp0;
        if (cb < C) lpart[(size_t)cb * S + s] = lp1;
    }
}

template <int DT, int NW, int BN_, int SPLIT, bool MK8>
__global__ void __launch_bounds__(32 * NW * SPLIT, SPLIT == 1 ? 8 / NW : 1)
k_lr_grad(const double* __restrict__ q, const double* __restrict__ X,
          const double* __restrict__ y, double* __restrict__ part, double* __restrict__ lpart,
          unsigned C, unsigned D, unsigned n_obs, unsigned L, unsigned S, int vecX) {
    extern __shared__ __align__(16) double lr_smem[];
    lr_grad_body<DT, NW, BN_, SPLIT, MK8, true>(q, X, y, part, lpart, C, D, n_obs, L, S, vecX,
                                                blockIdx.x, blockIdx.y, lr_smem);
}

// ---- general path: residual over Z from the GEMM -------------------------------------

constexpr int kRT = 256;  // residual kernel threads
constexpr int kRE = 4;    // observations per residual thread

// R = y - sigmoid(Z) in place; lpart[c][blk] = sum over the block's j of
// y z - softplus(z).
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
            double te;
            zr[j] = lr_resid(zr[j], y[j], te);
            t = add_(t, te);
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

// ---- fold + leapfrog update ----------------------------------------------------------

constexpr int kFT = 1024;  // fold threads per chain (10 slice groups of a 100-dim chain)

// In-order sum of a[t * stride] for t in [t0, t1), t1 > t0: the loads of a
// block of 8 are all issued before its additions (the partials come from L2;
// a load behind each addition would leave the fold latency-bound).
// COH: the data were written earlier in the same (persistent) kernel by other
// CTAs: load through L2 (ld.global.cg), never from a non-coherent cache.
template <bool COH>
__device__ __forceinline__ double ld_part(const double* p) {
    if constexpr (COH) return __ldcg(p);
    else return *p;
}

template <bool COH = false>
__device__ __forceinline__ double sum_rows(const double* __restrict__ a, size_t stride, int t0,
                                           int t1) {
    double s = 0.0;
    for (int t = t0; t < t1; t += 8) {
        double v[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
            v[u] = t + u < t1 ? ld_part<COH>(a + (size_t)(t + u) * stride) : 0.0;
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (t + u < t1) s = t + u == t0 ? v[u] : add_(s, v[u]);
    }
    return s;
}

// One CTA per chain: g = sum_s part[s] - q.  With H > 1 the S slices are cut
// into H contiguous groups, thread (h, i) sums group h of element i in slice
// order and the H group sums are added in group order (a fixed order, so the
// result is deterministic).  With write_step: p = p + he*g, rows of step k
// written to the trajectories and logp[c][k] = sum lpart - 0.5 |q|^2.  With
// drift: the next step's half-kick and drift, p_h = p + he*g;
// q = q + eps*p_h; p = p_h  (inverse mass 1).
// fold_sm: [H][D] doubles; sm: one double per warp of the CTA.  Every thread
// of the CTA calls it (H * D <= blockDim.x).
template <bool COH>
__device__ __forceinline__ void lr_fold_chain(
    unsigned c, const double* __restrict__ part, int S, int H, size_t CD, double* __restrict__ q,
    double* __restrict__ p, const double* __restrict__ lpart, unsigned nblk, size_t D, double eps,
    double he, int write_step, int drift, unsigned k, unsigned K, double* qc, double* pc,
    double* gc, double* logp, double* fold_sm, double* sm) {
    __syncthreads();  // fold_sm and sm may still be read for the previous chain
    const double* pc0 = part + (size_t)c * D;
    // this thread's position and momentum (D <= blockDim.x in the fused
    // path), loaded while the partials are summed
    const bool one = D <= blockDim.x && threadIdx.x < D;
    const double q_pre = one ? q[(size_t)c * D + threadIdx.x] : 0.0;
    const double p_pre = one ? p[(size_t)c * D + threadIdx.x] : 0.0;
    // and the chain's logp partials (lane j: j, j + 32, j + 64, ...)
    double l = 0.0;
    if (write_step && threadIdx.x < 32) {
        const double* lp = lpart + (size_t)c * nblk;
        for (unsigned j0 = threadIdx.x; j0 < nblk; j0 += 4 * 32) {
            double v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                v[u] = j0 + 32 * u < nblk ? ld_part<COH>(lp + j0 + 32 * u) : 0.0;
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (j0 + 32 * u < nblk) l = add_(l, v[u]);
        }
    }
    if (H > 1) {
        const unsigned tid = threadIdx.x;
        if (tid < (unsigned)H * D) {
            const unsigned h = tid / (unsigned)D, i = tid - h * (unsigned)D;
            const int t0 = (int)((size_t)h * S / H), t1 = (int)((size_t)(h + 1) * S / H);
            fold_sm[tid] = sum_rows<COH>(pc0 + i, CD, t0, t1);
        }
        __syncthreads();
    }
    double qq = 0.0;
    for (size_t i = threadIdx.x; i < D; i += blockDim.x) {
        const size_t o = (size_t)c * D + i;
        double s;
        if (H > 1) {
            s = fold_sm[i];
            for (int h = 1; h < H; h++) s = add_(s, fold_sm[(size_t)h * D + i]);
        } else {
            s = sum_rows<COH>(pc0 + i, CD, 0, S);
        }
        double qi = one ? q_pre : q[o];
        double gi = sub_(s, qi);
        qq = add_(qq, mul_(qi, qi));
        double pi = one ? p_pre : p[o];
        if (write_step) {
            pi = add_(pi, mul_(he, gi));
            size_t row = ((size_t)c * K + k) * D + i;
            qc[row] = qi;
            pc[row] = pi;
            gc[row] = gi;
        }
        if (drift) {
            double ph = add_(pi, mul_(he, gi));
            q[o] = add_(qi, mul_(eps, ph));
            pi = ph;
        }
        p[o] = pi;
    }
    if (!write_step) return;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) qq = add_(qq, __shfl_down_sync(0xffffffffu, qq, off));
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = qq;
    __syncthreads();
    if (threadIdx.x < 32) {
        // the chain's logp partials: lane j summed partials j, j + 32, ...
        // above (their loads issued together), then a fixed shuffle tree; the
        // order is the same on every call, so the result is deterministic
        const unsigned lane = threadIdx.x;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l = add_(l, __shfl_down_sync(0xffffffffu, l, off));
        if (lane == 0) {
            double sq = sm[0];
            for (int w = 1; w < (int)(blockDim.x >> 5); w++) sq = add_(sq, sm[w]);
            logp[(size_t)c * K + k] = sub_(l, mul_(0.5, sq));
        }
    }
}

__global__ void __launch_bounds__(kFT, 2)
k_lr_fold(const double* __restrict__ part, int S, int H, size_t CD, double* __restrict__ q,
          double* __restrict__ p, const double* __restrict__ lpart, unsigned nblk, size_t D,
          double eps, double he, int write_step, int drift, unsigned k, unsigned K, double* qc,
          double* pc, double* gc, double* logp) {
    extern __shared__ double fold_sm[];  // [H][D] group sums when H > 1
    __shared__ double sm[kFT / 32];
    // programmatic dependent launch: the partials of the gradient kernel
    // just before are read only after it has completed
    griddep_wait();
    griddep_launch();
    lr_fold_chain<false>(blockIdx.x, part, S, H, CD, q, p, lpart, nblk, D, eps, he, write_step,
                         drift, k, K, qc, pc, gc, logp, fold_sm, sm);
}

// NXV_LR_MK=4 keeps Z on the k = 4 MMA shape (default k = 8).
bool lr_mk8() {
    const char* e = getenv("NXV_LR_MK");
    return !(e && atoi(e) == 4);
}

template <int DT, int NW, int BN, int SPLIT, bool MK8>
int launch_lr_grad_mk(Ctx& c, const double* q, const double* X, const double* y, double* part,
                      double* lpart, unsigned C, unsigned D, unsigned n_obs, unsigned L,
                      unsigned S, int vecX) {
    using G = LrCfg<DT, NW, BN>;
    const size_t smem = G::BYTES;
    cudaError_t e = cudaFuncSetAttribute(k_lr_grad<DT, NW, BN, SPLIT, MK8>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_lr_grad)");
    dim3 grid(S, (C + G::BC - 1) / G::BC);
    return launch_pdl(c, k_lr_grad<DT, NW, BN, SPLIT, MK8>, grid, dim3(G::NT * SPLIT), smem,
                      "k_lr_grad", q, X, y, part, lpart, C, D, n_obs, L, S, vecX);
}

template <int DT, int NW, int BN, int SPLIT>
int launch_lr_grad(Ctx& c, const double* q, const double* X, const double* y, double* part,
                   double* lpart, unsigned C, unsigned D, unsigned n_obs, unsigned L, unsigned S,
                   int vecX) {
    if (lr_mk8())
        return launch_lr_grad_mk<DT, NW, BN, SPLIT, true>(c, q, X, y, part, lpart, C, D, n_obs,
                                                          L, S, vecX);
    return launch_lr_grad_mk<DT, NW, BN, SPLIT, false>(c, q, X, y, part, lpart, C, D, n_obs, L,
                                                       S, vecX);
}

// ---- persistent trajectory kernel -------------------------------------------------
//
// One cooperative launch per chain call: CTA (s, cb) computes its slice's
// gradient partials, all CTAs meet at a grid barrier, every CTA folds a
// share of the chains (chain c by CTA c mod the grid: slice sums in slice
// order, kick, drift, trajectory rows, logp), and a second barrier makes the
// new positions visible before the next gradient.  This replaces two
// launches per leapfrog step (the gradient kernel's 148 CTAs of 203 KB and
// the fold's) with two barriers.  Cooperative launch keeps every CTA
// resident, so a barrier cannot wait on a CTA that never runs; each wait is
// still bounded (about a second): on timeout the kernel records g_lr_error,
// leaves no copy in flight and returns.

__device__ int g_lr_error;  // 1 when a grid barrier's bounded wait ran out

// bar[0]: arrivals of the current barrier, bar[1]: generation.  Returns
// false (on every thread of the CTA) when the wait ran out here or another
// CTA reported a timeout.
__device__ __forceinline__ bool lr_grid_barrier(unsigned* bar, unsigned nctas) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        volatile unsigned* vgen = bar + 1;
        const unsigned gen = *vgen;
        __threadfence();
        if (atomicAdd(bar, 1u) == nctas - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            for (unsigned i = 0; *vgen == gen; i++) {
                if (i > (1u << 22)) {
                    ok = 0;
                    atomicExch(&g_lr_error, 1);
                    break;
                }
                if (i > 64) __nanosleep(256);
            }
        }
        __threadfence();
        s_ok = ok && *(volatile int*)&g_lr_error == 0;
    }
    __syncthreads();
    return s_ok != 0;
}

template <int DT, int NW, int BN_, int SPLIT, bool MK8>
__global__ void __launch_bounds__(32 * NW * SPLIT, 1)
k_lr_traj(const double* __restrict__ X, const double* __restrict__ y, double* __restrict__ q,
          double* __restrict__ p, double* __restrict__ part, double* __restrict__ lpart,
          unsigned C, unsigned D, unsigned n_obs, unsigned L, unsigned S, int vecX, int H,
          double eps, double he, unsigned K, double* qc, double* pc, double* gc, double* logp,
          unsigned* bar) {
    extern __shared__ __align__(16) double lr_smem[];
    __shared__ double sm_red[NW * SPLIT];
    const unsigned nctas = gridDim.x * gridDim.y;
    const unsigned cta = blockIdx.y * gridDim.x + blockIdx.x;
    const size_t CD = (size_t)C * D;
    for (unsigned it = 0; it <= K; it++) {
        lr_grad_body<DT, NW, BN_, SPLIT, MK8, false>(q, X, y, part, lpart, C, D, n_obs, L, S,
                                                     vecX, blockIdx.x, blockIdx.y, lr_smem);
        if (!lr_grid_barrier(bar, nctas)) return;
        // it = 0: the gradient at q0, then step 0's half-kick and drift;
        // it = k + 1: step k's final half-kick and rows, then step k+1's drift
        for (unsigned c = cta; c < C; c += nctas)
            lr_fold_chain<true>(c, part, (int)S, H, CD, q, p, lpart, S, D, eps, he, it > 0 ? 1 : 0,
                          it < K ? 1 : 0, it > 0 ? it - 1 : 0, K, qc, pc, gc, logp, lr_smem,
                          sm_red);
        if (it < K && !lr_grid_barrier(bar, nctas)) return;
    }
}

// NXV_LR_PERSIST=1 selects the persistent kernel.  It is off by default:
// measured on B200 for 256 chains x X[10000, 100], L = 16, one trajectory
// takes 1.140 ms persistent against 0.985 ms with two launches per step on
// programmatic dependent launch -- the fold with one 512-thread CTA per SM
// (2 chains on most CTAs) and the two barriers cost more than the launches
// they replace, which the dependent launch already overlaps.
bool lr_persist() {
    const char* e = getenv("NXV_LR_PERSIST");
    return e && e[0] == '1';
}

// Launches k_lr_traj when the grid fits the GPU at once (cooperative
// launch); E_KERNEL when it does not (the caller takes the per-step
// launches).
template <int DT, int NW, int BN, int SPLIT, bool MK8>
int launch_lr_traj_mk(Ctx& c, const double* X, const double* y, double* q, double* p,
                      double* part, double* lpart, unsigned C, unsigned D, unsigned n_obs,
                      unsigned L, unsigned S, int vecX, int H, double eps, double he, unsigned K,
                      double* qc, double* pc, double* gc, double* logp, unsigned* bar) {
    using G = LrCfg<DT, NW, BN>;
    const size_t smem = G::BYTES;
    auto kern = k_lr_traj<DT, NW, BN, SPLIT, MK8>;
    if ((size_t)H * D > (size_t)G::NT * SPLIT || (size_t)H * D * 8 > smem) return E_KERNEL;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_lr_traj)");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, G::NT * SPLIT, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    const dim3 grid(S, (C + G::BC - 1) / G::BC);
    if ((size_t)grid.x * grid.y > (size_t)per_sm * c.dev->sm_count) return E_KERNEL;
    NXV_CK(cudaMemsetAsync(bar, 0, 2 * sizeof(unsigned), c.stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(G::NT * SPLIT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, X, y, q, p, part, lpart, C, D, n_obs, L, S, vecX, H, eps,
                           he, K, qc, pc, gc, logp, bar);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(k_lr_traj)");
    count_launch();
    return OK;
}

template <int DT, int NW, int BN, int SPLIT>
int launch_lr_traj(Ctx& c, const double* X, const double* y, double* q, double* p, double* part,
                   double* lpart, unsigned C, unsigned D, unsigned n_obs, unsigned L, unsigned S,
                   int vecX, int H, double eps, double he, unsigned K, double* qc, double* pc,
                   double* gc, double* logp, unsigned* bar) {
    if (lr_mk8())
        return launch_lr_traj_mk<DT, NW, BN, SPLIT, true>(c, X, y, q, p, part, lpart, C, D, n_obs,
                                                          L, S, vecX, H, eps, he, K, qc, pc, gc,
                                                          logp, bar);
    return launch_lr_traj_mk<DT, NW, BN, SPLIT, false>(c, X, y, q, p, part, lpart, C, D, n_obs, L,
                                                       S, vecX, H, eps, he, K, qc, pc, gc, logp,
                                                       bar);
}


}  // namespace

int lr_traj_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_lr_error, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) {
        int z = 0;
        cudaMemcpyToSymbol(g_lr_error, &z, sizeof(int));
    }
    return v;
}

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
    const bool fused = D <= 104;
    const double he = 0.5 * eps;
    size_t S, L;
    unsigned nblk;
    // chains per fused-gradient CTA: 128, or 32 / 64 when there are no more
    // chains than that (a shard of the chains on each of several GPUs), so
    // that no CTA carries empty chain blocks: 32 chains 0.468 -> 0.383 ms per
    // trajectory (two 32-chain CTAs per SM: 0.389)
    const int lr_nw = C <= 32 ? 2 : (C <= 64 ? 4 : 8);
    if (fused) {
        // Slices: enough CTAs to cover the SMs once; L a multiple of 8.
        const size_t cblk = (C + 16 * lr_nw - 1) / (16 * lr_nw);
        S = ((size_t)c.dev->sm_count + cblk - 1) / cblk;
        L = ((n_obs + S - 1) / S + 7) & ~(size_t)7;
        S = (n_obs + L - 1) / L;
        nblk = (unsigned)S;
    } else {
        // split-K slices for G = R . X: enough CTAs to cover the SMs.
        const size_t ctas_mn = ((C + 127) / 128) * ((D + 127) / 128);
        S = (2 * (size_t)c.dev->sm_count + ctas_mn - 1) / ctas_mn;
        L = (n_obs + S - 1) / S;
        L = (L + 15) & ~(size_t)15;  // keep slice starts 16-byte aligned, BK multiple
        S = (n_obs + L - 1) / L;
        nblk = (unsigned)((n_obs + kRT * kRE - 1) / (kRT * kRE));
    }
    // scratch: q | p [C][D] | lpart [C][nblk] | part [S][C][D] | (general) Xt [D][N], Z [C][N]
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += (bytes + 255) & ~(size_t)255;
        return o;
    };
    size_t oq = take(CD * 8), op = take(CD * 8), oL = take(C * nblk * 8), oP = take(S * CD * 8);
    size_t oB = take(2 * sizeof(unsigned));  // grid-barrier state of the persistent kernel
    size_t oXt = fused ? 0 : take(D * n_obs * 8), oZ = fused ? 0 : take(C * n_obs * 8);
    ScratchGuard guard(c);
    char* base = (char*)scratch(c, off);
    if (!base) return E_CUDA;
    double* q = (double*)(base + oq);
    double* p = (double*)(base + op);
    double* lp = (double*)(base + oL);
    double* part = (double*)(base + oP);
    NXV_CK(cudaMemcpyAsync(q, q0, CD * 8, cudaMemcpyDeviceToDevice, c.stream));
    NXV_CK(cudaMemcpyAsync(p, p0, CD * 8, cudaMemcpyDeviceToDevice, c.stream));

    std::function<int()> grad;
    GemmP<double> G1{}, G2{};
    if (fused) {
        const int vecX = (D % 2 == 0) && ((uintptr_t)X % 16 == 0);
        const unsigned Cu = (unsigned)C, Du = (unsigned)D, Nu = (unsigned)n_obs,
                       Lu = (unsigned)L, Su = (unsigned)S;
        const double* Xd = (const double*)X;
        const double* yd = (const double*)y;
        // warps per 16-chain block: 2 by default (0.955 vs 1.042 ms per
        // trajectory of the 256-chain X[10000,100] workload); NXV_LR_SPLIT=1
        // selects one warp per block.
        const char* sv = getenv("NXV_LR_SPLIT");
        const int split = (sv && atoi(sv) == 1) ? 1 : 2;
        grad = [=, &c]() -> int {
            if (split == 2 && lr_nw == 2) {
                if (D <= 32)
                    return launch_lr_grad<4, 2, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
                if (D <= 64)
                    return launch_lr_grad<8, 2, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
                return launch_lr_grad<13, 2, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
            }
            if (split == 2 && lr_nw == 4) {
                if (D <= 32)
                    return launch_lr_grad<4, 4, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
                if (D <= 64)
                    return launch_lr_grad<8, 4, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
                return launch_lr_grad<13, 4, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
            }
            if (split == 2) {
                if (D <= 32)
                    return launch_lr_grad<4, 8, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
                if (D <= 64)
                    return launch_lr_grad<8, 8, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
                return launch_lr_grad<13, 8, 32, 2>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
            }
            if (D <= 32)
                return launch_lr_grad<4, 8, 32, 1>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
            if (D <= 64)
                return launch_lr_grad<8, 8, 32, 1>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
            return launch_lr_grad<13, 8, 32, 1>(c, q, Xd, yd, part, lp, Cu, Du, Nu, Lu, Su, vecX);
        };
    } else {
        double* Xt = (double*)(base + oXt);
        double* Z = (double*)(base + oZ);
        int rc = enqueue_transpose(c, F64, Xt, X, (unsigned)n_obs, (unsigned)D);
        if (rc) return rc;
        G1.A = q; G1.B = Xt; G1.C = Z;  // Z = Q . Xt
        G1.M = (int)C; G1.N = (int)n_obs; G1.K = (int)D;
        G1.lda = (int)D; G1.ldb = (int)n_obs; G1.ldc = (int)n_obs;
        G1.batch = 1;
        G2.A = Z; G2.B = (const double*)X; G2.C = part;  // part[s] = R[:, s] . X[s, :]
        G2.M = (int)C; G2.N = (int)D; G2.K = (int)n_obs;
        G2.lda = (int)n_obs; G2.ldb = (int)D; G2.ldc = (int)D;
        G2.sC = (long long)CD; G2.ksplit = (int)L; G2.batch = (int)S;
        grad = [&, Z, nblk]() -> int {
            int r = gemm_f64(c, G1);
            if (r) return r;
            dim3 rg(nblk, (unsigned)C);
            k_lr_resid<<<rg, kRT, 0, c.stream>>>(Z, (const double*)y, n_obs, lp, nblk);
            count_launch();
            return gemm_f64(c, G2);
        };
    }
    // slice groups of the fold: as many as fit kFT threads, at most S
    const int H = (D <= (size_t)kFT / 2) ? (int)std::min<size_t>(S, kFT / D) : 1;
    const size_t fold_smem = H > 1 ? (size_t)H * D * 8 : 0;
    auto fold = [&](int write_step, int drift, unsigned k) {
        return launch_pdl(c, k_lr_fold, dim3((unsigned)C), dim3(kFT), fold_smem, "k_lr_fold",
                          (const double*)part, (int)S, H, CD, q, p, (const double*)lp, nblk, D,
                          eps, he, write_step, drift, k, K, (double*)qc, (double*)pc,
                          (double*)gc, (double*)logp);
    };
    if (fused && lr_persist() && D % 2 == 0) {
        // (even D: the gradient loads its Q block by cp.async.cg, through L2,
        // which sees the positions the previous fold wrote in the same kernel)
        // one cooperative launch for the whole trajectory when the grid fits
        const int vecX = (D % 2 == 0) && ((uintptr_t)X % 16 == 0);
        const char* sv = getenv("NXV_LR_SPLIT");
        const int split = (sv && atoi(sv) == 1) ? 1 : 2;
        const unsigned Cu = (unsigned)C, Du = (unsigned)D, Nu = (unsigned)n_obs,
                       Lu = (unsigned)L, Su = (unsigned)S;
        const int Hp = (int)std::max<size_t>(1, std::min<size_t>(S, (size_t)(256 * split) / D));
        const double* Xd = (const double*)X;
        const double* yd = (const double*)y;
        unsigned* bar = (unsigned*)(base + oB);
        double *qcd = (double*)qc, *pcd = (double*)pc, *gcd = (double*)gc, *lgd = (double*)logp;
        int rc;
        if (split == 2) {
            if (D <= 32)
                rc = launch_lr_traj<4, 8, 32, 2>(c, Xd, yd, q, p, part, lp, Cu, Du, Nu, Lu, Su, vecX,
                                                 Hp, eps, he, K, qcd, pcd, gcd, lgd, bar);
            else if (D <= 64)
                rc = launch_lr_traj<8, 8, 32, 2>(c, Xd, yd, q, p, part, lp, Cu, Du, Nu, Lu, Su, vecX,
                                                 Hp, eps, he, K, qcd, pcd, gcd, lgd, bar);
            else
                rc = launch_lr_traj<13, 8, 32, 2>(c, Xd, yd, q, p, part, lp, Cu, Du, Nu, Lu, Su,
                                                  vecX, Hp, eps, he, K, qcd, pcd, gcd, lgd, bar);
        } else {
            if (D <= 32)
                rc = launch_lr_traj<4, 8, 32, 1>(c, Xd, yd, q, p, part, lp, Cu, Du, Nu, Lu, Su, vecX,
                                                 Hp, eps, he, K, qcd, pcd, gcd, lgd, bar);
            else if (D <= 64)
                rc = launch_lr_traj<8, 8, 32, 1>(c, Xd, yd, q, p, part, lp, Cu, Du, Nu, Lu, Su, vecX,
                                                 Hp, eps, he, K, qcd, pcd, gcd, lgd, bar);
            else
                rc = launch_lr_traj<13, 8, 32, 1>(c, Xd, yd, q, p, part, lp, Cu, Du, Nu, Lu, Su,
                                                  vecX, Hp, eps, he, K, qcd, pcd, gcd, lgd, bar);
        }
        if (rc == OK) return finish(c);
        if (rc != E_KERNEL) return rc;
    }
    // gradient at q0, then step 0's half-kick and drift
    int rc = grad();
    if (rc) return rc;
    if ((rc = fold(0, 1, 0))) return rc;
    for (unsigned k = 0; k < K; k++) {
        rc = grad();
        if (rc) return rc;
        if ((rc = fold(1, k + 1 < K, k))) return rc;
    }
    return finish(c);
}

}  // namespace nxv
