// k_nuts.cu -- the NUTS tree builder's per-level logic on the device.
//
// eXMC's NUTS tree builder (PLAN_FUSED_LEAPFROG.md:331-358) extends every
// chain speculatively with the fused leapfrog chain and then walks the new
// leaves: divergence, the generalized U-turn checks of the balanced subtree
// and of its merge with the tree so far, multinomial selection of a leaf and
// the biased move into the subtree (Betancourt 2017, "A Conceptual
// Introduction to Hamiltonian Monte Carlo", A.3-A.4).  These kernels do that
// walk where the leaves are -- in a device store that the chain calls write
// into -- so that no trajectory crosses PCIe.  Two drivers: nxv_nuts_start /
// nxv_nuts_level take the store rows of each active chain's next leaves from
// a host that keeps that bookkeeping (speculative extension, as eXMC calls
// the chain); nxv_nuts_start_layout / nxv_nuts_level_layout keep the tree
// ends, depth and leaf counts on the device, with every chain's level-l
// leaves at fixed store rows, so that a host only launches one start, one
// chain call and one level kernel per level and reads one flag.
//
// Store: q, p (p in the sign it was integrated with: negated for backward
// leaves), logp and kinetic energy per row; H = -logp + KE.
#include "../../include/nx_vulkan_shim.h"
#include "kernels.h"
#include "ops_common.cuh"

#include <math.h>

#include <algorithm>
#include <mutex>

namespace nxv {
namespace {

constexpr int kNT = 256;          // threads per chain
constexpr int kNW = kNT / 32;
constexpr int kMaxLeaves = 2048;  // leaves per level: 2^(max depth - 1), max depth 12
constexpr int kMaxDepth = 12;
static_assert(kMaxLeaves == 1 << (kMaxDepth - 1), "a level holds 2^(depth - 1) leaves");
constexpr double kMaxDeltaH = 1000.0;

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = add_(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
__device__ __forceinline__ double warp_max(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// Block sums of R values (every thread passes its R partials; all threads
// get the totals, added in warp order).
template <int R>
__device__ __forceinline__ void block_sums(double (&v)[R], double (*sm)[kNW]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < R; r++) v[r] = warp_sum(v[r]);
    __syncthreads();
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; r++) sm[r][warp] = v[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; r++) {
        double s = sm[r][0];
        for (int w = 1; w < kNW; w++) s = add_(s, sm[r][w]);
        v[r] = s;
    }
}

struct LevelArgs {
    const long long* rows;  // [A][n] store rows of the level's leaves, in time order
    const int* chain;       // [A] chain of each active slot
    const int* fwd;         // [A] 1: the subtree extends the tree forward in time
    const double* u_sel;    // [A] uniform for the leaf within the subtree
    const double* u_move;   // [A] uniform for the move into the subtree
    int n, d;
    const double* st_q;
    const double* st_p;
    const double* st_logp;
    const double* st_ke;
    const double* m;        // [d] inverse mass
    const double* H0;       // [C]
    double* logw;           // [C] log of the tree's weight
    double* rho;            // [C][d] the tree's summed momentum
    double* end_p;          // [2][C][d] momentum at the left (0) / right (1) end
    double* end_ps;         // [2][C][d] velocity at the ends
    double* sample;         // [C][d]
    int* active;            // [C] 1 while the tree keeps growing
    int* divergent;         // [C]
    double* node;           // [A][n][d] scratch: summed momenta of subtree nodes
    int C;
};

// One CTA per active chain.  Subtree U-turn check: node [a, b) of the
// balanced subtree is the merge of [a, m) and [m, b); level by level the
// node sums are built in `node` (node[a] holds the sum of [a, a + size)),
// and every merge is tested as the host tree builder tests it:
//   ps_first . rho > 0 and ps_last . rho > 0 (rho = rho_A + rho_B),
//   (rho_A + p_B,first) against ps_A,first and ps_B,first,
//   (rho_B + p_A,last) against ps_A,last and ps_B,last.
// The walk of chain c over its level's leaves rows(0) .. rows(n - 1) (time
// order); nd: the chain's [n][d] node scratch.
template <class Rows>
__device__ __forceinline__ void level_walk(const LevelArgs& a, int c, bool fwd, double u_sel,
                                           double u_move, double* nd, Rows rows) {
    __shared__ double h[kMaxLeaves];
    __shared__ double cs[kMaxLeaves];
    __shared__ double red[8][kNW];
    __shared__ int s_ok, s_sel;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = a.n, d = a.d;
    const double sg = fwd ? 1.0 : -1.0;  // backward leaves were integrated with -p
    const double H0 = a.H0[c];
    // the merge's operands (the tree's summed momentum and ends, the
    // subtree's first and last leaf, the inverse mass): nothing before the
    // merge changes them, so with one element per thread (d <= kNT) they
    // are loaded here, under the latency of the walk's first loads
    const size_t CD = (size_t)a.C * d;
    double* rho = a.rho + (size_t)c * d;
    const double* lp = a.end_p + (size_t)c * d;        // tree, left end
    const double* lps = a.end_ps + (size_t)c * d;
    const double* rp = a.end_p + CD + (size_t)c * d;   // tree, right end
    const double* rps = a.end_ps + CD + (size_t)c * d;
    const double* p_first = a.st_p + (size_t)rows(0) * d;
    const double* p_last = a.st_p + (size_t)rows(n - 1) * d;
    const bool pre = d <= kNT;
    double x_rho = 0.0, x_lp = 0.0, x_lps = 0.0, x_rp = 0.0, x_rps = 0.0, x_pf = 0.0,
           x_pl = 0.0, x_m = 0.0;
    if (pre && tid < d) {
        x_rho = rho[tid];
        x_lp = lp[tid];
        x_lps = lps[tid];
        x_rp = rp[tid];
        x_rps = rps[tid];
        x_pf = p_first[tid];
        x_pl = p_last[tid];
        x_m = a.m[tid];
    }

    // H of every leaf, divergence (NaN counts as divergent)
    int div_l = 0;
    for (int j = tid; j < n; j += kNT) {
        const long long r = rows(j);
        const double hj = sub_(a.st_ke[r], a.st_logp[r]);
        h[j] = hj;
        if (!(sub_(hj, H0) <= kMaxDeltaH)) div_l = 1;
    }
    const int div = __syncthreads_or(div_l);

    // a single leaf is its own node sum; with two or more, the first round
    // (size 2) reads the leaves themselves
    if (n == 1 && warp == 0) {
        const double* src = a.st_p + (size_t)rows(0) * d;
        for (int i = lane; i < d; i += 32) nd[i] = mul_(sg, src[i]);
    }
    if (tid == 0) s_ok = 1;
    __syncthreads();
    for (int size = 2; size <= n; size *= 2) {
        const int half = size / 2;
        for (int t = warp; t < n / size; t += kNW) {
            const int a0 = t * size, mid = a0 + half, b1 = a0 + size - 1;
            const double* pf = a.st_p + (size_t)rows(a0) * d;
            const double* pal = a.st_p + (size_t)rows(mid - 1) * d;
            const double* pbf = a.st_p + (size_t)rows(mid) * d;
            const double* pl = a.st_p + (size_t)rows(b1) * d;
            double s[6] = {0, 0, 0, 0, 0, 0};
            for (int i = lane; i < d; i += 32) {
                const double mi = a.m[i];
                const double vf = mul_(sg, pf[i]), val = mul_(sg, pal[i]);
                const double vbf = mul_(sg, pbf[i]), vl = mul_(sg, pl[i]);
                // size 2: the halves are single leaves (a0 = mid - 1, mid = b1)
                const double rA = size == 2 ? vf : nd[(size_t)a0 * d + i];
                const double rB = size == 2 ? vbf : nd[(size_t)mid * d + i];
                const double r = add_(rA, rB);
                const double v2 = add_(rA, vbf), v3 = add_(rB, val);
                s[0] = add_(s[0], mul_(mul_(mi, vf), r));
                s[1] = add_(s[1], mul_(mul_(mi, vl), r));
                s[2] = add_(s[2], mul_(mul_(mi, vf), v2));
                s[3] = add_(s[3], mul_(mul_(mi, vbf), v2));
                s[4] = add_(s[4], mul_(mul_(mi, val), v3));
                s[5] = add_(s[5], mul_(mul_(mi, vl), v3));
                nd[(size_t)a0 * d + i] = r;
            }
            bool ok = true;
#pragma unroll
            for (int k = 0; k < 6; k++) ok = ok && warp_sum(s[k]) > 0.0;
            if (lane == 0 && !ok) s_ok = 0;
        }
        __syncthreads();
    }
    const bool ok_sub = s_ok != 0 && !div;

    // multinomial choice of a leaf: w = -H (0 for every leaf of a divergent
    // subtree), weights exp(w - max w), chosen where the running sum first
    // reaches u * total
    double wmax = -INFINITY;
    for (int j = tid; j < n; j += kNT) wmax = fmax(wmax, div ? 0.0 : -h[j]);
    wmax = warp_max(wmax);
    if (lane == 0) red[0][warp] = wmax;
    __syncthreads();
    wmax = red[0][0];
    for (int w = 1; w < kNW; w++) wmax = fmax(wmax, red[0][w]);
    // per-thread contiguous chunk: local prefix sums, then chunk offsets
    const int per = (n + kNT - 1) / kNT, j0 = tid * per, j1 = min(n, j0 + per);
    double run = 0.0;
    for (int j = j0; j < j1; j++) {
        run = add_(run, exp(sub_(div ? 0.0 : -h[j], wmax)));
        cs[j] = run;
    }
    __shared__ double chunk[kNT];
    chunk[tid] = run;
    __syncthreads();
    if (tid == 0) {
        double acc = 0.0;
        const int nch = (n + per - 1) / per;  // chunks that hold leaves
        for (int t = 0; t < nch; t++) {
            const double v = chunk[t];
            chunk[t] = acc;  // offset of chunk t
            acc = add_(acc, v);
        }
        red[1][0] = acc;  // total
        s_sel = n - 1;
    }
    __syncthreads();
    const double tot = red[1][0], target = mul_(u_sel, tot);
    for (int j = j0; j < j1; j++) {
        const double cdf = add_(cs[j], chunk[tid]);
        if (!(cdf < target)) {
            atomicMin(&s_sel, j);
            break;
        }
    }
    __syncthreads();
    const int sel = s_sel;
    const double logw_sub = add_(wmax, log(tot));
    const double logw_old = a.logw[c];
    const bool move = u_move < exp(fmin(0.0, sub_(logw_sub, logw_old)));
    if (ok_sub && move) {
        const double* src = a.st_q + (size_t)rows(sel) * d;
        for (int i = tid; i < d; i += kNT) a.sample[(size_t)c * d + i] = src[i];
    }

    // merge with the tree so far; A is the earlier of (tree, subtree) in time
    const double* rho_sub = nd;  // node[0]: the sum of all n leaves
    double s[6] = {0, 0, 0, 0, 0, 0};
    for (int i = tid; i < d; i += kNT) {
        const double mi = pre ? x_m : a.m[i];
        const double rhoi = pre ? x_rho : rho[i];
        const double lpi = pre ? x_lp : lp[i], lpsi = pre ? x_lps : lps[i];
        const double rpi = pre ? x_rp : rp[i], rpsi = pre ? x_rps : rps[i];
        const double fp = mul_(sg, pre ? x_pf : p_first[i]);
        const double lsp = mul_(sg, pre ? x_pl : p_last[i]);
        const double fps = mul_(mi, fp), lps_ = mul_(mi, lsp);
        const double rA = fwd ? rhoi : rho_sub[i], rB = fwd ? rho_sub[i] : rhoi;
        const double pAl = fwd ? rpi : lsp;
        const double psAf = fwd ? lpsi : fps, psAl = fwd ? rpsi : lps_;
        const double pBf = fwd ? fp : lpi;
        const double psBf = fwd ? fps : lpsi, psBl = fwd ? lps_ : rpsi;
        const double r = add_(rA, rB), v2 = add_(rA, pBf), v3 = add_(rB, pAl);
        s[0] = add_(s[0], mul_(psAf, r));
        s[1] = add_(s[1], mul_(psBl, r));
        s[2] = add_(s[2], mul_(psAf, v2));
        s[3] = add_(s[3], mul_(psBf, v2));
        s[4] = add_(s[4], mul_(psAl, v3));
        s[5] = add_(s[5], mul_(psBl, v3));
    }
    block_sums<6>(s, red);
    bool ok_m = true;
#pragma unroll
    for (int k = 0; k < 6; k++) ok_m = ok_m && s[k] > 0.0;
    const bool cont = ok_sub && ok_m;
    // every thread has read rho, the ends and node[0] (block_sums synchronised)
    for (int i = tid; i < d; i += kNT) {
        if (cont) rho[i] = add_(pre ? x_rho : rho[i], rho_sub[i]);
        if (ok_sub) {
            // the subtree's far end becomes the tree's end on its side
            const double pe = pre ? (fwd ? x_pl : x_pf) : (fwd ? p_last : p_first)[i];
            const double v = mul_(sg, pe);
            double* ep = a.end_p + (fwd ? CD : 0) + (size_t)c * d;
            double* eps_ = a.end_ps + (fwd ? CD : 0) + (size_t)c * d;
            ep[i] = v;
            eps_[i] = mul_(pre ? x_m : a.m[i], v);
        }
    }
    if (tid == 0) {
        if (ok_sub) {
            // log(e^logw + e^logw_sub)
            const double hi = fmax(logw_old, logw_sub), lo = fmin(logw_old, logw_sub);
            a.logw[c] = hi == -INFINITY ? hi : add_(hi, log1p(exp(sub_(lo, hi))));
        }
        a.active[c] = cont ? 1 : 0;
        if (div) a.divergent[c] = 1;
    }
}

// One CTA per active slot: store rows, chain, direction and uniforms from
// the host.
__global__ void __launch_bounds__(kNT) k_nuts_level(LevelArgs a) {
    const int slot = blockIdx.x;
    const long long* rows = a.rows + (size_t)slot * a.n;
    level_walk(a, a.chain[slot], a.fwd[slot] != 0, a.u_sel[slot], a.u_move[slot],
               a.node + (size_t)slot * a.n * a.d, [rows](int j) { return rows[j]; });
}

// Device-driven levels: every chain's n leaves of this level are store rows
// base + c n .. base + c n + n - 1 in integration order; u[0][C] decides
// the direction (forward when >= 0.5), u[1][C] the leaf and u[2][C] the
// move.  One CTA per chain; chains whose tree has stopped return at once.
struct LayoutArgs {
    long long base;
    const double* u;       // [3][C] uniforms of this level
    long long* end_row;    // [2][C] store row of the tree's left / right end leaf (-1: the start)
    int* depth;            // [C]
    int* n_leapfrog;       // [C]
    int* any;              // optional: set to 1 by every chain that keeps building
    int level;
};

// Starting point of chain c's next extension: its tree's end leaf on the
// side u_dir picks, or (q0[c], +-p0[c]) while that side has none (or the
// row is outside the store).
__device__ __forceinline__ void start_point(double* qs, double* ps, const double* q0,
                                            const double* p0, const double* st_q,
                                            const double* st_p, const long long* end_row,
                                            double u_dir, int c, int C, int d,
                                            long long st_rows) {
    const bool fwd = u_dir >= 0.5;
    long long r = end_row[(fwd ? C : 0) + c];
    if (r >= st_rows) r = -1;  // not a row of this store: restart from the initial point
    const double sg = fwd ? 1.0 : -1.0;
    for (int k = threadIdx.x; k < d; k += kNT) {
        const size_t o = (size_t)c * d + k;
        if (r >= 0) {
            qs[o] = st_q[(size_t)r * d + k];
            ps[o] = st_p[(size_t)r * d + k];
        } else {
            qs[o] = q0[o];
            ps[o] = mul_(sg, p0[o]);
        }
    }
}

__global__ void __launch_bounds__(kNT) k_nuts_level_layout(LevelArgs a, LayoutArgs L) {
    const int c = blockIdx.x, n = a.n, C = a.C;
    if (a.active[c] == 0) return;
    const bool fwd = L.u[c] >= 0.5;
    const long long first = L.base + (long long)c * n;
    level_walk(a, c, fwd, L.u[C + c], L.u[2 * C + c], a.node + (size_t)c * n * a.d,
               [first, fwd, n](int j) { return fwd ? first + j : first + (n - 1 - j); });
    if (threadIdx.x == 0) {
        // the last leaf integrated is the tree's new end on its side
        L.end_row[(fwd ? C : 0) + c] = first + n - 1;
        L.depth[c] = L.level + 1;
        L.n_leapfrog[c] += n;
        if (L.any && a.active[c]) *L.any = 1;  // written by this thread in level_walk
    }
}

// H0 = -logp(q) + KE(p) for the Gaussian target, logp(q) = -0.5 sum
// prec (q - mu)^2 + logp_const; one warp per chain.
__global__ void __launch_bounds__(kNT) k_nuts_energy(double* H0, double* neg_H0, const double* q,
                                                     const double* p, const double* prec,
                                                     const double* m, double mu,
                                                     double logp_const, int C, int d) {
    const int c = blockIdx.x * kNW + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (c >= C) return;
    double u = 0.0, k = 0.0;
    for (int i = lane; i < d; i += 32) {
        const double dq = sub_(q[(size_t)c * d + i], mu), pi = p[(size_t)c * d + i];
        u = add_(u, mul_(mul_(prec[i], dq), dq));
        k = add_(k, mul_(mul_(pi, pi), m[i]));
    }
    u = warp_sum(u);
    k = warp_sum(k);
    if (lane == 0) {
        const double h = add_(sub_(mul_(0.5, u), logp_const), mul_(0.5, k));
        H0[c] = h;
        if (neg_H0) neg_H0[c] = -h;  // the tree's initial log weight
    }
}

// Starting points of a speculative extension: chain chain[i] continues from
// store row src_row[i] (the last leaf in its direction), or from the
// initial point (q0, dir[i] * p0) when src_row[i] < 0.
__global__ void __launch_bounds__(kNT) k_nuts_start(double* qs, double* ps, const double* q0,
                                                    const double* p0, const double* st_q,
                                                    const double* st_p, const int* chain,
                                                    const long long* src_row, const int* dir,
                                                    int d) {
    const int i = blockIdx.x, c = chain[i];
    const long long r = src_row[i];
    for (int k = threadIdx.x; k < d; k += kNT) {
        if (r >= 0) {
            qs[(size_t)i * d + k] = st_q[(size_t)r * d + k];
            ps[(size_t)i * d + k] = st_p[(size_t)r * d + k];
        } else {
            qs[(size_t)i * d + k] = q0[(size_t)c * d + k];
            ps[(size_t)i * d + k] = mul_((double)dir[i], p0[(size_t)c * d + k]);
        }
    }
}

// Starting points of a device-driven level: chain c continues from its
// tree's end leaf on the side u_dir[c] picks (the initial point (q0, +-p0)
// while that side has none).
__global__ void __launch_bounds__(kNT) k_nuts_start_layout(double* qs, double* ps,
                                                           const double* q0, const double* p0,
                                                           const double* st_q, const double* st_p,
                                                           const long long* end_row,
                                                           const double* u_dir, int C, int d,
                                                           long long st_rows) {
    start_point(qs, ps, q0, p0, st_q, st_p, end_row, u_dir[blockIdx.x], blockIdx.x, C, d,
                st_rows);
}

// Starting points of level `level` computed from the directions alone, so
// that the level's chain call can run while the previous level's walk
// does: a chain still building at this level extended its tree at level j
// in direction u_j, and its end on a side is the last leaf of the latest
// level in that direction (the initial point while there is none).
// spec_end [2][C] holds those rows (the level kernels keep their own
// end_row); level - 1's last leaf is row prev_base + c n_prev + n_prev - 1.
// For chains that stopped, the point is never used.
__global__ void __launch_bounds__(kNT) k_nuts_start_spec(double* qs, double* ps,
                                                         const double* q0, const double* p0,
                                                         const double* st_q, const double* st_p,
                                                         long long* spec_end, const double* u_dir,
                                                         const double* u_prev, long long prev_base,
                                                         long long n_prev, int C, int d,
                                                         long long st_rows) {
    const int c = blockIdx.x;
    const bool fwd = u_dir[c] >= 0.5;
    long long r = -1;
    if (u_prev) {
        const bool fwd_prev = u_prev[c] >= 0.5;
        const long long last = prev_base + (long long)c * n_prev + n_prev - 1;
        r = fwd == fwd_prev ? last : spec_end[(fwd ? C : 0) + c];  // never the side written
        if (threadIdx.x == 0) spec_end[(fwd_prev ? C : 0) + c] = last;
    }
    if (r >= st_rows) r = -1;
    const double sg = fwd ? 1.0 : -1.0;
    for (int k = threadIdx.x; k < d; k += kNT) {
        const size_t o = (size_t)c * d + k;
        if (r >= 0) {
            qs[o] = st_q[(size_t)r * d + k];
            ps[o] = st_p[(size_t)r * d + k];
        } else {
            qs[o] = q0[o];
            ps[o] = mul_(sg, p0[o]);
        }
    }
}

// A transition's initial state, one CTA per chain: p0 = z / sqrt(inv_mass)
// in place (z: standard normal draws), sample = q0, rho and both tree ends
// = p0, end velocities p0 * inv_mass, flags (active, divergent, depth,
// leapfrog count) = (1, 0, 0, 0), end rows -1, the per-level flags 0.
__global__ void __launch_bounds__(kNT) k_nuts_init(double* z, const double* q0, const double* m,
                                                   double* sample, double* rho, double* end_p,
                                                   double* end_ps, int* flags,
                                                   long long* end_row, long long* spec_end,
                                                   int* any, int levels, int C, int d) {
    const int c = blockIdx.x;
    if (c == 0 && threadIdx.x < levels) any[threadIdx.x] = 0;  // per-level "still growing"
    const size_t CD = (size_t)C * d;
    for (int k = threadIdx.x; k < d; k += kNT) {
        const size_t o = (size_t)c * d + k;
        const double p = div_(z[o], __dsqrt_rn(m[k]));
        z[o] = p;
        sample[o] = q0[o];
        rho[o] = p;
        end_p[o] = p;
        end_p[CD + o] = p;
        const double v = mul_(p, m[k]);
        end_ps[o] = v;
        end_ps[CD + o] = v;
    }
    if (threadIdx.x == 0) {
        flags[c] = 1;
        flags[C + c] = 0;
        flags[2 * C + c] = 0;
        flags[3 * C + c] = 0;
        end_row[c] = -1;
        end_row[C + c] = -1;
        spec_end[c] = -1;
        spec_end[C + c] = -1;
    }
}

// Pinned host word per device for the per-level "any tree still growing" read.
std::mutex g_any_mu;
int* g_any_host[64] = {};

// Per device: a second stream for the level kernels of the one-call
// transition (the chain calls stay on the caller's stream) and two events.
struct NutsStreams {
    cudaStream_t aux = nullptr;
    cudaEvent_t chain_done = nullptr, level_done = nullptr;
};
NutsStreams g_nuts_streams[64];

NutsStreams* nuts_streams(int dev) {
    std::lock_guard<std::mutex> lk(g_any_mu);
    if (dev < 0 || dev >= 64) return nullptr;
    NutsStreams& s = g_nuts_streams[dev];
    if (!s.aux) {
        if (cudaStreamCreateWithFlags(&s.aux, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&s.chain_done, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&s.level_done, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
    }
    return &s;
}

int* any_host(int dev) {
    std::lock_guard<std::mutex> lk(g_any_mu);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!g_any_host[dev] && cudaHostAlloc(&g_any_host[dev], sizeof(int), cudaHostAllocDefault) !=
                                cudaSuccess) {
        cudaGetLastError();
        g_any_host[dev] = nullptr;
    }
    return g_any_host[dev];
}

}  // namespace
}  // namespace nxv

using namespace nxv;

namespace {
bool holds(const void* h, size_t bytes) { return h && nbytes(h) >= bytes; }
}  // namespace

extern "C" {

int nxv_nuts_energy(void* H0, void* q, void* p, void* prec, void* inv_mass, double mu,
                    double logp_const, unsigned int n_chains, unsigned int d) {
    if (!H0 || !q || !p || !prec || !inv_mass) return E_NULL;
    Ctx c;
    int rc = begin(c, {H0, q, p, prec, inv_mass});
    if (rc) return rc;
    const size_t CD = (size_t)n_chains * d * 8;
    if (!holds(H0, (size_t)n_chains * 8) || !holds(q, CD) || !holds(p, CD) ||
        !holds(prec, (size_t)d * 8) || !holds(inv_mass, (size_t)d * 8)) {
        set_error("nuts_energy: a buffer is smaller than n_chains x d");
        return E_ARG;
    }
    if (n_chains == 0 || d == 0) return OK;
    k_nuts_energy<<<(n_chains + kNW - 1) / kNW, kNT, 0, c.stream>>>(
        (double*)dptr(H0), nullptr, (const double*)dptr(q), (const double*)dptr(p),
        (const double*)dptr(prec), (const double*)dptr(inv_mass), mu, logp_const, (int)n_chains,
        (int)d);
    count_launch();
    return finish(c);
}

int nxv_nuts_start(void* qs, void* ps, void* q0, void* p0, void* st_q, void* st_p, void* chain,
                   void* src_row, void* dir, unsigned int n_need, unsigned int n_chains,
                   unsigned int d) {
    if (!qs || !ps || !q0 || !p0 || !st_q || !st_p || !chain || !src_row || !dir) return E_NULL;
    Ctx c;
    int rc = begin(c, {qs, ps, q0, p0, st_q, st_p, chain, src_row, dir});
    if (rc) return rc;
    const size_t ND = (size_t)n_need * d * 8, CD = (size_t)n_chains * d * 8;
    if (!holds(qs, ND) || !holds(ps, ND) || !holds(q0, CD) || !holds(p0, CD) ||
        !holds(chain, (size_t)n_need * 4) || !holds(src_row, (size_t)n_need * 8) ||
        !holds(dir, (size_t)n_need * 4)) {
        set_error("nuts_start: a buffer is smaller than its extent");
        return E_ARG;
    }
    if (n_need == 0 || d == 0) return OK;
    k_nuts_start<<<n_need, kNT, 0, c.stream>>>(
        (double*)dptr(qs), (double*)dptr(ps), (const double*)dptr(q0), (const double*)dptr(p0),
        (const double*)dptr(st_q), (const double*)dptr(st_p), (const int*)dptr(chain),
        (const long long*)dptr(src_row), (const int*)dptr(dir), (int)d);
    count_launch();
    return finish(c);
}

int nxv_nuts_level(void* rows, void* chain, void* fwd, void* u_sel, void* u_move,
                   unsigned int n_active, unsigned int n, unsigned int d, void* st_q, void* st_p,
                   void* st_logp, void* st_ke, void* inv_mass, void* H0, void* logw, void* rho,
                   void* end_p, void* end_ps, void* sample, void* active, void* divergent,
                   void* node, unsigned int n_chains) {
    if (!rows || !chain || !fwd || !u_sel || !u_move || !st_q || !st_p || !st_logp || !st_ke ||
        !inv_mass || !H0 || !logw || !rho || !end_p || !end_ps || !sample || !active ||
        !divergent || !node)
        return E_NULL;
    if (n == 0 || n > (unsigned)kMaxLeaves || (n & (n - 1)) != 0) {
        set_error("nuts_level: n must be a power of two up to %d", kMaxLeaves);
        return E_ARG;
    }
    Ctx c;
    int rc = begin(c, {rows, chain, fwd, u_sel, u_move, st_q, st_p, st_logp, st_ke, inv_mass, H0,
                       logw, rho, end_p, end_ps, sample, active, divergent, node});
    if (rc) return rc;
    const size_t A = n_active, C = n_chains, CD = C * d * 8;
    if (!holds(rows, A * n * 8) || !holds(chain, A * 4) || !holds(fwd, A * 4) ||
        !holds(u_sel, A * 8) || !holds(u_move, A * 8) || !holds(inv_mass, (size_t)d * 8) ||
        !holds(H0, C * 8) || !holds(logw, C * 8) || !holds(rho, CD) || !holds(end_p, 2 * CD) ||
        !holds(end_ps, 2 * CD) || !holds(sample, CD) || !holds(active, C * 4) ||
        !holds(divergent, C * 4) || !holds(node, A * n * d * 8)) {
        set_error("nuts_level: a buffer is smaller than its extent");
        return E_ARG;
    }
    if (A == 0 || d == 0) return OK;
    const size_t st_rows = nbytes(st_logp) / 8;
    if (!holds(st_q, st_rows * d * 8) || !holds(st_p, st_rows * d * 8) ||
        !holds(st_ke, st_rows * 8)) {
        set_error("nuts_level: the store's q/p/ke hold fewer rows than its logp");
        return E_ARG;
    }
    LevelArgs g;
    g.rows = (const long long*)dptr(rows);
    g.chain = (const int*)dptr(chain);
    g.fwd = (const int*)dptr(fwd);
    g.u_sel = (const double*)dptr(u_sel);
    g.u_move = (const double*)dptr(u_move);
    g.n = (int)n;
    g.d = (int)d;
    g.st_q = (const double*)dptr(st_q);
    g.st_p = (const double*)dptr(st_p);
    g.st_logp = (const double*)dptr(st_logp);
    g.st_ke = (const double*)dptr(st_ke);
    g.m = (const double*)dptr(inv_mass);
    g.H0 = (const double*)dptr(H0);
    g.logw = (double*)dptr(logw);
    g.rho = (double*)dptr(rho);
    g.end_p = (double*)dptr(end_p);
    g.end_ps = (double*)dptr(end_ps);
    g.sample = (double*)dptr(sample);
    g.active = (int*)dptr(active);
    g.divergent = (int*)dptr(divergent);
    g.node = (double*)dptr(node);
    g.C = (int)C;
    k_nuts_level<<<(unsigned)A, kNT, 0, c.stream>>>(g);
    count_launch();
    return finish(c);
}

int nxv_nuts_start_layout(void* qs, void* ps, void* q0, void* p0, void* st_q, void* st_p,
                          void* end_row, void* u_dir, unsigned int n_chains, unsigned int d) {
    if (!qs || !ps || !q0 || !p0 || !st_q || !st_p || !end_row || !u_dir) return E_NULL;
    Ctx c;
    int rc = begin(c, {qs, ps, q0, p0, st_q, st_p, end_row, u_dir});
    if (rc) return rc;
    const size_t CD = (size_t)n_chains * d * 8;
    if (!holds(qs, CD) || !holds(ps, CD) || !holds(q0, CD) || !holds(p0, CD) ||
        !holds(end_row, (size_t)n_chains * 16) || !holds(u_dir, (size_t)n_chains * 8)) {
        set_error("nuts_start_layout: a buffer is smaller than its extent");
        return E_ARG;
    }
    if (n_chains == 0 || d == 0) return OK;
    // end rows are read only below the store's row count
    const long long st_rows = (long long)std::min(nbytes(st_q), nbytes(st_p)) / ((long long)d * 8);
    k_nuts_start_layout<<<n_chains, kNT, 0, c.stream>>>(
        (double*)dptr(qs), (double*)dptr(ps), (const double*)dptr(q0), (const double*)dptr(p0),
        (const double*)dptr(st_q), (const double*)dptr(st_p), (const long long*)dptr(end_row),
        (const double*)dptr(u_dir), (int)n_chains, (int)d, st_rows);
    count_launch();
    return finish(c);
}

int nxv_nuts_level_layout(unsigned long long base_row, unsigned int n, unsigned int d, void* u,
                          void* st_q, void* st_p, void* st_logp, void* st_ke, void* inv_mass,
                          void* H0, void* logw, void* rho, void* end_p, void* end_ps,
                          void* sample, void* active, void* divergent, void* end_row,
                          void* depth, void* n_leapfrog, void* node, unsigned int n_chains,
                          unsigned int level) {
    if (!u || !st_q || !st_p || !st_logp || !st_ke || !inv_mass || !H0 || !logw || !rho ||
        !end_p || !end_ps || !sample || !active || !divergent || !end_row || !depth ||
        !n_leapfrog || !node)
        return E_NULL;
    if (n == 0 || n > (unsigned)kMaxLeaves || (n & (n - 1)) != 0) {
        set_error("nuts_level_layout: n must be a power of two up to %d", kMaxLeaves);
        return E_ARG;
    }
    Ctx c;
    int rc = begin(c, {u, st_q, st_p, st_logp, st_ke, inv_mass, H0, logw, rho, end_p, end_ps,
                       sample, active, divergent, end_row, depth, n_leapfrog, node});
    if (rc) return rc;
    const size_t C = n_chains, CD = C * d * 8;
    if (!holds(u, 3 * C * 8) || !holds(inv_mass, (size_t)d * 8) || !holds(H0, C * 8) ||
        !holds(logw, C * 8) || !holds(rho, CD) || !holds(end_p, 2 * CD) ||
        !holds(end_ps, 2 * CD) || !holds(sample, CD) || !holds(active, C * 4) ||
        !holds(divergent, C * 4) || !holds(end_row, 2 * C * 8) || !holds(depth, C * 4) ||
        !holds(n_leapfrog, C * 4) || !holds(node, C * n * d * 8)) {
        set_error("nuts_level_layout: a buffer is smaller than its extent");
        return E_ARG;
    }
    if (C == 0 || d == 0) return OK;
    const size_t rows_needed = (size_t)base_row + C * n;
    if (!holds(st_logp, rows_needed * 8) || !holds(st_ke, rows_needed * 8) ||
        !holds(st_q, rows_needed * d * 8) || !holds(st_p, rows_needed * d * 8)) {
        set_error("nuts_level_layout: the store holds fewer than base_row + n_chains * n rows");
        return E_ARG;
    }
    LevelArgs g{};
    g.n = (int)n;
    g.d = (int)d;
    g.st_q = (const double*)dptr(st_q);
    g.st_p = (const double*)dptr(st_p);
    g.st_logp = (const double*)dptr(st_logp);
    g.st_ke = (const double*)dptr(st_ke);
    g.m = (const double*)dptr(inv_mass);
    g.H0 = (const double*)dptr(H0);
    g.logw = (double*)dptr(logw);
    g.rho = (double*)dptr(rho);
    g.end_p = (double*)dptr(end_p);
    g.end_ps = (double*)dptr(end_ps);
    g.sample = (double*)dptr(sample);
    g.active = (int*)dptr(active);
    g.divergent = (int*)dptr(divergent);
    g.node = (double*)dptr(node);
    g.C = (int)C;
    LayoutArgs L;
    L.base = (long long)base_row;
    L.u = (const double*)dptr(u);
    L.end_row = (long long*)dptr(end_row);
    L.depth = (int*)dptr(depth);
    L.n_leapfrog = (int*)dptr(n_leapfrog);
    L.any = nullptr;
    L.level = (int)level;
    k_nuts_level_layout<<<(unsigned)C, kNT, 0, c.stream>>>(g, L);
    count_launch();
    return finish(c);
}

int nxv_nuts_transition_layout(void* sample, void* flags, void* H0, void* q0, void* inv_mass,
                               void* prec, double mu, double logp_const, double eps,
                               unsigned int n_chains, unsigned int d, unsigned int max_depth,
                               unsigned int seed) {
    if (!sample || !flags || !H0 || !q0 || !inv_mass || !prec) return E_NULL;
    if (max_depth == 0 || max_depth > (unsigned)kMaxDepth) {
        set_error("nuts_transition_layout: max_depth must be 1 .. %d", kMaxDepth);
        return E_ARG;
    }
    Ctx c;
    int rc = begin(c, {sample, flags, H0, q0, inv_mass, prec});
    if (rc) return rc;
    const size_t C = n_chains, D = d, CD = C * D;
    if (!holds(sample, CD * 8) || !holds(flags, 4 * C * 4) || !holds(H0, C * 8) ||
        !holds(q0, CD * 8) || !holds(inv_mass, D * 8) || !holds(prec, D * 8)) {
        set_error("nuts_transition_layout: a buffer is smaller than its extent");
        return E_ARG;
    }
    if (C == 0 || D == 0) return OK;
    const size_t L = max_depth, nmax = size_t(1) << (L - 1), R = C * ((size_t(1) << L) - 1);
    // scratch regions, each 256-byte aligned: momenta (z -> p0), uniforms,
    // rho, tree ends and end velocities, log weight, start points, end rows,
    // the flag word, the leaf store (q, p, logp, ke) and the level scratch
    // (node sums, the chain call's gradients)
    size_t off = 0;
    auto take = [&off](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~size_t(255);
        return o;
    };
    const size_t o_z = take(CD * 8), o_u = take(L * 3 * C * 8), o_rho = take(CD * 8),
                 o_ep = take(2 * CD * 8), o_eps = take(2 * CD * 8), o_logw = take(C * 8),
                 o_qs = take(CD * 8), o_ps = take(CD * 8), o_er = take(2 * C * 8),
                 o_se = take(2 * C * 8),
                 o_any = take(L * 4), o_cst = take(8), o_sq = take(R * D * 8), o_sp = take(R * D * 8),
                 o_sl = take(R * 8), o_sk = take(R * 8), o_node = take(C * nmax * D * 8),
                 o_grad = take(C * nmax * D * 8);
    ScratchGuard guard(c);
    char* base = (char*)scratch(c, off, kScratchNuts);
    if (!base) return E_CUDA;
    int* any_h = any_host(c.dev->id);
    NutsStreams* ns = nuts_streams(c.dev->id);
    if (!any_h || !ns) {
        set_error("nuts_transition_layout: pinned host word or stream creation failed");
        return E_CUDA;
    }
    double* z = (double*)(base + o_z);
    const double* u = (const double*)(base + o_u);
    long long* end_row = (long long*)(base + o_er);
    long long* spec_end = (long long*)(base + o_se);
    int* any = (int*)(base + o_any);
    double* st_q = (double*)(base + o_sq);
    double* st_p = (double*)(base + o_sp);
    double* st_logp = (double*)(base + o_sl);
    double* st_ke = (double*)(base + o_sk);
    double* qs = (double*)(base + o_qs);
    double* ps = (double*)(base + o_ps);
    const double* m = (const double*)dptr(inv_mass);
    const double* pr = (const double*)dptr(prec);
    const double* q0d = (const double*)dptr(q0);
    int* fl = (int*)dptr(flags);
    // Philox keys of the momenta and of the uniforms
    const uint32_t kp = seed, ku = seed ^ 0x5BD1E995u;
    if ((rc = launch_random(c, F64, z, CD, kp, 1))) return rc;
    if ((rc = launch_random(c, F64, base + o_u, L * 3 * C, ku, 0))) return rc;
    k_nuts_init<<<(unsigned)C, kNT, 0, c.stream>>>(
        z, q0d, m, (double*)dptr(sample), (double*)(base + o_rho), (double*)(base + o_ep),
        (double*)(base + o_eps), fl, end_row, spec_end, any, (int)L, (int)C, (int)D);
    k_nuts_energy<<<(unsigned)((C + kNW - 1) / kNW), kNT, 0, c.stream>>>(
        (double*)dptr(H0), (double*)(base + o_logw), q0d, z, pr, m, mu, logp_const, (int)C,
        (int)D);
    count_launch(2);
    // the chain's log-density constant, once for every level's chain call
    if ((rc = launch_gauss_const(c, pr, D, base + o_cst))) return rc;
    LevelArgs g{};
    g.d = (int)D;
    g.st_q = st_q;
    g.st_p = st_p;
    g.st_logp = st_logp;
    g.st_ke = st_ke;
    g.m = m;
    g.H0 = (const double*)dptr(H0);
    g.logw = (double*)(base + o_logw);
    g.rho = (double*)(base + o_rho);
    g.end_p = (double*)(base + o_ep);
    g.end_ps = (double*)(base + o_eps);
    g.sample = (double*)dptr(sample);
    g.active = fl;
    g.divergent = fl + C;
    g.node = (double*)(base + o_node);
    g.C = (int)C;
    LayoutArgs Lg{};
    Lg.end_row = end_row;
    Lg.depth = fl + 2 * C;
    Lg.n_leapfrog = fl + 3 * C;
    // Two streams: the caller's runs the start kernels and the chain calls,
    // the library's second stream the level kernels.  The starting points
    // of level l + 1 depend only on the directions and on rows written by
    // earlier chain calls (k_nuts_start_spec), so level l + 1's chain call
    // runs while level l's walk does; level l + 1's walk waits for both.
    // When the flag after level l says that every tree has stopped, the
    // chain call of level l + 1 has been issued for nothing.
    const long long RR = (long long)R;
    auto chain_level = [&](size_t level) -> int {
        const size_t n = size_t(1) << level, row0 = C * (n - 1);
        const double* ul = u + level * 3 * C;
        const double* up = level ? ul - 3 * C : nullptr;
        const long long nprev = level ? (long long)(n / 2) : 0;
        const long long prev0 = level ? (long long)(C * (n / 2 - 1)) : 0;
        k_nuts_start_spec<<<(unsigned)C, kNT, 0, c.stream>>>(qs, ps, q0d, z, st_q, st_p, spec_end,
                                                           ul, up, prev0, nprev, (int)C, (int)D,
                                                           RR);
        count_launch();
        int r2 = launch_chain_gauss_f64(c, st_q + row0 * D, st_p + row0 * D, base + o_grad,
                                        st_logp + row0, qs, ps, m, pr, 0.0, mu, D, C,
                                        (unsigned)n, eps, st_ke + row0, true, base + o_cst);
        if (r2) return r2;
        cudaError_t e = cudaEventRecord(ns->chain_done, c.stream);
        return e == cudaSuccess ? OK : cuda_fail(e, "nuts_transition_layout: event");
    };
    if ((rc = chain_level(0))) return rc;
    for (size_t level = 0; level < L; level++) {
        const size_t n = size_t(1) << level, row0 = C * (n - 1);
        g.n = (int)n;
        Lg.base = (long long)row0;
        Lg.u = u + level * 3 * C;
        Lg.level = (int)level;
        Lg.any = any + level;
        cudaError_t e = cudaStreamWaitEvent(ns->aux, ns->chain_done, 0);
        if (e != cudaSuccess) return cuda_fail(e, "nuts_transition_layout: stream wait");
        k_nuts_level_layout<<<(unsigned)C, kNT, 0, ns->aux>>>(g, Lg);
        count_launch();
        // one 4-byte read per level from the third on (the first two levels
        // always continue: for chains whose tree has stopped, a level's
        // kernels change nothing but scratch, and a level of 1, 2 or 4
        // steps costs less than a wait for the flag)
        const bool check = level >= 2 && level + 1 < L;
        if (check)
            e = cudaMemcpyAsync(any_h, any + level, sizeof(int), cudaMemcpyDeviceToHost, ns->aux);
        if (e == cudaSuccess) e = cudaEventRecord(ns->level_done, ns->aux);
        if (e != cudaSuccess) return cuda_fail(e, "nuts_transition_layout: level");
        if (level + 1 < L && (rc = chain_level(level + 1))) return rc;
        if (check) {
            e = cudaEventSynchronize(ns->level_done);
            if (e != cudaSuccess) return cuda_fail(e, "nuts_transition_layout: flag read");
            if (*any_h == 0) break;
        }
    }
    // the outputs (and the next call's use of the scratch) follow the last
    // level kernel in the caller's stream order
    cudaError_t e = cudaStreamWaitEvent(c.stream, ns->level_done, 0);
    if (e != cudaSuccess) return cuda_fail(e, "nuts_transition_layout: stream wait");
    return finish(c);
}

}  // extern "C"
