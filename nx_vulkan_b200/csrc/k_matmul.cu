// k_matmul.cu -- dense C = A . B (row-major), batched over blockIdx.z.
//
// f64: DMMA tensor cores (mma.sync m16n8k4 .f64).  tcgen05 has no f64 kind,
// so the FP64 tensor path on sm_100a is the warp-level DMMA instruction.
// f32: 3xTF32 split on the warp-level TF32 MMA (mma.sync m16n8k8 .tf32):
// x = hi + lo with hi = x rounded to nearest TF32 and lo = tf32(x - hi);
// C += Ahi.Bhi + Ahi.Blo + Alo.Bhi, accumulated in f32.  The error is of the
// order of f32 rounding (the dropped lo.lo term is ~2^-22 relative).
//
// Tiles: f64 products by default on 64x64 CTA tiles (4 warps, 32x32 warp
// tiles, BK 16, three CTAs per SM); the 128x128 schedule -- 8 warps in a 2
// (M) x 4 (N) grid with a 64x32 warp tile, one CTA per SM, a stream-K tail
// for the last wave -- serves the f32 path and NXV_GEMM_TILE=128.  Both: a
// 3-stage cp.async pipeline, shared-memory rows padded so that every
// fragment load is bank-conflict free (A rows are BK+4 elements; B rows are
// BN+4 doubles -- 4 mod 16 in 8-byte bank pairs -- or BN+8 floats -- 8 mod 32
// in 4-byte banks), zero-filled out-of-range chunks, and a scalar loader
// when a row is not 16-byte aligned.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "kernels.h"

namespace nxv {

namespace {

constexpr int BM = 128, BN = 128, STAGES = 3, NTH = 256;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int sz = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

}  // namespace

namespace {

// CTA tile geometry: BM x BN tiles, BK-deep k-tiles, WARPS_M x WARPS_N warps
// with (BM / WARPS_M) x (BN / WARPS_N) warp tiles, at least MINB CTAs per SM
// (launch bounds).  The default is the 128 x 128 tile of the stream-K
// schedule.
template <typename T, int BK_, int BM_ = BM, int BN_ = BN, int WARPS_M_ = 2, int WARPS_N_ = 4,
          int MINB_ = 1>
struct Cfg {
    using type = T;
    static constexpr int BM = BM_, BN = BN_, BK = BK_;
    static constexpr int WARPS_N = WARPS_N_, NTH = 32 * WARPS_M_ * WARPS_N_, MINB = MINB_;
    static constexpr int MI = BM / WARPS_M_ / 16, NJ = BN / WARPS_N_ / 8;  // fragments per warp
    static constexpr int AS = BK + 4;      // A row stride (elements)
    static constexpr int BS = BN + (sizeof(T) == 8 ? 4 : 8);  // B row stride (elements)
    static constexpr int A_ELEMS = BM * AS;
    static constexpr int B_ELEMS = BK * BS;
    static constexpr int STAGE = A_ELEMS + B_ELEMS;
    static constexpr size_t BYTES = (size_t)STAGES * STAGE * sizeof(T);
};

// 64 x 64 f64 tiles: 4 warps with 32 x 32 warp tiles, BK 16 -- 57 KB of
// shared memory and 150 registers per thread, so three CTAs share an SM and
// hide each other's pipeline fill and epilogue, and a product's tiles
// spread over the SMs to within a tile (64 x 256^3: 1024 tiles, 6.9 per SM,
// against 1.7 of the 128 x 128 tiles).  A and B rows of 20 and 68 doubles
// (4 mod 16) keep the fragment loads conflict-free as in the large tile.
using Small64 = Cfg<double, 16, 64, 64, 2, 2, 3>;

// Load one BMxBK tile of A and one BKxBN tile of B into stage buffers.
template <class S, typename T = typename S::type>
__device__ __forceinline__ void load_tile(T* sA, T* sB, const T* A, const T* B, int M, int N,
                                          int K, int lda, int ldb, int m0, int n0, int k0,
                                          bool vecA, bool vecB) {
    constexpr int EPC = 16 / sizeof(T);  // elements per 16-byte chunk
    constexpr int BM = S::BM, BN = S::BN, BK = S::BK, NTH = S::NTH;
    const int tid = threadIdx.x;
    // A: BM rows x BK cols
    constexpr int A_CHUNKS = BM * BK / EPC;
    for (int ch = tid; ch < A_CHUNKS; ch += NTH) {
        int r = ch / (BK / EPC), cc = (ch % (BK / EPC)) * EPC;
        int gm = m0 + r, gk = k0 + cc;
        T* dst = sA + r * S::AS + cc;
        if (vecA) {
            bool in = gm < M && gk + EPC <= K;
            const T* src = in ? A + (size_t)gm * lda + gk : A;
            if (in || !(gm < M && gk < K)) {
                cp_async16(dst, src, in);
            } else {
#pragma unroll
                for (int e = 0; e < EPC; e++) dst[e] = (gk + e < K) ? A[(size_t)gm * lda + gk + e] : T(0);
            }
        } else {
#pragma unroll
            for (int e = 0; e < EPC; e++)
                dst[e] = (gm < M && gk + e < K) ? A[(size_t)gm * lda + gk + e] : T(0);
        }
    }
    constexpr int B_CHUNKS = BK * BN / EPC;
    for (int ch = tid; ch < B_CHUNKS; ch += NTH) {
        int r = ch / (BN / EPC), cc = (ch % (BN / EPC)) * EPC;
        int gk = k0 + r, gn = n0 + cc;
        T* dst = sB + r * S::BS + cc;
        if (vecB) {
            bool in = gk < K && gn + EPC <= N;
            const T* src = in ? B + (size_t)gk * ldb + gn : B;
            if (in || !(gk < K && gn < N)) {
                cp_async16(dst, src, in);
            } else {
#pragma unroll
                for (int e = 0; e < EPC; e++) dst[e] = (gn + e < N) ? B[(size_t)gk * ldb + gn + e] : T(0);
            }
        } else {
#pragma unroll
            for (int e = 0; e < EPC; e++)
                dst[e] = (gk < K && gn + e < N) ? B[(size_t)gk * ldb + gn + e] : T(0);
        }
    }
}

// ---- f64 DMMA -----------------------------------------------------------------------

__device__ __forceinline__ void dmma_16x8x4(double (&d)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%0,%1,%2,%3};\n"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

template <int MK>
__device__ __forceinline__ void dmma(double (&d)[4], const double* a, const double* b);
template <>
__device__ __forceinline__ void dmma<4>(double (&d)[4], const double* a, const double* b) {
    dmma_16x8x4(d, a[0], a[1], b[0]);
}
template <>
__device__ __forceinline__ void dmma<8>(double (&d)[4], const double* a, const double* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}
template <>
__device__ __forceinline__ void dmma<16>(double (&d)[4], const double* a, const double* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, "
        "{%4,%5,%6,%7,%8,%9,%10,%11}, {%12,%13,%14,%15}, {%0,%1,%2,%3};\n"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]),
          "d"(b[0]), "d"(b[1]), "d"(b[2]), "d"(b[3]));
}

__device__ __forceinline__ unsigned f2tf32_rn(float x) {
    unsigned r;
    asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void tmma_16x8x8(float (&d)[4], const unsigned (&a)[4],
                                            const unsigned (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Interior tile: every 16-byte chunk of the A and B tiles is in range and
// aligned, so the loads need no guards.
template <class S, typename T = typename S::type>
__device__ __forceinline__ void load_tile_fast(T* sA, T* sB, const T* A, const T* B, int lda,
                                               int ldb, int m0, int n0, int k0) {
    constexpr int EPC = 16 / sizeof(T);
    constexpr int BM = S::BM, BN = S::BN, BK = S::BK, NTH = S::NTH;
    const int tid = threadIdx.x;
    constexpr int A_CHUNKS = BM * BK / EPC;
#pragma unroll
    for (int ch = tid; ch < A_CHUNKS; ch += NTH) {
        const int r = ch / (BK / EPC), cc = (ch % (BK / EPC)) * EPC;
        cp_async16(sA + r * S::AS + cc, A + (size_t)(m0 + r) * lda + k0 + cc, true);
    }
    constexpr int B_CHUNKS = BK * BN / EPC;
#pragma unroll
    for (int ch = tid; ch < B_CHUNKS; ch += NTH) {
        const int r = ch / (BN / EPC), cc = (ch % (BN / EPC)) * EPC;
        cp_async16(sB + r * S::BS + cc, B + (size_t)(k0 + r) * ldb + n0 + cc, true);
    }
}

// Tile coordinates of linear tile `lin`: z (batch or K slice), m0, n0.
struct TileAt {
    int z, m0, n0;
};
template <typename T, int TM = BM, int TN = BN>
__device__ __forceinline__ TileAt tile_at(const GemmP<T>& P, long long lin) {
    const int tm = (P.M + TM - 1) / TM, tn = (P.N + TN - 1) / TN;
    const long long per_z = (long long)tm * tn;
    const int z = (int)(lin / per_z);
    const int r = (int)(lin - (long long)z * per_z);
    return TileAt{z, (r / tn) * TM, (r % tn) * TN};
}

// Operands of slice/batch z: A, B advanced and the K extent of the slice.
template <typename T>
__device__ __forceinline__ void operands_at(const GemmP<T>& P, int z, const T*& A, const T*& B,
                                            int& K) {
    A = P.A;
    B = P.B;
    K = P.K;
    if (P.ksplit > 0) {
        // split-K: slice z covers k in [z*ksplit, min(K, (z+1)*ksplit))
        const int kb = z * P.ksplit;
        K = (K - kb) < P.ksplit ? (K - kb) : P.ksplit;
        A += kb;
        B += (size_t)kb * P.ldb;
    } else {
        A += z * P.sA;
        B += z * P.sB;
    }
}

// acc += A[m0.., k] . B[k, n0..] over k-tiles [kt0, kt1) of this operand pair,
// through the STAGES-deep cp.async pipeline in `smem`.
template <class S, int MK, typename T = typename S::type>
__device__ __forceinline__ void gemm_mainloop(const GemmP<T>& P, const T* __restrict__ A,
                                              const T* __restrict__ B, int K, int m0, int n0,
                                              int kt0, int kt1, T* smem,
                                              T (&acc)[S::MI][S::NJ][4]) {
    constexpr int BM = S::BM, BN = S::BN, BK = S::BK, MI = S::MI, NJ = S::NJ;
    const int M = P.M, N = P.N, lda = P.lda, ldb = P.ldb;
    const bool vecA = P.vecA, vecB = P.vecB;
    const bool inner_mn = vecA && vecB && m0 + BM <= M && n0 + BN <= N;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int wm = (warp / S::WARPS_N) * (MI * 16), wn = (warp % S::WARPS_N) * (NJ * 8);
    auto load = [&](int st, int kt) {
        T* sA = smem + st * S::STAGE;
        T* sB = sA + S::A_ELEMS;
        const int k0 = kt * BK;
        if (inner_mn && k0 + BK <= K)
            load_tile_fast<S>(sA, sB, A, B, lda, ldb, m0, n0, k0);
        else
            load_tile<S>(sA, sB, A, B, M, N, K, lda, ldb, m0, n0, k0, vecA, vecB);
    };
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (kt0 + s < kt1) load(s, kt0 + s);
        cp_commit();
    }
    for (int kt = kt0; kt < kt1; kt++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        {
            const int nk = kt + STAGES - 1;
            if (nk < kt1) load((nk - kt0) % STAGES, nk);
            cp_commit();
        }
        const T* sA = smem + ((kt - kt0) % STAGES) * S::STAGE;
        const T* sB = sA + S::A_ELEMS;
        if constexpr (sizeof(T) == 8) {
            // DMMA m16n8kMK: A fragment register r holds (row g + 8*(r%2),
            // col tig + 4*(r/2)); B register r holds (row tig + 4r, col g).
            constexpr int AR = MK / 2, BR = MK / 4;
#pragma unroll
            for (int kk = 0; kk < BK; kk += MK) {
                double af[MI][AR], bf[NJ][BR];
#pragma unroll
                for (int i = 0; i < MI; i++)
#pragma unroll
                    for (int r = 0; r < AR; r++)
                        af[i][r] = sA[(wm + i * 16 + g + 8 * (r % 2)) * S::AS + kk + tig + 4 * (r / 2)];
#pragma unroll
                for (int j = 0; j < NJ; j++)
#pragma unroll
                    for (int r = 0; r < BR; r++) bf[j][r] = sB[(kk + tig + 4 * r) * S::BS + wn + j * 8 + g];
#pragma unroll
                for (int i = 0; i < MI; i++)
#pragma unroll
                    for (int j = 0; j < NJ; j++)
                        dmma<MK>(*reinterpret_cast<double(*)[4]>(acc[i][j]), af[i], bf[j]);
            }
        } else {
#pragma unroll
            for (int kk = 0; kk < BK; kk += 8) {
                unsigned ahi[MI][4], alo[MI][4], bhi[NJ][2], blo[NJ][2];
#pragma unroll
                for (int i = 0; i < MI; i++) {
                    const float* pa = reinterpret_cast<const float*>(sA) + (wm + i * 16 + g) * S::AS + kk + tig;
                    float x[4] = {pa[0], pa[8 * S::AS], pa[4], pa[8 * S::AS + 4]};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        ahi[i][e] = f2tf32_rn(x[e]);
                        alo[i][e] = f2tf32_rn(x[e] - __uint_as_float(ahi[i][e]));
                    }
                }
#pragma unroll
                for (int j = 0; j < NJ; j++) {
                    const float* pb = reinterpret_cast<const float*>(sB) + (kk + tig) * S::BS + wn + j * 8 + g;
                    float x[2] = {pb[0], pb[4 * S::BS]};
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        bhi[j][e] = f2tf32_rn(x[e]);
                        blo[j][e] = f2tf32_rn(x[e] - __uint_as_float(bhi[j][e]));
                    }
                }
#pragma unroll
                for (int i = 0; i < MI; i++)
#pragma unroll
                    for (int j = 0; j < NJ; j++) {
                        float(&d)[4] = *reinterpret_cast<float(*)[4]>(acc[i][j]);
                        tmma_16x8x8(d, alo[i], bhi[j]);
                        tmma_16x8x8(d, ahi[i], blo[j]);
                        tmma_16x8x8(d, ahi[i], bhi[j]);
                    }
            }
        }
    }
    cp_wait<0>();
    __syncthreads();  // the caller may reuse smem or start another tile
}

template <typename T, int MI, int NJ>
__device__ __forceinline__ void zero_acc(T (&acc)[MI][NJ][4]) {
#pragma unroll
    for (int i = 0; i < MI; i++)
#pragma unroll
        for (int j = 0; j < NJ; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[i][j][e] = T(0);
}

// Data-parallel kernel: CTA b computes linear tile tile_base + b over its
// whole K and writes C (bounds-checked).
template <class S, int MK = 4, typename T = typename S::type>
__global__ void __launch_bounds__(S::NTH, S::MINB) k_gemm(GemmP<T> P, long long tile_base) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* smem = reinterpret_cast<T*>(smem_raw);
    constexpr int MI = S::MI, NJ = S::NJ;
    const TileAt ta = tile_at<T, S::BM, S::BN>(P, tile_base + blockIdx.x);
    const T* A;
    const T* B;
    int K;
    operands_at(P, ta.z, A, B, K);
    T* __restrict__ C = P.C + ta.z * P.sC;
    T acc[MI][NJ][4];
    zero_acc(acc);
    gemm_mainloop<S, MK>(P, A, B, K, ta.m0, ta.n0, 0, (K + S::BK - 1) / S::BK, smem, acc);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int wm = (warp / S::WARPS_N) * (MI * 16), wn = (warp % S::WARPS_N) * (NJ * 8);
    const int M = P.M, N = P.N, ldc = P.ldc;
    // accumulator (i, j): c0,c1 at (g, 2tig..2tig+1), c2,c3 at (g+8, 2tig..)
#pragma unroll
    for (int i = 0; i < MI; i++)
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int col = ta.n0 + wn + j * 8 + 2 * tig;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int row = ta.m0 + wm + i * 16 + g + h * 8;
                if (row >= M) continue;
                T* dst = C + (size_t)row * ldc + col;
                T v0 = acc[i][j][2 * h], v1 = acc[i][j][2 * h + 1];
                if constexpr (sizeof(T) == 4) {
                    // 3xTF32: non-finite results are recomputed exactly
                    if (P.ksplit == 0 && !isfinite(v0) && col < N)
                        v0 = exact_dot_f32(A + (size_t)row * P.lda, B + col, K, P.ldb);
                    if (P.ksplit == 0 && !isfinite(v1) && col + 1 < N)
                        v1 = exact_dot_f32(A + (size_t)row * P.lda, B + col + 1, K, P.ldb);
                }
                if (col + 1 < N) {
                    dst[0] = v0;
                    dst[1] = v1;
                } else if (col < N) {
                    dst[0] = v0;
                }
            }
        }
}

// ---- stream-K tail --------------------------------------------------------------------
//
// The tiles after the last full wave (tile_base .. tile_base + tail) would
// leave SMs idle.  Their tail * KT k-tile iterations are cut into G equal
// contiguous ranges, range p = [W p / G, W (p+1) / G) with W = tail * KT.  A
// range is shorter than KT (tail < G), so it touches at most two tiles; CTA p
// writes the partial sum of each touched tile to workspace slot 2p or 2p+1
// (dense BM x BN).  k_gemm_fix then adds each tile's partials in range order
// -- that is, in k order -- and writes C: the result does not depend on
// timing.

__host__ __device__ inline long long sk_lo(long long p, long long W, int G) { return p * W / G; }

template <typename T, int BK, int MK = 4>
__global__ void __launch_bounds__(NTH, 1)
k_gemm_sk(GemmP<T> P, long long tile_base, long long W, int G, int KT, T* __restrict__ ws) {
    using S = Cfg<T, BK>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* smem = reinterpret_cast<T*>(smem_raw);
    const int p = blockIdx.x;
    const long long hi = sk_lo(p + 1, W, G);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;
    int slot = 0;
    for (long long it = sk_lo(p, W, G); it < hi && slot < 2; slot++) {
        const long long t = it / KT;
        const int kt0 = (int)(it - t * KT);
        const int kt1 = (int)((hi - it) < (long long)(KT - kt0) ? kt0 + (hi - it) : KT);
        const TileAt ta = tile_at(P, tile_base + t);
        const T* A;
        const T* B;
        int K;
        operands_at(P, ta.z, A, B, K);
        T acc[4][4][4];
        zero_acc(acc);
        gemm_mainloop<S, MK>(P, A, B, K, ta.m0, ta.n0, kt0, kt1, smem, acc);
        T* dst = ws + ((size_t)p * 2 + slot) * (BM * BN);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int row = wm + i * 16 + g + h * 8, col = wn + j * 8 + 2 * tig;
                    dst[row * BN + col] = acc[i][j][2 * h];
                    dst[row * BN + col + 1] = acc[i][j][2 * h + 1];
                }
        it += kt1 - kt0;
    }
}

// CTA (t, f) of the fix-up sums part f of tail tile t's elements over the
// tile's partials in range order.  The contributing ranges (at most G) are
// listed once in shared memory; four partials are loaded per step.
constexpr int kMaxSkRanges = 1024;

template <typename T> struct alignas(16) V16 {
    T x[16 / sizeof(T)];
};

template <typename T>
__global__ void __launch_bounds__(NTH)
k_gemm_fix(GemmP<T> P, long long tile_base, long long W, int G, int KT,
           const T* __restrict__ ws) {
    __shared__ int src_slot[kMaxSkRanges];  // workspace slot of each contributor, in k order
    __shared__ int n_src;
    const long long t = blockIdx.x;
    const int per = (BM * BN) / gridDim.y;  // elements of this CTA
    const int e0 = blockIdx.y * per;
    if (threadIdx.x == 0) {
        const long long i0 = t * KT, i1 = i0 + KT;
        int p0 = (int)(i0 * G / W);  // first range holding iteration i0
        while (p0 + 1 < G && sk_lo(p0 + 1, W, G) <= i0) p0++;
        while (p0 > 0 && sk_lo(p0, W, G) > i0) p0--;
        int n = 0;
        for (int q = p0; q < G && n < kMaxSkRanges; q++) {
            const long long lo = sk_lo(q, W, G);
            if (lo >= i1) break;
            src_slot[n++] = q * 2 + ((lo / KT == t) ? 0 : 1);
        }
        n_src = n;
    }
    __syncthreads();
    const int n = n_src;
    const TileAt ta = tile_at(P, tile_base + t);
    T* __restrict__ C = P.C + ta.z * P.sC;
    const int M = P.M, N = P.N, ldc = P.ldc;
    constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
    for (int e = e0 + threadIdx.x * V; e < e0 + per; e += NTH * V) {
        auto at = [&](int q) {
            return *reinterpret_cast<const V16<T>*>(ws + (size_t)src_slot[q] * (BM * BN) + e);
        };
        T sum[V];
        {
            const V16<T> v = at(0);
#pragma unroll
            for (int u = 0; u < V; u++) sum[u] = v.x[u];
        }
        int q = 1;
        for (; q + 4 <= n; q += 4) {
            const V16<T> v0 = at(q), v1 = at(q + 1), v2 = at(q + 2), v3 = at(q + 3);
#pragma unroll
            for (int u = 0; u < V; u++) sum[u] = (((sum[u] + v0.x[u]) + v1.x[u]) + v2.x[u]) + v3.x[u];
        }
        for (; q < n; q++) {
            const V16<T> v = at(q);
#pragma unroll
            for (int u = 0; u < V; u++) sum[u] = sum[u] + v.x[u];
        }
        const int row = ta.m0 + e / BN, col0 = ta.n0 + e % BN;
        if (row >= M) continue;
        if constexpr (sizeof(T) == 4) {
            // 3xTF32 partials: a non-finite sum is recomputed exactly
            if (P.ksplit == 0 && P.A != nullptr) {
                const T* A = P.A + ta.z * P.sA + (size_t)row * P.lda;
                const T* B = P.B + ta.z * P.sB;
#pragma unroll
                for (int u = 0; u < V; u++)
                    if (col0 + u < N && !isfinite(sum[u]))
                        sum[u] = exact_dot_f32(A, B + col0 + u, P.K, P.ldb);
            }
        }
#pragma unroll
        for (int u = 0; u < V; u++)
            if (col0 + u < N) C[(size_t)row * ldc + col0 + u] = sum[u];
    }
}

// Stream-K is used for plain products (no K slicing) whose last wave leaves
// SMs idle for at least 6 k-tile times in total per SM -- the fix-up costs
// about that much.  NXV_GEMM_SK=0 disables it.
bool sk_enabled() {
    const char* v = getenv("NXV_GEMM_SK");
    return !(v && strcmp(v, "0") == 0);
}

template <typename T, int BK, int MK = 4>
int run_gemm_p(Ctx& c, GemmP<T> P) {
    constexpr int EPC = 16 / sizeof(T);
    P.vecA = ((uintptr_t)P.A % 16 == 0) && (P.lda % EPC == 0) && (P.ksplit % EPC == 0);
    P.vecB = ((uintptr_t)P.B % 16 == 0) && (P.ldb % EPC == 0);
    using S = Cfg<T, BK>;
    size_t smem = S::BYTES;
    const long long tiles = (long long)((P.M + BM - 1) / BM) * ((P.N + BN - 1) / BN) * P.batch;
    if (tiles <= 0) return finish(c);
    if (tiles > 0x7fffffffLL) {
        set_error("matmul grid out of range");
        return E_ARG;
    }
    const int KT = (P.K + BK - 1) / BK;
    const SkPlan pl = P.ksplit == 0 ? gemm_sk_plan(tiles, KT, c.dev->sm_count, 6) : SkPlan{};
    if (pl.tail == 0) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm<S, MK>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
        k_gemm<S, MK><<<(unsigned)tiles, NTH, smem, c.stream>>>(P, 0);
        count_launch();
        return finish(c);
    }
    const long long dp = pl.dp, tail = pl.tail, W = pl.W;
    const int G = pl.G;
    ScratchGuard guard(c);
    T* ws = (T*)scratch(c, (size_t)G * 2 * BM * BN * sizeof(T), kScratchGemm);
    if (!ws) return E_CUDA;
    cudaError_t e = cudaFuncSetAttribute(k_gemm<S, MK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k_gemm_sk<T, BK, MK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    if (dp > 0) {
        k_gemm<S, MK><<<(unsigned)dp, NTH, smem, c.stream>>>(P, 0);
        count_launch();
    }
    k_gemm_sk<T, BK, MK><<<G, NTH, smem, c.stream>>>(P, dp, W, G, KT, ws);
    count_launch();
    // fix-up: split each tile's elements over f CTAs so that about 2 CTAs per
    // SM run (f divides BM*BN / (NTH * 16 bytes) evenly for f <= 16, a power of 2)
    int f = 1;
    while (f < 16 && tail * f < 2LL * c.dev->sm_count) f *= 2;
    k_gemm_fix<T><<<dim3((unsigned)tail, f), NTH, 0, c.stream>>>(P, dp, W, G, KT, ws);
    count_launch();
    return finish(c);
}

// Fills the GEMM parameters of a plain (batched, dense) product.
template <typename T>
int plain_params(GemmP<T>& P, T* C, const T* A, const T* B, size_t batch, size_t m, size_t n,
                 size_t k) {
    if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff || batch > 65535) {
        set_error("matmul extents out of range");
        return E_ARG;
    }
    P = GemmP<T>{};
    P.A = A;
    P.B = B;
    P.C = C;
    P.M = (int)m;
    P.N = (int)n;
    P.K = (int)k;
    P.lda = (int)k;
    P.ldb = (int)n;
    P.ldc = (int)n;
    P.sA = (long long)(m * k);
    P.sB = (long long)(k * n);
    P.sC = (long long)(m * n);
    P.ksplit = 0;
    P.batch = (int)batch;
    return OK;
}

// f64 configuration: BK x MMA-K, default 32x4.  NXV_DMMA="BKxMK" (16x4,
// 16x8, 16x16, 32x8, 32x16) overrides it.
int dmma_cfg() {
    const char* v = getenv("NXV_DMMA");
    if (v && *v) {
        int bk = 0, mk = 0;
        if (sscanf(v, "%dx%d", &bk, &mk) == 2) return bk * 100 + mk;
    }
    return 3204;
}

// f64 products run on the 64 x 64 tile (Small64) unless NXV_GEMM_TILE=128
// selects the 128 x 128 schedule with its stream-K tail.  Measured on B200
// (TF/s, 64 x 64 / 128 x 128 / cuBLAS): 64 x 256^3 batched 28.1 / 23.6 / 29.4;
// 256 x 128^3 24.5 / 20.5 / 24.9; 1024^3 26.0 / 23.5 / 26.1; 2048^3 31.9 /
// 30.3 / 33.7; 4096^3 33.3 / 32.0 / 35.4; 3000 x 3000 x 512 30.5 / 26.3 /
// 32.1; 256 x 10000 x 104 18.4 / 10.0 / 19.8; 8 x 512^3 24.4 / 25.3 / 27.1.
bool small64_pick() {
    const char* v = getenv("NXV_GEMM_TILE");
    return !(v && strcmp(v, "128") == 0);
}

int run_gemm_small(Ctx& c, GemmP<double> P) {
    using S = Small64;
    constexpr int EPC = 2;
    P.vecA = ((uintptr_t)P.A % 16 == 0) && (P.lda % EPC == 0) && (P.ksplit % EPC == 0);
    P.vecB = ((uintptr_t)P.B % 16 == 0) && (P.ldb % EPC == 0);
    const long long tiles = (long long)((P.M + S::BM - 1) / S::BM) * ((P.N + S::BN - 1) / S::BN) * P.batch;
    if (tiles <= 0) return finish(c);
    if (tiles > 0x7fffffffLL) {
        set_error("matmul grid out of range");
        return E_ARG;
    }
    cudaError_t e = cudaFuncSetAttribute(k_gemm<S, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)S::BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm 64x64)");
    k_gemm<S, 4><<<(unsigned)tiles, S::NTH, S::BYTES, c.stream>>>(P, 0);
    count_launch();
    return finish(c);
}

int gemm_f64_dispatch(Ctx& c, const GemmP<double>& P) {
    if (small64_pick()) return run_gemm_small(c, P);
    switch (dmma_cfg()) {
        case 1608: return run_gemm_p<double, 16, 8>(c, P);
        case 1616: return run_gemm_p<double, 16, 16>(c, P);
        case 1604: return run_gemm_p<double, 16, 4>(c, P);
        case 3208: return run_gemm_p<double, 32, 8>(c, P);
        case 3216: return run_gemm_p<double, 32, 16>(c, P);
        default: return run_gemm_p<double, 32, 4>(c, P);
    }
}

template <typename T, int BK>
int run_gemm(Ctx& c, T* C, const T* A, const T* B, size_t batch, size_t m, size_t n, size_t k) {
    if (batch == 0 || m == 0 || n == 0) return OK;
    if (k == 0) {
        cudaError_t e = cudaMemsetAsync(C, 0, batch * m * n * sizeof(T), c.stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
        return finish(c);
    }
    GemmP<T> P;
    int rc = plain_params(P, C, A, B, batch, m, n, k);
    if (rc) return rc;
    if constexpr (sizeof(T) == 8) return gemm_f64_dispatch(c, P);
    return run_gemm_p<T, BK>(c, P);
}

}  // namespace

int launch_matmul_f64(Ctx& c, void* C, const void* A, const void* B, size_t batch, size_t m,
                      size_t n, size_t k) {
    return run_gemm<double, 16>(c, (double*)C, (const double*)A, (const double*)B, batch, m, n, k);
}

int launch_matmul_f32(Ctx& c, void* C, const void* A, const void* B, size_t batch, size_t m,
                      size_t n, size_t k) {
    // Default: tcgen05 3xTF32 (k_matmul_tc.cu).  NXV_MATMUL_F32=mma selects the
    // warp-level mma.sync 3xTF32 kernel below.
    const char* v = getenv("NXV_MATMUL_F32");
    if (!(v && strcmp(v, "mma") == 0)) return launch_matmul_f32_tc(c, C, A, B, batch, m, n, k);
    return run_gemm<float, 32>(c, (float*)C, (const float*)A, (const float*)B, batch, m, n, k);
}

int gemm_f64(Ctx& c, const GemmP<double>& P) { return gemm_f64_dispatch(c, P); }

bool gemm_sk_enabled() { return sk_enabled(); }

SkPlan gemm_sk_plan(long long tiles, int KT, int sms, int min_idle) {
    SkPlan pl{};
    pl.tail = tiles % sms;
    if (!(sk_enabled() && pl.tail > 0 && (sms - pl.tail) * (long long)KT >= (long long)min_idle * sms)) {
        pl.tail = 0;
        return pl;
    }
    pl.dp = tiles - pl.tail;
    pl.W = pl.tail * KT;
    pl.G = (int)std::min<long long>(std::min<long long>(std::min<long long>(pl.W, sms), 32 * pl.tail),
                                    kMaxSkRanges);
    return pl;
}

int launch_gemm_fix_f32(Ctx& c, float* C, const float* A, const float* B, int M, int N, int K,
                        int batch, const SkPlan& pl, int KT, const float* ws) {
    GemmP<float> P{};
    P.A = A;
    P.B = B;
    P.C = C;
    P.M = M;
    P.N = N;
    P.K = K;
    P.lda = K;
    P.ldb = N;
    P.ldc = N;
    P.sA = (long long)M * K;
    P.sB = (long long)K * N;
    P.sC = (long long)M * N;
    P.batch = batch;
    int f = 1;
    while (f < 16 && pl.tail * f < 2LL * c.dev->sm_count) f *= 2;
    k_gemm_fix<float><<<dim3((unsigned)pl.tail, f), NTH, 0, c.stream>>>(P, pl.dp, pl.W, pl.G, KT, ws);
    count_launch();
    return OK;
}

}  // namespace nxv
