// k_matmul.cu -- dense C = A . B (row-major), batched over blockIdx.z.
//
// f64: DMMA tensor cores (mma.sync m16n8k4 .f64).  tcgen05 has no f64 kind,
// so the FP64 tensor path on sm_100a is the warp-level DMMA instruction.
// f32: 3xTF32 split on the warp-level TF32 MMA (mma.sync m16n8k8 .tf32):
// x = hi + lo with hi = x rounded toward zero to TF32 and lo = tf32(x - hi);
// C += Ahi.Bhi + Ahi.Blo + Alo.Bhi, accumulated in f32.  The error is of the
// order of f32 rounding (the dropped lo.lo term is ~2^-22 relative).
//
// Both kernels: CTA tile 128x128, 8 warps in a 2 (M) x 4 (N) grid with a
// 64x32 warp tile, a 3-stage cp.async pipeline, shared-memory rows padded so
// that every fragment load is bank-conflict free (A rows are BK+4 elements,
// B rows are 128+8 elements), zero-filled out-of-range chunks, and a
// scalar loader when a row is not 16-byte aligned.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

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

template <typename T, int BK>
struct Smem {
    static constexpr int AS = BK + 4;      // A row stride (elements)
    static constexpr int BS = BN + 8;      // B row stride (elements)
    static constexpr int A_ELEMS = BM * AS;
    static constexpr int B_ELEMS = BK * BS;
    static constexpr int STAGE = A_ELEMS + B_ELEMS;
    static constexpr size_t BYTES = (size_t)STAGES * STAGE * sizeof(T);
};

// Load one BMxBK tile of A and one BKxBN tile of B into stage buffers.
template <typename T, int BK>
__device__ __forceinline__ void load_tile(T* sA, T* sB, const T* A, const T* B, int M, int N,
                                          int K, int lda, int ldb, int m0, int n0, int k0,
                                          bool vecA, bool vecB) {
    constexpr int EPC = 16 / sizeof(T);  // elements per 16-byte chunk
    using S = Smem<T, BK>;
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

__device__ __forceinline__ unsigned f2tf32_rz(float x) { return __float_as_uint(x) & 0xFFFFE000u; }
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

template <typename T, int BK, int MK = 4>
__global__ void __launch_bounds__(NTH, 1) k_gemm(GemmP<T> P) {
    using S = Smem<T, BK>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* smem = reinterpret_cast<T*>(smem_raw);
    const int bz = blockIdx.z;
    const T* __restrict__ A = P.A;
    const T* __restrict__ B = P.B;
    T* __restrict__ C = P.C + bz * P.sC;
    const int M = P.M, N = P.N, lda = P.lda, ldb = P.ldb, ldc = P.ldc;
    int K = P.K;
    if (P.ksplit > 0) {
        // split-K: slice bz covers k in [bz*ksplit, min(K, (bz+1)*ksplit))
        int kb = bz * P.ksplit;
        K = (K - kb) < P.ksplit ? (K - kb) : P.ksplit;
        A += kb;
        B += (size_t)kb * ldb;
    } else {
        A += bz * P.sA;
        B += bz * P.sB;
    }
    const bool vecA = P.vecA, vecB = P.vecB;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;

    constexpr int NACC = sizeof(T) == 8 ? 4 : 4;
    T acc[4][4][NACC];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int e = 0; e < NACC; e++) acc[i][j][e] = T(0);

    const int KT = (K + BK - 1) / BK;
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < KT) load_tile<T, BK>(smem + s * S::STAGE, smem + s * S::STAGE + S::A_ELEMS, A, B, M,
                                     N, K, lda, ldb, m0, n0, s * BK, vecA, vecB);
        cp_commit();
    }
    for (int kt = 0; kt < KT; kt++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        {
            int nk = kt + STAGES - 1;
            if (nk < KT) {
                int st = nk % STAGES;
                load_tile<T, BK>(smem + st * S::STAGE, smem + st * S::STAGE + S::A_ELEMS, A, B, M, N,
                                 K, lda, ldb, m0, n0, nk * BK, vecA, vecB);
            }
            cp_commit();
        }
        const T* sA = smem + (kt % STAGES) * S::STAGE;
        const T* sB = sA + S::A_ELEMS;
        if constexpr (sizeof(T) == 8) {
            // DMMA m16n8kMK: A fragment register r holds (row g + 8*(r%2),
            // col tig + 4*(r/2)); B register r holds (row tig + 4r, col g).
            constexpr int AR = MK / 2, BR = MK / 4;
#pragma unroll
            for (int kk = 0; kk < BK; kk += MK) {
                double af[4][AR], bf[4][BR];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int r = 0; r < AR; r++)
                        af[i][r] = sA[(wm + i * 16 + g + 8 * (r % 2)) * S::AS + kk + tig + 4 * (r / 2)];
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int r = 0; r < BR; r++) bf[j][r] = sB[(kk + tig + 4 * r) * S::BS + wn + j * 8 + g];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        dmma<MK>(*reinterpret_cast<double(*)[4]>(acc[i][j]), af[i], bf[j]);
            }
        } else {
#pragma unroll
            for (int kk = 0; kk < BK; kk += 8) {
                unsigned ahi[4][4], alo[4][4], bhi[4][2], blo[4][2];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float* pa = reinterpret_cast<const float*>(sA) + (wm + i * 16 + g) * S::AS + kk + tig;
                    float x[4] = {pa[0], pa[8 * S::AS], pa[4], pa[8 * S::AS + 4]};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        ahi[i][e] = f2tf32_rz(x[e]);
                        alo[i][e] = f2tf32_rn(x[e] - __uint_as_float(ahi[i][e]));
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float* pb = reinterpret_cast<const float*>(sB) + (kk + tig) * S::BS + wn + j * 8 + g;
                    float x[2] = {pb[0], pb[4 * S::BS]};
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        bhi[j][e] = f2tf32_rz(x[e]);
                        blo[j][e] = f2tf32_rn(x[e] - __uint_as_float(bhi[j][e]));
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        float(&d)[4] = *reinterpret_cast<float(*)[4]>(acc[i][j]);
                        tmma_16x8x8(d, alo[i], bhi[j]);
                        tmma_16x8x8(d, ahi[i], blo[j]);
                        tmma_16x8x8(d, ahi[i], bhi[j]);
                    }
            }
        }
    }
    cp_wait<0>();
    // epilogue: c0,c1 at (g, 2tig..2tig+1), c2,c3 at (g+8, 2tig..)
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int col = n0 + wn + j * 8 + 2 * tig;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                int row = m0 + wm + i * 16 + g + h * 8;
                if (row >= M) continue;
                T* dst = C + (size_t)row * ldc + col;
                if (col + 1 < N) {
                    dst[0] = acc[i][j][2 * h];
                    dst[1] = acc[i][j][2 * h + 1];
                } else if (col < N) {
                    dst[0] = acc[i][j][2 * h];
                }
            }
        }
}

template <typename T, int BK, int MK = 4>
int run_gemm_p(Ctx& c, GemmP<T> P) {
    constexpr int EPC = 16 / sizeof(T);
    P.vecA = ((uintptr_t)P.A % 16 == 0) && (P.lda % EPC == 0) && (P.ksplit % EPC == 0);
    P.vecB = ((uintptr_t)P.B % 16 == 0) && (P.ldb % EPC == 0);
    size_t smem = Smem<T, BK>::BYTES;
    cudaError_t e = cudaFuncSetAttribute(k_gemm<T, BK, MK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    dim3 grid((unsigned)((P.N + BN - 1) / BN), (unsigned)((P.M + BM - 1) / BM), (unsigned)P.batch);
    if (grid.y > 65535 || grid.z > 65535) {
        set_error("matmul grid out of range");
        return E_ARG;
    }
    k_gemm<T, BK, MK><<<grid, NTH, smem, c.stream>>>(P);
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

// f64 configuration: BK x MMA-K.  NXV_DMMA="BKxMK" (16x4, 16x8, 16x16,
// 32x8, 32x16) overrides the default.
int dmma_cfg() {
    const char* v = getenv("NXV_DMMA");
    if (v && *v) {
        int bk = 0, mk = 0;
        if (sscanf(v, "%dx%d", &bk, &mk) == 2) return bk * 100 + mk;
    }
    return 1604;
}

int gemm_f64_dispatch(Ctx& c, const GemmP<double>& P) {
    switch (dmma_cfg()) {
        case 1608: return run_gemm_p<double, 16, 8>(c, P);
        case 1616: return run_gemm_p<double, 16, 16>(c, P);
        case 3208: return run_gemm_p<double, 32, 8>(c, P);
        case 3216: return run_gemm_p<double, 32, 16>(c, P);
        default: return run_gemm_p<double, 16, 4>(c, P);
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

}  // namespace nxv
