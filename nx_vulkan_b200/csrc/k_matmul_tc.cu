// k_matmul_tc.cu -- f32 GEMM as 3xTF32 on the sm_100a tensor cores (tcgen05).
//
// C = A . B with A [M][K], B [K][N], C [M][N] row-major f32, batched.
// Split: x = hi + lo with hi = x rounded to TF32 and lo = x - hi rounded to
// TF32 (both exact TF32 values);
// C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi accumulated in f32 in tensor memory
// (three accumulators, summed in the epilogue).  The dropped A_lo.B_lo term
// and the rounding of lo are ~2^-22 relative and unbiased, so the result has
// f32 accuracy (as close to the exact product as an f32 FMA GEMM).  An element whose accumulated value is
// not finite is recomputed exactly in the epilogue (exact_dot_f32), so
// infinities and NaNs in the inputs give IEEE results.
//
// Pipeline (one CTA per 128 x 128 tile of C, 4 warps; the tiles after the
// last full wave of SMs run stream-K, see k_gemm_tc):
//   pre-pass  split A -> A_hi, A_lo [M][Kp] and B -> B^T_hi, B^T_lo [N][Kp]
//             (K padded to a multiple of 32 with zeros): both operands
//             K-major, every TMA box starts at an x multiple of 32.
//   warp 0    lane 0: TMA producer -- per k-block of 32, four 2-D boxes
//             (128 rows x 128 bytes, 128-byte swizzle) into one of 3 stages
//             of 64 KB, completion counted on the stage's mbarrier.
//   warp 1    lane 0: MMA issuer -- for each of the 4 K-steps of 8 in a
//             k-block: tcgen05.mma kind::tf32 (lo.hi, hi.lo, hi.hi) into a
//             128 x 128 f32 accumulator in TMEM; tcgen05.commit frees the
//             stage, a last commit signals the epilogue.
//   all       epilogue: warp q reads TMEM lanes 32q..32q+31 (its rows) with
//             tcgen05.ld 32x32b.x8 and stores C.
// Every mbarrier wait is bounded: on timeout the kernel records an error
// flag, drains its own TMA loads (bounded), frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "kernels.h"

#include <algorithm>

namespace nxv {

namespace {

constexpr int TBM = 128, TBN = 128, TBK = 32, TSTAGES = 3;
constexpr int TILE_BYTES = TBM * TBK * 4;        // 16 KB: 128 rows x 128 B
constexpr int STAGE_BYTES = 4 * TILE_BYTES;      // A_hi, A_lo, B_hi, B_lo
constexpr int SMEM_BYTES = TSTAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
// Three 128 x 128 f32 accumulators in tensor memory (columns 0, 128, 256 of
// a 512-column allocation): ACC_HI0 and ACC_HI1 take the A_hi.B_hi products
// of the first and second half of every k-block, ACC_X the two cross terms.
// The tensor core's accumulation loses up to ~1/2 ulp of the running sum per
// MMA, with a bias; keeping the small cross terms apart and splitting the
// large sum in two cuts the additions into each large sum by 6 and halves
// its magnitude.  The epilogue adds the three in f32.  Measured on B200 for
// 2048^3 with N(0, 1/2048) entries, max |error| against the exact product:
// one accumulator, truncated split 1.82e-6; three accumulators 3.3e-7.
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t ACC_HI0 = 0, ACC_HI1 = 128, ACC_X = 256;

__device__ int g_tc_error;  // 1 when a bounded wait ran out

__device__ __forceinline__ uint32_t su32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait (about a second at most); false and the error flag on timeout.
__device__ __noinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); i++) {
        if (mbar_try(b, parity)) return true;
        if (i > 128) __nanosleep(200);
    }
    atomicExch(&g_tc_error, 1);
    return false;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(su32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(su32(bar))
        : "memory");
}

// Shared-memory matrix descriptor: K-major operand tile of rows of 128 bytes
// with the 128-byte swizzle; 8-row groups 1024 bytes apart (SBO), version 1
// (sm_100 format), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::tf32: D f32 (bits 4-5 = 1), A and B TF32
// (bits 7-9, 10-12 = 2), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TBN >> 3) << 17) |
                           ((uint32_t)(TBM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(IDESC), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     su32(b))
                 : "memory");
}

// One CTA computes up to two work items, each a 128 x 128 tile of C over a
// range of k-blocks:
//   mode 0 (data-parallel): tile tile_base + blockIdx.x over all KB k-blocks,
//            written to C;
//   mode 1 (stream-K tail): CTA p takes k-block iterations
//            [W p / G, W (p+1) / G) of the tiles after tile_base (KB
//            iterations per tile), at most two tiles, and writes each
//            partial sum to workspace slot 2p or 2p+1 (dense 128 x 128 f32);
//            a fix-up adds every tile's slots in order.
// The producer and the MMA issuer count pipeline iterations across the items
// (stage = it % TSTAGES, parity from it / TSTAGES); the accumulator is
// drained between items behind a block barrier.
__global__ void __launch_bounds__(128, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap mA_hi, const __grid_constant__ CUtensorMap mA_lo,
          const __grid_constant__ CUtensorMap mB_hi, const __grid_constant__ CUtensorMap mB_lo,
          float* __restrict__ C, int M, int N, int Kp, long long sC, long long tile_base, int mode,
          long long W, int G, float* __restrict__ ws, const float* __restrict__ A0,
          const float* __restrict__ B0, int K) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t base = su32(smem_raw);
    unsigned char* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + TSTAGES * STAGE_BYTES);
    uint64_t* empty = full + TSTAGES;
    uint64_t* done = empty + TSTAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int s_err;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KB = Kp / TBK;
    const int tm = (M + TBM - 1) / TBM, tn = (N + TBN - 1) / TBN;

    // work items: (linear tile, first k-block, end k-block, workspace slot)
    long long it_tile[2];
    int it_k0[2], it_k1[2], n_items = 0;
    if (mode == 0) {
        it_tile[0] = tile_base + blockIdx.x;
        it_k0[0] = 0;
        it_k1[0] = KB;
        n_items = 1;
    } else {
        const long long p = blockIdx.x;
        long long it = p * W / G;
        const long long hi = (p + 1) * W / G;
        while (it < hi && n_items < 2) {
            const long long t = it / KB;
            const int k0 = (int)(it - t * KB);
            const int k1 = (int)((hi - it) < (long long)(KB - k0) ? k0 + (hi - it) : KB);
            it_tile[n_items] = tile_base + t;
            it_k0[n_items] = k0;
            it_k1[n_items] = k1;
            n_items++;
            it += k1 - k0;
        }
    }

    if (tid == 0) {
        s_err = 0;
        for (int s = 0; s < TSTAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         su32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    int issued = 0;    // producer: pipeline iterations whose loads were issued
    int pipe_it = 0;   // pipeline iterations of the items before this one
    for (int item = 0; item < n_items; item++) {
        const long long lin = it_tile[item];
        const int bz = (int)(lin / ((long long)tm * tn));
        const int rr = (int)(lin - (long long)bz * tm * tn);
        const int m0 = (rr / tn) * TBM, n0 = (rr % tn) * TBN;
        const int k0 = it_k0[item], k1 = it_k1[item];
        if (warp == 0 && lane == 0) {
            for (int kb = k0; kb < k1; kb++) {
                const int it = pipe_it + (kb - k0);
                const int s = it % TSTAGES;
                if (it >= TSTAGES && !mbar_wait(&empty[s], ((it / TSTAGES) + 1) & 1)) {
                    s_err = 1;
                    break;
                }
                unsigned char* st = smem + s * STAGE_BYTES;
                mbar_expect_tx(&full[s], STAGE_BYTES);
                tma_load_3d(st, &mA_hi, kb * TBK, m0, bz, &full[s]);
                tma_load_3d(st + TILE_BYTES, &mA_lo, kb * TBK, m0, bz, &full[s]);
                tma_load_3d(st + 2 * TILE_BYTES, &mB_hi, kb * TBK, n0, bz, &full[s]);
                tma_load_3d(st + 3 * TILE_BYTES, &mB_lo, kb * TBK, n0, bz, &full[s]);
                issued = it + 1;
            }
        } else if (warp == 1 && lane == 0) {
            bool ok = true;
            for (int kb = k0; kb < k1; kb++) {
                const int it = pipe_it + (kb - k0);
                const int s = it % TSTAGES;
                if (!mbar_wait(&full[s], (it / TSTAGES) & 1)) {
                    s_err = 1;
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t st = su32(smem + s * STAGE_BYTES);
                const uint64_t ahi = sdesc(st), alo = sdesc(st + TILE_BYTES);
                const uint64_t bhi = sdesc(st + 2 * TILE_BYTES), blo = sdesc(st + 3 * TILE_BYTES);
#pragma unroll
                for (int j = 0; j < TBK / 8; j++) {
                    const uint64_t adv = (uint64_t)(j * 32) >> 4;  // 8 f32 = 32 bytes along K
                    const uint32_t acc_hi = tmem + (j < TBK / 16 ? ACC_HI0 : ACC_HI1);
                    const bool first = kb == k0 && j == 0;
                    const uint32_t first_hi = (kb == k0 && (j == 0 || j == TBK / 16)) ? 0u : 1u;
                    umma_tf32(tmem + ACC_X, alo + adv, bhi + adv, first ? 0u : 1u);
                    umma_tf32(tmem + ACC_X, ahi + adv, blo + adv, 1);
                    umma_tf32(acc_hi, ahi + adv, bhi + adv, first_hi);
                }
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(done);
        }
        __syncwarp();
        pipe_it += k1 - k0;
        // Epilogue: wait for the accumulator (done completes once per item),
        // then each thread drains its row to C or to the workspace slot.
        bool have = mbar_wait(done, item & 1);
        if (!have) s_err = 1;
        __syncthreads();
        if (s_err != 0 || !have) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int lrow = warp * 32 + lane;
        const int row = m0 + lrow;
        float* crow = (mode == 0) ? C + bz * sC + (size_t)row * N
                                  : ws + ((size_t)blockIdx.x * 2 + item) * (TBM * TBN) + (size_t)lrow * TBN;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
        for (int c0 = 0; c0 < TBN; c0 += 8) {
            uint32_t r[8], h1[8], x[8];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                  "=r"(r[6]), "=r"(r[7])
                : "r"(tl + ACC_HI0 + c0));
            asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                    : "=r"(h1[0]), "=r"(h1[1]), "=r"(h1[2]), "=r"(h1[3]), "=r"(h1[4]), "=r"(h1[5]),
                      "=r"(h1[6]), "=r"(h1[7])
                    : "r"(tl + ACC_HI1 + c0));
            asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                    : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]),
                      "=r"(x[6]), "=r"(x[7])
                    : "r"(tl + ACC_X + c0));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int e = 0; e < 8; e++)
                r[e] = __float_as_uint(__fadd_rn(
                    __fadd_rn(__uint_as_float(r[e]), __uint_as_float(h1[e])), __uint_as_float(x[e])));
            if (mode == 1) {  // dense slot, every element
                float4* d4 = reinterpret_cast<float4*>(crow + c0);
                d4[0] = make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]),
                                    __uint_as_float(r[2]), __uint_as_float(r[3]));
                d4[1] = make_float4(__uint_as_float(r[4]), __uint_as_float(r[5]),
                                    __uint_as_float(r[6]), __uint_as_float(r[7]));
            } else if (row < M) {
                const int col = n0 + c0;
#pragma unroll
                for (int e = 0; e < 8; e++)
                    if (!isfinite(__uint_as_float(r[e])) && col + e < N)
                        r[e] = __float_as_uint(exact_dot_f32(A0 + ((size_t)bz * M + row) * K,
                                                             B0 + (size_t)bz * K * N + col + e, K, N));
                if (col + 8 <= N && (((uintptr_t)(crow + col)) & 15) == 0) {
                    float4* d4 = reinterpret_cast<float4*>(crow + col);
                    d4[0] = make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]),
                                        __uint_as_float(r[2]), __uint_as_float(r[3]));
                    d4[1] = make_float4(__uint_as_float(r[4]), __uint_as_float(r[5]),
                                        __uint_as_float(r[6]), __uint_as_float(r[7]));
                } else {
                    for (int e = 0; e < 8; e++)
                        if (col + e < N) crow[col + e] = __uint_as_float(r[e]);
                }
            }
        }
        // the next item's MMAs overwrite the accumulator: every read is done
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    if (s_err != 0 && tid == 0) {
        // error path: let every TMA load this CTA issued land before the CTA
        // (and its shared memory) goes away; each wait is bounded.
        for (int it = (issued > TSTAGES ? issued - TSTAGES : 0); it < issued; it++)
            mbar_wait(&full[it % TSTAGES], (it / TSTAGES) & 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}
// hi = x rounded to nearest TF32, lo = (x - hi) rounded to nearest TF32:
// |lo| <= 2^-11 |x| with no sign bias, so the dropped lo.lo term averages
// out (truncating hi leaves lo with x's sign and up to twice the size:
// 1x1x3 products err by 1.3e-6 instead of 2.4e-8).  The tensor core reads
// both exactly.  An infinite x gives hi = inf, lo = NaN (see the header).
__device__ __forceinline__ float tf32_hi(float x) { return tf32_rna(x); }
__device__ __forceinline__ float tf32_lo(float x, float hi) { return tf32_rna(__fsub_rn(x, hi)); }

// One launch splits both operands (blockIdx.y: the batch entry).
//   CTAs [0, ga): A [M][K] -> A_hi, A_lo [M][Kp], one warp per row, lane l
//     taking 4-column groups l, l+32, ... with 8 groups' loads in flight
//     and 16-byte accesses when rows are 16-byte aligned;
//   CTAs [ga, ga + gb): B [K][N] -> B^T_hi, B^T_lo [N][Kp] in tiles of
//     32 k x 128 n through shared memory (rows padded to 129 floats: the
//     column reads are conflict-free), 16 loads in flight per thread,
//     grid-stride over the tiles.
// Columns k in [K, Kp) are written as zeros.  Four CTAs per SM (64
// registers): 128 KB of A or 64 KB of B loads in flight per SM.
constexpr int kSplitU = 8;

__global__ void __launch_bounds__(256, 4)
k_split_ab(const float* __restrict__ A, float* __restrict__ ahi, float* __restrict__ alo, int M,
           const float* __restrict__ B, float* __restrict__ bhi, float* __restrict__ blo, int N,
           int K, int Kp, long long sA, long long sB, long long sOA, long long sOB, int ga,
           int gb) {
    __shared__ float t[32][129];
    const int bz = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if ((int)blockIdx.x < ga) {
        A += bz * sA;
        ahi += bz * sOA;
        alo += bz * sOA;
        const bool vec = (K & 3) == 0 && (((uintptr_t)A) & 15) == 0;
        for (int r = blockIdx.x * 8 + warp; r < M; r += ga * 8) {
            const float* src = A + (size_t)r * K;
            float* h = ahi + (size_t)r * Kp;
            float* l = alo + (size_t)r * Kp;
            // Kp % 32 == 0, so groups never straddle Kp
            for (int k0 = lane * 4; k0 < Kp; k0 += 128 * kSplitU) {
                float x[kSplitU][4];
#pragma unroll
                for (int u = 0; u < kSplitU; u++) {
                    const int k = k0 + u * 128;
                    if (k >= Kp) continue;
                    if (vec && k + 4 <= K) {
                        const float4 v = *reinterpret_cast<const float4*>(src + k);
                        x[u][0] = v.x, x[u][1] = v.y, x[u][2] = v.z, x[u][3] = v.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; e++) x[u][e] = k + e < K ? src[k + e] : 0.0f;
                    }
                }
#pragma unroll
                for (int u = 0; u < kSplitU; u++) {
                    const int k = k0 + u * 128;
                    if (k >= Kp) continue;
                    float4 vh, vl;
                    vh.x = tf32_hi(x[u][0]), vh.y = tf32_hi(x[u][1]);
                    vh.z = tf32_hi(x[u][2]), vh.w = tf32_hi(x[u][3]);
                    vl.x = tf32_lo(x[u][0], vh.x), vl.y = tf32_lo(x[u][1], vh.y);
                    vl.z = tf32_lo(x[u][2], vh.z), vl.w = tf32_lo(x[u][3], vh.w);
                    *reinterpret_cast<float4*>(h + k) = vh;
                    *reinterpret_cast<float4*>(l + k) = vl;
                }
            }
        }
        return;
    }
    B += bz * sB;
    bhi += bz * sOB;
    blo += bz * sOB;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    const long long ntn = (N + 127) / 128, ntiles = ntn * (Kp / 32);
    for (long long tile = (long long)blockIdx.x - ga; tile < ntiles; tile += gb) {
        const int n0 = (int)(tile % ntn) * 128, k0 = (int)(tile / ntn) * 32;
#pragma unroll
        for (int r = ty; r < 32; r += 8) {
            const int k = k0 + r;
#pragma unroll
            for (int c = 0; c < 128; c += 32) {
                const int n = n0 + c + tx;
                t[r][c + tx] = (k < K && n < N) ? B[(size_t)k * N + n] : 0.0f;
            }
        }
        __syncthreads();
        const int k = k0 + tx;
#pragma unroll 4
        for (int r = ty; r < 128; r += 8) {
            const int n = n0 + r;
            if (n < N) {
                const float x = t[tx][r];
                const float h = tf32_hi(x);
                bhi[(size_t)n * Kp + k] = h;
                blo[(size_t)n * Kp + k] = tf32_lo(x, h);
            }
        }
        __syncthreads();  // the tile is refilled next iteration
    }
}

// The driver's tensor-map encoder, looked up once (a function-local static:
// initialised once even when several threads make their first GEMM call at
// the same time).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        cudaGetLastError();
        return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    }();
    return fn;
}

// 3-D map over [batch][rows][Kp] f32, box 32 (k) x 128 (rows) x 1, 128-byte swizzle.
int make_map(CUtensorMap* map, const float* base, int rows, int Kp, int batch) {
    auto fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return E_CUDA;
    }
    cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)Kp * 4, (cuuint64_t)Kp * 4 * (cuuint64_t)rows};
    cuuint32_t box[3] = {(cuuint32_t)TBK, (cuuint32_t)TBM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return E_CUDA;
    }
    return OK;
}

}  // namespace

int tc_gemm_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) {
        int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

int launch_matmul_f32_tc(Ctx& c, void* C, const void* A, const void* B, size_t batch, size_t m,
                         size_t n, size_t k) {
    if (batch == 0 || m == 0 || n == 0) return OK;
    if (k == 0) {
        cudaError_t e = cudaMemsetAsync(C, 0, batch * m * n * sizeof(float), c.stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
        return finish(c);
    }
    if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffe0 || batch > 65535) {
        set_error("matmul extents out of range");
        return E_ARG;
    }
    const size_t Kp = (k + TBK - 1) / TBK * TBK;  // < 2^31: int indexing in the kernels
    ScratchGuard guard(c);
    const size_t a_elems = batch * m * Kp, b_elems = batch * n * Kp;
    float* s = (float*)scratch(c, (2 * a_elems + 2 * b_elems) * sizeof(float) + 256);
    if (!s) return E_CUDA;
    float* ahi = s;
    float* alo = ahi + a_elems;
    float* bhi = alo + a_elems;
    float* blo = bhi + b_elems;
    {
        // one launch for both splits: a row per warp for A, 32 x 128 tiles
        // for B, each part at most a few CTAs per SM
        const int ga = (int)std::min<size_t>((m + 7) / 8, (size_t)c.dev->sm_count * 4);
        const size_t btiles = (n + 127) / 128 * (Kp / 32);
        const int gb = (int)std::min<size_t>(btiles, (size_t)c.dev->sm_count * 8);
        k_split_ab<<<dim3((unsigned)(ga + gb), (unsigned)batch), 256, 0, c.stream>>>(
            (const float*)A, ahi, alo, (int)m, (const float*)B, bhi, blo, (int)n, (int)k, (int)Kp,
            (long long)(m * k), (long long)(k * n), (long long)(m * Kp), (long long)(n * Kp), ga,
            gb);
        count_launch();
    }
    CUtensorMap mah, mal, mbh, mbl;
    int rc;
    if ((rc = make_map(&mah, ahi, (int)m, (int)Kp, (int)batch))) return rc;
    if ((rc = make_map(&mal, alo, (int)m, (int)Kp, (int)batch))) return rc;
    if ((rc = make_map(&mbh, bhi, (int)n, (int)Kp, (int)batch))) return rc;
    if ((rc = make_map(&mbl, blo, (int)n, (int)Kp, (int)batch))) return rc;
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_gemm_tc)");
    const long long tiles = (long long)((m + TBM - 1) / TBM) * ((n + TBN - 1) / TBN) * batch;
    if (tiles > 0x7fffffffLL) {
        set_error("matmul grid out of range");
        return E_ARG;
    }
    const int KB = (int)(Kp / TBK);
    // A 32-deep k-block takes ~0.7 us here: stream-K needs ~24 idle k-blocks
    // per SM to repay its fix-up (2048^3 with a 73 % last wave does not).
    const SkPlan pl = gemm_sk_plan(tiles, KB, c.dev->sm_count, 24);
    const long long dp = pl.tail ? pl.dp : tiles;
    if (dp > 0) {
        k_gemm_tc<<<(unsigned)dp, 128, SMEM_BYTES, c.stream>>>(
            mah, mal, mbh, mbl, (float*)C, (int)m, (int)n, (int)Kp, (long long)(m * n), 0, 0, 0, 1,
            nullptr, (const float*)A, (const float*)B, (int)k);
        count_launch();
    }
    if (pl.tail) {
        // workspace: 2 slots of 128 x 128 f32 per range, in the GEMM's own
        // scratch slot (the split planes above hold the op scratch)
        float* wsp = (float*)scratch(c, (size_t)pl.G * 2 * TBM * TBN * sizeof(float), kScratchGemm);
        if (!wsp) return E_CUDA;
        k_gemm_tc<<<(unsigned)pl.G, 128, SMEM_BYTES, c.stream>>>(
            mah, mal, mbh, mbl, (float*)C, (int)m, (int)n, (int)Kp, (long long)(m * n), pl.dp, 1,
            pl.W, pl.G, wsp, (const float*)A, (const float*)B, (int)k);
        count_launch();
        int rc2 = launch_gemm_fix_f32(c, (float*)C, (const float*)A, (const float*)B, (int)m,
                                      (int)n, (int)k, (int)batch, pl, KB, wsp);
        if (rc2) return rc2;
    }
    return finish(c);
}

}  // namespace nxv
