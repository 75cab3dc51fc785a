// k_reduce.cu -- deterministic reductions, argmax, logsumexp, kinetic energy.
//
// Layout: every reduction is over the middle axis of a virtual
// (outer, R, inner) row-major tensor (c_src/nx_vulkan_shim.h:129-134); a full
// reduce is (1, n, 1).  Two kernel shapes:
//   rows (inner == 1): a CTA reduces one segment of one row with 16-byte
//     vector loads; S segments per row when rows are few (a full reduce uses
//     up to 4 CTAs per SM), each segment's partial goes to scratch and a
//     second launch folds the S partials of a row in index order;
//   cols (inner > 1): a thread owns one (o, j) column and walks r in order,
//     loads coalesced across j; R is split into S segments the same way when
//     outer*inner is too small to fill the GPU.
// The grid shape depends only on (outer, R, inner) and the SM count, and
// every combine happens in a fixed tree, so results are bit-reproducible.
// Accumulators: f32 sums in f64 (rounded once), f64 sums in double-double,
// max/min in the input type with NaN propagation, argmax as (value, index)
// under a total order (NaN first, then larger value, then lower index).
#include "kernels.h"
#include "ops_common.cuh"

#include <math.h>

namespace nxv {

namespace {

constexpr int kThreads = 256;

// ---- reducers -----------------------------------------------------------------

template <typename T> struct SumR;
// kU: 16-byte vectors in flight per thread in the segmented kernel (k_rows).
template <> struct SumR<float> {
    static constexpr int kU = 8;
    using Acc = double;
    using Out = float;
    __device__ static Acc init() { return 0.0; }
    __device__ static Acc add(Acc a, float x, long long) { return __dadd_rn(a, (double)x); }
    __device__ static Acc combine(Acc a, Acc b) { return __dadd_rn(a, b); }
    __device__ static Acc shfl(Acc a, int off) { return __shfl_down_sync(0xffffffffu, a, off); }
    __device__ static Out out(Acc a) { return (float)a; }
};
template <> struct SumR<double> {
    static constexpr int kU = 8;
    using Acc = dd;
    using Out = double;
    __device__ static Acc init() { return dd{0.0, 0.0}; }
    __device__ static Acc add(Acc a, double x, long long) { return dd_add_d(a, x); }
    __device__ static Acc combine(Acc a, Acc b) { return dd_add(a, b); }
    __device__ static Acc shfl(Acc a, int off) {
        return dd{__shfl_down_sync(0xffffffffu, a.hi, off), __shfl_down_sync(0xffffffffu, a.lo, off)};
    }
    __device__ static Out out(Acc a) { return dd_value(a); }
};

template <typename T, bool MAX> struct MaxR {
    static constexpr int kU = 8;
    using Acc = T;
    using Out = T;
    __device__ static Acc init() { return MAX ? -INFINITY : INFINITY; }
    // NaN propagates: a if a is NaN, else b if b is NaN, else the max (min).
    // f32 as selects (faster for the f32 kernels), f64 as early returns (the
    // select form measured 1.4x slower in the f64 segmented kernel); the
    // two forms give identical results.
    __device__ static Acc combine(Acc a, Acc b) {
        if constexpr (sizeof(T) == 4) {
            T r = MAX ? ((b > a) ? b : a) : ((b < a) ? b : a);
            r = (b != b) ? b : r;
            return (a != a) ? a : r;
        } else {
            if (a != a) return a;
            if (b != b) return b;
            return MAX ? ((b > a) ? b : a) : ((b < a) ? b : a);
        }
    }
    __device__ static Acc add(Acc a, T x, long long) { return combine(a, x); }
    __device__ static Acc shfl(Acc a, int off) { return __shfl_down_sync(0xffffffffu, a, off); }
    __device__ static Out out(Acc a) { return a; }
};

template <typename T> struct ArgAcc {
    T v;
    int i;  // index along the reduced axis (R < 2^31), -1 = empty
};
template <typename T, bool MIN> struct ArgR {
    static constexpr int kU = 4;
    using Acc = ArgAcc<T>;
    using Out = long long;
    __device__ static Acc init() { return Acc{MIN ? (T)INFINITY : (T)-INFINITY, -1}; }
    // Per-element update.  Every accumulator sees its elements in increasing
    // index order, so a strict comparison keeps the lowest index on ties, and
    // a NaN replaces only a non-NaN (the first NaN wins).
    __device__ static Acc add(Acc a, T x, long long idx) {
        const bool take = (a.i < 0) || (MIN ? (x < a.v) : (x > a.v)) || (x != x && a.v == a.v);
        return take ? Acc{x, (int)idx} : a;
    }
    // true when b should replace a
    __device__ static bool better(Acc a, Acc b) {
        if (b.i < 0) return false;
        if (a.i < 0) return true;
        bool an = a.v != a.v, bn = b.v != b.v;
        if (an || bn) {
            if (an && bn) return b.i < a.i;
            return bn;
        }
        if (b.v == a.v) return b.i < a.i;
        return MIN ? (b.v < a.v) : (b.v > a.v);
    }
    __device__ static Acc combine(Acc a, Acc b) { return better(a, b) ? b : a; }
    __device__ static Acc shfl(Acc a, int off) {
        return Acc{__shfl_down_sync(0xffffffffu, a.v, off), __shfl_down_sync(0xffffffffu, a.i, off)};
    }
    __device__ static Out out(Acc a) { return a.i < 0 ? 0 : a.i; }
};

template <class R>
__device__ typename R::Acc block_reduce(typename R::Acc a) {
    __shared__ typename R::Acc sm[kThreads / 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a = R::combine(a, R::shfl(a, off));
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) sm[w] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
        a = sm[0];
        for (int k = 1; k < (int)(blockDim.x >> 5); k++) a = R::combine(a, sm[k]);
    }
    return a;  // valid in thread 0
}

template <class R, typename T>
__device__ void write_out(void* out, size_t idx, typename R::Acc a, int index_bytes) {
    if constexpr (sizeof(typename R::Out) == 8 && !std::is_floating_point<typename R::Out>::value) {
        long long v = R::out(a);
        if (index_bytes == 4) ((int*)out)[idx] = (int)v;
        else ((long long*)out)[idx] = v;
    } else {
        ((typename R::Out*)out)[idx] = R::out(a);
    }
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// rows kernel: grid (S, rows).  Segment s of row r covers [s*L, min(R, (s+1)*L)).
// final: S == 1, writes the output; else writes Acc partial [r][s].  It lets
// its dependent (the fold, launched with programmatic dependent launch)
// start at once: the fold's CTAs wait for this grid to complete, so they are
// resident and begin the moment the last partial is written.  Launched
// itself with programmatic dependent launch (the segmented path), it waits
// for the previous kernel before its loads, or -- `early`: its input is not
// that kernel's output -- only before its writes (the previous call's fold
// may still be reading the partials).
template <class R, typename T>
__global__ void __launch_bounds__(kThreads)
k_rows(const T* __restrict__ a, size_t R_, size_t L, void* out, typename R::Acc* partial,
       int S, int index_bytes, int early) {
    griddep_launch();
    if (!early) griddep_wait();
    size_t r = blockIdx.y;
    size_t s = blockIdx.x;
    size_t beg = s * L, end = beg + L < R_ ? beg + L : R_;
    const T* row = a + r * R_;
    typename R::Acc acc = R::init();
    constexpr int W = (int)(16 / sizeof(T));
    constexpr int U = R::kU;  // vectors in flight per thread, one accumulator each
    // vector body when the segment start is 16-byte aligned
    size_t i = beg;
    if ((((uintptr_t)(row + beg)) & 15) == 0) {
        const size_t nv = (end - beg) / W;
        const size_t step = (size_t)blockDim.x * U;
        typename R::Acc part[U];
#pragma unroll
        for (int u = 0; u < U; u++) part[u] = R::init();
        size_t v = threadIdx.x;
        for (; v + (U - 1) * blockDim.x < nv; v += step) {
            T x[U][W];
#pragma unroll
            for (int u = 0; u < U; u++) vload(row + beg + (v + u * blockDim.x) * W, x[u]);
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int j = 0; j < W; j++)
                    part[u] = R::add(part[u], x[u][j], (long long)(beg + (v + u * blockDim.x) * W + j));
        }
        for (int u = 0; u < U; u++, v += blockDim.x) {
            if (v < nv) {
                T x[W];
                vload(row + beg + v * W, x);
#pragma unroll
                for (int j = 0; j < W; j++) part[u] = R::add(part[u], x[j], (long long)(beg + v * W + j));
            }
        }
        acc = part[0];
#pragma unroll
        for (int u = 1; u < U; u++) acc = R::combine(acc, part[u]);
        i = beg + nv * W;
    }
    for (size_t e = i + threadIdx.x; e < end; e += blockDim.x) acc = R::add(acc, row[e], (long long)e);
    acc = block_reduce<R>(acc);
    if (early) griddep_wait();
    if (threadIdx.x == 0) {
        if (S == 1) write_out<R, T>(out, r, acc, index_bytes);
        else partial[r * S + s] = acc;
    }
}

// Many rows: one warp per row, RPC rows (warps) per CTA, no shared memory or
// barrier.  Lane l takes vectors l, l+32, ... into U accumulators (vector v
// goes to accumulator (v / 32) % U, so each accumulator sees increasing
// indices; U = 8 for f64, 4 for f32); the U accumulators are combined in
// order, then a shuffle tree (lane i takes lane i + off) -- a fixed order.
// Small CTAs (RPC = 2) spread the rows evenly over the SMs: with 8 rows per
// CTA, 4096 rows leave some SMs 4 CTAs and others 3.  Requires R_ < 2^31
// (32-bit element index).
template <class R, typename T, int RPC>
__global__ void __launch_bounds__(32 * RPC)
k_rows_warp(const T* __restrict__ a, size_t outer, unsigned R_, void* out, int index_bytes,
            int early) {
    const size_t r = (size_t)blockIdx.x * RPC + (threadIdx.x >> 5);
    const unsigned lane = threadIdx.x & 31;
    if (r >= outer) return;  // the whole warp leaves together
    if (!early) griddep_wait();  // see pdl_row_launch
    const T* row = a + r * R_;
    constexpr int W = (int)(16 / sizeof(T));
    constexpr int U = sizeof(T) == 8 ? 8 : 4;  // 16-byte vectors in flight per lane
    typename R::Acc part[U];
#pragma unroll
    for (int u = 0; u < U; u++) part[u] = R::init();
    unsigned tail = 0;  // first element not covered by the vector body
    if ((((uintptr_t)row) & 15) == 0) {
        const unsigned nv = R_ / W;
        unsigned v = lane;
        for (; v + (U - 1) * 32 < nv; v += 32 * U) {
            T x[U][W];
#pragma unroll
            for (int u = 0; u < U; u++) vload(row + (size_t)(v + u * 32) * W, x[u]);
#pragma unroll
            for (int u = 0; u < U; u++)
#pragma unroll
                for (int j = 0; j < W; j++)
                    part[u] = R::add(part[u], x[u][j], (long long)((v + u * 32) * W + j));
        }
#pragma unroll
        for (int u = 0; u < U; u++, v += 32) {
            if (v < nv) {
                T x[W];
                vload(row + (size_t)v * W, x);
#pragma unroll
                for (int j = 0; j < W; j++) part[u] = R::add(part[u], x[j], (long long)(v * W + j));
            }
        }
        tail = nv * W;
    }
    for (unsigned e = tail + lane; e < R_; e += 32) part[U - 1] = R::add(part[U - 1], row[e], (long long)e);
    typename R::Acc acc = part[0];
#pragma unroll
    for (int u = 1; u < U; u++) acc = R::combine(acc, part[u]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = R::combine(acc, R::shfl(acc, off));
    if (early) griddep_wait();
    griddep_launch();
    if (lane == 0) write_out<R, T>(out, r, acc, index_bytes);
}

// Rows (warps) per CTA of the row kernels: NXV_ROW_CTA = 2, 4 or 8 (default 2).
int rows_per_cta() {
    if (const char* e = getenv("NXV_ROW_CTA")) {
        const int g = atoi(e);
        if (g == 2 || g == 4 || g == 8) return g;
    }
    return 2;
}

// The one-pass row kernels (k_rows_warp, k_lse_rows) run on programmatic
// dependent launch unless NXV_MAP_PDL=0: a kernel whose input is not the
// output of the previous programmatic launch on the stream (`early`, from
// the per-stream record) reads and reduces its rows while that kernel
// finishes and waits for it only before writing its results; otherwise it
// waits before its first load.  Either way it lets the next kernel start
// only after its own wait.
template <typename... KArgs, typename... Args>
int pdl_row_launch(Ctx& c, void (*kern)(KArgs...), unsigned grid, unsigned block, const void* in,
                   size_t in_bytes, const void* out, Args... args) {
    const char* ev = getenv("NXV_MAP_PDL");
    const bool pdl = !(ev && ev[0] == '0');
    const void* ins[1] = {in};
    const int early = pdl && pdl_independent_and_record(c, ins, 1, in_bytes, out) ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args..., early);
    return e == cudaSuccess ? OK : cuda_fail(e, "cudaLaunchKernelEx(row kernel)");
}

template <class R, typename T>
int launch_rows_warp(Ctx& c, const T* a, size_t outer, unsigned R_, void* out, int index_bytes) {
    const int rpc = rows_per_cta();
    const unsigned ctas = (unsigned)((outer + rpc - 1) / rpc);
    const size_t nb = outer * (size_t)R_ * sizeof(T);
    if (rpc == 8)
        return pdl_row_launch(c, k_rows_warp<R, T, 8>, ctas, 256, a, nb, out, a, outer, R_, out,
                              index_bytes);
    if (rpc == 4)
        return pdl_row_launch(c, k_rows_warp<R, T, 4>, ctas, 128, a, nb, out, a, outer, R_, out,
                              index_bytes);
    return pdl_row_launch(c, k_rows_warp<R, T, 2>, ctas, 64, a, nb, out, a, outer, R_, out,
                          index_bytes);
}

// Fold S partials per output in index order.
template <class R, typename T>
__global__ void k_fold(const typename R::Acc* __restrict__ partial, size_t n_out, int S,
                       size_t inner, void* out, int index_bytes) {
    // partial layout: [o][s][j] with n_out = outer*inner; rows case has inner = 1.
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_out) return;
    size_t o = t / inner, j = t - o * inner;
    typename R::Acc acc = partial[(o * S) * inner + j];
    for (int s = 1; s < S; s++) acc = R::combine(acc, partial[(o * S + s) * inner + j]);
    write_out<R, T>(out, t, acc, index_bytes);
}

// Rows case: one CTA folds the S partials of one row.  Thread t combines
// partials t, t+256, ... in order, then the fixed block tree finishes.
template <class R, typename T>
__global__ void __launch_bounds__(kThreads)
k_fold_rows(const typename R::Acc* __restrict__ partial, int S, void* out, int index_bytes) {
    griddep_wait();  // every partial of the segment kernel is written
    griddep_launch();
    const size_t o = blockIdx.x;
    typename R::Acc acc = R::init();
    for (int s = threadIdx.x; s < S; s += blockDim.x) acc = R::combine(acc, partial[o * S + s]);
    acc = block_reduce<R>(acc);
    if (threadIdx.x == 0) write_out<R, T>(out, o, acc, index_bytes);
}

// cols kernel: grid (ceil(inner/256), S, outer); thread owns column j.
template <class R, typename T>
__global__ void __launch_bounds__(kThreads)
k_cols(const T* __restrict__ a, size_t R_, size_t inner, size_t L, void* out,
       typename R::Acc* partial, int S, int index_bytes) {
    size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t s = blockIdx.y, o = blockIdx.z;
    if (j >= inner) return;
    size_t beg = s * L, end = beg + L < R_ ? beg + L : R_;
    const T* base = a + o * R_ * inner + j;
    typename R::Acc acc = R::init();
    for (size_t r = beg; r < end; r++) acc = R::add(acc, base[r * inner], (long long)r);
    if (S == 1) write_out<R, T>(out, o * inner + j, acc, index_bytes);
    else partial[(o * S + s) * inner + j] = acc;
}

template <class R, typename T>
int run_reduce(Ctx& c, const T* a, size_t outer, size_t R_, size_t inner, void* out,
               int index_bytes) {
    if (outer == 0 || inner == 0) return OK;
    using Acc = typename R::Acc;
    ScratchGuard guard(c);
    const size_t sms = (size_t)c.dev->sm_count;
    if (inner == 1) {
        // Segments per row: enough CTAs to fill the GPU, each >= 4096 elements.
        size_t S = 1;
        if (outer < 2 * sms) {
            size_t want = (4 * sms + outer - 1) / outer;
            size_t max_by_len = (R_ + 4095) / 4096;
            S = want < max_by_len ? want : max_by_len;
            if (S < 1) S = 1;
        }
        size_t L = (R_ + S - 1) / S;
        // keep segment starts 16-byte aligned when rows are
        L = (L + 3) & ~(size_t)3;
        if (L == 0) L = 4;
        S = (R_ + L - 1) / L;
        if (S == 0) S = 1;
        if (S == 1 && R_ < 0x80000000ull) {
            if ((outer + 1) / 2 > 0x7fffffffull) {
                set_error("too many rows for a reduce");
                return E_ARG;
            }
            int rc = launch_rows_warp<R, T>(c, a, outer, (unsigned)R_, out, index_bytes);
            if (rc) return rc;
            count_launch();
            return finish(c);
        }
        Acc* part = nullptr;
        if (S > 1) {
            part = (Acc*)scratch(c, outer * S * sizeof(Acc));
            if (!part) return E_CUDA;
        }
        if (outer > 65535 && S > 1) {
            set_error("too many rows for a segmented reduce");
            return E_ARG;
        }
        if (outer > 65535) {
            // one launch per 65535-row slab (grid.y limit)
            for (size_t r0 = 0; r0 < outer; r0 += 65535) {
                size_t rows = outer - r0 < 65535 ? outer - r0 : 65535;
                dim3 grid(1, (unsigned)rows);
                void* o2 = (char*)out + r0 * (index_bytes ? (size_t)index_bytes : sizeof(typename R::Out));
                k_rows<R, T><<<grid, kThreads, 0, c.stream>>>(a + r0 * R_, R_, L, o2, nullptr, 1,
                                                              index_bytes, 0);
                count_launch();
            }
            return finish(c);
        }
        dim3 grid((unsigned)S, (unsigned)outer);
        {
            // programmatic dependent launch unless NXV_MAP_PDL=0
            const char* ev = getenv("NXV_MAP_PDL");
            const bool pdl = !(ev && ev[0] == '0');
            const void* ins[1] = {a};
            const int early =
                pdl && pdl_independent_and_record(c, ins, 1, outer * R_ * sizeof(T), out) ? 1 : 0;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = grid;
            cfg.blockDim = dim3(kThreads);
            cfg.stream = c.stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = pdl ? 1 : 0;
            cudaError_t e = cudaLaunchKernelEx(&cfg, k_rows<R, T>, a, R_, L, out, part, (int)S,
                                               index_bytes, early);
            if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(k_rows)");
        }
        count_launch();
        if (S > 1) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)outer);
            cfg.blockDim = dim3(kThreads);
            cfg.stream = c.stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t e = cudaLaunchKernelEx(&cfg, k_fold_rows<R, T>,
                                               (const typename R::Acc*)part, (int)S, out,
                                               index_bytes);
            if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(k_fold_rows)");
            count_launch();
        }
        return finish(c);
    }
    size_t cols = outer * inner;
    size_t S = 1;
    size_t target = 4 * sms * kThreads;
    if (cols < target && R_ > 256) {
        S = (target + cols - 1) / cols;
        size_t max_s = R_ / 64;
        if (S > max_s) S = max_s;
        if (S > 1024) S = 1024;
        if (S < 1) S = 1;
    }
    size_t L = (R_ + S - 1) / S;
    S = (R_ + L - 1) / L;
    if (S == 0) S = 1;
    if (outer > 65535) {
        set_error("outer extent %zu exceeds the grid limit", outer);
        return E_ARG;
    }
    Acc* part = nullptr;
    if (S > 1) {
        part = (Acc*)scratch(c, cols * S * sizeof(Acc));
        if (!part) return E_CUDA;
    }
    dim3 grid((unsigned)((inner + kThreads - 1) / kThreads), (unsigned)S, (unsigned)outer);
    k_cols<R, T><<<grid, kThreads, 0, c.stream>>>(a, R_, inner, L, out, part, (int)S, index_bytes);
    count_launch();
    if (S > 1) {
        k_fold<R, T><<<(unsigned)((cols + 127) / 128), 128, 0, c.stream>>>(part, cols, (int)S, inner,
                                                                          out, index_bytes);
        count_launch();
    }
    return finish(c);
}

// ---- logsumexp (f32 in/out, f64 math) --------------------------------------------

// One warp per row, one pass over the row (online logsumexp).  Each lane
// keeps a running max m and s = sum of exp(x - m) over the elements it has
// seen (double); when a group of 16 elements raises the max, s is rescaled by
// exp(m_old - m_new).  The 32 lane states merge in a fixed shuffle tree:
// s = s_a exp(m_a - M) + s_b exp(m_b - M).  The special values follow the
// two-pass definition the oracle uses (max ignoring NaN, then sum of
// exp(x - max)): a NaN, a +inf, or a row of only -inf/NaN gives NaN (lanes
// whose elements are all -inf, or that have none, hold m = -inf, s = 0).  NaN
// never enters m (fmaxf ignores it); while m is -inf every element seen was
// -inf or NaN, and terms are taken against 0 so that NaN propagates and -inf
// adds 0.  EX: exp in f64 (the oracle's evaluation; NXV_EXACT_F32=1), else
// the hardware exponential __expf of the f32 difference, 16 terms summed in
// f32 before the double add.  __expf's error grows with |x - max|, but a
// term's weight in the sum falls as e^(x - max), so the result stays within
// 4 ulp of the f64 evaluation rounded once (measured over rows of 1 to
// 100,003 N(0, 100) elements; exact with EX) -- 13.9 us instead of 15.1 us
// with expf on [4096, 4096].
template <bool EX>
struct LseLane {
    float m = -INFINITY;
    double s = 0.0;
    __device__ __forceinline__ void raise_to(float bm) {
        if (bm > m) {
            if constexpr (EX) s *= exp((double)m - (double)bm);
            else s *= (double)expf(m - bm);
            m = bm;
        }
    }
    __device__ __forceinline__ float ref() const { return m == -INFINITY ? 0.f : m; }
    __device__ __forceinline__ double term(float x, float r) const {
        if constexpr (EX) return exp((double)x - (double)r);
        else return (double)expf(x - r);
    }
};

template <bool EX, int U>
__device__ __forceinline__ void lse_group(LseLane<EX>& L, const float4 (&x)[U]) {
    float bm = -INFINITY;
#pragma unroll
    for (int u = 0; u < U; u++) bm = fmaxf(bm, fmaxf(fmaxf(x[u].x, x[u].y), fmaxf(x[u].z, x[u].w)));
    L.raise_to(bm);
    const float r = L.ref();
    if constexpr (EX) {
        double t = 0.0;
#pragma unroll
        for (int u = 0; u < U; u++)
            t = __dadd_rn(t, __dadd_rn(__dadd_rn(L.term(x[u].x, r), L.term(x[u].y, r)),
                                       __dadd_rn(L.term(x[u].z, r), L.term(x[u].w, r))));
        L.s = __dadd_rn(L.s, t);
    } else {
        float t = 0.f;
#pragma unroll
        for (int u = 0; u < U; u++)
            t = add_(t, add_(add_(__expf(x[u].x - r), __expf(x[u].y - r)),
                             add_(__expf(x[u].z - r), __expf(x[u].w - r))));
        L.s = __dadd_rn(L.s, (double)t);
    }
}

template <bool EX>
__device__ __forceinline__ void lse_merge(LseLane<EX>& L, float mo, double so) {
    const float M = fmaxf(L.m, mo);
    // factor 1 for the side that holds the max (also when both are -inf:
    // two lanes without finite elements must not make 0 * exp(NaN))
    const double fa = L.m == M ? 1.0 : exp((double)L.m - (double)M);
    const double fb = mo == M ? 1.0 : exp((double)mo - (double)M);
    L.s = __dadd_rn(__dmul_rn(L.s, fa), __dmul_rn(so, fb));
    L.m = M;
}

// One warp per row, RPC rows per CTA (as k_rows_warp).
template <bool EX, int RPC>
__global__ void __launch_bounds__(32 * RPC)
k_lse_rows(const float* __restrict__ a, size_t outer, unsigned R_, float* __restrict__ out,
           int early) {
    const size_t r = (size_t)blockIdx.x * RPC + (threadIdx.x >> 5);
    const unsigned lane = threadIdx.x & 31;
    if (r >= outer) return;
    if (!early) griddep_wait();  // see pdl_row_launch
    const float* row = a + r * R_;
    const bool vec = (((uintptr_t)row) & 15) == 0;
    const unsigned nv = vec ? R_ / 4 : 0;
    const float4* rv = reinterpret_cast<const float4*>(row);
    constexpr int U = EX ? 2 : 4;  // 16-byte loads in flight per lane (EX: f64 exp is register-heavy)
    LseLane<EX> L;
    unsigned v = lane;
    for (; v + (U - 1) * 32 < nv; v += 32 * U) {
        float4 x[U];
#pragma unroll
        for (int u = 0; u < U; u++) x[u] = __ldcs(rv + v + u * 32);
        lse_group<EX, U>(L, x);
    }
    for (; v < nv; v += 32) {
        float4 x[1] = {__ldcs(rv + v)};
        lse_group<EX, 1>(L, x);
    }
    for (unsigned e = nv * 4 + lane; e < R_; e += 32) {
        const float x = row[e];
        L.raise_to(x);
        L.s = __dadd_rn(L.s, L.term(x, L.ref()));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        lse_merge(L, __shfl_down_sync(0xffffffffu, L.m, off), __shfl_down_sync(0xffffffffu, L.s, off));
    if (early) griddep_wait();
    griddep_launch();
    if (lane == 0)
        out[r] = L.m == -INFINITY ? __int_as_float(0x7fc00000) : (float)(log(L.s) + (double)L.m);
}

template <bool EX>
int launch_lse_rows(Ctx& c, const float* a, size_t outer, unsigned R_, float* out) {
    const int rpc = rows_per_cta();
    const unsigned ctas = (unsigned)((outer + rpc - 1) / rpc);
    const size_t nb = outer * (size_t)R_ * 4;
    if (rpc == 8) return pdl_row_launch(c, k_lse_rows<EX, 8>, ctas, 256, a, nb, out, a, outer, R_, out);
    if (rpc == 4) return pdl_row_launch(c, k_lse_rows<EX, 4>, ctas, 128, a, nb, out, a, outer, R_, out);
    return pdl_row_launch(c, k_lse_rows<EX, 2>, ctas, 64, a, nb, out, a, outer, R_, out);
}

__global__ void __launch_bounds__(kThreads)
k_lse_cols(const float* __restrict__ a, size_t R_, size_t inner, float* out) {
    size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t o = blockIdx.y;
    if (j >= inner) return;
    const float* base = a + o * R_ * inner + j;
    double mx = -INFINITY;
    for (size_t r = 0; r < R_; r++) {
        double v = base[r * inner];
        if (v > mx) mx = v;
    }
    double s = 0.0;
    for (size_t r = 0; r < R_; r++) s += exp((double)base[r * inner] - mx);
    out[o * inner + j] = (float)(log(s) + mx);
}

// ---- kinetic energy partials -------------------------------------------------------

// out[g] = 0.5 * sum over the 256 elements of group g of (p*p)*m (the
// reference's per-workgroup partials).  One warp per group: lane l takes
// elements 8l .. 8l+7 (two 16-byte loads of p and of m when aligned),
// terms in f32 as (p*p)*m, sums in double, then a fixed shuffle tree.
__global__ void __launch_bounds__(kThreads)
k_kinetic(const float* __restrict__ p, const float* __restrict__ m, size_t n, float* out) {
    const size_t grp = (size_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    const unsigned lane = threadIdx.x & 31;
    const size_t ngrp = (n + 255) / 256;
    if (grp >= ngrp) return;
    const size_t i0 = grp * 256 + (size_t)lane * 8;
    double t = 0.0;
    if (i0 + 8 <= n && (((uintptr_t)(p + i0)) & 15) == 0 && (((uintptr_t)(m + i0)) & 15) == 0) {
        const float4 p0 = *reinterpret_cast<const float4*>(p + i0);
        const float4 p1 = *reinterpret_cast<const float4*>(p + i0 + 4);
        const float4 m0 = *reinterpret_cast<const float4*>(m + i0);
        const float4 m1 = *reinterpret_cast<const float4*>(m + i0 + 4);
        const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) t = __dadd_rn(t, (double)mul_(mul_(pv[e], pv[e]), mv[e]));
    } else {
        for (int e = 0; e < 8; e++) {
            const size_t i = i0 + e;
            if (i < n) t = __dadd_rn(t, (double)mul_(mul_(p[i], p[i]), m[i]));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t = __dadd_rn(t, __shfl_down_sync(0xffffffffu, t, off));
    if (lane == 0) out[grp] = (float)(0.5 * t);
}

}  // namespace

int launch_reduce_full(Ctx& c, int dt, void* out_dev, const void* a, size_t n, unsigned op) {
    if (n == 0) {
        set_error("reduce of an empty tensor");
        return E_ARG;
    }
    if (dt == F32) {
        const float* x = (const float*)a;
        if (op == 0) return run_reduce<SumR<float>, float>(c, x, 1, n, 1, out_dev, 0);
        if (op == 1) return run_reduce<MaxR<float, false>, float>(c, x, 1, n, 1, out_dev, 0);
        return run_reduce<MaxR<float, true>, float>(c, x, 1, n, 1, out_dev, 0);
    }
    const double* x = (const double*)a;
    if (op == 0) return run_reduce<SumR<double>, double>(c, x, 1, n, 1, out_dev, 0);
    if (op == 1) return run_reduce<MaxR<double, false>, double>(c, x, 1, n, 1, out_dev, 0);
    return run_reduce<MaxR<double, true>, double>(c, x, 1, n, 1, out_dev, 0);
}

int launch_reduce_axis(Ctx& c, int dt, void* out, const void* a, size_t outer, size_t R,
                       size_t inner, unsigned op) {
    if (R == 0) {
        set_error("reduce over an empty axis");
        return E_ARG;
    }
    if (dt == F32) {
        const float* x = (const float*)a;
        if (op == 0) return run_reduce<SumR<float>, float>(c, x, outer, R, inner, out, 0);
        if (op == 1) return run_reduce<MaxR<float, true>, float>(c, x, outer, R, inner, out, 0);
        return run_reduce<MaxR<float, false>, float>(c, x, outer, R, inner, out, 0);
    }
    const double* x = (const double*)a;
    if (op == 0) return run_reduce<SumR<double>, double>(c, x, outer, R, inner, out, 0);
    if (op == 1) return run_reduce<MaxR<double, true>, double>(c, x, outer, R, inner, out, 0);
    return run_reduce<MaxR<double, false>, double>(c, x, outer, R, inner, out, 0);
}

int launch_argmax(Ctx& c, int dt, void* out, const void* a, size_t outer, size_t R,
                  size_t inner, int is_min, int index_bytes) {
    if (R == 0) {
        set_error("argmax over an empty axis");
        return E_ARG;
    }
    if (R > 0x7fffffffull) {
        set_error("argmax axis of %zu elements exceeds 2^31 - 1", R);
        return E_ARG;
    }
    if (dt == F32) {
        if (is_min) return run_reduce<ArgR<float, true>, float>(c, (const float*)a, outer, R, inner, out, index_bytes);
        return run_reduce<ArgR<float, false>, float>(c, (const float*)a, outer, R, inner, out, index_bytes);
    }
    if (is_min) return run_reduce<ArgR<double, true>, double>(c, (const double*)a, outer, R, inner, out, index_bytes);
    return run_reduce<ArgR<double, false>, double>(c, (const double*)a, outer, R, inner, out, index_bytes);
}

int launch_logsumexp(Ctx& c, void* out, const void* a, size_t outer, size_t R, size_t inner) {
    if (R == 0 || outer == 0 || inner == 0) return OK;
    if (inner == 1) {
        if ((outer + 1) / 2 > 0x7fffffff || R > 0xffffffffull) {
            set_error("logsumexp extents out of range");
            return E_ARG;
        }
        const int rc =
            fast_f32() ? launch_lse_rows<false>(c, (const float*)a, outer, (unsigned)R, (float*)out)
                       : launch_lse_rows<true>(c, (const float*)a, outer, (unsigned)R, (float*)out);
        if (rc) return rc;
    } else {
        if (outer > 65535) return E_ARG;
        dim3 grid((unsigned)((inner + kThreads - 1) / kThreads), (unsigned)outer);
        k_lse_cols<<<grid, kThreads, 0, c.stream>>>((const float*)a, R, inner, (float*)out);
    }
    count_launch();
    return finish(c);
}

int launch_kinetic_energy(Ctx& c, void* out, const void* p, const void* m, size_t n) {
    if (n == 0) return OK;
    const size_t groups = (n + 255) / 256;
    const size_t ctas = (groups + kThreads / 32 - 1) / (kThreads / 32);
    k_kinetic<<<(unsigned)ctas, kThreads, 0, c.stream>>>((const float*)p, (const float*)m, n,
                                                         (float*)out);
    count_launch();
    return finish(c);
}

}  // namespace nxv
