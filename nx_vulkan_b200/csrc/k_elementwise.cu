// k_elementwise.cu -- binary, unary, cast, broadcast, transpose and the
// fused op-tape kernels (sm_100a).
//
// All of these are HBM-bound: bytes per element are (inputs + 1) * sizeof(T)
// and the arithmetic is a few instructions.  Design:
//   - 128-bit vector loads/stores (float4 / double2) when every pointer is
//     16-byte aligned (pool buffers always are), scalar path otherwise;
//   - grid-stride loops with a grid of up to 8 CTAs x 256 threads per SM and
//     4 vectors in flight per thread (all loads issued before the math);
//   - the op tape (lib/nx_vulkan.ex:457-538, c_src/nx_vulkan_shim.cpp:865-929)
//     is interpreted from kernel parameters with every operand preloaded, and
//     hot chains have compile-time specialisations with no dispatch at all.
#include "kernels.h"
#include "ops_common.cuh"

#include <algorithm>
#include <type_traits>

namespace nxv {

namespace {

constexpr int kThreads = 256;
// The f64 pipelined map runs 128-thread CTAs: with the same registers per
// SM a CTA of the next call can start as soon as any 128 threads of the
// current one finish (config 1 f64 7.42 -> 7.19 us against 256 threads).
constexpr int kPipeThreads = 128;
// The exact-f32 staged map (its shared-memory slots are per thread).
constexpr int kStagedThreads = 256;
constexpr int kUnroll = 4;

inline bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// ---- generic n-ary map ------------------------------------------------------

// NXV_MAP_WIDE=0: small vector maps keep kUnroll vectors per thread.
bool map_wide() {
    const char* e = getenv("NXV_MAP_WIDE");
    return !(e && e[0] == '0');
}

// F: T operator()(const T* in_vals) over NIN inputs.
template <typename T, int NIN, class F, bool VEC>
__global__ void __launch_bounds__(kThreads)
k_map(T* __restrict__ out, const T* __restrict__ in0, const T* __restrict__ in1,
      const T* __restrict__ in2, const T* __restrict__ in3, size_t n, F f) {
    const T* ins[4] = {in0, in1, in2, in3};
    constexpr int W = VEC ? (int)(16 / sizeof(T)) : 1;
    const size_t nv = n / W;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; v + (kUnroll - 1) * stride < nv; v += kUnroll * stride) {
        T x[kUnroll][NIN > 0 ? NIN : 1][W];
#pragma unroll
        for (int u = 0; u < kUnroll; u++)
#pragma unroll
            for (int q = 0; q < NIN; q++) {
                const T* src = ins[q] + (v + u * stride) * W;
                if constexpr (VEC) {
                    vload(src, *reinterpret_cast<T(*)[16 / sizeof(T)]>(x[u][q]));
                } else {
                    x[u][q][0] = src[0];
                }
            }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            T r[W];
#pragma unroll
            for (int j = 0; j < W; j++) {
                T args[NIN > 0 ? NIN : 1];
#pragma unroll
                for (int q = 0; q < NIN; q++) args[q] = x[u][q][j];
                r[j] = f(args);
            }
            T* dst = out + (v + u * stride) * W;
            if constexpr (VEC) {
                vstore(dst, *reinterpret_cast<T(*)[16 / sizeof(T)]>(r));
            } else {
                dst[0] = r[0];
            }
        }
    }
    // the rest, one vector per step (the whole array when the grid covers it
    // with one vector per thread); every input's load is issued before the math
    for (; v < nv; v += stride) {
        T x[NIN > 0 ? NIN : 1][W];
#pragma unroll
        for (int q = 0; q < NIN; q++) {
            if constexpr (VEC) {
                vload(ins[q] + v * W, *reinterpret_cast<T(*)[16 / sizeof(T)]>(x[q]));
            } else {
                x[q][0] = ins[q][v];
            }
        }
        T r[W];
#pragma unroll
        for (int j = 0; j < W; j++) {
            T args[NIN > 0 ? NIN : 1];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = x[q][j];
            r[j] = f(args);
        }
        if constexpr (VEC) {
            vstore(out + v * W, *reinterpret_cast<T(*)[16 / sizeof(T)]>(r));
        } else {
            out[v] = r[0];
        }
    }
    if (VEC && blockIdx.x == 0) {  // tail of n % W elements
        size_t t = nv * W + threadIdx.x;
        if (t < n) {
            T args[NIN > 0 ? NIN : 1];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = ins[q][t];
            out[t] = f(args);
        }
    }
}

// ---- one-wave map with programmatic dependent launch ---------------------------
//
// Small f32 maps (a grid of one vector per thread that fits the SMs in one
// wave, 2^20 elements and below) are bound by the launch, the DRAM latency of
// their first loads and the drain of their last stores, not by bandwidth.
// k_map1 runs them in one wave (launch bounds of 8 CTAs x 256 threads per SM)
// and is launched with programmatic dependent launch: its CTAs may start while
// the previous kernel on the stream finishes.  Each CTA
//   1. loads its inputs at once when none of them overlaps the output of the
//      previous kernel launched this way on the stream (`early`; the host
//      tracks that range per stream, Device::pdl_last),
//   2. waits for the previous kernel to complete (griddepcontrol.wait),
//   3. lets the next kernel's CTAs launch (griddepcontrol.launch_dependents),
//   4. loads its inputs now if it did not in step 1, computes and stores.
// Every kernel passes step 2 before step 3, so when a kernel's CTAs start,
// every kernel but the one immediately before it has completed: an early
// load never reads memory that a running kernel writes, and no store happens
// before the previous kernel has completed.  A predecessor that is not
// launched this way (any other kernel) lets its dependents start only when it
// completes.  NXV_MAP_PDL=0 launches k_map1 without the attribute.

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename T, int NIN, class F>
__global__ void __launch_bounds__(kThreads, 8)
k_map1(T* __restrict__ out, const T* __restrict__ in0, const T* __restrict__ in1,
       const T* __restrict__ in2, const T* __restrict__ in3, size_t n, F f, int early) {
    constexpr int W = (int)(16 / sizeof(T));
    const T* ins[4] = {in0, in1, in2, in3};
    const size_t nv = n / W;
    const size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool have = v < nv;
    T x[NIN > 0 ? NIN : 1][W];
    if (early && have) {
#pragma unroll
        for (int q = 0; q < NIN; q++) vload(ins[q] + v * W, x[q]);
    }
    griddep_wait();
    griddep_launch();
    if (!early && have) {
#pragma unroll
        for (int q = 0; q < NIN; q++) vload(ins[q] + v * W, x[q]);
    }
    if (have) {
        T r[W];
#pragma unroll
        for (int j = 0; j < W; j++) {
            T args[NIN > 0 ? NIN : 1];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = x[q][j];
            r[j] = f(args);
        }
        vstore(out + v * W, r);
    }
    if (blockIdx.x == 0) {  // tail of n % W elements
        const size_t t = nv * W + threadIdx.x;
        if (t < n) {
            T args[NIN > 0 ? NIN : 1];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = ins[q][t];
            out[t] = f(args);
        }
    }
}

// Functors whose f32 arithmetic goes through f64 (the exact mode) need more
// registers than k_map1's launch bounds allow; they keep the grid-stride map.
template <class F, class = void> struct Heavy { static constexpr bool value = false; };
template <class F> struct Heavy<F, std::void_t<decltype(F::kHeavy)>> {
    static constexpr bool value = F::kHeavy;
};

bool map_pdl() {
    const char* e = getenv("NXV_MAP_PDL");
    return !(e && e[0] == '0');
}

// Launches a map kernel (k_map1, k_map_pipe or k_map_staged: parameters
// out, in0..in3, n, f, early) of `block` threads per CTA with programmatic
// dependent launch unless NXV_MAP_PDL=0.
template <typename T, class F>
int launch_pdl(Ctx& c, void (*kern)(T*, const T*, const T*, const T*, const T*, size_t, F, int),
               const char* name, unsigned grid, T* out, const T* i0, const T* i1, const T* i2,
               const T* i3, size_t n, F f, int nin, int block = kThreads) {
    const void* ins[4] = {i0, i1, i2, i3};
    const bool pdl = map_pdl();
    const int early = pdl && pdl_independent_and_record(c, ins, nin, n * sizeof(T), out) ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, out, i0, i1, i2, i3, n, f, early);
    if (e != cudaSuccess) return cuda_fail(e, name);
    count_launch();
    return finish(c);
}

// Resident CTAs of k_map1<T, NIN, F> per SM (looked up once per instantiation).
template <typename T, int NIN, class F>
int map1_per_sm() {
    static const int occ = []() {
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_map1<T, NIN, F>, kThreads, 0) !=
            cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return o;
    }();
    return occ;
}

// ---- software-pipelined map for arithmetic-heavy functors ------------------------
//
// f64 maps and the exact f32 mode spend about as long in FP64 arithmetic as in
// moving their bytes.  k_map_pipe (the f64 maps) runs one wave of CTAs whose threads walk
// the array one vector at a time and keep the next two vectors' loads in
// flight while they do the math of the current one (the grid-stride form
// with all loads first and all math after serialises the two across the
// whole GPU when one wave covers the array).  Two vectors ahead rather than
// one: config 1 exact f32 6.59 -> 6.12 us, f64 8.03 -> 8.00 us.  Under
// programmatic dependent launch the first two vectors are loaded before the
// wait only when no input overlaps the previous kernel's output.

template <typename T, int NIN, class F>
__global__ void __launch_bounds__(kPipeThreads)
k_map_pipe(T* __restrict__ out, const T* __restrict__ in0, const T* __restrict__ in1,
           const T* __restrict__ in2, const T* __restrict__ in3, size_t n, F f, int early) {
    constexpr int W = (int)(16 / sizeof(T));
    const T* ins[4] = {in0, in1, in2, in3};
    const size_t nv = n / W;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    T nx[NIN > 0 ? NIN : 1][W], ny[NIN > 0 ? NIN : 1][W];
    if (early) {
        if (v < nv) {
#pragma unroll
            for (int q = 0; q < NIN; q++) vload(ins[q] + v * W, nx[q]);
        }
        if (v + stride < nv) {
#pragma unroll
            for (int q = 0; q < NIN; q++) vload(ins[q] + (v + stride) * W, ny[q]);
        }
    }
    griddep_wait();
    griddep_launch();
    if (!early) {
        if (v < nv) {
#pragma unroll
            for (int q = 0; q < NIN; q++) vload(ins[q] + v * W, nx[q]);
        }
        if (v + stride < nv) {
#pragma unroll
            for (int q = 0; q < NIN; q++) vload(ins[q] + (v + stride) * W, ny[q]);
        }
    }
    for (; v < nv; v += stride) {
        T x[NIN > 0 ? NIN : 1][W];
#pragma unroll
        for (int q = 0; q < NIN; q++)
#pragma unroll
            for (int j = 0; j < W; j++) {
                x[q][j] = nx[q][j];
                nx[q][j] = ny[q][j];
            }
        const size_t vn = v + 2 * stride;
        if (vn < nv) {
#pragma unroll
            for (int q = 0; q < NIN; q++) vload(ins[q] + vn * W, ny[q]);
        }
        T r[W];
#pragma unroll
        for (int j = 0; j < W; j++) {
            T args[NIN > 0 ? NIN : 1];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = x[q][j];
            r[j] = f(args);
        }
        vstore(out + v * W, r);
    }
    if (blockIdx.x == 0) {  // tail of n % W elements
        const size_t t = nv * W + threadIdx.x;
        if (t < n) {
            T args[NIN > 0 ? NIN : 1];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = ins[q][t];
            out[t] = f(args);
        }
    }
}

// The exact-f32 functors keep fewer values live than the f64 ones, and their
// math wants more resident warps than registers allow with two vectors
// held in registers: k_map_staged keeps the vectors in flight in shared
// memory instead (cp.async, three stages of 16 bytes per thread and input),
// which brings it to 38-40 registers and six CTAs per SM (config 1 exact
// 6.11 -> 5.95 us; the f64 chain is slower this way, 7.4 -> 8.2 us).  Each
// thread reads back only the slots it filled, after cp.async.wait_group,
// and refills a slot only after the math that used its values.

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T, int NIN, class F>
__global__ void __launch_bounds__(kStagedThreads)
k_map_staged(T* __restrict__ out, const T* __restrict__ in0, const T* __restrict__ in1,
             const T* __restrict__ in2, const T* __restrict__ in3, size_t n, F f, int early) {
    constexpr int W = (int)(16 / sizeof(T));
    constexpr int NB = NIN > 0 ? NIN : 1;
    constexpr int S = 3;  // the current vector and the next two in flight
    __shared__ uint4 slot[S][NB][kStagedThreads];
    const T* ins[4] = {in0, in1, in2, in3};
    const size_t nv = n / W;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    // one commit group per vector (empty past the end), so that
    // wait_group S - 1 always means "the oldest vector has landed"
    auto issue = [&](int st, size_t u) {
        if (u < nv) {
#pragma unroll
            for (int q = 0; q < NIN; q++) cp_async16(&slot[st][q][threadIdx.x], ins[q] + u * W);
        }
        cp_async_commit();
    };
    if (early) {
        issue(0, v);
        issue(1, v + stride);
    }
    griddep_wait();
    griddep_launch();
    if (!early) {
        issue(0, v);
        issue(1, v + stride);
    }
    int st = 0;
    for (; v < nv; v += stride) {
        issue(st == 0 ? S - 1 : st - 1, v + (S - 1) * stride);
        cp_async_wait<S - 1>();
        T r[W];
        T x[NB][W];
#pragma unroll
        for (int q = 0; q < NIN; q++) {
            const uint4 raw = slot[st][q][threadIdx.x];
            const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int j = 0; j < W; j++) x[q][j] = e[j];
        }
#pragma unroll
        for (int j = 0; j < W; j++) {
            T args[NB];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = x[q][j];
            r[j] = f(args);
        }
        vstore(out + v * W, r);
        st = st == S - 1 ? 0 : st + 1;
    }
    cp_async_wait<0>();
    if (blockIdx.x == 0) {  // tail of n % W elements
        const size_t t = nv * W + threadIdx.x;
        if (t < n) {
            T args[NB];
#pragma unroll
            for (int q = 0; q < NIN; q++) args[q] = ins[q][t];
            out[t] = f(args);
        }
    }
}

// Resident CTAs of a map kernel per SM (looked up once per instantiation).
template <typename T, int NIN, class F, bool STAGED>
int map_per_sm() {
    static const int occ = []() {
        int o = 0;
        cudaError_t e;
        if constexpr (STAGED)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_map_staged<T, NIN, F>,
                                                              kStagedThreads, 0);
        else
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, k_map_pipe<T, NIN, F>,
                                                              kPipeThreads, 0);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return o;
    }();
    return occ;
}

// NXV_MAP_PIPE=0: arithmetic-heavy maps use the grid-stride kernel.
bool map_pipe() {
    const char* e = getenv("NXV_MAP_PIPE");
    return !(e && e[0] == '0');
}

template <typename T, int NIN, class F>
int run_map(Ctx& c, T* out, const T* i0, const T* i1, const T* i2, const T* i3, size_t n, F f) {
    if (n == 0) return OK;
    bool vec = al16(out) && al16(i0) && (NIN < 2 || al16(i1)) && (NIN < 3 || al16(i2)) &&
               (NIN < 4 || al16(i3));
    constexpr int W = (int)(16 / sizeof(T));
    if constexpr (sizeof(T) == 4 && !Heavy<F>::value) {
        // one vector per thread in a single wave
        const size_t nv = n / W;
        const size_t wave = (size_t)c.dev->sm_count * map1_per_sm<T, NIN, F>() * kThreads;
        if (vec && map_wide() && nv >= 1 && nv <= wave)
            return launch_pdl(c, k_map1<T, NIN, F>, "cudaLaunchKernelEx(k_map1)",
                              (unsigned)((nv + kThreads - 1) / kThreads), out, i0, i1, i2, i3,
                              n, f, NIN);
    }
    if constexpr (sizeof(T) == 8 || Heavy<F>::value) {
        const size_t nv = n / W;
        constexpr bool staged = sizeof(T) == 4;  // exact f32 math
        const int occ = map_per_sm<T, NIN, F, staged>();
        if (vec && map_pipe() && nv >= 1 && occ > 0) {
            constexpr int bt = staged ? kStagedThreads : kPipeThreads;
            const size_t want = (nv + bt - 1) / bt;
            const unsigned g =
                (unsigned)std::min<size_t>(want, (size_t)c.dev->sm_count * (size_t)occ);
            if constexpr (staged)
                return launch_pdl(c, k_map_staged<T, NIN, F>, "cudaLaunchKernelEx(k_map_staged)",
                                  g, out, i0, i1, i2, i3, n, f, NIN, bt);
            else
                return launch_pdl(c, k_map_pipe<T, NIN, F>, "cudaLaunchKernelEx(k_map_pipe)", g,
                                  out, i0, i1, i2, i3, n, f, NIN, bt);
        }
    }
    if (vec) {
        // f32 arrays that one full grid covers with a vector or so per thread
        // run wide (one vector per thread, up to 8 CTAs per SM): 2^20
        // elements 5.3 -> 4.8 us.  Larger arrays, and f64 (whose
        // transcendentals want several vectors per thread: 2^20 10.2 -> 10.9
        // us wide), take kUnroll vectors per thread per step.
        const size_t nv = n / W;
        const size_t full = (size_t)c.dev->sm_count * 8 * kThreads;
        unsigned g = (sizeof(T) == 4 && map_wide() && nv <= full * kUnroll)
                         ? grid_for(c, nv, kThreads, 8)
                         : grid_for(c, (nv + kUnroll - 1) / kUnroll, kThreads, 8);
        k_map<T, NIN, F, true><<<g, kThreads, 0, c.stream>>>(out, i0, i1, i2, i3, n, f);
    } else {
        unsigned g = grid_for(c, (n + kUnroll - 1) / kUnroll, kThreads, 8);
        k_map<T, NIN, F, false><<<g, kThreads, 0, c.stream>>>(out, i0, i1, i2, i3, n, f);
    }
    count_launch();
    return finish(c);
}

// EX: f32 transcendentals evaluated in f64 and rounded (Nx.BinaryBackend
// semantics) when true, f32 library functions when false (the default;
// NXV_EXACT_F32=1 selects the first).
template <typename T, bool EX> struct BinF {
    static constexpr bool kHeavy = EX;  // f64 math: many registers
    unsigned op;
    __device__ T operator()(const T* x) const { return bin_op<T, EX>(x[0], x[1], op); }
};
template <typename T, bool EX> struct UnF {
    static constexpr bool kHeavy = EX;  // f64 math: many registers
    unsigned op;
    __device__ T operator()(const T* x) const { return un_op<T, EX>(x[0], op); }
};

// ---- fused op tape: generic interpreter --------------------------------------

template <typename T> struct TapeDev {
    unsigned n_ops;
    unsigned ops[8];
    unsigned src[8];
    T imm[8];
};

template <typename T, bool EX> struct TapeF {
    static constexpr bool kHeavy = EX;  // f64 math: many registers
    TapeDev<T> t;
    // x[0] = a, x[1] = b, x[2] = c, x[3] = d (unused ones are never read)
    __device__ T operator()(const T* x) const {
        T r = x[0];
#pragma unroll 1
        for (unsigned k = 0; k < t.n_ops; k++) {
            unsigned op = t.ops[k];
            if (op < 100) {
                unsigned s = t.src[k];
                T rhs = (s == 0) ? t.imm[k] : x[s];
                r = bin_op<T, EX>(r, rhs, op);
            } else if (op != 255) {
                r = un_op<T, EX>(r, op - 100);
            }
        }
        return r;
    }
};

// ---- fused op tape: compile-time specialisations of hot chains -------------

// tanh(exp(a*b + c) - imm0): the Nx.Defn chain tanh(exp(x*y + z) - 1.0).
template <typename T, bool EX> struct ChainMulAddExpSubTanh {
    static constexpr bool kHeavy = EX;  // f64 math: many registers
    T imm;
    __device__ T operator()(const T* x) const {
        return un_op<T, EX>(sub_(un_op<T, EX>(add_(mul_(x[0], x[1]), x[2]), 0), imm), 6);
    }
};
// a*b + c: Fast.leapfrog_position / fused_chain_4 [{mul,1},{add,2}].
template <typename T> struct ChainMulAdd {
    __device__ T operator()(const T* x) const { return add_(mul_(x[0], x[1]), x[2]); }
};
// a*b*c + d: Fast.leapfrog_momentum_half [{mul,1},{mul,2},{add,3}].
template <typename T> struct ChainMulMulAdd {
    __device__ T operator()(const T* x) const {
        return add_(mul_(mul_(x[0], x[1]), x[2]), x[3]);
    }
};

bool tape_is(const Tape& t, std::initializer_list<unsigned> ops,
             std::initializer_list<unsigned> src) {
    // Compares the tape after dropping nops; src entries of unary ops are
    // given as 9 (don't care).
    unsigned k = 0;
    auto so = src.begin();
    for (unsigned want : ops) {
        while (k < t.n_ops && t.ops[k] == 255) k++;
        if (k >= t.n_ops || t.ops[k] != want) return false;
        if (want < 100 && *so != 9 && t.src[k] != *so) return false;
        k++;
        ++so;
    }
    while (k < t.n_ops && t.ops[k] == 255) k++;
    return k == t.n_ops;
}

template <typename T, bool EX>
int fused_typed(Ctx& c, T* out, const T* a, const T* b, const T* cc, const T* d, size_t n,
                const Tape& t) {
    // Hot chains first.
    if (tape_is(t, {1, 0, 100, 2, 106}, {1, 2, 9, 0, 9}) && b && cc) {
        unsigned k = 0;
        while (t.ops[k] == 255 || t.ops[k] != 2) k++;
        ChainMulAddExpSubTanh<T, EX> f{(T)t.imm[k]};
        return run_map<T, 3>(c, out, a, b, cc, nullptr, n, f);
    }
    if (tape_is(t, {1, 0}, {1, 2}) && b && cc)
        return run_map<T, 3>(c, out, a, b, cc, nullptr, n, ChainMulAdd<T>{});
    if (tape_is(t, {1, 1, 0}, {1, 2, 3}) && b && cc && d)
        return run_map<T, 4>(c, out, a, b, cc, d, n, ChainMulMulAdd<T>{});
    // Generic interpreter.  Pass the operands the tape reads; an operand the
    // tape never reads is aliased to `a` so the kernel has a valid pointer.
    bool used[4] = {true, false, false, false};
    for (unsigned k = 0; k < t.n_ops; k++)
        if (t.ops[k] < 100 && t.src[k] >= 1 && t.src[k] <= 3) used[t.src[k]] = true;
    TapeF<T, EX> f;
    f.t.n_ops = t.n_ops;
    for (int k = 0; k < 8; k++) {
        f.t.ops[k] = t.ops[k];
        f.t.src[k] = t.src[k];
        f.t.imm[k] = (T)t.imm[k];
    }
    const T* bb = used[1] ? b : a;
    const T* c2 = used[2] ? cc : a;
    const T* dd = used[3] ? d : a;
    int nin = used[3] ? 4 : (used[2] ? 3 : (used[1] ? 2 : 1));
    switch (nin) {
        case 1: return run_map<T, 1>(c, out, a, nullptr, nullptr, nullptr, n, f);
        case 2: return run_map<T, 2>(c, out, a, bb, nullptr, nullptr, n, f);
        case 3: return run_map<T, 3>(c, out, a, bb, c2, nullptr, n, f);
        default: return run_map<T, 4>(c, out, a, bb, c2, dd, n, f);
    }
}

// ---- cast -------------------------------------------------------------------

// f32 <-> f64.  Vector path (both pointers 16-byte aligned): a thread
// converts groups of 4 elements -- one float4 and two double2 -- with
// kUnroll groups in flight; the n % 4 tail is scalar.
template <typename To, typename From>
__global__ void __launch_bounds__(kThreads) k_cast(To* __restrict__ out,
                                                  const From* __restrict__ a, size_t n, int vec) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t done = 0;
    if (vec) {
        const size_t ng = n / 4;
        for (; t + (kUnroll - 1) * stride < ng; t += kUnroll * stride) {
            From x[kUnroll][4];
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                const From* src = a + (t + u * stride) * 4;
                if constexpr (sizeof(From) == 4) {
                    const float4 v = *reinterpret_cast<const float4*>(src);
                    x[u][0] = v.x, x[u][1] = v.y, x[u][2] = v.z, x[u][3] = v.w;
                } else {
                    const double2 v0 = reinterpret_cast<const double2*>(src)[0];
                    const double2 v1 = reinterpret_cast<const double2*>(src)[1];
                    x[u][0] = v0.x, x[u][1] = v0.y, x[u][2] = v1.x, x[u][3] = v1.y;
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; u++) {
                To* dst = out + (t + u * stride) * 4;
                if constexpr (sizeof(To) == 8) {
                    reinterpret_cast<double2*>(dst)[0] = make_double2((double)x[u][0], (double)x[u][1]);
                    reinterpret_cast<double2*>(dst)[1] = make_double2((double)x[u][2], (double)x[u][3]);
                } else {
                    *reinterpret_cast<float4*>(dst) = make_float4((float)x[u][0], (float)x[u][1],
                                                                  (float)x[u][2], (float)x[u][3]);
                }
            }
        }
        for (; t < ng; t += stride)
#pragma unroll
            for (int e = 0; e < 4; e++) out[t * 4 + e] = (To)a[t * 4 + e];
        done = ng * 4;
        t = done + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    }
    for (; t < n; t += stride) out[t] = (To)a[t];
}

// f32 -> f64 with every warp-wide store covering one contiguous span: a lane
// converts one float2 into one double2 (the warp reads 256 B and writes
// 512 B per vector), 8 pairs in flight per lane; the odd last element is
// scalar.  Needs out 16-byte and a 8-byte aligned.
__global__ void __launch_bounds__(kThreads) k_cast_up(double* __restrict__ out,
                                                     const float* __restrict__ a, size_t n) {
    constexpr int U = 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t np = n / 2;
    const float2* a2 = reinterpret_cast<const float2*>(a);
    double2* o2 = reinterpret_cast<double2*>(out);
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; t + (U - 1) * stride < np; t += U * stride) {
        float2 x[U];
#pragma unroll
        for (int u = 0; u < U; u++) x[u] = __ldcs(a2 + t + u * stride);
#pragma unroll
        for (int u = 0; u < U; u++) __stcs(o2 + t + u * stride, make_double2((double)x[u].x, (double)x[u].y));
    }
    for (; t < np; t += stride) {
        const float2 x = a2[t];
        o2[t] = make_double2((double)x.x, (double)x.y);
    }
    if ((n & 1) && blockIdx.x == 0 && threadIdx.x == 0) out[n - 1] = (double)a[n - 1];
}

// ---- broadcast --------------------------------------------------------------

struct Bcast {
    unsigned ndim;
    unsigned shape[4];
    unsigned as[4];
    unsigned bs[4];
};

// Flat over output vectors; each vector lies in one row of the innermost
// dim (inner % W == 0 on the vector path).  Row offsets of a and b come
// from the row's coordinates on the outer dims.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads)
k_bcast(T* __restrict__ out, const T* __restrict__ a, const T* __restrict__ b, Bcast g,
        unsigned op, size_t n) {
    constexpr int W = VEC ? (int)(16 / sizeof(T)) : 1;
    const unsigned last = g.ndim - 1;
    const size_t inner = g.shape[last];
    const size_t nv = n / W;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
        size_t e = v * W;
        size_t row = e / inner;
        size_t col = e - row * inner;
        size_t oa = col * g.as[last], ob = col * g.bs[last];
        size_t rem = row;
        for (int d = (int)last - 1; d >= 0; d--) {
            size_t cd = rem % g.shape[d];
            rem /= g.shape[d];
            oa += cd * g.as[d];
            ob += cd * g.bs[d];
        }
        T xa[W], xb[W], r[W];
        if constexpr (VEC) {
            if (g.as[last] == 1) vload(a + oa, xa);
            else {
#pragma unroll
                for (int j = 0; j < W; j++) xa[j] = a[oa];
            }
            if (g.bs[last] == 1) vload(b + ob, xb);
            else {
#pragma unroll
                for (int j = 0; j < W; j++) xb[j] = b[ob];
            }
        } else {
            xa[0] = a[oa];
            xb[0] = b[ob];
        }
#pragma unroll
        for (int j = 0; j < W; j++) r[j] = bin_op<T>(xa[j], xb[j], op);
        if constexpr (VEC) vstore(out + e, r);
        else out[e] = r[0];
    }
}

// Vector path for outputs of fewer than 2^32 elements: the flat vector
// index is decoded into coordinates with exact multiply-high division
// (Lemire, Kaser & Kurz 2019: for M = ceil(2^64 / d) and 32-bit n, d,
// floor(n / d) = umulhi64(M, n)), and each thread keeps 4 vectors in flight.
// NXV_BCAST_ROWS=0: every vector broadcast on the flat-index kernel.
bool bcast_rows_enabled() {
    const char* e = getenv("NXV_BCAST_ROWS");
    return !(e && e[0] == '0');
}

struct FastDiv {
    unsigned long long m[4];  // ceil(2^64 / shape[d]); 0 when shape[d] == 1
};

__device__ __forceinline__ unsigned fdiv(unsigned x, unsigned long long m) {
    return m ? (unsigned)__umul64hi(m, (unsigned long long)x) : x;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
k_bcast_fast(T* __restrict__ out, const T* __restrict__ a, const T* __restrict__ b, Bcast g,
             FastDiv fd, unsigned op, unsigned nv) {
    constexpr int W = (int)(16 / sizeof(T));
    constexpr int U = 4;
    const int last = (int)g.ndim - 1;
    const bool va = g.as[last] == 1, vb = g.bs[last] == 1;
    const unsigned stride = gridDim.x * blockDim.x;
    for (unsigned v0 = blockIdx.x * blockDim.x + threadIdx.x; v0 < nv; v0 += stride * U) {
        T xa[U][W], xb[U][W];
        unsigned ev[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const unsigned v = v0 + u * stride;
            ev[u] = v;
            if (v >= nv) continue;
            unsigned rem = v * W, oa = 0, ob = 0;
#pragma unroll
            for (int d = 3; d >= 0; d--) {
                if (d > last) continue;
                const unsigned q = fdiv(rem, fd.m[d]);
                const unsigned cd = rem - q * g.shape[d];
                rem = q;
                oa += cd * g.as[d];
                ob += cd * g.bs[d];
            }
            if (va) vload(a + oa, xa[u]);
            else {
#pragma unroll
                for (int j = 0; j < W; j++) xa[u][j] = a[oa];
            }
            if (vb) vload(b + ob, xb[u]);
            else {
#pragma unroll
                for (int j = 0; j < W; j++) xb[u][j] = b[ob];
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (ev[u] >= nv) continue;
            T r[W];
#pragma unroll
            for (int j = 0; j < W; j++) r[j] = bin_op<T>(xa[u][j], xb[u][j], op);
            vstore(out + (size_t)ev[u] * W, r);
        }
    }
}

// Row path (same conditions as the vector path): the innermost dimension, of
// Lv vectors, is contiguous in the output and has stride 1 or 0 in each
// operand.  A task is one chunk of kThreads * 4 vectors of one row; the row's
// operand offsets are decoded once per task, so per element only the loads,
// the op (a template constant) and the store remain.
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads)
k_bcast_rows(T* __restrict__ out, const T* __restrict__ a, const T* __restrict__ b, Bcast g,
             FastDiv fd, unsigned rows, unsigned Lv, unsigned chunks) {
    constexpr int W = (int)(16 / sizeof(T));
    constexpr int U = 4;
    const int last = (int)g.ndim - 1;
    const bool va = g.as[last] == 1, vb = g.bs[last] == 1;
    const unsigned ntask = rows * chunks;
    for (unsigned task = blockIdx.x; task < ntask; task += gridDim.x) {
        const unsigned r = task / chunks, ch = task - r * chunks;
        unsigned rem = r, oa = 0, ob = 0;
#pragma unroll
        for (int d = 2; d >= 0; d--) {
            if (d >= last) continue;
            const unsigned q = fdiv(rem, fd.m[d]);
            const unsigned cd = rem - q * g.shape[d];
            rem = q;
            oa += cd * g.as[d];
            ob += cd * g.bs[d];
        }
        const T* ar = a + oa;
        const T* br = b + ob;
        T* orow = out + (size_t)r * Lv * W;
        const unsigned v0 = ch * (kThreads * U) + threadIdx.x;
        T xa[U][W], xb[U][W];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const unsigned v = v0 + u * kThreads;
            if (v >= Lv) continue;
            if (va) vload(ar + (size_t)v * W, xa[u]);
            else {
#pragma unroll
                for (int j = 0; j < W; j++) xa[u][j] = ar[0];
            }
            if (vb) vload(br + (size_t)v * W, xb[u]);
            else {
#pragma unroll
                for (int j = 0; j < W; j++) xb[u][j] = br[0];
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const unsigned v = v0 + u * kThreads;
            if (v >= Lv) continue;
            T r2[W];
#pragma unroll
            for (int j = 0; j < W; j++) r2[j] = bin_op<T>(xa[u][j], xb[u][j], OP);
            vstore(orow + (size_t)v * W, r2);
        }
    }
}

template <typename T, int OP>
void launch_bcast_rows(Ctx& c, T* out, const T* a, const T* b, const Bcast& g, const FastDiv& fd,
                       unsigned rows, unsigned Lv) {
    const unsigned chunks = (Lv + kThreads * 4 - 1) / (kThreads * 4);
    const size_t tasks = (size_t)rows * chunks;
    const size_t cap = (size_t)c.dev->sm_count * 8;
    const unsigned grid = (unsigned)(tasks < cap ? tasks : cap);
    k_bcast_rows<T, OP><<<grid, kThreads, 0, c.stream>>>(out, a, b, g, fd, rows, Lv, chunks);
}

template <typename T>
void bcast_rows_op(Ctx& c, unsigned op, T* out, const T* a, const T* b, const Bcast& g,
                   const FastDiv& fd, unsigned rows, unsigned Lv) {
    switch (op) {
        case 0: return launch_bcast_rows<T, 0>(c, out, a, b, g, fd, rows, Lv);
        case 1: return launch_bcast_rows<T, 1>(c, out, a, b, g, fd, rows, Lv);
        case 2: return launch_bcast_rows<T, 2>(c, out, a, b, g, fd, rows, Lv);
        case 3: return launch_bcast_rows<T, 3>(c, out, a, b, g, fd, rows, Lv);
        case 4: return launch_bcast_rows<T, 4>(c, out, a, b, g, fd, rows, Lv);
        case 5: return launch_bcast_rows<T, 5>(c, out, a, b, g, fd, rows, Lv);
        case 6: return launch_bcast_rows<T, 6>(c, out, a, b, g, fd, rows, Lv);
        case 7: return launch_bcast_rows<T, 7>(c, out, a, b, g, fd, rows, Lv);
        case 8: return launch_bcast_rows<T, 8>(c, out, a, b, g, fd, rows, Lv);
        default: return launch_bcast_rows<T, 9>(c, out, a, b, g, fd, rows, Lv);
    }
}

// ---- transpose --------------------------------------------------------------

// TS x TS tile through shared memory (padded rows: conflict-free column
// reads), 32 x 8 threads, each moving (TS/32) x (TS/8) elements: coalesced
// row reads of A and row writes of the output.  TS = 64 for f32 (16 KB per
// CTA in flight), 32 for f64 (8 KB).
template <typename T, int TS>
__global__ void __launch_bounds__(256) k_transpose(T* __restrict__ out, const T* __restrict__ a,
                                                   unsigned m, unsigned n) {
    __shared__ T tile[TS][TS + 1];
    const unsigned bx = blockIdx.x * TS, by = blockIdx.y * TS;
#pragma unroll
    for (int j = 0; j < TS; j += 8) {
        const unsigned y = by + threadIdx.y + j;
#pragma unroll
        for (int i = 0; i < TS; i += 32) {
            const unsigned x = bx + threadIdx.x + i;
            if (x < n && y < m) tile[threadIdx.y + j][threadIdx.x + i] = a[(size_t)y * n + x];
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < TS; j += 8) {
        const unsigned oy = bx + threadIdx.y + j;  // out is n x m
#pragma unroll
        for (int i = 0; i < TS; i += 32) {
            const unsigned ox = by + threadIdx.x + i;
            if (ox < m && oy < n) out[(size_t)oy * m + ox] = tile[threadIdx.x + i][threadIdx.y + j];
        }
    }
}

// ---- HMC elementwise helpers (f32) ---------------------------------------------

// normal_logpdf.spv: ((z*z)*-0.5 - log sigma) - log sqrt(2 pi), z = (x-mu)/sigma
// (op order from lib/nx_vulkan/fast.ex:153-161).
// EX: log sigma in f64 rounded once (the oracle's evaluation,
// NXV_EXACT_F32=1), else logf (within 1 ulp).
template <bool EX> struct NormalLogpdfF {
    static constexpr bool kHeavy = EX;
    __device__ float operator()(const float* x) const {
        float z = div_(sub_(x[0], x[1]), x[2]);
        float z2 = mul_(z, z);
        const float ls = EX ? (float)log((double)x[2]) : logf(x[2]);
        return sub_(sub_(mul_(z2, -0.5f), ls), 0.918938533204672742f);
    }
};

__global__ void __launch_bounds__(kThreads)
k_leapfrog_step(float* __restrict__ qn, float* __restrict__ pn, const float* __restrict__ q,
                const float* __restrict__ p, const float* __restrict__ m, size_t n, float eps,
                float mu, float inv_var) {
    float he = mul_(0.5f, eps);
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float g = -mul_(sub_(q[i], mu), inv_var);
        float ph = add_(p[i], mul_(he, g));
        float qq = add_(q[i], mul_(mul_(eps, m[i]), ph));
        float gn = -mul_(sub_(qq, mu), inv_var);
        qn[i] = qq;
        pn[i] = add_(ph, mul_(he, gn));
    }
}

}  // namespace

int launch_binary(Ctx& c, int dt, void* out, const void* a, const void* b, size_t n,
                  unsigned op) {
    if (dt == F32 && fast_f32())
        return run_map<float, 2>(c, (float*)out, (const float*)a, (const float*)b, nullptr,
                                 nullptr, n, BinF<float, false>{op});
    if (dt == F32)
        return run_map<float, 2>(c, (float*)out, (const float*)a, (const float*)b, nullptr,
                                 nullptr, n, BinF<float, true>{op});
    return run_map<double, 2>(c, (double*)out, (const double*)a, (const double*)b, nullptr,
                              nullptr, n, BinF<double, true>{op});
}

int launch_unary(Ctx& c, int dt, void* out, const void* a, size_t n, unsigned op) {
    if (dt == F32 && fast_f32())
        return run_map<float, 1>(c, (float*)out, (const float*)a, nullptr, nullptr, nullptr, n,
                                 UnF<float, false>{op});
    if (dt == F32)
        return run_map<float, 1>(c, (float*)out, (const float*)a, nullptr, nullptr, nullptr, n,
                                 UnF<float, true>{op});
    return run_map<double, 1>(c, (double*)out, (const double*)a, nullptr, nullptr, nullptr, n,
                              UnF<double, true>{op});
}

int launch_cast(Ctx& c, int to_f64, void* out, const void* a, size_t n) {
    if (n == 0) return OK;
    const int vec = al16(out) && al16(a);
    unsigned g = grid_for(c, vec ? (n / 4 + kUnroll - 1) / kUnroll : n, kThreads, 8);
    if (to_f64 && al16(out) && (((uintptr_t)a) & 7) == 0) {
        const unsigned g2 = grid_for(c, (n / 2 + 7) / 8, kThreads, 8);
        k_cast_up<<<g2, kThreads, 0, c.stream>>>((double*)out, (const float*)a, n);
    } else if (to_f64)
        k_cast<double, float><<<g, kThreads, 0, c.stream>>>((double*)out, (const float*)a, n, vec);
    else
        k_cast<float, double><<<g, kThreads, 0, c.stream>>>((float*)out, (const double*)a, n, vec);
    count_launch();
    return finish(c);
}

int launch_broadcast(Ctx& c, int dt, void* out, const void* a, const void* b, unsigned op,
                     unsigned ndim, const unsigned* shape, const unsigned* as,
                     const unsigned* bs) {
    Bcast g{};
    g.ndim = ndim;
    size_t n = 1;
    for (unsigned d = 0; d < 4; d++) {
        g.shape[d] = d < ndim ? shape[d] : 1;
        g.as[d] = d < ndim ? as[d] : 0;
        g.bs[d] = d < ndim ? bs[d] : 0;
        if (d < ndim) n *= shape[d];
    }
    if (n == 0) return OK;
    const size_t esz = dt == F32 ? 4 : 8;
    const unsigned W = (unsigned)(16 / esz);
    const unsigned last = ndim - 1;
    bool vec = al16(out) && al16(a) && al16(b) && g.shape[last] % W == 0 &&
               g.as[last] <= 1 && g.bs[last] <= 1;
    for (unsigned d = 0; vec && d < last; d++)
        if ((g.as[last] == 1 && g.as[d] % W) || (g.bs[last] == 1 && g.bs[d] % W)) vec = false;
    // Fast vector path when every index fits 32 bits.
    size_t amax = 0, bmax = 0;
    for (unsigned d = 0; d < ndim; d++) {
        amax += (size_t)(g.shape[d] - 1) * g.as[d];
        bmax += (size_t)(g.shape[d] - 1) * g.bs[d];
    }
    if (vec && n < (1ull << 32) && amax + W < (1ull << 32) && bmax + W < (1ull << 32)) {
        FastDiv fd{};
        for (unsigned d = 0; d < 4; d++) {
            const unsigned long long sd = g.shape[d];
            fd.m[d] = (sd <= 1) ? 0ull : (~0ull) / sd + 1ull;  // ceil(2^64 / sd), sd >= 2
        }
        const unsigned nv = (unsigned)(n / W);
        const unsigned Lv = g.shape[last] / W;
        if (Lv >= 64 && bcast_rows_enabled()) {
            const unsigned rows = (unsigned)(n / g.shape[last]);
            if (dt == F32)
                bcast_rows_op<float>(c, op, (float*)out, (const float*)a, (const float*)b, g, fd,
                                     rows, Lv);
            else
                bcast_rows_op<double>(c, op, (double*)out, (const double*)a, (const double*)b, g, fd,
                                      rows, Lv);
            count_launch();
            return finish(c);
        }
        unsigned grid = grid_for(c, (nv + 3) / 4, kThreads, 8);
        if (dt == F32)
            k_bcast_fast<float><<<grid, kThreads, 0, c.stream>>>((float*)out, (const float*)a,
                                                                 (const float*)b, g, fd, op, nv);
        else
            k_bcast_fast<double><<<grid, kThreads, 0, c.stream>>>((double*)out, (const double*)a,
                                                                  (const double*)b, g, fd, op, nv);
        count_launch();
        return finish(c);
    }
    unsigned grid = grid_for(c, vec ? n / W : n, kThreads, 8);
    if (dt == F32) {
        if (vec) k_bcast<float, true><<<grid, kThreads, 0, c.stream>>>((float*)out, (const float*)a, (const float*)b, g, op, n);
        else k_bcast<float, false><<<grid, kThreads, 0, c.stream>>>((float*)out, (const float*)a, (const float*)b, g, op, n);
    } else {
        if (vec) k_bcast<double, true><<<grid, kThreads, 0, c.stream>>>((double*)out, (const double*)a, (const double*)b, g, op, n);
        else k_bcast<double, false><<<grid, kThreads, 0, c.stream>>>((double*)out, (const double*)a, (const double*)b, g, op, n);
    }
    count_launch();
    return finish(c);
}

int launch_fused(Ctx& c, int dt, void* out, const void* a, const void* b, const void* cc,
                 const void* d, size_t n, const Tape& t) {
    if (dt == F32 && fast_f32())
        return fused_typed<float, false>(c, (float*)out, (const float*)a, (const float*)b,
                                         (const float*)cc, (const float*)d, n, t);
    if (dt == F32)
        return fused_typed<float, true>(c, (float*)out, (const float*)a, (const float*)b,
                                        (const float*)cc, (const float*)d, n, t);
    return fused_typed<double, true>(c, (double*)out, (const double*)a, (const double*)b,
                                     (const double*)cc, (const double*)d, n, t);
}

int launch_transpose(Ctx& c, int dt, void* out, const void* a, unsigned m, unsigned n) {
    int rc = enqueue_transpose(c, dt, out, a, m, n);
    return rc ? rc : finish(c);
}

int enqueue_transpose(Ctx& c, int dt, void* out, const void* a, unsigned m, unsigned n) {
    if (m == 0 || n == 0) return OK;
    const dim3 block(32, 8);
    if (dt == F32) {
        const dim3 grid((n + 63) / 64, (m + 63) / 64);
        k_transpose<float, 64><<<grid, block, 0, c.stream>>>((float*)out, (const float*)a, m, n);
    } else {
        const dim3 grid((n + 31) / 32, (m + 31) / 32);
        k_transpose<double, 32><<<grid, block, 0, c.stream>>>((double*)out, (const double*)a, m, n);
    }
    count_launch();
    return OK;
}

int launch_normal_logpdf(Ctx& c, void* out, const void* x, const void* mu, const void* sigma,
                         size_t n) {
    if (fast_f32())
        return run_map<float, 3>(c, (float*)out, (const float*)x, (const float*)mu,
                                 (const float*)sigma, nullptr, n, NormalLogpdfF<false>{});
    return run_map<float, 3>(c, (float*)out, (const float*)x, (const float*)mu,
                             (const float*)sigma, nullptr, n, NormalLogpdfF<true>{});
}

int launch_leapfrog_step_f32(Ctx& c, void* qn, void* pn, const void* q, const void* p,
                             const void* m, size_t n, float eps, float mu, float sigma) {
    if (n == 0) return OK;
    float inv_var = 1.0f / (sigma * sigma);
    unsigned g = grid_for(c, n, kThreads, 8);
    k_leapfrog_step<<<g, kThreads, 0, c.stream>>>((float*)qn, (float*)pn, (const float*)q,
                                                   (const float*)p, (const float*)m, n, eps, mu,
                                                   inv_var);
    count_launch();
    return finish(c);
}

}  // namespace nxv
