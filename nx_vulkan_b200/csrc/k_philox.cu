// k_philox.cu -- counter-based Philox-2x32-10 (Salmon et al., SC'11).
//
// The reference runs Random123 Philox 2x32-10 (PLAN_FUSED_LEAPFROG.md:27-29)
// but its counter layout exists only inside a compiled shader, so this
// library defines and documents its own mapping (identical in the CPU
// oracle, which pins it bit for bit):
//   f32 uniform:  element i <- word (i & 1) of philox(ctr = (i >> 1, 0), key = seed),
//                 u = (w >> 8) * 2^-24 in [0, 1)
//   f32 normal:   pair c <- u1 = ((w0 >> 8) + 1) * 2^-24, u2 = (w1 >> 8) * 2^-24,
//                 r = sqrt(-2 ln u1): (r cos 2 pi u2, r sin 2 pi u2) -- in f32
//                 (logf, sqrtf, sincospif: within 4 ulp) by default, in f64 and
//                 rounded once with NXV_EXACT_F32=1
//   f64 uniform:  element i <- philox((i, 1), seed): (((w0 << 32) | w1) >> 11) * 2^-53
//   f64 normal:   pair c <- u1 = philox((2c, 1)) + 2^-53, u2 = philox((2c + 1, 1)),
//                 (r cos 2 pi u2, r sin 2 pi u2) through sincospi(2 u2)
// One thread per four f32 outputs (two counters) or per f64 output, with
// vector stores when aligned.
#include "kernels.h"

#include <math.h>

namespace nxv {

namespace {

__device__ __forceinline__ void philox2x32(uint32_t x0, uint32_t x1, uint32_t key, uint32_t& o0,
                                           uint32_t& o1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        // one 32 x 32 -> 64-bit product gives both halves (one wide multiply)
        const unsigned long long prod = (unsigned long long)x0 * 0xD256D193ull;
        const uint32_t lo = (uint32_t)prod, hi = (uint32_t)(prod >> 32);
        x0 = hi ^ key ^ x1;
        x1 = lo;
        key += 0x9E3779B9u;
    }
    o0 = x0;
    o1 = x1;
}

constexpr double kTwoPi = 6.283185307179586476925286766559;

template <bool EX>
__device__ __forceinline__ void f32_pair(uint32_t c, uint32_t seed, unsigned dist, float& v0, float& v1) {
    uint32_t w0, w1;
    philox2x32(c, 0u, seed, w0, w1);
    if (dist == 0) {
        v0 = (float)(w0 >> 8) * 0x1.0p-24f;
        v1 = (float)(w1 >> 8) * 0x1.0p-24f;
    } else if (EX) {
        double u1 = ((double)(w0 >> 8) + 1.0) * 0x1.0p-24;
        double u2 = (double)(w1 >> 8) * 0x1.0p-24;
        double r = sqrt(-2.0 * log(u1));
        double a = kTwoPi * u2;
        v0 = (float)(r * cos(a));
        v1 = (float)(r * sin(a));
    } else {
        const float u1 = (float)((w0 >> 8) + 1u) * 0x1.0p-24f;  // exact: <= 2^24
        const float u2 = (float)(w1 >> 8) * 0x1.0p-24f;
        const float r = sqrtf(-2.0f * logf(u1));
        float sn, cs;
        sincospif(2.0f * u2, &sn, &cs);  // sin, cos of 2 pi u2 (2 u2 exact)
        v0 = r * cs;
        v1 = r * sn;
    }
}

// A thread makes elements 4q .. 4q+3 (counters 2q, 2q+1) per step with one
// 16-byte store when the output is 16-byte aligned; the last n % 4 elements
// (or every element of an unaligned output) go through the pair path.
template <bool EX>
__global__ void k_random_f32(float* __restrict__ out, size_t n, uint32_t seed, unsigned dist) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t done = 0;
    if ((((uintptr_t)out) & 15) == 0) {
        const size_t quads = n / 4;
        for (size_t q = t0; q < quads; q += stride) {
            float4 v;
            f32_pair<EX>((uint32_t)(2 * q), seed, dist, v.x, v.y);
            f32_pair<EX>((uint32_t)(2 * q + 1), seed, dist, v.z, v.w);
            *reinterpret_cast<float4*>(out + 4 * q) = v;
        }
        done = quads * 4;
    }
    const size_t pairs = (n + 1) / 2;
    for (size_t c = done / 2 + t0; c < pairs; c += stride) {
        float v0, v1;
        f32_pair<EX>((uint32_t)c, seed, dist, v0, v1);
        out[2 * c] = v0;
        if (2 * c + 1 < n) out[2 * c + 1] = v1;
    }
}

__device__ __forceinline__ double u53(uint32_t i, uint32_t seed) {
    uint32_t w0, w1;
    philox2x32(i, 1u, seed, w0, w1);
    unsigned long long v = ((((unsigned long long)w0) << 32) | w1) >> 11;
    return (double)v * 0x1.0p-53;
}

__global__ void k_random_f64(double* __restrict__ out, size_t n, uint32_t seed, unsigned dist) {
    size_t stride = (size_t)gridDim.x * blockDim.x;
    if (dist == 0) {
        // two elements per thread and step, one 16-byte store when aligned
        const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        size_t done = 0;
        if ((((uintptr_t)out) & 15) == 0) {
            const size_t np = n / 2;
            for (size_t p = t0; p < np; p += stride)
                *reinterpret_cast<double2*>(out + 2 * p) =
                    make_double2(u53((uint32_t)(2 * p), seed), u53((uint32_t)(2 * p + 1), seed));
            done = np * 2;
        }
        for (size_t i = done + t0; i < n; i += stride) out[i] = u53((uint32_t)i, seed);
        return;
    }
    size_t pairs = (n + 1) / 2;
    for (size_t c = (size_t)blockIdx.x * blockDim.x + threadIdx.x; c < pairs; c += stride) {
        double u1 = u53((uint32_t)(2 * c), seed) + 0x1.0p-53;
        double u2 = u53((uint32_t)(2 * c + 1), seed);
        double r = sqrt(-2.0 * log(u1));
        double sn, cs;
        sincospi(2.0 * u2, &sn, &cs);  // sin, cos of 2 pi u2 in one call (2 u2 exact)
        out[2 * c] = r * cs;
        if (2 * c + 1 < n) out[2 * c + 1] = r * sn;
    }
}

}  // namespace

int launch_random(Ctx& c, int dt, void* out, size_t n, uint32_t seed, unsigned dist) {
    if (n == 0) return OK;
    if (n > 0x100000000ull) {
        set_error("random: at most 2^32 elements per call (32-bit counter)");
        return E_ARG;
    }
    unsigned g = grid_for(c, (n + 3) / 4, 256, 8);
    if (dt == F32) {
        if (fast_f32()) k_random_f32<false><<<g, 256, 0, c.stream>>>((float*)out, n, seed, dist);
        else k_random_f32<true><<<g, 256, 0, c.stream>>>((float*)out, n, seed, dist);
    }
    else k_random_f64<<<g, 256, 0, c.stream>>>((double*)out, n, seed, dist);
    count_launch();
    return finish(c);
}

}  // namespace nxv
