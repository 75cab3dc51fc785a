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
//                 (r cos 2 pi u2, r sin 2 pi u2) with a table-driven ln and
//                 sin/cos of pi x on an exactly reduced x (within 3 ulp of the
//                 exact transform)
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

// ---- the f64 Box-Muller transform's ln and sin/cos ------------------------
//
// ln u for u in [2^-53, 1] (table-driven after P. T. P. Tang, "Table-driven
// implementation of the logarithm function in IEEE floating-point
// arithmetic", ACM TOMS 16(4), 1990): u = 2^e m with m in [sqrt(1/2),
// sqrt(2)), F = j/64 the nearest multiple of 1/64 (j = 45 .. 91), r =
// (m - F) / F (m - F exact), ln u = e ln2 + ln F + ln(1 + r) with ln(1 + r)
// by its series to r^8 (|r| <= 0.0112: truncation below 2^-55 relative).
// ln F as a head and a tail, ln 2 as a 42-bit head (e * head exact) and a
// tail; u near 1 takes F = 1, ln F = 0 and e = 0, so nothing cancels.
// Constants computed from their definitions with 80-digit decimal
// arithmetic.  Within two units of 2^-53 of the C library's log on the
// tested draws.
struct LogRow {
    double inv_f, ln_hi, ln_lo;
};
__device__ const LogRow kLogTab[47] = {
    {0x1.6c16c16c16c17p+0, -0x1.68ac83e9c6a14p-2, -0x1.a64eadd740178p-58},  // j = 45
    {0x1.642c8590b2164p+0, -0x1.522ae0738a3d8p-2, 0x1.8f7e9b38a6979p-57},  // j = 46
    {0x1.5c9882b931057p+0, -0x1.3c25277333184p-2, 0x1.2ad27e50a8ec6p-56},  // j = 47
    {0x1.5555555555555p+0, -0x1.269621134db92p-2, -0x1.e0efadd9db02bp-56},  // j = 48
    {0x1.4e5e0a72f0539p+0, -0x1.1178e8227e47cp-2, 0x1.0e63a5f01c691p-57},  // j = 49
    {0x1.47ae147ae147bp+0, -0x1.f991c6cb3b379p-3, -0x1.f665066f980a2p-57},  // j = 50
    {0x1.4141414141414p+0, -0x1.d1037f2655e7bp-3, -0x1.60629242471a2p-57},  // j = 51
    {0x1.3b13b13b13b14p+0, -0x1.a93ed3c8ad9e3p-3, -0x1.bcafa9de97203p-57},  // j = 52
    {0x1.3521cfb2b78c1p+0, -0x1.823c16551a3c2p-3, 0x1.1232ce70be781p-57},  // j = 53
    {0x1.2f684bda12f68p+0, -0x1.5bf406b543db2p-3, 0x1.1f5b44c0df7e7p-61},  // j = 54
    {0x1.29e4129e4129ep+0, -0x1.365fcb0159016p-3, -0x1.7d411a5b944adp-58},  // j = 55
    {0x1.2492492492492p+0, -0x1.1178e8227e47cp-3, 0x1.0e63a5f01c691p-58},  // j = 56
    {0x1.1f7047dc11f70p+0, -0x1.da727638446a2p-4, -0x1.401fa71733019p-58},  // j = 57
    {0x1.1a7b9611a7b96p+0, -0x1.9335e5d594989p-4, 0x1.478a85704ccb7p-58},  // j = 58
    {0x1.15b1e5f75270dp+0, -0x1.4d3115d207eacp-4, -0x1.769f42c7842ccp-58},  // j = 59
    {0x1.1111111111111p+0, -0x1.08598b59e3a07p-4, 0x1.dd7009902bf32p-58},  // j = 60
    {0x1.0c9714fbcda3bp+0, -0x1.894aa149fb343p-5, -0x1.a8be97660a23dp-60},  // j = 61
    {0x1.0842108421084p+0, -0x1.0415d89e74444p-5, -0x1.c05cf1d753622p-59},  // j = 62
    {0x1.0410410410410p+0, -0x1.0205658935847p-6, -0x1.27c8e8416e71fp-60},  // j = 63
    {0x1.0000000000000p+0, 0x0.0p+0, 0x0.0p+0},  // j = 64
    {0x1.f81f81f81f820p-1, 0x1.fc0a8b0fc03e4p-7, -0x1.83092c59642a1p-62},  // j = 65
    {0x1.f07c1f07c1f08p-1, 0x1.f829b0e783300p-6, 0x1.33e3f04f1ef23p-60},  // j = 66
    {0x1.e9131abf0b767p-1, 0x1.77458f632dcfcp-5, 0x1.18d3ca87b9296p-59},  // j = 67
    {0x1.e1e1e1e1e1e1ep-1, 0x1.f0a30c01162a6p-5, 0x1.85f325c5bbacdp-59},  // j = 68
    {0x1.dae6076b981dbp-1, 0x1.341d7961bd1d1p-4, -0x1.b599f227becbbp-58},  // j = 69
    {0x1.d41d41d41d41dp-1, 0x1.6f0d28ae56b4cp-4, -0x1.906d99184b992p-58},  // j = 70
    {0x1.cd85689039b0bp-1, 0x1.a926d3a4ad563p-4, 0x1.942f48aa70ea9p-58},  // j = 71
    {0x1.c71c71c71c71cp-1, 0x1.e27076e2af2e6p-4, -0x1.61578001e0162p-60},  // j = 72
    {0x1.c0e070381c0e0p-1, 0x1.0d77e7cd08e59p-3, 0x1.9a5dc5e9030acp-57},  // j = 73
    {0x1.bacf914c1bad0p-1, 0x1.29552f81ff523p-3, 0x1.301771c407dbfp-57},  // j = 74
    {0x1.b4e81b4e81b4fp-1, 0x1.44d2b6ccb7d1ep-3, 0x1.9f4f6543e1f88p-57},  // j = 75
    {0x1.af286bca1af28p-1, 0x1.5ff3070a793d4p-3, -0x1.bc60efafc6f6ep-58},  // j = 76
    {0x1.a98ef606a63bep-1, 0x1.7ab890210d909p-3, 0x1.be36b2d6a0608p-59},  // j = 77
    {0x1.a41a41a41a41ap-1, 0x1.9525a9cf456b4p-3, 0x1.d904c1d4e2e26p-57},  // j = 78
    {0x1.9ec8e951033d9p-1, 0x1.af3c94e80bff3p-3, -0x1.398cff3641985p-58},  // j = 79
    {0x1.999999999999ap-1, 0x1.c8ff7c79a9a22p-3, -0x1.4f689f8434012p-57},  // j = 80
    {0x1.948b0fcd6e9e0p-1, 0x1.e27076e2af2e6p-3, -0x1.61578001e0162p-59},  // j = 81
    {0x1.8f9c18f9c18fap-1, 0x1.fb9186d5e3e2bp-3, -0x1.caaae64f21acbp-57},  // j = 82
    {0x1.8acb90f6bf3aap-1, 0x1.0a324e27390e3p-2, 0x1.7dcfde8061c03p-56},  // j = 83
    {0x1.8618618618618p-1, 0x1.1675cababa60ep-2, 0x1.ce63eab883717p-61},  // j = 84
    {0x1.8181818181818p-1, 0x1.22941fbcf7966p-2, -0x1.76f5eb09628afp-56},  // j = 85
    {0x1.7d05f417d05f4p-1, 0x1.2e8e2bae11d31p-2, -0x1.8f4cdb95ebdf9p-56},  // j = 86
    {0x1.78a4c8178a4c8p-1, 0x1.3a64c556945eap-2, -0x1.c68651945f97cp-57},  // j = 87
    {0x1.745d1745d1746p-1, 0x1.4618bc21c5ec2p-2, 0x1.f42decdeccf1dp-56},  // j = 88
    {0x1.702e05c0b8170p-1, 0x1.51aad872df82dp-2, 0x1.3927ac19f55e3p-59},  // j = 89
    {0x1.6c16c16c16c17p-1, 0x1.5d1bdbf5809cap-2, 0x1.4236383dc7fe1p-56},  // j = 90
    {0x1.6816816816817p-1, 0x1.686c81e9b14afp-2, -0x1.ddea0f7f58e3dp-57},  // j = 91
};
constexpr double kLn2Hi = 0x1.62e42fefa3800p-1, kLn2Lo = 0x1.ef35793c76730p-45;
constexpr double kSqrt2 = 1.4142135623730951;  // sqrt(2) rounded: the top of the range of m
constexpr double kShift52 = 0x1.8p52;
constexpr double kPi = 0x1.921fb54442d18p+1;

__device__ __forceinline__ double ln_unit(double u) {
    const int hi = __double2hiint(u), lo = __double2loint(u);
    int e = (hi >> 20) - 1023;
    double m = __hiloint2double((hi & 0x000fffff) | 0x3ff00000, lo);  // [1, 2)
    const bool big = m >= kSqrt2;
    m = big ? __dmul_rn(0.5, m) : m;
    e += big ? 1 : 0;
    const double t = __fma_rn(m, 64.0, kShift52);
    const int j = __double2loint(t);
    const double f = __fma_rn(__dsub_rn(t, kShift52), -0.015625, m);  // m - j/64, exact
    const LogRow row = kLogTab[j - 45];
    const double r = __dmul_rn(f, row.inv_f);
    // ln(1 + r) = r + r^2 (-1/2 + r (1/3 + r (-1/4 + r (1/5 + r (-1/6 + r (1/7 - r/8))))))
    double q = __fma_rn(r, -0.125, 1.0 / 7.0);
    q = __fma_rn(r, q, -1.0 / 6.0);
    q = __fma_rn(r, q, 0.2);
    q = __fma_rn(r, q, -0.25);
    q = __fma_rn(r, q, 1.0 / 3.0);
    q = __fma_rn(r, q, -0.5);
    const double p = __fma_rn(__dmul_rn(r, r), q, r);
    const double ed = (double)e;
    const double head = __fma_rn(ed, kLn2Hi, row.ln_hi);  // e * kLn2Hi is exact
    return __dadd_rn(head, __dadd_rn(p, __fma_rn(ed, kLn2Lo, row.ln_lo)));
}

// sin(pi x) and cos(pi x) for x in [0, 2): x = k/2 + r with |r| <= 1/4
// (exact), t = pi r, sin t and cos t by their Taylor series to t^17 and t^18
// (truncation below 2^-62 for |t| <= pi/4), then the quadrant k mod 4.
__device__ __forceinline__ void sincospi_unit2(double x, double& sn, double& cs) {
    const double tk = __fma_rn(x, 2.0, kShift52);
    const int k = __double2loint(tk);
    const double r = __fma_rn(__dsub_rn(tk, kShift52), -0.5, x);
    const double t = __dmul_rn(r, kPi), z = __dmul_rn(t, t);
    double ps = __fma_rn(z, 1.0 / 355687428096000.0, -1.0 / 1307674368000.0);
    ps = __fma_rn(z, ps, 1.0 / 6227020800.0);
    ps = __fma_rn(z, ps, -1.0 / 39916800.0);
    ps = __fma_rn(z, ps, 1.0 / 362880.0);
    ps = __fma_rn(z, ps, -1.0 / 5040.0);
    ps = __fma_rn(z, ps, 1.0 / 120.0);
    ps = __fma_rn(z, ps, -1.0 / 6.0);
    const double s = __fma_rn(__dmul_rn(t, z), ps, t);
    double pc = __fma_rn(z, -1.0 / 6402373705728000.0, 1.0 / 20922789888000.0);
    pc = __fma_rn(z, pc, -1.0 / 87178291200.0);
    pc = __fma_rn(z, pc, 1.0 / 479001600.0);
    pc = __fma_rn(z, pc, -1.0 / 3628800.0);
    pc = __fma_rn(z, pc, 1.0 / 40320.0);
    pc = __fma_rn(z, pc, -1.0 / 720.0);
    pc = __fma_rn(z, pc, 1.0 / 24.0);
    pc = __fma_rn(z, pc, -0.5);
    const double c = __fma_rn(z, pc, 1.0);
    switch (k & 3) {
        case 0: sn = s; cs = c; break;
        case 1: sn = c; cs = -s; break;
        case 2: sn = -s; cs = -c; break;
        default: sn = -c; cs = s; break;
    }
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
        double r = __dsqrt_rn(-2.0 * ln_unit(u1));
        double sn, cs;
        sincospi_unit2(2.0 * u2, sn, cs);  // sin, cos of 2 pi u2 (2 u2 exact)
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
