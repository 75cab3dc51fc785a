// shim.cu -- the extern "C" nxv_* entry points (include/nx_vulkan_shim.h).
//
// Each entry point validates its arguments the way the reference's NIF and
// shim did (native/nx_vulkan_native/src/lib.rs: equal byte sizes, op ranges,
// K > 0, matmul extents; c_src/nx_vulkan_shim.cpp: null checks), maps the
// spv basename to a kernel family, checks buffer sizes against the element
// counts it is asked to touch (the reference trusted the caller here), and
// launches on the current device's stream.
#include <string.h>

#include "../../include/nx_vulkan_shim.h"
#include "kernels.h"

using namespace nxv;

namespace {

// Buffer must hold at least `need` bytes.
bool fits(const void* h, size_t need) { return nxv::nbytes(h) >= need; }

int need(const void* h, size_t bytes, const char* what) {
    if (!fits(h, bytes)) {
        set_error("%s: buffer of %zu bytes, op needs %zu", what, nbytes(h), bytes);
        return E_ARG;
    }
    return OK;
}

// A batched chain's inverse mass is one [n] f64 row shared by every chain
// when its buffer holds exactly n elements and there are several chains
// (Nx broadcasting of an [n] tensor over [chain][n]); otherwise it must be
// [chain][n].
bool shared_row(const void* m, size_t n, size_t chains) {
    return chains > 1 && nbytes(m) == n * 8;
}

#define NEED(h, bytes, what)                       \
    do {                                           \
        int rc_ = need((h), (bytes), (what));      \
        if (rc_) return rc_;                       \
    } while (0)

#define BEGIN(...)                                 \
    Ctx c;                                         \
    do {                                           \
        int rc_ = begin(c, {__VA_ARGS__});         \
        if (rc_) return rc_;                       \
    } while (0)

int bad_kernel(const std::string& b) {
    set_error("no kernel for spv basename '%s'", b.c_str());
    return E_KERNEL;
}

}  // namespace

extern "C" {

int nxv_init(void) { return init_default(); }

void nxv_destroy(void) { destroy_all(); }

const char* nxv_device_name(void) {
    if (!is_initialised()) return nullptr;
    Ctx c;
    if (begin(c, {}) != OK) return nullptr;
    return c.dev->name.c_str();
}

int nxv_has_f64(void) { return is_initialised() ? 1 : 0; }

void* nxv_buf_alloc(unsigned long n_bytes) { return buf_alloc((size_t)n_bytes); }
void nxv_buf_free(void* handle) { buf_free(handle); }
void nxv_pool_clear(void) {
    if (is_initialised()) pool_clear();
}
void nxv_pool_stats(unsigned long* hits, unsigned long* misses, unsigned long* freed,
                    unsigned long* size_classes, unsigned long* total_pooled) {
    pool_stats(hits, misses, freed, size_classes, total_pooled);
}

int nxv_buf_upload(void* handle, const void* data, unsigned long n_bytes) {
    if (!handle || (!data && n_bytes)) return E_NULL;
    return buf_upload(handle, data, (size_t)n_bytes);
}

int nxv_buf_download(void* handle, void* data, unsigned long n_bytes) {
    if (!handle || (!data && n_bytes)) return E_NULL;
    return buf_download(handle, data, (size_t)n_bytes);
}

int nxv_buf_copy_2d(void* dst, unsigned long dst_offset, unsigned long dst_pitch, void* src,
                    unsigned long src_offset, unsigned long src_pitch, unsigned long width,
                    unsigned long rows) {
    if (!dst || !src) return E_NULL;
    if (rows == 0 || width == 0) return OK;
    if (width > dst_pitch || width > src_pitch) {
        set_error("copy_2d: row width %lu exceeds a pitch (%lu, %lu)", width, dst_pitch,
                  src_pitch);
        return E_ARG;
    }
    BEGIN(dst, src);
    NEED(dst, (size_t)dst_offset + (size_t)(rows - 1) * dst_pitch + width, "copy_2d dst");
    NEED(src, (size_t)src_offset + (size_t)(rows - 1) * src_pitch + width, "copy_2d src");
    cudaError_t e = cudaMemcpy2DAsync(static_cast<char*>(dptr(dst)) + dst_offset, dst_pitch,
                                      static_cast<const char*>(dptr(src)) + src_offset,
                                      src_pitch, width, rows, cudaMemcpyDeviceToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync");
    return finish(c);
}

// ---- elementwise ------------------------------------------------------------

int nxv_apply_binary(void* out, void* a, void* b, unsigned int n, unsigned int op,
                     const char* spv_path) {
    if (!out || !a || !b || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    int dt;
    if (k == "elementwise_binary.spv") dt = F32;
    else if (k == "elementwise_binary_f64.spv") dt = F64;
    else return bad_kernel(k);
    if (op > 9) {
        set_error("binary op %u out of range 0..9", op);
        return E_ARG;
    }
    BEGIN(out, a, b);
    size_t es = dt == F32 ? 4 : 8, bytes = (size_t)n * es;
    NEED(a, bytes, "apply_binary a");
    NEED(b, bytes, "apply_binary b");
    NEED(out, bytes, "apply_binary out");
    return launch_binary(c, dt, dptr(out), dptr(a), dptr(b), n, op);
}

int nxv_apply_unary(void* out, void* a, unsigned int n, unsigned int op, const char* spv_path) {
    if (!out || !a || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    int dt;
    if (k == "elementwise_unary.spv") dt = F32;
    else if (k == "elementwise_unary_f64.spv") dt = F64;
    else return bad_kernel(k);
    if (op > 14) {
        set_error("unary op %u out of range 0..14", op);
        return E_ARG;
    }
    BEGIN(out, a);
    size_t bytes = (size_t)n * (dt == F32 ? 4 : 8);
    NEED(a, bytes, "apply_unary a");
    NEED(out, bytes, "apply_unary out");
    return launch_unary(c, dt, dptr(out), dptr(a), n, op);
}

int nxv_cast(void* out, void* a, unsigned int n, const char* spv_path) {
    if (!out || !a || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    int to64;
    if (k == "cast_f32_to_f64.spv") to64 = 1;
    else if (k == "cast_f64_to_f32.spv") to64 = 0;
    else return bad_kernel(k);
    BEGIN(out, a);
    NEED(a, (size_t)n * (to64 ? 4 : 8), "cast in");
    NEED(out, (size_t)n * (to64 ? 8 : 4), "cast out");
    return launch_cast(c, to64, dptr(out), dptr(a), n);
}

int nxv_apply_binary_broadcast(void* out, void* a, void* b, unsigned int op, unsigned int ndim,
                               const unsigned int* out_shape, const unsigned int* a_strides,
                               const unsigned int* b_strides, const char* spv_path) {
    if (!out || !a || !b || !out_shape || !a_strides || !b_strides || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    int dt;
    if (k == "elementwise_binary_broadcast.spv") dt = F32;
    else if (k == "elementwise_binary_broadcast_f64.spv") dt = F64;
    else return bad_kernel(k);
    if (op > 9 || ndim == 0 || ndim > 4) {
        set_error("broadcast: op %u / ndim %u out of range", op, ndim);
        return E_ARG;
    }
    BEGIN(out, a, b);
    size_t es = dt == F32 ? 4 : 8, n = 1, amax = 0, bmax = 0;
    for (unsigned d = 0; d < ndim; d++) {
        n *= out_shape[d];
        if (out_shape[d]) {
            amax += (size_t)(out_shape[d] - 1) * a_strides[d];
            bmax += (size_t)(out_shape[d] - 1) * b_strides[d];
        }
    }
    if (n == 0) return OK;
    NEED(out, n * es, "broadcast out");
    NEED(a, (amax + 1) * es, "broadcast a");
    NEED(b, (bmax + 1) * es, "broadcast b");
    return launch_broadcast(c, dt, dptr(out), dptr(a), dptr(b), op, ndim, out_shape, a_strides,
                            b_strides);
}

int nxv_transpose(void* out, void* a, unsigned int m, unsigned int n, const char* spv_path) {
    if (!out || !a || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    int dt;
    if (k == "transpose.spv") dt = F32;
    else if (k == "transpose_f64.spv") dt = F64;
    else return bad_kernel(k);
    BEGIN(out, a);
    size_t bytes = (size_t)m * n * (dt == F32 ? 4 : 8);
    NEED(a, bytes, "transpose in");
    NEED(out, bytes, "transpose out");
    return launch_transpose(c, dt, dptr(out), dptr(a), m, n);
}

// ---- fused op tape ------------------------------------------------------------

static int fused_common(void* out, void* a, void* b, void* cc, void* d, unsigned n,
                        unsigned n_ops, const unsigned* ops, const unsigned* src, const double* imm,
                        int dt, unsigned max_bin_op) {
    if (n_ops == 0 || n_ops > 8) {
        set_error("fused chain needs 1..8 ops, got %u", n_ops);
        return E_ARG;
    }
    Tape t{};
    t.n_ops = n_ops;
    for (unsigned k = 0; k < 8; k++) {
        t.ops[k] = k < n_ops ? ops[k] : 255;
        t.src[k] = (k < n_ops && src) ? src[k] : 1;
        t.imm[k] = (k < n_ops && imm) ? imm[k] : 0.0;
    }
    void* srcs[4] = {a, b, cc, d};
    for (unsigned k = 0; k < n_ops; k++) {
        unsigned op = t.ops[k];
        bool binary = op <= max_bin_op, unary = op >= 100 && op <= 114;
        if (!(binary || unary || op == 255)) {
            set_error("fused op %u at step %u is not a valid op code", op, k);
            return E_ARG;
        }
        if (binary) {
            if (t.src[k] > 3) {
                set_error("fused step %u: operand index %u out of range", k, t.src[k]);
                return E_ARG;
            }
            if (t.src[k] == 0 && !imm) return E_NULL;
            if (t.src[k] >= 1 && !srcs[t.src[k]]) return E_NULL;
        }
    }
    BEGIN(out, a, b, cc, d);
    size_t bytes = (size_t)n * (dt == F32 ? 4 : 8);
    NEED(a, bytes, "fused a");
    NEED(out, bytes, "fused out");
    for (unsigned k = 0; k < n_ops; k++)
        if (t.ops[k] <= max_bin_op && t.src[k] >= 1) NEED(srcs[t.src[k]], bytes, "fused operand");
    return launch_fused(c, dt, dptr(out), dptr(a), dptr(b), dptr(cc), dptr(d), n, t);
}

int nxv_fused_chain(void* out, void* a, void* b, unsigned int n, unsigned int n_ops,
                    const unsigned int* ops, const char* spv_path) {
    if (!out || !a || !b || !ops || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "fused_elementwise.spv") return bad_kernel(k);
    return fused_common(out, a, b, nullptr, nullptr, n, n_ops, ops, nullptr, nullptr, F32, 6);
}

int nxv_fused_chain_4(void* out, void* a, void* b, void* c, void* d, unsigned int n,
                      unsigned int n_ops, const unsigned int* ops, const unsigned int* buf_idx,
                      const char* spv_path) {
    if (!out || !a || !b || !c || !d || !ops || !buf_idx || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "fused_elementwise_4in.spv") return bad_kernel(k);
    unsigned src[8];
    for (unsigned i = 0; i < 8; i++) {
        unsigned s = i < n_ops ? buf_idx[i] : 1;
        // buf_idx is 1..3 in the reference; 0 is not an immediate there.
        src[i] = (s >= 1 && s <= 3) ? s : 99;
    }
    for (unsigned i = 0; i < n_ops && i < 8; i++)
        if (ops[i] <= 6 && src[i] == 99) {
            set_error("fused_chain_4: buf_idx[%u] = %u is not 1..3", i, buf_idx[i]);
            return E_ARG;
        }
    return fused_common(out, a, b, c, d, n, n_ops, ops, src, nullptr, F32, 6);
}

int nxv_fused_chain_imm(void* out, void* a, void* b, void* c, void* d, unsigned int n,
                        unsigned int n_ops, const unsigned int* ops, const unsigned int* src,
                        const double* imm, unsigned int dtype, const char* spv_path) {
    if (!out || !a || !ops || !src || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "fused_elementwise_imm.spv") return bad_kernel(k);
    if (dtype > 1) {
        set_error("dtype %u is not 0 (f32) or 1 (f64)", dtype);
        return E_ARG;
    }
    return fused_common(out, a, b, c, d, n, n_ops, ops, src, imm, (int)dtype, 9);
}

// ---- reductions ------------------------------------------------------------------

int nxv_reduce(float* out_scalar, void* in, unsigned int n, unsigned int op, const char* spv_path) {
    if (!out_scalar || !in || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "reduce.spv") return bad_kernel(k);
    if (op > 2) {
        set_error("reduce op %u out of range 0..2", op);
        return E_ARG;
    }
    BEGIN(in);
    NEED(in, (size_t)n * 4, "reduce in");
    float* dv = (float*)scratch(c, 0);  // re-fetched below after the launch
    (void)dv;
    void* res = buf_alloc(4);
    if (!res) return E_CUDA;
    int rc = launch_reduce_full(c, F32, dptr(res), dptr(in), n, op);
    if (rc == OK) rc = buf_download(res, out_scalar, 4);
    buf_free(res);
    return rc;
}

int nxv_reduce_f64(double* out_scalar, void* in, unsigned long n, unsigned int op,
                   const char* spv_path) {
    if (!out_scalar || !in || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "reduce_full_f64.spv") return bad_kernel(k);
    if (op > 2) {
        set_error("reduce op %u out of range 0..2", op);
        return E_ARG;
    }
    BEGIN(in);
    NEED(in, (size_t)n * 8, "reduce_f64 in");
    void* res = buf_alloc(8);
    if (!res) return E_CUDA;
    int rc = launch_reduce_full(c, F64, dptr(res), dptr(in), n, op);
    if (rc == OK) rc = buf_download(res, out_scalar, 8);
    buf_free(res);
    return rc;
}

int nxv_reduce_to_buf(void* out, void* in, unsigned long n, unsigned int op, unsigned int dtype,
                      const char* spv_path) {
    if (!out || !in || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "reduce.spv" && k != "reduce_full_f64.spv") return bad_kernel(k);
    if (op > 2 || dtype > 1) {
        set_error("reduce_to_buf: op %u / dtype %u out of range", op, dtype);
        return E_ARG;
    }
    BEGIN(out, in);
    size_t es = dtype == 0 ? 4 : 8;
    NEED(in, (size_t)n * es, "reduce_to_buf in");
    NEED(out, es, "reduce_to_buf out");
    return launch_reduce_full(c, (int)dtype, dptr(out), dptr(in), n, op);
}

int nxv_reduce_axis(void* out, void* a, unsigned int outer, unsigned int reduce_size,
                    unsigned int inner, unsigned int op, const char* spv_path) {
    if (!out || !a || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    bool lse = k == "logsumexp.spv";
    int dt;
    if (k == "reduce_axis.spv" || lse) dt = F32;
    else if (k == "reduce_axis_f64.spv") dt = F64;
    else return bad_kernel(k);
    if (!lse && op > 2) {
        set_error("reduce_axis op %u out of range 0..2", op);
        return E_ARG;
    }
    BEGIN(out, a);
    size_t es = dt == F32 ? 4 : 8;
    size_t nin = (size_t)outer * reduce_size * inner, nout = (size_t)outer * inner;
    NEED(a, nin * es, "reduce_axis in");
    NEED(out, nout * es, "reduce_axis out");
    if (nout == 0) return OK;
    if (lse) return launch_logsumexp(c, dptr(out), dptr(a), outer, reduce_size, inner);
    return launch_reduce_axis(c, dt, dptr(out), dptr(a), outer, reduce_size, inner, op);
}

int nxv_argmax_axis(void* out, void* a, unsigned int outer, unsigned int reduce_size,
                    unsigned int inner, unsigned int is_min, unsigned int dtype,
                    unsigned int index_bytes, const char* spv_path) {
    if (!out || !a || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "argmax_axis.spv") return bad_kernel(k);
    if (dtype > 1 || is_min > 1 || (index_bytes != 4 && index_bytes != 8)) {
        set_error("argmax: dtype %u / is_min %u / index_bytes %u out of range", dtype, is_min,
                  index_bytes);
        return E_ARG;
    }
    BEGIN(out, a);
    size_t es = dtype == 0 ? 4 : 8;
    size_t nin = (size_t)outer * reduce_size * inner, nout = (size_t)outer * inner;
    NEED(a, nin * es, "argmax in");
    NEED(out, nout * index_bytes, "argmax out");
    if (nout == 0) return OK;
    return launch_argmax(c, (int)dtype, dptr(out), dptr(a), outer, reduce_size, inner,
                         (int)is_min, (int)index_bytes);
}

// ---- matmul -------------------------------------------------------------------------

static int matmul_common(void* out, void* a, void* b, size_t batch, size_t m, size_t n, size_t k,
                         int dt) {
    BEGIN(out, a, b);
    size_t es = dt == F32 ? 4 : 8;
    NEED(a, batch * m * k * es, "matmul a");
    NEED(b, batch * k * n * es, "matmul b");
    NEED(out, batch * m * n * es, "matmul out");
    if (dt == F32) return launch_matmul_f32(c, dptr(out), dptr(a), dptr(b), batch, m, n, k);
    return launch_matmul_f64(c, dptr(out), dptr(a), dptr(b), batch, m, n, k);
}

static bool is_matmul_spv(const std::string& k) {
    return k == "matmul.spv" || k == "matmul_tiled.spv" || k == "matmul_tiled32.spv" ||
           k == "matmul_tiled16x2.spv";
}

int nxv_matmul(void* out, void* a, void* b, unsigned int m, unsigned int n, unsigned int k,
               const char* spv_path) {
    if (!out || !a || !b || !spv_path) return E_NULL;
    std::string s = spv_base(spv_path);
    if (!is_matmul_spv(s)) return bad_kernel(s);
    return matmul_common(out, a, b, 1, m, n, k, F32);
}

int nxv_matmul_v(void* out, void* a, void* b, unsigned int m, unsigned int n, unsigned int k,
                 unsigned int tile_m, unsigned int tile_n, const char* spv_path) {
    (void)tile_m;
    (void)tile_n;
    return nxv_matmul(out, a, b, m, n, k, spv_path);
}

int nxv_matmul_batched(void* out, void* a, void* b, unsigned int batch, unsigned int m,
                       unsigned int n, unsigned int k, unsigned int dtype, const char* spv_path) {
    if (!out || !a || !b || !spv_path) return E_NULL;
    std::string s = spv_base(spv_path);
    if (s != "matmul_batched.spv") return bad_kernel(s);
    if (dtype > 1) {
        set_error("dtype %u is not 0 (f32) or 1 (f64)", dtype);
        return E_ARG;
    }
    return matmul_common(out, a, b, batch, m, n, k, (int)dtype);
}

// ---- random -------------------------------------------------------------------------

int nxv_random(void* out, unsigned int n, unsigned int seed, unsigned int dist,
               const char* spv_path) {
    if (!out || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "random_philox.spv") return bad_kernel(k);
    if (dist > 1) {
        set_error("random dist %u out of range 0..1", dist);
        return E_ARG;
    }
    BEGIN(out);
    NEED(out, (size_t)n * 4, "random out");
    return launch_random(c, F32, dptr(out), n, seed, dist);
}

int nxv_random_f64(void* out, unsigned long n, unsigned int seed, unsigned int dist,
                   const char* spv_path) {
    if (!out || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "random_philox_f64.spv") return bad_kernel(k);
    if (dist > 1) {
        set_error("random dist %u out of range 0..1", dist);
        return E_ARG;
    }
    BEGIN(out);
    NEED(out, (size_t)n * 8, "random_f64 out");
    return launch_random(c, F64, dptr(out), n, seed, dist);
}

// ---- HMC primitives ---------------------------------------------------------------------

int nxv_kinetic_energy(void* out, void* p, void* inv_mass, unsigned int n, const char* spv_path) {
    if (!out || !p || !inv_mass || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "kinetic_energy.spv") return bad_kernel(k);
    BEGIN(out, p, inv_mass);
    NEED(p, (size_t)n * 4, "kinetic_energy p");
    NEED(inv_mass, (size_t)n * 4, "kinetic_energy inv_mass");
    NEED(out, (size_t)((n + 255) / 256) * 4, "kinetic_energy out");
    return launch_kinetic_energy(c, dptr(out), dptr(p), dptr(inv_mass), n);
}

int nxv_normal_logpdf(void* out, void* x, void* mu, void* sigma, unsigned int n,
                      const char* spv_path) {
    if (!out || !x || !mu || !sigma || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "normal_logpdf.spv") return bad_kernel(k);
    BEGIN(out, x, mu, sigma);
    size_t bytes = (size_t)n * 4;
    NEED(x, bytes, "normal_logpdf x");
    NEED(mu, bytes, "normal_logpdf mu");
    NEED(sigma, bytes, "normal_logpdf sigma");
    NEED(out, bytes, "normal_logpdf out");
    return launch_normal_logpdf(c, dptr(out), dptr(x), dptr(mu), dptr(sigma), n);
}

int nxv_leapfrog_normal(void* q_new, void* p_new, void* q, void* p, void* inv_mass,
                        unsigned int n, float eps, float mu, float sigma, const char* spv_path) {
    if (!q_new || !p_new || !q || !p || !inv_mass || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "leapfrog_normal.spv") return bad_kernel(k);
    BEGIN(q_new, p_new, q, p, inv_mass);
    size_t bytes = (size_t)n * 4;
    NEED(q, bytes, "leapfrog q");
    NEED(p, bytes, "leapfrog p");
    NEED(inv_mass, bytes, "leapfrog inv_mass");
    NEED(q_new, bytes, "leapfrog q_new");
    NEED(p_new, bytes, "leapfrog p_new");
    return launch_leapfrog_step_f32(c, dptr(q_new), dptr(p_new), dptr(q), dptr(p), dptr(inv_mass),
                                    n, eps, mu, sigma);
}

// ---- leapfrog chains -------------------------------------------------------------------------

static int chain_f32(void* qc, void* pc, void* gc, void* lc, void* q0, void* p0, void* m,
                     unsigned n, unsigned K, float eps, int fam, const float* prm,
                     const char* spv_path, const char* want, int mode, unsigned nwg) {
    if (!qc || !pc || !gc || !lc || !q0 || !p0 || !m || !spv_path) return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != want) return bad_kernel(k);
    if (K == 0) {
        set_error("K must be positive");
        return E_ARG;
    }
    BEGIN(qc, pc, gc, lc, q0, p0, m);
    size_t vec = (size_t)n * 4, chain = vec * K;
    NEED(q0, vec, "chain q_init");
    NEED(p0, vec, "chain p_init");
    NEED(m, vec, "chain inv_mass");
    NEED(qc, chain, "q_chain");
    NEED(pc, chain, "p_chain");
    NEED(gc, chain, "grad_chain");
    if (mode == 1) {
        unsigned want_wg = (n + 255) / 256;
        if (nwg != want_wg) {
            set_error("num_workgroups %u != ceil(n/256) = %u", nwg, want_wg);
            return E_ARG;
        }
        NEED(lc, (size_t)K * nwg * 4, "partial_logp");
    } else {
        NEED(lc, (size_t)K * 4, "logp_chain");
    }
    return launch_chain_f32(c, fam, prm, dptr(qc), dptr(pc), dptr(gc), dptr(lc), dptr(q0),
                            dptr(p0), dptr(m), n, 1, K, eps, mode);
}

int nxv_leapfrog_chain_normal(void* q_chain, void* p_chain, void* grad_chain, void* logp_chain,
                              void* q_init, void* p_init, void* inv_mass, unsigned int n,
                              unsigned int K, float eps, float mu, float sigma,
                              const char* spv_path) {
    float prm[2] = {mu, sigma};
    return chain_f32(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, n, K, eps,
                     FAM_NORMAL, prm, spv_path, "leapfrog_chain_normal.spv", 0, 0);
}

int nxv_leapfrog_chain_normal_lg(void* q_chain, void* p_chain, void* grad_chain,
                                 void* partial_logp, void* q_init, void* p_init, void* inv_mass,
                                 unsigned int n, unsigned int K, unsigned int num_workgroups,
                                 float eps, float mu, float sigma, const char* spv_path) {
    float prm[2] = {mu, sigma};
    return chain_f32(q_chain, p_chain, grad_chain, partial_logp, q_init, p_init, inv_mass, n, K,
                     eps, FAM_NORMAL, prm, spv_path, "leapfrog_chain_normal_lg.spv", 1,
                     num_workgroups);
}

int nxv_leapfrog_chain_exponential(void* q_chain, void* p_chain, void* grad_chain,
                                   void* logp_chain, void* q_init, void* p_init, void* inv_mass,
                                   unsigned int n, unsigned int K, float eps, float lambda,
                                   const char* spv_path) {
    float prm[1] = {lambda};
    return chain_f32(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, n, K, eps,
                     FAM_EXP, prm, spv_path, "leapfrog_chain_exponential.spv", 0, 0);
}

int nxv_leapfrog_chain_studentt(void* q_chain, void* p_chain, void* grad_chain, void* logp_chain,
                                void* q_init, void* p_init, void* inv_mass, unsigned int n,
                                unsigned int K, float eps, float mu, float sigma, float nu,
                                float logp_const, const char* spv_path) {
    float prm[4] = {mu, sigma, nu, logp_const};
    return chain_f32(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, n, K, eps,
                     FAM_STUDENTT, prm, spv_path, "leapfrog_chain_studentt.spv", 0, 0);
}

int nxv_leapfrog_chain_cauchy(void* q_chain, void* p_chain, void* grad_chain, void* logp_chain,
                              void* q_init, void* p_init, void* inv_mass, unsigned int n,
                              unsigned int K, float eps, float loc, float scale,
                              float log_pi_scale, const char* spv_path) {
    float prm[3] = {loc, scale, log_pi_scale};
    return chain_f32(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, n, K, eps,
                     FAM_CAUCHY, prm, spv_path, "leapfrog_chain_cauchy.spv", 0, 0);
}

int nxv_leapfrog_chain_halfnormal(void* q_chain, void* p_chain, void* grad_chain,
                                  void* logp_chain, void* q_init, void* p_init, void* inv_mass,
                                  unsigned int n, unsigned int K, float eps, float sigma,
                                  float log_const, const char* spv_path) {
    float prm[2] = {sigma, log_const};
    return chain_f32(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, n, K, eps,
                     FAM_HALFNORMAL, prm, spv_path, "leapfrog_chain_halfnormal.spv", 0, 0);
}

int nxv_leapfrog_chain_weibull(void* q_chain, void* p_chain, void* grad_chain, void* logp_chain,
                               void* q_init, void* p_init, void* inv_mass, unsigned int n,
                               unsigned int K, float eps, float k, float lambda, float logp_const,
                               const char* spv_path) {
    float prm[3] = {k, lambda, logp_const};
    return chain_f32(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, n, K, eps,
                     FAM_WEIBULL, prm, spv_path, "leapfrog_chain_weibull.spv", 0, 0);
}

int nxv_leapfrog_chain_normal_f64(void* q_chain, void* p_chain, void* grad_chain,
                                  void* logp_chain, void* q_init, void* p_init, void* inv_mass,
                                  unsigned int n, unsigned int K, double eps, double mu,
                                  double sigma, const char* spv_path) {
    if (!q_chain || !p_chain || !grad_chain || !logp_chain || !q_init || !p_init || !inv_mass ||
        !spv_path)
        return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "leapfrog_chain_normal_f64.spv") return bad_kernel(k);
    if (K == 0) {
        set_error("K must be positive");
        return E_ARG;
    }
    BEGIN(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass);
    size_t vec = (size_t)n * 8, chain = vec * K;
    NEED(q_init, vec, "q_init");
    NEED(p_init, vec, "p_init");
    NEED(inv_mass, vec, "inv_mass");
    NEED(q_chain, chain, "q_chain");
    NEED(p_chain, chain, "p_chain");
    NEED(grad_chain, chain, "grad_chain");
    NEED(logp_chain, (size_t)K * 8, "logp_chain");
    double prec = 1.0 / (sigma * sigma);
    return launch_chain_gauss_f64(c, dptr(q_chain), dptr(p_chain), dptr(grad_chain),
                                  dptr(logp_chain), dptr(q_init), dptr(p_init), dptr(inv_mass),
                                  nullptr, prec, mu, n, 1, K, eps);
}

int nxv_leapfrog_chain_gauss_f64_batched(void* q_chain, void* p_chain, void* grad_chain,
                                         void* logp_chain, void* q_init, void* p_init,
                                         void* inv_mass, void* prec, unsigned int n,
                                         unsigned int n_chains, unsigned int K, double eps,
                                         double mu, const char* spv_path) {
    if (!q_chain || !p_chain || !grad_chain || !logp_chain || !q_init || !p_init || !inv_mass ||
        !prec || !spv_path)
        return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "leapfrog_chain_gauss_f64_batched.spv") return bad_kernel(k);
    if (K == 0) {
        set_error("K must be positive");
        return E_ARG;
    }
    BEGIN(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, inv_mass, prec);
    size_t vec = (size_t)n * 8 * n_chains, chain = vec * K;
    NEED(q_init, vec, "q_init");
    NEED(p_init, vec, "p_init");
    const bool m_shared = shared_row(inv_mass, n, n_chains);
    if (!m_shared) NEED(inv_mass, vec, "inv_mass");
    NEED(prec, (size_t)n * 8, "prec");
    NEED(q_chain, chain, "q_chain");
    NEED(p_chain, chain, "p_chain");
    NEED(grad_chain, chain, "grad_chain");
    NEED(logp_chain, (size_t)K * n_chains * 8, "logp_chain");
    return launch_chain_gauss_f64(c, dptr(q_chain), dptr(p_chain), dptr(grad_chain),
                                  dptr(logp_chain), dptr(q_init), dptr(p_init), dptr(inv_mass),
                                  dptr(prec), 0.0, mu, n, n_chains, K, eps, nullptr, m_shared);
}

int nxv_leapfrog_chain_gauss_f64_batched_ke(void* q_chain, void* p_chain, void* grad_chain,
                                            void* logp_chain, void* ke_chain, void* q_init,
                                            void* p_init, void* inv_mass, void* prec,
                                            unsigned int n, unsigned int n_chains, unsigned int K,
                                            double eps, double mu, const char* spv_path) {
    if (!q_chain || !p_chain || !grad_chain || !logp_chain || !ke_chain || !q_init || !p_init ||
        !inv_mass || !prec || !spv_path)
        return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "leapfrog_chain_gauss_f64_batched.spv") return bad_kernel(k);
    if (K == 0) {
        set_error("K must be positive");
        return E_ARG;
    }
    BEGIN(q_chain, p_chain, grad_chain, logp_chain, ke_chain, q_init, p_init, inv_mass, prec);
    size_t vec = (size_t)n * 8 * n_chains, chain = vec * K;
    NEED(q_init, vec, "q_init");
    NEED(p_init, vec, "p_init");
    const bool m_shared = shared_row(inv_mass, n, n_chains);
    if (!m_shared) NEED(inv_mass, vec, "inv_mass");
    NEED(prec, (size_t)n * 8, "prec");
    NEED(q_chain, chain, "q_chain");
    NEED(p_chain, chain, "p_chain");
    NEED(grad_chain, chain, "grad_chain");
    NEED(logp_chain, (size_t)K * n_chains * 8, "logp_chain");
    NEED(ke_chain, (size_t)K * n_chains * 8, "ke_chain");
    return launch_chain_gauss_f64(c, dptr(q_chain), dptr(p_chain), dptr(grad_chain),
                                  dptr(logp_chain), dptr(q_init), dptr(p_init), dptr(inv_mass),
                                  dptr(prec), 0.0, mu, n, n_chains, K, eps, dptr(ke_chain),
                                  m_shared);
}

int nxv_leapfrog_logreg_f64_batched(void* q_chain, void* p_chain, void* grad_chain,
                                    void* logp_chain, void* q_init, void* p_init, void* X,
                                    void* y, unsigned int n_obs, unsigned int n_dim,
                                    unsigned int n_chains, unsigned int K, double eps,
                                    const char* spv_path) {
    if (!q_chain || !p_chain || !grad_chain || !logp_chain || !q_init || !p_init || !X || !y ||
        !spv_path)
        return E_NULL;
    std::string k = spv_base(spv_path);
    if (k != "leapfrog_logreg_f64_batched.spv") return bad_kernel(k);
    if (K == 0) {
        set_error("K must be positive");
        return E_ARG;
    }
    BEGIN(q_chain, p_chain, grad_chain, logp_chain, q_init, p_init, X, y);
    size_t vec = (size_t)n_dim * 8 * n_chains, chain = vec * K;
    NEED(q_init, vec, "q_init");
    NEED(p_init, vec, "p_init");
    NEED(X, (size_t)n_obs * n_dim * 8, "X");
    NEED(y, (size_t)n_obs * 8, "y");
    NEED(q_chain, chain, "q_chain");
    NEED(p_chain, chain, "p_chain");
    NEED(grad_chain, chain, "grad_chain");
    NEED(logp_chain, (size_t)K * n_chains * 8, "logp_chain");
    return launch_chain_logreg_f64(c, dptr(q_chain), dptr(p_chain), dptr(grad_chain),
                                   dptr(logp_chain), dptr(q_init), dptr(p_init), dptr(X), dptr(y),
                                   n_obs, n_dim, n_chains, K, eps);
}

// ---- devices / interop -------------------------------------------------------------------------

int nxv_init_devices(const int* ids, int n) { return init_devices(ids, n); }
int nxv_set_device(int id) { return set_current(id); }
int nxv_set_stream(void* cuda_stream) { return set_stream((cudaStream_t)cuda_stream); }

int nxv_synchronize(void) {
    BEGIN();
    int rc = sync(c);
    if (rc == OK && tc_gemm_error()) {
        set_error("tensor-core GEMM: a bounded pipeline wait ran out; results are invalid");
        return E_CUDA;
    }
    if (rc == OK && lr_traj_error()) {
        set_error("logistic trajectory kernel: a grid barrier's bounded wait ran out; results "
                  "are invalid");
        return E_CUDA;
    }
    return rc;
}

void* nxv_buf_wrap(void* device_ptr, unsigned long n_bytes) {
    if (!device_ptr && n_bytes) return nullptr;
    return buf_wrap(device_ptr, (size_t)n_bytes);
}

void* nxv_buf_device_ptr(void* handle) {
    Buf* b = as_buf(handle);
    return b ? b->ptr : nullptr;
}

unsigned long nxv_buf_size(void* handle) {
    Buf* b = as_buf(handle);
    return b ? (unsigned long)b->n_bytes : 0;
}

const char* nxv_last_error(void) { return last_error(); }

unsigned long nxv_launch_count(void) { return g_launches.load(); }

}  // extern "C"
