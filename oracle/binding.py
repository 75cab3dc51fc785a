"""numpy binding of liboracle.so (the C restatement in oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for libnxv_b200.so.  Builds the
library from oracle.c with the committed Makefile on first use.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    srcs = [HERE / "oracle.c", HERE / "oracle.h", HERE / "Makefile"]
    if not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True,
                       capture_output=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB))
        _lib.orc_reduce_full_f32.restype = C.c_double
        _lib.orc_reduce_full_f64.restype = C.c_double
        _lib.orc_sum_exact_f64.restype = C.c_double
        _lib.orc_sum_abs_f64.restype = C.c_double
        _lib.orc_kinetic_energy_f32.restype = C.c_double
        _lib.orc_max_threads.restype = C.c_int
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _u32(vals, n=8, fill=0):
    vals = list(vals) + [fill] * (n - len(vals))
    return (C.c_uint * n)(*vals)


def _f64s(vals, n=8):
    vals = list(vals) + [0.0] * (n - len(vals))
    return (C.c_double * n)(*vals)


def f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def f64(x):
    return np.ascontiguousarray(x, dtype=np.float64)


def binary(a, b, op):
    a = np.ascontiguousarray(a)
    out = np.empty_like(a)
    fn = lib().orc_binary_f32 if a.dtype == np.float32 else lib().orc_binary_f64
    fn(_p(out), _p(a), _p(np.ascontiguousarray(b, dtype=a.dtype)), C.c_size_t(a.size), C.c_uint(op))
    return out


def unary(a, op):
    a = np.ascontiguousarray(a)
    out = np.empty_like(a)
    fn = lib().orc_unary_f32 if a.dtype == np.float32 else lib().orc_unary_f64
    fn(_p(out), _p(a), C.c_size_t(a.size), C.c_uint(op))
    return out


def broadcast(a, b, op, ndim, shape, a_strides, b_strides):
    a = np.ascontiguousarray(a)
    n = int(np.prod(shape[:ndim]))
    out = np.empty(n, dtype=a.dtype)
    fn = lib().orc_broadcast_f32 if a.dtype == np.float32 else lib().orc_broadcast_f64
    fn(_p(out), _p(a), _p(np.ascontiguousarray(b, dtype=a.dtype)), C.c_uint(op), C.c_uint(ndim),
       _u32(shape, 4), _u32(a_strides, 4), _u32(b_strides, 4))
    return out


def fused(a, operands, ops, src=None, imm=None, nthreads=0):
    """Op tape: ops codes (binary 0..9 / unary 100..114), src 0 imm, 1..3 operand."""
    a = np.ascontiguousarray(a)
    dt = a.dtype
    ops_l = list(ops)
    srcs = [np.ascontiguousarray(o, dtype=dt) if o is not None else None
            for o in (list(operands) + [None] * 3)[:3]]
    src_l = list(src) if src is not None else [1] * len(ops_l)
    imm_l = list(imm) if imm is not None else [0.0] * len(ops_l)
    out = np.empty_like(a)
    if dt == np.float32 and nthreads:
        lib().orc_fused_f32_mt(_p(out), _p(a), *(_p(s) for s in srcs), C.c_size_t(a.size),
                               C.c_uint(len(ops_l)), _u32(ops_l, 8, 255), _u32(src_l, 8, 1),
                               _f64s(imm_l), C.c_int(nthreads))
        return out
    fn = lib().orc_fused_f32 if dt == np.float32 else lib().orc_fused_f64
    fn(_p(out), _p(a), *(_p(s) for s in srcs), C.c_size_t(a.size), C.c_uint(len(ops_l)),
       _u32(ops_l, 8, 255), _u32(src_l, 8, 1), _f64s(imm_l))
    return out


def reduce_full(a, op):
    a = np.ascontiguousarray(a)
    fn = lib().orc_reduce_full_f32 if a.dtype == np.float32 else lib().orc_reduce_full_f64
    return fn(_p(a), C.c_size_t(a.size), C.c_uint(op))


def sum_exact(a):
    a = f64(a)
    return lib().orc_sum_exact_f64(_p(a), C.c_size_t(a.size))


def sum_abs(a):
    a = f64(a)
    return lib().orc_sum_abs_f64(_p(a), C.c_size_t(a.size))


def reduce_axis(a, outer, R, inner, op):
    a = np.ascontiguousarray(a)
    out = np.empty(outer * inner, dtype=a.dtype)
    fn = lib().orc_reduce_axis_f32 if a.dtype == np.float32 else lib().orc_reduce_axis_f64
    fn(_p(out), _p(a), C.c_size_t(outer), C.c_size_t(R), C.c_size_t(inner), C.c_uint(op))
    return out


def argmax_axis(a, outer, R, inner, is_min=False):
    a = np.ascontiguousarray(a)
    out = np.empty(outer * inner, dtype=np.int64)
    fn = lib().orc_argmax_axis_f32 if a.dtype == np.float32 else lib().orc_argmax_axis_f64
    fn(_p(out), _p(a), C.c_size_t(outer), C.c_size_t(R), C.c_size_t(inner), C.c_int(int(is_min)))
    return out


def logsumexp(a, outer, R, inner):
    a = f32(a)
    out = np.empty(outer * inner, dtype=np.float32)
    lib().orc_logsumexp_f32(_p(out), _p(a), C.c_size_t(outer), C.c_size_t(R), C.c_size_t(inner))
    return out


def matmul(a, b, m, n, k, batch=1):
    a = np.ascontiguousarray(a)
    out = np.empty(batch * m * n, dtype=a.dtype)
    b = np.ascontiguousarray(b, dtype=a.dtype)
    if a.dtype == np.float32:
        lib().orc_matmul_batched_f32(_p(out), _p(a), _p(b), C.c_size_t(batch), C.c_size_t(m),
                                     C.c_size_t(n), C.c_size_t(k))
    else:
        lib().orc_matmul_batched_f64(_p(out), _p(a), _p(b), C.c_size_t(batch), C.c_size_t(m),
                                     C.c_size_t(n), C.c_size_t(k))
    return out


def transpose(a, m, n):
    a = f32(a)
    out = np.empty(m * n, dtype=np.float32)
    lib().orc_transpose_f32(_p(out), _p(a), C.c_uint(m), C.c_uint(n))
    return out


def random_f32(n, seed, dist):
    out = np.empty(n, dtype=np.float32)
    lib().orc_random_f32(_p(out), C.c_size_t(n), C.c_uint32(seed), C.c_uint(dist))
    return out


def random_f64(n, seed, dist):
    out = np.empty(n, dtype=np.float64)
    lib().orc_random_f64(_p(out), C.c_size_t(n), C.c_uint32(seed), C.c_uint(dist))
    return out


def philox2x32(c0, c1, key):
    o0, o1 = C.c_uint32(0), C.c_uint32(0)
    lib().orc_philox2x32(C.c_uint32(c0), C.c_uint32(c1), C.c_uint32(key), C.byref(o0), C.byref(o1))
    return o0.value, o1.value


def kinetic_energy(p, m):
    p, m = f32(p), f32(m)
    return lib().orc_kinetic_energy_f32(_p(p), _p(m), C.c_size_t(p.size))


def normal_logpdf(x, mu, sigma):
    x = f32(x)
    out = np.empty_like(x)
    lib().orc_normal_logpdf_f32(_p(out), _p(x), _p(f32(mu)), _p(f32(sigma)), C.c_size_t(x.size))
    return out


def leapfrog_step_f32(q, p, m, eps, mu, sigma):
    q, p, m = f32(q), f32(p), f32(m)
    qn, pn = np.empty_like(q), np.empty_like(p)
    lib().orc_leapfrog_normal_step_f32(_p(qn), _p(pn), _p(q), _p(p), _p(m), C.c_size_t(q.size),
                                       C.c_float(eps), C.c_float(mu), C.c_float(sigma))
    return qn, pn


FAMILIES = {"normal": 0, "exponential": 1, "studentt": 2, "cauchy": 3, "halfnormal": 4,
            "weibull": 5}


def chain_f32(family, prm, q0, p0, m, n, chains, K, eps):
    q0, p0, m = f32(q0), f32(p0), f32(m)
    qc = np.empty(chains * K * n, np.float32)
    pc, gc = np.empty_like(qc), np.empty_like(qc)
    lp = np.empty(chains * K, np.float32)
    pr = (C.c_float * 8)(*(list(prm) + [0.0] * (8 - len(prm))))
    lib().orc_leapfrog_chain_f32(C.c_int(FAMILIES[family]), pr, _p(qc), _p(pc), _p(gc), _p(lp),
                                 _p(q0), _p(p0), _p(m), C.c_size_t(n), C.c_size_t(chains),
                                 C.c_uint(K), C.c_float(eps))
    return qc, pc, gc, lp


def chain_gauss_f64(q0, p0, m, prec, mu, n, chains, K, eps, nthreads=1):
    q0, p0, m, prec = f64(q0), f64(p0), f64(m), f64(prec)
    qc = np.empty(chains * K * n, np.float64)
    pc, gc = np.empty_like(qc), np.empty_like(qc)
    lp = np.empty(chains * K, np.float64)
    lib().orc_leapfrog_gauss_f64(_p(qc), _p(pc), _p(gc), _p(lp), _p(q0), _p(p0), _p(m), _p(prec),
                                 C.c_double(mu), C.c_size_t(n), C.c_size_t(chains), C.c_uint(K),
                                 C.c_double(eps), C.c_int(nthreads))
    return qc, pc, gc, lp


def chain_logreg_f64(q0, p0, X, y, n_obs, n_dim, chains, K, eps, nthreads=1):
    q0, p0, X, y = f64(q0), f64(p0), f64(X), f64(y)
    qc = np.empty(chains * K * n_dim, np.float64)
    pc, gc = np.empty_like(qc), np.empty_like(qc)
    lp = np.empty(chains * K, np.float64)
    lib().orc_leapfrog_logreg_f64(_p(qc), _p(pc), _p(gc), _p(lp), _p(q0), _p(p0), _p(X), _p(y),
                                  C.c_size_t(n_obs), C.c_size_t(n_dim), C.c_size_t(chains),
                                  C.c_uint(K), C.c_double(eps), C.c_int(nthreads))
    return qc, pc, gc, lp


def max_threads():
    return lib().orc_max_threads()
