"""ctypes binding of libnxv_b200.so, the nxv_* C ABI (include/nx_vulkan_shim.h).

This is the host-side equivalent of the reference's extern "C" block in
native/nx_vulkan_native/src/lib.rs:30-295: one declaration per exported
function, with the exact C signature.  Loading fails loudly when the library
has not been built: there is no CPU fallback for any nxv_* operation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libnxv_b200.so"

vp = C.c_void_p
u32 = C.c_uint
ul = C.c_ulong
f32 = C.c_float
f64 = C.c_double
cstr = C.c_char_p
u32p = C.POINTER(C.c_uint)
ulp = C.POINTER(C.c_ulong)
f32p = C.POINTER(C.c_float)
f64p = C.POINTER(C.c_double)
intp = C.POINTER(C.c_int)

CHAIN7 = [vp] * 7

# name -> (restype, argtypes); mirrors include/nx_vulkan_shim.h line by line.
SIGNATURES: dict[str, tuple] = {
    "nxv_init": (C.c_int, []),
    "nxv_destroy": (None, []),
    "nxv_device_name": (cstr, []),
    "nxv_has_f64": (C.c_int, []),
    "nxv_buf_alloc": (vp, [ul]),
    "nxv_buf_free": (None, [vp]),
    "nxv_pool_clear": (None, []),
    "nxv_pool_stats": (None, [ulp, ulp, ulp, ulp, ulp]),
    "nxv_buf_upload": (C.c_int, [vp, vp, ul]),
    "nxv_buf_download": (C.c_int, [vp, vp, ul]),
    "nxv_apply_binary": (C.c_int, [vp, vp, vp, u32, u32, cstr]),
    "nxv_apply_unary": (C.c_int, [vp, vp, u32, u32, cstr]),
    "nxv_cast": (C.c_int, [vp, vp, u32, cstr]),
    "nxv_apply_binary_broadcast": (C.c_int, [vp, vp, vp, u32, u32, u32p, u32p, u32p, cstr]),
    "nxv_transpose": (C.c_int, [vp, vp, u32, u32, cstr]),
    "nxv_fused_chain": (C.c_int, [vp, vp, vp, u32, u32, u32p, cstr]),
    "nxv_fused_chain_4": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32p, u32p, cstr]),
    "nxv_fused_chain_imm": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32p, u32p, f64p, u32, cstr]),
    "nxv_reduce": (C.c_int, [f32p, vp, u32, u32, cstr]),
    "nxv_reduce_axis": (C.c_int, [vp, vp, u32, u32, u32, u32, cstr]),
    "nxv_reduce_f64": (C.c_int, [f64p, vp, ul, u32, cstr]),
    "nxv_reduce_to_buf": (C.c_int, [vp, vp, ul, u32, u32, cstr]),
    "nxv_argmax_axis": (C.c_int, [vp, vp, u32, u32, u32, u32, u32, u32, cstr]),
    "nxv_matmul": (C.c_int, [vp, vp, vp, u32, u32, u32, cstr]),
    "nxv_matmul_v": (C.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, cstr]),
    "nxv_matmul_batched": (C.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, cstr]),
    "nxv_random": (C.c_int, [vp, u32, u32, u32, cstr]),
    "nxv_random_f64": (C.c_int, [vp, ul, u32, u32, cstr]),
    "nxv_kinetic_energy": (C.c_int, [vp, vp, vp, u32, cstr]),
    "nxv_normal_logpdf": (C.c_int, [vp, vp, vp, vp, u32, cstr]),
    "nxv_leapfrog_normal": (C.c_int, [vp, vp, vp, vp, vp, u32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_normal": (C.c_int, CHAIN7 + [u32, u32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_normal_lg": (C.c_int, CHAIN7 + [u32, u32, u32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_exponential": (C.c_int, CHAIN7 + [u32, u32, f32, f32, cstr]),
    "nxv_leapfrog_chain_studentt": (C.c_int, CHAIN7 + [u32, u32, f32, f32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_cauchy": (C.c_int, CHAIN7 + [u32, u32, f32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_halfnormal": (C.c_int, CHAIN7 + [u32, u32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_weibull": (C.c_int, CHAIN7 + [u32, u32, f32, f32, f32, f32, cstr]),
    "nxv_leapfrog_chain_normal_f64": (C.c_int, CHAIN7 + [u32, u32, f64, f64, f64, cstr]),
    "nxv_leapfrog_chain_gauss_f64_batched": (C.c_int, CHAIN7 + [vp, u32, u32, u32, f64, f64, cstr]),
    "nxv_leapfrog_chain_gauss_f64_batched_ke": (C.c_int, [vp] * 9 + [u32, u32, u32, f64, f64, cstr]),
    "nxv_leapfrog_chain_gauss_f64_batched_noalloc": (C.c_int, [vp] * 8 + [u32, u32, u32, f64, f64]),
    "nxv_leapfrog_logreg_f64_batched": (C.c_int, [vp] * 8 + [u32, u32, u32, u32, f64, cstr]),
    "nxv_nuts_energy": (C.c_int, [vp] * 5 + [f64, f64, u32, u32]),
    "nxv_nuts_start": (C.c_int, [vp] * 9 + [u32, u32, u32]),
    "nxv_nuts_level": (C.c_int, [vp] * 5 + [u32, u32, u32] + [vp] * 14 + [u32]),
    "nxv_nuts_start_layout": (C.c_int, [vp] * 8 + [u32, u32]),
    "nxv_nuts_level_layout": (C.c_int, [C.c_ulonglong, u32, u32] + [vp] * 18 + [u32, u32]),
    "nxv_nuts_transition_layout": (C.c_int, [vp] * 6 + [f64, f64, f64, u32, u32, u32, u32]),
    "nxv_init_devices": (C.c_int, [intp, C.c_int]),
    "nxv_set_device": (C.c_int, [C.c_int]),
    "nxv_set_stream": (C.c_int, [vp]),
    "nxv_synchronize": (C.c_int, []),
    "nxv_buf_copy_2d": (C.c_int, [vp, ul, ul, vp, ul, ul, ul, ul]),
    "nxv_buf_wrap": (vp, [vp, ul]),
    "nxv_buf_device_ptr": (vp, [vp]),
    "nxv_buf_size": (ul, [vp]),
    "nxv_last_error": (cstr, []),
    "nxv_launch_count": (ul, []),
}

_lib = None


def load(path: str | os.PathLike | None = None):
    """Load the CUDA library (once) and declare every signature."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"libnxv_b200.so not found at {p}; build it with `python -m nx_vulkan_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return (load().nxv_last_error() or b"").decode()


def u32_array(vals) -> C.Array:
    vals = list(vals)
    return (C.c_uint * max(1, len(vals)))(*vals)


def f64_array(vals) -> C.Array:
    vals = list(vals)
    return (C.c_double * max(1, len(vals)))(*vals)
