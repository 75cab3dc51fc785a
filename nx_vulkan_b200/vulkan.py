"""Host-side mirror of the reference's `Nx.Vulkan` module and NIF layer.

The reference's host code is Elixir (lib/nx_vulkan.ex) over a Rustler NIF
(native/nx_vulkan_native/src/lib.rs).  No Elixir or Rust toolchain exists
here, so this module restates that layer in Python over the same C ABI, with
the same function names, argument meaning and error behaviour:

  * results are ``("ok", value)`` or ``("error", atom)`` like ``{:ok, v}`` /
    ``{:error, :size_mismatch}``; the atoms are the NIF's
    (lib.rs:15-27: no_device, alloc_failed, upload_failed, download_failed,
    size_mismatch, dispatch_failed, bad_op);
  * the NIF-level validation is kept (equal byte sizes, op ranges, K > 0,
    matmul byte sizes, download size == buffer size, lib.rs:420-422);
  * outputs are allocated from the pool before the op and freed again when
    the op fails (lib.rs:489-492);
  * a `VulkanTensor` owns its device buffer and returns it to the pool when
    garbage collected (the ResourceArc Drop, lib.rs:330-342).

Everything computes on the GPU through libnxv_b200.so; nothing here
evaluates tensor math on the host.  Like the reference module, this module
defines `max`, `min`, `sum` and `abs` as GPU ops; internal code uses
`_builtins` for the Python ones.
"""
from __future__ import annotations

import builtins as _builtins
import ctypes as C
import math
import struct
from typing import Iterable, Sequence

from . import _native

OK = "ok"
ERROR = "error"

_SHADERS = "priv/shaders"


def shader_path(name: str) -> bytes:
    """lib/nx_vulkan.ex:171-177: priv/shaders/<name>.  Only the basename matters."""
    return f"{_SHADERS}/{name}".encode()


class VulkanTensor:
    """A device buffer handle with its byte size (lib.rs:330-342)."""

    __slots__ = ("handle", "n_bytes", "__weakref__")

    def __init__(self, handle: int, n_bytes: int):
        self.handle = handle
        self.n_bytes = n_bytes

    def __del__(self):
        h, self.handle = getattr(self, "handle", None), None
        if h and _native._lib is not None:
            _native._lib.nxv_buf_free(h)

    @property
    def device_ptr(self) -> int:
        return _native.load().nxv_buf_device_ptr(self.handle) or 0


def _lib():
    return _native.load()


def _alloc(n_bytes: int):
    h = _lib().nxv_buf_alloc(n_bytes)
    if not h:
        return None
    return VulkanTensor(h, n_bytes)


def _dispatch(outs: Sequence[VulkanTensor], rc: int):
    if rc != 0:
        for o in outs:
            o.__del__()
        return (ERROR, "dispatch_failed")
    return (OK, outs[0] if len(outs) == 1 else tuple(outs))


# ---- lifecycle (lib/nx_vulkan.ex:41-53; lib.rs:344-386) ------------------------

_initialised = False


def init():
    """`Nx.Vulkan.init/0`: idempotent; ``"ok"`` or ``("error", "no_device")``."""
    global _initialised
    if _initialised:
        return OK
    if _lib().nxv_init() == 0:
        _initialised = True
        return OK
    return (ERROR, "no_device")


def init_devices(ids: Sequence[int]):
    """Select the GPUs this process drives (one process per GPU: [local_rank])."""
    global _initialised
    arr = (C.c_int * len(ids))(*ids)
    if _lib().nxv_init_devices(arr, len(ids)) == 0:
        _initialised = True
        return OK
    return (ERROR, "no_device")


def device_name():
    if not _initialised:
        return None
    s = _lib().nxv_device_name()
    return s.decode() if s else None


def has_f64() -> bool:
    return _lib().nxv_has_f64() != 0


# ---- transfers (lib/nx_vulkan.ex:55-137; lib.rs:388-453) ------------------------

def upload_binary(data) -> tuple:
    mv = memoryview(data).cast("B")
    n = mv.nbytes
    t = _alloc(n)
    if t is None:
        return (ERROR, "alloc_failed")
    if n:
        buf = (C.c_char * n).from_buffer_copy(mv) if mv.readonly else (C.c_char * n).from_buffer(mv)
        if _lib().nxv_buf_upload(t.handle, buf, n) != 0:
            t.__del__()
            return (ERROR, "upload_failed")
    return (OK, t)


def upload_f32(values: Iterable[float]):
    vals = list(values)
    return upload_binary(struct.pack(f"<{len(vals)}f", *vals))


def upload_f64(values: Iterable[float]):
    vals = list(values)
    return upload_binary(struct.pack(f"<{len(vals)}d", *vals))


def download_binary(t: VulkanTensor, n_bytes: int):
    if n_bytes != t.n_bytes:
        return (ERROR, "size_mismatch")
    buf = (C.c_char * _builtins.max(1, n_bytes))()
    if _lib().nxv_buf_download(t.handle, buf, n_bytes) != 0:
        return (ERROR, "download_failed")
    return (OK, bytes(buf)[:n_bytes])


def _decode(x: float):
    # lib/nx_vulkan.ex:85-127: non-finite values decode to atoms.
    if math.isnan(x):
        return "nan"
    if math.isinf(x):
        return "infinity" if x > 0 else "neg_infinity"
    return x


def download_f32(t: VulkanTensor, n: int):
    r = download_binary(t, n * 4)
    if r[0] != OK:
        return r
    return (OK, [_decode(v) for v in struct.unpack(f"<{n}f", r[1])])


def download_f64(t: VulkanTensor, n: int):
    r = download_binary(t, n * 8)
    if r[0] != OK:
        return r
    return (OK, [_decode(v) for v in struct.unpack(f"<{n}d", r[1])])


def byte_size(t: VulkanTensor) -> int:
    return t.n_bytes


# ---- elementwise (lib/nx_vulkan.ex:139-240; lib.rs:455-530, 965-1034) ------------

OPS_BINARY = {"add": 0, "multiply": 1, "subtract": 2, "divide": 3, "pow": 4, "max": 5,
              "min": 6, "equal": 7, "less": 8, "greater": 9}
OPS_UNARY = {"exp": 0, "log": 1, "sqrt": 2, "abs": 3, "negate": 4, "sigmoid": 5, "tanh": 6,
             "relu": 7, "ceil": 8, "floor": 9, "sign": 10, "reciprocal": 11, "square": 12,
             "erf": 13, "expm1": 14}


def apply_binary(a: VulkanTensor, b: VulkanTensor, op: int, spv: bytes, elt: int = 4,
                 max_op: int = 9):
    if op > max_op:
        return (ERROR, "bad_op")
    if a.n_bytes != b.n_bytes:
        return (ERROR, "size_mismatch")
    out = _alloc(a.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_apply_binary(out.handle, a.handle, b.handle, a.n_bytes // elt, op, spv)
    return _dispatch([out], rc)


def apply_unary(a: VulkanTensor, op: int, spv: bytes, elt: int = 4):
    if op > 14:
        return (ERROR, "bad_op")
    out = _alloc(a.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_apply_unary(out.handle, a.handle, a.n_bytes // elt, op, spv)
    return _dispatch([out], rc)


def _mk_binary(name, code):
    def f(a, b):
        return apply_binary(a, b, code, shader_path("elementwise_binary.spv"))
    f.__name__ = name
    f.__doc__ = f"Elementwise `{name}` of two f32 GPU tensors of equal length."
    return f


def _mk_unary(name, code):
    def f(a):
        return apply_unary(a, code, shader_path("elementwise_unary.spv"))
    f.__name__ = name
    f.__doc__ = f"Elementwise `{name}` of an f32 GPU tensor."
    return f


for _n, _c in OPS_BINARY.items():
    globals()[_n] = _mk_binary(_n, _c)
for _n, _c in OPS_UNARY.items():
    globals()[_n] = _mk_unary(_n, _c)


def apply_binary_f64(a, b, op: str):
    return apply_binary(a, b, OPS_BINARY[op], shader_path("elementwise_binary_f64.spv"), 8, 9)


def apply_unary_f64(a, op: str):
    return apply_unary(a, OPS_UNARY[op], shader_path("elementwise_unary_f64.spv"), 8)


# ---- broadcast (lib/nx_vulkan.ex:768-842; lib.rs:740-789, 876-925) ------------------

def _pad4(xs):
    xs = list(xs)[:4]
    return xs + [0] * (4 - len(xs))


def broadcast_strides(src_shape: Sequence[int], out_shape: Sequence[int]):
    """lib/nx_vulkan.ex:808-835: right-aligned, stride 0 on broadcast axes."""
    src, out = list(src_shape), list(out_shape)
    src = [1] * (len(out) - len(src)) + src
    strides, running = [], 1
    for sd, od in reversed(list(zip(src, out))):
        if sd == od:
            strides.insert(0, running)
            running *= sd
        elif sd == 1:
            strides.insert(0, 0)
        else:
            raise ValueError(f"shapes don't broadcast: {tuple(src_shape)} -> {tuple(out_shape)}")
    return _pad4(strides)


def _broadcast(a, b, op_code, ndim, out_shape, a_strides, b_strides, spv, elt):
    if op_code > 9:
        return (ERROR, "bad_op")
    if ndim == 0 or ndim > 4 or len(out_shape) != 4 or len(a_strides) != 4 or len(b_strides) != 4:
        return (ERROR, "bad_op")
    n = 1
    for d in range(ndim):
        n *= out_shape[d]
    out = _alloc(n * elt)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_apply_binary_broadcast(out.handle, a.handle, b.handle, op_code, ndim,
                                           _native.u32_array(out_shape),
                                           _native.u32_array(a_strides),
                                           _native.u32_array(b_strides), spv)
    return _dispatch([out], rc)


def apply_binary_broadcast(a, b, op: str, ndim, out_shape, a_strides, b_strides):
    return _broadcast(a, b, OPS_BINARY[op], ndim, _pad4(out_shape), _pad4(a_strides),
                      _pad4(b_strides), shader_path("elementwise_binary_broadcast.spv"), 4)


def apply_binary_broadcast_f64(a, b, op: str, ndim, out_shape, a_strides, b_strides):
    return _broadcast(a, b, OPS_BINARY[op], ndim, _pad4(out_shape), _pad4(a_strides),
                      _pad4(b_strides), shader_path("elementwise_binary_broadcast_f64.spv"), 8)


# ---- reductions (lib/nx_vulkan.ex:226-275, 441-451; lib.rs:533-559, 701-735) ----------

def _reduce_scalar(t, op):
    if op > 2:
        return (ERROR, "bad_op")
    out = C.c_float(0.0)
    rc = _lib().nxv_reduce(C.byref(out), t.handle, t.n_bytes // 4, op,
                           shader_path("reduce.spv"))
    if rc != 0:
        return (ERROR, "dispatch_failed")
    return (OK, out.value)


def sum(t):  # noqa: A001 - mirrors Nx.Vulkan.sum/1
    return _reduce_scalar(t, 0)


def reduce_min(t):
    return _reduce_scalar(t, 1)


def reduce_max(t):
    return _reduce_scalar(t, 2)


def mean(t):
    r = sum(t)
    if r[0] != OK:
        return r
    return (OK, r[1] / (t.n_bytes // 4))


def reduce_f64(t, op: int):
    """Full f64 reduce (wires reduce_full_f64.spv, unwired in the reference)."""
    if op > 2:
        return (ERROR, "bad_op")
    out = C.c_double(0.0)
    rc = _lib().nxv_reduce_f64(C.byref(out), t.handle, t.n_bytes // 8, op,
                               shader_path("reduce_full_f64.spv"))
    if rc != 0:
        return (ERROR, "dispatch_failed")
    return (OK, out.value)


def _out_buffer(out, n_bytes):
    """The caller's output buffer (checked to hold n_bytes), or a new one."""
    if out is not None:
        return out if out.n_bytes >= n_bytes else None
    return _alloc(n_bytes)


def _dispatch_into(out, given, rc):
    if given is not None:
        return (OK, out) if rc == 0 else (ERROR, "dispatch_failed")
    return _dispatch([out], rc)


def _reduce_axis(a, outer, r, inner, op, spv, elt, out=None):
    if op > 2:
        return (ERROR, "bad_op")
    o = _out_buffer(out, outer * inner * elt)
    if o is None:
        return (ERROR, "alloc_failed" if out is None else "size_mismatch")
    rc = _lib().nxv_reduce_axis(o.handle, a.handle, outer, r, inner, op, spv)
    return _dispatch_into(o, out, rc)


def reduce_axis(a, outer, reduce_size, inner, op, out=None):
    """(outer, reduce, inner) -> (outer, inner); op 0 sum, 1 max, 2 min.
    `out`: an existing buffer to write the result into (e.g. wrap_tensor)."""
    return _reduce_axis(a, outer, reduce_size, inner, op, shader_path("reduce_axis.spv"), 4, out)


def reduce_axis_f64(a, outer, reduce_size, inner, op, out=None):
    return _reduce_axis(a, outer, reduce_size, inner, op, shader_path("reduce_axis_f64.spv"), 8,
                        out)


def logsumexp(a, outer, reduce_size, inner):
    return _reduce_axis(a, outer, reduce_size, inner, 0, shader_path("logsumexp.spv"), 4)


def argmax_axis(a, outer, reduce_size, inner, *, dtype="f32", is_min=False, index_bytes=8,
                out=None):
    """argmax/argmin over the middle axis; lowest index wins ties (Nx :low)."""
    o = _out_buffer(out, outer * inner * index_bytes)
    if o is None:
        return (ERROR, "alloc_failed" if out is None else "size_mismatch")
    rc = _lib().nxv_argmax_axis(o.handle, a.handle, outer, reduce_size, inner, int(is_min),
                                0 if dtype == "f32" else 1, index_bytes,
                                shader_path("argmax_axis.spv"))
    return _dispatch_into(o, out, rc)


# ---- matmul (lib/nx_vulkan.ex:277-347; lib.rs:563-598, 1038-1078) --------------------

def pick_matmul(m, n, k):
    """lib/nx_vulkan.ex:330-342 (kept for API compatibility; every choice runs
    the same tensor-core kernel)."""
    flops = m * n * k
    if flops < 4096:
        return ("matmul.spv", 16, 16)
    if flops >= 16_777_216:
        return ("matmul_tiled16x2.spv", 32, 16)
    return ("matmul_tiled.spv", 16, 16)


_VARIANT_TILES = {"matmul": (16, 16), "matmul_tiled": (16, 16), "matmul_tiled32": (32, 32),
                  "matmul_tiled16x2": (32, 16)}


def matmul_variant(a, b, m, n, k, variant, tile_m=None, tile_n=None):
    if tile_m is None:
        if variant not in _VARIANT_TILES:
            raise ValueError(f"unknown matmul variant {variant!r}")
        tile_m, tile_n = _VARIANT_TILES[variant]
        name = f"{variant}.spv"
    else:
        name = variant
    if a.n_bytes != m * k * 4 or b.n_bytes != k * n * 4:
        return (ERROR, "size_mismatch")
    out = _alloc(m * n * 4)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_matmul_v(out.handle, a.handle, b.handle, m, n, k, tile_m, tile_n,
                             shader_path(name))
    return _dispatch([out], rc)


def matmul(a, b, m, n, k):
    shader, tm, tn = pick_matmul(m, n, k)
    return matmul_variant(a, b, m, n, k, shader, tm, tn)


def matmul_batched(a, b, batch, m, n, k, dtype="f64", out=None):
    elt = 4 if dtype == "f32" else 8
    if a.n_bytes != batch * m * k * elt or b.n_bytes != batch * k * n * elt:
        return (ERROR, "size_mismatch")
    o = _out_buffer(out, batch * m * n * elt)
    if o is None:
        return (ERROR, "alloc_failed" if out is None else "size_mismatch")
    rc = _lib().nxv_matmul_batched(o.handle, a.handle, b.handle, batch, m, n, k,
                                   0 if dtype == "f32" else 1, shader_path("matmul_batched.spv"))
    return _dispatch_into(o, out, rc)


def wrap_tensor(t):
    """Non-owning handle over the memory of a torch CUDA tensor (nxv_buf_wrap),
    for calls that write their result into it in place.  The tensor must stay
    alive while work using the handle can run."""
    n = t.numel() * t.element_size()
    h = _lib().nxv_buf_wrap(C.c_void_p(t.data_ptr()), n)
    return VulkanTensor(h, n) if h else None



# ---- random (lib/nx_vulkan.ex:349-361; lib.rs:602-635) ----------------------------------

def random(n, seed, dist):
    if dist > 1:
        return (ERROR, "bad_op")
    out = _alloc(n * 4)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_random(out.handle, n, seed, dist, shader_path("random_philox.spv"))
    return _dispatch([out], rc)


def uniform(n, seed=42):
    return random(n, seed, 0)


def normal(n, seed=42):
    return random(n, seed, 1)


def random_f64(n, seed, dist):
    out = _alloc(n * 8)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_random_f64(out.handle, n, seed, dist, shader_path("random_philox_f64.spv"))
    return _dispatch([out], rc)


# ---- compositions (lib/nx_vulkan.ex:363-412) -----------------------------------------------

def _upload_constant(value, n):
    return upload_f32([float(value)] * n)


def select(cond, t, f):
    """cond * t + (1 - cond) * f (lib/nx_vulkan.ex:376-387)."""
    n = cond.n_bytes // 4
    ok, ones = _upload_constant(1.0, n)
    if ok != OK:
        return (ok, ones)
    steps = [subtract(ones, cond)]
    if steps[-1][0] != OK:
        return steps[-1]
    on_t = multiply(cond, t)
    on_f = multiply(steps[-1][1], f)
    if on_t[0] != OK:
        return on_t
    if on_f[0] != OK:
        return on_f
    return add(on_t[1], on_f[1])


def clip(a, low, high):
    """max(low, min(high, a)) (lib/nx_vulkan.ex:396-406)."""
    n = a.n_bytes // 4
    lo = _upload_constant(low, n)
    hi = _upload_constant(high, n)
    capped = min(a, hi[1])  # noqa: A001
    if capped[0] != OK:
        return capped
    return max(lo[1], capped[1])  # noqa: A001


# ---- transpose / cast (lib/nx_vulkan.ex:419-439; lib.rs:637-700) ---------------------------

def transpose_2d(a, m, n):
    if a.n_bytes != m * n * 4:
        return (ERROR, "size_mismatch")
    out = _alloc(a.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    return _dispatch([out], _lib().nxv_transpose(out.handle, a.handle, m, n,
                                                 shader_path("transpose.spv")))


def cast(a, n, out_elt, spv):
    out = _alloc(n * out_elt)
    if out is None:
        return (ERROR, "alloc_failed")
    return _dispatch([out], _lib().nxv_cast(out.handle, a.handle, n, spv))


def cast_f32_to_f64(a, n):
    return cast(a, n, 8, shader_path("cast_f32_to_f64.spv"))


def cast_f64_to_f32(a, n):
    return cast(a, n, 4, shader_path("cast_f64_to_f32.spv"))


# ---- fused chains (lib/nx_vulkan.ex:453-538; lib.rs:794-835, 1705-1756) ---------------------

OP_CODES = {"add": 0, "multiply": 1, "subtract": 2, "divide": 3, "pow": 4, "max": 5, "min": 6,
            "exp": 100, "log": 101, "sqrt": 102, "abs": 103, "negate": 104, "sigmoid": 105,
            "tanh": 106, "relu": 107, "ceil": 108, "floor": 109, "sign": 110,
            "reciprocal": 111, "square": 112, "erf": 113, "expm1": 114}


def fused_chain(a, b, ops: Sequence[str]):
    codes = [OP_CODES[o] for o in ops]  # KeyError on unknown atoms, like Map.fetch!
    if not codes or len(codes) > 8:
        return (ERROR, "bad_op")
    if a.n_bytes != b.n_bytes:
        return (ERROR, "size_mismatch")
    out = _alloc(a.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    arr = _native.u32_array(codes + [255] * (8 - len(codes)))
    rc = _lib().nxv_fused_chain(out.handle, a.handle, b.handle, a.n_bytes // 4, len(codes), arr,
                                shader_path("fused_elementwise.spv"))
    return _dispatch([out], rc)


def fused_chain_4(a, b, c, d, ops_with_buf):
    codes, idx = [], []
    for item in ops_with_buf:
        if isinstance(item, tuple):
            codes.append(OP_CODES[item[0]])
            idx.append(item[1])
        else:
            codes.append(OP_CODES[item])
            idx.append(1)
    if not codes or len(codes) > 8:
        return (ERROR, "bad_op")
    if not (a.n_bytes == b.n_bytes == c.n_bytes == d.n_bytes):
        return (ERROR, "size_mismatch")
    out = _alloc(a.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_fused_chain_4(out.handle, a.handle, b.handle, c.handle, d.handle,
                                  a.n_bytes // 4, len(codes),
                                  _native.u32_array(codes + [255] * (8 - len(codes))),
                                  _native.u32_array(idx + [1] * (8 - len(idx))),
                                  shader_path("fused_elementwise_4in.spv"))
    return _dispatch([out], rc)


def fused_chain_imm(a, operands: Sequence, ops: Sequence, *, dtype="f32"):
    """Op tape with immediates: ops items are unary atoms or (binary_atom, src)
    where src is 1..3 (operand b/c/d) or ("imm", value)."""
    elt = 4 if dtype == "f32" else 8
    codes, src, imm = [], [], []
    bin_codes = dict(OPS_BINARY)
    for item in ops:
        if isinstance(item, tuple):
            name, s = item
            codes.append(bin_codes[name])
            if isinstance(s, tuple) and s[0] == "imm":
                src.append(0)
                imm.append(float(s[1]))
            else:
                src.append(int(s))
                imm.append(0.0)
        else:
            codes.append(OP_CODES[item])
            src.append(1)
            imm.append(0.0)
    if not codes or len(codes) > 8:
        return (ERROR, "bad_op")
    ops_b = list(operands) + [None] * (3 - len(operands))
    for o in ops_b:
        if o is not None and o.n_bytes != a.n_bytes:
            return (ERROR, "size_mismatch")
    out = _alloc(a.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    pad = 8 - len(codes)
    rc = _lib().nxv_fused_chain_imm(out.handle, a.handle,
                                    *(o.handle if o is not None else None for o in ops_b),
                                    a.n_bytes // elt, len(codes),
                                    _native.u32_array(codes + [255] * pad),
                                    _native.u32_array(src + [1] * pad),
                                    _native.f64_array(imm + [0.0] * pad),
                                    0 if dtype == "f32" else 1,
                                    shader_path("fused_elementwise_imm.spv"))
    return _dispatch([out], rc)


# ---- HMC primitives (lib/nx_vulkan.ex:540-580; lib.rs:1082-1241) ----------------------------

def kinetic_energy(p, inv_mass):
    if p.n_bytes != inv_mass.n_bytes:
        return (ERROR, "size_mismatch")
    n = p.n_bytes // 4
    out = _alloc(((n + 255) // 256) * 4)
    if out is None:
        return (ERROR, "alloc_failed")
    return _dispatch([out], _lib().nxv_kinetic_energy(out.handle, p.handle, inv_mass.handle, n,
                                                      shader_path("kinetic_energy.spv")))


def normal_logpdf(x, mu, sigma):
    if not (x.n_bytes == mu.n_bytes == sigma.n_bytes):
        return (ERROR, "size_mismatch")
    out = _alloc(x.n_bytes)
    if out is None:
        return (ERROR, "alloc_failed")
    return _dispatch([out], _lib().nxv_normal_logpdf(out.handle, x.handle, mu.handle, sigma.handle,
                                                     x.n_bytes // 4,
                                                     shader_path("normal_logpdf.spv")))


def leapfrog_normal(q, p, inv_mass, eps, mu, sigma):
    if not (q.n_bytes == p.n_bytes == inv_mass.n_bytes):
        return (ERROR, "size_mismatch")
    qn, pn = _alloc(q.n_bytes), _alloc(q.n_bytes)
    if qn is None or pn is None:
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_leapfrog_normal(qn.handle, pn.handle, q.handle, p.handle, inv_mass.handle,
                                    q.n_bytes // 4, eps, mu, sigma,
                                    shader_path("leapfrog_normal.spv"))
    return _dispatch([qn, pn], rc)


def _chain(fn_name, spv, q, p, m, k, scalars, elt=4, partial_groups=None):
    """The allocate-4 / dispatch / return-4-tuple pattern of lib.rs:1307-1662."""
    if not (q.n_bytes == p.n_bytes == m.n_bytes):
        return (ERROR, "size_mismatch")
    if k <= 0:
        return (ERROR, "bad_op")
    n = q.n_bytes // elt
    chain_bytes = q.n_bytes * k
    logp_bytes = k * elt * (partial_groups or 1)
    outs = [_alloc(chain_bytes), _alloc(chain_bytes), _alloc(chain_bytes), _alloc(logp_bytes)]
    if any(o is None for o in outs):
        return (ERROR, "alloc_failed")
    extra = [partial_groups] if partial_groups else []
    rc = getattr(_lib(), fn_name)(*(o.handle for o in outs), q.handle, p.handle, m.handle, n, k,
                                  *extra, *scalars, shader_path(spv))
    return _dispatch(outs, rc)


def leapfrog_chain_normal(q, p, m, k, eps, mu, sigma):
    return _chain("nxv_leapfrog_chain_normal", "leapfrog_chain_normal.spv", q, p, m, k,
                  [eps, mu, sigma])


def leapfrog_chain_normal_lg(q, p, m, k, eps, mu, sigma):
    n = q.n_bytes // 4
    return _chain("nxv_leapfrog_chain_normal_lg", "leapfrog_chain_normal_lg.spv", q, p, m, k,
                  [eps, mu, sigma], partial_groups=(n + 255) // 256)


def leapfrog_chain_exponential(q, p, m, k, eps, lam):
    return _chain("nxv_leapfrog_chain_exponential", "leapfrog_chain_exponential.spv", q, p, m, k,
                  [eps, lam])


def leapfrog_chain_studentt(q, p, m, k, eps, mu, sigma, nu, logp_const):
    return _chain("nxv_leapfrog_chain_studentt", "leapfrog_chain_studentt.spv", q, p, m, k,
                  [eps, mu, sigma, nu, logp_const])


def leapfrog_chain_cauchy(q, p, m, k, eps, loc, scale, log_pi_scale):
    return _chain("nxv_leapfrog_chain_cauchy", "leapfrog_chain_cauchy.spv", q, p, m, k,
                  [eps, loc, scale, log_pi_scale])


def leapfrog_chain_halfnormal(q, p, m, k, eps, sigma, log_const):
    return _chain("nxv_leapfrog_chain_halfnormal", "leapfrog_chain_halfnormal.spv", q, p, m, k,
                  [eps, sigma, log_const])


def leapfrog_chain_weibull(q, p, m, k_steps, eps, weibull_k, lam, logp_const):
    return _chain("nxv_leapfrog_chain_weibull", "leapfrog_chain_weibull.spv", q, p, m, k_steps,
                  [eps, weibull_k, lam, logp_const])


def leapfrog_chain_normal_f64(q, p, m, k, eps, mu, sigma):
    return _chain("nxv_leapfrog_chain_normal_f64", "leapfrog_chain_normal_f64.spv", q, p, m, k,
                  [eps, mu, sigma], elt=8)


def leapfrog_chain_gauss_f64_batched(q, p, m, prec, n_chains, k, eps, mu=0.0, kinetic=False):
    """Batched anisotropic Gaussian chains: q, p are [chain][n] f64, m is
    [chain][n] or one [n] row broadcast over the chains, prec [n].
    Returns q, p, grad trajectories [chain][k][n] and logp [chain][k]; with
    kinetic=True also the kinetic energy 0.5 * sum(p^2 m) [chain][k]."""
    if q.n_bytes != p.n_bytes or k <= 0 or n_chains <= 0:
        return (ERROR, "size_mismatch" if k > 0 else "bad_op")
    n = q.n_bytes // 8 // n_chains
    if n * 8 * n_chains != q.n_bytes or prec.n_bytes != n * 8:
        return (ERROR, "size_mismatch")
    if m.n_bytes not in (q.n_bytes, n * 8):
        return (ERROR, "size_mismatch")
    outs = [_alloc(q.n_bytes * k), _alloc(q.n_bytes * k), _alloc(q.n_bytes * k),
            _alloc(n_chains * k * 8)]
    if kinetic:
        outs.append(_alloc(n_chains * k * 8))
    if any(o is None for o in outs):
        return (ERROR, "alloc_failed")
    spv = shader_path("leapfrog_chain_gauss_f64_batched.spv")
    if kinetic:
        rc = _lib().nxv_leapfrog_chain_gauss_f64_batched_ke(
            *(o.handle for o in outs), q.handle, p.handle, m.handle, prec.handle, n, n_chains, k,
            eps, mu, spv)
    else:
        rc = _lib().nxv_leapfrog_chain_gauss_f64_batched(
            *(o.handle for o in outs), q.handle, p.handle, m.handle, prec.handle, n, n_chains, k,
            eps, mu, spv)
    return _dispatch(outs, rc)


def leapfrog_logreg_f64_batched(q, p, X, y, n_obs, n_dim, n_chains, k, eps):
    if q.n_bytes != p.n_bytes or q.n_bytes != n_chains * n_dim * 8 or k <= 0:
        return (ERROR, "size_mismatch" if k > 0 else "bad_op")
    if X.n_bytes != n_obs * n_dim * 8 or y.n_bytes != n_obs * 8:
        return (ERROR, "size_mismatch")
    outs = [_alloc(q.n_bytes * k), _alloc(q.n_bytes * k), _alloc(q.n_bytes * k),
            _alloc(n_chains * k * 8)]
    if any(o is None for o in outs):
        return (ERROR, "alloc_failed")
    rc = _lib().nxv_leapfrog_logreg_f64_batched(
        *(o.handle for o in outs), q.handle, p.handle, X.handle, y.handle, n_obs, n_dim,
        n_chains, k, eps, shader_path("leapfrog_logreg_f64_batched.spv"))
    return _dispatch(outs, rc)


# ---- pool (lib/nx_vulkan.ex:844-867; lib.rs:1680-1703) ------------------------------------------

def pool_clear():
    _lib().nxv_pool_clear()
    return OK


def pool_stats():
    v = [C.c_ulong(0) for _ in range(5)]
    _lib().nxv_pool_stats(*(C.byref(x) for x in v))
    keys = ("hits", "misses", "freed", "size_classes", "total_pooled")
    return (OK, dict(zip(keys, (x.value for x in v))))


def synchronize():
    return OK if _lib().nxv_synchronize() == 0 else (ERROR, "dispatch_failed")


def launch_count() -> int:
    return int(_lib().nxv_launch_count())
