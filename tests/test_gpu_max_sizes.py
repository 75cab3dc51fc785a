"""Maximum sizes: element counts past 2^31 and 2^32 (the reference passes
counts as u32 push constants, so 2^32 - 1 elements is its largest call),
run through the C ABI on device memory owned by torch (nxv_buf_wrap) and
checked on the device with size-independent properties: IEEE-exact ops
against the same op in torch on the same data, max/min/argmax exactly, sums
against a float64 torch sum within the sum tolerance.  Inputs come from the
library's own Philox generator.  About 26-43 GB of device memory per test,
released after it."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

N31 = (1 << 31) + 7   # f32 elements past the signed 32-bit range


@pytest.fixture(scope="module")
def lib(nxv):
    from nx_vulkan_b200 import _native
    return _native.load()


def need_gb(gb):
    free, _ = torch.cuda.mem_get_info()
    if free < gb * 1e9:
        pytest.skip(f"needs {gb} GB of free device memory, {free / 1e9:.0f} GB free")


class Wrapped:
    """nxv handles over torch tensors, released (records only) on exit."""

    def __init__(self, lib):
        self.lib, self.handles = lib, []

    def __call__(self, t):
        h = self.lib.nxv_buf_wrap(C.c_void_p(t.data_ptr()), t.numel() * t.element_size())
        assert h
        self.handles.append(h)
        return h

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        for h in self.handles:
            self.lib.nxv_buf_free(h)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def sp(nxv, name):
    return nxv.shader_path(name)


def test_binary_and_full_reduce_past_2_31(nxv, lib):
    need_gb(45)
    a = torch.empty(N31, dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    out = torch.empty_like(a)
    torch.cuda.synchronize()
    with Wrapped(lib) as w:
        ha, hb, ho = w(a), w(b), w(out)
        assert lib.nxv_random(ha, N31, 11, 0, sp(nxv, "random_philox.spv")) == 0
        assert lib.nxv_random(hb, N31, 12, 1, sp(nxv, "random_philox.spv")) == 0
        assert lib.nxv_apply_binary(ho, ha, hb, N31, 0, sp(nxv, "elementwise_binary.spv")) == 0
        assert lib.nxv_apply_binary(ho, ho, ha, N31, 1, sp(nxv, "elementwise_binary.spv")) == 0
        assert lib.nxv_synchronize() == 0
        assert torch.equal(out, (a + b) * a)  # IEEE add and mul, bit for bit
        assert bool((a[-8:] != 0).any())       # the generator reached the last elements
        # full reduce: sum (f64 accumulation, one rounding), min, max
        v = C.c_float()
        assert lib.nxv_reduce(C.byref(v), ha, N31, 0, sp(nxv, "reduce.spv")) == 0
        want = torch.sum(a, dtype=torch.float64).item()
        assert abs(v.value - want) <= 1e-5 * abs(want) + 1e-6
        for op, fn in ((1, torch.min), (2, torch.max)):
            assert lib.nxv_reduce(C.byref(v), hb, N31, op, sp(nxv, "reduce.spv")) == 0
            assert v.value == fn(b).item()
    del a, b, out


def test_argmax_at_the_largest_axis(nxv, lib):
    """argmax over R = 2^31 - 1 (the largest axis it accepts): a planted
    maximum near the end, tied once after it -- the lower index wins."""
    need_gb(10)
    R = (1 << 31) - 1
    x = torch.empty(R, dtype=torch.float32, device="cuda")
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    with Wrapped(lib) as w:
        hx, ho = w(x), w(out)
        assert lib.nxv_random(hx, R, 5, 0, sp(nxv, "random_philox.spv")) == 0
        assert lib.nxv_synchronize() == 0  # the library's stream is not torch's
        x[R - 5] = 2.0
        x[R - 3] = 2.0
        x[7] = -1.0
        torch.cuda.synchronize()
        assert lib.nxv_argmax_axis(ho, hx, 1, R, 1, 0, 0, 8, sp(nxv, "argmax_axis.spv")) == 0
        assert lib.nxv_synchronize() == 0
        assert out[0].item() == R - 5
        assert lib.nxv_argmax_axis(ho, hx, 1, R, 1, 1, 0, 8, sp(nxv, "argmax_axis.spv")) == 0
        assert lib.nxv_synchronize() == 0
        assert out[0].item() == 7
        # one past the largest axis is refused, not truncated
        assert lib.nxv_argmax_axis(ho, hx, 1, R + 1, 1, 0, 0, 8, sp(nxv, "argmax_axis.spv")) != 0
    del x, out


def test_f64_sum_past_2_31(nxv, lib):
    """Double-double f64 sum over 2^31 + 3 elements against torch's float64 sum
    (whose own error is ~log2(n) eps |sum|)."""
    need_gb(19)
    n = (1 << 31) + 3
    x = torch.empty(n, dtype=torch.float64, device="cuda")
    with Wrapped(lib) as w:
        hx = w(x)
        assert lib.nxv_random_f64(hx, n, 21, 1, sp(nxv, "random_philox_f64.spv")) == 0
        v = C.c_double()
        assert lib.nxv_reduce_f64(C.byref(v), hx, n, 0, sp(nxv, "reduce_full_f64.spv")) == 0
        want = torch.sum(x).item()
        absum = torch.sum(x.abs()).item()
        assert abs(v.value - want) <= 1e-12 * abs(want) + 64 * 2.2e-16 * absum
        assert lib.nxv_reduce_f64(C.byref(v), hx, n, 2, sp(nxv, "reduce_full_f64.spv")) == 0
        assert v.value == torch.max(x).item()
    del x


def test_broadcast_output_past_2_32(nxv, lib):
    """out [2, 2^31 + 1] = a [2, 1] + b [2^31 + 1]: 2^32 + 2 output elements,
    past the 32-bit index path of the broadcast kernels."""
    need_gb(45)
    L = (1 << 31) + 1
    a = torch.tensor([[0.5], [-3.0]], dtype=torch.float32, device="cuda")
    b = torch.empty(L, dtype=torch.float32, device="cuda")
    out = torch.empty((2, L), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()  # a is written on torch's stream
    with Wrapped(lib) as w:
        ha, hb, ho = w(a), w(b), w(out)
        assert lib.nxv_random(hb, L, 9, 1, sp(nxv, "random_philox.spv")) == 0
        shape = (C.c_uint * 4)(2, L, 0, 0)
        sa = (C.c_uint * 4)(1, 0, 0, 0)
        sb = (C.c_uint * 4)(0, 1, 0, 0)
        assert lib.nxv_apply_binary_broadcast(ho, ha, hb, 0, 2, shape, sa, sb,
                                              sp(nxv, "elementwise_binary_broadcast.spv")) == 0
        assert lib.nxv_synchronize() == 0
        assert torch.equal(out[0], b + 0.5)
        assert torch.equal(out[1], b - 3.0)
    del a, b, out
