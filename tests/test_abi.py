"""CPU checks of the drop-in boundary: the CUDA library loads here (no GPU
needed to dlopen it) and exports every function that include/nx_vulkan_shim.h
declares, including every name of the reference's C ABI
(c_src/nx_vulkan_shim.h:20-280).  No compute calls: there is no GPU here."""
import ctypes
import re

import pytest

from conftest import GOLDEN, ROOT

HEADER = (ROOT / "include" / "nx_vulkan_shim.h").read_text()

# Every entry point of the reference's shim header (c_src/nx_vulkan_shim.h).
REFERENCE_ABI = [
    "nxv_init", "nxv_destroy", "nxv_device_name", "nxv_has_f64", "nxv_buf_alloc",
    "nxv_buf_free", "nxv_pool_clear", "nxv_pool_stats", "nxv_buf_upload", "nxv_buf_download",
    "nxv_apply_binary", "nxv_apply_unary", "nxv_reduce", "nxv_matmul", "nxv_matmul_v",
    "nxv_random", "nxv_transpose", "nxv_cast", "nxv_reduce_axis", "nxv_apply_binary_broadcast",
    "nxv_fused_chain", "nxv_fused_chain_4", "nxv_kinetic_energy", "nxv_normal_logpdf",
    "nxv_leapfrog_normal", "nxv_leapfrog_chain_normal", "nxv_leapfrog_chain_normal_lg",
    "nxv_leapfrog_chain_exponential", "nxv_leapfrog_chain_studentt", "nxv_leapfrog_chain_cauchy",
    "nxv_leapfrog_chain_halfnormal", "nxv_leapfrog_chain_weibull",
    "nxv_leapfrog_chain_normal_f64",
]


def declared():
    body = re.sub(r"/\*.*?\*/", "", HEADER, flags=re.S)
    return sorted(set(re.findall(r"\b(nxv_[a-z0-9_]+)\s*\(", body)))


@pytest.fixture(scope="module")
def lib():
    from nx_vulkan_b200 import build
    build.build()
    return ctypes.CDLL(str(build.LIB))


def test_header_declares_reference_abi():
    d = declared()
    for name in REFERENCE_ABI:
        assert name in d, name


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from nx_vulkan_b200 import _native
    assert sorted(_native.SIGNATURES) == declared()


def test_binding_loads_and_reports_no_device_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from nx_vulkan_b200 import vulkan
    # nxv_init returns non-zero without a device; the mirror maps it to :no_device
    assert vulkan.init() == ("error", "no_device")
    # every op refuses to run before init, with -5 (not initialised)
    from nx_vulkan_b200 import _native
    lib = _native.load()
    assert lib.nxv_buf_alloc(16) is None
    assert lib.nxv_apply_binary(None, None, None, 0, 0, b"elementwise_binary.spv") == -1


@pytest.mark.parametrize("case", GOLDEN["broadcast_strides"], ids=lambda c: str(c["src"]))
def test_broadcast_strides(case):
    from nx_vulkan_b200 import vulkan
    assert vulkan.broadcast_strides(tuple(case["src"]), tuple(case["out"])) == case["want"]


def test_broadcast_strides_rejects():
    from nx_vulkan_b200 import vulkan
    with pytest.raises(ValueError):
        vulkan.broadcast_strides((3,), (2, 4))


@pytest.mark.parametrize("case", GOLDEN["pick_matmul"], ids=lambda c: str(c["mnk"]))
def test_pick_matmul(case):
    from nx_vulkan_b200 import vulkan
    assert list(vulkan.pick_matmul(*case["mnk"])) == case["want"]


def test_unknown_fused_op_is_key_error():
    # test/nx_vulkan_test.exs:1042-1052: unknown op atoms fail before the NIF.
    from nx_vulkan_b200 import vulkan
    with pytest.raises(KeyError):
        vulkan.OP_CODES["not_a_real_op"]


def test_product_package_never_imports_the_oracle():
    """The oracle is test infrastructure: no module of the product package
    imports it (the CPU restatement is never one import away from the
    product path)."""
    pkg = ROOT / "nx_vulkan_b200"
    offenders = [p.name for p in pkg.rglob("*.py")
                 if re.search(r"^\s*(from|import)\s+oracle\b", p.read_text(), flags=re.M)]
    assert not offenders, offenders


def test_nuts_layout_entry_points_validate_before_any_device_work():
    """The device-driven NUTS calls reject a missing buffer (-1) and a level
    width that is not a power of two up to 2048 (-3) before touching a
    device (none exists here)."""
    from nx_vulkan_b200 import _native
    lib = _native.load()
    p = ctypes.c_void_p(16)  # never dereferenced on these paths
    bufs = [p] * 18
    assert lib.nxv_nuts_level_layout(0, 4, 8, None, *bufs[1:], 2, 0) == -1
    assert lib.nxv_nuts_level_layout(0, 3, 8, *bufs, 2, 1) == -3
    assert lib.nxv_nuts_level_layout(0, 4096, 8, *bufs, 2, 12) == -3
    assert lib.nxv_nuts_start_layout(None, p, p, p, p, p, p, p, 2, 8) == -1
    assert lib.nxv_nuts_transition_layout(p, None, p, p, p, p, 0.0, 0.0, 0.1, 2, 8, 4, 1) == -1
    assert lib.nxv_nuts_transition_layout(p, p, p, p, p, p, 0.0, 0.0, 0.1, 2, 8, 0, 1) == -3
    assert lib.nxv_nuts_transition_layout(p, p, p, p, p, p, 0.0, 0.0, 0.1, 2, 8, 13, 1) == -3
