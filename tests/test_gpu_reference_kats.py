"""The reference test suite's known answers (test/nx_vulkan_test.exs), run
through the Nx.Vulkan mirror on the GPU.  Each test cites the reference
test it restates."""
import math
import threading

import numpy as np
import pytest

from conftest import GOLDEN, atoms_equal
from gpu_util import down, unwrap, up

pytestmark = pytest.mark.gpu

BIN_NAMES = {v: k for k, v in {"add": 0, "multiply": 1, "subtract": 2, "divide": 3, "pow": 4,
                               "max": 5, "min": 6, "equal": 7, "less": 8, "greater": 9}.items()}
UN_NAMES = {0: "exp", 1: "log", 2: "sqrt", 7: "relu", 13: "erf", 14: "expm1"}


def test_init_and_device(nxv):
    assert nxv.init() == "ok"
    assert "B200" in nxv.device_name() or nxv.device_name()
    assert nxv.has_f64() is True


def test_round_trip(nxv):
    t = unwrap(nxv.upload_f32([1.0, 2.0, 3.0, 4.0]))
    assert nxv.download_f32(t, 4) == ("ok", [1.0, 2.0, 3.0, 4.0])
    assert nxv.download_f32(t, 3) == ("error", "size_mismatch")


@pytest.mark.parametrize("case", GOLDEN["binary_f32"], ids=lambda c: c["cite"])
def test_binary(nxv, case):
    a = unwrap(nxv.upload_f32(case["a"]))
    b = unwrap(nxv.upload_f32(case["b"]))
    c = unwrap(getattr(nxv, BIN_NAMES[case["op"]])(a, b))
    got = unwrap(nxv.download_f32(c, len(case["a"])))
    atoms_equal(got, case["want"], case["tol"])


def test_size_mismatch(nxv):
    # test/nx_vulkan_test.exs:156-160
    a = unwrap(nxv.upload_f32([1.0, 2.0]))
    b = unwrap(nxv.upload_f32([1.0, 2.0, 3.0]))
    assert nxv.add(a, b) == ("error", "size_mismatch")


def test_chained(nxv):
    c = GOLDEN["chained_f32"][0]
    a, b = unwrap(nxv.upload_f32(c["a"])), unwrap(nxv.upload_f32(c["b"]))
    d = unwrap(nxv.multiply(unwrap(nxv.add(a, b)), a))
    assert unwrap(nxv.download_f32(d, 3)) == c["want"]


def test_1024_elements(nxv):
    # test/nx_vulkan_test.exs:171-179
    x = [float(i) for i in range(1, 1025)]
    a, b = unwrap(nxv.upload_f32(x)), unwrap(nxv.upload_f32(x))
    r = unwrap(nxv.download_f32(unwrap(nxv.add(a, b)), 1024))
    assert r[0] == 2.0 and r[-1] == 2048.0


@pytest.mark.parametrize("case", GOLDEN["unary_f32"], ids=lambda c: c["cite"])
def test_unary(nxv, case):
    a = unwrap(nxv.upload_f32(case["a"]))
    c = unwrap(getattr(nxv, UN_NAMES[case["op"]])(a))
    atoms_equal(unwrap(nxv.download_f32(c, len(case["a"]))), case["want"], case["tol"])


def test_f64_ops(nxv):
    c = GOLDEN["binary_f64"][0]
    a, b = unwrap(nxv.upload_f64(c["a"])), unwrap(nxv.upload_f64(c["b"]))
    assert unwrap(nxv.download_f64(unwrap(nxv.apply_binary_f64(a, b, "add")), 3)) == c["want"]
    c = GOLDEN["unary_f64"][0]
    a = unwrap(nxv.upload_f64(c["a"]))
    assert unwrap(nxv.download_f64(unwrap(nxv.apply_unary_f64(a, "sqrt")), 3)) == c["want"]
    c = GOLDEN["f64_precision"][0]
    a = unwrap(nxv.upload_f64(c["a"]))
    s = unwrap(nxv.download_f64(unwrap(nxv.apply_binary_f64(a, a, "add")), 2))[0]
    assert c["lo"] < s < c["hi"]


@pytest.mark.parametrize("case", GOLDEN["reduce_full_f32"], ids=lambda c: c["cite"])
def test_reduce_full(nxv, case):
    a = unwrap(nxv.upload_f32(case["a"]))
    fn = {0: nxv.sum, 1: nxv.reduce_min, 2: nxv.reduce_max}[case["op"]]
    assert fn(a) == ("ok", case["want"])


def test_mean(nxv):
    c = GOLDEN["mean_f32"][0]
    assert nxv.mean(unwrap(nxv.upload_f32(c["a"]))) == ("ok", c["want"])


@pytest.mark.parametrize("case", GOLDEN["reduce_axis_f32"], ids=lambda c: c["cite"])
def test_reduce_axis(nxv, case):
    a = unwrap(nxv.upload_f32(case["a"]))
    out = unwrap(nxv.reduce_axis(a, case["outer"], case["R"], case["inner"], case["op"]))
    assert unwrap(nxv.download_f32(out, case["outer"] * case["inner"])) == case["want"]


@pytest.mark.parametrize("case", GOLDEN["matmul_f32"], ids=lambda c: c["cite"])
def test_matmul(nxv, case):
    a, b = unwrap(nxv.upload_f32(case["a"])), unwrap(nxv.upload_f32(case["b"]))
    c = unwrap(nxv.matmul(a, b, case["m"], case["n"], case["k"]))
    got = unwrap(nxv.download_f32(c, case["m"] * case["n"]))
    assert all(abs(g - w) < 1e-5 for g, w in zip(got, case["want"]))


def test_matmul_variants(nxv):
    # test/nx_vulkan_test.exs:1065-1076: every variant gives the same product
    a = unwrap(nxv.upload_f32([1.0, 2.0, 3.0, 4.0]))
    b = unwrap(nxv.upload_f32([5.0, 6.0, 7.0, 8.0]))
    for v in ["matmul", "matmul_tiled", "matmul_tiled16x2"]:
        c = unwrap(nxv.matmul_variant(a, b, 2, 2, 2, v))
        assert unwrap(nxv.download_f32(c, 4)) == [19.0, 22.0, 43.0, 50.0]


def test_uniform_determinism_and_range(nxv):
    r1, r2 = unwrap(nxv.uniform(8, 42)), unwrap(nxv.uniform(8, 42))
    l1, l2 = unwrap(nxv.download_f32(r1, 8)), unwrap(nxv.download_f32(r2, 8))
    assert l1 == l2 and all(0.0 <= x < 1.0 for x in l1)
    assert nxv.download_f32(unwrap(nxv.uniform(8, 1)), 8) != nxv.download_f32(unwrap(nxv.uniform(8, 2)), 8)


def test_concurrent_threads(nxv):
    # test/nx_vulkan_test.exs:309-331 (20 concurrent tasks x 5 iterations)
    inputs = [i / 1.0 for i in range(1, 257)]
    heads, errs = [], []

    def task():
        try:
            for _ in range(5):
                a, b = unwrap(nxv.upload_f32(inputs)), unwrap(nxv.upload_f32(inputs))
                heads.append(unwrap(nxv.download_f32(unwrap(nxv.add(a, b)), 256))[0])
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ts = [threading.Thread(target=task) for _ in range(20)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert not errs and len(heads) == 100 and all(h == 2.0 for h in heads)


def test_5000_alloc_free_cycles(nxv):
    # test/nx_vulkan_test.exs:352-363
    for _ in range(5000):
        unwrap(nxv.upload_f32([42.0]))
    t = unwrap(nxv.upload_f32([1.0, 2.0, 3.0]))
    assert nxv.download_f32(t, 3) == ("ok", [1.0, 2.0, 3.0])


def test_select_and_clip(nxv):
    # test/nx_vulkan_test.exs:393-412
    cond = unwrap(nxv.upload_f32([1.0, 0.0, 1.0, 0.0]))
    t = unwrap(nxv.upload_f32([10.0, 20.0, 30.0, 40.0]))
    f = unwrap(nxv.upload_f32([100.0, 200.0, 300.0, 400.0]))
    assert nxv.download_f32(unwrap(nxv.select(cond, t, f)), 4) == ("ok", [10.0, 200.0, 30.0, 400.0])
    a = unwrap(nxv.upload_f32([-2.0, -0.5, 0.0, 1.5, 3.0, 7.0]))
    assert nxv.download_f32(unwrap(nxv.clip(a, 0.0, 5.0)), 6) == ("ok", [0.0, 0.0, 0.0, 1.5, 3.0, 5.0])
    a = unwrap(nxv.upload_f32([1.0, 2.0, 3.0]))
    assert nxv.download_f32(unwrap(nxv.clip(a, -10.0, 10.0)), 3) == ("ok", [1.0, 2.0, 3.0])


@pytest.mark.parametrize("case", GOLDEN["cast"], ids=lambda c: c["cite"] + c["dir"])
def test_cast(nxv, case):
    if case["dir"] == "f32_to_f64":
        a = unwrap(nxv.upload_f32(case["a"]))
        got = unwrap(nxv.download_f64(unwrap(nxv.cast_f32_to_f64(a, len(case["a"]))), len(case["a"])))
    else:
        a = unwrap(nxv.upload_f64(case["a"]))
        got = unwrap(nxv.download_f32(unwrap(nxv.cast_f64_to_f32(a, len(case["a"]))), len(case["a"])))
    assert got == case["want"]


def test_pool(nxv):
    # test/nx_vulkan_test.exs:1095-1136
    nxv.pool_clear()
    s0 = unwrap(nxv.pool_stats())
    t1 = unwrap(nxv.upload_f32([1.0, 2.0, 3.0, 4.0]))
    del t1
    unwrap(nxv.upload_f32([9.0, 10.0, 11.0, 12.0]))
    s1 = unwrap(nxv.pool_stats())
    assert s1["misses"] + s1["hits"] >= s0["misses"] + s0["hits"] + 2
    assert s1["hits"] >= s0["hits"] + 1  # the freed 16-byte buffer was reused
    for _ in range(5):
        unwrap(nxv.upload_f32([0.0, 0.0]))
    nxv.pool_clear()
    s = unwrap(nxv.pool_stats())
    assert s["total_pooled"] == 0 and s["size_classes"] == 0


@pytest.mark.parametrize("case", GOLDEN["broadcast_f32"], ids=lambda c: c["cite"])
def test_broadcast(nxv, case):
    a, b = unwrap(nxv.upload_f32(case["a"])), unwrap(nxv.upload_f32(case["b"]))
    name = BIN_NAMES[case["op"]]
    out = unwrap(nxv.apply_binary_broadcast(a, b, name, case["ndim"], case["shape"], case["as"], case["bs"]))
    assert unwrap(nxv.download_f32(out, len(case["want"]))) == case["want"]


NAMES = {0: "add", 1: "multiply", 2: "subtract", 3: "divide", 100: "exp", 101: "log",
         102: "sqrt", 112: "square", 113: "erf", 114: "expm1"}


@pytest.mark.parametrize("case", GOLDEN["fused_chain_f32"], ids=lambda c: c["cite"])
def test_fused_chain(nxv, case):
    a, b = unwrap(nxv.upload_f32(case["a"])), unwrap(nxv.upload_f32(case["b"]))
    out = unwrap(nxv.fused_chain(a, b, [NAMES[o] for o in case["ops"]]))
    got = unwrap(nxv.download_f32(out, len(case["a"])))
    assert all(abs(g - w) <= case["tol"] for g, w in zip(got, case["want"]))


def test_fused_chain_rejects(nxv):
    a, b = unwrap(nxv.upload_f32([1.0, 2.0])), unwrap(nxv.upload_f32([1.0, 1.0]))
    with pytest.raises(KeyError):
        nxv.fused_chain(a, b, ["not_a_real_op"])
    assert nxv.fused_chain(a, b, []) == ("error", "bad_op")


@pytest.mark.parametrize("case", GOLDEN["fused_chain_4_f32"], ids=lambda c: c["cite"])
def test_fused_chain_4(nxv, case):
    t = [unwrap(nxv.upload_f32(case[k])) for k in "abcd"]
    ops = [(NAMES[o], i) if o < 100 else NAMES[o] for o, i in zip(case["ops"], case["idx"])]
    out = unwrap(nxv.fused_chain_4(*t, ops))
    got = unwrap(nxv.download_f32(out, len(case["a"])))
    assert all(abs(g - w) <= case["tol"] for g, w in zip(got, case["want"]))


@pytest.mark.parametrize("case", GOLDEN["kinetic_energy_f32"], ids=lambda c: c["cite"])
def test_kinetic_energy(nxv, case):
    p, m = unwrap(nxv.upload_f32(case["p"])), unwrap(nxv.upload_f32(case["m"]))
    parts = unwrap(nxv.download_f32(unwrap(nxv.kinetic_energy(p, m)), 1))
    assert abs(sum(parts) - case["want"]) <= case["tol"]


def test_normal_logpdf(nxv):
    c = GOLDEN["normal_logpdf_f32"][0]
    t = [unwrap(nxv.upload_f32(c[k])) for k in ("x", "mu", "sigma")]
    got = unwrap(nxv.download_f32(unwrap(nxv.normal_logpdf(*t)), 3))
    assert all(abs(g - w) <= c["tol"] for g, w in zip(got, c["want"]))


def test_weibull_chain_kat(nxv):
    c = GOLDEN["leapfrog_chain_kat"][0]
    n = c["n"]
    q = unwrap(nxv.upload_f32([c["q0"]] * n))
    p = unwrap(nxv.upload_f32([c["p0"]] * n))
    m = unwrap(nxv.upload_f32([c["m"]] * n))
    qc, pc, gc, lc = unwrap(nxv.leapfrog_chain_weibull(q, p, m, c["K"], c["eps"], *c["prm"]))
    assert abs(unwrap(nxv.download_f32(qc, n))[0] - c["want_q0"]) <= c["tol"]
    assert abs(unwrap(nxv.download_f32(pc, n))[0] - c["want_p0"]) <= c["tol"]
    assert abs(unwrap(nxv.download_f32(lc, 1))[0] - c["want_logp0"]) <= c["tol"]


def test_chain_rejects_k0_and_size_mismatch(nxv):
    q = unwrap(nxv.upload_f32([0.0] * 4))
    p3 = unwrap(nxv.upload_f32([0.0] * 3))
    assert nxv.leapfrog_chain_normal(q, q, q, 0, 0.1, 0.0, 1.0) == ("error", "bad_op")
    assert nxv.leapfrog_chain_normal(q, p3, q, 4, 0.1, 0.0, 1.0) == ("error", "size_mismatch")


def test_ieee_specials_round_trip(nxv):
    # test/nx_vulkan_test.exs:1755-1773
    import struct
    t = unwrap(nxv.upload_binary(struct.pack("<3I", 0x7F800000, 0xFF800000, 0x7FC00000)))
    assert unwrap(nxv.download_f32(t, 3)) == ["infinity", "neg_infinity", "nan"]
