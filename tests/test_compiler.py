"""The chain compiler (the reference's Nx.Vulkan.Compiler path): detection
and lowering are host logic and run on CPU; execution is gpu-marked."""
import numpy as np
import pytest

from nx_vulkan_b200.compiler import detect_chain, jit, nx, trace, Tensor


def lower(fun, arity):
    ch = detect_chain(trace(fun, arity), arity)
    return None if ch is None else (ch.start, ch.ops, ch.src, ch.imm, ch.operands)


def test_config1_chain_fuses_with_literal():
    # tanh(exp(x*y + z) - 1.0): one tape, the literal as an immediate
    f = lambda x, y, z: nx.tanh(nx.subtract(nx.exp(nx.add(nx.multiply(x, y), z)), 1.0))
    assert lower(f, 3) == (0, [1, 0, 100, 2, 106], [1, 2, 1, 0, 1], [0.0, 0.0, 0.0, 1.0, 0.0], [1, 2])


def test_reference_chains():
    # compiler.ex:1220-1309 shapes: fn(a, b) -> exp(a*b + b); fn(q, eps, p) -> q + eps*p
    assert lower(lambda a, b: nx.exp(nx.add(nx.multiply(a, b), b)), 2) == (0, [1, 0, 100], [1, 1, 1], [0, 0, 0], [1])
    # q + eps*p: the register starts at eps (commutative swaps), operands p then q
    st, ops, src, imm, operands = lower(lambda q, eps, p: nx.add(q, nx.multiply(eps, p)), 3)
    assert ops == [1, 0] and len(operands) == 2
    assert lower(lambda x: nx.sqrt(nx.abs(nx.negate(x))), 1) == (0, [104, 103, 102], [1, 1, 1], [0, 0, 0], [])


def test_left_literal_subtract_is_negated():
    st, ops, src, imm, _ = lower(lambda x: 1.0 - nx.exp(x), 1)
    assert ops == [100, 2, 104] and src[1] == 0 and imm[1] == 1.0


def test_non_chains_do_not_fuse():
    # two register paths (x*x appears on both sides) and division by the register
    assert lower(lambda x, y: nx.add(nx.exp(x), nx.log(x)), 2) is None
    assert lower(lambda x: 2.0 / x, 1) is None
    # more than 8 ops
    def long(x):
        for _ in range(9):
            x = nx.exp(x)
        return x
    assert lower(long, 1) is None


@pytest.mark.gpu
def test_jit_config1_one_launch(nxv, orc):
    from nx_vulkan_b200 import vulkan
    n = 1 << 20
    r = np.random.default_rng(0)
    x, y, z = (r.uniform(-1, 1, n).astype(np.float32) for _ in range(3))
    f = jit(lambda x, y, z: nx.tanh(nx.subtract(nx.exp(nx.add(nx.multiply(x, y), z)), 1.0)))
    tx, ty, tz = (Tensor.from_numpy(v) for v in (x, y, z))
    f(tx, ty, tz)
    before = vulkan.launch_count()
    out = f(tx, ty, tz).numpy()
    assert vulkan.launch_count() - before == 1
    want = orc.fused(x, [y, z], [1, 0, 100, 2, 106], [1, 2, 1, 0, 1], [0, 0, 0, 1.0, 0])
    assert np.max(np.abs(out - want) - (1e-5 * np.abs(want) + 1e-6)) <= 0


@pytest.mark.gpu
def test_jit_fallback_op_by_op(nxv, orc):
    from nx_vulkan_b200 import vulkan
    r = np.random.default_rng(1)
    x, y = r.uniform(0.5, 2, 1000), r.uniform(0.5, 2, 1000)
    f = jit(lambda x, y: nx.add(nx.exp(x), nx.log(nx.multiply(x, y))) - 2.0)
    before = vulkan.launch_count()
    out = f(Tensor.from_numpy(x), Tensor.from_numpy(y)).numpy()
    assert vulkan.launch_count() - before == 5  # exp, mul, log, add, -2.0
    assert np.allclose(out, np.exp(x) + np.log(x * y) - 2.0, rtol=1e-12, atol=1e-12)
