"""CUDA path vs the CPU oracle on identical seeded inputs.

Tolerances (written per assertion): bit-exact for integer/index work and for
IEEE-exact ops (+ - * / sqrt, compare, max/min, abs, neg, ceil, floor, sign,
relu, square, reciprocal, casts, transposes, uniform Philox); f32
transcendentals within 1e-5 relative + 1e-6 absolute; f64 within 1e-12
relative (+1e-14 absolute for results near zero)."""
import numpy as np
import pytest

from gpu_util import chain_error_bound, close, close_bound, down, ulp_diff, unwrap, up

pytestmark = pytest.mark.gpu

SIZES = [1, 3, 4, 255, 256, 257, 1000, 4097, 65536 + 3]
EXACT_BIN = [0, 1, 2, 3, 5, 6, 7, 8, 9]
EXACT_UN = [2, 3, 4, 7, 8, 9, 10, 11, 12]
TRANS_UN = [0, 1, 5, 6, 13, 14]


def data(seed, n, dtype, lo=-2.0, hi=2.0):
    return np.random.default_rng(seed).uniform(lo, hi, n).astype(dtype)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_binary_all_ops(nxv, orc, n, dt):
    a, b = data(1, n, dt), data(2, n, dt)
    b[::7] = a[::7]  # exercise equal / ties of max-min
    spv = nxv.shader_path("elementwise_binary.spv" if dt == np.float32 else "elementwise_binary_f64.spv")
    ta, tb = up(nxv, a), up(nxv, b)
    for op in range(10):
        got = down(nxv, unwrap(nxv.apply_binary(ta, tb, op, spv, a.itemsize, 9)), dt)
        want = orc.binary(a, b, op)
        if op in EXACT_BIN:
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)) or np.array_equal(got, want), op
        else:  # pow
            pa = np.abs(a) + 0.1
            got = down(nxv, unwrap(nxv.apply_binary(up(nxv, pa), tb, op, spv, a.itemsize, 9)), dt)
            want = orc.binary(pa, b, op)
            if dt == np.float32:
                close_bound(got, want, chain_error_bound(pa, [b], [4], dtype=np.float32))
            else:
                close(got, want, 1e-12, 1e-14)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_unary_all_ops(nxv, orc, n, dt):
    a = data(3, n, dt, -3, 3)
    a[:1] = 0.0
    spv = nxv.shader_path("elementwise_unary.spv" if dt == np.float32 else "elementwise_unary_f64.spv")
    ta = up(nxv, a)
    for op in range(15):
        src = np.abs(a) + 0.01 if op in (1, 2) else a
        t = ta if src is a else up(nxv, src)
        got = down(nxv, unwrap(nxv.apply_unary(t, op, spv, a.itemsize)), dt)
        want = orc.unary(src, op)
        if op in EXACT_UN:
            assert np.array_equal(got, want), op
        elif dt == np.float32:
            close_bound(got, want, chain_error_bound(src, [], [100 + op]))
        else:
            close(got, want, 1e-12, 1e-14)


def test_unary_specials(nxv, orc):
    a = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 1e-40, -1e-40, 88.0, -104.0], np.float32)
    spv = nxv.shader_path("elementwise_unary.spv")
    ta = up(nxv, a)
    for op in range(15):
        got = down(nxv, unwrap(nxv.apply_unary(ta, op, spv, 4)), np.float32)
        close_bound(got, orc.unary(a, op), chain_error_bound(a, [], [100 + op]))


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_broadcast_shapes(nxv, orc, dt):
    r = np.random.default_rng(5)
    cases = [((3, 5), (5,)), ((3, 5), (3, 1)), ((2, 3, 4), (3, 1)), ((2, 1, 4, 3), (5, 1, 1)),
             ((4, 8), (1, 8)), ((7,), ()), ((64, 256), (256,)), ((3, 1, 5), (1, 4, 1)),
             # vector path with 32-bit index decoding: large and odd outer dims,
             # broadcast on either side and on middle dims
             ((3, 70001, 4), (70001, 1)), ((8,), (6, 8)), ((2, 3, 5, 8), (3, 1, 8)),
             ((1000, 12), (1000, 1)), ((5, 131072), (5, 1)), ((6, 1, 16), (7, 1)),
             # row path: innermost extent of >= 64 vectors, several chunks per row
             ((3, 4, 512), (4, 1)), ((2, 3, 5, 1024), (3, 1, 1024)), ((7, 1032), (1032,)),
             ((2, 4100), (4100,)), ((1, 2048), (9, 2048)), ((3, 1, 8192), (5, 1))]
    spv = nxv.shader_path("elementwise_binary_broadcast.spv" if dt == np.float32
                          else "elementwise_binary_broadcast_f64.spv")
    for sa, sb in cases:
        out = np.broadcast_shapes(sa, sb)
        a, b = r.normal(size=sa).astype(dt), r.normal(size=sb).astype(dt)
        ast, bst = nxv.broadcast_strides(sa, out), nxv.broadcast_strides(sb, out)
        for op in (0, 1, 2, 3, 5, 8):
            t = unwrap(nxv._broadcast(up(nxv, a.reshape(-1) if a.size else a), up(nxv, b.reshape(-1)),
                                      op, len(out), nxv._pad4(out), ast, bst, spv, a.itemsize))
            got = down(nxv, t, dt)
            want = orc.broadcast(a.reshape(-1), b.reshape(-1), op, len(out), list(out), ast, bst)
            assert np.array_equal(got, want), (sa, sb, op)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_broadcast_rows_all_ops(nxv, orc, dt):
    """Every binary op on the row path (one kernel instantiation per op)."""
    r = np.random.default_rng(6)
    a = np.abs(r.normal(size=(33, 1536))).astype(dt) + 0.5
    b = r.normal(size=(1536,)).astype(dt)
    b[::7] = a[0, ::7]   # some equal pairs for the comparisons
    out = (33, 1536)
    ast, bst = nxv.broadcast_strides(a.shape, out), nxv.broadcast_strides(b.shape, out)
    spv = nxv.shader_path("elementwise_binary_broadcast.spv" if dt == np.float32
                          else "elementwise_binary_broadcast_f64.spv")
    for op in range(10):
        t = unwrap(nxv._broadcast(up(nxv, a.reshape(-1)), up(nxv, b), op, 2, nxv._pad4(out), ast, bst,
                                  spv, a.itemsize))
        got = down(nxv, t, dt)
        want = orc.broadcast(a.reshape(-1), b, op, 2, list(out), ast, bst)
        if op == 4:   # pow: f64 evaluation rounded once on both sides
            close(got, want, 1e-6 if dt == np.float32 else 1e-14, 0.0)
        else:
            assert np.array_equal(got, want), op


def test_broadcast_config_rows(nxv, orc):
    """x f32/f64[4096,4096] + b[4096] along rows (the reductions+broadcast workload)."""
    for dt in (np.float32, np.float64):
        r = np.random.default_rng(1)
        x = r.normal(size=(4096, 4096)).astype(dt)
        b = r.normal(size=4096).astype(dt)
        spv = "elementwise_binary_broadcast.spv" if dt == np.float32 else "elementwise_binary_broadcast_f64.spv"
        t = unwrap(nxv._broadcast(up(nxv, x), up(nxv, b), 0, 2, [4096, 4096, 0, 0], [4096, 1, 0, 0],
                                  [0, 1, 0, 0], nxv.shader_path(spv), x.itemsize))
        assert np.array_equal(down(nxv, t, dt).reshape(4096, 4096), x + b)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_fused_chain_config1(nxv, orc, dt):
    """tanh(exp(x*y + z) - 1.0) on [1,048,576] ~ U(-1,1), seed 0, one kernel.

    f32: 1e-5 relative + 1e-6 absolute.  f64: exp(u) - 1 cancels near u = 0,
    so the bound is 1e-12 relative to the largest intermediate, 2 + |e^u|."""
    n = 1 << 20
    r = np.random.default_rng(0)
    x, y, z = (r.uniform(-1, 1, n).astype(dt) for _ in range(3))
    ops, src, imm = [1, 0, 100, 2, 106], [1, 2, 1, 0, 1], [0, 0, 0, 1.0, 0]
    t = unwrap(nxv.fused_chain_imm(up(nxv, x), [up(nxv, y), up(nxv, z)],
                                   [("multiply", 1), ("add", 2), "exp", ("subtract", ("imm", 1.0)), "tanh"],
                                   dtype="f32" if dt == np.float32 else "f64"))
    got = down(nxv, t, dt)
    want = orc.fused(x, [y, z], ops, src, imm)
    if dt == np.float32:
        close(got, want, 1e-5, 1e-6)  # well conditioned: the flat tolerance holds
        close_bound(got, want, chain_error_bound(x, [y, z], ops, src, imm))
    else:
        scale = 2.0 + np.exp(x.astype(np.float64) * y + z)
        assert np.all(np.abs(got - want) <= 1e-12 * np.maximum(np.abs(want), scale))


@pytest.mark.parametrize("n", [1, 5, 1000, 100003])
def test_fused_generic_tapes(nxv, orc, n):
    r = np.random.default_rng(9)
    a, b, c, d = (r.uniform(0.1, 2, n).astype(np.float32) for _ in range(4))
    tapes = [
        ([0, 1, 2, 3, 112, 100, 101, 102], [1, 1, 1, 1, 1, 1, 1, 1]),
        ([103, 105, 1, 2, 106], [1, 1, 2, 3, 1]),
        ([1, 0], [1, 2]),
        ([1, 1, 0], [1, 2, 3]),
        ([110, 107, 108, 109, 104, 111, 0], [1, 1, 1, 1, 1, 1, 3]),
        ([5, 6, 4], [2, 3, 1]),
    ]
    ta, tb, tc, td = (up(nxv, v) for v in (a, b, c, d))
    names = {0: "add", 1: "multiply", 2: "subtract", 3: "divide", 4: "pow", 5: "max", 6: "min"}
    unames = {v: k for k, v in nxv.OP_CODES.items() if v >= 100}
    for ops, src in tapes:
        items = [(names[o], s) if o < 100 else unames[o] for o, s in zip(ops, src)]
        got = down(nxv, unwrap(nxv.fused_chain_imm(ta, [tb, tc, td], items)), np.float32)
        close_bound(got, orc.fused(a, [b, c, d], ops, src), chain_error_bound(a, [b, c, d], ops, src))


@pytest.mark.parametrize("shape", [(1, 1, 1), (1, 16777216, 1), (4096, 4096, 1), (1, 4096, 4096),
                                   (3, 1000, 7), (2, 5, 100003), (100003, 3, 1), (1, 257, 1),
                                   (70000, 2, 1), (7, 3, 1)])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_reduce_axis_and_full(nxv, orc, shape, dt):
    outer, R, inner = shape
    if outer * R * inner > 16777216 and dt == np.float64 and shape != (4096, 4096, 1):
        pytest.skip("size")
    x = np.random.default_rng(1).normal(size=outer * R * inner).astype(dt)
    t = up(nxv, x)
    spv = "reduce_axis.spv" if dt == np.float32 else "reduce_axis_f64.spv"
    for op in (0, 1, 2):
        got = down(nxv, unwrap(nxv._reduce_axis(t, outer, R, inner, op, nxv.shader_path(spv), x.itemsize)), dt)
        want = orc.reduce_axis(x, outer, R, inner, op)
        if op == 0:
            if dt == np.float32:
                close(got, want, 1e-5, 1e-6)
            else:  # |got - seq| <= 1e-12 |seq| + 4 eps sum|x| (tree vs sequential order)
                xs = np.abs(x.reshape(outer, R, inner)).sum(axis=1).reshape(-1)
                assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want) + 4 * 2.2e-16 * xs)
        else:
            assert np.array_equal(got, want)
    if inner == 1 and outer == 1:
        if dt == np.float32:
            for op in (0, 1, 2):
                g = {0: nxv.sum, 1: nxv.reduce_min, 2: nxv.reduce_max}[op](t)[1]
                w = orc.reduce_full(x, op)
                assert abs(g - w) <= 1e-5 * abs(w) + 1e-6 if op == 0 else g == w
        else:
            for op in (0, 1, 2):
                g = unwrap(nxv.reduce_f64(t, op))
                w = orc.reduce_full(x, op)
                if op == 0:
                    exact = orc.sum_exact(x)
                    assert abs(g - exact) <= 1e-12 * abs(exact) + 1e-15 * orc.sum_abs(x)
                    assert abs(g - w) <= 1e-12 * abs(w) + 4 * 2.2e-16 * orc.sum_abs(x)
                else:
                    assert g == w


@pytest.mark.parametrize("shape", [(4096, 4096, 1), (1, 16777216, 1), (3, 1000, 7), (1, 1, 1),
                                   (5, 4097, 3), (100003, 2, 1)])
@pytest.mark.parametrize("dt", [np.float32, np.float64])
def test_argmax_bit_exact(nxv, orc, shape, dt):
    outer, R, inner = shape
    r = np.random.default_rng(1)
    x = r.normal(size=outer * R * inner).astype(dt)
    x[:: 97] = np.round(x[:: 97])  # plant ties
    t = up(nxv, x)
    for is_min in (False, True):
        for ib in (8, 4):
            got = down(nxv, unwrap(nxv.argmax_axis(t, outer, R, inner, dtype="f32" if dt == np.float32 else "f64",
                                                   is_min=is_min, index_bytes=ib)),
                       np.int64 if ib == 8 else np.int32)
            want = orc.argmax_axis(x, outer, R, inner, is_min)
            assert np.array_equal(got.astype(np.int64), want)


@pytest.mark.parametrize("g", ["2", "4", "8"])
def test_row_kernels_all_cta_sizes(nxv, orc, monkeypatch, g):
    """The row kernels (>= 296 rows; one warp per row) with 2, 4 and 8 rows per
    CTA: max, min and argmax bit-exact, sums and logsumexp within their
    tolerances; rows of aligned and unaligned starts, shorter than one warp
    chunk, and long; row counts that leave the last CTA partly empty."""
    monkeypatch.setenv("NXV_ROW_CTA", g)
    for outer, R in ((300, 4096), (1001, 7), (5001, 1001), (333, 10003)):
        for dt in (np.float32, np.float64):
            x = np.random.default_rng(8).normal(size=outer * R).astype(dt)
            x[::53] = np.round(x[::53])
            t = up(nxv, x)
            spv = nxv.shader_path("reduce_axis.spv" if dt == np.float32 else "reduce_axis_f64.spv")
            for op in (0, 1, 2):
                got = down(nxv, unwrap(nxv._reduce_axis(t, outer, R, 1, op, spv, x.itemsize)), dt)
                want = orc.reduce_axis(x, outer, R, 1, op)
                if op == 0:
                    xs = np.abs(x.reshape(outer, R)).astype(np.float64).sum(axis=1)
                    tol = 1e-5 * np.abs(want) + 1e-6 if dt == np.float32 else 1e-12 * np.abs(want) + 4 * 2.2e-16 * xs
                    assert np.all(np.abs(got - want) <= tol)
                else:
                    assert np.array_equal(got, want)
            dts = "f32" if dt == np.float32 else "f64"
            got = down(nxv, unwrap(nxv.argmax_axis(t, outer, R, 1, dtype=dts)), np.int64)
            assert np.array_equal(got, orc.argmax_axis(x, outer, R, 1, False))
            if dt == np.float32:
                got = down(nxv, unwrap(nxv.logsumexp(t, outer, R, 1)), np.float32)
                close(got, orc.logsumexp(x, outer, R, 1), 1e-5, 1e-6)


def test_argmax_ties_and_nan(nxv, orc):
    x = np.array([1, 3, 3, 2, 5, 5, np.nan, 5, np.nan, 0, 0, 0], np.float32)
    t = up(nxv, x)
    got = down(nxv, unwrap(nxv.argmax_axis(t, 3, 4, 1)), np.int64)
    assert np.array_equal(got, orc.argmax_axis(x, 3, 4, 1))
    assert list(got) == [1, 2, 0]


@pytest.mark.parametrize("exact", ["0", "1"])
def test_logsumexp(nxv, orc, monkeypatch, exact):
    """f32 in/out within 1e-5 relative and within 4 ulp of the oracle (its
    f64 evaluation rounded once) with the hardware exponential (default),
    1 ulp with exp in f64 (NXV_EXACT_F32=1); sums in double.  Rows of
    1..4096+ elements, odd and unaligned lengths, the cols kernel."""
    monkeypatch.setenv("NXV_EXACT_F32", exact)
    worst = 0
    for shape in [(64, 1000, 1), (3, 50, 17), (4096, 4096, 1), (1, 100003, 1), (5000, 7, 1),
                  (9, 1, 1), (33, 4097, 1)]:
        x = np.random.default_rng(2).normal(size=int(np.prod(shape))).astype(np.float32) * 10
        got = down(nxv, unwrap(nxv.logsumexp(up(nxv, x), *shape)), np.float32)
        want = orc.logsumexp(x, *shape)
        close(got, want, 1e-5, 1e-6)
        worst = max(worst, int(ulp_diff(got, want).max()))
    print(f"logsumexp exact={exact}: worst {worst} ulp")
    assert worst <= (1 if exact == "1" else 4)


@pytest.mark.parametrize("exact", ["0", "1"])
def test_logsumexp_special_values(nxv, orc, monkeypatch, exact):
    """IEEE specials as in the two-pass definition: -inf elements add 0,
    a NaN or +inf gives NaN, a row of only -inf gives NaN; the max moving
    late in a row (ascending rows) exercises the rescaling."""
    monkeypatch.setenv("NXV_EXACT_F32", exact)
    R = 600
    rows = np.random.default_rng(4).normal(size=(12, R)).astype(np.float32)
    rows[0, :500] = -np.inf               # leading -inf, finite max later
    rows[1, :] = -np.inf                  # only -inf
    rows[2, 17] = np.nan
    rows[3, 599] = np.inf
    rows[4, :] = np.nan
    rows[5, :] = np.sort(rows[5]) * 30    # ascending: the max rises at every group
    rows[6, :] = np.sort(rows[6])[::-1] * 30
    rows[7, :] = 88.0                      # exp would overflow without the shift
    rows[8, ::2] = -np.inf
    rows[9, :300] = np.nan
    rows[9, 300:] = -np.inf
    rows[10, :] = -1e30
    rows[11, 0] = 1e30
    x = rows.reshape(-1)
    got = down(nxv, unwrap(nxv.logsumexp(up(nxv, x), 12, R, 1)), np.float32)
    want = orc.logsumexp(x, 12, R, 1)
    assert np.array_equal(np.isnan(got), np.isnan(want)), (got, want)
    ok = ~np.isnan(want)
    close(got[ok], want[ok], 1e-5, 1e-6)
    # one more column of -inf: rows of 601 start unaligned (scalar path) and
    # the results do not change
    x2 = np.concatenate([rows, np.full((12, 1), -np.inf, np.float32)], axis=1).reshape(-1)
    got2 = down(nxv, unwrap(nxv.logsumexp(up(nxv, x2), 12, R + 1, 1)), np.float32)
    assert np.array_equal(np.isnan(got2), np.isnan(want))
    close(got2[ok], want[ok], 1e-5, 1e-6)


@pytest.mark.parametrize("mnk", [(1, 1, 1), (2, 2, 2), (17, 33, 9), (128, 128, 128), (130, 70, 257),
                                 (256, 512, 100), (1, 300, 1000)])
def test_matmul_f64(nxv, orc, mnk):
    m, n, k = mnk
    r = np.random.default_rng(2)
    a, b = r.normal(size=m * k), r.normal(size=k * n)
    got = down(nxv, unwrap(nxv.matmul_batched(up(nxv, a), up(nxv, b), 1, m, n, k, "f64")), np.float64)
    want = orc.matmul(a, b, m, n, k)
    bound = np.abs(a.reshape(m, k)) @ np.abs(b.reshape(k, n))
    assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want) + 2 * k * 2.2e-16 * bound.reshape(-1))


def f32_dot_bound(k, absprod):
    """Forward error bound of an f32 dot product of length k (the bound a true
    f32 FMA GEMM obeys): (k + 8) * 2^-24 * sum|a||b| (accumulation plus the
    3xTF32 split terms, each <= 2^-22 relative)."""
    return (k + 8) * 2.0 ** -24 * absprod


@pytest.mark.parametrize("mnk", [(1, 1, 3), (2, 2, 2), (17, 33, 9), (128, 128, 128), (130, 70, 257),
                                 (333, 129, 65)])
def test_matmul_f32_3xtf32(nxv, orc, mnk):
    """3xTF32 stays within f32 accuracy: |err| <= 1e-5 |C| + 1e-6 + f32 dot bound.

    Inputs ~ N(0, 1): outputs that cancel to near zero cannot meet the flat
    1e-5 / 1e-6 tolerance in any f32-accumulating GEMM (the accumulator's own
    rounding is ~2^-24 of the partial sums), so the dot bound is added.  The
    fraction of elements inside the flat tolerance is printed beside that of
    the host's f32 BLAS product (numpy float32 matmul) on the same inputs,
    and must not be lower by more than 0.5 %.  Inputs scaled as the matmul
    workload's (N(0, 1/k)) meet the flat tolerance everywhere
    (test_matmul_config_sizes)."""
    m, n, k = mnk
    r = np.random.default_rng(3)
    a, b = r.normal(size=m * k).astype(np.float32), r.normal(size=k * n).astype(np.float32)
    got = down(nxv, unwrap(nxv.matmul(up(nxv, a), up(nxv, b), m, n, k)), np.float32)
    want = orc.matmul(a, b, m, n, k)
    bound = (np.abs(a.reshape(m, k)).astype(np.float64) @ np.abs(b.reshape(k, n))).reshape(-1)
    err = np.abs(got.astype(np.float64) - want)
    tol = 1e-5 * np.abs(want) + 1e-6
    host = (a.reshape(m, k) @ b.reshape(k, n)).reshape(-1).astype(np.float64)
    flat, flat_host = (err <= tol).mean(), (np.abs(host - want) <= tol).mean()
    print(f"f32 {m}x{n}x{k}: {flat:.4%} within 1e-5|C|+1e-6 (host f32 BLAS {flat_host:.4%}); "
          f"worst |err| {err.max():.3e} (host {np.abs(host - want).max():.3e}) "
          f"= {np.max(err / f32_dot_bound(k, bound)):.3e} of the dot bound")
    assert flat >= flat_host - 0.005
    assert np.all(err <= tol + f32_dot_bound(k, bound))


@pytest.mark.parametrize("mnk", [(1, 1, 2_200_003), (2, 3, 2_097_153)])
def test_matmul_f32_deep_k(nxv, orc, mnk):
    """k past 65535 tiles of 32 (2,097,120): the transposing split of B
    walks its k tiles grid-stride instead of one grid row per tile."""
    m, n, k = mnk
    r = np.random.default_rng(13)
    a, b = r.normal(size=m * k).astype(np.float32), r.normal(size=k * n).astype(np.float32)
    got = down(nxv, unwrap(nxv.matmul(up(nxv, a), up(nxv, b), m, n, k)), np.float32)
    want = orc.matmul(a, b, m, n, k)
    bound = (np.abs(a.reshape(m, k)).astype(np.float64) @ np.abs(b.reshape(k, n))).reshape(-1)
    assert np.all(np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-6 + f32_dot_bound(k, bound))


@pytest.mark.parametrize("impl", ["tc", "mma"])
@pytest.mark.parametrize("mnk", [(5, 7, 9), (130, 70, 257), (128, 128, 4096), (300, 260, 64)])
def test_matmul_f32_ieee_specials(nxv, orc, monkeypatch, impl, mnk):
    """inf, -inf and NaN inputs and an f32 overflow give the oracle's IEEE
    results (NaN where it has NaN, the same signed infinity where it has one);
    finite elements stay within the f32 dot bound.  128x128x4096 runs the
    tcgen05 kernel's stream-K tail (one tile, 128 k-blocks)."""
    if impl == "mma":
        monkeypatch.setenv("NXV_MATMUL_F32", "mma")
    m, n, k = mnk
    r = np.random.default_rng(11)
    a = r.normal(size=(m, k)).astype(np.float32)
    b = r.normal(size=(k, n)).astype(np.float32)
    a[0, k // 2] = np.inf               # row 0: +-inf unless a column of B meets 0 or NaN
    a[min(2, m - 1), 0] = -np.inf
    b[min(3, k - 1), min(1, n - 1)] = np.nan  # column 1: NaN everywhere
    b[k // 2, n - 1] = 0.0              # inf * 0 in row 0, last column: NaN
    b[k // 2, 0] = 1.0                  # exact TF32 value (lo = 0) times inf: inf
    if m > 4:
        a[4] = 3.0e38                   # row 4: f32 overflow of finite inputs
        b[:, min(2, n - 1)] = np.abs(b[:, min(2, n - 1)]) + 1.0
    got = down(nxv, unwrap(nxv.matmul(up(nxv, a), up(nxv, b), m, n, k)), np.float32)
    want = orc.matmul(a.reshape(-1), b.reshape(-1), m, n, k)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    inf = np.isinf(want)
    assert np.array_equal(np.isinf(got), inf)
    assert np.array_equal(np.sign(got[inf]), np.sign(want[inf]))
    assert inf.any() and np.isnan(want).any()
    fin = np.isfinite(want)
    bound = (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)).reshape(-1)
    assert np.all(np.abs(got[fin] - want[fin]) <= 1e-5 * np.abs(want[fin]) + 1e-6 + f32_dot_bound(k, bound[fin]))


def test_matmul_config_sizes(nxv, orc):
    """A.B with A,B [2048,2048] ~ N(0, 1/2048) (f32 and f64), batched f64 64x256^3.
    Checked on 256 sampled rows against the oracle; the f32 product is held
    to the flat f32 tolerance (1e-5 relative + 1e-6 absolute per element),
    not just the f32 dot bound."""
    r = np.random.default_rng(2)
    n = 2048
    rows = r.choice(n, 256, replace=False)
    for dt in (np.float64, np.float32):
        a = (r.normal(size=(n, n)) / np.sqrt(n)).astype(dt)
        b = (r.normal(size=(n, n)) / np.sqrt(n)).astype(dt)
        if dt == np.float64:
            t = unwrap(nxv.matmul_batched(up(nxv, a), up(nxv, b), 1, n, n, n, "f64"))
        else:
            t = unwrap(nxv.matmul(up(nxv, a), up(nxv, b), n, n, n))
        got = down(nxv, t, dt).reshape(n, n)[rows]
        want = orc.matmul(np.ascontiguousarray(a[rows]), b, 256, n, n).reshape(256, n)
        bound = np.abs(a[rows]).astype(np.float64) @ np.abs(b).astype(np.float64)
        if dt == np.float64:
            assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want) + 2 * n * 2.2e-16 * bound)
        else:
            err = np.abs(got.astype(np.float64) - want)
            rel = err / np.maximum(np.abs(want), 1e-30)
            print(f"f32 2048^3 (256 rows): max |err| {err.max():.3e}, max rel err {rel.max():.3e}, "
                  f"max |err|/(1e-5|C|+1e-6) {np.max(err / (1e-5 * np.abs(want) + 1e-6)):.3f}, "
                  f"max |err|/dot bound {np.max(err / f32_dot_bound(n, bound)):.3e}")
            assert np.all(err <= 1e-5 * np.abs(want) + 1e-6)
    a = r.normal(size=(64, 256, 256)) / 16
    b = r.normal(size=(64, 256, 256)) / 16
    got = down(nxv, unwrap(nxv.matmul_batched(up(nxv, a), up(nxv, b), 64, 256, 256, 256, "f64")), np.float64)
    want = orc.matmul(a, b, 256, 256, 256, batch=64)
    bound = np.einsum("bik,bkj->bij", np.abs(a), np.abs(b)).reshape(-1)
    assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want) + 2 * 256 * 2.2e-16 * bound)


@pytest.mark.parametrize("exact", ["0", "1"])
@pytest.mark.parametrize("n", [1, 2, 4, 6, 7, 1024, 1000001])
def test_philox_matches_oracle(nxv, orc, monkeypatch, n, exact):
    """Uniforms bit-exact; f32 normals within 1e-6 (f32 math by default,
    f64 math rounded once with NXV_EXACT_F32=1); f64 normals within 1e-12."""
    monkeypatch.setenv("NXV_EXACT_F32", exact)
    for seed in (0, 42, 0xDEADBEEF):
        u = down(nxv, unwrap(nxv.uniform(n, seed)), np.float32)
        assert np.array_equal(u, orc.random_f32(n, seed, 0))  # bit-exact
        g = down(nxv, unwrap(nxv.normal(n, seed)), np.float32)
        close(g, orc.random_f32(n, seed, 1), 1e-6, 1e-6)
        u64 = down(nxv, unwrap(nxv.random_f64(n, seed, 0)), np.float64)
        assert np.array_equal(u64, orc.random_f64(n, seed, 0))
        g64 = down(nxv, unwrap(nxv.random_f64(n, seed, 1)), np.float64)
        close(g64, orc.random_f64(n, seed, 1), 1e-12, 1e-14)


def test_f64_normals_against_exact_box_muller(nxv):
    """f64 normals against the Box-Muller transform of the same uniforms
    (pair c: u1 = uniform 2c + 2^-53, u2 = uniform 2c + 1) evaluated in
    50-digit arithmetic: within 4 units in the last place of each result,
    near the zeros of sin and cos too (sin(pi r) is evaluated on an exactly
    reduced r)."""
    import mpmath

    mpmath.mp.dps = 50
    n, seed = 4000, 77
    u = down(nxv, unwrap(nxv.random_f64(n, seed, 0)), np.float64)
    g = down(nxv, unwrap(nxv.random_f64(n, seed, 1)), np.float64)
    worst = 0.0
    for c in range(n // 2):
        u1 = mpmath.mpf(float(u[2 * c])) + mpmath.mpf(2) ** -53
        u2 = mpmath.mpf(float(u[2 * c + 1]))
        r = mpmath.sqrt(-2 * mpmath.log(u1))
        for got, want in ((g[2 * c], r * mpmath.cos(2 * mpmath.pi * u2)),
                          (g[2 * c + 1], r * mpmath.sin(2 * mpmath.pi * u2))):
            w = float(want)
            ulp = np.spacing(abs(w)) if w != 0 else np.finfo(np.float64).tiny
            worst = max(worst, float(abs(mpmath.mpf(float(got)) - want) / ulp))
    print(f"f64 normals: max {worst:.2f} ulp against the exact transform")
    assert worst <= 4.0


def test_f32_normals_against_exact_box_muller(nxv, monkeypatch):
    """Default f32 normals (f32 arithmetic) against the Box-Muller transform
    of the same uniforms (pair c: u1 = uniform 2c + 2^-24, u2 = uniform
    2c + 1) in 50-digit arithmetic: within 4 f32 units in the last place."""
    import mpmath

    monkeypatch.setenv("NXV_EXACT_F32", "0")
    mpmath.mp.dps = 50
    n, seed = 4000, 91
    u = down(nxv, unwrap(nxv.uniform(n, seed)), np.float32)
    g = down(nxv, unwrap(nxv.normal(n, seed)), np.float32)
    worst = 0.0
    for c in range(n // 2):
        u1 = mpmath.mpf(float(u[2 * c])) + mpmath.mpf(2) ** -24
        u2 = mpmath.mpf(float(u[2 * c + 1]))
        r = mpmath.sqrt(-2 * mpmath.log(u1))
        for got, want in ((g[2 * c], r * mpmath.cos(2 * mpmath.pi * u2)),
                          (g[2 * c + 1], r * mpmath.sin(2 * mpmath.pi * u2))):
            w = np.float32(float(want))
            ulp = float(np.spacing(abs(w))) if w != 0 else float(np.finfo(np.float32).tiny)
            worst = max(worst, float(abs(mpmath.mpf(float(got)) - want) / ulp))
    print(f"f32 normals: max {worst:.2f} ulp against the exact transform")
    assert worst <= 4.0


@pytest.mark.parametrize("mn", [(1, 1), (3, 5), (33, 65), (1000, 17), (4096, 4096), (8, 3000), (3000, 9)])
def test_transpose_and_cast(nxv, orc, mn):
    m, n = mn
    a = np.random.default_rng(4).normal(size=m * n).astype(np.float32)
    got = down(nxv, unwrap(nxv.transpose_2d(up(nxv, a), m, n)), np.float32)
    assert np.array_equal(got, orc.transpose(a, m, n))
    d = down(nxv, unwrap(nxv.cast_f32_to_f64(up(nxv, a), m * n)), np.float64)
    assert np.array_equal(d, a.astype(np.float64))
    b = np.random.default_rng(5).normal(size=m * n) * 1e3
    f = down(nxv, unwrap(nxv.cast_f64_to_f32(up(nxv, b), m * n)), np.float32)
    assert np.array_equal(f, b.astype(np.float32))


@pytest.mark.parametrize("n", [1, 255, 256, 257, 100003, 1 << 20])
def test_kinetic_energy_partials(nxv, orc, n):
    """One partial per 256-element group: 0.5 * sum((p*p)*m) of the group,
    the f32 products summed in double (within 1e-6 of numpy per group)."""
    r = np.random.default_rng(n)
    p, m = r.normal(size=n).astype(np.float32), r.uniform(0.5, 2, n).astype(np.float32)
    parts = down(nxv, unwrap(nxv.kinetic_energy(up(nxv, p), up(nxv, m))), np.float32)
    assert parts.size == (n + 255) // 256
    terms = ((p * p) * m).astype(np.float64)
    pad = np.zeros(parts.size * 256)
    pad[:n] = terms
    want = 0.5 * pad.reshape(-1, 256).sum(axis=1)
    close(parts, want, 1e-6, 1e-6)
    # an unaligned p (offset by one element) takes the scalar path
    if n > 1:
        p2, m2 = p[1:].copy(), m[1:].copy()
        pt = unwrap(nxv.upload_f32(np.concatenate([[0.0], p2]).astype(np.float32)))
        from nx_vulkan_b200 import _native
        lib = _native.load()
        base = lib.nxv_buf_device_ptr(pt.handle)
        hp = lib.nxv_buf_wrap(base + 4, (n - 1) * 4)
        hm = up(nxv, m2)
        out = unwrap(nxv.upload_f32(np.zeros((n - 1 + 255) // 256, np.float32)))
        assert lib.nxv_kinetic_energy(out.handle, hp, hm.handle, n - 1,
                                      nxv.shader_path("kinetic_energy.spv")) == 0
        lib.nxv_buf_free(hp)
        got2 = down(nxv, out, np.float32)
        t2 = ((p2 * p2) * m2).astype(np.float64)
        pad2 = np.zeros(got2.size * 256)
        pad2[:n - 1] = t2
        close(got2, 0.5 * pad2.reshape(-1, 256).sum(axis=1), 1e-6, 1e-6)


def test_kinetic_energy_and_logpdf_large(nxv, orc):
    r = np.random.default_rng(6)
    n = 100003
    p, m = r.normal(size=n).astype(np.float32), r.uniform(0.5, 2, n).astype(np.float32)
    parts = down(nxv, unwrap(nxv.kinetic_energy(up(nxv, p), up(nxv, m))), np.float32)
    assert parts.size == (n + 255) // 256
    assert abs(parts.astype(np.float64).sum() - orc.kinetic_energy(p, m)) <= 1e-5 * orc.kinetic_energy(p, m)
    x, mu, s = r.normal(size=n).astype(np.float32), r.normal(size=n).astype(np.float32), r.uniform(0.5, 2, n).astype(np.float32)
    got = down(nxv, unwrap(nxv.normal_logpdf(up(nxv, x), up(nxv, mu), up(nxv, s))), np.float32)
    close(got, orc.normal_logpdf(x, mu, s), 1e-5, 1e-6)


def test_errors_are_reported(nxv):
    from nx_vulkan_b200 import _native
    lib = _native.load()
    a = unwrap(nxv.upload_f32([1.0] * 8))
    # unknown kernel basename
    assert lib.nxv_apply_unary(a.handle, a.handle, 8, 0, b"nope.spv") == -2
    # element count beyond the buffer
    assert lib.nxv_apply_unary(a.handle, a.handle, 9, 0, nxv.shader_path("elementwise_unary.spv")) == -3
    assert "buffer" in _native.last_error()
    # bad op
    assert lib.nxv_apply_binary(a.handle, a.handle, a.handle, 8, 10, nxv.shader_path("elementwise_binary.spv")) == -3
    # empty tensor ops are no-ops, not errors
    e = unwrap(nxv.upload_f32([]))
    assert lib.nxv_apply_unary(e.handle, e.handle, 0, 0, nxv.shader_path("elementwise_unary.spv")) == 0


@pytest.mark.parametrize("bmnk", [(1, 1, 1, 1), (1, 128, 128, 32), (1, 129, 257, 33), (3, 130, 70, 257),
                                  (2, 256, 384, 1000), (64, 256, 256, 256)])
def test_matmul_f32_tensor_core_vs_oracle_and_mma(nxv, orc, monkeypatch, bmnk):
    """tcgen05 3xTF32 (default) against the oracle and against the mma.sync
    3xTF32 kernel; both within the f32 dot-product bound."""
    batch, m, n, k = bmnk
    r = np.random.default_rng(11)
    a = r.normal(size=batch * m * k).astype(np.float32)
    b = r.normal(size=batch * k * n).astype(np.float32)
    ta, tb = up(nxv, a), up(nxv, b)
    got = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f32")), np.float32)
    monkeypatch.setenv("NXV_MATMUL_F32", "mma")
    legacy = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f32")), np.float32)
    want = orc.matmul(a, b, m, n, k, batch=batch)
    bound = np.concatenate([
        (np.abs(a.reshape(batch, m, k)[q]).astype(np.float64) @ np.abs(b.reshape(batch, k, n)[q])).reshape(-1)
        for q in range(batch)])
    tol = 1e-5 * np.abs(want) + 1e-6 + f32_dot_bound(k, bound)
    assert np.all(np.abs(got - want) <= tol)
    assert np.all(np.abs(legacy - want) <= tol)
    from nx_vulkan_b200 import _native
    assert _native.load().nxv_synchronize() == 0  # no pipeline timeout recorded


@pytest.mark.parametrize("cfg", ["16x4", "16x8", "16x16", "32x4", "32x8", "32x16"])
@pytest.mark.parametrize("bmnk", [(1, 130, 70, 257), (2, 256, 256, 100), (1, 33, 200, 17)])
def test_matmul_f64_dmma_shapes(nxv, orc, monkeypatch, cfg, bmnk):
    """Every DMMA configuration (k-tile x MMA K-shape) of the 128 x 128 tile
    against the oracle."""
    monkeypatch.setenv("NXV_DMMA", cfg)
    monkeypatch.setenv("NXV_GEMM_TILE", "128")
    batch, m, n, k = bmnk
    r = np.random.default_rng(12)
    a, b = r.normal(size=batch * m * k), r.normal(size=batch * k * n)
    got = down(nxv, unwrap(nxv.matmul_batched(up(nxv, a), up(nxv, b), batch, m, n, k, "f64")), np.float64)
    want = orc.matmul(a, b, m, n, k, batch=batch)
    bound = np.concatenate([
        (np.abs(a.reshape(batch, m, k)[q]) @ np.abs(b.reshape(batch, k, n)[q])).reshape(-1)
        for q in range(batch)])
    assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want) + 2 * k * 2.2e-16 * bound)


@pytest.mark.parametrize("bmnk", [(1, 1000, 700, 513), (3, 300, 260, 700), (1, 1100, 1300, 640),
                                  (1, 2304, 1152, 320), (1, 100, 120, 3000)])
def test_matmul_f64_stream_k(nxv, orc, monkeypatch, bmnk):
    """Tile counts that leave a partial last wave run their tail as stream-K
    (k-ranges split evenly over the SMs, partials summed in k order) on the
    128 x 128 schedule (NXV_GEMM_TILE=128).  The result is within the f64
    bound, identical bit for bit on a second call, and within the bound of
    the plain data-parallel schedule (NXV_GEMM_SK=0) and of the default
    64 x 64 tiles."""
    batch, m, n, k = bmnk
    r = np.random.default_rng(13)
    a, b = r.normal(size=batch * m * k), r.normal(size=batch * k * n)
    ta, tb = up(nxv, a), up(nxv, b)
    small = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f64")), np.float64)
    monkeypatch.setenv("NXV_GEMM_TILE", "128")
    got = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f64")), np.float64)
    again = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f64")), np.float64)
    assert np.array_equal(got, again)
    monkeypatch.setenv("NXV_GEMM_SK", "0")
    plain = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f64")), np.float64)
    want = orc.matmul(a, b, m, n, k, batch=batch)
    bound = np.concatenate([
        (np.abs(a.reshape(batch, m, k)[q]) @ np.abs(b.reshape(batch, k, n)[q])).reshape(-1)
        for q in range(batch)])
    tol = 1e-12 * np.abs(want) + 2 * k * 2.2e-16 * bound
    assert np.all(np.abs(got - want) <= tol)
    assert np.all(np.abs(plain - want) <= tol)
    assert np.all(np.abs(small - want) <= tol)


@pytest.mark.parametrize("bmnk", [(1, 1, 1, 1), (1, 33, 200, 17), (2, 65, 129, 31), (5, 64, 64, 64),
                                  (1, 300, 1, 7), (3, 100, 120, 3000), (64, 256, 256, 256),
                                  (1, 256, 10000, 104)])
def test_matmul_f64_tile64(nxv, orc, bmnk):
    """The default f64 tile (64 x 64, three CTAs per SM): ragged edges, odd K
    (rows not 16-byte aligned: the scalar loader), deep K, many batches and
    the batched and logistic-gradient shapes, within the f64 bound and
    identical bit for bit on a second call."""
    batch, m, n, k = bmnk
    r = np.random.default_rng(14)
    a, b = r.normal(size=batch * m * k), r.normal(size=batch * k * n)
    ta, tb = up(nxv, a), up(nxv, b)
    got = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f64")), np.float64)
    again = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f64")), np.float64)
    assert np.array_equal(got, again)
    want = orc.matmul(a, b, m, n, k, batch=batch)
    bound = np.concatenate([
        (np.abs(a.reshape(batch, m, k)[q]) @ np.abs(b.reshape(batch, k, n)[q])).reshape(-1)
        for q in range(batch)])
    assert np.all(np.abs(got - want) <= 1e-12 * np.abs(want) + 2 * k * 2.2e-16 * bound)


@pytest.mark.parametrize("bmnk", [(1, 100, 120, 3000), (1, 500, 400, 4000), (2, 256, 256, 2048),
                                  (1, 2560, 1024, 2048)])
def test_matmul_f32_stream_k(nxv, orc, monkeypatch, bmnk):
    """tcgen05 3xTF32 with a stream-K tail (few tiles over a deep K, and a
    full wave plus 12 tail tiles): within the f32 dot-product bound,
    identical bit for bit on a second call, and within the bound of the
    data-parallel schedule (NXV_GEMM_SK=0)."""
    batch, m, n, k = bmnk
    r = np.random.default_rng(14)
    a = r.normal(size=batch * m * k).astype(np.float32)
    b = r.normal(size=batch * k * n).astype(np.float32)
    ta, tb = up(nxv, a), up(nxv, b)
    got = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f32")), np.float32)
    again = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f32")), np.float32)
    assert np.array_equal(got, again)
    monkeypatch.setenv("NXV_GEMM_SK", "0")
    plain = down(nxv, unwrap(nxv.matmul_batched(ta, tb, batch, m, n, k, "f32")), np.float32)
    want = orc.matmul(a, b, m, n, k, batch=batch)
    bound = np.concatenate([
        (np.abs(a.reshape(batch, m, k)[q]).astype(np.float64) @ np.abs(b.reshape(batch, k, n)[q])).reshape(-1)
        for q in range(batch)])
    tol = 1e-5 * np.abs(want) + 1e-6 + f32_dot_bound(k, bound)
    assert np.all(np.abs(got - want) <= tol)
    assert np.all(np.abs(plain - want) <= tol)
    from nx_vulkan_b200 import _native
    assert _native.load().nxv_synchronize() == 0  # no pipeline timeout recorded
