"""Helpers for GPU tests: numpy <-> device buffers through the nxv_* ABI."""
import numpy as np


def up(nxv, arr):
    ok, t = nxv.upload_binary(np.ascontiguousarray(arr))
    assert ok == "ok", t
    return t


def down(nxv, t, dtype, n=None):
    dtype = np.dtype(dtype)
    nb = t.n_bytes if n is None else n * dtype.itemsize
    ok, b = nxv.download_binary(t, t.n_bytes)
    assert ok == "ok", b
    return np.frombuffer(b[:nb], dtype=dtype).copy()


def unwrap(r):
    assert r[0] == "ok", r
    return r[1]


EXACT_OPS = {0, 1, 2, 3, 5, 6, 7, 8, 9, 102, 103, 104, 107, 108, 109, 110, 111, 112}


def chain_error_bound(a, operands, ops, src=None, imm=None, dtype=np.float32, ulps=4.0):
    """First-order forward error bound of an op tape evaluated in `dtype`.

    Each op contributes 0.5 ulp of its result (IEEE-exact ops) or `ulps` ulp
    (transcendentals: the f32 library functions are within 2-4 ulp), and
    scales the incoming error by |d op / d r|.  Elements where the register
    lies within its error of a discontinuity (ceil/floor/sign/compare) get an
    infinite bound.  Returns the bound per element (float64)."""
    a = np.asarray(a, np.float64)
    ops = list(ops)
    src = list(src) if src is not None else [1] * len(ops)
    imm = list(imm) if imm is not None else [0.0] * len(ops)
    ins = [None] + [np.asarray(o, np.float64) if o is not None else None for o in operands]
    r = a.copy()
    err = np.zeros_like(r)
    spacing = lambda v: np.spacing(np.abs(v).astype(dtype)).astype(np.float64)
    with np.errstate(all="ignore"):
        for op, s, im in zip(ops, src, imm):
            if op == 255:
                continue
            c = 0.5 if op in EXACT_OPS else ulps
            if op < 100:
                rhs = np.full_like(r, np.float64(dtype(im))) if s == 0 else ins[s]
                if op in (0, 2):
                    f, new = 1.0, (r + rhs if op == 0 else r - rhs)
                elif op == 1:
                    f, new = np.abs(rhs), r * rhs
                elif op == 3:
                    f, new = 1.0 / np.abs(rhs), r / rhs
                elif op == 4:
                    new = np.power(r, rhs)
                    f = np.abs(rhs * np.power(r, rhs - 1))
                elif op in (5, 6):
                    f, new = 1.0, (np.maximum(r, rhs) if op == 5 else np.minimum(r, rhs))
                else:
                    new = {7: r == rhs, 8: r < rhs, 9: r > rhs}[op].astype(np.float64)
                    f = np.where(np.abs(r - rhs) <= err, np.inf, 0.0)
            else:
                u = op - 100
                if u == 0:
                    new = np.exp(r); f = new
                elif u == 1:
                    new = np.log(r); f = 1 / np.abs(r)
                elif u == 2:
                    new = np.sqrt(r); f = 0.5 / new
                elif u in (3, 4):
                    new = np.abs(r) if u == 3 else -r; f = 1.0
                elif u == 5:
                    new = 1 / (1 + np.exp(-r)); f = new * (1 - new)
                elif u == 6:
                    new = np.tanh(r); f = 1 - new * new
                elif u == 7:
                    new = np.maximum(r, 0); f = 1.0
                elif u in (8, 9):
                    new = np.ceil(r) if u == 8 else np.floor(r)
                    f = np.where(np.abs(r - np.round(r)) <= err, np.inf, 0.0)
                elif u == 10:
                    new = np.sign(r); f = np.where(np.abs(r) <= err, np.inf, 0.0)
                elif u == 11:
                    new = 1 / r; f = 1 / (r * r)
                elif u == 12:
                    new = r * r; f = 2 * np.abs(r)
                elif u == 13:
                    import math
                    new = np.vectorize(math.erf)(r); f = 2 / np.sqrt(np.pi) * np.exp(-r * r)
                else:
                    new = np.expm1(r); f = np.exp(r)
            err = np.nan_to_num(f * err, nan=np.inf) + c * spacing(new)
            r = new
    return err


def close_bound(got, want, bound, rtol=1e-5, atol=1e-6):
    """|got - want| <= rtol |want| + atol + 2 * propagated bound."""
    close(got, want, rtol, atol + 2 * np.asarray(bound))


def close(got, want, rtol, atol):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    both_nan = np.isnan(got) & np.isnan(want)
    same_inf = np.isinf(got) & np.isinf(want) & (np.sign(got) == np.sign(want))
    with np.errstate(invalid="ignore"):
        ok = both_nan | same_inf | (got == want) | (np.abs(got - want) <= atol + rtol * np.abs(want))
    if not ok.all():
        i = np.flatnonzero(~ok)[:5]
        raise AssertionError(f"{(~ok).sum()} mismatches, e.g. idx {i}: got {got[i]} want {want[i]}")


def ulp_diff(got, want):
    """|got - want| in units in the last place of f32 (adjacent floats differ
    by 1; +0 and -0 are equal).  Both arrays f32; NaN positions must match
    and count 0."""
    g = np.asarray(got, np.float32)
    w = np.asarray(want, np.float32)
    assert np.array_equal(np.isnan(g), np.isnan(w))

    def ordered(x):
        i = x.view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)

    d = np.abs(ordered(g) - ordered(w))
    d[np.isnan(w)] = 0
    return d
