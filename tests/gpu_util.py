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


def close(got, want, rtol, atol):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    both_nan = np.isnan(got) & np.isnan(want)
    same_inf = np.isinf(got) & np.isinf(want) & (np.sign(got) == np.sign(want))
    ok = both_nan | same_inf | (np.abs(got - want) <= atol + rtol * np.abs(want))
    if not ok.all():
        i = np.flatnonzero(~ok)[:5]
        raise AssertionError(f"{(~ok).sum()} mismatches, e.g. idx {i}: got {got[i]} want {want[i]}")
