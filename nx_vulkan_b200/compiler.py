"""Elementwise chain compiler: the `Nx.Vulkan.Compiler` path of the reference.

The reference's Defn compiler (lib/nx_vulkan/compiler.ex:91-120, 175-405)
traces a function, looks for a linear chain of at most 8 elementwise ops
whose binary steps take a *parameter* as the second operand, and runs it
as one `fused_chain(_4)` dispatch; anything else goes op by op through
`Nx.Defn.Evaluator`.  This module does the same for Python functions over
GPU tensors:

  * `jit(fun)` traces `fun` once per (arity, dtype, size) signature into an
    expression DAG (the reference re-traced on every call,
    compiler.ex:86-89) and caches the lowering;
  * the chain detector walks from the output towards each parameter in turn
    (compiler.ex:213-285): every binary step on the path must have a
    parameter or a scalar literal on its other side; add/multiply/max/min
    may swap sides; `c - r` becomes `-(r - c)` (bit-identical in IEEE);
  * literals become immediates of the op tape, so a chain such as
    tanh(exp(x*y + z) - 1.0) -- which the reference cannot fuse because
    1.0 is not a parameter (compiler.ex:291-307) -- runs as ONE kernel
    (`nxv_fused_chain_imm`);
  * anything else is evaluated node by node with the elementwise kernels
    (the Evaluator path), still entirely on the GPU.
"""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from . import vulkan as V

BINARY = {"add": 0, "multiply": 1, "subtract": 2, "divide": 3, "pow": 4, "max": 5, "min": 6,
          "equal": 7, "less": 8, "greater": 9}
UNARY = dict(V.OPS_UNARY)
COMMUTATIVE = {"add", "multiply", "max", "min", "equal"}


@dataclass
class Tensor:
    """A GPU tensor: device buffer + element type + shape."""

    data: V.VulkanTensor
    dtype: str  # "f32" | "f64"
    shape: tuple

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @classmethod
    def from_numpy(cls, a: np.ndarray) -> "Tensor":
        a = np.ascontiguousarray(a)
        dt = {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64"}[a.dtype]
        ok, t = V.upload_binary(a)
        if ok != V.OK:
            raise RuntimeError(f"upload failed: {t}")
        return cls(t, dt, a.shape)

    def numpy(self) -> np.ndarray:
        ok, b = V.download_binary(self.data, self.data.n_bytes)
        if ok != V.OK:
            raise RuntimeError(f"download failed: {b}")
        return np.frombuffer(b, dtype=np.float32 if self.dtype == "f32" else np.float64).reshape(self.shape)


# ---- expression graph -----------------------------------------------------------

@dataclass(eq=False)
class Expr:
    op: str                       # "parameter" | "constant" | unary | binary name
    args: tuple = ()
    index: int = -1               # parameter position
    value: float = 0.0            # constant value

    def _b(self, op, other, swap=False):
        o = other if isinstance(other, Expr) else Expr("constant", value=float(other))
        return Expr(op, (o, self) if swap else (self, o))

    def __add__(self, o): return self._b("add", o)
    def __radd__(self, o): return self._b("add", o, True)
    def __sub__(self, o): return self._b("subtract", o)
    def __rsub__(self, o): return self._b("subtract", o, True)
    def __mul__(self, o): return self._b("multiply", o)
    def __rmul__(self, o): return self._b("multiply", o, True)
    def __truediv__(self, o): return self._b("divide", o)
    def __rtruediv__(self, o): return self._b("divide", o, True)
    def __pow__(self, o): return self._b("pow", o)
    def __neg__(self): return Expr("negate", (self,))


def _lift(x):
    return x if isinstance(x, Expr) else Expr("constant", value=float(x))


class _Nx:
    """The Nx function names used inside traced functions (Nx.add, Nx.exp ...)."""

    def __getattr__(self, name):
        if name in BINARY:
            return lambda a, b: Expr(name, (_lift(a), _lift(b)))
        if name in UNARY:
            return lambda a: Expr(name, (_lift(a),))
        raise AttributeError(name)


nx = _Nx()


# ---- chain detection --------------------------------------------------------------

@dataclass
class Chain:
    start: int                          # parameter index of the register
    ops: list = field(default_factory=list)   # op codes
    src: list = field(default_factory=list)   # 0 imm, 1..3 operand slot
    imm: list = field(default_factory=list)
    operands: list = field(default_factory=list)  # parameter index per slot 1..3


def _find_chain_to(target: int, e: Expr, ch: Chain) -> bool:
    """Append, in execution order, the ops from parameter `target` up to `e`."""
    if e.op == "parameter":
        return e.index == target
    if e.op in UNARY:
        if not _find_chain_to(target, e.args[0], ch):
            return False
        ch.ops.append(100 + UNARY[e.op]); ch.src.append(1); ch.imm.append(0.0)
        return True
    if e.op not in BINARY:
        return False
    first, second = e.args
    mark = (len(ch.ops), list(ch.operands))
    if _find_chain_to(target, first, ch):
        return _leaf(e.op, second, ch, negate_after=False)
    del ch.ops[mark[0]:], ch.src[mark[0]:], ch.imm[mark[0]:]
    ch.operands[:] = mark[1]
    if e.op in COMMUTATIVE and _find_chain_to(target, second, ch):
        return _leaf(e.op, first, ch, negate_after=False)
    if e.op == "subtract" and _find_chain_to(target, second, ch):
        # c - r == -(r - c) exactly
        return _leaf("subtract", first, ch, negate_after=True)
    return False


def _leaf(op: str, other: Expr, ch: Chain, negate_after: bool) -> bool:
    if other.op == "constant":
        ch.ops.append(BINARY[op]); ch.src.append(0); ch.imm.append(other.value)
    elif other.op == "parameter":
        if other.index in ch.operands:
            slot = ch.operands.index(other.index) + 1
        elif len(ch.operands) < 3:
            ch.operands.append(other.index)
            slot = len(ch.operands)
        else:
            return False
        ch.ops.append(BINARY[op]); ch.src.append(slot); ch.imm.append(0.0)
    else:
        return False
    if negate_after:
        ch.ops.append(100 + UNARY["negate"]); ch.src.append(1); ch.imm.append(0.0)
    return True


def detect_chain(root: Expr, arity: int):
    """Try every parameter as the register start; first success wins."""
    for start in range(arity):
        ch = Chain(start)
        if _find_chain_to(start, root, ch) and 1 <= len(ch.ops) <= 8:
            return ch
    return None


# ---- jit ---------------------------------------------------------------------------

class Compiled:
    def __init__(self, fun: Callable, root: Expr, arity: int):
        self.fun, self.root, self.arity = fun, root, arity
        self.chain = detect_chain(root, arity)
        if os.environ.get("NXV_FUSE_DEBUG"):
            msg = (f"fused: ops={self.chain.ops} src={self.chain.src} imm={self.chain.imm}"
                   if self.chain else "not fusable: op-by-op")
            print(f"[nx_vulkan_b200.compiler] {getattr(fun, '__name__', 'fun')}: {msg}",
                  file=sys.stderr)

    def __call__(self, *args: Tensor) -> Tensor:
        if self.chain is not None:
            return self._run_fused(args)
        return self._evaluate(self.root, args, {})

    def _run_fused(self, args):
        ch = self.chain
        a = args[ch.start]
        items = []
        for op, s, im in zip(ch.ops, ch.src, ch.imm):
            if op >= 100:
                items.append({v + 100: k for k, v in UNARY.items()}[op])
            else:
                name = {v: k for k, v in BINARY.items()}[op]
                items.append((name, ("imm", im) if s == 0 else s))
        operands = [args[i].data for i in ch.operands]
        ok, out = V.fused_chain_imm(a.data, operands, items, dtype=a.dtype)
        if ok != V.OK:
            raise RuntimeError(f"fused chain failed: {out}: {V._native.last_error()}")
        return Tensor(out, a.dtype, a.shape)

    def _evaluate(self, e: Expr, args, memo):
        """Op-by-op evaluation on the GPU (the Evaluator path)."""
        if id(e) in memo:
            return memo[id(e)]
        if e.op == "parameter":
            r = args[e.index]
        elif e.op == "constant":
            raise ValueError("a bare constant cannot be evaluated without a shape")
        elif e.op in UNARY:
            x = self._evaluate(e.args[0], args, memo)
            spv = "elementwise_unary.spv" if x.dtype == "f32" else "elementwise_unary_f64.spv"
            ok, t = V.apply_unary(x.data, UNARY[e.op], V.shader_path(spv), 4 if x.dtype == "f32" else 8)
            r = _check(ok, t, x)
        else:
            lhs, rhs = e.args
            if rhs.op == "constant" or lhs.op == "constant":
                # scalar literal: one fused step with an immediate
                x = self._evaluate(rhs if lhs.op == "constant" else lhs, args, memo)
                c = (lhs if lhs.op == "constant" else rhs).value
                if lhs.op == "constant":
                    if e.op in COMMUTATIVE:
                        items = [(e.op, ("imm", c))]
                    elif e.op == "subtract":
                        items = [("subtract", ("imm", c)), "negate"]
                    else:
                        raise ValueError(f"unsupported literal on the left of {e.op}")
                else:
                    items = [(e.op, ("imm", c))]
                ok, t = V.fused_chain_imm(x.data, [], items, dtype=x.dtype)
                r = _check(ok, t, x)
            else:
                a = self._evaluate(lhs, args, memo)
                b = self._evaluate(rhs, args, memo)
                if a.size != b.size:
                    raise ValueError("op-by-op evaluation needs equal sizes")
                spv = "elementwise_binary.spv" if a.dtype == "f32" else "elementwise_binary_f64.spv"
                ok, t = V.apply_binary(a.data, b.data, BINARY[e.op], V.shader_path(spv),
                                       4 if a.dtype == "f32" else 8)
                r = _check(ok, t, a)
        memo[id(e)] = r
        return r


def _check(ok, t, like: Tensor) -> Tensor:
    if ok != V.OK:
        raise RuntimeError(f"kernel failed: {t}: {V._native.last_error()}")
    return Tensor(t, like.dtype, like.shape)


def trace(fun: Callable, arity: int) -> Expr:
    params = [Expr("parameter", index=i) for i in range(arity)]
    root = fun(*params)
    if not isinstance(root, Expr):
        raise TypeError("traced function must return an expression of its arguments")
    return root


def jit(fun: Callable) -> Callable:
    """`Nx.Vulkan.jit/2` for elementwise functions: trace once per signature,
    fuse when the body is a linear chain, else run op by op on the GPU."""
    cache: dict = {}

    def run(*args: Tensor) -> Tensor:
        key = tuple((a.dtype, a.size) for a in args)
        comp = cache.get(key)
        if comp is None:
            comp = cache[key] = Compiled(fun, trace(fun, len(args)), len(args))
        return comp(*args)

    run.compiled = lambda *args: cache.get(tuple((a.dtype, a.size) for a in args))
    return run
