"""Front-end of the host scalar oracle (TEST INFRASTRUCTURE ONLY).

A `Program` records porch API calls as the text program that
oracle/oracle.cpp evaluates. It offers the same functions as
porch_b200.api (`tensor`, operators, `matmul`, `reshape`, ..., `softmax`), so
a test writes each graph once as `f(M, ...)` and runs it with M = the product
API and M = a Program. Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg use this module, and only as the checker.
"""

from __future__ import annotations

import builtins as _builtins
import ctypes
import os
import struct
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path
from typing import Sequence

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIBRARY = ORACLE_DIR / "_build" / "liboracle.so"

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            from . import build as _b

            _b.build_oracle()
        # A C++ extension loaded earlier (numpy's) can leave the C++ runtime
        # outside the global symbol scope, which breaks iostream number
        # parsing in later-loaded C++ libraries; put it there first.
        ctypes.CDLL("libstdc++.so.6", mode=ctypes.RTLD_GLOBAL)
        L = ctypes.CDLL(str(LIBRARY))
        L.oracle_last_error.restype = c_char_p
        L.oracle_shape.argtypes = [c_char_p, POINTER(c_void_p), POINTER(POINTER(c_int64)),
                                   POINTER(c_size_t), c_size_t, POINTER(c_int64), c_size_t,
                                   POINTER(c_size_t)]
        L.oracle_shape.restype = c_int
        L.oracle_eval.argtypes = [c_char_p, POINTER(c_void_p), POINTER(POINTER(c_int64)),
                                  POINTER(c_size_t), c_size_t, POINTER(c_float), c_size_t, c_int]
        L.oracle_eval.restype = c_int
        _lib = L
    return _lib


class OracleInvalidArgument(ValueError):
    pass


class OracleOutOfRange(IndexError):
    pass


def _raise(status: int) -> None:
    msg = lib().oracle_last_error().decode()
    if status == 1:
        raise OracleInvalidArgument(msg)
    if status == 2:
        raise OracleOutOfRange(msg)
    raise RuntimeError(msg)


class _All:
    pass


ALL = _All()


class Node:
    """A program value: an expression, or a tensor handle (`is_tensor`)."""

    def __init__(self, prog: "Program", vid: int, is_tensor: bool = False):
        self.prog = prog
        self.id = vid
        self.is_tensor = is_tensor

    def shape(self) -> list[int]:
        return self.prog.shape_of(self)

    def rank(self) -> int:
        return len(self.shape())

    def numel(self) -> int:
        n = 1
        for s in self.shape():
            n *= s
        return n

    def __add__(self, o):
        return self.prog._bin("add", self, o)

    def __radd__(self, o):
        return self.prog._bin("add", o, self)

    def __sub__(self, o):
        return self.prog._bin("subtract", self, o)

    def __rsub__(self, o):
        return self.prog._bin("subtract", o, self)

    def __mul__(self, o):
        return self.prog._bin("multiply", self, o)

    def __rmul__(self, o):
        return self.prog._bin("multiply", o, self)

    def __truediv__(self, o):
        return self.prog._bin("divide", self, o)

    def __rtruediv__(self, o):
        return self.prog._bin("divide", o, self)

    def __getitem__(self, key):
        if not self.is_tensor:
            raise TypeError("indexing applies to tensors (tensor::operator[])")
        if not isinstance(key, tuple):
            key = (key,)
        specs = []
        for k in key:
            if k is ALL or (hasattr(k, "__class__") and k.__class__.__name__ == "_All"):
                specs.append("a")
            elif isinstance(k, slice):
                start = 0 if k.start is None else int(k.start)
                stop = 2**62 if k.stop is None else int(k.stop)
                step = 1 if k.step is None else int(k.step)
                specs.append(f"s{start}:{stop}:{step}")
            else:
                specs.append(f"i{int(k)}")
        return self.prog._emit(f"index {self.id} {';'.join(specs) or '-'}", deps=(self.id,))

    def cpu(self) -> np.ndarray:
        return self.prog.evaluate(self)


class Program:
    """Records porch API calls for the oracle; mirrors porch_b200.api."""

    all = ALL

    def __init__(self, threads: int | None = None):
        self.lines: list[str] = []
        self.deps: list[tuple[int, ...]] = []
        self.inputs: list[np.ndarray] = []
        self.threads = threads or os.cpu_count() or 1

    # -- plumbing
    def _emit(self, text: str, is_tensor: bool = False, deps: tuple[int, ...] = ()) -> Node:
        vid = len(self.lines)
        self.lines.append(f"{vid} {text}")
        self.deps.append(deps)
        return Node(self, vid, is_tensor)

    def _val(self, x) -> Node:
        if isinstance(x, Node):
            return x
        if isinstance(x, (int, float, np.floating, np.integer)):
            bits = struct.unpack("<I", struct.pack("<f", float(x)))[0]
            return self._emit(f"scalar {bits:08x}")
        raise TypeError(f"cannot convert {type(x).__name__}")

    def _bin(self, op: str, a, b) -> Node:
        a, b = self._val(a), self._val(b)
        return self._emit(f"{op} {a.id} {b.id}", deps=(a.id, b.id))

    def _un(self, op: str, a) -> Node:
        a = self._val(a)
        return self._emit(f"{op} {a.id}", deps=(a.id,))

    def program_text(self, upto: Node) -> str:
        """The lines `upto` depends on, in recording order."""
        need = set()
        stack = [upto.id]
        while stack:
            v = stack.pop()
            if v in need:
                continue
            need.add(v)
            stack.extend(self.deps[v])
        return "\n".join(self.lines[i] for i in sorted(need)) + "\n"

    def _marshal(self):
        n = len(self.inputs)
        ptrs = (c_void_p * _builtins.max(1, n))()
        shapes = (POINTER(c_int64) * _builtins.max(1, n))()
        ranks = (c_size_t * _builtins.max(1, n))()
        keep = []
        for i, arr in enumerate(self.inputs):
            ptrs[i] = arr.ctypes.data_as(c_void_p)
            sh = (c_int64 * _builtins.max(1, arr.ndim))(*arr.shape)
            keep.append(sh)
            shapes[i] = ctypes.cast(sh, POINTER(c_int64))
            ranks[i] = arr.ndim
        return ptrs, shapes, ranks, keep

    def shape_of(self, node: Node) -> list[int]:
        ptrs, shapes, ranks, keep = self._marshal()
        out = (c_int64 * 16)()
        rank = c_size_t(0)
        st = lib().oracle_shape(self.program_text(node).encode(), ptrs, shapes, ranks,
                                len(self.inputs), out, 16, ctypes.byref(rank))
        if st:
            _raise(st)
        return [out[i] for i in range(rank.value)]

    def evaluate(self, node: Node) -> np.ndarray:
        shape = self.shape_of(node)
        n = 1
        for s in shape:
            n *= s
        out = np.empty(n, dtype=np.float32)
        ptrs, shapes, ranks, keep = self._marshal()
        st = lib().oracle_eval(self.program_text(node).encode(), ptrs, shapes, ranks,
                               len(self.inputs), out.ctypes.data_as(POINTER(c_float)), n,
                               int(self.threads))
        if st:
            _raise(st)
        return out.reshape(shape)

    # -- the porch API
    def tensor(self, shape: Sequence[int], values, device: int = 0) -> Node:
        arr = np.ascontiguousarray(np.asarray(values, dtype=np.float32)).reshape(-1)
        expected = 1
        for s in shape:
            if s < 0:
                raise OracleInvalidArgument("tensor shape extents must be non-negative")
            expected *= int(s)
        if arr.size != expected:
            raise OracleInvalidArgument("tensor data size does not match shape")
        self.inputs.append(arr.reshape([int(s) for s in shape]))
        return self._emit(f"input {len(self.inputs) - 1}", is_tensor=True)

    def full(self, shape, value, device: int = 0) -> Node:
        n = 1
        for s in shape:
            n *= int(s)
        return self.tensor(shape, np.full(n, value, dtype=np.float32), device)

    def zeros(self, shape, device: int = 0) -> Node:
        return self.full(shape, 0.0, device)

    def as_tensor(self, e) -> Node:
        e = self._val(e)
        return self._emit(f"tensor {e.id}", is_tensor=True, deps=(e.id,))

    def materialize(self, e) -> Node:
        e = self._val(e)
        return self._emit(f"materialize {e.id}", is_tensor=True, deps=(e.id,))

    def add(self, a, b):
        return self.materialize(self._bin("add", a, b))

    def subtract(self, a, b):
        return self.materialize(self._bin("subtract", a, b))

    def multiply(self, a, b):
        return self.materialize(self._bin("multiply", a, b))

    def divide(self, a, b):
        return self.materialize(self._bin("divide", a, b))

    def matmul(self, a, b):
        return self._bin("matmul", a, b)

    def maximum(self, a, b):
        return self._bin("maximum", a, b)

    def minimum(self, a, b):
        return self._bin("minimum", a, b)

    def exp(self, a):
        return self._un("exp", a)

    def reciprocal(self, a):
        return self._un("reciprocal", a)

    def transpose(self, a):
        return self._un("transpose", a)

    def relu(self, a):
        return self._un("relu", a)

    def logistic(self, a):
        return self._un("logistic", a)

    def reshape(self, a, shape):
        dims = ",".join(str(int(s)) for s in shape) or "-"
        a = self._val(a)
        return self._emit(f"reshape {a.id} {dims}", deps=(a.id,))

    def broadcast_to(self, a, shape):
        dims = ",".join(str(int(s)) for s in shape) or "-"
        a = self._val(a)
        return self._emit(f"broadcast {a.id} {dims}", deps=(a.id,))

    def unsqueeze(self, a, axis: int):
        a = self._val(a)
        return self._emit(f"unsqueeze {a.id} {int(axis)}", deps=(a.id,))

    def concat(self, a, b, axis: int):
        a, b = self._val(a), self._val(b)
        return self._emit(f"concat {a.id} {b.id} {int(axis)}", deps=(a.id, b.id))

    def sum(self, a, axis: int, keepdim: bool = False):  # noqa: A003
        a = self._val(a)
        return self._emit(f"sum {a.id} {int(axis)} {int(bool(keepdim))}", deps=(a.id,))

    def max(self, a, axis: int, keepdim: bool = False):  # noqa: A003
        a = self._val(a)
        return self._emit(f"max {a.id} {int(axis)} {int(bool(keepdim))}", deps=(a.id,))

    def softmax(self, a, axis: int):
        a = self._val(a)
        return self._emit(f"softmax {a.id} {int(axis)}", deps=(a.id,))
