"""Graph programs shared by the three arms of the parity tests.

A program is the oracle's text format (one porch API call per line, see
oracle/oracle.cpp). `build(M, program, inputs)` replays it through a module M
with porch's API: porch_b200.api (the product), an oracle.graph.Program (the
host oracle) — and oracle/ref_runner.cpp replays the same text through the
reference's C++ API on the GPU box.
"""

from __future__ import annotations

import random
import struct
from typing import Sequence

import numpy as np


def scalar_hex(x: float) -> str:
    return f"{struct.unpack('<I', struct.pack('<f', float(x)))[0]:08x}"


def build(M, program: str, inputs: Sequence[np.ndarray]):
    """Replays `program` through module M; returns the last value."""
    tensors = [M.tensor(list(a.shape), a.reshape(-1)) for a in inputs]
    vals: dict[int, object] = {}
    last = None
    for line in program.strip().splitlines():
        parts = line.split()
        vid, op, args = int(parts[0]), parts[1], parts[2:]
        v = lambda k: vals[int(args[k])]  # noqa: E731
        if op == "input":
            out = tensors[int(args[0])]
        elif op == "scalar":
            out = struct.unpack("<f", struct.pack("<I", int(args[0], 16)))[0]
        elif op in ("add", "subtract", "multiply", "divide"):
            a, b = v(0), v(1)
            out = {"add": lambda: a + b, "subtract": lambda: a - b,
                   "multiply": lambda: a * b, "divide": lambda: a / b}[op]()
        elif op in ("maximum", "minimum", "matmul"):
            out = getattr(M, op)(v(0), v(1))
        elif op in ("exp", "reciprocal", "transpose", "relu", "logistic"):
            out = getattr(M, op)(v(0))
        elif op == "softmax":
            out = M.softmax(v(0), int(args[1]))
        elif op in ("reshape", "broadcast"):
            dims = [] if args[1] == "-" else [int(x) for x in args[1].split(",")]
            out = M.reshape(v(0), dims) if op == "reshape" else M.broadcast_to(v(0), dims)
        elif op == "unsqueeze":
            out = M.unsqueeze(v(0), int(args[1]))
        elif op == "concat":
            out = M.concat(v(0), v(1), int(args[2]))
        elif op in ("sum", "max"):
            out = getattr(M, op)(v(0), int(args[1]), bool(int(args[2])))
        elif op == "tensor":
            out = M.as_tensor(v(0))
        elif op == "materialize":
            out = M.materialize(v(0))
        elif op == "index":
            spec = args[1]
            key = []
            for sp in ([] if spec == "-" else spec.split(";")):
                if sp[0] == "i":
                    key.append(int(sp[1:]))
                elif sp[0] == "s":
                    a, b, c = (int(x) for x in sp[1:].split(":"))
                    key.append(slice(a, b, c))
                else:
                    key.append(M.all)
            out = v(0)[tuple(key)]
        else:
            raise ValueError(op)
        vals[vid] = out
        last = out
    return last


def evaluate_product(api, program: str, inputs: Sequence[np.ndarray]) -> np.ndarray:
    out = build(api, program, inputs)
    t = api.materialize(out)
    return t.cpu().reshape(t.shape())


def evaluate_oracle(program: str, inputs: Sequence[np.ndarray], threads: int | None = None) -> np.ndarray:
    from oracle.graph import Program

    P = Program(threads=threads)
    out = build(P, program, inputs)
    if not hasattr(out, "id"):
        raise ValueError("program output is a scalar")
    return P.evaluate(out)


# ------------------------------------------------------------- fuzzing ----
class _Gen:
    """Random well-formed programs over small shapes."""

    def __init__(self, rng: random.Random, integer_values: bool, large: bool = False):
        self.rng = rng
        self.lines: list[str] = []
        self.inputs: list[np.ndarray] = []
        self.integer_values = integer_values
        self.has_inexact = False
        # Large mode: extents up to thousands (at most LARGE_LIMIT elements
        # per operand); the default draws are unchanged, seed for seed.
        self.large = large

    LARGE_LIMIT = 1 << 21

    def _too_big(self, shape) -> bool:
        return self.large and int(np.prod(shape)) > self.LARGE_LIMIT

    def emit(self, text: str) -> int:
        self.lines.append(f"{len(self.lines)} {text}")
        return len(self.lines) - 1

    def new_input(self, shape: list[int]) -> int:
        n = int(np.prod(shape)) if shape else 1
        if self.integer_values:
            vals = np.array([self.rng.randint(-8, 8) for _ in range(n)], dtype=np.float32)
        else:
            vals = np.array([self.rng.uniform(-2, 2) for _ in range(n)], dtype=np.float32)
        self.inputs.append(vals.reshape(shape))
        return self.emit(f"input {len(self.inputs) - 1}")

    def rand_shape(self) -> list[int]:
        if self.large:
            r = self.rng.choice([1, 2, 2, 3])
            ext = {1: [1000, 4096, 65536], 2: [1, 3, 64, 100, 257, 512], 3: [1, 3, 16, 33, 64]}[r]
            return [self.rng.choice(ext) for _ in range(r)]
        r = self.rng.choice([1, 2, 2, 2, 3])
        return [self.rng.choice([1, 2, 3, 4, 5, 7, 8, 16, 33]) for _ in range(r)]

    def expr(self, shape: list[int], depth: int) -> int:
        """An expression of exactly `shape`."""
        rng = self.rng
        if depth <= 0 or rng.random() < 0.25:
            return self.new_input(shape)
        choice = rng.random()
        if choice < 0.35:
            op = rng.choice(["add", "subtract", "multiply", "maximum", "minimum", "divide"])
            a = self.expr(shape, depth - 1)
            if rng.random() < 0.3:
                b = self.emit(f"scalar {scalar_hex(rng.choice([0.5, 2.0, -1.0, 3.0, 0.25]))}")
                if rng.random() < 0.5:
                    a, b = b, a
            else:
                b = self.expr(shape, depth - 1)
            return self.emit(f"{op} {a} {b}")
        if choice < 0.45 and len(shape) == 2:
            # transpose of a transposed-shape expression
            a = self.expr([shape[1], shape[0]], depth - 1)
            return self.emit(f"transpose {a}")
        if choice < 0.55:
            # broadcast from a smaller source
            src = [s if rng.random() < 0.5 else 1 for s in shape]
            drop = rng.randint(0, len(src) - 1) if len(src) > 1 and rng.random() < 0.4 else 0
            src = src[drop:]
            a = self.expr(src, depth - 1)
            return self.emit(f"broadcast {a} {','.join(map(str, shape))}")
        if choice < 0.65:
            # slice of a realised/lazy tensor: grow each dim, then slice back
            steps = [rng.choice([1, 1, 2, 3]) for _ in shape]
            starts = [rng.randint(0, 2) for _ in shape]
            big = [st + (s - 1) * k + 1 + rng.randint(0, 2) for s, st, k in zip(shape, starts, steps)]
            if self._too_big(big):
                return self.new_input(shape)
            a = self.expr(big, depth - 1)
            t = self.emit(f"tensor {a}")
            spec = ";".join(f"s{st}:{st + (s - 1) * k + 1}:{k}" for s, st, k in zip(shape, starts, steps))
            return self.emit(f"index {t} {spec}")
        if choice < 0.72:
            # concat along a random axis
            ax = rng.randrange(len(shape))
            if shape[ax] >= 2:
                cut = rng.randint(1, shape[ax] - 1)
                l = list(shape)
                r = list(shape)
                l[ax] = cut
                r[ax] = shape[ax] - cut
                a = self.expr(l, depth - 1)
                b = self.expr(r, depth - 1)
                return self.emit(f"concat {a} {b} {ax}")
            return self.new_input(shape)
        if choice < 0.78:
            # reshape from a different factorisation
            n = int(np.prod(shape))
            src = [n] if len(shape) > 1 else ([1, n] if rng.random() < 0.5 else [n])
            a = self.expr(src, depth - 1)
            return self.emit(f"reshape {a} {','.join(map(str, shape))}")
        if choice < 0.84 and any(s == 1 for s in shape):
            ax = shape.index(1)
            a = self.expr(shape[:ax] + shape[ax + 1:], depth - 1) if len(shape) > 1 else self.new_input([])
            return self.emit(f"unsqueeze {a} {ax}")
        if choice < 0.9:
            # reduction producing `shape`
            ax = rng.randrange(len(shape) + 1)
            keep = rng.random() < 0.5
            n = rng.choice([1, 33, 257, 1000] if self.large else [1, 3, 8, 33])
            if keep:
                if ax >= len(shape) or shape[ax] != 1:
                    return self.new_input(shape)
                src = list(shape)
                src[ax] = n
            else:
                src = shape[:ax] + [n] + shape[ax:]
                if len(shape) == 1 and shape[0] == 1 and rng.random() < 0.5:
                    src = [n]
                    ax = 0
            if self._too_big(src):
                return self.new_input(shape)
            a = self.expr(src, depth - 1)
            op = rng.choice(["sum", "max"])
            if op == "sum":
                self.has_inexact = True
            return self.emit(f"{op} {a} {ax} {int(keep)}")
        if choice < 0.95:
            a = self.expr(shape, depth - 1)
            op = rng.choice(["relu", "exp", "logistic", "reciprocal"])
            if op in ("exp", "logistic"):
                self.has_inexact = True
            return self.emit(f"{op} {a}")
        if len(shape) == 2:
            k = rng.choice([8, 64, 300] if self.large else [1, 3, 8, 17])
            a = self.expr([shape[0], k], depth - 1)
            b = self.expr([k, shape[1]], depth - 1)
            self.has_inexact = True
            return self.emit(f"matmul {a} {b}")
        return self.new_input(shape)


def random_program(seed: int, integer_values: bool = True, depth: int = 4, large: bool = False):
    """Returns (program text, inputs, exact). `exact` says the program uses
    only operations whose fp32 result is fixed by IEEE rounding (+ - * /,
    reciprocal, maximum/minimum, max reductions and data movement), so the
    product must match the oracle bit for bit; exp, sum, softmax and matmul
    are compared with a tolerance."""
    rng = random.Random(seed)
    g = _Gen(rng, integer_values, large)
    shape = g.rand_shape()
    root = g.expr(shape, depth)
    if rng.random() < 0.15 and len(shape) >= 1:
        # Mostly the last axis (the row kernel); otherwise any axis (the
        # pattern then lowers as reductions plus an elementwise pass).
        ax = len(shape) - 1 if rng.random() < 0.6 else rng.randrange(len(shape))
        root = g.emit(f"softmax {root} {ax}")
        g.has_inexact = True
    text = "\n".join(g.lines) + "\n"
    return text, g.inputs, not g.has_inexact
