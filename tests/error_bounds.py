"""Forward error bounds of fp32 evaluation, for the parity tests' inexact
programs.

A relative bar (1e-5 per element) cannot hold where a result cancels: a sum
of signed terms, exp(x) - y or a matmul row whose products cancel to near
zero has no fp32 evaluation order whose result is within 1e-5 of a tiny
exact value. For those elements the tests use a rigorous bound instead:
`evaluate(program, inputs)` replays the program in fp64 (numpy) and carries,
next to every value v, an absolute bound e on how far ANY fp32 evaluation of
the same graph (each operation rounded once to nearest, sums and matmul
accumulated in any order) can be from v. Both the product and the oracle are
such evaluations, so |got - oracle| <= 2 e.

Rules (u = 2^-24, unit roundoff of fp32; e_x the operands' bounds):
- x + y, x - y: e_x + e_y + u|v|
- x * y:        |y| e_x + |x| e_y + e_x e_y + u|v|
- x / y:        (e_x + |v| e_y) / (|y| - e_y) + u|v|   (unbounded if |y| <= e_y)
- exp(x):       exp(x) (expm1(e_x) + c(x) exp(e_x)), c(x) = 8u + 2u|x|: the
                fast exponential (src/tensor.cpp:857 uses __expf) rounds
                x * log2(e) (relative u, i.e. u|x| in the result) and then
                approximates 2^y within a few ulp
- maximum, minimum, relu, max over an axis: the largest operand bound
  (a selection is exact; a perturbed comparison picks a value within it)
- sum of n terms: sum e_i + (n - 1) u sum |v_i|  (any order)
- matmul over K: |A| e_B + e_A |B| + e_A e_B + (2K + 4) u |A||B|  (any
  accumulation order, plus the 3xTF32 split: the dropped lo*lo term and the
  rounding of lo are each <= 2^-22 of a product)
- logistic and softmax as their defining graphs (src/ops.cpp:5-18), softmax
  with one more rounding for a reciprocal-then-multiply normalisation
- data movement (slice, transpose, reshape, broadcast, unsqueeze, concat)
  moves bounds with values.
Results below the normal range may flush to zero: every exp adds 2^-126.
"""

from __future__ import annotations

import numpy as np

U = 2.0 ** -24
TINY = 2.0 ** -126


class _V:
    __slots__ = ("v", "e", "scalar")

    def __init__(self, v, e, scalar=False):
        self.v = v
        self.e = e
        self.scalar = scalar


def _div(a: _V, b: _V) -> _V:
    with np.errstate(all="ignore"):
        v = a.v / b.v
        den = np.abs(b.v) - b.e
        e = np.where(den > 0, (a.e + np.abs(v) * b.e) / np.where(den > 0, den, 1.0), np.inf) + U * np.abs(v)
    return _V(v, e, a.scalar and b.scalar)


def _exp(a: _V) -> _V:
    with np.errstate(all="ignore"):
        v = np.exp(a.v)
        c = 8 * U + 2 * U * np.abs(a.v)
        e = v * (np.expm1(a.e) + c * np.exp(a.e)) + TINY
    return _V(v, e, a.scalar)


def _add(a: _V, b: _V, sign: float = 1.0) -> _V:
    with np.errstate(all="ignore"):
        v = a.v + sign * b.v
        e = a.e + b.e + U * np.abs(v)
    return _V(v, e, a.scalar and b.scalar)


def _mul(a: _V, b: _V) -> _V:
    with np.errstate(all="ignore"):
        v = a.v * b.v
        e = np.abs(b.v) * a.e + np.abs(a.v) * b.e + a.e * b.e + U * np.abs(v)
    return _V(v, e, a.scalar and b.scalar)


def _select(a: _V, b: _V, take_a) -> _V:
    va, vb = np.broadcast_arrays(np.asarray(a.v, np.float64), np.asarray(b.v, np.float64))
    ea, eb = np.broadcast_arrays(np.asarray(a.e, np.float64), np.asarray(b.e, np.float64))
    v = np.where(take_a(va, vb), va, vb)
    return _V(v, np.maximum(ea, eb), a.scalar and b.scalar)


def _reduce_shape(r, keepdim: bool):
    r = np.asarray(r)
    return r.reshape(1) if r.ndim == 0 else r


def _sum(a: _V, axis: int, keepdim: bool) -> _V:
    n = a.v.shape[axis]
    v = np.sum(a.v, axis=axis, keepdims=keepdim)
    e = np.sum(a.e, axis=axis, keepdims=keepdim) + max(n - 1, 0) * U * np.sum(np.abs(a.v), axis=axis,
                                                                              keepdims=keepdim)
    return _V(_reduce_shape(v, keepdim), _reduce_shape(e, keepdim))


def _max(a: _V, axis: int, keepdim: bool) -> _V:
    v = np.max(a.v, axis=axis, keepdims=keepdim)
    e = np.max(a.e, axis=axis, keepdims=keepdim)
    return _V(_reduce_shape(v, keepdim), _reduce_shape(e, keepdim))


def _matmul(a: _V, b: _V) -> _V:
    k = a.v.shape[1]
    aa, ab = np.abs(a.v), np.abs(b.v)
    with np.errstate(all="ignore"):
        v = a.v @ b.v
        e = aa @ b.e + a.e @ ab + a.e @ b.e + (2 * k + 4) * U * (aa @ ab)
    return _V(v, e)


def _map(a: _V, f) -> _V:
    return _V(f(np.asarray(a.v)), f(np.asarray(a.e)), a.scalar)


def _softmax(x: _V, axis: int) -> _V:
    m = _max(x, axis, True)
    d = _add(x, _V(np.broadcast_to(m.v, x.v.shape), np.broadcast_to(m.e, x.v.shape)), -1.0)
    ex = _exp(d)
    s = _sum(ex, axis, True)
    out = _div(ex, _V(np.broadcast_to(s.v, x.v.shape), np.broadcast_to(s.e, x.v.shape)))
    out.e = out.e + U * np.abs(out.v)
    return out


def _logistic(x: _V) -> _V:
    zero = _V(np.float64(0.0), np.float64(0.0), True)
    one = _V(np.float64(1.0), np.float64(0.0), True)
    return _div(one, _add(one, _exp(_add(zero, x, -1.0))))


def evaluate(program: str, inputs) -> tuple[np.ndarray, np.ndarray]:
    """Returns (value, bound) of the program's last node, both float64 arrays
    of its shape."""
    vals: dict[int, _V] = {}
    last = None
    for line in program.strip().splitlines():
        p = line.split()
        vid, op, a = int(p[0]), p[1], p[2:]

        def v(k):
            return vals[int(a[k])]

        if op == "input":
            x = np.asarray(inputs[int(a[0])], dtype=np.float32).astype(np.float64)
            r = _V(x, np.zeros_like(x))
        elif op == "scalar":
            s = float(np.frombuffer(bytes.fromhex(a[0])[::-1], dtype=np.float32)[0])
            r = _V(np.float64(s), np.float64(0.0), True)
        elif op == "add":
            r = _add(v(0), v(1))
        elif op == "subtract":
            r = _add(v(0), v(1), -1.0)
        elif op == "multiply":
            r = _mul(v(0), v(1))
        elif op == "divide":
            r = _div(v(0), v(1))
        elif op == "reciprocal":
            r = _div(_V(np.float64(1.0), np.float64(0.0), True), v(0))
        elif op == "maximum":
            r = _select(v(0), v(1), lambda x, y: x > y)
        elif op == "minimum":
            r = _select(v(0), v(1), lambda x, y: x < y)
        elif op == "relu":
            r = _select(v(0), _V(np.float64(0.0), np.float64(0.0), True), lambda x, y: x > y)
        elif op == "exp":
            r = _exp(v(0))
        elif op == "logistic":
            r = _logistic(v(0))
        elif op == "softmax":
            r = _softmax(v(0), int(a[1]))
        elif op == "matmul":
            r = _matmul(v(0), v(1))
        elif op == "transpose":
            r = _map(v(0), lambda x: np.ascontiguousarray(x.T))
        elif op == "reshape":
            dims = [] if a[1] == "-" else [int(s) for s in a[1].split(",")]
            r = _map(v(0), lambda x: x.reshape(dims))
        elif op == "broadcast":
            dims = [int(s) for s in a[1].split(",")]
            r = _map(v(0), lambda x: np.broadcast_to(x, dims).copy())
        elif op == "unsqueeze":
            r = _map(v(0), lambda x: np.expand_dims(x, int(a[1])))
        elif op == "concat":
            ax = int(a[2])
            r = _V(np.concatenate([v(0).v, v(1).v], axis=ax), np.concatenate([v(0).e, v(1).e], axis=ax))
        elif op == "sum":
            r = _sum(v(0), int(a[1]), bool(int(a[2])))
        elif op == "max":
            r = _max(v(0), int(a[1]), bool(int(a[2])))
        elif op in ("tensor", "materialize"):
            r = v(0)
        elif op == "index":
            key = []
            for sp in ([] if a[1] == "-" else a[1].split(";")):
                if sp[0] == "i":
                    key.append(int(sp[1:]))
                elif sp[0] == "s":
                    s0, s1, s2 = (int(t) for t in sp[1:].split(":"))
                    key.append(slice(s0, s1, s2))
                else:
                    key.append(slice(None))
            r = _map(v(0), lambda x: np.ascontiguousarray(x[tuple(key)]))
        else:
            raise ValueError(op)
        vals[vid] = r
        last = r
    return np.asarray(last.v, np.float64), np.asarray(last.e, np.float64)


def check(got: np.ndarray, want: np.ndarray, bound: np.ndarray, rel: float, what: str) -> dict:
    """Every element must be within `rel` of `want` (relative), or, where
    cancellation makes that bar unattainable, within 2 x the forward error
    bound of fp32 evaluation. Non-finite results must agree in class.
    Returns how many elements needed the second bar."""
    want = np.asarray(want, np.float64)
    bound = np.broadcast_to(np.asarray(bound, np.float64), want.shape).reshape(-1)
    got = np.asarray(got, np.float64).reshape(-1)
    want = want.reshape(-1)
    fin = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), fin), f"{what}: finite/non-finite pattern differs"
    nan_w, nan_g = np.isnan(want), np.isnan(got)
    assert np.array_equal(nan_w, nan_g), f"{what}: NaN pattern differs"
    inf = ~fin & ~nan_w
    assert np.array_equal(np.sign(got[inf]), np.sign(want[inf])), f"{what}: infinities differ in sign"
    err = np.abs(got - want)
    rel_ok = err <= rel * np.abs(want) + 1e-30
    fwd_ok = err <= 2 * bound + 1e-30
    bad = fin & ~rel_ok & ~fwd_ok
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} of {got.size} elements exceed both the {rel} relative "
                             f"bar and the fp32 forward bound; first at {i}: got {got[i]!r} want {want[i]!r} "
                             f"bound {bound[i]:.3e}")
    return {"elements": int(got.size), "cancellation_bound": int((fin & ~rel_ok).sum())}
