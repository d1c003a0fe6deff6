"""The host oracle against the reference's own known answers
(tests/golden/known_answers.json, from AkhilSamavedam/porch
tests/tensor_test.cpp) and against an independent numpy restatement."""

import json
from pathlib import Path

import numpy as np
import pytest

import graphs
from tolerances import assert_bitwise

GOLDEN = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())["cases"]


def _inputs(case):
    return [np.asarray(v, dtype=np.float32).reshape(s) for s, v in case["inputs"]]


@pytest.mark.parametrize("case", GOLDEN, ids=[c["name"] for c in GOLDEN])
def test_oracle_known_answers(oracle_lib, case):
    ins = _inputs(case)
    if case["error"]:
        with pytest.raises(ValueError):
            graphs.evaluate_oracle(case["program"], ins)
        return
    got = graphs.evaluate_oracle(case["program"], ins)
    if case["shape"] is not None:
        assert list(got.shape) == case["shape"]
    if case["expect"] is not None:
        assert_bitwise(got, np.asarray(case["expect"], dtype=np.float32), case["name"])
    if case["interval"] is not None:
        flat = got.reshape(-1)
        for i, (lo, hi) in enumerate(case["interval"]):
            assert lo <= flat[i] <= hi, (case["name"], i, flat[i])
    for i, v in (case["exact_at"] or {}).items():
        assert got.reshape(-1)[int(i)] == np.float32(v)


def test_oracle_rejects_like_reference(oracle_lib):
    from oracle.graph import OracleInvalidArgument, OracleOutOfRange, Program

    P = Program()
    a = P.tensor([2, 3], np.zeros(6))
    b = P.tensor([2, 2], np.zeros(4))
    with pytest.raises(OracleInvalidArgument, match="shapes must match"):
        P.evaluate(a + b)
    with pytest.raises(OracleInvalidArgument, match="inner dimensions"):
        P.evaluate(P.matmul(a, b))
    with pytest.raises(OracleInvalidArgument, match="rank-2"):
        P.evaluate(P.transpose(P.reshape(a, [6])))
    with pytest.raises(OracleOutOfRange):
        P.evaluate(a[5])
    with pytest.raises(OracleInvalidArgument, match="step must be positive"):
        P.evaluate(a[slice(0, 2, 0)])
    with pytest.raises(OracleInvalidArgument, match="data size"):
        P.tensor([2, 2], np.zeros(3))


def _numpy_eval(program, inputs):
    """Independent numpy restatement of the same semantics (used only to
    cross-check the C++ oracle on exact programs)."""
    vals = {}
    tensors = {}
    for line in program.strip().splitlines():
        p = line.split()
        vid, op, a = int(p[0]), p[1], p[2:]
        v = lambda k: vals[int(a[k])]  # noqa: E731
        if op == "input":
            r = inputs[int(a[0])].astype(np.float32)
        elif op == "scalar":
            r = np.frombuffer(bytes.fromhex(a[0])[::-1], dtype=np.float32)[0]
        elif op in ("add", "subtract", "multiply", "divide"):
            x, y = np.float32(v(0)) if np.ndim(v(0)) == 0 else v(0), v(1)
            with np.errstate(all="ignore"):
                r = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply,
                     "divide": np.divide}[op](x, y, dtype=np.float32)
        elif op == "maximum":
            x, y = np.broadcast_arrays(np.float32(v(0)), np.float32(v(1)))
            r = np.where(x > y, x, y).astype(np.float32)
        elif op == "minimum":
            x, y = np.broadcast_arrays(np.float32(v(0)), np.float32(v(1)))
            r = np.where(x < y, x, y).astype(np.float32)
        elif op == "reciprocal":
            with np.errstate(all="ignore"):
                r = np.divide(np.float32(1.0), v(0), dtype=np.float32)
        elif op == "relu":
            x = v(0)
            r = np.where(x > 0, x, np.float32(0)).astype(np.float32)
        elif op == "transpose":
            r = np.ascontiguousarray(v(0).T)
        elif op == "reshape":
            r = v(0).reshape([int(s) for s in a[1].split(",")])
        elif op == "broadcast":
            r = np.broadcast_to(v(0), [int(s) for s in a[1].split(",")]).copy()
        elif op == "unsqueeze":
            r = np.expand_dims(v(0), int(a[1]))
        elif op == "concat":
            r = np.concatenate([v(0), v(1)], axis=int(a[2]))
        elif op == "max":
            r = np.max(v(0), axis=int(a[1]), keepdims=bool(int(a[2])))
            if r.ndim == 0:
                r = r.reshape(1)
        elif op == "tensor":
            r = v(0)
        elif op == "index":
            x = v(0)
            key = []
            for sp in a[1].split(";"):
                if sp[0] == "i":
                    key.append(int(sp[1:]))
                elif sp[0] == "s":
                    s0, s1, s2 = (int(t) for t in sp[1:].split(":"))
                    key.append(slice(s0, s1, s2))
                else:
                    key.append(slice(None))
            r = np.ascontiguousarray(x[tuple(key)])
        else:
            return None
        vals[vid] = r
    return vals[max(vals)]


@pytest.mark.parametrize("seed", range(60))
def test_oracle_matches_numpy_restatement(oracle_lib, seed):
    text, ins, exact = graphs.random_program(seed)
    if not exact:
        pytest.skip("inexact program")
    want = _numpy_eval(text, ins)
    if want is None:
        pytest.skip("op outside the numpy restatement")
    got = graphs.evaluate_oracle(text, ins)
    assert_bitwise(got, np.broadcast_to(want, got.shape), f"seed {seed}")
