"""Parity against outputs of the reference itself (tests/golden/ref_golden.*,
produced by tests/golden/make_ref_golden.py running AkhilSamavedam/porch's
own NVRTC-JIT path, compiled from its sources, on a B200).

Criteria (tests/tolerances.py):
- programs of IEEE-exact operations only: bit for bit, oracle and CUDA path;
- exp/logistic elementwise graphs: bit for bit on the CUDA path (both it and
  the reference use the __expf intrinsic, src/tensor.cpp:857), within
  REL_TOL for the host oracle (libm expf);
- sum / softmax (no matmul): relative error <= REL_TOL per element;
- programs with a matmul: |got - want| <= MATMUL_TOL * sqrt(K_MAX) *
  max(|want|, rms(want)); every matmul in these fixtures has K <= 128.
"""

import json
from pathlib import Path

import numpy as np
import pytest

import graphs
from tolerances import MATMUL_TOL, REL_TOL, assert_bitwise, assert_relative

GOLDEN = Path(__file__).parent / "golden"
MANIFEST = json.loads((GOLDEN / "ref_golden.json").read_text())["cases"]
ARRAYS = np.load(GOLDEN / "ref_golden.npz")
K_MAX = 128
IDS = [c["name"] for c in MANIFEST]


def _ops(program):
    return {line.split()[1] for line in program.strip().splitlines()}


def _case(i):
    c = MANIFEST[i]
    ins = [ARRAYS[f"c{i}_in{j}"] for j in range(c["n_inputs"])]
    out = ARRAYS[f"c{i}_out"] if c["error"] is None else None
    return c, ins, out


def _assert_matmul_close(got, want, what):
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    assert got.shape == want.shape, what
    fin = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), fin), what
    if not fin.any():
        return
    rms = float(np.sqrt(np.mean(want[fin] ** 2)))
    scale = np.maximum(np.abs(want[fin]), rms)
    scale = np.where(scale == 0, 1.0, scale)
    err = float(np.max(np.abs(got[fin] - want[fin]) / scale))
    assert err <= MATMUL_TOL * np.sqrt(K_MAX), (what, err)


def _compare(got, want, ops, exp_bitwise, what):
    assert list(got.shape) == list(want.shape), what
    if not ops & {"exp", "logistic", "sum", "softmax", "matmul"}:
        assert_bitwise(got, want, what)
    elif "matmul" in ops:
        _assert_matmul_close(got, want, what)
    elif exp_bitwise and not ops & {"sum", "softmax"}:
        assert_bitwise(got, want, what)
    else:
        assert_relative(got, want, REL_TOL, what)


def test_fixtures_cover_the_reference_paths():
    kinds = set()
    for c in MANIFEST:
        kinds |= _ops(c["program"])
    assert {"matmul", "softmax", "sum", "max", "concat", "index", "transpose", "broadcast",
            "reshape", "unsqueeze", "exp", "logistic", "relu", "materialize"} <= kinds
    assert len(MANIFEST) >= 100
    assert sum(c["error"] is None for c in MANIFEST) >= 100


@pytest.mark.parametrize("i", range(len(MANIFEST)), ids=IDS)
def test_oracle_against_reference_outputs(oracle_lib, i):
    c, ins, want = _case(i)
    if c["error"]:
        with pytest.raises(ValueError):
            graphs.evaluate_oracle(c["program"], ins)
        return
    got = graphs.evaluate_oracle(c["program"], ins)
    _compare(got, want, _ops(c["program"]), False, c["name"])


@pytest.mark.gpu
@pytest.mark.parametrize("i", range(len(MANIFEST)), ids=IDS)
def test_cuda_path_against_reference_outputs(gpu, i):
    c, ins, want = _case(i)
    if c["error"]:
        with pytest.raises(ValueError):
            graphs.evaluate_product(gpu, c["program"], ins)
        return
    got = graphs.evaluate_product(gpu, c["program"], ins)
    _compare(got, want, _ops(c["program"]), True, c["name"])
