"""The forward error bounds (tests/error_bounds.py) pinned on the CPU: the
host oracle is itself an fp32 evaluation of each program (operations
rounded once, exp/sums/matmul accumulated in double and rounded), so it must
lie within the bound of the fp64 restatement's value on every element, for
the same random programs the GPU parity tests use."""

import numpy as np
import pytest

import error_bounds
import graphs


def _holds(text, ins):
    want = graphs.evaluate_oracle(text, ins).astype(np.float64)
    v, e = error_bounds.evaluate(text, ins)
    assert np.shape(v) == want.shape, (np.shape(v), want.shape)
    e = np.broadcast_to(e, want.shape).reshape(-1)
    want, v = want.reshape(-1), np.asarray(v).reshape(-1)
    fin = np.isfinite(want) & np.isfinite(v)
    err = np.abs(want[fin] - v[fin])
    assert np.all(err <= e[fin] + 1e-30), float(np.max(err - e[fin]))
    return fin


@pytest.mark.parametrize("seed", range(160))
def test_oracle_within_forward_bound(oracle_lib, seed):
    text, ins, _ = graphs.random_program(seed, integer_values=seed % 2 == 0)
    try:
        graphs.evaluate_oracle(text, ins)
    except (ValueError, IndexError):
        pytest.skip("program rejected")
    _holds(text, ins)


@pytest.mark.parametrize("seed", [7000, 7003, 7011, 7019, 7026, 7033])
def test_oracle_within_forward_bound_large(oracle_lib, seed):
    text, ins, _ = graphs.random_program(seed, integer_values=True, depth=4, large=True)
    try:
        graphs.evaluate_oracle(text, ins)
    except (ValueError, IndexError):
        pytest.skip("program rejected")
    _holds(text, ins)


def test_bound_is_tight_enough_to_fail_a_wrong_sum(oracle_lib):
    """A sum missing one of its 1000 terms is outside the bound."""
    rng = np.random.default_rng(3)
    x = rng.uniform(-2, 2, (4, 1000)).astype(np.float32)
    text = "0 input 0\n1 sum 0 1 0\n"
    v, e = error_bounds.evaluate(text, [x])
    wrong = x[:, :-1].astype(np.float64).sum(axis=1)
    assert np.all(np.abs(wrong - v) > 2 * e)


def test_check_accepts_shaped_arrays():
    want = np.arange(12, dtype=np.float64).reshape(3, 4) + 1
    bound = np.full((3, 4), 1e-9)
    got = want.astype(np.float32)
    out = error_bounds.check(got, want, bound, 1e-5, "shaped")
    assert out["elements"] == 12
    with pytest.raises(AssertionError):
        error_bounds.check(got + 1, want, bound, 1e-5, "shaped")
