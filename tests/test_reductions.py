"""sum / max over leading and middle axes (reference: src/tensor.cpp:316,
819-855, 896-962; tests/tensor_test.cpp:550 reduces axis 0).

A reduction whose outputs alone give too few CTAs to fill the GPU (a tall
tensor reduced over axis 0) is split into row chunks: pass 1 writes one
partial per (chunk, output), pass 2 combines them in chunk order.
CPU: the plans. GPU: parity with the host oracle (max bit for bit -- the
maximum does not depend on the order -- sum within the reduction tolerance).
"""

import numpy as np
import pytest

import graphs
from tolerances import REL_TOL, assert_bitwise, assert_relative, assert_sum_close

CASES = [
    # (shape, axis, keepdim, op, prologue)
    ([65536, 64], 0, False, "sum", None),
    ([65536, 64], 0, True, "max", None),
    ([20000, 300], 0, False, "sum", "exp"),
    ([4096, 4096], 0, False, "max", "relu"),
    ([64, 4096, 8], 1, False, "sum", None),
    ([3, 1000, 5], 1, True, "max", None),
    ([8, 8], 0, False, "sum", None),
]


def _program(shape, axis, keepdim, op, prologue):
    lines = ["0 input 0"]
    src = 0
    if prologue is not None:
        lines.append(f"1 {prologue} 0")
        src = 1
    lines.append(f"{len(lines)} {op} {src} {axis} {int(keepdim)}")
    return "\n".join(lines) + "\n"


def _inputs(shape, seed):
    rng = np.random.default_rng(seed)
    return [rng.normal(0, 1, shape).astype(np.float32)]


def _placeholder_expr(api, program, shape):
    orig = api.tensor
    try:
        api.tensor = lambda s, values, device=0: api.placeholder(list(s))
        return graphs.build(api, program, [np.zeros(shape, np.float32)])
    finally:
        api.tensor = orig


def test_tall_leading_axis_reduction_plans_two_passes(api):
    e = _placeholder_expr(api, _program([65536, 64], 0, False, "sum", None), [65536, 64])
    plan = api.describe(e)
    kernels = [line for line in plan.splitlines() if line.startswith("kernel ")]
    assert len(kernels) == 2, plan
    assert "pass 1" in kernels[0] and "pass 2" in kernels[1], plan


def test_wide_row_reduction_stays_one_pass(api):
    e = _placeholder_expr(api, _program([4096, 4096], 1, False, "sum", None), [4096, 4096])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert len(kernels) == 1


@pytest.mark.parametrize("case", CASES, ids=[f"{c[3]}{c[0]}ax{c[1]}" for c in CASES])
def test_oracle_reductions_match_numpy(oracle_lib, case):
    shape, axis, keepdim, op, prologue = case
    if np.prod(shape) > 1 << 22:
        pytest.skip("large case: GPU test only")
    ins = _inputs(shape, 3)
    got = graphs.evaluate_oracle(_program(shape, axis, keepdim, op, prologue), ins)
    x = ins[0].astype(np.float64)
    if prologue == "exp":
        x = np.exp(x)
    elif prologue == "relu":
        x = np.maximum(x, 0)
    if op == "sum":
        assert_sum_close(got, x.sum(axis=axis, keepdims=keepdim), np.abs(x).sum(axis=axis, keepdims=keepdim),
                         shape[axis], REL_TOL, str(case))
    else:
        assert_relative(got, x.max(axis=axis, keepdims=keepdim).astype(np.float32), REL_TOL, str(case))


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[f"{c[3]}{c[0]}ax{c[1]}" for c in CASES])
def test_cuda_reductions_match_oracle(gpu, case):
    shape, axis, keepdim, op, prologue = case
    program = _program(shape, axis, keepdim, op, prologue)
    ins = _inputs(shape, 11)
    got = graphs.evaluate_product(gpu, program, ins)
    want = graphs.evaluate_oracle(program, ins)
    if op == "max" and prologue != "exp":
        assert_bitwise(got, want, str(case))
    elif op == "max":
        assert_relative(got, want, REL_TOL, str(case))
    else:
        x = ins[0].astype(np.float64)
        x = np.exp(x) if prologue == "exp" else (np.maximum(x, 0) if prologue == "relu" else x)
        abs_sum = np.abs(x).sum(axis=axis, keepdims=keepdim)
        assert_sum_close(got, want, abs_sum, shape[axis], REL_TOL, str(case))
