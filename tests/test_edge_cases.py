"""Edge cases: zero-size dimensions, NaN/Inf operands, and tensors past 2^31
elements (the 64-bit index paths).

The reference's rules (src/tensor.cpp): an empty result launches nothing
(:1023-1028); IEEE arithmetic in the generated code (:616-683) with
`(l > r ? l : r)` maxima, so NaN handling follows from the comparison form;
its matmul is an fp32 FMA chain, so Inf/NaN operands give Inf/NaN exactly
as IEEE says (the 3xTF32 path hands such operands to the same chain).
"""

import numpy as np
import pytest

import error_bounds
import graphs
from tolerances import (MATMUL_TOL, REL_TOL, assert_bitwise, assert_relative, assert_sum_close,
                        matmul_error)

ZERO_SIZE = [
    ("0 input 0\n1 exp 0\n", [[0, 5]]),
    ("0 input 0\n1 input 1\n2 add 0 1\n", [[3, 0], [3, 0]]),
    ("0 input 0\n1 sum 0 1 0\n", [[4, 0]]),
    ("0 input 0\n1 max 0 0 1\n", [[0, 6]]),
    ("0 input 0\n1 transpose 0\n", [[0, 7]]),
    ("0 input 0\n1 input 1\n2 concat 0 1 0\n", [[0, 3], [2, 3]]),
    ("0 input 0\n1 tensor 0\n2 index 1 s2:2:1;s0:3:1\n", [[4, 3]]),
]


# Where the output is not empty but an input is, the reference refuses the
# launch; the oracle restates that rule and the CUDA path must agree.
REFUSED = {2: "CUDA reduction input is empty", 3: "CUDA reduction input is empty",
           5: "CUDA elementwise input is empty"}


@pytest.mark.parametrize("case", range(len(ZERO_SIZE)))
def test_oracle_zero_size_rules(oracle_lib, case):
    program, shapes = ZERO_SIZE[case]
    ins = [np.zeros(s, np.float32) for s in shapes]
    if case in REFUSED:
        with pytest.raises(ValueError, match=REFUSED[case]):
            graphs.evaluate_oracle(program, ins)
    else:
        assert graphs.evaluate_oracle(program, ins).size == 0


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(ZERO_SIZE)))
def test_zero_size_dimensions_match_oracle(gpu, case):
    program, shapes = ZERO_SIZE[case]
    rng = np.random.default_rng(1)
    ins = [rng.normal(0, 1, s).astype(np.float32) for s in shapes]
    if case in REFUSED:
        with pytest.raises(ValueError, match=REFUSED[case]):
            graphs.evaluate_product(gpu, program, ins)
        return
    want = graphs.evaluate_oracle(program, ins)
    got = graphs.evaluate_product(gpu, program, ins)
    assert list(got.shape) == list(want.shape)
    assert_bitwise(got, want, program)


SPECIALS = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1.0, -2.5, 3.4e38, -3.4e38, 1e-45],
                    dtype=np.float32)
# A NaN inside a max reduction makes `(m > x ? m : x)` depend on the order
# in which values are combined (the reference's 256-wide block tree, the
# host oracle's loop and this library's warp tree all differ), so the
# reductions and softmax get +-Inf and extremes but no NaN.
NO_NAN = {"softmax", "max"}
NONFINITE_PROGRAMS = [
    ("0 input 0\n1 input 1\n2 add 0 1\n", True),
    ("0 input 0\n1 input 1\n2 multiply 0 1\n", True),
    ("0 input 0\n1 input 1\n2 divide 0 1\n", True),
    ("0 input 0\n1 input 1\n2 maximum 0 1\n", True),
    ("0 input 0\n1 input 1\n2 minimum 0 1\n", True),
    ("0 input 0\n1 relu 0\n", True),
    ("0 input 0\n1 reciprocal 0\n", True),
    ("0 input 0\n1 exp 0\n", False),
    ("0 input 0\n1 logistic 0\n", False),
    ("0 input 0\n1 softmax 0 1\n", False),
    ("0 input 0\n1 max 0 1 0\n", True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("program,exact", NONFINITE_PROGRAMS)
def test_nan_and_inf_operands_match_oracle(gpu, program, exact):
    # Every pair of special values, as rows of a [10, 10] grid.
    specials = SPECIALS
    if {line.split()[1] for line in program.strip().splitlines()} & NO_NAN:
        specials = np.where(np.isnan(SPECIALS), np.float32(7.0), SPECIALS).astype(np.float32)
    a = np.repeat(specials[:, None], 10, axis=1)
    b = np.repeat(specials[None, :], 10, axis=0)
    n_inputs = program.count("input")
    ins = [a, b][:n_inputs]
    want = graphs.evaluate_oracle(program, ins)
    got = graphs.evaluate_product(gpu, program, ins)
    if exact:
        assert_bitwise(got, want, program)
    else:
        assert_relative(got, want, 1e-5, program)


@pytest.mark.gpu
def test_nonfinite_matmul_operands_match_the_reference(gpu):
    """Inf and NaN in tensor-core-eligible operands: the same non-finite
    pattern as the reference's own fp32 chain, finite entries within the
    matmul tolerance of it."""
    import test_ref_fullsize as ref

    rng = np.random.default_rng(9)
    m = k = n = 512
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    a[3, 7] = np.inf
    a[10, 100] = -np.inf
    a[200, :4] = np.nan
    b[5, 9] = np.inf
    b[7, 300] = 0.0  # inf * 0 -> NaN in row 3 only where the chain meets it
    prog = "0 input 0\n1 input 1\n2 matmul 0 1\n"
    assert "tcgen05" in gpu.describe(gpu.matmul(gpu.tensor([m, k], a), gpu.tensor([k, n], b)))
    got = graphs.evaluate_product(gpu, prog, [a, b])
    want = ref._run_reference(prog, [a, b])
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(np.isposinf(got), np.isposinf(want))
    assert np.array_equal(np.isneginf(got), np.isneginf(want))
    # Finite entries: 1e-5 relative or, where they cancel, within the fp32
    # forward error bound (both sides are fp32 evaluations).
    _, bound = error_bounds.evaluate(prog, [a, b])
    error_bounds.check(got, want, bound, REL_TOL, "non-finite operands")
    # And with finite operands the same plan takes the tensor-core path: the
    # CUDA-core kernel returns at once (results equal to the reference's
    # within the 3xTF32 tolerance).
    a2, b2 = np.nan_to_num(a, posinf=1.0, neginf=-1.0), np.nan_to_num(b, posinf=1.0, neginf=-1.0)
    got2 = graphs.evaluate_product(gpu, prog, [a2, b2])
    want2 = ref._run_reference(prog, [a2, b2])
    _, bound2 = error_bounds.evaluate(prog, [a2, b2])
    error_bounds.check(got2, want2, bound2, REL_TOL, "finite operands")
    assert matmul_error(got2, a2.astype(np.float64) @ b2.astype(np.float64), k) <= MATMUL_TOL


BIG = (1 << 31) + 8


@pytest.mark.gpu
def test_elementwise_past_2_31_elements(gpu):
    api = gpu
    c = api.tensor([1], np.array([1.5], dtype=np.float32))
    y = api.materialize(api.broadcast_to(c, [BIG]) * 2.0 + 1.0)
    assert y.shape() == [BIG]
    tail = api.materialize(y[BIG - 16:BIG]).cpu()
    head = api.materialize(y[0:16]).cpu()
    assert np.all(tail == 4.0) and np.all(head == 4.0)


@pytest.mark.gpu
def test_softmax_and_column_sum_past_2_31_elements(gpu):
    api = gpu
    rows, cols = (1 << 21) + 1, 1024
    rng = np.random.default_rng(3)
    row = rng.normal(0, 1, (1, cols)).astype(np.float32)
    x = api.broadcast_to(api.tensor([1, cols], row), [rows, cols])
    p = api.materialize(api.softmax(x, 1))
    last = api.materialize(p[rows - 2:rows, 0:cols]).cpu()
    want = graphs.evaluate_oracle("0 input 0\n1 softmax 0 1\n", [row])
    assert_relative(last[0:1], want, 1e-5, "first of the last two rows")
    assert_relative(last[1:2], want, 1e-5, "last row")
    ones = api.broadcast_to(api.tensor([1, cols], np.ones((1, cols), np.float32)), [rows, cols])
    s = api.materialize(api.sum(ones, 0)).cpu()
    assert np.all(s == np.float32(rows))  # exact: integers below 2^24


@pytest.mark.gpu
def test_graph_reading_many_distinct_tensors(gpu):
    """300 distinct inputs in one fused kernel (more than 64 kernel
    arguments; the reference passes its inputs as one parameter vector)."""
    api = gpu
    rng = np.random.default_rng(21)
    arrays = [rng.integers(-4, 5, 1000).astype(np.float32) for _ in range(300)]
    tensors = [api.tensor([1000], a) for a in arrays]
    expr = tensors[0] + 0.0
    for t in tensors[1:]:
        expr = expr + t
    got = api.materialize(expr).cpu()
    want = np.zeros(1000, np.float32)
    for a in arrays:
        want = (want + a).astype(np.float32)
    assert_bitwise(got, want, "300-input sum")


# A reduced axis followed by extent-1 dimensions can have any stride (the
# row-vectorised loads need unit stride), and a softmax over an axis other
# than the last lowers as its two reductions and an elementwise pass
# (reference: src/ops.cpp:7-14 builds softmax from max, exp, sum, divide).
STRIDED_AXIS = [
    ("0 input 0\n1 transpose 0\n2 reshape 1 4,100,1\n3 sum 2 1 0\n", [[100, 4]]),
    ("0 input 0\n1 transpose 0\n2 reshape 1 8,64,1\n3 max 2 1 1\n", [[64, 8]]),
    ("0 input 0\n1 softmax 0 1\n", [[4, 100, 3]]),
    ("0 input 0\n1 transpose 0\n2 reshape 1 4,100,1\n3 softmax 2 1\n", [[100, 4]]),
    ("0 input 0\n1 softmax 0 0\n", [[64, 8]]),
]


def _strided_inputs(shapes, seed):
    rng = np.random.default_rng(seed)
    return [rng.normal(0, 1, s).astype(np.float32) for s in shapes]


def _numpy_of(program, x):
    """numpy restatement of the five STRIDED_AXIS programs."""
    x = x.astype(np.float64)
    lines = program.strip().splitlines()
    last = lines[-1].split()
    if "transpose" in program:
        x = x.T.reshape([int(d) for d in lines[2].split()[3].split(",")])
    axis = int(last[3])
    if last[1] == "sum":
        return x.sum(axis=axis, keepdims=last[4] == "1")
    if last[1] == "max":
        return x.max(axis=axis, keepdims=last[4] == "1")
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return e / e.sum(axis=axis, keepdims=True)


@pytest.mark.parametrize("case", range(len(STRIDED_AXIS)))
def test_oracle_strided_axis_and_inner_softmax(oracle_lib, case):
    program, shapes = STRIDED_AXIS[case]
    ins = _strided_inputs(shapes, 5)
    got = graphs.evaluate_oracle(program, ins)
    want = _numpy_of(program, ins[0])
    if " sum " in program:
        abs_sum = np.abs(ins[0].astype(np.float64)).T.reshape(4, 100, 1).sum(axis=1)
        assert_sum_close(got, want, abs_sum, 100, 1e-5, program)
    else:
        assert_relative(got, want.astype(np.float32), 1e-5, program)


@pytest.mark.parametrize("case", range(len(STRIDED_AXIS)))
def test_strided_axis_plans(api, case):
    """Plans on placeholders: no softmax row kernel for an inner axis, and no
    four-wide loads along a strided reduced axis."""
    program, shapes = STRIDED_AXIS[case]
    orig = api.tensor
    try:
        api.tensor = lambda s, values, device=0: api.placeholder(list(s))
        e = graphs.build(api, program, [np.zeros(sh, np.float32) for sh in shapes])
    finally:
        api.tensor = orig
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert kernels and not any("softmax row kernel" in k for k in kernels), kernels
    if "transpose" in program:
        assert not any("row reduction" in k and "V=4" in k for k in kernels), kernels


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(STRIDED_AXIS)))
def test_strided_axis_and_inner_softmax_match_oracle(gpu, case):
    program, shapes = STRIDED_AXIS[case]
    ins = _strided_inputs(shapes, 6)
    want = graphs.evaluate_oracle(program, ins)
    got = graphs.evaluate_product(gpu, program, ins)
    if " max " in program:
        assert_bitwise(got, want, program)
    elif " sum " in program:
        x = np.abs(ins[0].astype(np.float64)).T.reshape(4, 100, 1)
        assert_sum_close(got, want, x.sum(axis=1), 100, 1e-5, program)
    else:
        assert_relative(got, want, 1e-5, program)


@pytest.mark.gpu
def test_device_ordinal_not_present_runs_on_device_zero(gpu):
    """device{n} runs on GPU n when it is present. An ordinal with no GPU
    behind it keeps the reference's meaning -- metadata, with the work on
    device 0 (src/cuda_jit.cpp:446-450; its own test builds device{1}
    tensors, tests/tensor_test.cpp:17-31) -- and never lands on another
    present GPU (it used to wrap around to n % count)."""
    api = gpu
    count = api.device_count()
    values = np.arange(4, dtype=np.float32)
    t = api.tensor([4], values, device=count + 7)
    assert t.placement() == count + 7
    assert_bitwise(api.materialize(t + 1.0).cpu(), values + 1.0, "absent ordinal")
    with pytest.raises(ValueError, match="devices must match"):
        api.materialize(t + api.tensor([4], values, device=0))
    with pytest.raises(ValueError, match="non-negative"):
        api.tensor([4], values, device=-1)
    last = api.tensor([4], values, device=count - 1)
    assert_bitwise(api.materialize(last + 1.0).cpu(), values + 1.0, "last device")
