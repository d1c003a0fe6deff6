"""sum / max over leading and middle axes (reference: src/tensor.cpp:316,
819-855, 896-962; tests/tensor_test.cpp:550 reduces axis 0).

A reduction whose outputs alone give too few CTAs to fill the GPU (a tall
tensor reduced over axis 0) is split into row chunks: pass 1 writes one
partial per (chunk, output), pass 2 combines them in a fixed order. A 2-D
operand with unit-stride rows of at least 64 columns (a multiple of 4) is
read in 128-column tiles, a float4 per lane, eight rows in flight per warp.
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
    # Column tiles (unit-stride rows of >= 64 columns, a multiple of 4):
    ([262144, 256], 0, False, "sum", None),
    ([1000, 260], 0, False, "sum", "exp"),
    ([1003, 128], 0, True, "max", None),
    ([64, 128], 0, False, "max", "relu"),
    # Narrow rows: several rows per warp load (2, 4 and 8 rows).
    ([1048576, 64], 0, False, "sum", None),
    ([100000, 32], 0, True, "max", "relu"),
    ([65536, 16], 0, False, "sum", "exp"),
    ([333, 20], 0, False, "max", None),
    # The middle axis of [B, A, C]: column tiles, one batch per blockIdx.z.
    ([32, 2048, 1024], 1, False, "sum", None),
    ([7, 300, 260], 1, True, "max", "exp"),
    ([64, 4096, 64], 1, False, "sum", "relu"),
    ([2, 3, 5, 40], 2, False, "max", None),
    # Contiguous trailing dimensions merge: [A, B, C] over axis 0 reads as
    # [A, B*C]; [64, 32, 16, 8] over axis 1 as a batch of [32, 128].
    ([4096, 64, 256], 0, False, "sum", None),
    ([64, 32, 16, 8], 1, True, "max", "relu"),
    ([8, 3, 5, 7], 0, False, "sum", "exp"),
    # 4 and 8 columns: 32 and 16 rows per warp load.
    ([100000, 4], 0, False, "sum", None),
    ([300, 8], 0, False, "max", None),
    ([64, 4096, 8], 1, True, "sum", "exp"),
    # Columns not a multiple of 4, or transposed: thread per output.
    ([100000, 6], 0, False, "sum", None),
    ([2048, 384], 0, False, "sum", "transpose"),
    # Few long rows: a CTA per row (8 warps share it).
    ([4096, 16384], 1, False, "sum", None),
    ([300, 2049], 1, False, "max", "exp"),
    ([4, 50, 3000], 2, True, "sum", "relu"),
]


def _program(shape, axis, keepdim, op, prologue):
    lines = ["0 input 0"]
    src = 0
    if prologue is not None:
        lines.append(f"1 {prologue} 0")
        src = 1
    lines.append(f"{len(lines)} {op} {src} {axis} {int(keepdim)}")
    return "\n".join(lines) + "\n"


def _host_prologue(x, prologue):
    if prologue == "exp":
        return np.exp(x)
    if prologue == "relu":
        return np.maximum(x, 0)
    if prologue == "transpose":
        return x.T
    return x


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
    assert "column reduction (128-column tiles" in kernels[0] and "pass 2" in kernels[1], plan
    e = _placeholder_expr(api, _program([100000, 6], 0, False, "sum", None), [100000, 6])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert len(kernels) == 2 and "pass 1" in kernels[0] and "pass 2" in kernels[1], kernels


def test_unit_stride_columns_plan_column_tiles(api):
    e = _placeholder_expr(api, _program([262144, 256], 0, False, "sum", None), [262144, 256])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert len(kernels) == 2 and "column reduction (128-column tiles" in kernels[0], kernels
    assert "pass 2" in kernels[1] and "fixed order" in kernels[1], kernels
    # A transposed operand has strided columns: thread per output instead.
    e = _placeholder_expr(api, _program([2048, 384], 0, False, "sum", "transpose"), [2048, 384])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert "strided reduction" in kernels[0], kernels


def test_few_long_rows_plan_a_cta_per_row(api):
    e = _placeholder_expr(api, _program([4096, 16384], 1, False, "sum", None), [4096, 16384])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert len(kernels) == 1 and "per row" in kernels[0] and "CTA of 1024" in kernels[0] and "V=4" in kernels[0], kernels
    e = _placeholder_expr(api, _program([65536, 1024], 1, False, "sum", None), [65536, 1024])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert "warp per row" in kernels[0], kernels


def test_middle_axis_plans_batched_column_tiles(api):
    e = _placeholder_expr(api, _program([32, 2048, 1024], 1, False, "sum", None), [32, 2048, 1024])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert "column reduction (128-column tiles" in kernels[0] and "x32 block" in kernels[0], kernels


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
    x = _host_prologue(ins[0].astype(np.float64), prologue)
    if op == "sum":
        assert_sum_close(got, x.sum(axis=axis, keepdims=keepdim), np.abs(x).sum(axis=axis, keepdims=keepdim),
                         x.shape[axis], REL_TOL, str(case))
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
        x = _host_prologue(ins[0].astype(np.float64), prologue)
        abs_sum = np.abs(x).sum(axis=axis, keepdims=keepdim)
        assert_sum_close(got, want, abs_sum, x.shape[axis], REL_TOL, str(case))


def test_trailing_dimensions_merge_only_when_contiguous(api):
    e = _placeholder_expr(api, _program([4096, 64, 256], 0, False, "sum", None), [4096, 64, 256])
    kernels = [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]
    assert "column reduction (128-column tiles" in kernels[0] and "grid=128x" in kernels[0], kernels
    x = api.placeholder([64, 16, 300])
    kernels = [line for line in api.describe(api.sum(x[:, :, 0:256], 0)).splitlines() if line.startswith("kernel ")]
    assert "strided reduction" in kernels[0], kernels


@pytest.mark.gpu
def test_sliced_trailing_dimensions_match_oracle(gpu):
    """A slice breaks the contiguity of the trailing dimensions: no merge,
    thread per output; same results as the oracle."""
    rng = np.random.default_rng(17)
    x = rng.normal(0, 1, (512, 16, 300)).astype(np.float32)
    program = "0 input 0\n1 tensor 0\n2 index 1 s0:512:1;s0:16:1;s3:259:1\n3 sum 2 0 0\n"
    got = graphs.evaluate_product(gpu, program, [x])
    want = graphs.evaluate_oracle(program, [x])
    abs_sum = np.abs(x[:, :, 3:259].astype(np.float64)).sum(axis=0)
    assert_sum_close(got, want, abs_sum, 512, REL_TOL, "sliced sum over axis 0")
