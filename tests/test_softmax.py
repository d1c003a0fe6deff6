"""softmax over the last axis (reference: src/ops.cpp:7-14, max -> subtract
-> exp -> sum -> divide).

Rows of up to 64 values per thread (16384 columns at 256 threads) are held
in registers: one read and one write. When there are too few rows to fill
the GPU, rows of up to 8 x 16384 columns are spread over a thread-block
cluster of 2-8 CTAs, each holding its segment in registers, the CTAs'
maxima and sums exchanged through distributed shared memory: still one read
and one write. Otherwise longer rows take two passes: an online
pass keeps a running (max, sum) per thread, rescaling the sum whenever the
max grows, and the block combines the pairs; a second pass writes
exp(x - m) / s. CPU: the plans. GPU: parity with the host oracle within the
softmax tolerance (1e-5 relative).
"""

import numpy as np
import pytest

import graphs
from tolerances import assert_relative

LONG = [
    # (rows, columns, distribution)
    (64, 65536, "normal"),    # cluster of 4
    (37, 20000, "rising"),    # cluster of 2; the max sits in the last CTA
    (10, 100003, "normal"),   # cluster of 7, not a multiple of 4: scalar loads
    (3, 16388, "falling"),    # cluster of 2, the second CTA holds 2 columns
    (5, 131072, "rising"),    # cluster of 8
    (600, 20000, "rising"),   # rows enough to fill the GPU: streaming
    (4, 140000, "rising"),    # streaming: a rescale at every step
    (2, 300001, "falling"),   # streaming, scalar loads
]


def _rows(rows, cols, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return rng.normal(0, 3, (rows, cols)).astype(np.float32)
    ramp = np.linspace(-40.0, 40.0, cols, dtype=np.float64)
    if kind == "falling":
        ramp = ramp[::-1]
    return (ramp[None, :] + rng.normal(0, 0.5, (rows, cols))).astype(np.float32)


def _placeholder_plan(api, program, shapes):
    orig = api.tensor
    try:
        api.tensor = lambda s, values, device=0: api.placeholder(list(s))
        e = graphs.build(api, program, [np.zeros(s, np.float32) for s in shapes])
    finally:
        api.tensor = orig
    return [line for line in api.describe(e).splitlines() if line.startswith("kernel ")]


def test_long_rows_plan_cluster_or_online_kernels(api):
    prog = "0 input 0\n1 softmax 0 1\n"
    kernels = _placeholder_plan(api, prog, [[1000, 16384]])
    assert len(kernels) == 1 and "row in registers" in kernels[0], kernels
    kernels = _placeholder_plan(api, prog, [[64, 65536]])
    assert len(kernels) == 1 and "cluster of 4 CTAs" in kernels[0] and "grid=256x" in kernels[0], kernels
    kernels = _placeholder_plan(api, prog, [[10, 100003]])
    assert "V=1" in kernels[0] and "cluster of 7 CTAs" in kernels[0], kernels
    kernels = _placeholder_plan(api, prog, [[4, 140000]])
    assert len(kernels) == 1 and "online max/sum pass" in kernels[0], kernels
    kernels = _placeholder_plan(api, prog, [[600, 20000]])
    assert len(kernels) == 1 and "online max/sum pass" in kernels[0], kernels


@pytest.mark.parametrize("rows,cols,kind", LONG[:2])
def test_oracle_long_row_softmax_matches_numpy(oracle_lib, rows, cols, kind):
    x = _rows(min(rows, 4), cols, kind, 1)
    got = graphs.evaluate_oracle("0 input 0\n1 softmax 0 1\n", [x])
    x64 = x.astype(np.float64)
    e = np.exp(x64 - x64.max(axis=1, keepdims=True))
    assert_relative(got, (e / e.sum(axis=1, keepdims=True)).astype(np.float32), 1e-5, "oracle softmax")


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,kind", LONG)
def test_long_row_softmax_matches_oracle(gpu, rows, cols, kind):
    x = _rows(rows, cols, kind, 2)
    program = "0 input 0\n1 softmax 0 1\n"
    got = graphs.evaluate_product(gpu, program, [x])
    want = graphs.evaluate_oracle(program, [x])
    assert_relative(got, want, 1e-5, f"softmax [{rows}, {cols}] {kind}")


@pytest.mark.gpu
def test_long_row_softmax_with_broadcast_prologue(gpu):
    """Two leaves in the online pass: softmax(x + broadcast(b))."""
    rows, cols = 48, 40000
    rng = np.random.default_rng(3)
    x = rng.normal(0, 2, (rows, cols)).astype(np.float32)
    b = rng.normal(0, 2, (cols,)).astype(np.float32)
    program = f"0 input 0\n1 input 1\n2 broadcast 1 {rows},{cols}\n3 add 0 2\n4 softmax 3 1\n"
    got = graphs.evaluate_product(gpu, program, [x, b])
    want = graphs.evaluate_oracle(program, [x, b])
    assert_relative(got, want, 1e-5, "softmax(x + b)")
