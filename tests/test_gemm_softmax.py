"""softmax(A @ B + bias, 1) through the tensor-core GEMM's softmax epilogue.

The reference composes softmax as max, subtract, exp, sum and divide over a
realised matmul (src/ops.cpp:7-14, src/tensor.cpp:684-721): the product makes
a round trip through memory before four reduction/elementwise kernels. Here
each 128 x 256 GEMM tile writes exp(y - m) with its row maximum m and sum,
and one streaming pass rescales every tile by exp(m_t - M) / S. Bars:
softmax within 1e-5 relative of the fp64 softmax of the same GEMM's realised
output (which isolates the softmax steps), and that output within the
sqrt(K)-normalised 1e-5 matmul bar of fp64.
"""

import numpy as np
import pytest

import graphs
from tolerances import MATMUL_TOL, REL_TOL, assert_relative, matmul_error

pytestmark = pytest.mark.gpu


def _softmax64(z):
    z = np.asarray(z, np.float64)
    e = np.exp(z - z.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def _kernels(api, fn):
    api.synchronize()
    api.profile_enable(True)
    api.profile_read()
    try:
        out = fn()
        api.synchronize()
        return out, {k: n for k, (n, _) in api.profile_read().items()}
    finally:
        api.profile_enable(False)


@pytest.mark.parametrize("m,k,n", [(1024, 512, 4396), (640, 768, 1000), (256, 2048, 256),
                                   (512, 8192, 4096), (1024, 6144, 2048)])
def test_gemm_softmax_epilogue_matches_fp64(gpu, m, k, n):
    """The last two shapes have few tiles of long K: the GEMM splits K to
    fill its waves and the split-K combine runs the whole row softmax."""
    api = gpu
    rng = np.random.default_rng(m + k + n)
    s = 3.0 / np.sqrt(k)
    a = rng.uniform(-s, s, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    A, B, Bi = api.tensor([m, k], a), api.tensor([k, n], b), api.tensor([n], bias)
    z_expr = api.matmul(A, B) + api.broadcast_to(Bi, [m, n])
    plan = api.describe(api.softmax(z_expr, 1))
    split = k > 4096
    if split:
        assert "split-K softmax combine" in plan, plan
    else:
        assert "softmax epilogue" in plan and "pb_softmax_norm" in plan, plan
    P, kernels = _kernels(api, lambda: api.materialize(api.softmax(z_expr, 1)))
    fused = "pb_splitk_softmax" if split else "pb_softmax_norm"
    assert any(name.startswith(fused) for name in kernels), kernels
    got = P.cpu().reshape(m, n)
    z = api.materialize(z_expr).cpu().reshape(m, n)
    z64 = a.astype(np.float64) @ b.astype(np.float64) + bias.astype(np.float64)
    assert matmul_error(z, z64, k) <= MATMUL_TOL
    if _split_parts(api.describe(z_expr)) == _split_parts(plan):
        # The realised product summed K in the same parts as the fused GEMM:
        # the same z, so the softmax steps alone are measured.
        assert_relative(got, _softmax64(z), REL_TOL, f"gemm softmax {m}x{k}x{n}")
    else:
        # Different parts (a softmax epilogue splits only rows of a multiple
        # of 1024 columns): against fp64, the softmax bar plus the GEMM bar
        # carried through the softmax (|d log P| <= 2 max |dz|).
        zscale = np.maximum(np.abs(z64), np.sqrt(np.mean(z64 ** 2))).max(axis=1, keepdims=True)
        rel = np.abs(got - _softmax64(z64)) / _softmax64(z64)
        assert np.all(rel <= REL_TOL + 2 * MATMUL_TOL * np.sqrt(k) * zscale)
    assert np.allclose(got.sum(axis=1, dtype=np.float64), 1.0, atol=1e-5)


def _split_parts(plan: str) -> int:
    import re

    for line in plan.splitlines():
        if "pb_gemm_tc" in line:
            found = re.search(r"split-K x(\d+)", line)
            return int(found.group(1)) if found else 1
    return 1


def test_gemm_softmax_with_nonfinite_operand_takes_the_reference_steps(gpu, oracle_lib):
    """An Inf in A: the tensor-core kernels stand down, the CUDA-core GEMM
    and an in-place row softmax with the reference's own steps write the
    result (same non-finite pattern as the oracle, finite rows within 1e-5)."""
    api = gpu
    m, k, n = 256, 1024, 768
    rng = np.random.default_rng(11)
    a = rng.uniform(-0.05, 0.05, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    a[7, 3] = np.inf
    prog = "0 input 0\n1 input 1\n2 matmul 0 1\n3 softmax 2 1\n"
    got = graphs.evaluate_product(api, prog, [a, b])
    want = graphs.evaluate_oracle(prog, [a, b])
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = np.isfinite(want).all(axis=1)
    assert fin.sum() == m - 1
    assert_relative(got[fin], want[fin], REL_TOL, "finite rows")
    # And with the Inf removed the same plan runs the tensor-core path.
    a[7, 3] = 0.0
    got2 = graphs.evaluate_product(api, prog, [a, b])
    z64 = a.astype(np.float64) @ b.astype(np.float64)
    p64 = _softmax64(z64)
    rel = np.abs(got2 - p64) / p64
    # softmax relative bar plus the GEMM bar carried through (|d log P| <= 2 max|dz|)
    zscale = np.maximum(np.abs(z64), np.sqrt(np.mean(z64 ** 2))).max(axis=1, keepdims=True)
    assert np.all(rel <= REL_TOL + 2 * MATMUL_TOL * np.sqrt(k) * zscale)
