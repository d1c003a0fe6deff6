"""Batched (rank-3) matmul, an extension: [B, M, K] @ [B, K, N] -> [B, M, N].

The reference's matmul is rank 2 only (src/tensor.cpp:366-381), and
PB_MATMUL keeps that rule. pb_expr_batched_matmul runs one tcgen05 3xTF32
GEMM per batch when M * N * K >= 2^27 (every batch reuses the same compiled
kernels and split buffers through pointer offsets), else one CUDA-core
launch over all batches; an elementwise consumer of the product is fused
as each batch's GEMM epilogue. Checked bit for bit on integer-valued operands
(every product and sum exact in fp32), and within the sqrt(K)-normalised
1e-5 bar of fp64 on real-valued ones.
"""

import numpy as np
import pytest

from tolerances import MATMUL_TOL, assert_bitwise, matmul_error

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,m,k,n", [(4, 512, 1024, 512), (3, 640, 2052, 264), (6, 64, 96, 33), (1, 5, 7, 3)])
def test_batched_matmul_matches_numpy(gpu, b, m, k, n):
    api = gpu
    rng = np.random.default_rng(b * 1000 + m + k + n)
    xi = rng.integers(-3, 4, (b, m, k)).astype(np.float32)
    yi = rng.integers(-3, 4, (b, k, n)).astype(np.float32)
    X, Y = api.tensor([b, m, k], xi), api.tensor([b, k, n], yi)
    expr = api.batched_matmul(X, Y)
    assert expr.shape() == [b, m, n]
    plan = api.describe(expr)
    assert ("tcgen05" in plan) == (m * n * k >= (1 << 27)), plan
    want = np.matmul(xi.astype(np.float64), yi.astype(np.float64)).astype(np.float32)
    for _ in range(2):  # the second call reuses the kept splits of X and Y
        assert_bitwise(api.materialize(expr).cpu().reshape(b, m, n), want, f"batched {b}x{m}x{k}x{n}")
    # Real values against fp64, per batch, with a fused consumer after it.
    xr = rng.uniform(-1, 1, (b, m, k)).astype(np.float32)
    yr = rng.uniform(-1, 1, (b, k, n)).astype(np.float32)
    Xr, Yr = api.tensor([b, m, k], xr), api.tensor([b, k, n], yr)
    got = api.materialize(api.batched_matmul(Xr * 2.0, Yr) - 1.0).cpu().reshape(b, m, n)
    ref = np.matmul(2.0 * xr.astype(np.float64), yr.astype(np.float64)) - 1.0
    for t in range(b):
        assert matmul_error(got[t], ref[t], k) <= MATMUL_TOL, t


def test_batched_matmul_checks_its_operands(gpu):
    api = gpu
    z = lambda *s: api.tensor(list(s), np.zeros(int(np.prod(s)), np.float32))  # noqa: E731
    with pytest.raises(ValueError, match="rank-3"):
        api.batched_matmul(z(4, 4), z(4, 4))
    with pytest.raises(ValueError, match="batch dimensions"):
        api.batched_matmul(z(2, 4, 4), z(3, 4, 4))
    with pytest.raises(ValueError, match="inner dimensions"):
        api.batched_matmul(z(2, 4, 5), z(2, 4, 4))
    # The reference's rank-2 rule for PB_MATMUL stands.
    with pytest.raises(ValueError, match="rank-2"):
        api.materialize(api.matmul(z(2, 4, 4), z(2, 4, 4)))


@pytest.mark.parametrize("b,m,k,n", [(4, 512, 1024, 512), (3, 640, 2052, 264)])
def test_batched_matmul_fuses_its_elementwise_consumer(gpu, b, m, k, n):
    """relu(P * 2 + bias - Z) over P = X @ Y runs as the epilogue of each
    batch's GEMM (no elementwise kernel of its own): the leaves Z and bias
    are read at per-batch pointer offsets. Exact on integer operands."""
    api = gpu
    rng = np.random.default_rng(b * 7 + m + k + n)
    xi = rng.integers(-3, 4, (b, m, k)).astype(np.float32)
    yi = rng.integers(-3, 4, (b, k, n)).astype(np.float32)
    zi = rng.integers(-50, 51, (b, m, n)).astype(np.float32)
    bias = rng.integers(-9, 10, n).astype(np.float32)
    X, Y, Z, Bv = (api.tensor(list(v.shape), v) for v in (xi, yi, zi, bias))
    expr = api.relu(api.batched_matmul(X, Y) * 2.0 + api.broadcast_to(Bv, [b, m, n]) - Z)
    plan = api.describe(expr)
    assert "pb_elem" not in plan and plan.count("pb_gemm_tc") == b, plan
    prod = np.matmul(xi.astype(np.float64), yi.astype(np.float64))
    want = np.maximum(prod * 2.0 + bias - zi, 0.0).astype(np.float32)
    assert_bitwise(api.materialize(expr).cpu().reshape(b, m, n), want, f"fused batched {b}x{m}x{k}x{n}")


def test_batched_matmul_leaf_with_unaligned_batch_stride_runs_unfused(gpu):
    """A leaf whose batch stride (263 floats) would misalign the epilogue's
    16-byte loads is not fused: the product is realised, then an
    elementwise kernel adds the leaf. Same values."""
    api = gpu
    b, m, k, n = 3, 256, 2052, 263
    rng = np.random.default_rng(5)
    xi = rng.integers(-3, 4, (b, m, k)).astype(np.float32)
    yi = rng.integers(-3, 4, (b, k, n)).astype(np.float32)
    ci = rng.integers(-9, 10, (b, 1, n)).astype(np.float32)
    X, Y, C = (api.tensor(list(v.shape), v) for v in (xi, yi, ci))
    expr = api.batched_matmul(X, Y) + api.broadcast_to(C, [b, m, n])
    plan = api.describe(expr)
    assert "pb_elem" in plan and plan.count("pb_gemm_tc") == b, plan
    want = (np.matmul(xi.astype(np.float64), yi.astype(np.float64)) + ci).astype(np.float32)
    assert_bitwise(api.materialize(expr).cpu().reshape(b, m, n), want, "unfused batched epilogue")
