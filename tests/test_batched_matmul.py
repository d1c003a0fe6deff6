"""Batched (rank-3) matmul, an extension: [B, M, K] @ [B, K, N] -> [B, M, N].

The reference's matmul is rank 2 only (src/tensor.cpp:366-381), and
PB_MATMUL keeps that rule. pb_expr_batched_matmul runs one grouped tcgen05
3xTF32 GEMM over every batch's tiles when B * M * N * K >= 2^27 (A's rows of
all batches split as one matrix, B's batches transposed side by side into
one stacked buffer), else one CUDA-core launch over all batches; an
elementwise consumer of the product is fused as that GEMM's epilogue, its
leaves read at per-batch offsets. Checked bit for bit on integer-valued operands
(every product and sum exact in fp32), and within the sqrt(K)-normalised
1e-5 bar of fp64 on real-valued ones.
"""

import numpy as np
import pytest

from tolerances import MATMUL_TOL, assert_bitwise, matmul_error

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,m,k,n", [(4, 512, 1024, 512), (3, 640, 2052, 264), (6, 64, 96, 33), (1, 5, 7, 3),
                                     (32, 256, 512, 256),   # small GEMMs, tensor cores on the total
                                     (8, 100, 4096, 300)])  # a tile's rows past M belong to the next batch
def test_batched_matmul_matches_numpy(gpu, b, m, k, n):
    api = gpu
    rng = np.random.default_rng(b * 1000 + m + k + n)
    xi = rng.integers(-3, 4, (b, m, k)).astype(np.float32)
    yi = rng.integers(-3, 4, (b, k, n)).astype(np.float32)
    X, Y = api.tensor([b, m, k], xi), api.tensor([b, k, n], yi)
    expr = api.batched_matmul(X, Y)
    assert expr.shape() == [b, m, n]
    plan = api.describe(expr)
    assert ("tcgen05" in plan) == (b * m * n * k >= (1 << 27)), plan
    assert plan.count("kernel pb_gemm_tc_") == (1 if "tcgen05" in plan else 0), plan
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
    """relu(P * 2 + bias - Z) over P = X @ Y runs as the epilogue of the
    grouped GEMM (no elementwise kernel of its own): Z is read at per-batch
    offsets, bias the same for every batch. Exact on integer operands."""
    api = gpu
    rng = np.random.default_rng(b * 7 + m + k + n)
    xi = rng.integers(-3, 4, (b, m, k)).astype(np.float32)
    yi = rng.integers(-3, 4, (b, k, n)).astype(np.float32)
    zi = rng.integers(-50, 51, (b, m, n)).astype(np.float32)
    bias = rng.integers(-9, 10, n).astype(np.float32)
    X, Y, Z, Bv = (api.tensor(list(v.shape), v) for v in (xi, yi, zi, bias))
    expr = api.relu(api.batched_matmul(X, Y) * 2.0 + api.broadcast_to(Bv, [b, m, n]) - Z)
    plan = api.describe(expr)
    assert "pb_elem" not in plan and plan.count("kernel pb_gemm_tc_") == 1, plan
    assert f"{b} batches grouped in one launch" in plan, plan
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
    assert "pb_elem" in plan and plan.count("kernel pb_gemm_tc_") == 1, plan
    want = (np.matmul(xi.astype(np.float64), yi.astype(np.float64)) + ci).astype(np.float32)
    assert_bitwise(api.materialize(expr).cpu().reshape(b, m, n), want, "unfused batched epilogue")


def test_batched_matmul_nonfinite_operand_takes_the_cuda_core_path(gpu):
    """An Inf in one batch sends the grouped GEMM to its CUDA-core fallback,
    which runs every batch (blockIdx.y) with the fused epilogue's leaves at
    their batch offsets: Inf and NaN (Inf * 0) land where an fp32 FMA chain
    puts them, every other value exact on integer operands."""
    api = gpu
    b, m, k, n = 4, 512, 1024, 512
    rng = np.random.default_rng(12)
    xi = rng.integers(-3, 4, (b, m, k)).astype(np.float32)
    yi = rng.integers(-3, 4, (b, k, n)).astype(np.float32)
    zi = rng.integers(-50, 51, (b, m, n)).astype(np.float32)
    bias = rng.integers(-9, 10, n).astype(np.float32)
    xi[2, 3, 5] = np.inf
    X, Y, Z, Bv = (api.tensor(list(v.shape), v) for v in (xi, yi, zi, bias))
    expr = api.batched_matmul(X, Y) * 2.0 + api.broadcast_to(Bv, [b, m, n]) - Z
    assert "batches grouped in one launch" in api.describe(expr)
    with np.errstate(invalid="ignore"):
        prod = np.matmul(xi.astype(np.float64), yi.astype(np.float64))
        want = (prod * 2.0 + bias - zi).astype(np.float32)
    got = api.materialize(expr).cpu().reshape(b, m, n)
    assert np.isnan(want[2, 3]).any() and np.isinf(want[2, 3]).any()
    np.testing.assert_array_equal(got, want)


def test_batched_matmul_keeps_operand_splits(gpu):
    """Realised [B, M, K] and [B, K, N] operands keep their 3xTF32 splits
    like a 2-D matmul's: the second product of the same tensors launches no
    split pass and gives the same bits."""
    api = gpu
    b, m, k, n = 4, 512, 1024, 512
    rng = np.random.default_rng(14)
    X = api.tensor([b, m, k], rng.uniform(-1, 1, (b, m, k)).astype(np.float32))
    Y = api.tensor([b, k, n], rng.uniform(-1, 1, (b, k, n)).astype(np.float32))

    def run():
        api.synchronize()
        api.profile_enable(True)
        api.profile_read()
        try:
            out = api.materialize(api.batched_matmul(X, Y)).cpu()
            api.synchronize()
            kernels = {name: count for name, (count, _) in api.profile_read().items()}
        finally:
            api.profile_enable(False)
        splits = sum(c for name, c in kernels.items() if name.startswith(("pb_split_rows", "pb_split_transpose")))
        return out, splits

    first, s1 = run()
    second, s2 = run()
    assert s1 == 2 and s2 == 0, (s1, s2)
    assert_bitwise(second, first, "kept batched splits")
