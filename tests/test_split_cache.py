"""3xTF32 operand splits kept by realised tensors.

The tcgen05 GEMM multiplies hi/lo TF32 halves of each fp32 operand (Ootomo &
Yokota 2022); a split pass writes them before the GEMM. A realised input
whose device handle has never been handed out cannot change, so its storage
keeps the split: a weight used step after step is split once. Handing out
its handle (tensor::device_data(), pb_tensor_device_pointer) drops the kept
split, since the values may be written through it. The kept split carries
its operand's Inf/NaN flag, so a later GEMM still takes the reference's
fp32 chain for non-finite operands.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ints(shape, seed):
    return np.random.default_rng(seed).integers(-3, 4, shape).astype(np.float32)


def _run(api, fn):
    api.synchronize()
    api.profile_enable(True)
    api.profile_read()
    try:
        out = fn()
        api.synchronize()
        return out, {k: n for k, (n, _) in api.profile_read().items()}
    finally:
        api.profile_enable(False)


def _splits(kernels):
    return sum(n for k, n in kernels.items() if k.startswith(("pb_split_rows", "pb_split_transpose")))


def test_weight_split_is_kept_until_its_handle_escapes(gpu):
    api = gpu
    m, k, n = 256, 1024, 512  # tensor-core eligible
    w = _ints([k, n], 1)
    W = api.tensor([k, n], w)
    for step, seed in enumerate([2, 3, 4]):
        x = _ints([m, k], seed)
        X = api.tensor([m, k], x)
        C, kernels = _run(api, lambda: api.materialize(api.matmul(X, W)))
        assert any(name.startswith("pb_gemm_tc") for name in kernels), kernels
        # Step 0 splits X and W; later steps split only their new X.
        assert _splits(kernels) == (2 if step == 0 else 1), (step, kernels)
        want = (x.astype(np.float64) @ w.astype(np.float64)).astype(np.float32)
        assert np.array_equal(C.cpu().reshape(m, n), want)
    # The handle escapes: the kept split is dropped and W is split again.
    W.device_data()
    x = _ints([m, k], 5)
    X = api.tensor([m, k], x)
    C, kernels = _run(api, lambda: api.materialize(api.matmul(X, W)))
    assert _splits(kernels) == 2, kernels
    assert np.array_equal(C.cpu().reshape(m, n), (x.astype(np.float64) @ w.astype(np.float64)).astype(np.float32))


def test_kept_split_keeps_its_nonfinite_flag(gpu):
    api = gpu
    m, k, n = 256, 1024, 512
    w = _ints([k, n], 6)
    w[17, 40] = np.inf
    W = api.tensor([k, n], w)
    for step, seed in enumerate([7, 8]):
        x = _ints([m, k], seed)
        x[:, 17] = np.where(x[:, 17] == 0, 1.0, x[:, 17])  # no inf * 0 except where chosen
        x[3, 17] = 0.0                                      # inf * 0 -> NaN in row 3, column 40
        X = api.tensor([m, k], x)
        C, kernels = _run(api, lambda: api.materialize(api.matmul(X, W)))
        assert _splits(kernels) == (2 if step == 0 else 1), kernels
        got = C.cpu().reshape(m, n)
        with np.errstate(invalid="ignore"):
            want = (x.astype(np.float64) @ w.astype(np.float64)).astype(np.float32)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        assert np.isnan(got[3, 40]) and np.isinf(got[0, 40])
        fin = np.isfinite(want)
        assert np.array_equal(got[fin], want[fin])
