"""CTA pairs (the default): the tensor-core GEMM runs a 256 x 256 tile on a
cluster of two CTAs (tcgen05.mma.cta_group::2, each CTA holding its own 128
rows of A and half of B, 32-wide k-blocks) wherever there are at least two
128-row tiles. The products and their accumulation order are those of the
one-CTA form (PORCH_B200_GEMM=single, 16-wide k-blocks, the same periods in
K), so every epilogue gives the same bits either way: plain and fused
epilogues, ragged edges (a pair whose second half lies past M), the
softmax epilogue, the split-output epilogue of an MLP, split-K and the
persistent schedule. Also checked against fp64 within the sqrt(K)-
normalised bar.
"""

import os

import numpy as np
import pytest

from tolerances import MATMUL_TOL, assert_bitwise, matmul_error

pytestmark = pytest.mark.gpu


def _both(api, build):
    """Realise build() with CTA pairs (the default), then with one CTA per
    tile; returns both results and both plan descriptions."""
    out = []
    for form in (None, "single"):
        if form is None:
            os.environ.pop("PORCH_B200_GEMM", None)
        else:
            os.environ["PORCH_B200_GEMM"] = form
        try:
            expr = build()
            out.append((api.materialize(expr).cpu(), api.describe(expr)))
        finally:
            os.environ.pop("PORCH_B200_GEMM", None)
    return out


@pytest.mark.parametrize("m,k,n,paired", [
    (256, 1024, 512, True),      # one pair row
    (1152, 512, 768, True),      # nine 128-row tiles: the last pair's second half is past M
    (1000, 1000, 1000, True),    # ragged M, N and K
    (384, 2048, 512, False),     # three tiles: one CTA per tile
    (2048, 4096, 2048, True),    # persistent pairs (K <= 4096)
    (256, 8192, 1024, True),     # few pair tiles: split-K
    (2048, 1024, 100, True),     # N = 100: the second CTA's half of B lies past N (zeros)
    (512, 1024, 4099, True),     # N not a multiple of 4: scalar epilogue loads and stores
])
def test_pairs_match_single_cta_tiles(gpu, m, k, n, paired):
    api = gpu
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = rng.uniform(-1, 1, n).astype(np.float32)
    A, B, C = api.tensor([m, k], a), api.tensor([k, n], b), api.tensor([n], c)
    (zp, dp), (zs, ds) = _both(api, lambda: api.relu(api.matmul(A, B) + api.broadcast_to(C, [m, n])))
    assert ("CTA pairs" in dp) == paired, dp
    assert "CTA pairs" not in ds, ds
    assert_bitwise(zp, zs, f"pairs vs single {m}x{k}x{n}")
    ref = np.maximum(a.astype(np.float64) @ b.astype(np.float64) + c, 0.0)
    assert matmul_error(zp.reshape(m, n), ref, k) <= MATMUL_TOL


def test_pairs_match_single_through_softmax_and_split_output(gpu):
    api = gpu
    m, d, h = 1024, 1024, 2048
    rng = np.random.default_rng(77)
    x = rng.normal(0, 1, (m, d)).astype(np.float32)
    w1 = rng.normal(0, 1 / 32, (d, h)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, h).astype(np.float32)
    w2 = rng.normal(0, 1 / 45, (h, d)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, d).astype(np.float32)
    X, W1, B1, W2, B2 = (api.tensor(list(v.shape), v) for v in (x, w1, b1, w2, b2))

    def mlp():
        hid = api.logistic(api.matmul(X, W1) + api.broadcast_to(B1, [m, h]))
        return api.softmax(api.matmul(hid, W2) + api.broadcast_to(B2, [m, d]), 1)

    (pp, dp), (ps, ds) = _both(api, mlp)
    assert "CTA pairs" in dp and "split-output" in dp, dp
    assert "softmax epilogue" in dp or "split-K softmax combine" in dp, dp
    assert "CTA pairs" not in ds, ds
    assert_bitwise(pp, ps, "MLP: pairs vs single")


def test_pairs_match_single_through_the_softmax_epilogue(gpu):
    # Enough pair tiles (8 x 16) that the softmax epilogue runs without split-K.
    api = gpu
    m, k, n = 2048, 1024, 4096
    rng = np.random.default_rng(78)
    h = rng.uniform(0, 1, (m, k)).astype(np.float32)
    w = rng.normal(0, 1 / 32, (k, n)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    H, W, B = api.tensor([m, k], h), api.tensor([k, n], w), api.tensor([n], b)
    (pp, dp), (ps, ds) = _both(api, lambda: api.softmax(api.matmul(H, W) + api.broadcast_to(B, [m, n]), 1))
    assert "CTA pairs" in dp and "softmax epilogue" in dp, dp
    assert "CTA pairs" not in ds, ds
    assert_bitwise(pp, ps, "softmax epilogue: pairs vs single")


def test_pairs_with_split_parts_of_odd_length(gpu):
    """256 x 1040 x 512: split-K x4 over 65 k-blocks of 16, parts of 17 for
    one CTA per tile; a pair's parts are whole 32-wide k-blocks (18 of 16,
    the last part reading zeros past K). The split points differ, so the
    two forms are compared with fp64, each within the sqrt(K)-normalised
    bar, not bit for bit."""
    api = gpu
    m, k, n = 256, 1040, 512
    rng = np.random.default_rng(81)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    A, B = api.tensor([m, k], a), api.tensor([k, n], b)
    (zp, dp), (zs, ds) = _both(api, lambda: api.matmul(A, B))
    assert "CTA pairs" in dp and "split-K x4" in dp, dp
    assert "CTA pairs" not in ds and "split-K x4" in ds, ds
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert matmul_error(zp.reshape(m, n), ref, k) <= MATMUL_TOL
    assert matmul_error(zs.reshape(m, n), ref, k) <= MATMUL_TOL
