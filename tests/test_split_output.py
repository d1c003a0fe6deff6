"""A GEMM whose result only feeds another GEMM writes it as that GEMM's
3xTF32 operand halves.

In config 5, H = logistic(X@W1 + b1) is read only by H@W2: its GEMM's
epilogue writes hi = rn_tf32(y) and lo = rn_tf32(y - hi) straight into the
second GEMM's operand buffers, so neither H in fp32 nor a split pass over it
exists. The halves are the same roundings of the same fp32 values the split
pass computes from a realised H, so the one-graph product equals the staged
one bit for bit. Non-finite values travel as hi with lo = 0 and a flag that
sends both GEMMs to the reference's fp32 chain.
"""

import numpy as np
import pytest

import error_bounds
import graphs
from tolerances import REL_TOL, assert_bitwise

pytestmark = pytest.mark.gpu


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


def test_split_output_equals_the_staged_product(gpu):
    api = gpu
    m, d, h = 512, 1024, 2048
    rng = np.random.default_rng(31)
    x = rng.normal(0, 1, (m, d)).astype(np.float32)
    w1 = rng.normal(0, 1 / 32, (d, h)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, h).astype(np.float32)
    w2 = rng.normal(0, 1 / 45, (h, d)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, d).astype(np.float32)
    X, W1, B1, W2, B2 = (api.tensor(list(a.shape), a) for a in (x, w1, b1, w2, b2))
    hid = api.logistic(api.matmul(X, W1) + api.broadcast_to(B1, [m, h]))
    z_graph = api.matmul(hid, W2) + api.broadcast_to(B2, [m, d])
    plan = api.describe(z_graph)
    assert "split-output epilogue" in plan, plan
    Z, kernels = _kernels(api, lambda: api.materialize(z_graph))
    # X and W1, W2 are split; H is not (it arrives as halves).
    assert sum(n for k, n in kernels.items() if k.startswith(("pb_split_rows", "pb_split_transpose"))) == 3, kernels
    H = api.materialize(hid)
    Zs = api.materialize(api.matmul(H, W2) + api.broadcast_to(B2, [m, d]))
    assert_bitwise(Z.cpu(), Zs.cpu(), "split-output GEMM vs staged")
    # And through the softmax epilogue, the benchmark's one graph.
    P = api.materialize(api.softmax(z_graph, 1)).cpu().reshape(m, d)
    Ps = api.materialize(api.softmax(Zs, 1)).cpu().reshape(m, d)
    assert np.allclose(P, Ps, rtol=REL_TOL, atol=0)


def test_split_output_carries_nonfinite_values(gpu, oracle_lib):
    api = gpu
    m, d, h = 256, 512, 1024
    rng = np.random.default_rng(32)
    x = rng.integers(-2, 3, (m, d)).astype(np.float32)
    w1 = rng.integers(-2, 3, (d, h)).astype(np.float32)
    w2 = rng.integers(-2, 3, (h, d)).astype(np.float32)
    x[4, 9] = np.inf
    prog = ("0 input 0\n1 input 1\n2 input 2\n3 matmul 0 1\n4 relu 3\n5 matmul 4 2\n")
    want = graphs.evaluate_oracle(prog, [x, w1, w2])
    got = graphs.evaluate_product(api, prog, [x, w1, w2])
    assert "split-output" in api.describe(api.matmul(api.relu(api.matmul(api.tensor([m, d], x), api.tensor([d, h], w1))),
                                                     api.tensor([h, d], w2)))
    _, bound = error_bounds.evaluate(prog, [x, w1, w2])
    error_bounds.check(got, want, bound, REL_TOL, "non-finite through split output")
