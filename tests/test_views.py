"""Realised data movement as strided views (no copy until values are read).

The reference realises a slice or transpose into a new contiguous buffer
(src/tensor.cpp:1002-1066, one elementwise kernel) and refuses
non-contiguous storage (src/tensor.cpp:1193-1197); its transpose is rank 2
only (src/tensor.cpp:430-437). Here materialising a graph that only slices,
transposes, permutes, unsqueezes or contiguously reshapes one realised tensor
launches nothing; later graphs -- the tcgen05 GEMM's operand split included --
read the view in place, and the values are copied out only when they are
read. Results are compared bit for bit with numpy (data movement, and
integer-valued GEMMs whose every product and sum is exact in fp32).
"""

import ctypes

import numpy as np
import pytest

from tolerances import assert_bitwise

pytestmark = pytest.mark.gpu


def _ints(shape, seed, lo=-3, hi=4):
    return np.random.default_rng(seed).integers(lo, hi, shape).astype(np.float32)


def _launched(api, fn):
    """Runs fn() with per-launch profiling; returns (result, {kernel: launches})."""
    api.synchronize()
    api.profile_enable(True)
    api.profile_read()
    try:
        out = fn()
        api.synchronize()
        prof = api.profile_read()
    finally:
        api.profile_enable(False)
    return out, {k: n for k, (n, _) in prof.items()}


def test_realised_slice_is_a_view_read_in_place(gpu):
    api = gpu
    x = _ints([64, 96], 1)
    X = api.tensor([64, 96], x)
    V, kernels = _launched(api, lambda: api.materialize(X[2:50:3, 5:90:2]))
    assert kernels == {}, kernels
    want = x[2:50:3, 5:90:2]
    assert V.shape() == list(want.shape)
    assert V.is_contiguous() and V.strides() == [want.shape[1], 1]
    # A graph over the view reads the base in place: one elementwise kernel.
    Y, kernels = _launched(api, lambda: api.materialize(V * 2.0 + 1.0))
    assert sum(kernels.values()) == 1 and all(k.startswith("pb_elem") for k in kernels), kernels
    assert_bitwise(Y.cpu().reshape(want.shape), want * np.float32(2) + np.float32(1), "graph over a view")
    # Reading the view's own values copies them out once.
    assert_bitwise(V.cpu().reshape(want.shape), want, "view values")


def test_chained_views_compose(gpu):
    api = gpu
    x = _ints([8, 6, 10], 2)
    X = api.tensor([8, 6, 10], x)

    def chain():
        a = api.materialize(X[1:7:2, api.all, 3:9])          # [3, 6, 6]
        b = api.materialize(api.permute(a, [2, 0, 1]))      # [6, 3, 6]
        c = api.materialize(api.unsqueeze(b, 1))            # [6, 1, 3, 6]
        d = api.materialize(c[0:5:2, 0, 1:, ::5])           # [3, 2, 2]
        return a, b, c, d

    (a, b, c, d), kernels = _launched(api, chain)
    assert kernels == {}, kernels
    wa = x[1:7:2, :, 3:9]
    wb = np.transpose(wa, (2, 0, 1))
    wc = wb[:, None]
    wd = wc[0:5:2, 0, 1:, ::5]
    for got, want, what in [(a, wa, "slice"), (b, wb, "permute"), (c, wc, "unsqueeze"), (d, wd, "re-slice")]:
        assert got.shape() == list(want.shape), what
        assert_bitwise(got.cpu().reshape(want.shape), want, what)
    # A contiguous reshape of a contiguous view is a view too; a reshape of a
    # transposed view is not (it is copied by a kernel).
    r, kernels = _launched(api, lambda: api.materialize(api.reshape(X[2:4], [120])))
    assert kernels == {}
    assert_bitwise(r.cpu(), x[2:4].reshape(-1), "reshape view")
    t, kernels = _launched(api, lambda: api.materialize(api.reshape(api.permute(X, [1, 0, 2]), [480])))
    assert sum(kernels.values()) == 1
    assert_bitwise(t.cpu(), np.transpose(x, (1, 0, 2)).reshape(-1), "reshape of a permute")


def test_views_feed_the_tensor_core_gemm_without_a_copy(gpu):
    """X realised, re-sliced and transposed as views, then the A operand of a
    tcgen05 GEMM: the launch list holds the GEMM's own kernels (operand
    splits, the GEMM, its guarded fallback) and no copy kernel."""
    api = gpu
    x = _ints([1024, 2048], 3)
    w = _ints([512, 1024], 4)
    X = api.tensor([1024, 2048], x)
    W = api.tensor([512, 1024], w)
    v1 = api.materialize(X[0::2, 1024:2048])          # [512, 1024] view, row stride 4096
    v2 = api.materialize(api.transpose(v1))           # [1024, 512] view, strides (1, 4096)
    C, kernels = _launched(api, lambda: api.materialize(api.relu(api.matmul(v2, W) + 1.0)))
    assert any(k.startswith("pb_gemm_tc") for k in kernels), kernels
    copies = [k for k in kernels if k.startswith(("pb_elem", "pb_gather"))]
    assert not copies, kernels
    a = np.ascontiguousarray(x[0::2, 1024:2048].T).astype(np.float64)
    want = np.maximum(a @ w.astype(np.float64) + 1.0, 0.0).astype(np.float32)
    assert_bitwise(C.cpu().reshape(1024, 1024), want, "gemm over views")
    # The B operand as a transposed view takes the row split (already K-major).
    wt = _ints([1024, 512], 5)
    Wt = api.tensor([1024, 512], wt)
    D, kernels = _launched(api, lambda: api.materialize(api.matmul(v2, api.materialize(api.transpose(Wt)))))
    assert not [k for k in kernels if k.startswith(("pb_elem", "pb_gather"))], kernels
    want = (a @ wt.T.astype(np.float64)).astype(np.float32)
    assert_bitwise(D.cpu().reshape(1024, 1024), want, "gemm with a transposed B view")


def test_view_is_a_snapshot_when_its_base_is_written(gpu):
    """Before a handle to the base's values leaves the library, its views
    are copied out, so writing the base afterwards leaves them unchanged
    (the reference's materialise is a copy)."""
    api = gpu
    from porch_b200._lib import lib

    x = _ints([16, 16], 6)
    X = api.tensor([16, 16], x)
    V = api.materialize(X[::2, 3:11])
    ptr, nbytes = X.device_data()  # the handle escapes: V is copied out first
    new = np.full(256, 7.0, dtype=np.float32)
    L = lib()
    stream = ctypes.c_void_p()
    assert L.pbrt_stream_current(0, ctypes.byref(stream)) == 0
    assert L.pbrt_memcpy_h2d_async(0, ptr, new.ctypes.data, nbytes, stream) == 0
    assert L.pbrt_stream_synchronize(0, stream) == 0
    assert_bitwise(V.cpu().reshape(8, 8), x[::2, 3:11], "view after its base was written")
    # New slices of the escaped base are copies of the new values.
    W, kernels = _launched(api, lambda: api.materialize(X[::2, 3:11]))
    assert sum(kernels.values()) == 1
    assert_bitwise(W.cpu(), np.full(64, 7.0, dtype=np.float32), "slice of the written base")


def test_permute_checks_its_axes(gpu):
    api = gpu
    X = api.tensor([2, 3, 4], np.zeros(24, dtype=np.float32))
    for bad in ([0, 1], [0, 1, 1], [0, 1, 3], [-1, 0, 1]):
        with pytest.raises(ValueError, match="permut"):
            api.permute(X, bad)
    # Transpose keeps the reference's rank-2 rule.
    with pytest.raises(ValueError, match="rank-2"):
        api.materialize(api.transpose(X))
    # A permute inside a larger graph lowers like any other index map.
    x = _ints([5, 7, 9], 7)
    Y = api.tensor([5, 7, 9], x)
    got = api.materialize(api.permute(Y, [1, 2, 0]) * 3.0).cpu().reshape(7, 9, 5)
    assert_bitwise(got, np.transpose(x, (1, 2, 0)) * np.float32(3), "permute in a graph")


def test_threads_reading_one_view_concurrently(gpu):
    """Several threads realise graphs over, and read the values of, the same
    view at once: each first read copies the view out; one copy wins, and
    every reader sees the same values."""
    import threading

    api = gpu
    x = _ints([256, 512], 8)
    X = api.tensor([256, 512], x)
    V = api.materialize(api.transpose(X[16:240:2, 100:400]))
    want = np.ascontiguousarray(x[16:240:2, 100:400].T)
    errors = []

    def reader(j):
        try:
            for _ in range(5):
                got = api.materialize(V * float(j + 1)).cpu().reshape(want.shape)
                assert np.array_equal(got, want * np.float32(j + 1))
                assert np.array_equal(V.cpu().reshape(want.shape), want)
        except Exception as exc:  # reported below
            errors.append(repr(exc))

    threads = [threading.Thread(target=reader, args=(j,)) for j in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    api.synchronize()
    assert not errors, errors
