"""pb_matmul_3xtf32_noalloc: a matmul entry point that allocates no device
memory. It exists for callers that cannot let a library allocate, such as
code whose device memory is owned by its own arena or allocator hook. The
caller passes input and output device buffers; the split operands live in a
fixed file-scope device array.

Checked through the C-ABI against the regular entry point
(pb_materialize(matmul(A, B))), on two calls in a row with different shapes
and values, within the matmul tolerance the other tests use. Collected last
(file name) so a run that stops at the first failure has already run every
other test; it also passes alone in a fresh process.
"""

import numpy as np
import pytest

from tolerances import MATMUL_TOL, matmul_error

pytestmark = pytest.mark.gpu


def _device_tensor(api, shape, values):
    # pb_tensor_create keeps no host mirror, so later reads come from device
    # memory (where the no-allocation call writes).
    return api.tensor(list(shape), values)


def test_noalloc_matmul_matches_regular_entry_point(gpu):
    api = gpu
    from porch_b200._lib import lib

    L = lib()
    for call, (m, k, n) in enumerate([(512, 512, 512), (256, 1024, 768)]):
        rng = np.random.default_rng(1000 + call)
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        A = _device_tensor(api, [m, k], a)
        B = _device_tensor(api, [k, n], b)
        C = _device_tensor(api, [m, n], np.full(m * n, np.nan, dtype=np.float32))
        pa, _ = A.device_data()
        pb, _ = B.device_data()
        pc, _ = C.device_data()
        status = L.pb_matmul_3xtf32_noalloc(pa, pb, pc, m, n, k, None)
        assert status == 0, L.pb_last_error().decode()
        got = C.cpu().reshape(m, n)
        want = api.materialize(api.matmul(A, B)).cpu().reshape(m, n)
        assert np.isfinite(got).all()
        assert matmul_error(got, want.astype(np.float64), k) <= MATMUL_TOL
        ref = a.astype(np.float64) @ b.astype(np.float64)
        assert matmul_error(got, ref, k) <= MATMUL_TOL


def test_noalloc_matmul_rejects_sizes_beyond_its_scratch(gpu):
    api = gpu
    from porch_b200._lib import lib

    L = lib()
    A = _device_tensor(api, [128, 64], np.zeros(128 * 64, dtype=np.float32))
    pa, _ = A.device_data()
    # 2 * (M*K + N*K) floats > the 64 MiB array: rejected before any work.
    status = L.pb_matmul_3xtf32_noalloc(pa, pa, pa, 4096, 4096, 4096, None)
    assert status == 1
    assert "scratch" in L.pb_last_error().decode()
    # Shapes the kernel cannot tile are rejected too.
    assert L.pb_matmul_3xtf32_noalloc(pa, pa, pa, 100, 256, 64, None) == 1


def test_noalloc_matmul_refuses_nonfinite_operands_and_recovers(gpu):
    api = gpu
    from porch_b200._lib import lib

    L = lib()
    m = k = n = 512
    rng = np.random.default_rng(77)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bad = a.copy()
    bad[5, 6] = np.inf
    A_bad = _device_tensor(api, [m, k], bad)
    A = _device_tensor(api, [m, k], a)
    B = _device_tensor(api, [k, n], b)
    C = _device_tensor(api, [m, n], np.zeros(m * n, dtype=np.float32))
    pab, _ = A_bad.device_data()
    pa, _ = A.device_data()
    pb, _ = B.device_data()
    pc, _ = C.device_data()
    assert L.pb_matmul_3xtf32_noalloc(pab, pb, pc, m, n, k, None) == 1
    assert "Inf or NaN" in L.pb_last_error().decode()
    # The flag was cleared: a finite call afterwards succeeds.
    assert L.pb_matmul_3xtf32_noalloc(pa, pb, pc, m, n, k, None) == 0, L.pb_last_error().decode()
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert matmul_error(C.cpu().reshape(m, n), ref, k) <= MATMUL_TOL
