"""A device-side bounded wait that expires, recovered from without a fault.

Every mbarrier wait in the tcgen05 GEMM is bounded by a clock64 budget
(about two seconds); on expiry the kernel records a code in the device's
error word, stops issuing, waits (bounded) for its own copies and MMAs in
flight, frees its tensor memory and returns. The test hook
pb_test_gemm_stall makes one CTA wait on an mbarrier that nothing arrives
on, so that path runs for real: the next synchronisation raises with the
site code, and the same GPU then realises GEMMs normally (which it could
not if the tensor memory had not been freed, or if the context were lost).
Nothing faults, traps or hangs the GPU.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_expired_gemm_wait_reports_and_the_gpu_recovers(gpu):
    api = gpu
    from porch_b200._lib import lib

    L = lib()
    m, k, n = 256, 1024, 512  # tensor-core eligible (M * N * K = 2^27)
    rng = np.random.default_rng(21)
    a = rng.integers(-3, 4, (m, k)).astype(np.float32)
    b = rng.integers(-3, 4, (k, n)).astype(np.float32)
    A, B = api.tensor([m, k], a), api.tensor([k, n], b)
    assert "tcgen05" in api.describe(api.matmul(A, B))
    assert L.pb_test_gemm_stall(1) == 0
    try:
        with pytest.raises(RuntimeError, match="kernel error code 31751"):  # 0x7c00 + site 7
            api.materialize(api.matmul(A, B)).cpu()
    finally:
        assert L.pb_test_gemm_stall(0) == 0
    # The error word was cleared, the context is usable and the tensor
    # memory was given back: the same GEMM (a normal plan) is exact again.
    want = (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)
    for _ in range(2):
        got = api.materialize(api.matmul(A, B)).cpu().reshape(m, n)
        assert np.array_equal(got, want)
    api.synchronize()
