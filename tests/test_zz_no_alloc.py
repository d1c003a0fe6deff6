"""pb_matmul_3xtf32_noalloc: a matmul entry point that allocates no device
memory. It exists for callers that cannot let a library allocate, such as
code whose device memory is owned by its own arena or allocator hook. The
caller passes input and output device buffers; the split operands live in a
fixed file-scope device array.

Checked through the C-ABI against the regular entry point
(pb_materialize(matmul(A, B))), on two calls in a row with different shapes
and values, within the matmul tolerance the other tests use; at the largest
K its 64 MiB array admits, within 4x a sequential fp32 chain's own error (the
bound the main GEMM's tests use); and a call after the first one on a device
leaves the device's free memory unchanged. Collected last (file name) so a
run that stops at the first failure has already run every other test; it
also passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest

from tolerances import MATMUL_TOL, matmul_error

pytestmark = pytest.mark.gpu


def _device_tensor(api, shape, values):
    # pb_tensor_create keeps no host mirror, so later reads come from device
    # memory (where the no-allocation call writes).
    return api.tensor(list(shape), values)


def _lib():
    from porch_b200._lib import lib

    return lib()


def test_noalloc_matmul_matches_regular_entry_point(gpu):
    api = gpu
    L = _lib()
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


def test_noalloc_matmul_at_its_largest_k_stays_within_the_fp32_chain(gpu):
    """K = 21824 is the largest multiple of 64 with 2*(M*K + N*K) within the
    64 MiB array at M = 128, N = 256. The accumulation is drained period by
    period, so the error stays within 4x the reference's sequential fp32
    chain (src/tensor.cpp:684-721 accumulates `sum += L * R` over k)."""
    api = gpu
    L = _lib()
    m, n, k = 128, 256, 21824
    rng = np.random.default_rng(4242)
    s = 1.0 / np.sqrt(k)
    a = rng.uniform(-s, s, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    A, B = _device_tensor(api, [m, k], a), _device_tensor(api, [k, n], b)
    C = _device_tensor(api, [m, n], np.zeros(m * n, dtype=np.float32))
    pa, _ = A.device_data()
    pb, _ = B.device_data()
    pc, _ = C.device_data()
    assert L.pb_matmul_3xtf32_noalloc(pa, pb, pc, m, n, k, None) == 0, L.pb_last_error().decode()
    got = C.cpu().reshape(m, n)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    chain = np.zeros((m, n), dtype=np.float32)
    for kk in range(k):
        chain = (chain + np.outer(a[:, kk], b[kk, :]).astype(np.float32)).astype(np.float32)
    err, chain_err = matmul_error(got, ref, k), matmul_error(chain, ref, k)
    print(f"K={k}: noalloc {err:.3e}, fp32 chain {chain_err:.3e}")
    assert err <= MATMUL_TOL
    assert err <= 4 * chain_err, (err, chain_err)
    # The regular entry point on the same operands agrees within the bound.
    want = api.materialize(api.matmul(A, B)).cpu().reshape(m, n)
    assert matmul_error(got, want.astype(np.float64), k) <= MATMUL_TOL


def test_noalloc_matmul_rejects_sizes_and_pointers_it_cannot_take(gpu):
    api = gpu
    L = _lib()
    A = _device_tensor(api, [128, 256], np.zeros(128 * 256, dtype=np.float32))
    pa, _ = A.device_data()
    # 2 * (M*K + N*K) floats > the 64 MiB array: rejected before any work.
    assert L.pb_matmul_3xtf32_noalloc(pa, pa, pa, 4096, 4096, 4096, None) == 1
    assert "scratch" in L.pb_last_error().decode()
    # Extents whose products would wrap 64 bits are rejected the same way.
    assert L.pb_matmul_3xtf32_noalloc(pa, pa, pa, (1 << 57) + 128, 256, 128, None) == 1
    assert "scratch" in L.pb_last_error().decode()
    # Shapes the kernel cannot tile are rejected too.
    assert L.pb_matmul_3xtf32_noalloc(pa, pa, pa, 100, 256, 64, None) == 1
    # A misaligned output (one float into a buffer) is refused before any
    # kernel runs: its 16-byte stores would fault.
    assert L.pb_matmul_3xtf32_noalloc(pa, pa, pa + 4, 128, 256, 64, None) == 1
    assert "aligned" in L.pb_last_error().decode()
    # Host memory is refused: the kernels would fault on it.
    host = np.zeros(128 * 256, dtype=np.float32)
    hp = host.ctypes.data
    assert L.pb_matmul_3xtf32_noalloc(hp, pa, pa, 128, 256, 64, None) == 1
    assert "device memory" in L.pb_last_error().decode() or "knows" in L.pb_last_error().decode()
    # After the refusals the entry point still works.
    B = _device_tensor(api, [64, 256], np.ones(64 * 256, dtype=np.float32))
    Cm = _device_tensor(api, [128, 256], np.zeros(128 * 256, dtype=np.float32))
    A2 = _device_tensor(api, [128, 64], np.ones(128 * 64, dtype=np.float32))
    p2, _ = A2.device_data()
    pb, _ = B.device_data()
    pc, _ = Cm.device_data()
    assert L.pb_matmul_3xtf32_noalloc(p2, pb, pc, 128, 256, 64, None) == 0, L.pb_last_error().decode()
    assert np.array_equal(Cm.cpu().reshape(-1), np.full(128 * 256, 64.0, dtype=np.float32))


def test_noalloc_matmul_refuses_nonfinite_operands_and_recovers(gpu):
    api = gpu
    L = _lib()
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


def _free_device_bytes(device: int = 0) -> int:
    """cuMemGetInfo on `device`'s primary context (the one the library and
    the CUDA runtime share)."""
    cu = ctypes.CDLL("libcuda.so.1")
    assert cu.cuInit(0) == 0
    ctx = ctypes.c_void_p()
    assert cu.cuDevicePrimaryCtxRetain(ctypes.byref(ctx), ctypes.c_int(device)) == 0
    try:
        assert cu.cuCtxPushCurrent_v2(ctx) == 0
        free, total = ctypes.c_size_t(), ctypes.c_size_t()
        assert cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
        popped = ctypes.c_void_p()
        assert cu.cuCtxPopCurrent_v2(ctypes.byref(popped)) == 0
    finally:
        cu.cuDevicePrimaryCtxRelease_v2(ctypes.c_int(device))
    return int(free.value)


def test_noalloc_matmul_allocates_no_device_memory(gpu):
    """After the first call on a device (which loads the kernels and the
    fixed array), further calls leave the device's free memory unchanged."""
    api = gpu
    L = _lib()
    m, k, n = 512, 1024, 512
    rng = np.random.default_rng(5)
    A = _device_tensor(api, [m, k], rng.uniform(-1, 1, (m, k)).astype(np.float32))
    B = _device_tensor(api, [k, n], rng.uniform(-1, 1, (k, n)).astype(np.float32))
    C = _device_tensor(api, [m, n], np.zeros(m * n, dtype=np.float32))
    pa, _ = A.device_data()
    pb, _ = B.device_data()
    pc, _ = C.device_data()
    assert L.pb_matmul_3xtf32_noalloc(pa, pb, pc, m, n, k, None) == 0, L.pb_last_error().decode()
    before = _free_device_bytes()
    for _ in range(3):
        assert L.pb_matmul_3xtf32_noalloc(pa, pb, pc, m, n, k, None) == 0, L.pb_last_error().decode()
    after = _free_device_bytes()
    assert after >= before, f"{before - after} bytes of device memory were allocated by the calls"
