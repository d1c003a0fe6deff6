"""Several host threads on one device (the reference's threading contract:
handles copy across threads, a shared lazy tensor materialises once,
streams are per thread -- include/porch/tensor.hpp, src/tensor.cpp:1070-1079,
src/cuda_jit.cpp:524-528).

Each thread builds and realises graphs of every kernel family on its own
stream, some shared across threads, first-use plan resolution included;
every result must equal the single-threaded one bit for bit.
"""

import threading

import numpy as np
import pytest


def _graphs(api, t):
    x, y, w = t["x"], t["y"], t["w"]
    return {
        "elementwise": (x + y) * 2.0 - 1.0,
        "view": api.concat(api.transpose(x[0::2, 0:64]) + 1.0, y[0:64, 0:256], 0),
        "softmax": api.softmax(x, 1),
        "reduce0": api.sum(x, 0),
        "reduce1": api.max(y, 1),
        "matmul": api.relu(api.matmul(x, w)),
    }


@pytest.mark.gpu
def test_threads_realise_the_same_values(gpu):
    api = gpu
    rng = np.random.default_rng(17)
    hx = rng.normal(0, 1, (512, 256)).astype(np.float32)
    hy = rng.normal(0, 1, (512, 256)).astype(np.float32)
    hw = rng.uniform(-1, 1, (256, 1024)).astype(np.float32) / 16
    shared = {"x": api.tensor([512, 256], hx), "y": api.tensor([512, 256], hy),
              "w": api.tensor([256, 1024], hw)}
    # A lazy tensor shared by every thread: realised exactly once.
    lazy = api.as_tensor(api.exp(shared["x"]) * 0.5)

    # The threads are the first to realise these graphs, so plan building,
    # compilation and per-device function resolution race as well.
    results = {}
    errors = []
    start = threading.Barrier(6)

    def worker(i):
        try:
            start.wait()
            for rep in range(4):
                # Half the threads reuse the shared inputs, half make their own.
                if i % 2:
                    t = shared
                else:
                    t = {"x": api.tensor([512, 256], hx), "y": api.tensor([512, 256], hy),
                         "w": api.tensor([256, 1024], hw)}
                for k, e in _graphs(api, t).items():
                    results[(i, rep, k)] = api.materialize(e).cpu()
                results[(i, rep, "lazy")] = lazy.cpu()
        except Exception as exc:  # reported below, not lost in the thread
            errors.append((i, repr(exc)))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(6)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads)
    assert not errors, errors[:10]

    want = {k: api.materialize(e).cpu() for k, e in _graphs(api, shared).items()}
    want["lazy"] = lazy.cpu()
    bad = [key for key, got in results.items()
           if not np.array_equal(got.view(np.uint32), want[key[2]].view(np.uint32))]
    assert len(results) == 6 * 4 * 7
    assert not bad, bad[:10]


@pytest.mark.gpu
def test_slab_allocator_serves_misses_without_driver_calls_and_releases(gpu):
    """Cache misses are carved from 256 MiB slabs: many distinct block sizes
    cost at most a slab or two, and dropping the cache gives a slab whose
    blocks are all gone back to the driver."""
    import ctypes

    api = gpu
    cu = ctypes.CDLL("libcuda.so.1")

    def free_bytes():
        ctx = ctypes.c_void_p()
        assert cu.cuDevicePrimaryCtxRetain(ctypes.byref(ctx), 0) == 0
        assert cu.cuCtxPushCurrent_v2(ctx) == 0
        f, t = ctypes.c_size_t(), ctypes.c_size_t()
        assert cu.cuMemGetInfo_v2(ctypes.byref(f), ctypes.byref(t)) == 0
        assert cu.cuCtxPopCurrent_v2(ctypes.byref(ctypes.c_void_p())) == 0
        cu.cuDevicePrimaryCtxRelease_v2(0)
        return f.value

    api.synchronize()
    api.empty_cache(0)
    base = free_bytes()
    api.host_profile_enable(True)
    api.host_profile_read()
    held = []
    for i in range(40):  # 40 distinct sizes from 40 KB to 1.6 MB: all misses
        n = 1024 * (i + 1) * 10
        held.append(api.materialize(api.tensor([n], np.ones(n, np.float32)) + float(i)))
    api.synchronize()
    counters = api.host_profile_read()
    api.host_profile_enable(False)
    assert counters.get("alloc_cache_miss", 0) >= 40
    assert counters.get("slab_alloc", 0) <= 2, counters
    for i in range(len(held)):
        assert float(held[i].cpu().reshape(-1)[0]) == 1.0 + i
    held.clear()
    api.synchronize()
    api.empty_cache(0)
    assert free_bytes() >= base - (64 << 20)


@pytest.mark.gpu
def test_async_uploads_order_each_reader_behind_its_own_copy(gpu):
    """pb_tensor_create_async returns before its copy is done; every reader
    (a kernel, a host read, a handed-out pointer) waits for that tensor's own
    copy. Five uploads, then graphs reading them in another order."""
    api = gpu
    rng = np.random.default_rng(3)
    arrays = [rng.integers(-8, 9, 1 << 22).astype(np.float32) for _ in range(5)]
    pinned = [api.PinnedBuffer(a.size) for a in arrays]
    for pb, a in zip(pinned, arrays):
        pb.array[:] = a
    for _ in range(3):
        ts = [api.tensor_from_pointer([a.size], pb.address, a.size, asynchronous=True)
              for a, pb in zip(arrays, pinned)]
        got = api.materialize((ts[4] - ts[0]) * 2.0 + ts[2]).cpu()
        assert np.array_equal(got, (arrays[4] - arrays[0]) * np.float32(2) + arrays[2])
        assert np.array_equal(ts[1].cpu(), arrays[1])
        ptr, nbytes = ts[3].device_data()
        assert ptr != 0 and nbytes == arrays[3].size * 4
        assert np.array_equal(ts[3].cpu(), arrays[3])
    api.synchronize()
