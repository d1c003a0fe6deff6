"""Python mirror of the porch tensor API over the flat C-ABI
(include/porch_b200.h), bound with ctypes.

Names and argument meanings follow porch's C++ API (include/porch/tensor.hpp,
ops.hpp): `tensor`, `full`, `zeros`, operators, `matmul`, `reshape`,
`unsqueeze`, `transpose`, `broadcast_to`, `concat`, `sum`, `max`, `maximum`,
`minimum`, `exp`, `reciprocal`, `materialize`, `relu`, `softmax`,
`logistic`, and the tensor boundaries `realize`, `synchronize`, `cpu`,
`data`, `device_data`. Errors keep the C++ exception classes' meaning:

  std::invalid_argument -> InvalidArgument (a ValueError)
  std::out_of_range     -> OutOfRange (an IndexError)
  compilation_error     -> CompilationError (a RuntimeError)
  std::runtime_error    -> RuntimeError
"""

from __future__ import annotations

import builtins as _builtins
import ctypes
from ctypes import byref, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from typing import Iterable, Sequence

import numpy as np

from ._lib import lib, pb_index

PB_ADD, PB_SUBTRACT, PB_MULTIPLY, PB_DIVIDE, PB_MAXIMUM, PB_MINIMUM, PB_MATMUL = range(7)
PB_EXP, PB_RECIPROCAL, PB_TRANSPOSE, PB_RELU, PB_LOGISTIC, PB_SUM, PB_MAX = range(7, 14)


class InvalidArgument(ValueError):
    """std::invalid_argument"""


class OutOfRange(IndexError):
    """std::out_of_range"""


class CompilationError(RuntimeError):
    """porch::cuda_jit::compilation_error"""


def _check(status: int) -> None:
    if status == 0:
        return
    msg = lib().pb_last_error().decode(errors="replace")
    if status == 1:
        raise InvalidArgument(msg)
    if status == 2:
        raise OutOfRange(msg)
    if status == 4:
        raise CompilationError(msg)
    raise RuntimeError(msg)


def _shape_arg(shape: Sequence[int]):
    arr = (c_int64 * _builtins.max(1, len(shape)))(*[int(s) for s in shape])
    return arr, len(shape)


class _All:
    def __repr__(self) -> str:
        return "porch.all"


all = _All()  # noqa: A001  (porch::all marker)


def is_available() -> bool:
    return lib().pb_is_available() == 1


def device_count() -> int:
    """CUDA devices visible to this process (0 without a driver)."""
    if not is_available():
        return 0
    n = c_int(0)
    _check_rt(lib().pbrt_device_count(byref(n)))
    return n.value


def _check_rt(status: int) -> None:
    if status != 0:
        raise RuntimeError(lib().pbrt_last_error().decode(errors="replace"))


def backend_name() -> str:
    return lib().pb_backend_name().decode()


def synchronize() -> None:
    _check(lib().pb_synchronize())


class Expr:
    """porch::tensor_expr"""

    __slots__ = ("_h",)

    def __init__(self, handle: int):
        self._h = c_void_p(handle)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().pb_expr_release(h)
            except Exception:  # interpreter shutdown
                pass
            self._h = c_void_p(None)

    # -- metadata
    def shape(self) -> list[int]:
        buf = (c_int64 * 16)()
        rank = c_size_t(0)
        _check(lib().pb_expr_shape(self._h, buf, 16, byref(rank)))
        return [buf[i] for i in range(rank.value)]

    def rank(self) -> int:
        return len(self.shape())

    def numel(self) -> int:
        n = 1
        for s in self.shape():
            n *= s
        return n

    def eval(self) -> "Tensor":
        return materialize(self)

    def to_tensor(self) -> "Tensor":
        """tensor_expr::operator tensor(): a lazy tensor."""
        out = c_void_p()
        _check(lib().pb_expr_to_tensor(self._h, byref(out)))
        return Tensor(out.value)

    def describe(self, with_source: bool = False) -> str:
        return describe(self, with_source)

    # -- operators
    def __add__(self, o):
        return _binary(PB_ADD, self, o)

    def __radd__(self, o):
        return _binary(PB_ADD, o, self)

    def __sub__(self, o):
        return _binary(PB_SUBTRACT, self, o)

    def __rsub__(self, o):
        return _binary(PB_SUBTRACT, o, self)

    def __mul__(self, o):
        return _binary(PB_MULTIPLY, self, o)

    def __rmul__(self, o):
        return _binary(PB_MULTIPLY, o, self)

    def __truediv__(self, o):
        return _binary(PB_DIVIDE, self, o)

    def __rtruediv__(self, o):
        return _binary(PB_DIVIDE, o, self)


def _expr(x) -> Expr:
    if isinstance(x, Expr):
        return x
    if isinstance(x, Tensor):
        out = c_void_p()
        _check(lib().pb_expr_from_tensor(x._h, byref(out)))
        return Expr(out.value)
    if isinstance(x, (int, float, np.floating, np.integer)):
        out = c_void_p()
        _check(lib().pb_expr_scalar(c_float(float(x)), byref(out)))
        return Expr(out.value)
    raise TypeError(f"cannot convert {type(x).__name__} to a tensor expression")


def _binary(op: int, a, b) -> Expr:
    ea, eb = _expr(a), _expr(b)
    out = c_void_p()
    _check(lib().pb_expr_binary(op, ea._h, eb._h, byref(out)))
    return Expr(out.value)


def _unary(op: int, a) -> Expr:
    ea = _expr(a)
    out = c_void_p()
    _check(lib().pb_expr_unary(op, ea._h, byref(out)))
    return Expr(out.value)


class Tensor:
    """porch::tensor (a shared handle)."""

    __slots__ = ("_h",)

    def __init__(self, handle: int):
        self._h = c_void_p(handle)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().pb_tensor_release(h)
            except Exception:
                pass
            self._h = c_void_p(None)

    # -- metadata
    def shape(self) -> list[int]:
        r = self.rank()
        buf = (c_int64 * _builtins.max(1, r))()
        _check(lib().pb_tensor_shape(self._h, buf, r))
        return [buf[i] for i in range(r)]

    def strides(self) -> list[int]:
        r = self.rank()
        buf = (c_int64 * _builtins.max(1, r))()
        _check(lib().pb_tensor_strides(self._h, buf, r))
        return [buf[i] for i in range(r)]

    def rank(self) -> int:
        r = c_size_t(0)
        _check(lib().pb_tensor_rank(self._h, byref(r)))
        return r.value

    def numel(self) -> int:
        n = c_size_t(0)
        _check(lib().pb_tensor_numel(self._h, byref(n)))
        return n.value

    def storage_offset(self) -> int:
        o = c_int64(0)
        _check(lib().pb_tensor_storage_offset(self._h, byref(o)))
        return o.value

    def is_contiguous(self) -> bool:
        c = c_int(0)
        _check(lib().pb_tensor_is_contiguous(self._h, byref(c)))
        return bool(c.value)

    def placement(self) -> int:
        d = c_int(0)
        _check(lib().pb_tensor_device(self._h, byref(d)))
        return d.value

    # -- boundaries
    def realize(self) -> "Tensor":
        _check(lib().pb_tensor_realize(self._h))
        return self

    def synchronize(self) -> None:
        _check(lib().pb_tensor_synchronize(self._h))

    def cpu(self, out: np.ndarray | None = None) -> np.ndarray:
        n = self.numel()
        if out is None:
            out = np.empty(n, dtype=np.float32)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == n
        _check(lib().pb_tensor_read(self._h, out.ctypes.data_as(c_void_p), n))
        return out.reshape(self.shape()) if out.ndim == 1 and self.rank() != 1 else out

    def data(self) -> np.ndarray:
        return self.cpu().reshape(-1)

    def device_data(self) -> tuple[int, int]:
        """(device address, size in bytes) of tensor::device_data()."""
        p = c_uint64(0)
        b = c_size_t(0)
        _check(lib().pb_tensor_device_pointer(self._h, byref(p), byref(b)))
        return p.value, b.value

    def __getitem__(self, key) -> Expr:
        if not isinstance(key, tuple):
            key = (key,)
        idx = (pb_index * _builtins.max(1, len(key)))()
        for i, k in enumerate(key):
            if k is all:
                idx[i].kind = 2
            elif isinstance(k, slice):
                idx[i].kind = 1
                idx[i].start = 0 if k.start is None else int(k.start)
                idx[i].stop = (2**62) if k.stop is None else int(k.stop)
                idx[i].step = 1 if k.step is None else int(k.step)
            else:
                idx[i].kind = 0
                idx[i].index = int(k)
        out = c_void_p()
        _check(lib().pb_tensor_index(self._h, idx, len(key), byref(out)))
        return Expr(out.value)

    # -- operators (tensor converts to tensor_expr, as in C++)
    def __add__(self, o):
        return _binary(PB_ADD, self, o)

    def __radd__(self, o):
        return _binary(PB_ADD, o, self)

    def __sub__(self, o):
        return _binary(PB_SUBTRACT, self, o)

    def __rsub__(self, o):
        return _binary(PB_SUBTRACT, o, self)

    def __mul__(self, o):
        return _binary(PB_MULTIPLY, self, o)

    def __rmul__(self, o):
        return _binary(PB_MULTIPLY, o, self)

    def __truediv__(self, o):
        return _binary(PB_DIVIDE, self, o)

    def __rtruediv__(self, o):
        return _binary(PB_DIVIDE, o, self)


# ----------------------------------------------------------------- builders --
def tensor(shape: Sequence[int], values, device: int = 0) -> Tensor:
    """porch::tensor(shape, values, device{device})"""
    vals = np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
    s, r = _shape_arg(shape)
    out = c_void_p()
    _check(lib().pb_tensor_create(s, r, vals.ctypes.data_as(ctypes.POINTER(c_float)),
                                  vals.size, int(device), byref(out)))
    return Tensor(out.value)


def tensor_from_pointer(shape: Sequence[int], pointer: int, count: int, device: int = 0,
                        asynchronous: bool = False) -> Tensor:
    """tensor from `count` floats at host address `pointer` (e.g. pinned).
    asynchronous=True enqueues the copy on this thread's upload stream and
    returns at once (pb_tensor_create_async): readers wait for it on the
    device, and the host memory must stay unchanged until it is done."""
    s, r = _shape_arg(shape)
    out = c_void_p()
    fn = lib().pb_tensor_create_async if asynchronous else lib().pb_tensor_create
    _check(fn(s, r, ctypes.cast(pointer, ctypes.POINTER(c_float)), count, int(device), byref(out)))
    return Tensor(out.value)


def placeholder(shape: Sequence[int], device: int = 0) -> Tensor:
    s, r = _shape_arg(shape)
    out = c_void_p()
    _check(lib().pb_tensor_placeholder(s, r, int(device), byref(out)))
    return Tensor(out.value)


def full(shape: Sequence[int], value: float, device: int = 0) -> Tensor:
    s, r = _shape_arg(shape)
    out = c_void_p()
    _check(lib().pb_tensor_full(s, r, c_float(value), int(device), byref(out)))
    return Tensor(out.value)


def zeros(shape: Sequence[int], device: int = 0) -> Tensor:
    return full(shape, 0.0, device)


def materialize(e) -> Tensor:
    ex = _expr(e)
    out = c_void_p()
    _check(lib().pb_materialize(ex._h, byref(out)))
    return Tensor(out.value)


def as_tensor(e) -> Tensor:
    """`porch::tensor t = expr;` (lazy)."""
    return _expr(e).to_tensor()


def add(a, b):
    return materialize(_binary(PB_ADD, a, b))


def subtract(a, b):
    return materialize(_binary(PB_SUBTRACT, a, b))


def multiply(a, b):
    return materialize(_binary(PB_MULTIPLY, a, b))


def divide(a, b):
    return materialize(_binary(PB_DIVIDE, a, b))


def matmul(a, b) -> Expr:
    return _binary(PB_MATMUL, a, b)


def maximum(a, b) -> Expr:
    return _binary(PB_MAXIMUM, a, b)


def minimum(a, b) -> Expr:
    return _binary(PB_MINIMUM, a, b)


def exp(a) -> Expr:
    return _unary(PB_EXP, a)


def reciprocal(a) -> Expr:
    return _unary(PB_RECIPROCAL, a)


def transpose(a) -> Expr:
    return _unary(PB_TRANSPOSE, a)


def relu(a) -> Expr:
    return _unary(PB_RELU, a)


def logistic(a) -> Expr:
    return _unary(PB_LOGISTIC, a)


def reshape(a, shape: Sequence[int]) -> Expr:
    ea = _expr(a)
    s, r = _shape_arg(shape)
    out = c_void_p()
    _check(lib().pb_expr_reshape(ea._h, s, r, byref(out)))
    return Expr(out.value)


def broadcast_to(a, shape: Sequence[int]) -> Expr:
    ea = _expr(a)
    s, r = _shape_arg(shape)
    out = c_void_p()
    _check(lib().pb_expr_broadcast(ea._h, s, r, byref(out)))
    return Expr(out.value)


def unsqueeze(a, axis: int) -> Expr:
    ea = _expr(a)
    out = c_void_p()
    _check(lib().pb_expr_unsqueeze(ea._h, int(axis), byref(out)))
    return Expr(out.value)


def batched_matmul(a, b) -> Expr:
    """[B, M, K] @ [B, K, N] -> [B, M, N]; an extension, the reference's
    matmul is rank 2 only."""
    ea, eb = _expr(a), _expr(b)
    out = c_void_p()
    _check(lib().pb_expr_batched_matmul(ea._h, eb._h, byref(out)))
    return Expr(out.value)


def permute(a, perm: Sequence[int]) -> Expr:
    """N-D axis permutation (output axis d = input axis perm[d]); an
    extension, the reference's transpose is rank 2 only."""
    ea = _expr(a)
    arr, n = _shape_arg(perm)
    out = c_void_p()
    _check(lib().pb_expr_permute(ea._h, arr, n, byref(out)))
    return Expr(out.value)


def concat(a, b, axis: int) -> Expr:
    ea, eb = _expr(a), _expr(b)
    out = c_void_p()
    _check(lib().pb_expr_concat(ea._h, eb._h, int(axis), byref(out)))
    return Expr(out.value)


def sum(a, axis: int, keepdim: bool = False) -> Expr:  # noqa: A001
    ea = _expr(a)
    out = c_void_p()
    _check(lib().pb_expr_reduce(PB_SUM, ea._h, int(axis), int(bool(keepdim)), byref(out)))
    return Expr(out.value)


def max(a, axis: int, keepdim: bool = False) -> Expr:  # noqa: A001
    ea = _expr(a)
    out = c_void_p()
    _check(lib().pb_expr_reduce(PB_MAX, ea._h, int(axis), int(bool(keepdim)), byref(out)))
    return Expr(out.value)


def softmax(a, axis: int) -> Expr:
    ea = _expr(a)
    out = c_void_p()
    _check(lib().pb_expr_softmax(ea._h, int(axis), byref(out)))
    return Expr(out.value)


def describe(e, with_source: bool = False) -> str:
    ex = _expr(e)
    need = c_size_t(0)
    _check(lib().pb_expr_describe(ex._h, int(with_source), None, 0, byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    _check(lib().pb_expr_describe(ex._h, int(with_source), buf, need.value, byref(need)))
    return buf.value.decode()


# -------------------------------------------------------------- utilities --
def fill_synthetic(out: np.ndarray, seed: int, dist: str, a: float, b: float) -> np.ndarray:
    """Seeded inputs: dist 'uniform' on [a, b) or 'normal' (mean a, stddev b)."""
    assert out.dtype == np.float32 and out.flags.c_contiguous
    code = {"uniform": 0, "normal": 1}[dist]
    _check(lib().pb_fill_synthetic(out.ctypes.data_as(c_void_p), out.size, int(seed), code,
                                   float(a), float(b)))
    return out


def compile_stats() -> dict[str, int]:
    """NVRTC compilations and on-disk cache hits in this process so far."""
    n, d = c_uint64(), c_uint64()
    lib().pbrt_compile_stats(byref(n), byref(d))
    return {"nvrtc_compiles": n.value, "disk_cache_hits": d.value}


def launch_count() -> int:
    return int(lib().pb_launch_count())


def profile_enable(on: bool = True) -> None:
    _check(lib().pb_profile_enable(int(on)))


def profile_read() -> dict[str, tuple[int, float]]:
    buf = ctypes.create_string_buffer(1 << 16)
    _check(lib().pb_profile_read(buf, len(buf)))
    out: dict[str, tuple[int, float]] = {}
    for line in buf.value.decode().splitlines():
        name, n, ms = line.split("\t")
        out[name] = (int(n), float(ms))
    return out


def host_profile_enable(on: bool = True) -> None:
    _check(lib().pb_host_profile_enable(int(on)))


def host_profile_read() -> dict[str, float]:
    buf = ctypes.create_string_buffer(4096)
    _check(lib().pb_host_profile_read(buf, len(buf)))
    out = {}
    for line in buf.value.decode().splitlines():
        k, v = line.split("\t")
        out[k] = float(v)
    return out


class DeviceTimer:
    """CUDA events on this thread's porch stream of `device`."""

    def __init__(self, device: int = 0):
        self.device = device
        self._t = c_void_p()

    def __enter__(self):
        _check(lib().pb_timer_begin(self.device, byref(self._t)))
        return self

    def __exit__(self, *exc):
        ms = c_float(0)
        _check(lib().pb_timer_end(self._t, byref(ms)))
        self.ms = ms.value
        return False


def device_synchronize(device: int = 0) -> None:
    _check(lib().pb_device_synchronize(int(device)))


def empty_cache(device: int = 0) -> int:
    """Returns every cached device block of `device` to the driver; the
    bytes released."""
    released = c_size_t()
    _check(lib().pb_empty_cache(int(device), byref(released)))
    return int(released.value)


class PinnedBuffer:
    """Page-locked host memory viewed as a float32 numpy array."""

    def __init__(self, count: int):
        self.count = int(count)
        self._p = c_void_p()
        _check(lib().pb_host_alloc(_builtins.max(4, self.count * 4), byref(self._p)))
        self.array = np.ctypeslib.as_array(
            ctypes.cast(self._p, ctypes.POINTER(c_float)), shape=(_builtins.max(1, self.count),))[: self.count]

    @property
    def address(self) -> int:
        return int(self._p.value)

    def free(self) -> None:
        if self._p.value:
            _check(lib().pb_host_free(self._p))
            self._p = c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def copy_bandwidth(device: int = 0, nbytes: int = 256 << 20, reps: int = 3) -> dict[str, float]:
    """Page-locked host <-> device copy rates in GB/s (best of `reps`, CUDA
    events on this thread's stream): the transfer bound of an end-to-end
    step whose inputs start in host memory and whose result ends there."""
    L = lib()
    stream = c_void_p()
    _check_rt(L.pbrt_stream_current(int(device), byref(stream)))
    dptr = c_uint64()
    _check_rt(L.pbrt_mem_alloc_async(int(device), int(nbytes), stream, byref(dptr)))
    host = PinnedBuffer(int(nbytes) // 4)
    ev = [c_void_p(), c_void_p()]
    for e in ev:
        _check_rt(L.pbrt_event_create(int(device), 1, byref(e)))
    out = {}
    try:
        copies = {
            "h2d": lambda: L.pbrt_memcpy_h2d_async(int(device), dptr.value, host.address, int(nbytes), stream),
            "d2h": lambda: L.pbrt_memcpy_d2h_async(int(device), host.address, dptr.value, int(nbytes), stream),
        }
        for name, copy in copies.items():
            best = float("inf")
            for _ in range(_builtins.max(1, reps)):
                _check_rt(L.pbrt_event_record(int(device), ev[0], stream))
                _check_rt(copy())
                _check_rt(L.pbrt_event_record(int(device), ev[1], stream))
                _check_rt(L.pbrt_event_synchronize(int(device), ev[1]))
                ms = c_float()
                _check_rt(L.pbrt_event_elapsed_ms(ev[0], ev[1], byref(ms)))
                best = _builtins.min(best, ms.value)
            out[name + "_gbs"] = nbytes / (best * 1e-3) / 1e9
    finally:
        for e in ev:
            L.pbrt_event_destroy(int(device), e)
        L.pbrt_mem_free_async(int(device), dptr.value, stream)
        L.pbrt_stream_synchronize(int(device), stream)
        host.free()
    return out


# ----------------------------------------------------------- row sharding --
def row_block(rows: int, rank: int, nranks: int) -> tuple[int, int]:
    """Rows [begin, end) of `rows` owned by `rank` of `nranks` (contiguous
    blocks; the first rows % nranks ranks hold one extra row)."""
    b, e = c_int64(), c_int64()
    _check(lib().pb_row_block(int(rows), int(rank), int(nranks), byref(b), byref(e)))
    return b.value, e.value


def comm_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (make on one rank, send to the rest)."""
    buf = ctypes.create_string_buffer(128)
    _check(lib().pb_comm_unique_id(buf))
    return buf.raw


class Communicator:
    """One rank of a one-process-per-GPU communicator (NCCL over NVLink)."""

    def __init__(self, nranks: int, unique_id: bytes, rank: int, device: int, timeout_s: float = 60.0):
        if len(unique_id) != 128:
            raise InvalidArgument("unique id must be 128 bytes")
        self._h = c_void_p()
        _check(lib().pb_comm_init(int(nranks), unique_id, int(rank), int(device), float(timeout_s),
                                  byref(self._h)))

    def info(self) -> tuple[int, int, int]:
        r, n, d = c_int(), c_int(), c_int()
        _check(lib().pb_comm_info(self._h, byref(r), byref(n), byref(d)))
        return r.value, n.value, d.value

    def allgather_rows(self, shard, total_rows: int, wait: bool = True) -> Tensor:
        """Whole [total_rows, ...] tensor from every rank's row block.
        wait=False enqueues the gather on the communicator's stream and
        returns at once (see wait())."""
        t = shard if isinstance(shard, Tensor) else materialize(shard)
        out = c_void_p()
        fn = lib().pb_allgather_rows if wait else lib().pb_allgather_rows_async
        _check(fn(self._h, t._h, int(total_rows), byref(out)))
        return Tensor(out.value)

    def wait(self) -> None:
        """Bounded wait for every asynchronous gather issued so far."""
        _check(lib().pb_comm_wait(self._h))

    def set_timeout(self, timeout_s: float) -> None:
        _check(lib().pb_comm_set_timeout(self._h, float(timeout_s)))

    def abort(self) -> None:
        _check(lib().pb_comm_abort(self._h))

    def close(self) -> None:
        if self._h.value:
            _check(lib().pb_comm_release(self._h))
            self._h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- configs --
# The five benchmark graphs named by the project's baseline (shapes only
# matter here; values come from fill_synthetic).
CONFIG_SHAPES = {
    "c1_elementwise": {"a": [1 << 24], "b": [1 << 24]},
    "c2_view": {"x": [8192, 8192], "bias": [4096], "y": [6144, 4096]},
    "c3a_softmax": {"x": [65536, 4096]},
    "c3b_relu_logistic": {"x": [65536, 4096]},
    "c4_matmul": {"a": [8192, 8192], "b": [8192, 8192], "bias": [8192]},
    "c5_mlp": {"x": [16384, 4096], "w1": [4096, 16384], "b1": [16384], "w2": [16384, 4096],
               "b2": [4096]},
}


def config_graph(name: str, t: dict) -> Expr:
    """Builds config `name`'s graph from tensors `t` (keyed as CONFIG_SHAPES)."""
    if name == "c1_elementwise":
        return (t["a"] + t["b"]) * 2.0 - 1.0
    if name == "c2_view":
        xs = t["x"][0::2, 1024:7168]
        return concat(transpose(xs) + broadcast_to(t["bias"], [6144, 4096]), t["y"], 0)
    if name == "c3a_softmax":
        return softmax(t["x"], 1)
    if name == "c3b_relu_logistic":
        return logistic(relu(t["x"]))
    if name == "c4_matmul":
        m = t["a"].shape()[0]
        n = t["b"].shape()[1]
        return relu(matmul(t["a"], t["b"]) + broadcast_to(t["bias"], [m, n]))
    if name == "c5_mlp":
        m = t["x"].shape()[0]
        h = logistic(matmul(t["x"], t["w1"]) + broadcast_to(t["b1"], [m, t["w1"].shape()[1]]))
        z = matmul(h, t["w2"]) + broadcast_to(t["b2"], [m, t["w2"].shape()[1]])
        return softmax(z, 1)
    raise KeyError(name)


def benchmark_graphs(placeholder: bool = True, device: int = 0) -> dict[str, Expr]:
    graphs = {}
    for name, shapes in CONFIG_SHAPES.items():
        ts = {k: (globals()["placeholder"](v, device)) for k, v in shapes.items()}
        graphs[name] = config_graph(name, ts)
    return graphs
