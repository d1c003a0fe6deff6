"""ctypes loader for libporch_b200.so (fails loudly when it is missing)."""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "lib" / "libporch_b200.so"


class pb_index(ctypes.Structure):
    _fields_ = [("kind", c_int), ("index", c_int64), ("start", c_int64),
                ("stop", c_int64), ("step", c_int64)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise ImportError(
                f"{LIBRARY} is not built; run `python -m porch_b200.build` "
                "(porch_b200 has no fallback implementation)")
        # The C++ runtime must be in the global symbol scope (as it is in any
        # C++ executable). In a Python process a C++ extension loaded earlier
        # (numpy's) can leave it outside, and iostream number formatting and
        # parsing in later-loaded C++ libraries then misbehave.
        ctypes.CDLL("libstdc++.so.6", mode=ctypes.RTLD_GLOBAL)
        L = ctypes.CDLL(str(LIBRARY), mode=ctypes.RTLD_GLOBAL)
        _declare(L)
        _lib = L
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    T = c_void_p  # opaque handles
    P = POINTER
    sig = {
        "pb_last_error": (c_char_p, []),
        "pb_is_available": (c_int, []),
        "pb_backend_name": (c_char_p, []),
        "pb_synchronize": (c_int, []),
        "pb_tensor_create": (c_int, [P(c_int64), c_size_t, P(c_float), c_size_t, c_int, P(T)]),
        "pb_tensor_create_async": (c_int, [P(c_int64), c_size_t, P(c_float), c_size_t, c_int, P(T)]),
        "pb_tensor_full": (c_int, [P(c_int64), c_size_t, c_float, c_int, P(T)]),
        "pb_tensor_placeholder": (c_int, [P(c_int64), c_size_t, c_int, P(T)]),
        "pb_tensor_release": (None, [T]),
        "pb_tensor_rank": (c_int, [T, P(c_size_t)]),
        "pb_tensor_shape": (c_int, [T, P(c_int64), c_size_t]),
        "pb_tensor_strides": (c_int, [T, P(c_int64), c_size_t]),
        "pb_tensor_numel": (c_int, [T, P(c_size_t)]),
        "pb_tensor_storage_offset": (c_int, [T, P(c_int64)]),
        "pb_tensor_is_contiguous": (c_int, [T, P(c_int)]),
        "pb_tensor_device": (c_int, [T, P(c_int)]),
        "pb_tensor_realize": (c_int, [T]),
        "pb_tensor_synchronize": (c_int, [T]),
        "pb_tensor_read": (c_int, [T, c_void_p, c_size_t]),
        "pb_tensor_device_pointer": (c_int, [T, P(c_uint64), P(c_size_t)]),
        "pb_tensor_index": (c_int, [T, P(pb_index), c_size_t, P(T)]),
        "pb_expr_from_tensor": (c_int, [T, P(T)]),
        "pb_expr_scalar": (c_int, [c_float, P(T)]),
        "pb_expr_release": (None, [T]),
        "pb_expr_binary": (c_int, [c_int, T, T, P(T)]),
        "pb_expr_unary": (c_int, [c_int, T, P(T)]),
        "pb_expr_reshape": (c_int, [T, P(c_int64), c_size_t, P(T)]),
        "pb_expr_broadcast": (c_int, [T, P(c_int64), c_size_t, P(T)]),
        "pb_expr_unsqueeze": (c_int, [T, c_size_t, P(T)]),
        "pb_expr_permute": (c_int, [T, P(c_int64), c_size_t, P(T)]),
        "pb_test_gemm_stall": (c_int, [c_int]),
        "pb_expr_batched_matmul": (c_int, [T, T, P(T)]),
        "pb_expr_concat": (c_int, [T, T, c_size_t, P(T)]),
        "pb_expr_reduce": (c_int, [c_int, T, c_size_t, c_int, P(T)]),
        "pb_expr_softmax": (c_int, [T, c_size_t, P(T)]),
        "pb_expr_shape": (c_int, [T, P(c_int64), c_size_t, P(c_size_t)]),
        "pb_expr_to_tensor": (c_int, [T, P(T)]),
        "pb_materialize": (c_int, [T, P(T)]),
        "pb_expr_describe": (c_int, [T, c_int, c_char_p, c_size_t, P(c_size_t)]),
        "pb_host_alloc": (c_int, [c_size_t, P(c_void_p)]),
        "pb_host_free": (c_int, [c_void_p]),
        "pb_timer_begin": (c_int, [c_int, P(c_void_p)]),
        "pb_timer_end": (c_int, [c_void_p, P(c_float)]),
        "pb_device_synchronize": (c_int, [c_int]),
        "pb_launch_count": (c_uint64, []),
        "pb_empty_cache": (c_int, [c_int, P(c_size_t)]),
        "pb_profile_enable": (c_int, [c_int]),
        "pb_profile_read": (c_int, [c_char_p, c_size_t]),
        "pb_host_profile_enable": (c_int, [c_int]),
        "pb_host_profile_read": (c_int, [c_char_p, c_size_t]),
        "pb_fill_synthetic": (c_int, [c_void_p, c_size_t, c_uint64, c_int, c_double, c_double]),
        "pb_matmul_3xtf32_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                             c_void_p]),
        "pb_comm_unique_id": (c_int, [c_char_p]),
        "pb_comm_init": (c_int, [c_int, c_char_p, c_int, c_int, c_double, P(c_void_p)]),
        "pb_comm_info": (c_int, [c_void_p, P(c_int), P(c_int), P(c_int)]),
        "pb_comm_abort": (c_int, [c_void_p]),
        "pb_comm_set_timeout": (c_int, [c_void_p, c_double]),
        "pb_comm_release": (c_int, [c_void_p]),
        "pb_row_block": (c_int, [c_int64, c_int, c_int, P(c_int64), P(c_int64)]),
        "pb_allgather_rows": (c_int, [c_void_p, c_void_p, c_int64, P(c_void_p)]),
        "pb_allgather_rows_async": (c_int, [c_void_p, c_void_p, c_int64, P(c_void_p)]),
        "pb_comm_wait": (c_int, [c_void_p]),
        "pbrt_available": (c_int, []),
        "pbrt_device_count": (c_int, [P(c_int)]),
        "pbrt_last_error": (c_char_p, []),
        "pbrt_fault_inject": (c_int, [c_char_p]),
        "pbrt_launch_count": (c_uint64, []),
        "pbrt_compile_stats": (None, [P(c_uint64), P(c_uint64)]),
        "pbrt_stream_current": (c_int, [c_int, P(c_void_p)]),
        "pbrt_stream_synchronize": (c_int, [c_int, c_void_p]),
        "pbrt_mem_alloc_async": (c_int, [c_int, c_size_t, c_void_p, P(c_uint64)]),
        "pbrt_mem_free_async": (c_int, [c_int, c_uint64, c_void_p]),
        "pbrt_mem_alloc": (c_int, [c_int, c_size_t, P(c_uint64)]),
        "pbrt_launch_ex": (c_int, [c_int, c_void_p, P(ctypes.c_uint32), P(ctypes.c_uint32), ctypes.c_uint32, c_void_p,
                                   P(c_void_p), P(ctypes.c_uint32), ctypes.c_uint]),
        "pbrt_mem_free": (c_int, [c_int, c_uint64]),
        "pbrt_memcpy_h2d_async": (c_int, [c_int, c_uint64, c_void_p, c_size_t, c_void_p]),
        "pbrt_memcpy_d2h_async": (c_int, [c_int, c_void_p, c_uint64, c_size_t, c_void_p]),
        "pbrt_event_create": (c_int, [c_int, c_int, P(c_void_p)]),
        "pbrt_event_destroy": (c_int, [c_int, c_void_p]),
        "pbrt_event_record": (c_int, [c_int, c_void_p, c_void_p]),
        "pbrt_event_synchronize": (c_int, [c_int, c_void_p]),
        "pbrt_event_elapsed_ms": (c_int, [c_void_p, c_void_p, P(c_float)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
