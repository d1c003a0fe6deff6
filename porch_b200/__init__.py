"""porch_b200: a B200-native (sm_100a) lowering and execution backend for
porch's lazy tensor graphs.

The product is the native library porch_b200/lib/libporch_b200.so: the drop-in
porch C++ API (include/porch/*.hpp), its flat C-ABI (include/porch_b200.h)
and the runtime C-ABI over the CUDA driver, NVRTC and NCCL
(include/porch_b200_rt.h). `porch_b200.api` binds the flat C-ABI with ctypes
for tests, benchmarks and Python callers.
"""

from .build import LIBRARY  # noqa: F401
