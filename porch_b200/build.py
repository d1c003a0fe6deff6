"""Build recipe for the porch_b200 native library.

Compiles every C++ source under porch_b200/csrc with g++ into
porch_b200/lib/libporch_b200.so. The library reaches CUDA only through
dlopen'ed libcuda / libnvrtc / libnccl, so it builds on a machine without a
GPU; the CUDA toolkit headers (cuda.h, nvrtc.h) and nccl.h are needed for
their type declarations only.

Kernels are hand-written templates that the library instantiates per graph
and compiles with NVRTC for sm_100a at run time. `check_kernels()` proves the
templates compile on a build machine: it lowers the benchmark graph shapes on
shape-only placeholder tensors (which runs NVRTC to sm_100a cubin) and also
compiles the same generated sources with nvcc -gencode
arch=compute_100a,code=sm_100a.

Usage: python -m porch_b200.build [--force] [--check]
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIB_DIR = PACKAGE / "lib"
OBJ_DIR = ROOT / "_build" / "obj"
LIBRARY = LIB_DIR / "libporch_b200.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
# The system g++ links the C++ runtime dynamically; a toolchain wrapper that
# embeds a private static copy would give this library its own exported
# libstdc++ and clash with other C++ code in the process.
CXX = os.environ.get("PORCH_B200_CXX", "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
CXXFLAGS = [
    "-std=c++20",
    "-O2",
    "-g1",
    "-fPIC",
    "-Wall",
    "-Wextra",
    "-Wno-unused-parameter",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC / 'front'}",
    f"-I{CUDA_HOME / 'include'}",
    "-I/usr/include",
]


NVCC = os.environ.get("NVCC", str(CUDA_HOME / "bin" / "nvcc"))
NVCCFLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
             "--fmad=false", "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}"]


def sources() -> list[Path]:
    return sorted(p for p in CSRC.rglob("*.cpp")) + sorted(p for p in CSRC.rglob("*.cu"))


def headers() -> list[Path]:
    hs = list(CSRC.rglob("*.hpp")) + list((ROOT / "include").rglob("*.h*"))
    return hs


def _compile(src: Path) -> Path:
    rel = src.relative_to(CSRC)
    obj = OBJ_DIR / rel.with_suffix(".o")
    obj.parent.mkdir(parents=True, exist_ok=True)
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCCFLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [CXX, *CXXFLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stderr}")
    return obj


def build(force: bool = False) -> Path:
    srcs = sources()
    newest = max(p.stat().st_mtime for p in srcs + headers() + [Path(__file__)])
    if LIBRARY.exists() and not force and LIBRARY.stat().st_mtime >= newest:
        return LIBRARY
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(_compile, srcs))
    tmp = LIBRARY.with_suffix(".so.tmp")
    # The CUDA runtime is linked statically for the one nvcc-compiled entry
    # point (pb_matmul_3xtf32_noalloc); everything else reaches the driver
    # through dlopen.
    cmd = [CXX, "-shared", "-o", str(tmp), *map(str, objs), f"-L{CUDA_HOME / 'lib64'}",
           "-lcudart_static", "-lrt", "-ldl", "-lpthread", "-Wl,--no-undefined"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


def check_kernels(out_dir: Path | None = None) -> list[str]:
    """Lower the benchmark graph shapes on placeholders (NVRTC -> sm_100a
    cubin inside the library), dump the generated sources and compile each
    with nvcc for sm_100a. Returns the kernel names checked."""
    from . import api  # noqa: WPS433 (import after the library is built)

    out_dir = out_dir or (ROOT / "_build" / "kernels")
    out_dir.mkdir(parents=True, exist_ok=True)
    names: list[str] = []
    sources_out: list[Path] = []
    for name, expr in api.benchmark_graphs(placeholder=True).items():
        text = api.describe(expr, with_source=True)
        chunks = text.split("extern \"C\" __global__")
        kernels = _split_kernels(text)
        for kname, src in kernels:
            path = out_dir / f"{name}_{kname}.cu"
            path.write_text(src)
            sources_out.append(path)
            names.append(kname)
        del chunks
    nvcc = shutil.which("nvcc") or str(CUDA_HOME / "bin" / "nvcc")
    if Path(nvcc).exists():
        def one(path: Path) -> None:
            cmd = [nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
                   "-O3", "--fmad=false", "-std=c++17", "-o", str(path.with_suffix(".cubin")),
                   str(path)]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed for {path}:\n{res.stderr}")
        with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
            list(ex.map(one, sources_out))
    return names


def _split_kernels(plan_text: str) -> list[tuple[str, str]]:
    """Pull each kernel's full source out of a plan description."""
    out: list[tuple[str, str]] = []
    lines = plan_text.splitlines(keepends=True)
    i = 0
    while i < len(lines):
        line = lines[i]
        if line.startswith("kernel "):
            kname = line.split()[1]
            i += 1
            buf = []
            while i < len(lines) and not lines[i].startswith("kernel "):
                buf.append(lines[i])
                i += 1
            out.append((kname, "".join(buf)))
        else:
            i += 1
    return out


if __name__ == "__main__":
    force = "--force" in sys.argv
    lib = build(force=force)
    print(lib)
    if "--check" in sys.argv:
        print("\n".join(check_kernels()))
