"""Build recipe for the checkers (TEST INFRASTRUCTURE ONLY).

  oracle/_build/liboracle.so   host scalar oracle (oracle/oracle.cpp),
                               -ffp-contract=off so no operation fuses
  oracle/_build/pb_runner      oracle/ref_runner.cpp against this repository's
                               drop-in headers and libporch_b200.so
  oracle/_ref/libporch_ref.a   the reference library, compiled directly from its
                               four sources under <reference>/src (no CMake)
  oracle/_ref/ref_runner       oracle/ref_runner.cpp against the reference
  oracle/_ref/ref_conformance  the reference's own tests/tensor_test.cpp against
                               the reference library
  oracle/_ref/pb_conformance   the same unmodified test file against
                               libporch_b200.so (the drop-in check)

The reference checkout (PORCH_REFERENCE, by default the `reference`
directory beside this repository) is read where it lies and never copied
into the repository; the _ref outputs are git-ignored and travel with the
repository to GPU machines, which have no checkout and use them prebuilt.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
ROOT = ORACLE.parent
BUILD = ORACLE / "_build"
REF_OUT = ORACLE / "_ref"
REFERENCE = Path(os.environ.get("PORCH_REFERENCE", str(ROOT.parent / "reference")))
# The system g++ links the C++ runtime dynamically; a toolchain wrapper that
# embeds a private static copy would give this library its own exported
# libstdc++ and clash with other C++ code in the process.
CXX = os.environ.get("PORCH_B200_CXX", "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
SYNTH = ROOT / "porch_b200" / "csrc" / "synth.cpp"
PB_LIB_DIR = ROOT / "porch_b200" / "lib"


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build_oracle() -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    out = BUILD / "liboracle.so"
    src = ORACLE / "oracle.cpp"
    if _stale(out, [src, Path(__file__)]):
        _run([CXX, "-std=c++20", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-Wall",
              "-Wextra", str(src), "-o", str(out), "-lpthread"])
    return out


def build_pb_runner() -> Path | None:
    lib = PB_LIB_DIR / "libporch_b200.so"
    if not lib.exists():
        return None
    out = BUILD / "pb_runner"
    src = ORACLE / "ref_runner.cpp"
    if _stale(out, [src, lib, SYNTH, Path(__file__)]):
        _run([CXX, "-std=c++20", "-O2", f"-I{ROOT / 'include'}", str(src), str(SYNTH),
              f"-L{PB_LIB_DIR}", "-lporch_b200", f"-Wl,-rpath,{PB_LIB_DIR}", "-lpthread",
              "-o", str(out)])
    return out


def build_reference() -> bool:
    """Compile the reference from its own sources; False when absent."""
    srcs = [REFERENCE / "src" / f for f in ("backend.cpp", "cuda_jit.cpp", "ops.cpp", "tensor.cpp")]
    if not all(s.exists() for s in srcs):
        return (REF_OUT / "ref_runner").exists()
    REF_OUT.mkdir(parents=True, exist_ok=True)
    inc = f"-I{REFERENCE / 'include'}"
    objs = []
    for s in srcs:
        o = REF_OUT / (s.stem + ".o")
        if _stale(o, [s, Path(__file__)]):
            # The reference's CMake build uses C++20 with no optimisation flag
            # unless a build type is given; -O2 is the fair (faster) choice.
            _run([CXX, "-std=c++20", "-O2", "-fPIC", inc, "-c", str(s), "-o", str(o)])
        objs.append(str(o))
    lib = REF_OUT / "libporch_ref.a"
    if _stale(lib, [Path(o) for o in objs]):
        if lib.exists():
            lib.unlink()
        _run(["ar", "rcs", str(lib), *objs])
    runner = REF_OUT / "ref_runner"
    if _stale(runner, [lib, ORACLE / "ref_runner.cpp", SYNTH]):
        _run([CXX, "-std=c++20", "-O2", inc, str(ORACLE / "ref_runner.cpp"), str(SYNTH), str(lib),
              "-ldl", "-lpthread", "-o", str(runner)])
    test_src = REFERENCE / "tests" / "tensor_test.cpp"
    if test_src.exists():
        conf = REF_OUT / "ref_conformance"
        if _stale(conf, [lib, test_src]):
            _run([CXX, "-std=c++20", "-O0", "-g", inc, str(test_src), str(lib), "-ldl", "-lpthread",
                  "-o", str(conf)])
        pb_lib = PB_LIB_DIR / "libporch_b200.so"
        if pb_lib.exists():
            pconf = REF_OUT / "pb_conformance"
            if _stale(pconf, [pb_lib, test_src]):
                _run([CXX, "-std=c++20", "-O0", "-g", f"-I{ROOT / 'include'}", str(test_src),
                      f"-L{PB_LIB_DIR}", "-lporch_b200", f"-Wl,-rpath,{PB_LIB_DIR}", "-lpthread",
                      "-o", str(pconf)])
    return True


def build_all() -> None:
    build_oracle()
    build_pb_runner()
    build_reference()


if __name__ == "__main__":
    build_all()
    print("ok", file=sys.stderr)
