"""The benchmark graphs at (or near) full size against the reference itself.

oracle/_ref/ref_runner is AkhilSamavedam/porch compiled from its sources
(oracle/build.py); `ref_runner eval` realises a program through the
reference's own public API and NVRTC-JIT path on the same GPU. Both sides
get the same seeded inputs (the bench's generator and distributions):
- configs 1, 2 and 3b: bit for bit (same IEEE operations in the same order;
  exp is the same __expf intrinsic, src/tensor.cpp:857);
- config 3a (softmax): within 1e-5 relative (the reductions associate in a
  different order);
- config 4: our 3xTF32 GEMM and the reference's fp32 FFMA chain
  (src/tensor.cpp:684-721) against fp64 on sampled rows: both within the
  1e-5 sqrt(K) bound, ours within 4x the reference's own error, and the two
  within that bound of each other;
- config 5 (staged, as the reference must run it): within tolerance.
"""

from __future__ import annotations

import struct
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest

import graphs
from tolerances import MATMUL_TOL, REL_TOL, assert_bitwise, assert_relative, matmul_error

ROOT = Path(__file__).resolve().parent.parent
RUNNER = ROOT / "oracle" / "_ref" / "ref_runner"
SEED = 20261201


def _inputs(api, specs):
    out = []
    for i, (shape, dist, a, b) in enumerate(specs):
        x = np.empty(int(np.prod(shape)), dtype=np.float32)
        api.fill_synthetic(x, SEED + i, dist, a, b)
        out.append(x.reshape(shape))
    return out


def _run_reference(program: str, inputs) -> np.ndarray:
    assert RUNNER.exists(), "oracle/_ref/ref_runner was not built (python -m oracle.build)"
    with tempfile.TemporaryDirectory() as td:
        tmp = Path(td)
        (tmp / "prog.txt").write_text(program)
        with open(tmp / "inputs.bin", "wb") as f:
            for arr in inputs:
                f.write(struct.pack("<q", arr.ndim))
                for d in arr.shape:
                    f.write(struct.pack("<q", d))
                f.write(np.ascontiguousarray(arr, dtype=np.float32).tobytes())
        res = subprocess.run([str(RUNNER), "eval", str(tmp / "prog.txt"), str(tmp / "inputs.bin"),
                              str(tmp / "out.bin")], capture_output=True, text=True, timeout=900)
        assert res.returncode == 0, res.stderr[-2000:]
        data = (tmp / "out.bin").read_bytes()
    rank = struct.unpack_from("<q", data, 0)[0]
    shape = list(struct.unpack_from(f"<{rank}q", data, 8))
    return np.frombuffer(data, dtype=np.float32, offset=8 + 8 * rank).reshape(shape).copy()


C1 = "0 input 0\n1 input 1\n2 add 0 1\n3 scalar 40000000\n4 multiply 2 3\n5 scalar 3f800000\n6 subtract 4 5\n"
C2 = ("0 input 0\n1 input 1\n2 input 2\n3 index 0 s0:8192:2;s1024:7168:1\n4 transpose 3\n"
      "5 broadcast 1 6144,4096\n6 add 4 5\n7 concat 6 2 0\n")
C3A = "0 input 0\n1 softmax 0 1\n"
C3B = "0 input 0\n1 relu 0\n2 logistic 1\n"


@pytest.mark.gpu
def test_c1_full_size_equals_reference(gpu):
    ins = _inputs(gpu, [([1 << 24], "uniform", -1, 1), ([1 << 24], "uniform", -1, 1)])
    assert_bitwise(graphs.evaluate_product(gpu, C1, ins), _run_reference(C1, ins), "config 1 vs reference")


@pytest.mark.gpu
def test_c2_full_size_equals_reference(gpu):
    ins = _inputs(gpu, [([8192, 8192], "normal", 0, 1), ([4096], "uniform", -0.5, 0.5),
                        ([6144, 4096], "normal", 0, 1)])
    assert_bitwise(graphs.evaluate_product(gpu, C2, ins), _run_reference(C2, ins), "config 2 vs reference")


@pytest.mark.gpu
def test_c3b_equals_reference(gpu):
    ins = _inputs(gpu, [([16384, 4096], "normal", 0, 2)])
    assert_bitwise(graphs.evaluate_product(gpu, C3B, ins), _run_reference(C3B, ins), "config 3b vs reference")


@pytest.mark.gpu
def test_c3a_softmax_matches_reference(gpu):
    ins = _inputs(gpu, [([16384, 4096], "normal", 0, 2)])
    assert_relative(graphs.evaluate_product(gpu, C3A, ins), _run_reference(C3A, ins), REL_TOL,
                    "config 3a vs reference")


@pytest.mark.gpu
def test_c4_matmul_against_reference_and_fp64(gpu):
    n = 8192
    s = 1 / 90.50966799187808
    ins = _inputs(gpu, [([n, n], "uniform", -s, s), ([n, n], "uniform", -s, s), ([n], "uniform", -0.1, 0.1)])
    # relu(A @ B + bias) with the bias and relu out of the way of the error
    # measurement: compare the product itself.
    prog = "0 input 0\n1 input 1\n2 matmul 0 1\n"
    ours = graphs.evaluate_product(gpu, prog, ins[:2])
    ref = _run_reference(prog, ins[:2])
    rows = np.arange(0, n, 131)
    want = ins[0][rows].astype(np.float64) @ ins[1].astype(np.float64)
    e_ours = matmul_error(ours[rows], want, n)
    e_ref = matmul_error(ref[rows], want, n)
    print(f"config 4 normalised error vs fp64: porch_b200 {e_ours:.3e}, reference {e_ref:.3e}")
    assert e_ours <= MATMUL_TOL and e_ref <= MATMUL_TOL, (e_ours, e_ref)
    assert e_ours <= 4 * e_ref, (e_ours, e_ref)
    assert matmul_error(ours[rows], ref[rows].astype(np.float64), n) <= MATMUL_TOL
    # The full fused graph of config 4 as well (bias + relu epilogue).
    full = ("0 input 0\n1 input 1\n2 input 2\n3 matmul 0 1\n4 broadcast 2 8192,8192\n5 add 3 4\n"
            "6 relu 5\n")
    ours_full = graphs.evaluate_product(gpu, full, ins)
    ref_full = _run_reference(full, ins)
    assert matmul_error(ours_full[rows], ref_full[rows].astype(np.float64), n) <= MATMUL_TOL


@pytest.mark.gpu
def test_c5_staged_matches_reference(gpu):
    m, d, h = 4096, 4096, 16384
    ins = _inputs(gpu, [([m, d], "normal", 0, 1), ([d, h], "normal", 0, 1 / 64), ([h], "uniform", -0.1, 0.1),
                        ([h, d], "normal", 0, 1 / 128), ([d], "uniform", -0.1, 0.1)])
    prog = (f"0 input 0\n1 input 1\n2 input 2\n3 input 3\n4 input 4\n5 matmul 0 1\n6 broadcast 2 {m},{h}\n"
            f"7 add 5 6\n8 logistic 7\n9 materialize 8\n10 matmul 9 3\n11 broadcast 4 {m},{d}\n"
            "12 add 10 11\n13 materialize 12\n14 softmax 13 1\n")
    ours = graphs.evaluate_product(gpu, prog, ins)
    ref = _run_reference(prog, ins)
    # P's rows sum to 1 with entries ~1/4096: compare each element against
    # the row scale (the matmuls' sqrt(K)-normalised error carries through).
    err = np.abs(ours.astype(np.float64) - ref.astype(np.float64)) / np.abs(ref).max(axis=1, keepdims=True)
    assert float(err.max()) <= 1e-4, float(err.max())


LARGE_SEEDS = list(range(7000, 7040))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", LARGE_SEEDS)
def test_large_random_programs_match_reference(gpu, seed):
    """Random programs over every node kind at extents up to thousands, with
    integer-valued inputs: every operation but exp/logistic/softmax is then
    exact in fp32 whatever the order (sums and matmul products of small
    integers included), so those programs must equal the reference's output
    bit for bit; programs with exp must still match within 1e-5 relative
    where no sum, softmax or matmul sits downstream of it, and within the
    reduction scale otherwise."""
    text, ins, _ = graphs.random_program(seed, integer_values=True, depth=4, large=True)
    ops = {line.split()[1] for line in text.strip().splitlines()}
    try:
        ref = _run_reference(text, ins)
    except AssertionError:
        # The reference rejects the program (or cannot realise a scalar):
        # ours must reject it as well.
        with pytest.raises((ValueError, IndexError, RuntimeError)):
            graphs.evaluate_product(gpu, text, ins)
        return
    got = graphs.evaluate_product(gpu, text, ins)
    assert list(got.shape) == list(ref.shape)
    if not ops & {"exp", "logistic", "softmax"}:
        assert_bitwise(got, ref, f"seed {seed}")
    elif not ops & {"sum", "softmax", "matmul"}:
        # The same __expf on both sides, in the same operation order.
        assert_bitwise(got, ref, f"seed {seed}")
    else:
        g64, r64 = got.astype(np.float64), ref.astype(np.float64)
        fin = np.isfinite(r64)
        assert np.array_equal(np.isfinite(g64), fin), f"seed {seed}"
        scale = np.maximum(np.abs(r64), np.sqrt(np.mean(r64[fin] ** 2)) if fin.any() else 1.0)
        err = np.abs(g64 - r64)[fin] / np.where(scale[fin] == 0, 1.0, scale[fin])
        assert err.size == 0 or float(err.max()) <= 1e-4, (f"seed {seed}", float(err.max()))
