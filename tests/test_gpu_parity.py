"""Parity of the CUDA path against the host oracle and the reference's own
test suite. Every test here runs kernels on the GPU through the C-ABI."""

import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import error_bounds
import graphs
from tolerances import REL_TOL, assert_bitwise, assert_relative, matmul_error

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())["cases"]


@pytest.mark.parametrize("case", GOLDEN, ids=[c["name"] for c in GOLDEN])
def test_known_answers(gpu, case):
    api = gpu
    ins = [np.asarray(v, dtype=np.float32).reshape(s) for s, v in case["inputs"]]
    if case["error"]:
        with pytest.raises(ValueError):
            graphs.evaluate_product(api, case["program"], ins)
        return
    got = graphs.evaluate_product(api, case["program"], ins)
    if case["shape"] is not None:
        assert list(got.shape) == case["shape"]
    if case["expect"] is not None:
        assert_bitwise(got, np.asarray(case["expect"], dtype=np.float32), case["name"])
    if case["interval"] is not None:
        flat = got.reshape(-1)
        for i, (lo, hi) in enumerate(case["interval"]):
            assert lo <= flat[i] <= hi, (case["name"], i, flat[i])
    for i, v in (case["exact_at"] or {}).items():
        assert got.reshape(-1)[int(i)] == np.float32(v)


CONFORMANCE = [
    "construction_tracks_shape_and_device", "tensor_is_small_handle",
    "construction_builds_contiguous_layout", "bracket_slice_selects_contiguous_copy",
    "bracket_slice_returns_lazy_expression", "bracket_slice_handles_multiple_dimensions",
    "zeros_fills_gpu_tensor", "add_uses_cuda_backend", "subtract_uses_cuda_backend",
    "multiply_uses_cuda_backend", "elementwise_arithmetic_matches_expected_values",
    "chained_arithmetic_matches_expected_values", "fused_expression_materializes_once",
    "multiline_expression_stays_lazy_with_auto", "tensor_assignment_keeps_graph_lazy",
    "explicit_gpu_sync_and_cpu_copy", "concurrent_same_lazy_tensor_materializes_once_safely",
    "concurrent_independent_lazy_tensors_use_thread_streams",
    "scalar_elementwise_ops_use_cuda_backend", "scalar_arithmetic_order_matches_expected_values",
    "matmul_uses_cuda_backend", "matmul_rectangular_values_are_correct",
    "matmul_returns_lazy_expression", "matmul_composes_with_elementwise_ir",
    "matmul_accepts_expression_operands", "matmul_rejects_invalid_shapes",
    "reshape_uses_lazy_device_ir", "transpose_uses_lazy_device_ir",
    "broadcast_to_uses_lazy_device_ir", "concat_uses_lazy_device_ir",
    "reductions_use_lazy_device_ir", "keepdim_reductions_use_lazy_device_ir",
    "block_reductions_handle_axis_larger_than_block",
    "nested_reductions_materialize_with_block_reduction",
    "softmax_style_expression_uses_nested_block_reduction", "relu_compound_op_uses_primitives",
    "softmax_compound_op_uses_primitives", "logistic_compound_op_uses_primitives",
    "exp_uses_lazy_device_ir", "divide_and_reciprocal_use_lazy_device_ir",
    "elementwise_minimum_maximum_use_lazy_device_ir",
    "unsqueeze_and_expression_shape_are_lazy_metadata", "rejects_invalid_shapes",
    "cuda_devices_select_cuda_jit_backend", "cuda_jit_availability_matches_backend_availability",
    "cuda_jit_compiles_or_reports_missing_nvrtc", "device_buffer_round_trips_values",
]


@pytest.mark.parametrize("name", CONFORMANCE)
def test_reference_test_suite_against_this_library(gpu, name):
    """The reference's unmodified tests/tensor_test.cpp linked against
    libporch_b200.so; each of its 47 cases must pass on the GPU (not skip)."""
    exe = ROOT / "oracle" / "_ref" / "pb_conformance"
    assert exe.exists(), "oracle/_ref/pb_conformance was not built"
    res = subprocess.run([str(exe), name], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "skipped" not in res.stdout, "the CUDA path did not run"


@pytest.mark.parametrize("seed", range(120))
def test_fuzz_against_oracle(gpu, oracle_lib, seed):
    text, ins, exact = graphs.random_program(seed, integer_values=seed % 2 == 0)
    want = graphs.evaluate_oracle(text, ins)
    got = graphs.evaluate_product(gpu, text, ins)
    assert list(got.shape) == list(want.shape)
    if exact:
        assert_bitwise(got, want, f"seed {seed}")
    else:
        # Inexact programs (exp, sum, softmax, matmul): every element within
        # 1e-5 relative of the oracle, or, where the result cancels and no
        # fp32 evaluation order can meet a relative bar, within the forward
        # error bound of fp32 evaluation (tests/error_bounds.py).
        _, bound = error_bounds.evaluate(text, ins)
        error_bounds.check(got, want, bound, REL_TOL, f"seed {seed}")


def _config_inputs(api, name, shapes, seed=20261201):
    specs = {
        "c1_elementwise": [("uniform", -1, 1)] * 2,
        "c2_view": [("normal", 0, 1), ("uniform", -0.5, 0.5), ("normal", 0, 1)],
        "c3a_softmax": [("normal", 0, 2)],
        "c3b_relu_logistic": [("normal", 0, 2)],
        "c4_matmul": [("uniform", -1 / 90.50966799187808, 1 / 90.50966799187808)] * 2 + [("uniform", -0.1, 0.1)],
        "c5_mlp": [("normal", 0, 1), ("normal", 0, 1 / 64), ("uniform", -0.1, 0.1),
                   ("normal", 0, 1 / 128), ("uniform", -0.1, 0.1)],
    }[name]
    arrays = []
    for i, ((dist, a, b), shape) in enumerate(zip(specs, shapes)):
        x = np.empty(int(np.prod(shape)), dtype=np.float32)
        api.fill_synthetic(x, seed + i, dist, a, b)
        arrays.append(x.reshape(shape))
    return arrays


def test_c1_full_size_bitwise(gpu):
    api = gpu
    a, b = _config_inputs(api, "c1_elementwise", [[1 << 24], [1 << 24]])
    out = api.materialize((api.tensor([1 << 24], a) + api.tensor([1 << 24], b)) * 2.0 - 1.0).cpu()
    want = (a + b) * np.float32(2.0) - np.float32(1.0)
    assert_bitwise(out, want, "c1")


def test_c2_full_size_bitwise(gpu):
    api = gpu
    x, bias, y = _config_inputs(api, "c2_view", [[8192, 8192], [4096], [6144, 4096]])
    X, B, Y = api.tensor([8192, 8192], x), api.tensor([4096], bias), api.tensor([6144, 4096], y)
    out = api.materialize(api.concat(api.transpose(X[0::2, 1024:7168]) + api.broadcast_to(B, [6144, 4096]),
                                     Y, 0)).cpu()
    want = np.concatenate([np.ascontiguousarray(x[0::2, 1024:7168].T) + bias[None, :], y], axis=0)
    assert_bitwise(out, want, "c2")


@pytest.mark.parametrize("rows,cols", [(65536, 4096), (257, 4096), (33, 1000), (5, 16385), (3, 7)])
def test_softmax_rows_against_oracle(gpu, oracle_lib, rows, cols):
    api = gpu
    (x,) = _config_inputs(api, "c3a_softmax", [[rows, cols]])
    got = api.materialize(api.softmax(api.tensor([rows, cols], x), 1)).cpu()
    # Row sums are 1; sampled rows match the oracle within 1e-5 relative.
    assert np.allclose(got.sum(axis=1, dtype=np.float64), 1.0, atol=1e-5)
    sample = sorted(set(np.linspace(0, rows - 1, num=min(rows, 256)).astype(int).tolist()))
    want = graphs.evaluate_oracle("0 input 0\n1 softmax 0 1\n", [x[sample]])
    assert_relative(got[sample], want, what=f"softmax {rows}x{cols}")


def test_relu_logistic_full_size(gpu, oracle_lib):
    api = gpu
    (x,) = _config_inputs(api, "c3b_relu_logistic", [[65536, 4096]])
    got = api.materialize(api.logistic(api.relu(api.tensor([65536, 4096], x)))).cpu()
    sample = x[::997]
    want = graphs.evaluate_oracle("0 input 0\n1 relu 0\n2 logistic 1\n", [sample])
    assert_relative(got[::997], want, what="relu->logistic")


@pytest.mark.parametrize("m,k,n", [(2, 3, 2), (64, 64, 64), (100, 37, 129), (512, 1024, 384)])
def test_matmul_epilogue_against_fp64(gpu, m, k, n):
    api = gpu
    rng = np.random.default_rng(m * 1000 + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    A, B, Bi = api.tensor([m, k], a), api.tensor([k, n], b), api.tensor([n], bias)
    got = api.materialize(api.relu(api.matmul(A, B) + api.broadcast_to(Bi, [m, n]))).cpu()
    ref = np.maximum(a.astype(np.float64) @ b.astype(np.float64) + bias, 0.0)
    assert matmul_error(got, ref, k) <= 1e-5


TC_SHAPES = [(512, 512, 512), (256, 1024, 768), (1024, 768, 512), (384, 512, 1024),
             # few tiles: split-K into 8, 8 and 16 K-ranges
             (128, 4096, 1024), (256, 2048, 512), (128, 8192, 1024),
             # edge tiles: M, N, K not multiples of the tile (zero fill past
             # the edges, masked stores), with and without split-K
             (1000, 520, 1004), (300, 4096, 772), (129, 4100, 260),
             # K past a multiple of 32: hi/lo rows padded with zeros to
             # 128-byte lines, the last accumulation period of a tile short
             (128, 4100, 4096), (2048, 2052, 2048),
             # N or K not multiples of 4: scalar A loads, column-checked
             # epilogue loads and stores, split-K partials on a padded pitch
             (1000, 999, 1001), (513, 4097, 515), (129, 1030, 2050), (300, 771, 4096),
             (2049, 515, 1027)]


@pytest.mark.parametrize("m,k,n", TC_SHAPES)
def test_tcgen05_3xtf32_matmul(gpu, m, k, n):
    """Shapes eligible for the tcgen05 path (M*N*K >= 2^27): the plan must
    use it, and the result must hold fp32 accuracy: within the
    normalised 1e-5 bound, and within 4x the error of the reference's
    sequential fp32 accumulation (a plain one-pass TF32 product is about
    1000x worse than fp32 and fails this)."""
    api = gpu
    rng = np.random.default_rng(m + 3 * k + 7 * n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    A, B, Bi = api.tensor([m, k], a), api.tensor([k, n], b), api.tensor([n], bias)
    expr = api.relu(api.matmul(A, B) + api.broadcast_to(Bi, [m, n]))
    assert "tcgen05" in api.describe(expr)
    got = api.materialize(expr).cpu()
    ref = np.maximum(a.astype(np.float64) @ b.astype(np.float64) + bias, 0.0)
    err = matmul_error(got, ref, k)
    assert err <= 1e-5, err
    # The reference's own arithmetic: a sequential fp32 chain over k (its
    # generated loop `sum += L * R`, src/tensor.cpp:684-721).
    chain = np.zeros((m, n), dtype=np.float32)
    for kk in range(k):
        chain = (chain + np.outer(a[:, kk], b[kk, :]).astype(np.float32)).astype(np.float32)
    chain = np.maximum(chain + bias, np.float32(0.0))
    chain_err = matmul_error(chain, ref, k)
    assert err <= 4 * chain_err, (err, chain_err)


def test_matmul_c4_full_size_sampled_rows(gpu):
    api = gpu
    a, b, bias = _config_inputs(api, "c4_matmul", [[8192, 8192], [8192, 8192], [8192]])
    A, B, Bi = api.tensor([8192, 8192], a), api.tensor([8192, 8192], b), api.tensor([8192], bias)
    got = api.materialize(api.relu(api.matmul(A, B) + api.broadcast_to(Bi, [8192, 8192]))).cpu()
    rows = np.linspace(0, 8191, 64).astype(int)
    ref = np.maximum(a[rows].astype(np.float64) @ b.astype(np.float64) + bias, 0.0)
    assert matmul_error(got[rows], ref, 8192) <= 1e-5
