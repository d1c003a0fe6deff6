"""Seeded random cases aimed at the specialised schedules: column-tile
reductions over axis 0, a CTA per row for few long rows, long-row softmax
(two-pass streaming and thread-block clusters), and the tcgen05 GEMM with N
or K off a multiple of 4 and a fused epilogue. Each case draws a shape, an
operation and a prologue (none, exp, relu, a broadcast bias, a strided
slice, a scalar multiply) from its seed.

CPU: every case plans the schedule it is meant to reach. GPU: parity with
the host oracle (max bit for bit; sums within the reduction tolerance;
softmax 1e-5 relative; matmul against fp64 within 1e-5 normalised by
sqrt(K)).
"""

import random

import numpy as np
import pytest

import graphs
from tolerances import assert_relative

MAX_ELEMENTS = 1 << 25


def _case(seed):
    rng = random.Random(seed)
    kind = rng.choice(["colred", "rowred", "softmax", "gemm"])
    if kind == "colred":
        shape = [rng.choice([1, 7, 64, 65, 999, 4096, 20000, 131071]),
                 rng.choice([64, 68, 128, 130, 256, 260, 516, 1000, 1024, 2052])]
        return kind, shape, rng.choice(["sum", "max"]), rng.randint(0, 1), \
            rng.choice([None, "exp", "relu", "bias", "slice"])
    if kind == "rowred":
        shape = [rng.choice([1, 3, 100, 1000, 4000]), rng.choice([2048, 2049, 4100, 8192, 9000, 16384, 50001])]
        return kind, shape, rng.choice(["sum", "max"]), rng.randint(0, 1), \
            rng.choice([None, "exp", "relu", "bias", "slice"])
    if kind == "softmax":
        shape = [rng.choice([1, 2, 7, 40, 150, 600]),
                 rng.choice([16385, 16388, 20000, 32768, 50001, 65536, 100000, 131072, 131073, 200000])]
        return kind, shape, "softmax", 0, rng.choice([None, "bias", "slice", "scale"])
    m, n, k = rng.randint(100, 3000), rng.randint(100, 3000), rng.randint(16, 3000)
    while m * n * k < (1 << 27):
        k *= 2
    return kind, [m, n, k], "matmul", 0, rng.choice([None, "bias", "relu_bias", "add"])


def _program(kind, shape, op, keep, pro):
    if kind == "gemm":
        m, n, k = shape
        ins = [[m, k], [k, n]]
        lines = ["0 input 0", "1 input 1", "2 matmul 0 1"]
        if pro in ("bias", "relu_bias"):
            ins.append([n])
            lines += ["3 input 2", f"4 broadcast 3 {m},{n}", "5 add 2 4"]
            if pro == "relu_bias":
                lines.append("6 relu 5")
        elif pro == "add":
            ins.append([m, n])
            lines += ["3 input 2", "4 add 2 3"]
        return "\n".join(lines) + "\n", ins
    rows, cols = shape
    if pro == "slice":
        ins = [[rows + 3, cols + 5]]
        lines = ["0 input 0", "1 tensor 0", f"2 index 1 s1:{rows + 1}:1;s3:{cols + 3}:1"]
    elif pro == "bias":
        ins = [[rows, cols], [cols]]
        lines = ["0 input 0", "1 input 1", f"2 broadcast 1 {rows},{cols}", "3 add 0 2"]
    elif pro in ("exp", "relu"):
        ins = [[rows, cols]]
        lines = ["0 input 0", f"1 {pro} 0"]
    elif pro == "scale":
        ins = [[rows, cols]]
        lines = ["0 input 0", "1 scalar 40000000", "2 multiply 0 1"]
    else:
        ins = [[rows, cols]]
        lines = ["0 input 0"]
    src = len(lines) - 1
    if kind == "softmax":
        lines.append(f"{len(lines)} softmax {src} 1")
    else:
        lines.append(f"{len(lines)} {op} {src} {0 if kind == 'colred' else 1} {keep}")
    return "\n".join(lines) + "\n", ins


def _size(kind, shape):
    if kind == "gemm":
        m, n, k = shape
        return max(m * k, k * n, m * n)
    return shape[0] * shape[1]


def _seeds(per_kind=7):
    picked = {"colred": [], "rowred": [], "softmax": [], "gemm": []}
    for s in range(90000, 91000):
        kind, shape = _case(s)[:2]
        if _size(kind, shape) <= MAX_ELEMENTS and len(picked[kind]) < per_kind:
            picked[kind].append(s)
    return sorted(s for v in picked.values() for s in v)


SEEDS = _seeds()
EXPECT = {"colred": "column reduction (128-column tiles", "rowred": "per row",
          "softmax": "softmax row kernel", "gemm": "tcgen05"}


@pytest.mark.parametrize("seed", SEEDS)
def test_case_plans_its_schedule(api, seed):
    kind, shape, op, keep, pro = _case(seed)
    text, shapes = _program(kind, shape, op, keep, pro)
    orig = api.tensor
    try:
        api.tensor = lambda s, values, device=0: api.placeholder(list(s))
        e = graphs.build(api, text, [np.zeros(s, np.float32) for s in shapes])
    finally:
        api.tensor = orig
    plan = api.describe(e)
    want = EXPECT[kind]
    if kind == "colred" and pro == "slice":
        # A slice whose rows are not 16-byte aligned reads one float at a
        # time: thread per output instead of column tiles.
        want = "reduction"
    assert want in plan, (seed, kind, shape, pro, plan)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", SEEDS)
def test_case_matches_oracle(gpu, seed):
    kind, shape, op, keep, pro = _case(seed)
    text, shapes = _program(kind, shape, op, keep, pro)
    rng = np.random.default_rng(seed)
    ins = [rng.normal(0, 1, s).astype(np.float32) for s in shapes]
    got = graphs.evaluate_product(gpu, text, ins)
    what = f"seed {seed}: {kind} {shape} {op} {pro}"
    if kind == "gemm":
        z = ins[0].astype(np.float64) @ ins[1].astype(np.float64)
        if pro in ("bias", "relu_bias", "add"):
            z = z + ins[2].astype(np.float64)
        if pro == "relu_bias":
            z = np.maximum(z, 0.0)
        rms = np.sqrt(np.mean(z ** 2))
        err = np.max(np.abs(got - z) / (np.maximum(np.abs(z), rms) * np.sqrt(shape[2])))
        assert err <= 1e-5, (what, err)
        return
    want = graphs.evaluate_oracle(text, ins)
    assert got.shape == want.shape, what
    if op == "max" and pro != "exp":
        assert np.array_equal(got, want), what
    elif op == "sum":
        n = shape[0] if kind == "colred" else shape[1]
        # Terms of magnitude ~1 (normal inputs; exp of them ~e): the error
        # bound scales with the sum of magnitudes, ~sqrt(n) per output here.
        scale = np.maximum(np.abs(want.astype(np.float64)), 3.0 * np.sqrt(n) + 1.0)
        rel = np.max(np.abs(got.astype(np.float64) - want) / scale)
        assert rel <= 4e-5, (what, rel)
    else:
        assert_relative(got, want, 1e-5, what)
