"""Realises one benchmark graph a few times, for a profiler to capture.

    python -m porch_b200.profile_case c3a_softmax --rows 16384 --steps 3

Builds the named configuration's graph (porch_b200.api.config_graph), or
one of the other kernel families' graphs below, on seeded synthetic inputs whose leading dimension is cut to --rows (0 keeps
the benchmark's full shape), realises it --steps times on --device and
synchronises. Nothing is timed here: under ncu the per-launch figures come
from the profiler; without it the run only checks that the case exits 0.
"""

from __future__ import annotations

import argparse

import numpy as np

from porch_b200 import api

DISTRIBUTIONS = {
    "c1_elementwise": [("uniform", -1, 1), ("uniform", -1, 1)],
    "c2_view": [("normal", 0, 1), ("uniform", -0.5, 0.5), ("normal", 0, 1)],
    "c3a_softmax": [("normal", 0, 2)],
    "c3b_relu_logistic": [("normal", 0, 2)],
    "c4_matmul": [("uniform", -1 / 90.50966799187808, 1 / 90.50966799187808)] * 2 + [("uniform", -0.1, 0.1)],
    "c5_mlp": [("normal", 0, 1), ("normal", 0, 1 / 64), ("uniform", -0.1, 0.1), ("normal", 0, 1 / 128),
               ("uniform", -0.1, 0.1)],
}
# Inputs whose leading dimension is the graph's row axis (cut by --rows).
ROW_INPUTS = {"c3a_softmax": {"x"}, "c3b_relu_logistic": {"x"}, "c4_matmul": {"a"}, "c5_mlp": {"x"}}
# Row graphs outside the benchmark configs: (shape, axis) of sum(x, axis),
# and long-row softmax shapes (streaming two-pass; a cluster per row).
REDUCTIONS = {"sum_axis0": ([262144, 256], 0), "sum_axis1": ([4096, 16384], 1)}
SOFTMAX = {"softmax_long": [4096, 32768], "softmax_cluster": [64, 65536]}
# Other kernel families: (input shapes, graph builder).
#  gather:       a reshape of a transpose, inside a sum, whose index map is
#                not affine (pb_gather_*), 268 MB in, 134 MB out;
#  reduce_part:  a sum over the middle axis of [8192, 2048, 3] (rows of 3:
#                no column tiles; pb_reduce_part_* + pb_reduce_comb_*);
#  splitk:       [128, 4096] @ [4096, 4096] (16 tiles: split-K x8,
#                pb_splitk_*);
#  gemm_simt:    [512, 512] @ [512, 256] (below the tensor-core threshold,
#                the CUDA-core GEMM);
#  split:        [2048, 8192] @ [8192, 8192] (the 3xTF32 split passes
#                pb_split_rows / pb_split_transpose; the GEMM itself too).
GRAPHS = {
    "gather": ([[8192, 4095], [4095 * 8192]],
               lambda t: api.reshape(api.transpose(t[0]), [4095 * 8192]) + t[1]),
    "reduce_part": ([[8192, 2048, 3]], lambda t: api.sum(t[0], 1)),
    "splitk": ([[128, 4096], [4096, 4096]], lambda t: api.matmul(t[0], t[1])),
    "gemm_simt": ([[512, 512], [512, 256]], lambda t: api.matmul(t[0], t[1])),
    "split": ([[2048, 8192], [8192, 8192]], lambda t: api.matmul(t[0], t[1])),
    # Config 5's first GEMM at 4096 rows writing H in fp32, and the same GEMM
    # writing H as the second GEMM's 3xTF32 halves (split output).
    "gemm1_plain": ([[4096, 4096], [4096, 16384], [16384]],
                    lambda t: api.logistic(api.matmul(t[0], t[1]) + api.broadcast_to(t[2], [4096, 16384]))),
    "gemm1_split": ([[4096, 4096], [4096, 16384], [16384], [16384, 4096]],
                    lambda t: api.matmul(api.logistic(api.matmul(t[0], t[1]) + api.broadcast_to(t[2], [4096, 16384])),
                                         t[3])),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("workload", choices=sorted(api.CONFIG_SHAPES) + sorted(REDUCTIONS) + sorted(SOFTMAX)
                    + sorted(GRAPHS))
    ap.add_argument("--rows", type=int, default=0)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args()
    if args.workload in GRAPHS:
        shapes, build = GRAPHS[args.workload]
        ts = []
        for i, shape in enumerate(shapes):
            arr = np.empty(int(np.prod(shape)), dtype=np.float32)
            api.fill_synthetic(arr, 20261201 + i, "uniform", -1, 1)
            t = api.tensor(shape, arr, device=args.device)
            t.device_data()  # handed out: every realisation splits its GEMM operands again
            ts.append(t)
        outs = [api.materialize(build(ts)) for _ in range(max(1, args.steps))]
        api.device_synchronize(args.device)
        print(f"{args.workload}: {len(outs)} realisations of shape {outs[-1].shape()}")
        return
    if args.workload in SOFTMAX:
        shape = list(SOFTMAX[args.workload])
        if args.rows:
            shape[0] = args.rows
        arr = np.empty(int(np.prod(shape)), dtype=np.float32)
        api.fill_synthetic(arr, 20261201, "normal", 0, 2)
        x = api.tensor(shape, arr, device=args.device)
        outs = [api.materialize(api.softmax(x, 1)) for _ in range(max(1, args.steps))]
        api.device_synchronize(args.device)
        print(f"{args.workload}: {len(outs)} realisations of shape {outs[-1].shape()}")
        return
    if args.workload in REDUCTIONS:
        shape, axis = REDUCTIONS[args.workload]
        shape = list(shape)
        if args.rows:
            shape[0] = args.rows
        arr = np.empty(int(np.prod(shape)), dtype=np.float32)
        api.fill_synthetic(arr, 20261201, "normal", 0, 1)
        x = api.tensor(shape, arr, device=args.device)
        outs = [api.materialize(api.sum(x, axis)) for _ in range(max(1, args.steps))]
        api.device_synchronize(args.device)
        print(f"{args.workload}: {len(outs)} realisations of shape {outs[-1].shape()}")
        return
    shapes = api.CONFIG_SHAPES[args.workload]
    tensors = {}
    for i, ((key, shape), (dist, a, b)) in enumerate(zip(shapes.items(), DISTRIBUTIONS[args.workload])):
        shape = list(shape)
        if args.rows and key in ROW_INPUTS.get(args.workload, ()):
            shape[0] = args.rows
        arr = np.empty(int(np.prod(shape)), dtype=np.float32)
        api.fill_synthetic(arr, 20261201 + i, dist, a, b)
        tensors[key] = api.tensor(shape, arr, device=args.device)
    graph = api.config_graph(args.workload, tensors)
    outs = [api.materialize(graph) for _ in range(max(1, args.steps))]
    api.device_synchronize(args.device)
    print(f"{args.workload}: {len(outs)} realisations of shape {outs[-1].shape()}")


if __name__ == "__main__":
    main()
