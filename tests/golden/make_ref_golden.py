"""Generates tests/golden/ref_golden.npz + ref_golden.json: outputs of the
REFERENCE ITSELF (AkhilSamavedam/porch, compiled from its sources into
oracle/_ref/ref_runner by oracle/build.py) on seeded small programs.

Run on a GPU box (the reference runs only on CUDA):
    python tests/golden/make_ref_golden.py <output dir>
and copy the two files into tests/golden/. The cases are:
  - every known-answer program of tests/golden/known_answers.json;
  - seeded random programs from tests/graphs.py (integer and float values);
  - the five benchmark graphs at reduced sizes with the benchmark's
    structure and value distributions.
Inputs are stored with the outputs, so the fixtures do not depend on the
input generator staying bit-stable.
"""

from __future__ import annotations

import json
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import graphs  # noqa: E402

RUNNER = ROOT / "oracle" / "_ref" / "ref_runner"


def hx(x: float) -> str:
    return f"{struct.unpack('<I', struct.pack('<f', float(x)))[0]:08x}"


def config_cases(rng: np.random.Generator):
    out = []
    # config 1 structure: (a + b) * 2 - 1
    a = rng.uniform(-1, 1, 4096).astype(np.float32)
    b = rng.uniform(-1, 1, 4096).astype(np.float32)
    out.append(("config1_small", f"0 input 0\n1 input 1\n2 add 0 1\n3 scalar {hx(2)}\n4 multiply 2 3\n"
                                 f"5 scalar {hx(1)}\n6 subtract 4 5\n", [a, b]))
    # config 2 structure: concat(transpose(X[0::2, 8:56]) + bcast(b), Y, 0)
    x = rng.normal(0, 1, (64, 64)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, 32).astype(np.float32)
    y = rng.normal(0, 1, (48, 32)).astype(np.float32)
    out.append(("config2_small", "0 input 0\n1 input 1\n2 input 2\n3 index 0 s0:64:2;s8:56:1\n"
                                 "4 transpose 3\n5 broadcast 1 48,32\n6 add 4 5\n7 concat 6 2 0\n",
                [x, bias, y]))
    # config 3a/3b structure
    for rows, cols in ((64, 257), (8, 4096), (3, 7)):
        xs = rng.normal(0, 2, (rows, cols)).astype(np.float32)
        out.append((f"config3a_small_{rows}x{cols}", "0 input 0\n1 softmax 0 1\n", [xs]))
        out.append((f"config3b_small_{rows}x{cols}", "0 input 0\n1 relu 0\n2 logistic 1\n", [xs]))
    # config 4 structure: relu(A @ B + bcast(bias))
    m, k, n = 64, 96, 128
    A = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    B = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    bb = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    out.append(("config4_small", f"0 input 0\n1 input 1\n2 input 2\n3 matmul 0 1\n4 broadcast 2 {m},{n}\n"
                                 "5 add 3 4\n6 relu 5\n", [A, B, bb]))
    # config 5 structure (staged like the reference must run it)
    m, d, h = 32, 64, 96
    X = rng.normal(0, 1, (m, d)).astype(np.float32)
    W1 = rng.normal(0, 1 / np.sqrt(d), (d, h)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, h).astype(np.float32)
    W2 = rng.normal(0, 1 / np.sqrt(h), (h, d)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, d).astype(np.float32)
    out.append(("config5_small", f"0 input 0\n1 input 1\n2 input 2\n3 input 3\n4 input 4\n5 matmul 0 1\n"
                                 f"6 broadcast 2 {m},{h}\n7 add 5 6\n8 logistic 7\n9 materialize 8\n"
                                 f"10 matmul 9 3\n11 broadcast 4 {m},{d}\n12 add 10 11\n13 materialize 12\n"
                                 "14 softmax 13 1\n", [X, W1, b1, W2, b2]))
    return out


def run_reference(program: str, inputs: list[np.ndarray], tmp: Path):
    (tmp / "prog.txt").write_text(program)
    with open(tmp / "inputs.bin", "wb") as f:
        for arr in inputs:
            f.write(struct.pack("<q", arr.ndim))
            for d in arr.shape:
                f.write(struct.pack("<q", d))
            f.write(np.ascontiguousarray(arr, dtype=np.float32).tobytes())
    res = subprocess.run([str(RUNNER), "eval", str(tmp / "prog.txt"), str(tmp / "inputs.bin"),
                          str(tmp / "out.bin")], capture_output=True, text=True, timeout=300)
    if res.returncode == 3:
        return None, "invalid_argument"
    if res.returncode == 4:
        return None, "out_of_range"
    if res.returncode != 0:
        return None, f"runner_failed rc={res.returncode}: {res.stderr.strip()[-200:]}"
    data = (tmp / "out.bin").read_bytes()
    rank = struct.unpack_from("<q", data, 0)[0]
    shape = list(struct.unpack_from(f"<{rank}q", data, 8))
    vals = np.frombuffer(data, dtype=np.float32, offset=8 + 8 * rank).copy()
    return vals.reshape(shape), None


def main(out_dir: Path) -> None:
    cases = []
    known = json.loads((ROOT / "tests" / "golden" / "known_answers.json").read_text())["cases"]
    for c in known:
        ins = [np.asarray(v, dtype=np.float32).reshape(s) for s, v in c["inputs"]]
        cases.append((f"known_{c['name']}", c["program"], ins))
    for seed in range(60):
        text, ins, _ = graphs.random_program(5000 + seed, integer_values=seed % 2 == 0, depth=4)
        cases.append((f"random_{5000 + seed}", text, ins))
    cases.extend(config_cases(np.random.default_rng(20261201)))

    arrays = {}
    manifest = {"reference": "AkhilSamavedam/porch built from source (oracle/build.py)",
                "runner": "oracle/ref_runner.cpp eval", "cases": []}
    with tempfile.TemporaryDirectory() as td:
        tmp = Path(td)
        for i, (name, program, ins) in enumerate(cases):
            out, err = run_reference(program, ins, tmp)
            entry = {"name": name, "program": program, "n_inputs": len(ins), "error": err,
                     "output_shape": None if out is None else list(out.shape)}
            for j, arr in enumerate(ins):
                arrays[f"c{i}_in{j}"] = arr
            if out is not None:
                arrays[f"c{i}_out"] = out
            manifest["cases"].append(entry)
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "ref_golden.npz", **arrays)
    (out_dir / "ref_golden.json").write_text(json.dumps(manifest, indent=1))
    print(f"{len(cases)} cases written to {out_dir}")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else ROOT / "tests" / "golden")
