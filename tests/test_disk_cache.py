"""The on-disk cubin cache (PORCH_B200_CACHE_DIR): a second process planning
the same graphs loads every image from disk and runs NVRTC for none of them
(the reference recompiles in every process, src/cuda_jit.cpp:647-703).
Planning compiles without a GPU, so this runs on CPU."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import json, sys
sys.path.insert(0, %r)
from porch_b200 import api
g = api.benchmark_graphs(placeholder=True)
for name in ("c1_elementwise", "c2_view", "c3a_softmax", "c4_matmul"):
    api.describe(g[name])
print(json.dumps(api.compile_stats()))
"""


def _child(cache_dir):
    env = dict(os.environ, PORCH_B200_CACHE_DIR=str(cache_dir))
    out = subprocess.run([sys.executable, "-c", CHILD % str(ROOT)], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_second_process_compiles_nothing(api, tmp_path):
    first = _child(tmp_path)
    assert first["nvrtc_compiles"] >= 5 and first["disk_cache_hits"] == 0, first
    files = sorted(p.name for p in tmp_path.iterdir())
    keys = [f for f in files if f.endswith(".key")]
    assert len(keys) == first["nvrtc_compiles"], files
    assert all(f.endswith((".key", ".img")) for f in files), files  # no temporaries left
    second = _child(tmp_path)
    assert second == {"nvrtc_compiles": 0, "disk_cache_hits": first["nvrtc_compiles"]}, second


def test_a_damaged_entry_is_recompiled(api, tmp_path):
    first = _child(tmp_path)
    # A key whose recorded source differs from the request (a hash
    # collision or a damaged file) is not trusted.
    key = next(p for p in tmp_path.iterdir() if p.name.endswith(".key"))
    key.write_bytes(b"something else")
    second = _child(tmp_path)
    assert second["nvrtc_compiles"] == 1, second
    assert second["disk_cache_hits"] == first["nvrtc_compiles"] - 1, second
