"""Plans of the tensor-core GEMM, on CPU (placeholders: planning compiles
every kernel with NVRTC but launches nothing).

The host side chooses the GEMM form, geometry and split-K:
- CTA pairs (`cta_group::2`, 256 x 256 tiles on a 2-CTA cluster, 32-wide
  k-blocks in 3 stages of 64 KB) where M has at least two 128-row tiles and
  pairing leaves at most a sliver of a pair idle (an even tile count, or 8
  or more);
- one CTA per 128 x 256 tile otherwise, or with PORCH_B200_GEMM=single
  (16-wide k-blocks, 4 stages of 48 KB);
- persistent grids for K <= 4096, sized to the resident units (148 CTAs,
  74 clusters of two);
- split-K when the units would leave SMs idle, over pair slots (74) or CTA
  slots (148).
"""

import os
import re

import pytest


def _gemm_lines(api, m, k, n, form=None):
    """The tcgen05 GEMM launches of relu(A @ B + bias) planned under `form`."""
    old = os.environ.pop("PORCH_B200_GEMM", None)
    try:
        if form is not None:
            os.environ["PORCH_B200_GEMM"] = form
        a, b, c = api.placeholder([m, k]), api.placeholder([k, n]), api.placeholder([n])
        plan = api.describe(api.relu(api.matmul(a, b) + api.broadcast_to(c, [m, n])))
    finally:
        os.environ.pop("PORCH_B200_GEMM", None)
        if old is not None:
            os.environ["PORCH_B200_GEMM"] = old
    return [line for line in plan.splitlines() if line.startswith("kernel pb_gemm_tc_")]


def _geometry(line):
    g = re.search(r"grid=(\d+)x1x1 block=(\d+) smem=(\d+)(?: cluster=(\d+))?", line)
    assert g, line
    return int(g.group(1)), int(g.group(2)), int(g.group(3)), int(g.group(4) or 1)


@pytest.mark.parametrize("m,paired", [
    (128, False),    # one 128-row tile
    (256, True),     # two
    (384, False),    # three: a pair row would sit half idle
    (640, False),    # five
    (1024, True),    # eight
    (1152, True),    # nine: one half-idle pair in five
    (4096, True),
])
def test_pairs_where_m_has_two_or_more_row_tiles(api, m, paired):
    (line,) = _gemm_lines(api, m, 4096, 2048)
    grid, block, smem, cluster = _geometry(line)
    assert ("CTA pairs" in line) == paired, line
    assert block == 320 and smem == 197632, line
    assert cluster == (2 if paired else 1), line
    assert grid % cluster == 0, line
    if paired:
        assert "256x256x32, 3-stage" in line and "128B swizzle" in line, line
    else:
        assert "128x256x16, 4-stage" in line and "64B swizzle" in line, line


def test_single_form_on_request(api):
    (pair,) = _gemm_lines(api, 4096, 4096, 4096)
    (single,) = _gemm_lines(api, 4096, 4096, 4096, form="single")
    assert "CTA pairs" in pair and "CTA pairs" not in single, (pair, single)
    # 4096 x 4096 tiles, K = 4096: persistent, one unit per slot
    assert _geometry(pair)[0] == 148 and _geometry(pair)[3] == 2, pair
    assert _geometry(single)[0] == 148 and _geometry(single)[3] == 1, single


def test_grids_and_split_k_in_pair_slots(api):
    # K = 8192 over 32 x 16 pair tiles (more than 4 waves of 74): no split,
    # not persistent, one cluster of two per tile.
    (line,) = _gemm_lines(api, 8192, 8192, 4096)
    assert "persistent" not in line and "split-K" not in line, line
    assert _geometry(line)[0] == 1024, line
    # 16 x 8 pair tiles fill 0.865 of their waves; split-K x4 fills 0.988,
    # and parts of 2048 of K run persistently.
    (line,) = _gemm_lines(api, 4096, 8192, 2048)
    assert "split-K x4" in line and "persistent" in line, line
    assert _geometry(line)[0] == 148, line
    # Few pair tiles: split-K to fill the 74 pair slots (1 x 4 tiles, K = 8192
    # -> 512 k-blocks of 16: x16 gives 64 units).
    (line,) = _gemm_lines(api, 256, 8192, 1024)
    assert "CTA pairs" in line and "split-K x16" in line, line
    # The same GEMM as one CTA per tile: 2 x 4 tiles, x16 -> 128 units.
    (line,) = _gemm_lines(api, 256, 8192, 1024, form="single")
    assert "CTA pairs" not in line and "split-K x16" in line, line


def test_config5_plans_pairs_for_both_gemms(api):
    plan = api.describe(api.benchmark_graphs(placeholder=True)["c5_mlp"])
    gemms = [line for line in plan.splitlines() if line.startswith("kernel pb_gemm_tc_")]
    assert len(gemms) == 2, plan
    g1, g2 = gemms
    assert "CTA pairs" in g1 and "split-output epilogue" in g1 and "persistent" in g1, g1
    assert "CTA pairs" in g2 and "softmax epilogue" in g2, g2
    assert _geometry(g1)[3] == 2 and _geometry(g2)[3] == 2, gemms
    # GEMM2: 64 x 16 pair tiles over K = 16384, one cluster each.
    assert _geometry(g2)[0] == 2048, g2
