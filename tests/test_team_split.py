"""The team kernel's split of a launch (sk_split and sk_warp_range in csrc/mv_streamk.cuh,
compiled here as host code): the CTAs' row tiles partition the matrix, each team is a run of
team_k consecutive warps, the warps of a team cut every tile's K blocks into consecutive
non-empty slices, and the teams of a CTA take its tiles round-robin exactly once. Checked on the
projection shapes of the 8B-, 1B- and 135M-shaped models at the warp counts the engine uses."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

CSRC = os.path.join(ROOT, "laicompute_b200", "csrc")


@pytest.fixture(scope="module")
def split_check(tmp_path_factory):
    from laicompute_b200 import build as B
    exe = str(tmp_path_factory.mktemp("split") / "split_check")
    subprocess.run([B.NVCC, "-std=c++17", *B.ARCH, f"-I{CSRC}", os.path.join(ROOT, "tests", "host", "split_check.cu"),
                    "-o", exe], check=True)
    return exe


SHAPES = [  # (rows, in, warps): 8B-shaped QKV, O, gate/up, down, lm_head; 1B; 135M; odd sizes
    (6144, 4096, 24), (4096, 4096, 24), (28672, 4096, 24), (4096, 14336, 24), (128256, 4096, 24),
    (3072, 2048, 16), (2048, 2048, 16), (16384, 2048, 16), (2048, 8192, 16), (128256, 2048, 16),
    (960, 576, 16), (576, 576, 16), (3072, 576, 16), (576, 1536, 16), (13, 96, 16), (200, 2048, 16),
]


@pytest.mark.parametrize("rows,cols,warps", SHAPES)
def test_split_covers_every_tile_block_once(split_check, rows, cols, warps):
    nb, ntiles = cols // 32, (rows + 15) // 16
    grid = max(1, min(148, ntiles))  # the engine's grid for the team kernel
    out = subprocess.run([split_check, str(nb), str(ntiles), str(grid), str(warps)], capture_output=True, text=True,
                         check=True).stdout.split("\n")
    k, teams = map(int, out[0].split())
    assert warps % k == 0 and teams == warps // k
    a = np.array([[int(v) for v in line.split()] for line in out[1:] if line.strip()], dtype=np.int64)
    assert a.shape == (grid * warps, 9)
    cover = np.zeros((ntiles, nb), dtype=np.int64)
    prev_hi = 0
    for cta in range(grid):
        r = a[a[:, 0] == cta]
        t_lo, t_hi = r[0, 5], r[0, 6]
        assert (r[:, 5] == t_lo).all() and (r[:, 6] == t_hi).all()
        assert t_lo == prev_hi and t_hi >= t_lo  # consecutive runs of whole tiles
        prev_hi = t_hi
        for team in range(teams):
            m = r[r[:, 2] == team]
            assert list(m[:, 1]) == list(range(team * k, team * k + k))  # a run of k warps
            assert (m[:, 4] == team * k).all() and list(m[:, 3]) == list(range(k))
            slices = m[:, 7:9]
            assert slices[0, 0] == 0 and slices[-1, 1] == nb and (slices[1:, 0] == slices[:-1, 1]).all()
            if nb >= k:
                assert (slices[:, 1] > slices[:, 0]).all()
            for t in range(t_lo + team, t_hi, teams):
                for b0, b1 in slices:
                    cover[t, b0:b1] += 1
    assert prev_hi == ntiles
    assert (cover == 1).all()
