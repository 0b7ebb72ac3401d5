"""The tile kernel's activation records (rec_off in csrc/mma_matvec.cuh, compiled here as host
code): every 16-byte record of a (block, hi/lo plane, sequence, 8-column group) has its own slot,
the records fill the buffer exactly, and the eight lanes of one shared-memory phase (two
sequences x four groups, the B fragments of mma.m16n8k16) read 128 consecutive bytes, so their
16-byte loads hit 32 distinct banks."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

CSRC = os.path.join(ROOT, "laicompute_b200", "csrc")


@pytest.fixture(scope="module")
def layout_check(tmp_path_factory):
    from laicompute_b200 import build as B
    exe = str(tmp_path_factory.mktemp("layout") / "layout_check")
    subprocess.run([B.NVCC, "-std=c++17", *B.ARCH, f"-I{CSRC}", os.path.join(ROOT, "tests", "host", "layout_check.cu"),
                    "-o", exe], check=True)
    return exe


@pytest.mark.parametrize("nb,nseq", [(18, 64), (48, 16), (4, 24), (3, 8)])
def test_records_tile_the_buffer_and_phases_are_contiguous(layout_check, nb, nseq):
    out = subprocess.run([layout_check, str(nb), str(nseq)], capture_output=True, text=True, check=True).stdout
    off = np.array([int(v) for v in out.split()], dtype=np.int64).reshape(nb, 2, nseq, 4)
    flat = np.sort(off.ravel())
    assert np.array_equal(flat, np.arange(nb * 2 * nseq * 4) * 16)  # a bijection onto the buffer
    for bl in range(nb):
        for part in range(2):
            for s0 in range(0, nseq - 1, 2):  # lanes 4g + c, g in {s0, s0 + 1}: one phase
                phase = np.sort(off[bl, part, s0:s0 + 2, :].ravel())
                assert phase[-1] - phase[0] == 112 and np.all(np.diff(phase) == 16)
                assert phase[0] % 128 == 0
