"""Work schedules the full grid does not reach: the grid capped to 1, 5 and 37 CTAs (environment QF_GRID_CAP, read
once per process, so each cap runs in a child process), GEMM and head checked against the oracle there."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("cap", [1, 5, 37])
def test_capped_grids_match_oracle(dev, cap):
    env = dict(os.environ, QF_GRID_CAP=str(cap))
    r = subprocess.run([sys.executable, "-m", "tests._grid_cap_case"], cwd=REPO, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
