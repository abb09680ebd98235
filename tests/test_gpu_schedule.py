"""Work schedules and kernel instances the default choice does not reach: the grid capped to 1, 5 and 37 CTAs
(environment QF_GRID_CAP) and every tile shape BN:KS forced (environment QF_TILES).  Both are read once per
process, so each setting runs in a child process that checks GEMM and head results against the oracle."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent

SETTINGS = [("1", ""), ("5", ""), ("37", ""),
            ("", "128:128"), ("", "128:256"), ("", "64:256"), ("", "64:512"), ("", "32:512"), ("", "32:1024"),
            ("5", "128:256"), ("37", "32:1024")]


@pytest.mark.parametrize("cap,tiles", SETTINGS, ids=lambda v: v or "-")
def test_schedules_and_tile_shapes_match_oracle(dev, cap, tiles):
    env = dict(os.environ)
    env.pop("QF_GRID_CAP", None)
    env.pop("QF_TILES", None)
    if cap:
        env["QF_GRID_CAP"] = cap
    if tiles:
        env["QF_TILES"] = tiles
    r = subprocess.run([sys.executable, "-m", "tests._grid_cap_case"], cwd=REPO, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
