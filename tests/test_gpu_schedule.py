"""Work schedules and kernel instances the default choice does not reach: the grid capped to 1, 5 and 37 CTAs
(environment QF_GRID_CAP), every tile shape BN:KS forced (environment QF_TILES), even or differently skewed
stream-K shares where every tile is split (environment QF_SK_SKEW), and stream-K reducers that do not wait for the
other shares (QF_PEER_WAIT_NS=0), so that the last share to finish reduces the tile, the all-bf16 activation path
(QF_F16_PATH=0) instead of the default fp16 conversion, and the opt-in tensor-core (tcgen05) consumers of the
128 x 256 tiles at 9..16 tokens (QF_TC=1).  The library reads these knobs only under QF_TEST_OVERRIDES=1,
once per process, so each setting runs in a child process that checks GEMM and head results against the oracle."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent

SETTINGS = [("1", "", "", ""), ("5", "", "", ""), ("37", "", "", ""),
            ("", "128:128", "", ""), ("", "128:256", "", ""), ("", "64:256", "", ""), ("", "64:512", "", ""),
            ("", "32:512", "", ""), ("", "32:1024", "", ""), ("5", "128:256", "", ""), ("37", "32:1024", "", ""),
            ("", "", "0", ""), ("", "", "1", ""), ("", "", "7", ""), ("100", "64:512", "5", ""),
            # reducers hand off at once: the last-arriving share reduces the tile (the not-co-resident path)
            ("", "", "", "0"), ("37", "", "", "0"), ("", "32:1024", "0", "0"), ("5", "128:256", "", "0")]
SETTINGS = [s + ("", "") for s in SETTINGS] + [
    # the exact bf16 activation path (QF_F16_PATH=0) on the default schedule and on forced schedules
    ("", "", "", "", "0", ""), ("37", "64:512", "", "0", "0", ""), ("", "128:256", "", "", "0", ""),
    # the tensor-core consumers of the 128 x 256 tiles at 9..16 tokens: forced shape, capped grid with reducers that
    # do not wait, the default schedule
    ("", "128:256", "", "", "", "1"), ("5", "128:256", "", "0", "", "1"), ("", "", "", "", "", "1")]


@pytest.mark.parametrize("cap,tiles,skew,peer,f16,tc", SETTINGS, ids=lambda v: v or "-")
def test_schedules_and_tile_shapes_match_oracle(dev, cap, tiles, skew, peer, f16, tc):
    env = dict(os.environ)
    for k in ("QF_GRID_CAP", "QF_TILES", "QF_SK_SKEW", "QF_PEER_WAIT_NS", "QF_F16_PATH", "QF_TC"):
        env.pop(k, None)
    env["QF_TEST_OVERRIDES"] = "1"
    if tc:
        env["QF_TC"] = tc
    if f16:
        env["QF_F16_PATH"] = f16
    if cap:
        env["QF_GRID_CAP"] = cap
    if tiles:
        env["QF_TILES"] = tiles
    if skew:
        env["QF_SK_SKEW"] = skew
    if peer:
        env["QF_PEER_WAIT_NS"] = peer
    r = subprocess.run([sys.executable, "-m", "tests._grid_cap_case"], cwd=REPO, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
