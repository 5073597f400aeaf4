"""CPU: the bench's reference arm (the oracle port timed on host cores).

`bench.py --impl reference` must run W untimed and exactly K timed steps, each
a bounded sample of the headline workload, and print one JSON line with the
arm's own step counts.
"""

from __future__ import annotations

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("gw_bench", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_sample_exact_steps():
    b = _bench()
    res = b.cpu_reference_sample(256, 128, 256, 0.5, "random", rows=32, budget_s=60.0, max_reps=3,
                                 exact=(2, 3))
    assert res["reps"] == 3 and res["rows"] == 32 and res["value"] > 0


def test_reference_sample_shrinks_rows_to_the_time_bound():
    b = _bench()
    res = b.cpu_reference_sample(256, 128, 256, 0.5, "random", rows=64, budget_s=1e-9, max_reps=4,
                                 exact=(1, 4))
    assert res["reps"] == 4 and res["rows"] == 16


def test_reference_sample_never_grows_a_small_sample():
    # A sample smaller than the 16-row floor stays as drawn, and the FLOP count
    # follows the rows actually multiplied.
    b = _bench()
    res = b.cpu_reference_sample(256, 128, 256, 0.5, "random", rows=8, budget_s=1e-9, max_reps=2,
                                 exact=(1, 2))
    assert res["rows"] == 8
    assert abs(res["value"] * 1e12 * res["seconds_per_sample"] - 2.0 * 8 * 128 * 128) < 1.0


def test_reference_arm_line():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "3"], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 3
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["value"] > 0
