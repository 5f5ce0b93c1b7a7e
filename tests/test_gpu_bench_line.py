"""bench.py end to end on a small decode case: one JSON line that keeps the contract.

Runs the bench as a user (and the round-end driver) would, on a reduced batch and pool so that it
takes seconds, and checks the line's keys and their consistency: the timed steps, the roofline
of the step's kernels, the instrumented pass, the end-to-end rate through host buffers, the
oracle's parity check and K1's bit-exact rows.
"""

from __future__ import annotations

import json
import subprocess
import sys

import pytest

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu


def test_default_decode_line_keeps_the_contract(cuda_device) -> None:  # type: ignore[no-untyped-def]
    steps, warmup = 5, 3
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--steps", str(steps), "--warmup", str(warmup),
         "--batch", "48", "--pool-blocks", "8192", "--no-extras", "--cpu-sample-seconds", "1"],
        capture_output=True, text=True, timeout=900, cwd=str(ROOT),
    )  # fmt: skip
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "roofline", "instrumented", "parity", "e2e", "gpu_launches", "clocks",
                "cpu_baseline"):  # fmt: skip
        assert key in line, key
    assert line["n_gpus"] == 1 and line["steps"] == steps and line["warmup"] >= 3
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True and line["value"] > 0
    roof = line["roofline"]
    assert roof["bound"] == "hbm" and roof["unit"] == "GB/s"
    # achieved = the step's algorithmic bytes over its measured time; a fraction far above 1
    # would mean the timed kernels are not doing the work
    assert abs(roof["achieved"] - roof["algorithmic_bytes_per_launch"] / roof["avg_launch_us"] / 1e3) \
        <= 0.01 * roof["achieved"]
    assert 0 < roof["frac"] < 1.3
    assert abs(roof["avg_launch_us"] / 1e3 - line["ms_per_step"]) <= 0.01 * line["ms_per_step"]
    assert line["instrumented"]["k2_launch_us"] > 0
    assert line["parity"]["ok"] is True and line["parity"]["k1_bitexact"] is True
    assert line["parity"]["seqs_checked"] > 0
    e2e = line["e2e"]
    assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    assert line["gpu_launches"] == 3 * steps  # K1, prep, decode per step
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["clocks"]["sm_max_mhz"] is None or line["clocks"]["sm_max_mhz"] > 0
