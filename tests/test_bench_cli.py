"""bench.py's command line and JSON plumbing on the CPU (no kernels run).

The bench only runs on a B200, so these checks keep its host-side parts honest between GPU runs:
the file compiles, every workload name parses, and the reference arm (transformers' eager
attention on the host cores) prints one JSON line with the contract's keys.
"""

from __future__ import annotations

import json
import py_compile
import subprocess
import sys

from tests.conftest import ROOT


def test_bench_compiles() -> None:
    py_compile.compile(str(ROOT / "bench.py"), doraise=True)


def test_bench_parses_every_workload() -> None:
    sys.path.insert(0, str(ROOT))
    import bench

    for w in ("decode", "prefill", "decode70b", "engine-tiny", "engine-8b", "engine-tiny-replay",
              "engine-8b-replay", "kv-ops", "swap"):  # fmt: skip
        sys.argv = ["bench.py", "--workload", w, "--collective", "pull"]
        args = bench.parse()
        assert args.workload == w and args.steps > 0
    assert bench.collective_for(bench.parse(), 1) == "none"
    assert bench.collective_for(bench.parse(), 8) == "pull"
    sys.argv = ["bench.py"]
    assert bench.collective_for(bench.parse(), 2) == "pull"
    assert bench.collective_for(bench.parse(), 4) == "pull"


def test_reference_arm_prints_one_json_line() -> None:
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0", "--batch", "16"],
        capture_output=True, text=True, timeout=600, cwd=str(ROOT),
    )  # fmt: skip
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):  # fmt: skip
        assert key in line, key
    # transformers' own eager attention (what HFBackend's Llama runs) when it imports
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] in ("reference", "port")
    assert "eager" in line["cpu_baseline"]["sample"]


def test_reference_attention_matches_the_oracle() -> None:
    """The attention the CPU legs time (transformers' eager_attention_forward, called as HFBackend
    runs it) gives the oracle's results on a decode row and on a causal chunk over a prefix."""
    import torch

    sys.path.insert(0, str(ROOT))
    import bench
    from oracle.attention import eager_attention_torch

    attend, kind, _ = bench.reference_attention(32, 8)
    assert kind in ("reference", "port")
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 32, 1, 128, generator=g)
    k, v = torch.randn(1, 8, 300, 128, generator=g), torch.randn(1, 8, 300, 128, generator=g)
    got = attend(q, k, v, None, 128**-0.5)  # [1, 1, 32, 128]
    assert torch.allclose(got[0], eager_attention_torch(q[0], k[0], v[0], 128**-0.5, causal=False),
                          atol=1e-6, rtol=1e-5)  # fmt: skip
    c, ctx = 20, 50
    qc = torch.randn(1, 32, c, 128, generator=g)
    kc, vc = torch.randn(1, 8, ctx, 128, generator=g), torch.randn(1, 8, ctx, 128, generator=g)
    visible = torch.arange(ctx)[None, :] <= torch.arange(ctx - c, ctx)[:, None]
    mask = torch.zeros(c, ctx).masked_fill(~visible, float("-inf"))[None, None]
    got = attend(qc, kc, vc, mask, 128**-0.5)
    ref = eager_attention_torch(qc[0], kc[0], vc[0], 128**-0.5, causal=True)
    assert torch.allclose(got[0], ref, atol=1e-6, rtol=1e-5)


def test_quiet_host_freezes_only_inside_the_region() -> None:
    import gc

    sys.path.insert(0, str(ROOT))
    import bench

    keep = [[i] for i in range(1000)]  # objects alive across the region
    before = gc.get_freeze_count()
    with bench.quiet_host():
        assert gc.get_freeze_count() >= before + len(keep)
    assert gc.get_freeze_count() < len(keep)  # the region's freeze is released
