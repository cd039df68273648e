"""The reference arm of bench.py (the CPU oracle port of the decode step)
prints one JSON line with the keys the benchmark contract asks for, on the
decode workload's config, with no GPU."""

from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3", "--cpu-seconds", "1"], capture_output=True, text=True, timeout=600,
                          cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "env-steps/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"].startswith("cached batched decode")


def test_reference_arm_under_torchrun_uses_every_core():
    """torchrun sets OMP_NUM_THREADS=1 for its ranks; the CPU arm lifts it to
    every usable core (affinity, capped by a CPU quota) and reports the
    threads it ran with."""
    env = dict(os.environ, OMP_NUM_THREADS="1")
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3", "--cpu-seconds", "1"], capture_output=True, text=True, timeout=600,
                          cwd=ROOT, env=env)
    assert proc.returncode == 0, proc.stderr[-2000:]
    d = json.loads([ln for ln in proc.stdout.splitlines() if ln.startswith("{")][0])
    sys.path.insert(0, ROOT)
    import bench

    assert d["cpu_baseline"]["cores"] == bench._usable_cores()


def test_unique_kv_tokens_counts_shared_pages_once():
    import numpy as np

    sys.path.insert(0, ROOT)
    import bench
    from mouse_core_b200.pages import PageTable

    class Sess:  # the attributes the helper reads
        page_size = 4

    s = Sess()
    s.pages = PageTable(3, 16, 4, 4)
    s.pages.allocate(np.array([3, 0, 0]))   # root: 10 tokens in 3 pages
    s.pages.share(1, 0, 2)                  # branch 1 shares the root's 2 full pages
    s.pages.share(2, 0, 2)                  # branch 2 as well
    s.pages.allocate(np.array([0, 1, 1]))   # each branch's own third page
    s._len = np.array([10, 11, 9])
    # branches: 8 shared tokens once + 3 + 1 private
    assert bench.unique_kv_tokens(s, np.array([1, 2])) == 8 + 3 + 1
    assert bench.unique_kv_tokens(s, np.array([0, 1, 2])) == 8 + 2 + 3 + 1
