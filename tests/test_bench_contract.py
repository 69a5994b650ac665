"""bench.py's reference arm on the host cores (no GPU needed): it prints one
JSON line with the keys the benchmark driver reads, and its end-to-end
figure moves no bytes between host and device."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2", "--warmup",
                          "1", "--ref-budget", "0.5"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, run.stdout[-2000:]
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 1 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_quietly():
    # Under torchrun only rank 0 times the host reference and prints the line;
    # the other ranks exit 0 without work or output.
    import os

    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps",
                          "2", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr[-2000:]
    assert not [ln for ln in run.stdout.splitlines() if ln.startswith("{")]


def test_roofline_traffic_comes_from_the_committed_profile():
    # roofline.traffic is read from profiles/decode_config3_ncu.md (an ncu
    # capture scaled to a full config-3 launch): it must parse, and DRAM bytes
    # may exceed the algorithmic bytes of one launch only by a few per cent
    # (the kernel reads every K/V byte once).
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_for_test", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    traffic = bench.profile_traffic()
    algorithmic = bench.BATCH * bench.bytes_per_seq()
    assert traffic is not None and 1.0 <= traffic / algorithmic <= 1.02, (traffic, algorithmic)
