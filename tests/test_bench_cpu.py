"""The bench's reference arm runs on host cores alone: its one JSON line keeps the
contract the driver reads (metric, unit and config of the main arm, the CPU
baseline it timed, an e2e object with no host-device bytes)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line_on_cpu():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == "w4a4_linear_tops" and line["unit"] == "TOPS" and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 3 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["config"]["workload"] == "config1_flux_double_block_linears"
    assert line["config"]["tokens"] == 4608
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["unit"] == "TOPS" and cpu["cores"] >= 1
    assert cpu["kind"] in ("reference", "port") and cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_bench_refuses_short_warmup():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                          cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode != 0 and "--warmup must be >= 3" in proc.stderr


def test_reference_arm_other_ranks_do_no_work():
    """Under torchrun only rank 0 times the reference; the others exit 0 silently."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                           "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert not [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_refuses_other_configs():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "4", "--steps", "1",
                           "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode != 0 and "config 1" in proc.stderr
