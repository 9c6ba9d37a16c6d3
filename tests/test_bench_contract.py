"""bench.py's command line and its reference arm (CPU): the JSON line carries
every key the benchmark contract names, with the reference arm's meaning."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_warmup_below_three_is_rejected():
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"],
                          capture_output=True, text=True, cwd=ROOT)
    assert done.returncode != 0 and "--warmup must be >= 3" in done.stderr


def test_reference_arm_json_line():
    """One small sample (1 layer, batch 1, 64 keys) of the oracle step: the line
    is the reference arm's, on the b200 arm's metric, unit and config."""
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3", "--batch", "1", "--layers", "1",
                           "--seq", "64"], capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert done.returncode == 0, done.stderr
    line = json.loads(done.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["config"]["global_batch"] == 1 and line["config"]["layers"] == 1
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["cpu_model"]
    # Whole steps were run, not extrapolated: the timed steps fit in the run.
    assert line["steps"] * line["ms_per_step"] / 1e3 <= line["timed_s"] * 1.001
    assert line["timed_s"] <= line["run_s"]


def test_reference_arm_under_torchrun_prints_once():
    """Launched the way the driver launches N > 1 (torchrun, 2 ranks on 127.0.0.1):
    rank 0 alone runs the sample and prints the one JSON line, every rank exits 0."""
    import socket
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    done = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                           "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                           "--master-port", str(port), str(ROOT / "bench.py"), "--impl",
                           "reference", "--gpus", "2", "--steps", "1", "--warmup", "3",
                           "--batch", "1", "--layers", "1", "--seq", "64"],
                          capture_output=True, text=True, cwd=ROOT, timeout=900)
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [ln for ln in done.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
