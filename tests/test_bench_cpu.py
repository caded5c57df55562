"""The bench's reference arm runs on the host only (the oracle port of the
reference's f64 row algorithms on every host thread), so its output line can
be checked here: one JSON line with the keys of the measurement contract,
printed by rank 0 alone when launched under torchrun."""

import json
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _json_lines(text: str) -> list:
    return [json.loads(line) for line in text.splitlines() if line.startswith("{")]


def _check_line(d: dict, n_gpus: int) -> None:
    assert d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 3 and d["warmup"] == 3 and d["n_gpus"] == n_gpus
    assert d["dtype"] == "f32" and d["data"] == "synthetic" and d["scaling"] == "weak"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "extrapolated" in cb["sample"] and d["config"]["extrapolated"] is True
    # the host path copies nothing between host and device
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check_line(lines[0], 1)


def test_reference_arm_under_torchrun_prints_on_rank_zero_only():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check_line(lines[0], 2)


def test_clock_summary_keeps_this_gpus_rows():
    """The clocks key: median SM clock and the throttle reasons seen on this
    process's GPU only (rows of other GPUs, by PCI bus id, are dropped)."""
    import tempfile

    sys.path.insert(0, str(ROOT))
    import bench

    rows = [
        "0, 00000000:1B:00.0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
        "1, 00000000:43:00.0, 1100, 1965, 300.0, 0x0, Active, Not Active, Not Active, Not Active",
        "0, 00000000:1B:00.0, 1815, 1965, 998.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 00000000:1B:00.0, 1920, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ]
    s = bench.ClockSampler("00000000:1B:00.0", enabled=False)
    s.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    s.file.write("\n".join(rows) + "\n")
    got = s.summary()
    assert got == {"sm_mhz": 1920.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    # nothing sampled (no nvidia-smi): marked as such, never as clean clocks
    assert bench.ClockSampler(None, enabled=False).summary()["reasons"] == ["unsampled"]
