"""bench.py's reference arm (the CPU port of the reference path) prints the
one-line JSON contract the driver reads: the same metric, unit and workload
as the B200 arm, plus `impl`, `cpu_baseline` and an `e2e` object with no
host-device traffic.  CPU only: run here on 8 sequences of the mix (the
default is the full 256), one warm-up and one timed full decode step through
the 36 Qwen3-8B layers and the LM head (about a minute)."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                           "--batch", "8"],
                          cwd=REPO, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    assert d["impl"] == "reference"
    assert d["metric"].startswith("decode tok/s") and d["unit"] == "tok/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    # the CPU arm runs at most one warm-up step and reports what it ran
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["steps_requested"] == 1 and d["warmup_requested"] == 3
    assert d["higher_is_better"] is True and d["dtype"] == "bf16"
    assert d["config"]["workload"] == "qwen3-8b-decode-mix256"
    assert d["config"]["batch"] == 8
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == "tok/s" and cb["sample"]
    e2e = d["e2e"]
    assert e2e["unit"] == "tok/s" and e2e["value"] > 0
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_clock_summary_reads_the_sampled_reasons(tmp_path):
    """The clock record that rides in the bench line: the median SM clock over
    the loaded samples, the max clock, and every throttle reason seen active
    (the driver rejects a run with a thermal or hardware slowdown)."""
    sys.path.insert(0, REPO)
    import bench
    import torch
    s = bench.ClockSampler(torch.device("cpu"))
    s.path = str(tmp_path / "clocks.csv")
    rows = ["0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
            "0, 1950, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active",
            "0, 1935, 1965, 1000.2, 0x4, Not Active, Not Active, Not Active, Active",
            "0, 210, 1965, 180.0, 0x1, Not Active, Not Active, Not Active, Not Active"]
    with open(s.path, "w") as f:
        f.write("\n".join(rows) + "\n")
    d = s.summary()
    assert d["sm_mhz"] == 1950 and d["sm_max_mhz"] == 1965 and d["samples"] == 4
    assert d["reasons"] == ["sw_power_cap"]
    # no file, or an empty one: marked unsampled rather than guessed
    s.path = str(tmp_path / "empty.csv")
    open(s.path, "w").close()
    assert s.summary()["reasons"] == ["unsampled"]
