"""bench.py's output contract, checked on the CPU through its reference arm (the C restatement
of the Go loops, timed on the host cores): one JSON line with the keys and types the driver
reads, printed by rank 0 alone when torchrun starts several ranks."""
import json
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

REQUIRED = {"metric": str, "value": float, "unit": str, "n_gpus": int, "steps": int, "warmup": int,
            "ms_per_step": float, "higher_is_better": bool, "scaling": str, "dtype": str, "data": str,
            "config": dict}


def run(cmd):
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]


def check_reference_line(d, n_gpus):
    for key, typ in REQUIRED.items():
        assert isinstance(d[key], typ), key
    assert d["impl"] == "reference" and d["n_gpus"] == n_gpus and d["vs_baseline"] is None
    assert d["config"]["workload"] == "ckpt_fp8_e4m3_llama3_8b" and d["unit"] == "elems/s" and d["higher_is_better"]
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_one_line():
    lines = run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert len(lines) == 1
    check_reference_line(lines[0], 1)


def test_reference_arm_under_torchrun_prints_once():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    lines = run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                 "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                 "--gpus", "2", "--steps", "1", "--warmup", "3"])
    assert len(lines) == 1
    check_reference_line(lines[0], 2)


def test_fewer_than_three_warmup_steps_are_refused():
    r = subprocess.run([sys.executable, "bench.py", "--warmup", "2"], cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode != 0 and "--warmup" in r.stderr
