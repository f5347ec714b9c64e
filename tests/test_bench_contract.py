"""bench.py's output contract on the host: the reference arm (the reference's CPU
recurrence) prints one JSON line with the keys the benchmark driver reads, at one
process and under torchrun with two ranks (rank 0 alone prints)."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.join(os.path.dirname(__file__), "..")


def _last_json(out: str) -> dict:
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out[-2000:]
    return json.loads(lines[0])


def _check(d: dict, n: int) -> None:
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["n_gpus"] == n and d["value"] > 0 and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["cores"] >= 1 and cpu["kind"] in ("reference", "port") and cpu["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    _check(_last_json(r.stdout), 1)


def test_reference_arm_two_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    _check(_last_json(r.stdout), 2)
