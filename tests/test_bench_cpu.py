"""The bench's reference arm on the CPU (it runs the oracle on the host cores,
so it needs no GPU): one step, and the JSON line carries the keys the bench
contract asks of it."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 0 and d["steps"] == 1
    # the line names what ran: one whole sequence of the prefill configuration
    assert d["config"]["global_batch"] == 1 and d["config"]["seq_len"] == 8192
    assert d["metric"].startswith("FastMKA prefill tokens/s") and d["unit"] == "tokens/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert "workload" in d["config"]
