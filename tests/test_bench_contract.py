"""The bench.py output contract, checked on CPU through its reference arm (the C
restatement of the reference path on the host cores): one JSON line with the
keys the driver reads, the reference arm's cpu_baseline and e2e objects, and
the same workload description the GPU arm prints for the same flags."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py")] + args, cwd=REPO, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    j = _run(["--impl", "reference", "--model", "tiny-llama", "--ctx", "96", "--steps", "2", "--warmup", "1",
              "--e2e-steps", "2"])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in j, k
    assert j["impl"] == "reference" and j["metric"] == "decode tok/s" and j["unit"] == "tok/s"
    assert j["value"] > 0 and j["higher_is_better"] is True
    cb = j["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == j["value"] and cb["sample"]
    assert j["e2e"] == {"value": j["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cfg = j["config"]
    assert cfg["model"] == "tiny-llama" and cfg["global_batch"] == 1 and cfg["seq_len"] == 96
    # prompt = ctx - warmup - steps - e2e_steps - 8, the GPU arm's workload
    assert cfg["prompt"] == 96 - 1 - 2 - 2 - 8 and "workload" in cfg
