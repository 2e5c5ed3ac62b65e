"""bench.py's reference arm on the host cores: the JSON line it prints (the
keys every bench line carries), the rank rule under torchrun, and the
bootstrapping mix's arm."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LINE_KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(args, env=None, timeout=300):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, capture_output=True, text=True,
                       timeout=timeout, env=e, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.strip()]


def _check_line(line):
    assert LINE_KEYS <= set(line)
    assert line["impl"] == "reference" and line["value"] > 0 and line["n_gpus"] == 1
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_hemul_line():
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    line = json.loads(lines[-1])
    _check_line(line)
    assert line["metric"].startswith("HE-Mult/s") and line["higher_is_better"] is True
    assert line["unit"] == "HE-Mult/s"


def test_reference_arm_bts_line():
    lines = _run(["--workload", "bts", "--impl", "reference", "--steps", "1", "--warmup", "0"])
    line = json.loads(lines[-1])
    _check_line(line)
    assert line["unit"] == "us" and line["higher_is_better"] is False
    assert set(line["by_kernel_us"]) == {"add", "mult", "automorph", "ntt_common", "basis_convert"}


@pytest.mark.parametrize("rank", ["1"])
def test_reference_arm_other_ranks_exit_quietly(rank):
    """Under torchrun only rank 0 runs the reference arm and prints."""
    assert _run(["--impl", "reference", "--steps", "1", "--warmup", "0"], env={"RANK": rank}, timeout=120) == []
