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


def _digits(total, dnum):
    """Sizes of the key-switch digits (ciphertext.py:329-419: ceil(total / dnum)
    limbs per digit, the last one shorter)."""
    alpha = -(-total // dnum)
    return [min(alpha, total - j * alpha) for j in range(-(-total // alpha))]


@pytest.mark.parametrize("workload,L,K,dnum,transforms", [("hemul", 24, 8, 3, 251), ("hemul", 35, 7, 5, 427),
                                                          ("herot", 24, 8, 3, 160)])
def test_operator_work_counts(workload, L, K, dnum, transforms):
    """The algorithmic work the roofline fractions divide by, restated from the
    operation sequence of hemul.py:153-217 / herot.py:183-302: limb-transforms
    per ciphertext (rescale: INTT of the last limb of 4 elements and NTT of the
    lift into L' limbs; key switch: INTT of d2, the NTT of every digit's
    converted limbs; ModDown: INTT of the K limbs and NTT of the L' limbs of 2
    elements) and the basis conversions' byte-plane contractions."""
    sys.path.insert(0, ROOT)
    import bench
    pt = bench.Point(workload, L, K, dnum, 64, 64)
    N = 65536
    if workload == "hemul":
        L1 = L - 1
        parts = _digits(L1, dnum)
        want_t = 4 + 4 * L1 + L1 + sum(L1 + K - a for a in parts) + 2 * K + 2 * L1
        convs = [(a, L1 + K - a) for a in parts] + [(K, L1), (K, L1)]
    else:
        parts = _digits(L, dnum)
        want_t = L + sum(L + K - a for a in parts) + 2 * K + 2 * L
        convs = [(a, L + K - a) for a in parts] + [(K, L), (K, L)]
    assert want_t == transforms == pt.transforms_per_ct()
    per_transform = 2 * 2 * (4 * 256) * (4 * 256) * 256      # two BAT stages of 2 (4K)(4K) per output row, K = 256
    assert per_transform == 32 * N * (256 + 256)
    want_ops = transforms * per_transform + sum(2 * N * (4 * sq) * (4 * sp) for sq, sp in convs)
    assert pt.int8_ops_per_ct() == pytest.approx(want_ops, rel=1e-12)
