"""The bootstrapping kernel mix's host side (tabIX.py:357-649): the invocation
table, the latency-log parser and the weighted accumulation, against an
independent restatement of the reference's accumulation rules."""
import re

import pytest

from cross_b200 import bts_mix

N = 65536


def _restated_total(rows, lat):
    """tabIX.py:582-617 restated: sum of latency x count over the table rows
    with a latency, the (1, 65536) ntt_common row counted once."""
    total = 0.0
    for kernel, dims, count in rows:
        v = lat.get((kernel, dims))
        if v is None:
            continue
        total += v if (kernel, dims) == ("ntt_common", (1, N)) else v * count
    return total


def test_invocation_table():
    rows = bts_mix.invocations()
    assert len(rows) == 162
    per = {}
    for k, dims, n in rows:
        per.setdefault(k, []).append((dims, n))
        assert dims[-1] == N and n > 0
        assert len(dims) == (3 if k == "basis_convert" else 2)
    assert set(per) == set(bts_mix.KERNELS)
    assert {k: len(v) for k, v in per.items()} == {"add": 32, "automorph": 24, "basis_convert": 41, "mult": 32,
                                                   "ntt_common": 33}
    assert {k: sum(n for _, n in v) for k, v in per.items()} == {"add": 1647, "automorph": 482,
                                                                "basis_convert": 245, "mult": 1852,
                                                                "ntt_common": 578}
    assert ("ntt_common", (1, N), 44) in rows
    assert ("basis_convert", (10, 21, N), 2) in rows
    assert rows[0] == ("add", (18, N), 2)


def test_parse_latency_log_reference_lines():
    log = "\n".join([
        "add(18,65536) - latency:12.5",
        "mult(18, 65536) - latency:3",
        "automorph(19,65536) - latency:7.25",
        "ntt_common(65536,1) b8 - latency:100.0",      # the single-modulus line with its batch
        "ntt_common(65536,7) - latency:40.5",
        "basis_convert(7,20) - latency:9.0",
        "unrelated line",
        "add(18,65536) - latency:13.5",                 # a later line for the same key wins
    ])
    got = bts_mix.parse_latency_log(log)
    assert got == {("add", "18,65536"): 13.5, ("mult", "18,65536"): 3.0, ("automorph", "19,65536"): 7.25,
                   ("ntt_common", "1,65536"): 100.0, ("ntt_common", "7,65536"): 40.5,
                   ("basis_convert", "7,20,65536"): 9.0}


def test_accumulate_and_ratios():
    log = ("add(18,65536) - latency:2\nntt_common(65536,1) - latency:100\n"
           "basis_convert(7,20) - latency:10\nmult(53,65536) - latency:1\n")
    # add (18) x 2, ntt_common (1) once, basis_convert (7, 20) x 3, mult (53) x 50
    assert bts_mix.accumulate_latency_from_log(log) == pytest.approx(2 * 2 + 100 + 10 * 3 + 1 * 50)
    r = bts_mix.latency_ratios(log)
    assert list(r) == ["mult", "ntt_common", "basis_convert", "add"]
    assert sum(r.values()) == pytest.approx(100.0)
    assert r["ntt_common"] == pytest.approx(100 * 100 / 184)


def test_latency_lines_round_trip_every_row():
    """Every row's line, in the reference's print format, parses back to that
    row's key; the weighted sum equals the restated rule."""
    rows = bts_mix.invocations()
    lat = {(k, d): 1.0 + 0.001 * i for i, (k, d, _) in enumerate(rows)}
    log = "\n".join(bts_mix.latency_line(k, d, v) for (k, d), v in lat.items())
    parsed = bts_mix.parse_latency_log(log)
    assert len(parsed) == len(rows)
    for (k, d), v in lat.items():
        assert parsed[(k, ",".join(map(str, d)))] == pytest.approx(v, abs=1e-4)
    assert bts_mix.accumulate_latency_from_log(log) == pytest.approx(_restated_total(rows, lat), rel=1e-6)
    s = bts_mix.summary(log)
    assert s["total_us"] == pytest.approx(sum(s["by_kernel_us"].values()))


def test_latency_line_has_no_exponent():
    line = bts_mix.latency_line("add", (18, N), 1.5e-7)
    assert re.search(r"latency:[0-9.]+$", line)
    assert "e" not in line.split("latency:")[1]


def test_missing_rows_are_skipped(capsys):
    assert bts_mix.accumulate_latency_from_log("") == 0.0
    assert bts_mix.latency_ratios("") == {}
    bts_mix.print_latency_ratios("add(18,65536) - latency:1\n")
    out = capsys.readouterr().out
    assert "add" in out and "100.00%" in out
