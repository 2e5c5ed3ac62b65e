"""Writes bts_invocations.csv: the invocation counts of the CKKS bootstrapping
kernel mix, read as text from the reference's tabIX.py (the
BTS_KERNEL_INVOCATION_CSV literal, tabIX.py:399-580).  The reference module
imports jax, so it is parsed, not imported.  The table is product data
(cross_b200/data/bts_invocations.csv, read by cross_b200.bts_mix); this
script only regenerates it.

    python tests/golden/make_bts_table.py <path of the reference's jaxite_word directory>
"""
import csv
import io
import os
import re
import sys


def extract(tabix_source: str) -> list:
    m = re.search(r'BTS_KERNEL_INVOCATION_CSV\s*=\s*"""(.*?)"""', tabix_source, re.S)
    if not m:
        raise ValueError("BTS_KERNEL_INVOCATION_CSV not found")
    rows = list(csv.DictReader(io.StringIO(m.group(1))))
    out = []
    for r in rows:
        dims = tuple(int(v) for v in r["dim"].strip("() ").split(","))
        out.append((r["kernel name"], dims, int(r["count"])))
    return out


def main(ref_dir: str) -> None:
    with open(os.path.join(ref_dir, "tabIX.py")) as f:
        rows = extract(f.read())
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = os.path.join(root, "cross_b200", "data", "bts_invocations.csv")
    with open(path, "w", newline="") as f:
        w = csv.writer(f, lineterminator="\n")
        w.writerow(["kernel", "dims", "count"])
        for k, dims, n in rows:
            w.writerow([k, " ".join(str(d) for d in dims), n])
    print(f"{len(rows)} rows -> {path}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_bts_table.py <jaxite_word directory of the reference>")
    main(sys.argv[1])
