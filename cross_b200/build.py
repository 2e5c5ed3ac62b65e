"""Build libcross_b200.so in-tree with nvcc for sm_100a.

    python -m cross_b200.build [--force]

Each translation unit compiles to an object under cross_b200/_build/ in its own
nvcc process (in parallel); the objects link into cross_b200/libcross_b200.so.
An object is rebuilt when its source or any header is newer.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "libcross_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "cross_b200.h")
SOURCES = ["errors.cu", "ntt.cu", "ntt_tc.cu", "ntt_shoup.cu", "ntt_noalloc.cu", "elementwise.cu", "bconv.cu",
           "bconv_var.cu", "hemul.cu", "ckks.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _headers():
    hs = [os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".cuh", ".hpp", ".h"))]
    return hs + [HEADER]


def _obj(src: str) -> str:
    return os.path.join(OBJ, src.replace(".cu", ".o"))


def _stale(src: str, newest_header: float) -> bool:
    o = _obj(src)
    if not os.path.exists(o):
        return True
    t = os.path.getmtime(o)
    return os.path.getmtime(os.path.join(SRC, src)) > t or newest_header > t


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(SRC, f) for f in os.listdir(SRC)] + [HEADER]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = True) -> str:
    if not force and not needs_build():
        return OUT
    os.makedirs(OBJ, exist_ok=True)
    newest = max(os.path.getmtime(h) for h in _headers())
    todo = [s for s in SOURCES if force or _stale(s, newest)]

    def compile_one(src):
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", os.path.join(SRC, src), "-o", _obj(src)]
        if verbose:
            print(" ".join(cmd), flush=True)
        return subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        results = list(ex.map(compile_one, todo))
    failed = [(s, r) for s, r in zip(todo, results) if r.returncode != 0]
    for s, r in zip(todo, results):
        if r.stdout or r.stderr:
            sys.stdout.write(r.stdout + r.stderr)
    if failed:
        raise subprocess.CalledProcessError(failed[0][1].returncode, f"nvcc {failed[0][0]}")
    cmd = [nvcc(), *ARCH, "-shared", "-o", OUT, *[_obj(s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv)
