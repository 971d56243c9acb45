"""Builds libptxstd.so in-tree (ptx-std_b200/libptxstd.so) from csrc/ with nvcc for sm_100a.

Each .cu / .cpp is compiled to an object under ptx-std_b200/_build/ (rebuilt when it or any
header is newer than its object), then linked with the CUDA runtime linked statically, so the
library does not depend on which libcudart the host process (e.g. torch) has loaded.

    python ptx-std_b200/build.py [--force] [-j N]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libptxstd.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I", os.path.join(ROOT, "include"), "-I", CSRC]
CUFLAGS = ARCH + COMMON + ["-lineinfo", "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [NVCC] + CUFLAGS + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, "-x", "cu"] + CUFLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    out = r.stdout + r.stderr
    if verbose:
        print(out, end="")
    return out


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    newest = max([os.path.getmtime(h) for h in _headers()] + [os.path.getmtime(__file__)])
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _stale(s, o, newest):
            todo.append((s, o))
    if todo:
        n = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(n) as ex:
            futs = [ex.submit(_compile, s, o, verbose) for s, o in todo]
            for f in futs:
                f.result()
    if todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB)
                                                for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + [
            "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
