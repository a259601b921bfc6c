"""Build the native library ``libkvs_b200.so`` in-tree.

Every ``.cu`` file under ``csrc/`` is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``), every ``.cpp`` by g++, and the
objects are linked by nvcc with a static CUDA runtime.  The library has no
link-time dependency on ``libcuda``: driver entry points (tensor-map
encoding) are fetched at run time with ``cudaGetDriverEntryPoint``, so the
library also loads on machines without a GPU driver (its CPU codec then
works and its device entry points return errors).

Usage: ``python -m kvserve_hpdps_b200.ops.build [-v] [--force]``.
Objects go to ``ops/_build/``; rebuilding is incremental on file mtimes.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_NAME = "libkvs_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> str:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and os.path.exists(os.path.join(cand, "bin", "nvcc")):
            return cand
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(nvcc))
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")))


def _stale(obj: str, src: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + deps)


def _compile(src: str, obj: str, cuda: str, verbose: bool) -> tuple[str, str]:
    if src.endswith(".cu"):
        cmd = [os.path.join(cuda, "bin", "nvcc"), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
               "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", CSRC, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
    else:
        cmd = ["g++", "-O3", "-fPIC", "-std=c++17", "-pthread", "-I", CSRC,
               "-I", os.path.join(cuda, "include"), "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return src, (res.stdout + res.stderr)


def build(verbose: bool = False, force: bool = False, jobs: int | None = None) -> str:
    """Compile and link; returns the library path."""
    cuda = _cuda_home()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    deps = _headers()
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _stale(o, s, deps):
            todo.append((s, o))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, cuda, verbose) for s, o in todo]
            for f in cf.as_completed(futs):
                src, log = f.result()
                if verbose and log.strip():
                    print(f"--- {os.path.basename(src)}\n{log}")
    if todo or force or not os.path.exists(LIB_PATH) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB_PATH) for o in objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [os.path.join(cuda, "bin", "nvcc"), *ARCH_FLAGS, "-shared", "-o", tmp, *objs,
               "-cudart", "static", "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-v", "--verbose", action="store_true", help="ptxas -v and compiler output")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    path = build(verbose=args.verbose, force=args.force)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
