"""Build recipe for liblotus_b200.so (sm_100a kernels + C ABI + C++ runtime).

Compiles every source under csrc/ with nvcc for ``sm_100a`` only, in
parallel, into ``_build/`` and links ``liblotus_b200.so`` next to this file,
so the library travels with the source tree.  Objects are rebuilt when their
source or a header they include (nvcc's dependency file next to the object)
is newer; without a dependency file, when any header is newer.

    python -m lotusinfer_b200.build [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "liblotus_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                     "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")) +
                  glob.glob(os.path.join(CSRC, "runtime", "*.cpp")) + glob.glob(os.path.join(CSRC, "runtime", "*.cu")))
    return srcs


def _headers():
    return (glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) +
            glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True) +
            glob.glob(os.path.join(CSRC, "**", "*.hpp"), recursive=True) +
            glob.glob(os.path.join(ROOT, "include", "*.h")))


def _obj(src: str) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _deps(obj: str):
    """Files listed in the object's dependency file, or None without one."""
    d = obj[:-2] + ".d"
    if not os.path.exists(d):
        return None
    txt = open(d).read().replace("\\\n", " ")
    files = txt.split(":", 1)[1].split() if ":" in txt else []
    return [f for f in files if f.strip()]


def _stale(src: str, obj: str, hdr_time: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = _deps(obj)
    if deps is None:
        return t < max(os.path.getmtime(src), hdr_time)
    return any(not os.path.exists(f) or os.path.getmtime(f) > t for f in [src] + deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    hdr_time = max([os.path.getmtime(h) for h in _headers()] + [0])
    jobs = []
    for src in _sources():
        obj = _obj(src)
        if force or _stale(src, obj, hdr_time):
            jobs.append([nvcc] + NVCC_FLAGS + ["-MD", "-MF", obj[:-2] + ".d", "-c", src, "-o", obj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 4)) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(failed))
    objs = [_obj(s) for s in _sources()]
    if force or jobs or not os.path.exists(LIB):
        cmd = [nvcc] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of liblotus_b200.so failed")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
