"""Builds libbarracuda_fhe.so in-tree for sm_100a (B200).

    python -m barracuda_b200.build            # incremental
    python -m barracuda_b200.build --clean    # rebuild everything

Every translation unit is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; host C++ files go
through nvcc too so that one toolchain links the library.  Objects live in
barracuda_b200/_build/, the library in barracuda_b200/lib/.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libbarracuda_fhe.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall",
              "-Xptxas", "-O3", "--expt-relaxed-constexpr", "-diag-suppress", "177",
              "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.hpp")) + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _obj(src: str) -> str:
    return os.path.join(BUILD, os.path.basename(src) + ".o")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, extra) -> str:
    obj = _obj(src)
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd[cmd.index("-c"):cmd.index("-c")] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr}{r.stdout}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(clean: bool = False, jobs: int | None = None, verbose: bool = False,
          extra_flags=()) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    todo = [s for s in srcs if _stale(_obj(s), [s, *hdrs, __file__])]
    jobs = jobs or min(len(todo), os.cpu_count() or 4) or 1
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj in ex.map(lambda s: _compile(s, list(extra_flags)), todo):
            if verbose:
                print("built", os.path.basename(obj))
    objs = [_obj(s) for s in srcs]
    if todo or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}{r.stdout}")
    build_probe()
    return LIB


PROBE_SRC = os.path.join(PKG, "probe", "op_latency.cpp")
PROBE = os.path.join(LIBDIR, "bc_op_latency")


def build_probe() -> str:
    """The C-ABI latency probe run by bench.py --op-latency (host code only)."""
    if _stale(PROBE, [PROBE_SRC, LIB, os.path.join(INCLUDE, "barracuda_fhe.h")]):
        cxx = shutil.which("g++") or shutil.which("c++")
        if not cxx:
            raise RuntimeError("g++ not found for the latency probe")
        cmd = [cxx, "-O2", "-std=c++17", "-I", INCLUDE, "-o", PROBE, PROBE_SRC, "-L", LIBDIR,
               "-lbarracuda_fhe", "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"latency probe build failed:\n{r.stderr}{r.stdout}")
    return PROBE


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(clean=a.clean or a.ptxas_verbose, jobs=a.jobs, verbose=a.verbose,
                extra_flags=extra))


if __name__ == "__main__":
    main()
