"""Builds libdmx_cuda.so (the C-ABI library of include/dmx.h) for sm_100a,
and the ``dmx`` command-line tool over it.

Every .cu under csrc/ is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into _build/ and
linked into ``libdmx_cuda.so`` next to this file (in-tree, so it travels with
the repository snapshot). ``cli/dmx_cli.cpp`` is compiled by g++ into the
executable ``dmx`` beside the library, which it finds through an $ORIGIN
rpath. Objects are rebuilt only when a source or header is newer than them.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libdmx_cuda.so")
CLI_SRC = os.path.join(HERE, "cli", "dmx_cli.cpp")
CLI = os.path.join(HERE, "dmx")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _newest_header():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src, obj, extra, verbose):
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = _newest_header()
    jobs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if ptxas_info or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr):
            jobs.append((src, obj))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = {ex.submit(_compile, s, o, extra, verbose): s for s, o in jobs}
        for f in concurrent.futures.as_completed(futs):
            log = f.result()
            if ptxas_info and log:
                print(f"== {os.path.basename(futs[f])}\n{log}")
    objs = [os.path.join(BUILD, os.path.basename(s) + ".o") for s in sources]
    if jobs or not os.path.exists(LIB):
        # link beside the library and rename over it, so a process that loads the
        # library (or a copy of the tree taken meanwhile) never sees a partial file
        tmp = LIB + f".tmp{os.getpid()}"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    build_cli(verbose)
    return LIB


def build_cli(verbose: bool = False) -> str:
    """Compiles the ``dmx`` executable (cli/dmx_cli.cpp) against libdmx_cuda.so."""
    newest = max(os.path.getmtime(CLI_SRC), os.path.getmtime(LIB),
                 os.path.getmtime(os.path.join(ROOT, "include", "dmx.h")))
    if os.path.exists(CLI) and os.path.getmtime(CLI) >= newest:
        return CLI
    tmp = CLI + f".tmp{os.getpid()}"
    cmd = [CXX, "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"), CLI_SRC,
           "-o", tmp, "-L", HERE, "-ldmx_cuda", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed on dmx_cli.cpp:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, CLI)
    return CLI


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv))
