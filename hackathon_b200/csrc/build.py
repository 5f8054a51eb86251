"""Builds libqlora_b200.so (all CUDA kernels + the C-ABI) in-tree for sm_100a.

    python -m hackathon_b200.csrc.build [--force] [-j N]

Every `.cu` file in this folder is compiled with nvcc into `hackathon_b200/_build/*.o`, then
linked into `hackathon_b200/libqlora_b200.so`. An object is rebuilt when its source or any header
(`*.cuh` here, `include/*.h`) is newer. The CUDA runtime is linked statically, so the library
needs only the driver at run time.
"""

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libqlora_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-DNDEBUG", "-I", INCLUDE, "-I", HERE]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build qlora_b200")
    return path


def _sources():
    return sorted(f for f in os.listdir(HERE) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(HERE, f) for f in os.listdir(HERE) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(obj, src, newest_header):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src, obj, verbose):
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose else ""


def build(force=False, jobs=None, verbose=False):
    """Compiles what is stale and relinks the library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    todo, objs = [], []
    for f in _sources():
        src = os.path.join(HERE, f)
        obj = os.path.join(BUILD, f[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, src, newest_header):
            todo.append((src, obj))
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        for log in ex.map(lambda so: _compile(*so, verbose), todo):
            if log:
                print(log, file=sys.stderr)
    if todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB)
                                              for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(a.force, a.j, a.verbose))


if __name__ == "__main__":
    main()
