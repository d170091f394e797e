"""Build the sqrt-block attention shared library in-tree with nvcc (sm_100a).

    python -m llm_training_b200.build [--force] [--debug]

Produces ``llm_training_b200/lib/libsqrtblock.so`` from ``csrc/*.cu``.  The
library exports the C ABI of ``include/sqrtblock.h`` and links the CUDA
runtime statically, so it depends only on the driver at run time.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIBNAME = "libsqrtblock.so"
LIBPATH = os.path.join(LIBDIR, LIBNAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sqrt-block CUDA library cannot be built")


def _flags(debug: bool):
    f = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-I", INCLUDE, "-I", CSRC,
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"] + ARCH_FLAGS
    if debug:
        f += ["-DSQB_DEBUG=1"]
    return f


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> str:
    """Compile every .cu for sm_100a and link the shared library; returns its path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    flags = _flags(debug)
    objs = []
    jobs = []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [s] + hdrs + [__file__]):
            jobs.append([nvcc, *flags, "-c", s, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for out in ex.map(run, jobs):
            if verbose and out.strip():
                print(out, flush=True)
    if force or jobs or _stale(LIBPATH, objs):
        tmp = LIBPATH + ".tmp"
        run([nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs])
        os.replace(tmp, LIBPATH)
    return LIBPATH


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true", help="build with device-side checks")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, debug=a.debug, verbose=a.verbose))


if __name__ == "__main__":
    sys.exit(main())
