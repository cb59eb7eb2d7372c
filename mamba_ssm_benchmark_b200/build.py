"""Builds libssm_b200.so (the C-ABI selective-scan library) in-tree for sm_100a.

    python -m mamba_ssm_benchmark_b200.build            # incremental
    python -m mamba_ssm_benchmark_b200.build --force    # rebuild everything

Each .cu file under csrc/ is compiled by nvcc in parallel into _build/, then linked into
mamba_ssm_benchmark_b200/_C/libssm_b200.so with the CUDA runtime linked statically, so the
library needs only the driver at run time.  nvcc cross-compiles: no GPU is needed to build.
"""

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
OUT_DIR = os.path.join(PKG, "_C")
LIB = os.path.join(OUT_DIR, "libssm_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _compile(src, obj, verbose):
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr[-8000:]}")
    return r.stderr


def build(force=False, verbose=False, jobs=None):
    """Compiles every CUDA source for sm_100a and links the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    newest_header = max(os.path.getmtime(h) for h in _headers())
    todo, objs = [], []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header):
            todo.append((src, obj))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(jobs) as ex:
            futs = {ex.submit(_compile, s, o, verbose): s for s, o in todo}
            for f in cf.as_completed(futs):
                log = f.result()
                if verbose and log:
                    sys.stderr.write(log)
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-8000:]}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="pass -Xptxas -v and print its report")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose, jobs=args.jobs))


if __name__ == "__main__":
    main()
