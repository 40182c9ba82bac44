"""Build libspatten_b200.so (the C-ABI library) for sm_100a with nvcc.

    python spatten_b200/build.py [--force] [--verbose] [--ptxas]

Each ``csrc/*.cu`` compiles to an object under ``spatten_b200/_build`` (in
parallel), then the objects link into ``spatten_b200/lib/libspatten_b200.so``
with the CUDA runtime linked statically, so the library depends on nothing
but the driver. The build is skipped when the library is newer than every
source and header.

``peaks/peaks.cu`` (the MUFU throughput microbenchmark the benchmark uses as
a roofline denominator) links separately into ``lib/libspatten_peaks.so``.
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libspatten_b200.so")
PEAKS_SRC = os.path.join(PKG, "peaks", "peaks.cu")
PEAKS_LIB = os.path.join(LIB_DIR, "libspatten_peaks.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) \
        + glob.glob(os.path.join(ROOT, "include", "*.h")) + [os.path.abspath(__file__)]


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build_peaks(force=False):
    """The measurement library (single source, no dependency on the main one)."""
    if not force and os.path.exists(PEAKS_LIB) and \
            os.path.getmtime(PEAKS_LIB) >= max(os.path.getmtime(PEAKS_SRC), os.path.getmtime(__file__)):
        return PEAKS_LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = PEAKS_LIB + ".tmp"
    cmd = [nvcc(), *ARCH, *FLAGS, "-shared", "-cudart", "static", "-o", tmp, PEAKS_SRC]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {PEAKS_SRC}:\n{r.stderr}")
    os.replace(tmp, PEAKS_LIB)
    return PEAKS_LIB


def build(force=False, verbose=False, ptxas_verbose=False):
    build_peaks(force)
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        if verbose or ptxas_verbose:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))
