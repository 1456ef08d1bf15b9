"""Build libmhc_b200.so (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python flagos-mhc_b200/build.py [--jobs J] [--debug]

Each csrc/*.cu is compiled to an object under _build/ (in parallel), then
linked into FlagOS_mhc/_lib/libmhc_b200.so, which the Python package loads.
"""
import argparse
import concurrent.futures as cf
import glob
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "FlagOS_mhc", "_lib")
LIB = os.path.join(LIB_DIR, "libmhc_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills", f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]


def _deps_hash(src, extra):
    h = hashlib.sha1()
    for f in [src] + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + \
            [os.path.join(ROOT, "include", "mhc_b200.h")]:
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(extra).encode())
    return h.hexdigest()[:16]


def _compile(src, extra, verbose):
    base = os.path.splitext(os.path.basename(src))[0]
    tag = _deps_hash(src, extra)
    obj = os.path.join(BUILD, f"{base}.{tag}.o")
    if os.path.exists(obj):
        return obj, ""
    for old in glob.glob(os.path.join(BUILD, f"{base}.*.o")):  # stale objects of this source
        os.remove(old)
    cmd = [NVCC] + ARCH + FLAGS + extra + ["-c", src, "-o", obj + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(obj + ".tmp", obj)
    return obj, (r.stdout + r.stderr) if verbose else ""


def build(jobs=None, debug=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    extra = ["-DMHC_DEBUG"] if debug else []
    extra += os.environ.get("MHC_EXTRA_NVCC_FLAGS", "").split()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        results = list(ex.map(lambda s: _compile(s, extra, verbose), srcs))
    for _, log in results:
        if log:
            print(log)
    objs = [o for o, _ in results]
    cmd = [NVCC] + ARCH + ["-shared", "-o", LIB + ".tmp"] + objs + ["-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.debug, a.verbose))
